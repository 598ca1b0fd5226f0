// kernels_ep.cu -- the token side of the expert-parallel MoE exchange (sm_100a).
//
// With the experts of every MoE layer split evenly over W ranks (rank r owns experts
// [r E/W, (r+1) E/W)), a rank routes its own T token rows (Lfm2Engine._moEFFN's router,
// lfm2-engine.js:417-447) and then:
//   plan    : for every destination rank r, the tokens with at least one (unmasked) routed slot on
//             r, in token order (one CTA per destination, a block-wide scan): their position in
//             r's send block, and per position the owner-local expert id of each slot (-1 for a
//             slot on another rank) and its routing weight;
//   gather  : the normalised token rows into the send blocks (each row sent once per
//             destination rank, however many of its slots that rank owns);
//   ... NCCL exchange, the owners' grouped expert GEMMs over the rows they received (weighted
//       partial sums of the slots they own), NCCL exchange back ...
//   combine : hidden[t] += sum over destination ranks, in rank order, of the partial sum that
//             came back for t (the JS slot-order sum, reassociated by rank).
// Blocks have a fixed capacity of C rows per destination, so no count crosses to the host.
#include "kernels.h"

namespace qq3 {

namespace {

constexpr int kEpPlanThreads = 1024;

__global__ void __launch_bounds__(kEpPlanThreads)
    k_ep_plan(const int* __restrict__ idx, const float* __restrict__ w, const uint32_t* __restrict__ mask, int T,
              int top_k, int per_rank, int C, int* __restrict__ pos, int* __restrict__ tok_of, int* __restrict__ ids,
              float* __restrict__ wts) {
    // CTA r plans destination r; thread t < T handles token t
    __shared__ int warp_tot[kEpPlanThreads / 32];
    const int r = blockIdx.x, t = threadIdx.x, lane = t & 31, wp = t >> 5;
    const int e0 = r * per_rank;
    int flag = 0;
    if (t < T)
        for (int s = 0; s < top_k; s++) {
            const int e = idx[t * top_k + s];
            const bool off = mask && ((mask[e >> 5] >> (e & 31)) & 1u);
            if (!off && e >= e0 && e < e0 + per_rank) flag = 1;
        }
    int incl = flag;
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[wp] = incl;
    __syncthreads();
    if (wp == 0) {
        int v = warp_tot[lane];
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += u;
        }
        warp_tot[lane] = v;  // inclusive over warps
    }
    __syncthreads();
    const int p = incl - flag + (wp ? warp_tot[wp - 1] : 0);
    const int count = warp_tot[kEpPlanThreads / 32 - 1];
    if (t < T) {
        pos[(size_t)r * T + t] = flag ? p : -1;
        if (flag) {
            tok_of[(size_t)r * C + p] = t;
            for (int s = 0; s < top_k; s++) {
                const int e = idx[t * top_k + s];
                const bool off = mask && ((mask[e >> 5] >> (e & 31)) & 1u);
                const bool mine = !off && e >= e0 && e < e0 + per_rank;
                ids[((size_t)r * C + p) * top_k + s] = mine ? e - e0 : -1;
                wts[((size_t)r * C + p) * top_k + s] = mine ? w[t * top_k + s] : 0.f;
            }
        }
    }
    // rows past the count carry no slot
    for (int q = count + t; q < C; q += kEpPlanThreads) {
        tok_of[(size_t)r * C + q] = -1;
        for (int s = 0; s < top_k; s++) {
            ids[((size_t)r * C + q) * top_k + s] = -1;
            wts[((size_t)r * C + q) * top_k + s] = 0.f;
        }
    }
}

// row q of destination block r = x[tok_of[r][q]] (float4 copies); rows without a token are zeroed
__global__ void k_ep_gather(const float* __restrict__ x, const int* __restrict__ tok_of, int W, int C, int E,
                            float* __restrict__ out) {
    const int E4 = E >> 2;
    const size_t n = (size_t)W * C * E4;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t row = i / E4;
        const int c = (int)(i % E4);
        const int t = tok_of[row];
        reinterpret_cast<float4*>(out)[i] =
            t >= 0 ? reinterpret_cast<const float4*>(x)[(size_t)t * E4 + c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// hidden[t] += sum over r of back[r][pos[r][t]] (rank order)
__global__ void k_ep_combine(const float* __restrict__ back, const int* __restrict__ pos, int W, int T, int C, int E,
                             float* __restrict__ hidden) {
    const size_t n = (size_t)T * E;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / E), c = (int)(i % E);
        float acc = 0.f;
        for (int r = 0; r < W; r++) {
            const int p = pos[(size_t)r * T + t];
            if (p >= 0) acc += back[((size_t)r * C + p) * E + c];
        }
        hidden[i] += acc;
    }
}

unsigned ep_grid(size_t n) { return (unsigned)std::min<size_t>((n + 255) / 256, (size_t)148 * 16); }

}  // namespace

void launch_ep_plan(const int* idx, const float* w, const uint32_t* mask, int T, int top_k, int n_expert, int W, int C,
                    int* pos, int* tok_of, int* ids, float* wts, cudaStream_t s) {
    QQ_CHECK(T >= 1 && T <= kEpPlanThreads && T <= C, -1, "expert-parallel plan: 1 <= T <= C, T <= 1024");
    QQ_CHECK(W >= 1 && n_expert % W == 0, -1, "expert-parallel plan: experts must split evenly over the ranks");
    k_ep_plan<<<W, kEpPlanThreads, 0, s>>>(idx, w, mask, T, top_k, n_expert / W, C, pos, tok_of, ids, wts);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_ep_gather(const float* x, const int* tok_of, int W, int C, int E, float* out, cudaStream_t s) {
    QQ_CHECK(E % 4 == 0, -1, "expert-parallel gather: E % 4 != 0");
    k_ep_gather<<<ep_grid((size_t)W * C * (E / 4)), 256, 0, s>>>(x, tok_of, W, C, E, out);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_ep_combine(const float* back, const int* pos, int W, int T, int C, int E, float* hidden, cudaStream_t s) {
    k_ep_combine<<<ep_grid((size_t)T * E), 256, 0, s>>>(back, pos, W, T, C, E, hidden);
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace qq3
