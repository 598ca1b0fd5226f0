// kernels_moe_grouped.cu -- the LFM2 MoE block for T token rows on the tensor cores.
//
// Lfm2Engine._moEFFN (lfm2-engine.js:413-487) runs per token: router, top-4, then for each
// routed expert gate/up (SwiGLU) and down, combined in slot order.  For T rows the same work is
// regrouped by expert so that each expert's weights stream once for all the rows routed to it:
//
//   plan     : histogram of the T*k routed (token, slot) pairs per expert, row order, and the
//              list of 128-row work items (expert, first row, rows) of the grouped GEMM;
//   gather   : X rows into expert order, as fp16 (the GEMM operand);
//   gate, up : grouped tensor-core GEMMs (kernels_gemm.cu) over the packed expert tensors;
//   swiglu   : h = silu(gate) * up, as fp16;
//   down     : grouped GEMM over the packed down tensor;
//   combine  : out[t] = sum over slots s of w[t][s] * down[row of (t, s)], in slot order.
#include "kernels.h"

namespace qq3 {

namespace {

constexpr int kPlanThreads = 1024;
constexpr int kMaxExperts = 256;

__global__ void __launch_bounds__(kPlanThreads)
    k_moe_plan(const int* __restrict__ idx, int P, int top_k, int n_expert, int* __restrict__ pos,
               int* __restrict__ row_token, int4* __restrict__ tiles, int* __restrict__ n_tiles) {
    // a pair whose expert id is outside [0, n_expert) (-1: a slot another rank serves, in the
    // expert-parallel exchange) is not computed: pos = -1, and the combine skips it
    __shared__ int cnt[kMaxExperts], cursor[kMaxExperts];
    __shared__ int n_valid;
    for (int e = threadIdx.x; e < n_expert; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int e = idx[i];
        if (e >= 0 && e < n_expert) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int off = 0, nt = 0;
        for (int e = 0; e < n_expert; e++) {
            cursor[e] = off;
            for (int m = 0; m < cnt[e]; m += 128) tiles[nt++] = make_int4(e, off + m, min(128, cnt[e] - m), 0);
            off += cnt[e];
        }
        *n_tiles = nt;
        n_valid = off;
    }
    __syncthreads();
    // any order of the rows inside an expert gives the same per-row results
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int e = idx[i];
        if (e < 0 || e >= n_expert) {
            pos[i] = -1;
            continue;
        }
        const int p = atomicAdd(&cursor[e], 1);
        pos[i] = p;
        row_token[p] = i / top_k;
    }
    for (int p = n_valid + threadIdx.x; p < P; p += blockDim.x) row_token[p] = 0;  // rows no GEMM reads
}

// GEMM operand of value v at index i: fp16(v), and when split (the exact GEMM) the scaled
// residual fp16((v - fp16(v)) * 2048) at index n + i
__device__ __forceinline__ void put_operand(__half* out, size_t i, size_t n, float v, bool split) {
    const __half h = __float2half_rn(v);
    out[i] = h;
    if (split) out[n + i] = __float2half_rn((v - __half2float(h)) * 2048.f);
}

__global__ void k_gather_rows_f16(const float* __restrict__ x, int K, const int* __restrict__ row_token, int P,
                                  bool split, __half* __restrict__ out) {
    const size_t n = (size_t)P * K;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int p = (int)(i / K), j = (int)(i % K);
        put_operand(out, i, n, x[(size_t)row_token[p] * K + j], split);
    }
}

__global__ void k_swiglu_f16(const float* __restrict__ g, const float* __restrict__ u, size_t n, bool split,
                             __half* __restrict__ h) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float a = g[i];
        put_operand(h, i, n, a * (1.0f / (1.0f + expf(-a))) * u[i], split);  // tensor.js:168-180
    }
}

__global__ void k_moe_combine(const float* __restrict__ down, const int* __restrict__ pos, const float* __restrict__ w,
                              const int* __restrict__ idx, const uint32_t* __restrict__ mask, int T, int top_k, int K,
                              float* __restrict__ out) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)T * K;
         i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / K), c = (int)(i % K);
        float acc = 0.f;
        for (int s = 0; s < top_k; s++) {  // slot order; a masked expert is skipped (lfm2-engine.js:459-486)
            const int p = pos[t * top_k + s];
            if (p < 0) continue;  // a slot served elsewhere
            if (mask) {
                const int e = idx[t * top_k + s];
                if ((mask[e >> 5] >> (e & 31)) & 1u) continue;
            }
            const float ws = w ? w[t * top_k + s] : 1.0f;  // no weights: each row of its own
            acc += ws * down[(size_t)p * K + c];
        }
        out[i] = acc;
    }
}

unsigned grid_for(size_t n) { return (unsigned)std::min<size_t>((n + 255) / 256, (size_t)148 * 32); }

}  // namespace

void launch_moe_combine_rows(const float* y, const int* pos, const float* w, int T, int top_k, int K, float* out,
                             cudaStream_t s) {
    if (T <= 0) return;
    k_moe_combine<<<grid_for((size_t)T * K), 256, 0, s>>>(y, pos, w, nullptr, nullptr, T, top_k, K, out);
    QQ_CUDA_TRY(cudaGetLastError());
}

size_t moe_grouped_scratch_bytes(int T, int top_k, int n_expert, int64_t K, int64_t F) {
    const size_t P = (size_t)T * top_k;
    const size_t tiles = (P + 127) / 128 + n_expert;
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t sp = gemm_exact() ? 2 : 1;  // hi (and lo) fp16 operands
    return al(P * 4) * 2 + al(tiles * 16) + al(4) + al(P * K * 2 * sp) + al(P * F * 4) * 2 + al(P * F * 2 * sp) +
           al(P * K * 4);
}

void launch_moe_grouped(const DTensor& gate, const DTensor& up, const DTensor& down, const int* idx, const float* w,
                        const uint32_t* mask, const float* x, int T, int top_k, int n_expert, void* scratch, float* out,
                        cudaStream_t s) {
    const int64_t K = gate.K, F = gate.rows / n_expert;
    QQ_CHECK(n_expert <= kMaxExperts && K % 32 == 0 && F % 32 == 0, -4, "grouped MoE: unsupported shape");
    const int P = T * top_k;
    const int max_tiles = (P + 127) / 128 + n_expert;
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    char* b = static_cast<char*>(scratch);
    int* pos = reinterpret_cast<int*>(b);
    b += al((size_t)P * 4);
    int* row_token = reinterpret_cast<int*>(b);
    b += al((size_t)P * 4);
    int4* tiles = reinterpret_cast<int4*>(b);
    b += al((size_t)max_tiles * 16);
    int* n_tiles = reinterpret_cast<int*>(b);
    b += al(4);
    const bool split = gemm_exact();
    const size_t sp = split ? 2 : 1;
    __half* xg = reinterpret_cast<__half*>(b);
    b += al((size_t)P * K * 2 * sp);
    float* g = reinterpret_cast<float*>(b);
    b += al((size_t)P * F * 4);
    float* u = reinterpret_cast<float*>(b);
    b += al((size_t)P * F * 4);
    __half* h = reinterpret_cast<__half*>(b);
    b += al((size_t)P * F * 2 * sp);
    float* dn = reinterpret_cast<float*>(b);

    k_moe_plan<<<1, kPlanThreads, 0, s>>>(idx, P, top_k, n_expert, pos, row_token, tiles, n_tiles);
    QQ_CUDA_TRY(cudaGetLastError());
    k_gather_rows_f16<<<grid_for((size_t)P * K), 256, 0, s>>>(x, (int)K, row_token, P, split, xg);
    QQ_CUDA_TRY(cudaGetLastError());
    const GemmGroups grp{tiles, n_tiles, max_tiles};
    launch_gemm_q8_f16(gate, F, xg, P, g, (int)F, &grp, s);
    launch_gemm_q8_f16(up, F, xg, P, u, (int)F, &grp, s);
    k_swiglu_f16<<<grid_for((size_t)P * F), 256, 0, s>>>(g, u, (size_t)P * F, split, h);
    QQ_CUDA_TRY(cudaGetLastError());
    launch_gemm_q8_f16(down, K, h, P, dn, (int)K, &grp, s);
    k_moe_combine<<<grid_for((size_t)T * K), 256, 0, s>>>(dn, pos, w, idx, mask, T, top_k, (int)K, out);
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace qq3
