// kernels_moe.cu -- LFM2-MoE routing (sm_100a).
//
// Replaces the router half of Lfm2Engine._moEFFN (lfm2-engine.js:417-447) and
// WGSL_MOE_SIGMOID_TOPK (webgpu.js:1243-1283): RMSNorm prologue, Q8_0 router GEMV
// (E_in -> n_expert), sigmoid, + selection bias, top-k on the biased score with ties to
// the lower expert id (the stable sort of lfm2-engine.js:434-435), weights = unbiased
// sigmoid normalised by (1e-6 + sum).  One CTA per token; warps split the router rows,
// warp 0 does the selection with shuffles.
#include "gemv_core.cuh"

namespace qq3 {

constexpr int kMaxExperts = 32;
constexpr int kMaxTopK = 8;

__global__ void __launch_bounds__(kGemvThreads)
    k_lfm2_router(const int8_t* __restrict__ rq, const __half* __restrict__ rd, const float* __restrict__ bias,
                  const float* __restrict__ x, int K, const float* __restrict__ norm_w, float eps, int n_expert,
                  int top_k, float* __restrict__ record, int* __restrict__ idx_out, float* __restrict__ w_out) {
    extern __shared__ float4 xs[];
    __shared__ double red[kGemvWarps];
    __shared__ float logits[kMaxExperts];
    const int t = blockIdx.x;
    XStage st;
    st.x[0] = x + (size_t)t * K;
    st.nvec = 1;
    st.K = K;
    st.norm_w = norm_w;
    st.eps = eps;
    stage_x(st, xs, red);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = K >> 4;
    for (int e = warp; e < n_expert; e += kGemvWarps) {
        const int8_t* q[1] = {rq + (size_t)e * K};
        const __half* d[1] = {rd + (size_t)e * (K >> 5)};
        const float4* xv[1] = {xs};
        const bool on[1] = {true};
        float acc[1] = {0.f};
        lane_dots<1>(q, d, xv, on, nch, acc);
        acc[0] = warp_sum(acc[0]);
        if (lane == 0) logits[e] = acc[0];
    }
    __syncthreads();
    if (warp != 0) return;
    // sigmoid stored to f32 (:421-424); selection score = f32(prob + bias) (:427-431)
    const bool live = lane < n_expert;
    const float prob = live ? 1.0f / (1.0f + expf(-logits[lane])) : 0.f;
    float sel = live ? prob + (bias ? bias[lane] : 0.f) : -INFINITY;
    bool taken = !live;
    double sum_w = 1e-6;
    int top_i[kMaxTopK];
    float top_p[kMaxTopK];
    for (int k = 0; k < top_k; k++) {
        // warp argmax: larger score first, lower expert id on ties
        float bv = taken ? -INFINITY : sel;
        int bi = taken ? 0x7fffffff : lane;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        // all lanes agree unless the scores are NaN; keep lane 0's choice and an in-range id
        bi = __shfl_sync(0xffffffffu, bi, 0);
        if (bi < 0 || bi >= n_expert) bi = 0;
        if (lane == bi) taken = true;
        top_i[k] = bi;
        top_p[k] = __shfl_sync(0xffffffffu, prob, bi & 31);
        sum_w += (double)top_p[k];
    }
    const double inv = 1.0 / sum_w;
    float* rec = record ? record + (size_t)t * (2 * top_k + n_expert) : nullptr;
    if (lane == 0) {
        for (int k = 0; k < top_k; k++) {
            const float wk = (float)((double)top_p[k] * inv);
            if (idx_out) idx_out[t * top_k + k] = top_i[k];
            if (w_out) w_out[t * top_k + k] = wk;
            if (rec) {
                rec[k] = (float)top_i[k];
                rec[top_k + k] = wk;
            }
        }
    }
    if (rec && live) rec[2 * top_k + lane] = prob;
}

void launch_lfm2_router(const DTensor& router, const float* bias, const float* x, int T, const float* norm_w,
                        float eps, int n_expert, int top_k, float* record, int* idx, float* w, cudaStream_t s) {
    QQ_CHECK(router.type == 8, -4, "router weight must be Q8_0");
    QQ_CHECK(n_expert >= 1 && n_expert <= kMaxExperts, -4, "router: at most 32 experts in this build");
    QQ_CHECK(top_k >= 1 && top_k <= kMaxTopK && top_k <= n_expert, -1, "router: bad top_k");
    QQ_CHECK(router.rows >= n_expert, -1, "router: fewer rows than experts");
    if (T <= 0) return;
    const int K = (int)router.K;
    QQ_CHECK(((uintptr_t)x & 15u) == 0 && ((uintptr_t)norm_w & 15u) == 0 && K % 32 == 0, -1,
             "router input must be 16-byte aligned with K % 32 == 0");
    const size_t smem = (size_t)K * sizeof(float);
    if (first_use_on_device(reinterpret_cast<const void*>(k_lfm2_router)))
        QQ_CUDA_TRY(cudaFuncSetAttribute(k_lfm2_router, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
    k_lfm2_router<<<T, kGemvThreads, smem, s>>>(router.qs, router.d, bias, x, K, norm_w, eps, n_expert, top_k, record,
                                                idx, w);
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace qq3
