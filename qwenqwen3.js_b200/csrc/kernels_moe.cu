// kernels_moe.cu -- MoE routing (sm_100a): the LFM2 sigmoid router and the Qwen3-MoE softmax router.
//
// Replaces the router half of Lfm2Engine._moEFFN (lfm2-engine.js:417-447) and
// WGSL_MOE_SIGMOID_TOPK (webgpu.js:1243-1283): RMSNorm prologue, Q8_0 router GEMV
// (E_in -> n_expert), sigmoid, + selection bias, top-k on the biased score with ties to
// the lower expert id (the stable sort of lfm2-engine.js:434-435), weights = unbiased
// sigmoid normalised by (1e-6 + sum).  One CTA per token; warps split the router rows,
// warp 0 does the selection with shuffles.
#include "gemv_core.cuh"

namespace qq3 {

constexpr int kMaxExperts = 128;          // experts a router scores (Qwen3-30B-A3B has 128)
constexpr int kPerLane = kMaxExperts / 32;  // experts per lane of the selecting warp
constexpr int kMaxTopK = 8;

// Router of one token per CTA.  softmax = false: the LFM2 rule (sigmoid, + selection bias, top-k
// on the biased score, weights = unbiased sigmoid / (1e-6 + their sum)); softmax = true: the
// Qwen3-MoE rule (qwen3-engine.js:304-321, webgpu.js:1181-1232): softmaxInPlace over the logits
// (f64 exp of (l - max), f32 stores, f64 sum), top-k of the probabilities, weights = probability /
// their f64 sum (0 when the sum is 0).  Ties go to the lower expert id in both (the stable sorts).
// Router rows are Q8_0 (rq, rd) or F32 (rf).
__global__ void __launch_bounds__(kGemvThreads)
    k_router(const int8_t* __restrict__ rq, const __half* __restrict__ rd, const float* __restrict__ rf,
             const float* __restrict__ bias, const float* __restrict__ x, int K, const float* __restrict__ norm_w,
             float eps, int n_expert, int top_k, int softmax, float* __restrict__ record, int* __restrict__ idx_out,
             float* __restrict__ w_out) {
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
        float acc = 0.f;
        if (rf) {  // F32 router row: lane-strided float4 dot (stage_x keeps float4 c at (c & 3) * nch + c / 4)
            const float4* row = reinterpret_cast<const float4*>(rf + (size_t)e * K);
            for (int c = lane; c < (K >> 2); c += 32) {
                const float4 a = __ldg(row + c), b = xs[(c & 3) * nch + (c >> 2)];
                acc = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc))));
            }
        } else {
            const int8_t* q[1] = {rq + (size_t)e * K};
            const __half* d[1] = {rd + (size_t)e * (K >> 5)};
            const float4* xv[1] = {xs};
            const bool on[1] = {true};
            float a1[1] = {0.f};
            lane_dots<1>(q, d, xv, on, nch, a1);
            acc = a1[0];
        }
        acc = warp_sum(acc);
        if (lane == 0) logits[e] = acc;
    }
    __syncthreads();
    if (warp != 0) return;
    float prob[kPerLane], sel[kPerLane];
    bool taken[kPerLane];
    if (softmax) {
        // softmaxInPlace (tensor.js:150-164): max, exp(l - max) in f64 stored f32, f64 sum, * 1/sum
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < kPerLane; j++) {
            const int e = lane + 32 * j;
            if (e < n_expert) mx = fmaxf(mx, logits[e]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        double sum = 0.0;
#pragma unroll
        for (int j = 0; j < kPerLane; j++) {
            const int e = lane + 32 * j;
            prob[j] = e < n_expert ? (float)exp((double)logits[e] - (double)mx) : 0.f;
            sum += (double)prob[j];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const double inv = 1.0 / sum;
#pragma unroll
        for (int j = 0; j < kPerLane; j++) {
            const int e = lane + 32 * j;
            prob[j] = (float)((double)prob[j] * inv);
            sel[j] = e < n_expert ? prob[j] : -INFINITY;
            taken[j] = e >= n_expert;
        }
    } else {
        // sigmoid stored to f32 (lfm2-engine.js:421-424); selection score = f32(prob + bias) (:427-431)
#pragma unroll
        for (int j = 0; j < kPerLane; j++) {
            const int e = lane + 32 * j;
            const bool live = e < n_expert;
            prob[j] = live ? 1.0f / (1.0f + expf(-logits[e])) : 0.f;
            sel[j] = live ? prob[j] + (bias ? bias[e] : 0.f) : -INFINITY;
            taken[j] = !live;
        }
    }
    double sum_w = softmax ? 0.0 : 1e-6;
    int top_i[kMaxTopK];
    float top_p[kMaxTopK];
    for (int k = 0; k < top_k; k++) {
        // warp argmax: larger score first, lower expert id on ties
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < kPerLane; j++) {
            const int e = lane + 32 * j;
            if (!taken[j] && (sel[j] > bv || (sel[j] == bv && e < bi))) {
                bv = sel[j];
                bi = e;
            }
        }
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
        float pk = 0.f;
#pragma unroll
        for (int j = 0; j < kPerLane; j++)
            if (lane + 32 * j == bi) {
                taken[j] = true;
                pk = prob[j];
            }
        top_i[k] = bi;
        top_p[k] = __shfl_sync(0xffffffffu, pk, bi & 31);
        sum_w += (double)top_p[k];
    }
    const double inv = softmax ? (sum_w > 0.0 ? 1.0 / sum_w : 0.0) : 1.0 / sum_w;
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
    if (rec) {
#pragma unroll
        for (int j = 0; j < kPerLane; j++) {
            const int e = lane + 32 * j;
            if (e < n_expert) rec[2 * top_k + e] = prob[j];
        }
    }
}

void launch_router(const DTensor& router, const float* bias, const float* x, int T, const float* norm_w, float eps,
                   int n_expert, int top_k, bool softmax, float* record, int* idx, float* w, cudaStream_t s) {
    QQ_CHECK(router.type == 8 || router.type == 0, -4, "router weight must be Q8_0 or F32");
    QQ_CHECK(n_expert >= 1 && n_expert <= kMaxExperts, -4, "router: at most 128 experts in this build");
    QQ_CHECK(top_k >= 1 && top_k <= kMaxTopK && top_k <= n_expert, -1, "router: bad top_k");
    QQ_CHECK(router.rows >= n_expert, -1, "router: fewer rows than experts");
    if (T <= 0) return;
    const int K = (int)router.K;
    QQ_CHECK(((uintptr_t)x & 15u) == 0 && ((uintptr_t)norm_w & 15u) == 0 && K % 32 == 0, -1,
             "router input must be 16-byte aligned with K % 32 == 0");
    const size_t smem = (size_t)K * sizeof(float);
    if (first_use_on_device(reinterpret_cast<const void*>(k_router)))
        QQ_CUDA_TRY(cudaFuncSetAttribute(k_router, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
    const bool f32 = router.type == 0;
    k_router<<<T, kGemvThreads, smem, s>>>(f32 ? nullptr : router.qs, f32 ? nullptr : router.d, f32 ? router.f32 : nullptr,
                                           bias, x, K, norm_w, eps, n_expert, top_k, softmax ? 1 : 0, record, idx, w);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_lfm2_router(const DTensor& router, const float* bias, const float* x, int T, const float* norm_w,
                        float eps, int n_expert, int top_k, float* record, int* idx, float* w, cudaStream_t s) {
    launch_router(router, bias, x, T, norm_w, eps, n_expert, top_k, false, record, idx, w, s);
}

}  // namespace qq3
