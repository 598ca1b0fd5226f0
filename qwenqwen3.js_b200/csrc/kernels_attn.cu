// kernels_attn.cu -- GQA decode attention over the device KV cache (sm_100a).
//
// Replaces, per attention layer: perHeadRMSNorm x2 (tensor.js:117-129), applyRoPE x2
// (tensor.js:132-147), KVCache.store (kv-cache.js:16-32) and the attention core
// (qwen3-engine.js:249-293, lfm2-engine.js:351-385), i.e. WGSL_RMSNORM / WGSL_ROPE /
// WGSL_COPY / WGSL_ATTENTION (webgpu.js:167-331), in ONE launch:
//
//   grid (n_kv, n_split): CTA (g, s) serves the G = n_head/n_kv query heads that share KV
//   head g, over the s-th slice of positions [0, pos].  Its prologue normalises and rotates
//   those query heads; the CTA whose slice holds `pos` also normalises/rotates K and appends
//   K/V at `pos`.  Four warps walk the slice with an online softmax (lane l owns head
//   dimensions [l*HD/32, (l+1)*HD/32)).  Each CTA writes (acc, max, sum) to scratch and the
//   last CTA to arrive for KV head g (atomic ticket, reset for the next launch) merges the
//   slices into the output.  There is no length cap (the WGSL shader stops at 2048).
//
// KV cache layout per layer (and sequence): [n_kv][max_ctx][HD] f32, as kv-cache.js:8-11.
#include "kernels.h"

namespace qq3 {

constexpr int kAttnWarps = 4;
constexpr int kMaxGroup = 8;
constexpr int kMinChunk = 32;

int attention_splits(int max_ctx) {
    int s = (max_ctx + kMinChunk - 1) / kMinChunk;
    if (s > 32) s = 32;
    if (s < 1) s = 1;
    return s;
}

// per-head RMSNorm + split-half RoPE of one head held in shared memory (HD floats)
template <int HD>
__device__ __forceinline__ void norm_rope_head(float* v, const float* __restrict__ w, float eps,
                                               const float* __restrict__ cs, double* red) {
    // called by one full warp
    const int lane = threadIdx.x & 31;
    double ss = 0.0;
    for (int i = lane; i < HD; i += 32) ss += (double)v[i] * v[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = (float)(1.0 / sqrt(ss / (double)HD + (double)eps));
    __syncwarp();
    for (int i = lane; i < HD; i += 32) v[i] = (w[i] * v[i]) * inv;
    __syncwarp();
    constexpr int half = HD / 2;
    for (int i = lane; i < half; i += 32) {
        const float c = cs[2 * i], s = cs[2 * i + 1];
        const float x0 = v[i], x1 = v[i + half];
        v[i] = x0 * c - x1 * s;
        v[i + half] = x0 * s + x1 * c;
    }
    __syncwarp();
}

template <int HD>
__global__ void __launch_bounds__(kAttnWarps * 32) k_attn_decode(AttnArgs a) {
    constexpr int PL = HD / 32;  // head dims per lane
    __shared__ float q_s[kMaxGroup][HD];
    __shared__ float kv_s[2][HD];
    __shared__ float m_s[kAttnWarps][kMaxGroup];
    __shared__ float l_s[kAttnWarps][kMaxGroup];
    __shared__ float acc_s[kAttnWarps][kMaxGroup][HD];
    __shared__ double red[kAttnWarps];
    __shared__ bool is_last;

    const int kvh = blockIdx.x, split = blockIdx.y;
    const int G = a.n_head / a.n_kv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = *a.pos;
    const int len = pos + 1;
    int chunk = (len + a.n_split - 1) / a.n_split;
    if (chunk < kMinChunk) chunk = kMinChunk;
    const int p0 = split * chunk;
    const int p1 = min(len, p0 + chunk);
    const float scale = (float)(1.0 / sqrt((double)HD));
    const float* cs = a.rope_cs + (size_t)pos * HD;  // [HD/2][2]
    float* kc = a.k_cache + (size_t)kvh * a.max_ctx * HD;
    float* vc = a.v_cache + (size_t)kvh * a.max_ctx * HD;

    if (p0 < p1) {
        // --- prologue: query heads of this group (QK-norm + RoPE)
        for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
            const int g = i / HD, d = i - g * HD;
            q_s[g][d] = a.qkv[(size_t)(kvh * G + g) * HD + d];
        }
        const bool owns_pos = (p0 <= pos && pos < p1);
        if (owns_pos) {
            const float* kraw = a.qkv + (size_t)a.n_head * HD + (size_t)kvh * HD;
            const float* vraw = a.qkv + (size_t)(a.n_head + a.n_kv) * HD + (size_t)kvh * HD;
            for (int d = threadIdx.x; d < HD; d += blockDim.x) {
                kv_s[0][d] = kraw[d];
                kv_s[1][d] = vraw[d];
            }
        }
        __syncthreads();
        for (int g = warp; g < G; g += kAttnWarps) norm_rope_head<HD>(q_s[g], a.q_norm, a.eps, cs, red);
        if (owns_pos && warp == kAttnWarps - 1) {
            norm_rope_head<HD>(kv_s[0], a.k_norm, a.eps, cs, red);
            for (int d = lane; d < HD; d += 32) {  // KVCache.store
                kc[(size_t)pos * HD + d] = kv_s[0][d];
                vc[(size_t)pos * HD + d] = kv_s[1][d];
            }
        }
        __syncthreads();

        // --- online softmax over this slice
        float m[kMaxGroup], l[kMaxGroup], acc[kMaxGroup][PL];
        float qv[kMaxGroup][PL];
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int j = 0; j < PL; j++) {
                acc[g][j] = 0.f;
                qv[g][j] = g < G ? q_s[g][lane * PL + j] : 0.f;
            }
        }
        for (int p = p0 + warp; p < p1; p += kAttnWarps) {
            float kr[PL], vr[PL];
            const float* kp = kc + (size_t)p * HD + lane * PL;
            const float* vp = vc + (size_t)p * HD + lane * PL;
#pragma unroll
            for (int j = 0; j < PL; j++) {
                kr[j] = kp[j];
                vr[j] = vp[j];
            }
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++) {
                if (g >= G) break;
                float dot = 0.f;
#pragma unroll
                for (int j = 0; j < PL; j++) dot = fmaf(qv[g][j], kr[j], dot);
                dot = warp_sum(dot);
                const float sc = dot * scale;
                const float mn = fmaxf(m[g], sc);
                const float cf = expf(m[g] - mn);
                const float pe = expf(sc - mn);
                l[g] = l[g] * cf + pe;
#pragma unroll
                for (int j = 0; j < PL; j++) acc[g][j] = fmaf(acc[g][j], cf, pe * vr[j]);
                m[g] = mn;
            }
        }
        // --- merge the warps of this CTA
        for (int g = 0; g < G; g++) {
            if (lane == 0) {
                m_s[warp][g] = m[g];
                l_s[warp][g] = l[g];
            }
#pragma unroll
            for (int j = 0; j < PL; j++) acc_s[warp][g][lane * PL + j] = acc[g][j];
        }
        __syncthreads();
        for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
            const int g = i / HD, d = i - g * HD;
            float M = -INFINITY;
            for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, m_s[w][g]);
            float L = 0.f, A = 0.f;
            for (int w = 0; w < kAttnWarps; w++) {
                if (m_s[w][g] == -INFINITY) continue;
                const float f = expf(m_s[w][g] - M);
                L += l_s[w][g] * f;
                A += acc_s[w][g][d] * f;
            }
            float* pp = a.part + ((size_t)(kvh * G + g) * a.n_split + split) * (HD + 2);
            pp[d] = A;
            if (d == 0) {
                pp[HD] = M;
                pp[HD + 1] = L;
            }
        }
    } else {
        for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
            const int g = i / HD, d = i - g * HD;
            float* pp = a.part + ((size_t)(kvh * G + g) * a.n_split + split) * (HD + 2);
            pp[d] = 0.f;
            if (d == 0) {
                pp[HD] = -INFINITY;
                pp[HD + 1] = 0.f;
            }
        }
    }

    // --- last CTA for this KV head merges the slices
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int t = atomicAdd(a.counter + kvh, 1u);
        is_last = (t == (unsigned)a.n_split - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int g = i / HD, d = i - g * HD;
        const float* base = a.part + (size_t)(kvh * G + g) * a.n_split * (HD + 2);
        float M = -INFINITY;
        for (int s = 0; s < a.n_split; s++) M = fmaxf(M, __ldcg(base + s * (HD + 2) + HD));
        float L = 0.f, A = 0.f;
        for (int s = 0; s < a.n_split; s++) {
            const float ms = __ldcg(base + s * (HD + 2) + HD);
            if (ms == -INFINITY) continue;
            const float f = expf(ms - M);
            L += __ldcg(base + s * (HD + 2) + HD + 1) * f;
            A += __ldcg(base + s * (HD + 2) + d) * f;
        }
        a.out[(size_t)(kvh * G + g) * HD + d] = A / L;
    }
    if (threadIdx.x == 0) a.counter[kvh] = 0u;
}

void launch_attention_decode(const AttnArgs& a, cudaStream_t s) {
    QQ_CHECK(a.n_head % a.n_kv == 0 && a.n_head / a.n_kv <= kMaxGroup, -4, "attention: unsupported GQA group size");
    dim3 grid(a.n_kv, a.n_split);
    if (a.hd == 64) k_attn_decode<64><<<grid, kAttnWarps * 32, 0, s>>>(a);
    else if (a.hd == 128) k_attn_decode<128><<<grid, kAttnWarps * 32, 0, s>>>(a);
    else QQ_CHECK(false, -4, "attention: head_dim must be 64 or 128");
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace qq3
