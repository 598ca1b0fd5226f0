// gemv_core.cuh -- shared inner loops of the Q8_0 dequant-GEMV kernels (sm_100a).
//
// Shared-memory layout of an input vector: float4 index (j * K/16 + c) holds elements
// [16c + 4j, 16c + 4j + 4), so the 32 lanes of a warp reading chunk c = base + lane at
// the same j touch 32 consecutive float4s (no bank conflicts).
#pragma once
#include "kernels.h"

namespace qq3 {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * kWarp;
constexpr int kUnroll = 4;  // 16-byte chunks in flight per lane per row

// Stage nvec vectors (optionally RMS-normalised) into the permuted shared layout.
__device__ __forceinline__ void stage_x(const XStage& st, float4* xs, double* red) {
    const int K = st.K;
    const int nch = K >> 4;
    const int K4 = K >> 2;
    float inv = 1.f;
    if (st.norm_w) {
        // rmsnorm: invRms = 1 / sqrt(sum(x^2)/n + eps), accumulated in double as the JS does
        double ss = 0.0;
        const float4* x4 = reinterpret_cast<const float4*>(st.x[0]);
        for (int i = threadIdx.x; i < K4; i += blockDim.x) {
            const float4 v = x4[i];
            ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
            red[0] = 1.0 / sqrt(t / (double)K + (double)st.eps);
        }
        __syncthreads();
        inv = (float)red[0];
    }
    for (int v = 0; v < st.nvec; v++) {
        const float4* x4 = reinterpret_cast<const float4*>(st.x[v]);
        float4* dst = xs + (size_t)v * K4;
        for (int i = threadIdx.x; i < K4; i += blockDim.x) {
            float4 val = x4[i];
            if (st.norm_w) {
                const float4 w = reinterpret_cast<const float4*>(st.norm_w)[i];
                val.x = (w.x * val.x) * inv;
                val.y = (w.y * val.y) * inv;
                val.z = (w.z * val.z) * inv;
                val.w = (w.w * val.w) * inv;
            }
            const int c = i >> 2, j = i & 3;
            dst[j * nch + c] = val;
        }
    }
    __syncthreads();
}

// Lane-partial dot products of S rows against their staged inputs.
template <int S>
__device__ __forceinline__ void lane_dots(const int8_t* const (&q)[S], const __half* const (&d)[S],
                                          const float4* const (&xv)[S], const bool (&on)[S], int nch,
                                          float (&acc)[S]) {
    const int lane = threadIdx.x & 31;
#pragma unroll 1
    for (int c0 = 0; c0 < nch; c0 += kWarp * kUnroll) {
        uint4 w[kUnroll][S];
        float dd[kUnroll][S];
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int c = c0 + u * kWarp + lane;
#pragma unroll
            for (int s = 0; s < S; s++) {
                if (on[s] && c < nch) {
                    w[u][s] = ld_stream_u4(q[s] + (size_t)c * 16);
                    dd[u][s] = __half2float(__ldg(d[s] + (c >> 1)));
                } else {
                    w[u][s] = make_uint4(0u, 0u, 0u, 0u);
                    dd[u][s] = 0.f;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int c = c0 + u * kWarp + lane;
            if (c < nch) {
#pragma unroll
                for (int s = 0; s < S; s++) {
                    const float4* x = xv[s] + c;
                    float p = dot4_i8(w[u][s].x, x[0]);
                    p += dot4_i8(w[u][s].y, x[nch]);
                    p += dot4_i8(w[u][s].z, x[2 * nch]);
                    p += dot4_i8(w[u][s].w, x[3 * nch]);
                    acc[s] = fmaf(p, dd[u][s], acc[s]);
                }
            }
        }
    }
}

// Row-source descriptor filled by a Map for one item.
template <int S>
struct Rows {
    const int8_t* q[S];
    const __half* d[S];
    int xsel[S];
    bool on[S];
};

}  // namespace qq3
