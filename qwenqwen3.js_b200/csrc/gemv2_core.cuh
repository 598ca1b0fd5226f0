// gemv2_core.cuh -- building blocks of the bulk-copy streamed GEMV (kernels_gemv2.cu) shared with
// the persistent decode kernel (kernels_decode.cu): activation digits, the shared-memory ring
// and its producer.
#pragma once
#include "gemv_core.cuh"
#include "pipe.cuh"

namespace qq3 {

constexpr int kCW = 8;                 // consumer warps
constexpr int kG = 4;                  // items per stage
constexpr int kSets = kCW / kG;        // consumer sets taking alternate stages (mode A)
constexpr int kThreads2 = (kCW + 1) * 32;
constexpr int kConsumerThreads = kCW * 32;
constexpr size_t kSmemBudget = 110 * 1024;  // leaves room for a second (PDL-overlapped) CTA per SM

__device__ __forceinline__ uint32_t round16(uint32_t v) { return (v + 15u) & ~15u; }

// --- activation digits -------------------------------------------------------------------
// Shared layout of one input vector of length K (nch = K/16 chunks, K/32 blocks):
//   dig [3][nch] uint4 : digit plane d of chunk c = 16 int8 digits (element 16c + 4w + b in
//                        byte b of word w), so lanes reading consecutive chunks never conflict
//   xsc [K/32] float   : block scale s
// The x-digit form: x ~= s * (d1 + d2/254 + d3/254^2) with s = max|x_block| / 127.

__host__ __device__ inline size_t digit_bytes(int K) { return (size_t)3 * (K >> 4) * 16 + (size_t)(K >> 5) * 4; }

// exact int -> float for |v| < 2^22 on the FMA/ALU pipes (1.5 * 2^23 has unit ulp)
__device__ __forceinline__ float i2f_small(int v) { return __int_as_float(v + 0x4B400000) - 12582912.0f; }
// round-to-nearest-even to an integer, |r| < 2^22, returning the integer and its float value
__device__ __forceinline__ int round_small(float r, float& rf) {
    const float t = r + 12582912.0f;
    rf = t - 12582912.0f;
    return __float_as_int(t) - 0x4B400000;
}

// Thread t of the nthreads consumer threads digitises elements [8t, 8t+8) of x (already
// normalised values in xv[8]).  Quads of threads share a 32-block.
__device__ __forceinline__ void digitise8(const float (&xv)[8], int e0, int K, uint4* dig, float* xsc) {
    const int nch = K >> 4;
    float m = 0.f;
    if (e0 < K) {
#pragma unroll
        for (int e = 0; e < 8; e++) m = fmaxf(m, fabsf(xv[e]));
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    if (e0 >= K) return;
    const float inv = m > 0.f ? 127.0f / m : 0.f;
    if ((e0 & 31) == 0) xsc[e0 >> 5] = m > 0.f ? m / 127.0f : 0.f;
    uint32_t wd[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
    for (int e = 0; e < 8; e++) {
        float f1, f2, f3;
        const float r0 = xv[e] * inv;
        const int d1 = round_small(r0, f1);
        const float r1 = (r0 - f1) * 254.0f;
        const int d2 = round_small(r1, f2);
        const int d3 = round_small((r1 - f2) * 254.0f, f3);
        const int sh = 8 * (e & 3);
        wd[0][e >> 2] |= ((uint32_t)d1 & 0xffu) << sh;
        wd[1][e >> 2] |= ((uint32_t)d2 & 0xffu) << sh;
        wd[2][e >> 2] |= ((uint32_t)d3 & 0xffu) << sh;
    }
    const int c = e0 >> 4, half = (e0 >> 3) & 1;  // 8 elements = words {2*half, 2*half+1} of chunk c
#pragma unroll
    for (int d = 0; d < 3; d++)
        reinterpret_cast<uint2*>(dig + (size_t)d * nch + c)[half] = make_uint2(wd[d][0], wd[d][1]);
}

// 12 dp4a of a 16-weight chunk against the three digit planes, combined in fp32
__device__ __forceinline__ float chunk_dot(const uint4 w, const uint4 g0, const uint4 g1, const uint4 g2) {
    int a1 = __dp4a((int)w.x, (int)g0.x, 0);
    int a2 = __dp4a((int)w.x, (int)g1.x, 0);
    int a3 = __dp4a((int)w.x, (int)g2.x, 0);
    a1 = __dp4a((int)w.y, (int)g0.y, a1);
    a2 = __dp4a((int)w.y, (int)g1.y, a2);
    a3 = __dp4a((int)w.y, (int)g2.y, a3);
    a1 = __dp4a((int)w.z, (int)g0.z, a1);
    a2 = __dp4a((int)w.z, (int)g1.z, a2);
    a3 = __dp4a((int)w.z, (int)g2.z, a3);
    a1 = __dp4a((int)w.w, (int)g0.w, a1);
    a2 = __dp4a((int)w.w, (int)g1.w, a2);
    a3 = __dp4a((int)w.w, (int)g2.w, a3);
    return fmaf(i2f_small(a3), 1.0f / 64516.0f, fmaf(i2f_small(a2), 1.0f / 254.0f, i2f_small(a1)));
}

// lane partials of S rows (shared memory) against one digitised input
template <int S, int CPL>
__device__ __forceinline__ void rows_dot(const int8_t* const (&q)[S], const __half* const (&d)[S],
                                         const bool (&on)[S], const uint4* dig, const float* xsc, int nch,
                                         float (&acc)[S]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < CPL; i++) {
        const int c = lane + 32 * i;
        if (c < nch) {
            const uint4 g0 = dig[c], g1 = dig[nch + c], g2 = dig[2 * nch + c];
            const float sx = xsc[c >> 1];
#pragma unroll
            for (int s = 0; s < S; s++) {
                if (!on[s]) continue;
                const uint4 w = *reinterpret_cast<const uint4*>(q[s] + 16 * c);
                const float dw = __half2float(d[s][c >> 1]);
                acc[s] = fmaf(chunk_dot(w, g0, g1, g2), dw * sx, acc[s]);
            }
        }
    }
}

// --- input staging (consumer threads only) ----------------------------------------------
// Loads x (K <= 2048, 8 elements per consumer thread), optionally applies RMSNorm
// (tensor.js:103-114; the sum of squares in double as the JS does), digitises into smem.
__device__ __forceinline__ void stage_digits(const float* __restrict__ x, const float* __restrict__ norm_w, float eps,
                                             int K, uint4* dig, float* xsc, double* red) {
    const int t = threadIdx.x;
    const int e0 = 8 * t;
    float xv[8];
    if (e0 < K) {
        const float4 a = reinterpret_cast<const float4*>(x + e0)[0];
        const float4 b = reinterpret_cast<const float4*>(x + e0)[1];
        xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w; xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) xv[e] = 0.f;
    }
    if (norm_w) {
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < 8; e++) ss += (double)xv[e] * xv[e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((t & 31) == 0) red[t >> 5] = ss;
        named_bar(1, kConsumerThreads);
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < kCW; w++) tot += red[w];
        const float inv = (float)(1.0 / sqrt(tot / (double)K + (double)eps));
        if (e0 < K) {
            const float4 a = reinterpret_cast<const float4*>(norm_w + e0)[0];
            const float4 b = reinterpret_cast<const float4*>(norm_w + e0)[1];
            const float wv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int e = 0; e < 8; e++) xv[e] = (wv[e] * xv[e]) * inv;
        }
    }
    digitise8(xv, e0, K, dig, xsc);
}

// --- the producer --------------------------------------------------------------------------

struct Ring {
    uint8_t* base;
    uint64_t* full;
    uint64_t* empty;
    int stages;
    uint32_t qs_bytes;  // per source per stage: kG * K
    uint32_t d_bytes;   // per source per stage: round16(kG * K / 16)
    uint32_t stage_bytes;
};

template <int S, class Map>
__device__ __forceinline__ void produce(const Map& map, const Ring& r, int K, int n_items, int* err,
                                        volatile int* abort_flag) {
    const int n_groups = (n_items + kG - 1) / kG;
    if (Map::kDependentRows) pdl_wait();
    int i = 0;
    for (int g = blockIdx.x; g < n_groups; g += gridDim.x, ++i) {
        const int slot = i % r.stages;
        const uint32_t use = (uint32_t)(i / r.stages);
        if (use > 0 && !mbar_wait(&r.empty[slot], (use - 1) & 1u, 200)) {
            set_err(err, kErrEmptyWait);
            *abort_flag = 1;
            return;
        }
        if (*abort_flag) return;
        const int item0 = g * kG;
        const int rows = min(kG, n_items - item0);
        const int8_t* q[S];
        const __half* d[S];
        bool on[S];
        map.group(item0, q, d, on);
        uint32_t tx = 0;
#pragma unroll
        for (int s = 0; s < S; s++)
            if (on[s]) tx += (uint32_t)rows * K + round16((uint32_t)rows * (K >> 4));
        uint8_t* sb = r.base + (size_t)slot * r.stage_bytes;
        mbar_arrive_expect_tx(&r.full[slot], tx);
#pragma unroll
        for (int s = 0; s < S; s++) {
            if (!on[s]) continue;
            bulk_g2s(sb + s * r.qs_bytes, q[s], (uint32_t)rows * K, &r.full[slot]);
            bulk_g2s(sb + S * r.qs_bytes + s * r.d_bytes, d[s], round16((uint32_t)rows * (K >> 4)), &r.full[slot]);
        }
    }
}

// Shared-memory carve-up: [stages][S][kG][K] qs | [S][d_bytes] | x staging | barriers
template <int S>
__device__ __forceinline__ Ring make_ring(uint8_t* smem, int K, int stages) {
    Ring r;
    r.stages = stages;
    r.qs_bytes = (uint32_t)kG * K;
    r.d_bytes = round16((uint32_t)kG * (K >> 4));
    r.stage_bytes = S * (r.qs_bytes + r.d_bytes);
    r.base = smem;
    return r;
}

__host__ __device__ inline size_t ring_bytes(int S, int K, int stages) {
    const size_t per = (size_t)S * ((size_t)kG * K + (((size_t)kG * (K >> 4) + 15) & ~(size_t)15));
    return per * stages;
}

}  // namespace qq3
