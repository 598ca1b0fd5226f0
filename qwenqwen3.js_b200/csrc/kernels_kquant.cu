// kernels_kquant.cu -- k-quant (Q2_K .. Q6_K) weights on the device (sm_100a).
//
// Real-world GGUF files (Q4_K_M and the like) mix k-quant tensors with Q8_0 and F32 ones.  The
// reference reads them element by element (matmulQ{2..6}KxF32 / _q{2..6}kColumn, tensor.js:
// 267-664; WGSL_MATMUL_KQUANT, webgpu.js:47-165): a 256-value superblock holds packed small
// integers, per-sub-block scales (and mins) and f16 super-scales, and element e is
//   Q2_K  d * (sc & 15) * q - dmin * (sc >> 4)          (q: 2 bits)
//   Q3_K  d * scale * ((q | hbit << 2) - 4)              (scale: 6 bits - 32)
//   Q4_K  d * sc * q - dmin * m                          (q: 4 bits, sc / m: 6 bits)
//   Q5_K  d * sc * (q | hbit << 4) - dmin * m
//   Q6_K  d * scale * ((ql | qh << 4) - 32)              (scale: int8)
// evaluated in JS doubles.  The blocks stay raw on the device (no repack).
//   * dequantisation: the same f64 expression, with the same operation order and no fused
//     multiply-add, rounded to f32 -- bit-exact with the reference's column readers;
//   * matmul: each lane of a warp owns 8 consecutive values of a superblock (32 lanes x 8 = one
//     superblock per warp step), evaluates them in f32 -- each product of an f16 scale and the
//     small integers is exact in f32, so one rounding gives the f64 value's f32 rounding -- and
//     dots them with up to kKqRows activation rows held in registers; warps own output rows.
#include "kernels.h"
#include "qq3.h"

namespace qq3 {

namespace {

constexpr int kKqThreads = 256;
constexpr int kKqRows = 8;  // activation rows per pass of the matmul

__device__ __forceinline__ float f16at(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// _q4kGetScaleMin (tensor.js:278-289)
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int sub, int& sc, int& mn) {
    if (sub < 4) {
        sc = s[sub] & 63;
        mn = s[sub + 4] & 63;
    } else {
        sc = (s[sub + 4] & 0xF) | ((s[sub - 4] >> 6) << 4);
        mn = (s[sub + 4] >> 4) | ((s[sub] >> 6) << 4);
    }
}

// _q3kGetScale (tensor.js:295-302)
__device__ __forceinline__ int q3k_scale(const uint8_t* s, int sub) {
    const int lo4 = (s[sub & 7] >> ((sub >> 3) << 2)) & 0xF;
    const int hi2 = (s[8 + (sub & 3)] >> ((sub >> 2) * 2)) & 0x3;
    return (lo4 | (hi2 << 4)) - 32;
}

// the integer parts of element e: value = a * b * c - m1 * m2 (as the JS evaluates it)
struct KqTerms {
    float a;   // super-scale d
    int b, c;  // sub-block scale, quantised value
    float m1;  // dmin (0 where there is no min)
    int m2;
};

__device__ __forceinline__ KqTerms kq_terms(int type, const uint8_t* bb, int e) {
    KqTerms t{0.f, 0, 0, 0.f, 0};
    switch (type) {
        case QQ_TYPE_Q2_K: {
            const int sb = bb[e >> 4];
            t.a = f16at(bb + 80);
            t.m1 = f16at(bb + 82);
            t.b = sb & 0xF;
            t.c = (bb[16 + (e >> 7) * 32 + ((e >> 4) & 1) * 16 + (e & 15)] >> (((e >> 5) & 3) * 2)) & 0x3;
            t.m2 = (sb >> 4) & 0xF;
            break;
        }
        case QQ_TYPE_Q3_K: {
            t.a = f16at(bb + 108);
            t.b = q3k_scale(bb + 96, e >> 4);
            const int hbit = (bb[((e >> 4) & 1) * 16 + (e & 15)] >> (e >> 5)) & 1;
            const int low2 = (bb[32 + (e >> 7) * 32 + ((e >> 4) & 1) * 16 + (e & 15)] >> (((e >> 5) & 3) * 2)) & 3;
            t.c = (low2 | (hbit << 2)) - 4;
            break;
        }
        case QQ_TYPE_Q4_K: {
            t.a = f16at(bb);
            t.m1 = f16at(bb + 2);
            q4k_scale_min(bb + 4, (e >> 6) * 2 + ((e >> 5) & 1), t.b, t.m2);
            const int qb = bb[16 + (e >> 6) * 32 + (e & 31)];
            t.c = ((e >> 5) & 1) ? (qb >> 4) & 0xF : qb & 0xF;
            break;
        }
        case QQ_TYPE_Q5_K: {
            t.a = f16at(bb);
            t.m1 = f16at(bb + 2);
            const int sub = (e >> 6) * 2 + ((e >> 5) & 1);
            q4k_scale_min(bb + 4, sub, t.b, t.m2);
            const int hbit = (bb[16 + (e & 31)] >> sub) & 1;
            const int qb = bb[48 + (e >> 6) * 32 + (e & 31)];
            t.c = (((e >> 5) & 1) ? (qb >> 4) & 0xF : qb & 0xF) | (hbit << 4);
            break;
        }
        default: {  // Q6_K
            t.a = f16at(bb + 208);
            const int ql = bb[(e >> 7) * 64 + ((e >> 5) & 1) * 32 + (e & 31)];
            const int low4 = ((e >> 6) & 1) ? (ql >> 4) & 0xF : ql & 0xF;
            const int high2 = (bb[128 + (e >> 7) * 32 + (e & 31)] >> (((e >> 5) & 3) * 2)) & 0x3;
            t.b = (int)(int8_t)bb[192 + (e >> 7) * 8 + ((e >> 5) & 3) * 2 + ((e & 31) >> 4)];
            t.c = (low4 | (high2 << 4)) - 32;
            break;
        }
    }
    return t;
}

// the reference's f64 value, rounded to f32 (explicit roundings: no contraction into FMA)
__device__ __forceinline__ float kq_exact(int type, const uint8_t* bb, int e) {
    const KqTerms t = kq_terms(type, bb, e);
    const double v = __dmul_rn(__dmul_rn((double)t.a, (double)t.b), (double)t.c);
    return (float)__dsub_rn(v, __dmul_rn((double)t.m1, (double)t.m2));
}

// the same value evaluated in f32: a*b is exact (f16 x <= 8-bit integer), (a*b)*c and m1*m2
// round once, so where the f64 expression is exact (always, short of f16 scales 2^30 apart)
// this is its f32 rounding
__device__ __forceinline__ float kq_fast(const KqTerms& t) {
    return __fsub_rn(__fmul_rn(__fmul_rn(t.a, (float)t.b), (float)t.c), __fmul_rn(t.m1, (float)t.m2));
}

__global__ void k_kq_dequant(int type, const uint8_t* __restrict__ raw, int bs, int64_t K, int64_t n,
                             float* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / K, k = i % K;
        const uint8_t* bb = raw + (row * (K >> 8) + (k >> 8)) * bs;
        out[i] = kq_exact(type, bb, (int)(k & 255));
    }
}

// y[m][n] (+)= W[n] . x[m] for rows m < M: warp per output row, lane = 8 values of a superblock
__global__ void __launch_bounds__(kKqThreads)
    k_kq_matmul(int type, const uint8_t* __restrict__ raw, int bs, int K, int N, const float* __restrict__ x, int M,
                float* __restrict__ y, int ldy) {
    const int lane = threadIdx.x & 31;
    const int warps = (int)(gridDim.x * (blockDim.x >> 5));
    const int nsb = K >> 8;
    for (int n = (int)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)); n < N; n += warps) {
        const uint8_t* rowp = raw + (size_t)n * nsb * bs;
        for (int m0 = 0; m0 < M; m0 += kKqRows) {
            float acc[kKqRows];
#pragma unroll
            for (int r = 0; r < kKqRows; r++) acc[r] = 0.f;
            for (int b = 0; b < nsb; b++) {
                const uint8_t* bb = rowp + (size_t)b * bs;
                float w[8];
#pragma unroll
                for (int j = 0; j < 8; j++) w[j] = kq_fast(kq_terms(type, bb, lane * 8 + j));
                const int k0 = b * 256 + lane * 8;
#pragma unroll
                for (int r = 0; r < kKqRows; r++) {
                    if (m0 + r < M) {
                        const float4* xr = reinterpret_cast<const float4*>(x + (size_t)(m0 + r) * K + k0);
                        const float4 p = __ldg(xr), q = __ldg(xr + 1);
                        acc[r] = fmaf(w[0], p.x, fmaf(w[1], p.y, fmaf(w[2], p.z, fmaf(w[3], p.w, acc[r]))));
                        acc[r] = fmaf(w[4], q.x, fmaf(w[5], q.y, fmaf(w[6], q.z, fmaf(w[7], q.w, acc[r]))));
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < kKqRows; r++) {
                float v = acc[r];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0 && m0 + r < M) y[(size_t)(m0 + r) * ldy + n] = v;
            }
        }
    }
}

// the embedding row of the token in *tok (device), k-quant column reader
__global__ void k_kq_embed(int type, const uint8_t* __restrict__ raw, int bs, int K, int V, const int* __restrict__ tok,
                           float* __restrict__ out) {
    int t = *tok;
    if (t < 0 || t >= V) t = 0;
    const uint8_t* rowp = raw + (size_t)t * (K >> 8) * bs;
    for (int k = threadIdx.x; k < K; k += blockDim.x) out[k] = kq_exact(type, rowp + (size_t)(k >> 8) * bs, k & 255);
}

__global__ void k_finish_token(const int* __restrict__ tok, int* __restrict__ ctl, int* __restrict__ trace) {
    const int p = ctl[1] + 1;
    ctl[0] = *tok;
    ctl[1] = p;
    trace[p] = *tok;
}

unsigned kq_grid(int64_t n) { return (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)148 * 32); }

}  // namespace

int kq_block_bytes(int type) {
    switch (type) {
        case QQ_TYPE_Q2_K: return 84;
        case QQ_TYPE_Q3_K: return 110;
        case QQ_TYPE_Q4_K: return 144;
        case QQ_TYPE_Q5_K: return 176;
        case QQ_TYPE_Q6_K: return 210;
        default: return 0;
    }
}

void launch_kq_dequant(const DTensor& W, int64_t row0, int64_t n_rows, float* out, cudaStream_t s) {
    const int bs = kq_block_bytes(W.type);
    QQ_CHECK(bs > 0 && W.K % 256 == 0, -1, "k-quant dequant: not a k-quant tensor with ne0 % 256 == 0");
    const int64_t n = n_rows * W.K;
    if (n <= 0) return;
    const uint8_t* raw = reinterpret_cast<const uint8_t*>(W.qs) + row0 * (W.K >> 8) * bs;
    k_kq_dequant<<<kq_grid(n), 256, 0, s>>>(W.type, raw, bs, W.K, n, out);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_kq_matmul(const DTensor& W, const float* x, int M, float* y, int ldy, cudaStream_t s) {
    const int bs = kq_block_bytes(W.type);
    QQ_CHECK(bs > 0 && W.K % 256 == 0, -1, "k-quant matmul: not a k-quant tensor with ne0 % 256 == 0");
    QQ_CHECK(((uintptr_t)x & 15u) == 0, -1, "k-quant matmul: input must be 16-byte aligned");
    if (M <= 0 || W.rows <= 0) return;
    const int warps_per_cta = kKqThreads / 32;
    const int64_t ctas = std::min<int64_t>((W.rows + warps_per_cta - 1) / warps_per_cta, (int64_t)num_sms() * 16);
    k_kq_matmul<<<(unsigned)ctas, kKqThreads, 0, s>>>(W.type, reinterpret_cast<const uint8_t*>(W.qs), bs, (int)W.K,
                                                      (int)W.rows, x, M, y, ldy);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_kq_embed(const DTensor& W, const int* tok_dev, int n_vocab, float* out, cudaStream_t s) {
    const int bs = kq_block_bytes(W.type);
    QQ_CHECK(bs > 0 && W.K % 256 == 0, -1, "k-quant embedding: not a k-quant tensor with ne0 % 256 == 0");
    k_kq_embed<<<1, 256, 0, s>>>(W.type, reinterpret_cast<const uint8_t*>(W.qs), bs, (int)W.K, n_vocab, tok_dev, out);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_finish_token(const int* tok, int* ctl, int* trace, cudaStream_t s) {
    k_finish_token<<<1, 1, 0, s>>>(tok, ctl, trace);
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace qq3
