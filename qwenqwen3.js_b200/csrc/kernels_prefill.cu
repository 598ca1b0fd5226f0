// kernels_prefill.cu -- batched prefill: T prompt tokens through a layer at once (sm_100a).
//
// The reference prefills one token at a time (`forward(t_i, i, true)`, qwen3-engine.js:397-457,
// lfm2-engine.js:523-583); a T-token call is semantically the same as T sequential calls.  Here
// the projections of all T tokens run as tensor-core GEMMs (kernels_gemm.cu) and the few
// sequential pieces are kernels over the T rows:
//   k_embed_rows      embedding rows of T tokens (tensor.js:56-77)
//   k_rope_rows       split-half RoPE of T x heads rows at positions pos0.. (tensor.js:132-147)
//   k_kv_append       K/V of T tokens into the cache at pos0.. (kv-cache.js:16-32)
//   k_conv_prefill    short-conv over the T tokens, carrying the 2-tap state (lfm2-engine.js:282-325)
//   k_attn_prefill    causal GQA attention of each token over positions 0..pos0+t
//                     (qwen3-engine.js:249-301, lfm2-engine.js:329-390)
//   k_add_rows / k_swiglu_rows   residual add and SwiGLU (tensor.js:168-185)
// The same pieces with a row map (`*_at`: row t is sequence seq[t] at position pos[t]) run one
// forward() step of several independent sequences at once, plus k_argmax_rows (sampleGreedy per
// row) for their greedy ids.
#include "kernels.h"
#include "pipe.cuh"

namespace qq3 {

// QQ3_ATTN_TILE=0 keeps the per-warp global-memory attention kernels (A/B measurements)
static bool tiled_attention_off() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("QQ3_ATTN_TILE");
        v = (e && atoi(e) == 0) ? 1 : 0;
    }
    return v == 1;
}

namespace {

unsigned grid_n(size_t n) { return (unsigned)std::min<size_t>((n + 255) / 256, (size_t)148 * 64); }

__global__ void k_embed_rows(const int8_t* __restrict__ qs, const __half* __restrict__ d, int K, const int* tok,
                             int T, int n_vocab, float* __restrict__ out) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)T * K; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / K), k = (int)(i % K);
        int v = tok[t];
        v = v < 0 || v >= n_vocab ? 0 : v;
        out[i] = (float)qs[(size_t)v * K + k] * __half2float(d[(size_t)v * (K >> 5) + (k >> 5)]);
    }
}

// x: [T][n_heads][hd], already RMS-normalised per head; rotate halves at position pos0 + t
__global__ void k_rope_rows(float* __restrict__ x, int T, int n_heads, int hd, const float* __restrict__ cs, int pos0) {
    const int half = hd / 2;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)T * n_heads * half;
         i += (size_t)gridDim.x * blockDim.x) {
        const int j = (int)(i % half);
        const size_t row = i / half;
        const int t = (int)(row / n_heads);
        float* v = x + row * hd;
        const float c = cs[(size_t)(pos0 + t) * hd + 2 * j], s = cs[(size_t)(pos0 + t) * hd + 2 * j + 1];
        const float x0 = v[j], x1 = v[j + half];
        v[j] = x0 * c - x1 * s;
        v[j + half] = x0 * s + x1 * c;
    }
}

// cache layout [n_kv][max_ctx][hd]; k, v: [T][n_kv][hd]
__global__ void k_kv_append(const float* __restrict__ k, const float* __restrict__ v, int T, int n_kv, int hd,
                            int max_ctx, int pos0, float* __restrict__ kc, float* __restrict__ vc) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)T * n_kv * hd;
         i += (size_t)gridDim.x * blockDim.x) {
        const int dd = (int)(i % hd);
        const int h = (int)((i / hd) % n_kv);
        const int t = (int)(i / ((size_t)hd * n_kv));
        const size_t dst = ((size_t)h * max_ctx + pos0 + t) * hd + dd;
        kc[dst] = k[i];
        vc[dst] = v[i];
    }
}

// bcx: [T][3E] = (B | C | x) rows of in_proj; conv taps w[E][3]; state[2][E] = (s0, s1)
__global__ void k_conv_prefill(const float* __restrict__ bcx, const float* __restrict__ w, float* __restrict__ state,
                               int T, int E, float* __restrict__ y) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= E) return;
    float s0 = state[c], s1 = state[E + c];
    const float k0 = w[c * 3], k1 = w[c * 3 + 1], k2 = w[c * 3 + 2];
    for (int t = 0; t < T; t++) {
        const float* r = bcx + (size_t)t * 3 * E;
        const float bx = r[c] * r[2 * E + c];
        const float co = k0 * s0 + k1 * s1 + k2 * bx;
        y[(size_t)t * E + c] = r[E + c] * co;
        s0 = s1;
        s1 = bx;
    }
    state[c] = s0;
    state[E + c] = s1;
}

__global__ void k_add_rows(float* __restrict__ x, const float* __restrict__ d, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] += d[i];
}

__global__ void k_swiglu_rows(const float* __restrict__ g, const float* __restrict__ u, size_t n, float* __restrict__ h) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float a = g[i];
        h[i] = a * (1.0f / (1.0f + expf(-a))) * u[i];
    }
}

// The fp16 operand form of one activation for the tensor-core products (the planes
// launch_f32_to_f16 writes): hi = fp16(v) at i and, when split, lo = fp16((v - hi) * 2048) at n + i
__device__ __forceinline__ void store_f16_split(__half* __restrict__ y16, size_t n, size_t i, float v, int split) {
    const __half h = __float2half_rn(v);
    y16[i] = h;
    if (split) y16[n + i] = __float2half_rn((v - __half2float(h)) * 2048.f);
}

// SwiGLU straight into the operand planes of the down projection (h itself is not stored)
__global__ void k_swiglu_rows_f16(const float* __restrict__ g, const float* __restrict__ u, size_t n,
                                  __half* __restrict__ y16, int split) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float a = g[i];
        store_f16_split(y16, n, i, a * (1.0f / (1.0f + expf(-a))) * u[i], split);
    }
}

// Residual add and the next RMS norm in one pass over a row (tensor.js:103-116, 181-186; block =
// row): x += d (d nullable), y = (w * x) / rms(x) with the sum of squares taken exactly as
// k_rmsnorm takes it (same thread striding and reduction order, so the same y), and y's operand
// planes when y16 is non-null (n_all = rows x n values per plane)
__global__ void k_add_rmsnorm_rows(float* __restrict__ x, const float* __restrict__ d, int n,
                                   const float* __restrict__ w, float eps, float* __restrict__ y,
                                   __half* __restrict__ y16, size_t n_all, int split) {
    __shared__ double red[32];
    const size_t r0 = (size_t)blockIdx.x * n;
    float* xr = x + r0;
    float* yr = y + r0;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = xr[i];
        if (d) {
            v += d[r0 + i];
            xr[i] = v;
        }
        ss += (double)v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
        red[0] = 1.0 / sqrt(t / (double)n + (double)eps);
    }
    __syncthreads();
    const float inv = (float)red[0];
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float o = (w[i] * xr[i]) * inv;
        yr[i] = o;
        if (y16) store_f16_split(y16, n_all, r0 + i, o, split);
    }
}

// The query / key head norms, RoPE and the K/V append of the rows in one launch.  Block
// (t, head), 128 threads: heads 0 .. n_head-1 are row t's query heads (normalised and rotated in
// place), heads n_head .. n_head+n_kv-1 its key heads (normalised, rotated and stored with the
// row's value head into the cache).  Row t is sequence seq[t] (nullable: the cache pointers are
// the sequence's own) at position pos[t] (nullable: pos0 + t).  The norm is k_rmsnorm's with 128
// threads and the rotation k_rope_rows' (tensor.js:117-147, kv-cache.js:16-32); hd <= 128, even.
__global__ void __launch_bounds__(128)
    k_qk_norm_rope_rows(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, int n_head,
                        int n_kv, int hd, const float* __restrict__ qw, const float* __restrict__ kw, float eps,
                        const float* __restrict__ cs, const int* __restrict__ seq, const int* __restrict__ pos,
                        int pos0, size_t seq_stride, int max_ctx, float* __restrict__ kc, float* __restrict__ vc) {
    __shared__ double red[4];
    __shared__ float xs[128];
    const int t = blockIdx.x, i = threadIdx.x;
    const bool is_q = (int)blockIdx.y < n_head;
    const int h = is_q ? (int)blockIdx.y : (int)blockIdx.y - n_head;
    const size_t src = is_q ? ((size_t)t * n_head + h) * hd : ((size_t)t * n_kv + h) * hd;
    const float xv = i < hd ? (is_q ? q[src + i] : k[src + i]) : 0.f;
    double ss = (double)xv * xv;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((i & 31) == 0) red[i >> 5] = ss;
    __syncthreads();
    if (i == 0) {
        double tt = 0.0;
        for (int j = 0; j < 4; j++) tt += red[j];
        red[0] = 1.0 / sqrt(tt / (double)hd + (double)eps);
    }
    __syncthreads();
    const float inv = (float)red[0];
    if (i < hd) xs[i] = ((is_q ? qw[i] : kw[i]) * xv) * inv;
    __syncthreads();
    const int half = hd >> 1;
    const size_t p = (size_t)(pos ? pos[t] : pos0 + t);
    float* dst;
    if (is_q) {
        dst = q + src;
    } else {
        const size_t at = (seq ? (size_t)seq[t] * seq_stride : 0) + ((size_t)h * max_ctx + p) * hd;
        dst = kc + at;
        if (i < hd) vc[at + i] = v[src + i];
    }
    if (i < half) {
        const float c = cs[p * hd + 2 * i], s = cs[p * hd + 2 * i + 1];
        const float x0 = xs[i], x1 = xs[i + half];
        dst[i] = x0 * c - x1 * s;
        dst[i + half] = x0 * s + x1 * c;
    }
}

// Causal GQA attention of one query head over positions 0..len-1 of one kv head's cache rows,
// by one warp: tiles of 32 positions (one per lane), online softmax, V accumulation (lane owns
// HD/32 dims).  qh: the normalised, rotated query; o: HD outputs.
template <int HD>
__device__ __forceinline__ void attn_row(const float* __restrict__ qh, const float* __restrict__ kb,
                                         const float* __restrict__ vb, int len, float* __restrict__ o) {
    constexpr int PL = HD / 32;
    const int lane = threadIdx.x & 31;
    const float scale = (float)(1.0 / sqrt((double)HD));
    float qv[HD];
#pragma unroll
    for (int j = 0; j < HD; j += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(qh + j);
        qv[j] = v4.x;
        qv[j + 1] = v4.y;
        qv[j + 2] = v4.z;
        qv[j + 3] = v4.w;
    }
    float m = -INFINITY, l = 0.f, acc[PL];
#pragma unroll
    for (int j = 0; j < PL; j++) acc[j] = 0.f;
    for (int p0 = 0; p0 < len; p0 += 32) {
        const int p = p0 + lane;
        float s = -INFINITY;
        if (p < len) {
            const float* kr = kb + (size_t)p * HD;
            float dot = 0.f;
#pragma unroll
            for (int j = 0; j < HD; j += 4) {
                const float4 k4 = __ldg(reinterpret_cast<const float4*>(kr + j));
                dot = fmaf(qv[j], k4.x, dot);
                dot = fmaf(qv[j + 1], k4.y, dot);
                dot = fmaf(qv[j + 2], k4.z, dot);
                dot = fmaf(qv[j + 3], k4.w, dot);
            }
            s = dot * scale;
        }
        const float m_new = fmaxf(m, warp_max(s));
        const float pl = p < len ? expf(s - m_new) : 0.f;
        const float cf = expf(m - m_new);
        l = l * cf + warp_sum(pl);
#pragma unroll
        for (int j = 0; j < PL; j++) acc[j] *= cf;
        const int n = min(32, len - p0);
        for (int jj = 0; jj < n; jj++) {
            const float pj = __shfl_sync(0xffffffffu, pl, jj);
            const float* vr = vb + (size_t)(p0 + jj) * HD + lane * PL;
#pragma unroll
            for (int j = 0; j < PL; j++) acc[j] = fmaf(pj, __ldg(vr + j), acc[j]);
        }
        m = m_new;
    }
    o += lane * PL;
#pragma unroll
    for (int j = 0; j < PL; j++) o[j] = acc[j] / l;
}

// The same over positions [p_begin, p_end) without the final division: writes the partial
// softmax state (HD accumulators, then max m and sum l) to part (HD + 2 floats); m = -inf and
// l = 0 for an empty range.
template <int HD>
__device__ __forceinline__ void attn_row_part(const float* __restrict__ qh, const float* __restrict__ kb,
                                              const float* __restrict__ vb, int p_begin, int p_end,
                                              float* __restrict__ part) {
    constexpr int PL = HD / 32;
    const int lane = threadIdx.x & 31;
    const float scale = (float)(1.0 / sqrt((double)HD));
    float qv[HD];
#pragma unroll
    for (int j = 0; j < HD; j += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(qh + j);
        qv[j] = v4.x;
        qv[j + 1] = v4.y;
        qv[j + 2] = v4.z;
        qv[j + 3] = v4.w;
    }
    float m = -INFINITY, l = 0.f, acc[PL];
#pragma unroll
    for (int j = 0; j < PL; j++) acc[j] = 0.f;
    for (int p0 = p_begin; p0 < p_end; p0 += 32) {
        const int p = p0 + lane;
        float s = -INFINITY;
        if (p < p_end) {
            const float* kr = kb + (size_t)p * HD;
            float dot = 0.f;
#pragma unroll
            for (int j = 0; j < HD; j += 4) {
                const float4 k4 = __ldg(reinterpret_cast<const float4*>(kr + j));
                dot = fmaf(qv[j], k4.x, dot);
                dot = fmaf(qv[j + 1], k4.y, dot);
                dot = fmaf(qv[j + 2], k4.z, dot);
                dot = fmaf(qv[j + 3], k4.w, dot);
            }
            s = dot * scale;
        }
        const float m_new = fmaxf(m, warp_max(s));
        const float pl = p < p_end ? expf(s - m_new) : 0.f;
        const float cf = expf(m - m_new);
        l = l * cf + warp_sum(pl);
#pragma unroll
        for (int j = 0; j < PL; j++) acc[j] *= cf;
        const int n = min(32, p_end - p0);
        for (int jj = 0; jj < n; jj++) {
            const float pj = __shfl_sync(0xffffffffu, pl, jj);
            const float* vr = vb + (size_t)(p0 + jj) * HD + lane * PL;
#pragma unroll
            for (int j = 0; j < PL; j++) acc[j] = fmaf(pj, __ldg(vr + j), acc[j]);
        }
        m = m_new;
    }
#pragma unroll
    for (int j = 0; j < PL; j++) part[lane * PL + j] = acc[j];
    if (lane == 0) {
        part[HD] = m;
        part[HD + 1] = l;
    }
}

// One CTA per (token t, kv head): warp g scores query head kvh*G + g against positions
// 0..pos0+t.  q: [T][n_head][HD] (normalised, rotated); out: [T][n_head][HD].
template <int HD>
__global__ void k_attn_prefill(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                               int pos0, int n_head, int n_kv, int max_ctx, float* __restrict__ out) {
    const int t = blockIdx.x, kvh = blockIdx.y;
    const int G = n_head / n_kv;
    const int warp = threadIdx.x >> 5;
    if (warp >= G) return;
    const int h = kvh * G + warp;
    attn_row<HD>(q + ((size_t)t * n_head + h) * HD, kc + (size_t)kvh * max_ctx * HD, vc + (size_t)kvh * max_ctx * HD,
                 pos0 + t + 1, out + ((size_t)t * n_head + h) * HD);
}

// Causal attention of a prompt chunk by query tiles (flash-attention form on the CUDA cores, f32):
// CTA (query tile, kv head) takes 64 query rows -- kPfTok = 64 / G consecutive tokens x the G query
// heads of the kv head, 16 rows per warp -- and walks the keys 0 .. (its last token's position) in
// tiles of 32: K is staged transposed (Kt[d][j], rows padded to 33), V as rows, each warp's queries
// transposed (Qs[d][r]); a lane scores its key against the warp's 16 rows (one K word and four
// broadcast float4 of queries per 16 FMAs), an online softmax per row, then a lane accumulates its
// HD/32 output dims of the 16 rows over the tile's 32 keys (the probabilities broadcast from
// shared memory).  Each K/V tile is read once per 64 query rows instead of once per query.
constexpr int kPfWarps = 4, kPfRows = 16, kPfKeys = 32;

template <int HD>
__global__ void __launch_bounds__(kPfWarps * 32)
    k_attn_prefill_tile(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc, int T,
                        int pos0, int n_head, int n_kv, int max_ctx, float* __restrict__ out) {
    constexpr int PL = HD / 32, H4 = HD / 4, KP = kPfKeys + 1;
    extern __shared__ __align__(16) float smf[];
    float* Kt = smf;                                    // [HD][KP]
    float* Vs = Kt + HD * KP;                           // [kPfKeys][HD]
    float* Qs = Vs + kPfKeys * HD;                      // [warp][HD][kPfRows]
    float* Ps = Qs + kPfWarps * HD * kPfRows;           // [warp][kPfKeys][kPfRows]
    const int G = n_head / n_kv;
    const int QT = (kPfWarps * kPfRows) / G;            // tokens per tile
    const int t0 = blockIdx.x * QT, kvh = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* qw = Qs + warp * HD * kPfRows;
    float* pw = Ps + warp * kPfKeys * kPfRows;
    // this warp's rows r = 16 warp + i: token t0 + r / G, head kvh G + r % G
    for (int i = 0; i < kPfRows; i++) {
        const int r = warp * kPfRows + i, t = t0 + r / G;
        const float* qr = q + ((size_t)t * n_head + kvh * G + r % G) * HD;
        for (int d = lane; d < HD; d += 32) qw[d * kPfRows + i] = t < T ? qr[d] : 0.f;
    }
    const float scale = (float)(1.0 / sqrt((double)HD));
    float m[kPfRows], l[kPfRows], acc[kPfRows][PL];
#pragma unroll
    for (int i = 0; i < kPfRows; i++) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int j = 0; j < PL; j++) acc[i][j] = 0.f;
    }
    const int t_last = min(T, t0 + QT) - 1;
    const int n_keys = pos0 + t_last + 1;  // keys 0 .. the tile's last position
    const float* kb = kc + (size_t)kvh * max_ctx * HD;
    const float* vb = vc + (size_t)kvh * max_ctx * HD;
    for (int k0 = 0; k0 < n_keys; k0 += kPfKeys) {
        __syncthreads();  // the previous tile's K / V are no longer read
        for (int f = threadIdx.x; f < kPfKeys * H4; f += kPfWarps * 32) {
            const int j = f / H4, d = (f % H4) * 4;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (k0 + j < n_keys) {
                kv = __ldg(reinterpret_cast<const float4*>(kb + (size_t)(k0 + j) * HD + d));
                vv = __ldg(reinterpret_cast<const float4*>(vb + (size_t)(k0 + j) * HD + d));
            }
            Kt[(d + 0) * KP + j] = kv.x;
            Kt[(d + 1) * KP + j] = kv.y;
            Kt[(d + 2) * KP + j] = kv.z;
            Kt[(d + 3) * KP + j] = kv.w;
            *reinterpret_cast<float4*>(Vs + j * HD + d) = vv;
        }
        __syncthreads();
        // scores of key k0 + lane against the warp's rows
        float sc[kPfRows];
#pragma unroll
        for (int i = 0; i < kPfRows; i++) sc[i] = 0.f;
#pragma unroll 4
        for (int d = 0; d < HD; d++) {
            const float kv = Kt[d * KP + lane];
            const float4* q4 = reinterpret_cast<const float4*>(qw + d * kPfRows);
#pragma unroll
            for (int c = 0; c < kPfRows / 4; c++) {
                const float4 qv = q4[c];
                sc[4 * c] = fmaf(qv.x, kv, sc[4 * c]);
                sc[4 * c + 1] = fmaf(qv.y, kv, sc[4 * c + 1]);
                sc[4 * c + 2] = fmaf(qv.z, kv, sc[4 * c + 2]);
                sc[4 * c + 3] = fmaf(qv.w, kv, sc[4 * c + 3]);
            }
        }
        const int key = k0 + lane;
#pragma unroll
        for (int i = 0; i < kPfRows; i++) {
            const int r = warp * kPfRows + i, t = t0 + r / G;
            const bool live = t < T && key <= pos0 + t;  // causal: keys up to the row's own position
            const float s = live ? sc[i] * scale : -INFINITY;
            const float mx = warp_max(s);
            const float m_new = fmaxf(m[i], mx);
            const float p = (live && m_new > -INFINITY) ? expf(s - m_new) : 0.f;
            const float cf = m_new > -INFINITY ? expf(m[i] - m_new) : 1.f;
            l[i] = l[i] * cf + warp_sum(p);
            m[i] = m_new;
#pragma unroll
            for (int j = 0; j < PL; j++) acc[i][j] *= cf;
            pw[lane * kPfRows + i] = p;
        }
        __syncwarp();
        // values: lane's HD/32 dims of the warp's rows over the tile's keys
        const int nk = min(kPfKeys, n_keys - k0);
        for (int jj = 0; jj < nk; jj++) {
            const float4* p4 = reinterpret_cast<const float4*>(pw + jj * kPfRows);
            float vv[PL];
#pragma unroll
            for (int j = 0; j < PL; j++) vv[j] = Vs[jj * HD + lane * PL + j];
#pragma unroll
            for (int c = 0; c < kPfRows / 4; c++) {
                const float4 pv = p4[c];
#pragma unroll
                for (int j = 0; j < PL; j++) {
                    acc[4 * c][j] = fmaf(pv.x, vv[j], acc[4 * c][j]);
                    acc[4 * c + 1][j] = fmaf(pv.y, vv[j], acc[4 * c + 1][j]);
                    acc[4 * c + 2][j] = fmaf(pv.z, vv[j], acc[4 * c + 2][j]);
                    acc[4 * c + 3][j] = fmaf(pv.w, vv[j], acc[4 * c + 3][j]);
                }
            }
        }
        __syncwarp();  // pw is rewritten by the next tile
    }
#pragma unroll
    for (int i = 0; i < kPfRows; i++) {
        const int r = warp * kPfRows + i, t = t0 + r / G;
        if (t >= T) continue;
        float* o = out + ((size_t)t * n_head + kvh * G + r % G) * HD + lane * PL;
        const float inv = 1.f / l[i];
#pragma unroll
        for (int j = 0; j < PL; j++) o[j] = acc[i][j] * inv;
    }
}

// ---- multi-sequence decode rows: row t is sequence seq[t] at position pos[t] ----------------
// (one forward() step of each of T independent sequences; the caches of sequence s start at
// seq_stride * s floats from the layer's base pointer)

__global__ void k_rope_rows_at(float* __restrict__ x, int T, int n_heads, int hd, const float* __restrict__ cs,
                               const int* __restrict__ pos) {
    const int half = hd / 2;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)T * n_heads * half;
         i += (size_t)gridDim.x * blockDim.x) {
        const int j = (int)(i % half);
        const size_t row = i / half;
        const int t = (int)(row / n_heads);
        float* v = x + row * hd;
        const size_t p = (size_t)pos[t];
        const float c = cs[p * hd + 2 * j], s = cs[p * hd + 2 * j + 1];
        const float x0 = v[j], x1 = v[j + half];
        v[j] = x0 * c - x1 * s;
        v[j + half] = x0 * s + x1 * c;
    }
}

__global__ void k_kv_append_at(const float* __restrict__ k, const float* __restrict__ v, int T, int n_kv, int hd,
                               int max_ctx, const int* __restrict__ seq, const int* __restrict__ pos,
                               size_t seq_stride, float* __restrict__ kc, float* __restrict__ vc) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)T * n_kv * hd;
         i += (size_t)gridDim.x * blockDim.x) {
        const int dd = (int)(i % hd);
        const int h = (int)((i / hd) % n_kv);
        const int t = (int)(i / ((size_t)hd * n_kv));
        const size_t dst = (size_t)seq[t] * seq_stride + ((size_t)h * max_ctx + pos[t]) * hd + dd;
        kc[dst] = k[i];
        vc[dst] = v[i];
    }
}

// The rows' attention split over positions: CTA (row t, kv head, split p) takes positions
// [p*chunk, min(len, (p+1)*chunk)) for the G query heads of its kv head (one warp each) and writes
// partial states part[(t * n_head + h) * n_split + p]; k_attn_merge then combines the splits of
// each (row, head) in split order: with M = max m_p, out = sum_p e^(m_p - M) acc_p / sum_p e^(m_p - M) l_p.
template <int HD>
__global__ void k_attn_rows_split(const float* __restrict__ q, const float* __restrict__ kc,
                                  const float* __restrict__ vc, const int* __restrict__ seq,
                                  const int* __restrict__ pos, size_t seq_stride, int n_head, int n_kv, int max_ctx,
                                  int chunk, int n_split, float* __restrict__ part) {
    const int t = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z;
    const int G = n_head / n_kv;
    const int warp = threadIdx.x >> 5;
    if (warp >= G) return;
    const int h = kvh * G + warp;
    const int len = pos[t] + 1;
    const int b = sp * chunk, e = min(len, b + chunk);
    const size_t base = (size_t)seq[t] * seq_stride + (size_t)kvh * max_ctx * HD;
    attn_row_part<HD>(q + ((size_t)t * n_head + h) * HD, kc + base, vc + base, b, e,
                      part + (((size_t)t * n_head + h) * n_split + sp) * (HD + 2));
}

// The same split over positions with the split's K and V rows staged once per CTA: one 1-D bulk
// copy each (a kv head's positions are contiguous, [pos][HD] f32) into shared memory, completing on
// an mbarrier; two warps per query head of the kv head then score and accumulate from shared
// memory, warp half 0 the split's 32-position steps 0, 2, .., half 1 steps 1, 3, .. (each its own
// online softmax), and half 0 combines the two states as the merge does (M = max, states scaled
// by e^(m - M)).  Lane l scores position p0 + l reading the K row's float4s in a lane-rotated
// order ((i + l) mod HD/4), so a quarter-warp's loads fall in distinct bank groups, in four
// independent FMA chains (one per float4 component); the query sits in shared memory read in the
// same order.  The V pass reads one row per step, lane l its HD/32 dims.  Chunk =
// attn_rows_chunk() positions; numerics as attn_row_part up to the f32 summation order.
template <int HD>
__global__ void __launch_bounds__(512)
    k_attn_rows_tile(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                     const int* __restrict__ seq, const int* __restrict__ pos, size_t seq_stride, int n_head, int n_kv,
                     int max_ctx, int chunk, int n_split, float* __restrict__ part, int* err) {
    constexpr int PL = HD / 32, H4 = HD / 4;
    extern __shared__ __align__(128) uint8_t sm_raw[];
    const int G = n_head / n_kv;
    float* ks = reinterpret_cast<float*>(sm_raw);
    float* vs = ks + (size_t)chunk * HD;
    float* qs = vs + (size_t)chunk * HD;  // [2 G][HD]: each warp's copy of its head's query
    float* xs = qs + (size_t)2 * G * HD;  // [G][HD + 2]: half 1's state for half 0
    __shared__ __align__(8) uint64_t bar;
    const int t = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = warp >> 1, half = warp & 1;
    const int len = pos[t] + 1;
    const int b = sp * chunk, e = min(len, b + chunk), n_pos = e - b;
    const size_t base = (size_t)seq[t] * seq_stride + (size_t)kvh * max_ctx * HD;
    if (n_pos > 0 && threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (n_pos > 0 && threadIdx.x == 0) {
        const uint32_t bytes = (uint32_t)n_pos * HD * 4u;
        mbar_arrive_expect_tx(&bar, 2u * bytes);
        bulk_g2s(ks, kc + base + (size_t)b * HD, bytes, &bar);
        bulk_g2s(vs, vc + base + (size_t)b * HD, bytes, &bar);
    }
    const int h = kvh * G + g;
    float* out = part + (((size_t)t * n_head + h) * n_split + sp) * (HD + 2);
    if (n_pos <= 0) {  // a split past this row's length (the whole CTA): an empty state
        if (half == 0) {
            for (int j = lane; j < HD; j += 32) out[j] = 0.f;
            if (lane == 0) {
                out[HD] = -INFINITY;
                out[HD + 1] = 0.f;
            }
        }
        return;
    }
    float* qw = qs + warp * HD;
    const float* qg = q + ((size_t)t * n_head + h) * HD;
    for (int j = lane; j < HD; j += 32) qw[j] = qg[j];
    __syncwarp();
    bool ok = mbar_wait(&bar, 0u);
    if (!ok) set_err(err, kErrFullWait);
    ok = __all_sync(0xffffffffu, ok);
    const float scale = (float)(1.0 / sqrt((double)HD));
    float m = -INFINITY, l = 0.f, acc[PL];
#pragma unroll
    for (int j = 0; j < PL; j++) acc[j] = 0.f;
    const float4* q4 = reinterpret_cast<const float4*>(qw);
    for (int p0 = 32 * half; ok && p0 < n_pos; p0 += 64) {
        const int pl_i = p0 + lane;
        float s = -INFINITY;
        if (pl_i < n_pos) {
            const float4* k4 = reinterpret_cast<const float4*>(ks + (size_t)pl_i * HD);
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 8
            for (int i = 0; i < H4; i++) {
                const int ii = (i + lane) & (H4 - 1);
                const float4 kv = k4[ii], qv = q4[ii];
                d0 = fmaf(qv.x, kv.x, d0);
                d1 = fmaf(qv.y, kv.y, d1);
                d2 = fmaf(qv.z, kv.z, d2);
                d3 = fmaf(qv.w, kv.w, d3);
            }
            s = ((d0 + d1) + (d2 + d3)) * scale;
        }
        const float m_new = fmaxf(m, warp_max(s));
        const float pl = pl_i < n_pos ? expf(s - m_new) : 0.f;
        const float cf = expf(m - m_new);
        l = l * cf + warp_sum(pl);
#pragma unroll
        for (int j = 0; j < PL; j++) acc[j] *= cf;
        const int n = min(32, n_pos - p0);
#pragma unroll 8
        for (int jj = 0; jj < n; jj++) {
            const float pj = __shfl_sync(0xffffffffu, pl, jj);
            const float* vr = vs + (size_t)(p0 + jj) * HD + lane * PL;
#pragma unroll
            for (int j = 0; j < PL; j++) acc[j] = fmaf(pj, vr[j], acc[j]);
        }
        m = m_new;
    }
    // half 1 hands its state to half 0 (an empty state when the split has <= 32 positions)
    float* xw = xs + (size_t)g * (HD + 2);
    if (half == 1) {
#pragma unroll
        for (int j = 0; j < PL; j++) xw[lane * PL + j] = acc[j];
        if (lane == 0) {
            xw[HD] = m;
            xw[HD + 1] = l;
        }
    }
    __syncthreads();
    if (half == 1) return;
    const float m1 = xw[HD], l1 = xw[HD + 1];
    const float M = fmaxf(m, m1);
    const float f0 = expf(m - M), f1 = expf(m1 - M);
#pragma unroll
    for (int j = 0; j < PL; j++) out[lane * PL + j] = acc[j] * f0 + xw[lane * PL + j] * f1;
    if (lane == 0) {
        out[HD] = M;
        out[HD + 1] = l * f0 + l1 * f1;
    }
}

// one warp per (row, head): lane owns HD/32 output dims
template <int HD>
__global__ void k_attn_merge(const float* __restrict__ part, const int* __restrict__ pos, int T, int n_head, int chunk,
                             int n_split, float* __restrict__ out, __half* __restrict__ out16, int split) {
    constexpr int PL = HD / 32;
    const int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (w >= T * n_head) return;
    const int t = w / n_head, h = w % n_head;
    const int used = (pos[t] + 1 + chunk - 1) / chunk;  // splits holding positions
    const float* pp = part + ((size_t)t * n_head + h) * n_split * (HD + 2);
    // the maximum over the splits: lane s reads splits s, s + 32, ... (all loads in flight)
    float M = -INFINITY;
    for (int sp = lane; sp < used; sp += 32) M = fmaxf(M, pp[sp * (HD + 2) + HD]);
    M = warp_max(M);
    // the weighted sums in split order, eight splits' loads issued before their first use
    float acc[PL], L = 0.f;
#pragma unroll
    for (int j = 0; j < PL; j++) acc[j] = 0.f;
    for (int s0 = 0; s0 < used; s0 += 8) {
        float mv[8], lv[8], av[8][PL];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const bool live = s0 + u < used;
            const float* q = pp + (size_t)(s0 + u) * (HD + 2);
            mv[u] = live ? q[HD] : -INFINITY;
            lv[u] = live ? q[HD + 1] : 0.f;
#pragma unroll
            for (int j = 0; j < PL; j++) av[u][j] = live ? q[lane * PL + j] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            if (s0 + u >= used) break;
            const float f = expf(mv[u] - M);
            L += f * lv[u];
#pragma unroll
            for (int j = 0; j < PL; j++) acc[j] = fmaf(f, av[u][j], acc[j]);
        }
    }
    const size_t o0 = ((size_t)t * n_head + h) * HD + lane * PL;
#pragma unroll
    for (int j = 0; j < PL; j++) {
        const float r = acc[j] / L;
        out[o0 + j] = r;
        if (out16) store_f16_split(out16, (size_t)T * n_head * HD, o0 + j, r, split);
    }
}

// one short-conv step per row with its sequence's 2-tap state (lfm2-engine.js:282-325);
// state of sequence s at state + s * state_stride: [s0 | s1] of E floats
__global__ void k_conv_rows_at(const float* __restrict__ bcx, const float* __restrict__ w, float* __restrict__ state,
                               size_t state_stride, const int* __restrict__ seq, int T, int E, float* __restrict__ y) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)T * E;
         i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / E), c = (int)(i % E);
        float* st = state + (size_t)seq[t] * state_stride;
        const float s0 = st[c], s1 = st[E + c];
        const float k0 = w[c * 3], k1 = w[c * 3 + 1], k2 = w[c * 3 + 2];
        const float* r = bcx + (size_t)t * 3 * E;
        const float bx = r[c] * r[2 * E + c];
        const float co = k0 * s0 + k1 * s1 + k2 * bx;
        y[i] = r[E + c] * co;
        st[c] = s1;
        st[E + c] = bx;
    }
}

// first-max argmax of each row of logits [T][V] (sampleGreedy, tensor.js:231-237), the id
// *suppress (>= 0) left out (thinking suppression, tensor.js:247-248), in two passes: CTA
// (row t, part p) reduces a slice of the row to a packed key (argmax_key: the larger value, then the
// lower index, wins), then one warp per row takes the largest of the kArgmaxParts keys
constexpr int kArgmaxThreads = 256;
constexpr int kArgmaxParts = 32;
__global__ void __launch_bounds__(kArgmaxThreads)
    k_argmax_rows_part(const float* __restrict__ logits, int V, const int* __restrict__ suppress, int idx0,
                       unsigned long long* __restrict__ keys) {
    const int t = blockIdx.x, p = blockIdx.y;
    const int skip = suppress ? *suppress : -1;
    const int per = (V + kArgmaxParts - 1) / kArgmaxParts;
    const int b = p * per, e = min(V, b + per);
    const float* r = logits + (size_t)t * V;
    unsigned long long best = 0ull;
    for (int i = b + threadIdx.x; i < e; i += blockDim.x)
        if (i != skip) {
            const unsigned long long k = argmax_key(r[i], idx0 + i);  // idx0: a vocab shard's first row
            best = k > best ? k : best;
        }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    __shared__ unsigned long long ks[kArgmaxThreads / 32];
    if ((threadIdx.x & 31) == 0) ks[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long m = 0ull;
        for (int w = 0; w < kArgmaxThreads / 32; w++) m = ks[w] > m ? ks[w] : m;
        keys[(size_t)t * kArgmaxParts + p] = m;
    }
}

__global__ void k_argmax_rows_final(const unsigned long long* __restrict__ keys, int T, int* __restrict__ out) {
    const int t = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    unsigned long long best = keys[(size_t)t * kArgmaxParts + lane];  // kArgmaxParts == 32 lanes
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if (lane == 0) out[t] = argmax_key_index(best);
}
static_assert(kArgmaxParts == 32, "one key per lane in k_argmax_rows_final");

}  // namespace

void launch_embed_rows(const DTensor& E, const int* tok, int T, int n_vocab, float* out, cudaStream_t s) {
    k_embed_rows<<<grid_n((size_t)T * E.K), 256, 0, s>>>(E.qs, E.d, (int)E.K, tok, T, n_vocab, out);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_rope_rows(float* x, int T, int n_heads, int hd, const float* cs, int pos0, cudaStream_t s) {
    k_rope_rows<<<grid_n((size_t)T * n_heads * hd / 2), 256, 0, s>>>(x, T, n_heads, hd, cs, pos0);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_kv_append(const float* k, const float* v, int T, int n_kv, int hd, int max_ctx, int pos0, float* kc,
                      float* vc, cudaStream_t s) {
    k_kv_append<<<grid_n((size_t)T * n_kv * hd), 256, 0, s>>>(k, v, T, n_kv, hd, max_ctx, pos0, kc, vc);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_conv_prefill(const float* bcx, const float* w, float* state, int T, int E, float* y, cudaStream_t s) {
    k_conv_prefill<<<(E + 127) / 128, 128, 0, s>>>(bcx, w, state, T, E, y);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_add_rows(float* x, const float* d, size_t n, cudaStream_t s) {
    k_add_rows<<<grid_n(n), 256, 0, s>>>(x, d, n);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_swiglu_rows(const float* g, const float* u, size_t n, float* h, cudaStream_t s) {
    k_swiglu_rows<<<grid_n(n), 256, 0, s>>>(g, u, n, h);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_swiglu_rows_f16(const float* g, const float* u, size_t n, __half* y16, cudaStream_t s) {
    if (n == 0) return;
    k_swiglu_rows_f16<<<grid_n(n), 256, 0, s>>>(g, u, n, y16, gemm_exact() ? 1 : 0);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_add_rmsnorm_rows(float* x, const float* d, int64_t n_rows, int n, const float* w, float eps, float* y,
                             __half* y16, cudaStream_t s) {
    if (n_rows <= 0) return;
    // the thread count launch_rmsnorm uses for rows of n values (the same sums)
    const int threads = n >= 2048 ? 1024 : (n >= 512 ? 256 : 128);
    k_add_rmsnorm_rows<<<(unsigned)n_rows, threads, 0, s>>>(x, d, n, w, eps, y, y16, (size_t)n_rows * n,
                                                            gemm_exact() ? 1 : 0);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_qk_norm_rope_rows(float* q, const float* k, const float* v, int T, int n_head, int n_kv, int hd,
                              const float* qw, const float* kw, float eps, const float* cs, const int* seq,
                              const int* pos, int pos0, size_t seq_stride, int max_ctx, float* kc, float* vc,
                              cudaStream_t s) {
    QQ_CHECK(hd >= 2 && hd <= 128 && hd % 2 == 0, -4, "head norm + RoPE: head_dim must be even and at most 128");
    if (T <= 0) return;
    k_qk_norm_rope_rows<<<dim3((unsigned)T, (unsigned)(n_head + n_kv)), 128, 0, s>>>(
        q, k, v, n_head, n_kv, hd, qw, kw, eps, cs, seq, pos, pos0, seq_stride, max_ctx, kc, vc);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_attn_prefill(const float* q, const float* kc, const float* vc, int T, int pos0, int n_head, int n_kv,
                         int hd, int max_ctx, float* out, cudaStream_t s) {
    const int G = n_head / n_kv;
    QQ_CHECK(G >= 1 && G <= 32 && n_head % n_kv == 0, -4, "prefill attention: unsupported head grouping");
    if (T <= 0) return;
    // tensor cores (kernels_attn_tc.cu) unless QQ3_ATTN_TC=0
    static const bool tc_off = [] {
        const char* e = getenv("QQ3_ATTN_TC");
        return e && atoi(e) == 0;
    }();
    if (!tc_off && attn_prefill_tc_supported(n_head, n_kv, hd)) {
        launch_attn_prefill_tc(q, kc, vc, T, pos0, n_head, n_kv, hd, max_ctx, out, s);
        return;
    }
    if (G <= kPfWarps * kPfRows && (kPfWarps * kPfRows) % G == 0 && !tiled_attention_off()) {
        // query tiles: K / V read once per 64 query rows (k_attn_prefill_tile)
        const int QT = kPfWarps * kPfRows / G;
        dim3 grid((unsigned)((T + QT - 1) / QT), (unsigned)n_kv);
        const size_t smem = ((size_t)hd * (kPfKeys + 1) + (size_t)kPfKeys * hd + (size_t)kPfWarps * hd * kPfRows +
                             (size_t)kPfWarps * kPfKeys * kPfRows) * sizeof(float);
        if (hd == 64) {
            if (first_use_on_device(reinterpret_cast<const void*>(k_attn_prefill_tile<64>)))
                QQ_CUDA_TRY(cudaFuncSetAttribute(k_attn_prefill_tile<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem));
            k_attn_prefill_tile<64><<<grid, kPfWarps * 32, smem, s>>>(q, kc, vc, T, pos0, n_head, n_kv, max_ctx, out);
        } else if (hd == 128) {
            if (first_use_on_device(reinterpret_cast<const void*>(k_attn_prefill_tile<128>)))
                QQ_CUDA_TRY(cudaFuncSetAttribute(k_attn_prefill_tile<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem));
            k_attn_prefill_tile<128><<<grid, kPfWarps * 32, smem, s>>>(q, kc, vc, T, pos0, n_head, n_kv, max_ctx, out);
        } else {
            QQ_CHECK(false, -4, "prefill attention: head_dim must be 64 or 128");
        }
        QQ_CUDA_TRY(cudaGetLastError());
        return;
    }
    dim3 grid((unsigned)T, (unsigned)n_kv);
    if (hd == 64) k_attn_prefill<64><<<grid, 32 * G, 0, s>>>(q, kc, vc, pos0, n_head, n_kv, max_ctx, out);
    else if (hd == 128) k_attn_prefill<128><<<grid, 32 * G, 0, s>>>(q, kc, vc, pos0, n_head, n_kv, max_ctx, out);
    else QQ_CHECK(false, -4, "prefill attention: head_dim must be 64 or 128");
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_rope_rows_at(float* x, int T, int n_heads, int hd, const float* cs, const int* pos, cudaStream_t s) {
    k_rope_rows_at<<<grid_n((size_t)T * n_heads * hd / 2), 256, 0, s>>>(x, T, n_heads, hd, cs, pos);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_kv_append_at(const float* k, const float* v, int T, int n_kv, int hd, int max_ctx, const int* seq,
                         const int* pos, size_t seq_stride, float* kc, float* vc, cudaStream_t s) {
    k_kv_append_at<<<grid_n((size_t)T * n_kv * hd), 256, 0, s>>>(k, v, T, n_kv, hd, max_ctx, seq, pos, seq_stride,
                                                                   kc, vc);
    QQ_CUDA_TRY(cudaGetLastError());
}

int attn_rows_chunk() { return 64; }



size_t attn_rows_part_floats(int T, int n_head, int hd, int max_ctx) {
    const int n_split = (max_ctx + attn_rows_chunk() - 1) / attn_rows_chunk();
    return (size_t)T * n_head * n_split * (hd + 2);
}

void launch_attn_rows_split(const float* q, const float* kc, const float* vc, int T, const int* seq, const int* pos,
                            int max_len, size_t seq_stride, int n_head, int n_kv, int hd, int max_ctx, float* part,
                            float* out, cudaStream_t s, __half* out16) {
    const int G = n_head / n_kv;
    QQ_CHECK(G >= 1 && G <= 32 && n_head % n_kv == 0, -4, "batched attention: unsupported head grouping");
    if (T <= 0) return;
    const int chunk = attn_rows_chunk(), n_split = (max_ctx + chunk - 1) / chunk;
    QQ_CHECK(n_split <= 65535 && max_len >= 1 && max_len <= max_ctx, -4, "batched attention: bad context length");
    // splits up to the longest row (max_len positions); a split past a row's own length writes an
    // empty state, and the merge reads only the splits that hold positions of its row
    dim3 grid((unsigned)T, (unsigned)n_kv, (unsigned)((max_len + chunk - 1) / chunk));
    const unsigned mg = (unsigned)(((size_t)T * n_head * 32 + 255) / 256);
    // K and V of a split staged in shared memory once for the G query heads (k_attn_rows_tile),
    // up to 8 heads per kv head; the per-warp global-memory form otherwise
    const bool tile = G <= 8 && !tiled_attention_off();
    const int split = gemm_exact() ? 1 : 0;
    // K, V, two query copies per head, half 1's states (k_attn_rows_tile)
    auto tile_smem = [&](int g) { return ((size_t)2 * chunk * hd + (size_t)2 * g * hd + (size_t)g * (hd + 2)) * sizeof(float); };
    const size_t smem = tile_smem(G);
    // the attribute is set once per device, to the largest size any head grouping needs (G = 8):
    // a launch may not ask for more dynamic shared memory than the attribute allows
    const size_t smem_max = tile_smem(8);
    if (hd == 64) {
        if (tile) {
            if (first_use_on_device(reinterpret_cast<const void*>(k_attn_rows_tile<64>)))
                QQ_CUDA_TRY(cudaFuncSetAttribute(k_attn_rows_tile<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem_max));
            k_attn_rows_tile<64><<<grid, 64 * G, smem, s>>>(q, kc, vc, seq, pos, seq_stride, n_head, n_kv, max_ctx,
                                                            chunk, n_split, part, kernel_err_ptr());
        } else {
            k_attn_rows_split<64><<<grid, 32 * G, 0, s>>>(q, kc, vc, seq, pos, seq_stride, n_head, n_kv, max_ctx, chunk,
                                                          n_split, part);
        }
        QQ_CUDA_TRY(cudaGetLastError());
        k_attn_merge<64><<<mg, 256, 0, s>>>(part, pos, T, n_head, chunk, n_split, out, out16, split);
    } else if (hd == 128) {
        if (tile) {
            if (first_use_on_device(reinterpret_cast<const void*>(k_attn_rows_tile<128>)))
                QQ_CUDA_TRY(cudaFuncSetAttribute(k_attn_rows_tile<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem_max));
            k_attn_rows_tile<128><<<grid, 64 * G, smem, s>>>(q, kc, vc, seq, pos, seq_stride, n_head, n_kv, max_ctx,
                                                             chunk, n_split, part, kernel_err_ptr());
        } else {
            k_attn_rows_split<128><<<grid, 32 * G, 0, s>>>(q, kc, vc, seq, pos, seq_stride, n_head, n_kv, max_ctx,
                                                           chunk, n_split, part);
        }
        QQ_CUDA_TRY(cudaGetLastError());
        k_attn_merge<128><<<mg, 256, 0, s>>>(part, pos, T, n_head, chunk, n_split, out, out16, split);
    } else {
        QQ_CHECK(false, -4, "batched attention: head_dim must be 64 or 128");
    }
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_conv_rows_at(const float* bcx, const float* w, float* state, size_t state_stride, const int* seq, int T,
                         int E, float* y, cudaStream_t s) {
    k_conv_rows_at<<<grid_n((size_t)T * E), 256, 0, s>>>(bcx, w, state, state_stride, seq, T, E, y);
    QQ_CUDA_TRY(cudaGetLastError());
}

size_t argmax_rows_scratch_bytes(int T) { return (size_t)T * kArgmaxParts * sizeof(unsigned long long); }

void launch_argmax_rows(const float* logits, int T, int V, const int* suppress, void* scratch, int* out,
                        cudaStream_t s) {
    if (T <= 0) return;
    unsigned long long* keys = static_cast<unsigned long long*>(scratch);
    k_argmax_rows_part<<<dim3((unsigned)T, kArgmaxParts), kArgmaxThreads, 0, s>>>(logits, V, suppress, 0, keys);
    QQ_CUDA_TRY(cudaGetLastError());
    k_argmax_rows_final<<<(unsigned)((T * 32 + 255) / 256), 256, 0, s>>>(keys, T, out);
    QQ_CUDA_TRY(cudaGetLastError());
}

namespace {
// out[t] = the index of the largest key of row t over the G ranks' kArgmaxParts keys each
// (keys [G][T][kArgmaxParts], rank-major as an all-gather leaves them)
__global__ void k_argmax_merge(const unsigned long long* __restrict__ keys, int G, int T, int* __restrict__ out) {
    const int t = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    unsigned long long best = 0ull;
    for (int g = 0; g < G; g++) {
        const unsigned long long k = keys[((size_t)g * T + t) * kArgmaxParts + lane];
        best = k > best ? k : best;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if (lane == 0) out[t] = argmax_key_index(best);
}
}  // namespace

void launch_argmax_rows_keys(const float* logits, int T, int V, const int* suppress, int idx0, void* keys,
                             cudaStream_t s) {
    if (T <= 0) return;
    k_argmax_rows_part<<<dim3((unsigned)T, kArgmaxParts), kArgmaxThreads, 0, s>>>(
        logits, V, suppress, idx0, static_cast<unsigned long long*>(keys));
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_argmax_merge(const void* keys, int G, int T, int* out, cudaStream_t s) {
    if (T <= 0) return;
    k_argmax_merge<<<(unsigned)((T * 32 + 255) / 256), 256, 0, s>>>(static_cast<const unsigned long long*>(keys), G,
                                                                     T, out);
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace qq3
