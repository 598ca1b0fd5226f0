/*
 * qq3_oracle.c -- CPU restatement of the QwenQwen3.js CPU inference path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker for libqq3cuda.so, never part of it).
 * Parity status: UNPINNED -- the reference is JavaScript with no tests or golden
 * vectors, and no JS runtime exists here; see qq3_oracle.h for the rules this
 * restatement follows (double accumulators, float rounding at Float32Array
 * stores, JS evaluation order, no FMA contraction).
 *
 * Citations are reference file:line (paths inside the QwenQwen3.js project).
 */
#include "qq3_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 1;

void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int orc_get_threads(void) { return g_threads; }

/* DataView.getFloat16(off, true): exact binary16 -> double (tensor.js:21-23). */
double orc_f16_to_double(uint16_t h) {
    int sign = h >> 15;
    int e = (h >> 10) & 0x1f;
    int m = h & 0x3ff;
    double v;
    if (e == 0) v = ldexp((double)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = ldexp((double)(m | 0x400), e - 25);
    return sign ? -v : v;
}

/* every binary16 value as a double (the values orc_f16_to_double gives), filled when the
 * library is loaded */
static double g_f16_tab[65536];
__attribute__((constructor)) static void f16_tab_fill(void) {
    for (int h = 0; h < 65536; h++) g_f16_tab[h] = orc_f16_to_double((uint16_t)h);
}
static inline double rd_f16(const uint8_t* p) { return g_f16_tab[p[0] | (p[1] << 8)]; }
static float rd_f32(const uint8_t* p) { float f; memcpy(&f, p, 4); return f; }

/* matmulQ80xF32 (tensor.js:26-53): output[c] = sum_b sum_i (x*q)*d, f64 sum, f32 store.
 * Four columns are walked together so that their four f64 sums form independent dependency
 * chains; each column's own sequence of operations (and so its result) is the JS loop's. */
static void matmul_q8(const uint8_t* w, int64_t in_dim, int64_t out_dim, const float* x, float* y) {
    const int64_t bpc = (in_dim + 31) / 32;
    const int64_t n4 = (out_dim + 3) / 4;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && out_dim >= 64)
    for (int64_t c4 = 0; c4 < n4; c4++) {
        const int64_t c0 = c4 * 4;
        if (c0 + 4 > out_dim) {
            for (int64_t c = c0; c < out_dim; c++) {
                double dot = 0;
                const uint8_t* col = w + (size_t)c * bpc * 34;
                for (int64_t b = 0; b < bpc; b++) {
                    const uint8_t* blk = col + b * 34;
                    const double d = rd_f16(blk);
                    const int8_t* qs = (const int8_t*)(blk + 2);
                    const int64_t eb = b * 32;
                    for (int i = 0; i < 32 && eb + i < in_dim; i++) dot += ((double)x[eb + i] * (double)qs[i]) * d;
                }
                y[c] = (float)dot;
            }
            continue;
        }
        double dot0 = 0, dot1 = 0, dot2 = 0, dot3 = 0;
        const uint8_t* col0 = w + (size_t)c0 * bpc * 34;
        const size_t cs = (size_t)bpc * 34;
        for (int64_t b = 0; b < bpc; b++) {
            const uint8_t* b0 = col0 + b * 34;
            const double d0 = rd_f16(b0), d1 = rd_f16(b0 + cs), d2 = rd_f16(b0 + 2 * cs), d3 = rd_f16(b0 + 3 * cs);
            const int8_t *q0 = (const int8_t*)(b0 + 2), *q1 = (const int8_t*)(b0 + cs + 2),
                         *q2 = (const int8_t*)(b0 + 2 * cs + 2), *q3 = (const int8_t*)(b0 + 3 * cs + 2);
            const int64_t eb = b * 32;
            for (int i = 0; i < 32 && eb + i < in_dim; i++) {
                const double xi = (double)x[eb + i];
                dot0 += (xi * (double)q0[i]) * d0;
                dot1 += (xi * (double)q1[i]) * d1;
                dot2 += (xi * (double)q2[i]) * d2;
                dot3 += (xi * (double)q3[i]) * d3;
            }
        }
        y[c0] = (float)dot0;
        y[c0 + 1] = (float)dot1;
        y[c0 + 2] = (float)dot2;
        y[c0 + 3] = (float)dot3;
    }
}

/* matmulF32xF32 (tensor.js:469-482). */
static void matmul_f32(const uint8_t* w, int64_t in_dim, int64_t out_dim, const float* x, float* y) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && out_dim >= 64)
    for (int64_t c = 0; c < out_dim; c++) {
        double dot = 0;
        const uint8_t* base = w + (size_t)c * in_dim * 4;
        for (int64_t i = 0; i < in_dim; i++) dot += (double)x[i] * (double)rd_f32(base + i * 4);
        y[c] = (float)dot;
    }
}

/* ---- k-quants (tensor.js:267-664) ----------------------------------------------------------
 * Column c of a [ne0, ne1] tensor is ceil(ne0 / 256) contiguous superblocks; element e of a
 * superblock is the JS expression below evaluated in doubles (JS numbers, the same operation
 * order), its f16 fields read exactly.  The JS layouts are restated as they are written there. */
#define ORC_QK_K 256

static int kq_block_bytes(int type) {
    switch (type) {
        case ORC_TYPE_Q2_K: return 84;   /* tensor.js:271 */
        case ORC_TYPE_Q3_K: return 110;  /* tensor.js:272 */
        case ORC_TYPE_Q4_K: return 144;  /* tensor.js:273 */
        case ORC_TYPE_Q5_K: return 176;  /* tensor.js:274 */
        case ORC_TYPE_Q6_K: return 210;  /* tensor.js:275 */
        default: return 0;
    }
}

static int is_kquant(int type) { return kq_block_bytes(type) != 0; }

/* _q4kGetScaleMin (tensor.js:278-289): 6-bit scale and min of sub-block sub of the 12-byte array */
static void q4k_scale_min(const uint8_t* s, int sub, int* sc, int* mn) {
    if (sub < 4) {
        *sc = s[sub] & 63;
        *mn = s[sub + 4] & 63;
    } else {
        const int ss = sub - 4;
        *sc = (s[sub + 4] & 0xF) | ((s[ss] >> 6) << 4);
        *mn = (s[sub + 4] >> 4) | ((s[sub] >> 6) << 4);
    }
}

/* _q3kGetScale (tensor.js:295-302): 6-bit scale minus 32 */
static int q3k_scale(const uint8_t* s, int sub) {
    const int lo4 = (s[sub & 7] >> ((sub >> 3) << 2)) & 0xF;
    const int hi2 = (s[8 + (sub & 3)] >> ((sub >> 2) * 2)) & 0x3;
    return (lo4 | (hi2 << 4)) - 32;
}

/* Element e (0..255) of the superblock at bb, as matmulQ{2..6}KxF32 and _q{2..6}kColumn compute
 * it (tensor.js:304-466, 551-664). */
static double kq_value(int type, const uint8_t* bb, int e) {
    switch (type) {
        case ORC_TYPE_Q2_K: { /* scales[16]@0 qs[64]@16 d@80 dmin@82 (tensor.js:304-334) */
            const double d = rd_f16(bb + 80), dmin = rd_f16(bb + 82);
            const int sb = bb[e >> 4];
            const int q = (bb[16 + (e >> 7) * 32 + ((e >> 4) & 1) * 16 + (e & 15)] >> (((e >> 5) & 3) * 2)) & 0x3;
            return d * (double)(sb & 0xF) * (double)q - dmin * (double)((sb >> 4) & 0xF);
        }
        case ORC_TYPE_Q3_K: { /* hmask[32]@0 qs[64]@32 scales[12]@96 d@108 (tensor.js:336-366) */
            const double d = rd_f16(bb + 108);
            const int scale = q3k_scale(bb + 96, e >> 4);
            const int hbit = (bb[((e >> 4) & 1) * 16 + (e & 15)] >> (e >> 5)) & 1;
            const int low2 = (bb[32 + (e >> 7) * 32 + ((e >> 4) & 1) * 16 + (e & 15)] >> (((e >> 5) & 3) * 2)) & 3;
            return d * (double)scale * (double)((low2 | (hbit << 2)) - 4);
        }
        case ORC_TYPE_Q4_K: { /* d@0 dmin@2 scales[12]@4 qs[128]@16 (tensor.js:368-397) */
            const double d = rd_f16(bb), dmin = rd_f16(bb + 2);
            int sc, mn;
            q4k_scale_min(bb + 4, (e >> 6) * 2 + ((e >> 5) & 1), &sc, &mn);
            const int qb = bb[16 + (e >> 6) * 32 + (e & 31)];
            const int q4 = ((e >> 5) & 1) ? (qb >> 4) & 0xF : qb & 0xF;
            return d * (double)sc * (double)q4 - dmin * (double)mn;
        }
        case ORC_TYPE_Q5_K: { /* d@0 dmin@2 scales[12]@4 qh[32]@16 qs[128]@48 (tensor.js:399-430) */
            const double d = rd_f16(bb), dmin = rd_f16(bb + 2);
            const int sub = (e >> 6) * 2 + ((e >> 5) & 1);
            int sc, mn;
            q4k_scale_min(bb + 4, sub, &sc, &mn);
            const int hbit = (bb[16 + (e & 31)] >> sub) & 1;
            const int qb = bb[48 + (e >> 6) * 32 + (e & 31)];
            const int low4 = ((e >> 5) & 1) ? (qb >> 4) & 0xF : qb & 0xF;
            return d * (double)sc * (double)(low4 | (hbit << 4)) - dmin * (double)mn;
        }
        case ORC_TYPE_Q6_K: { /* ql[128]@0 qh[64]@128 scales[16]@192 d@208 (tensor.js:432-466) */
            const double d = rd_f16(bb + 208);
            const int ql = bb[(e >> 7) * 64 + ((e >> 5) & 1) * 32 + (e & 31)];
            const int low4 = ((e >> 6) & 1) ? (ql >> 4) & 0xF : ql & 0xF;
            const int high2 = (bb[128 + (e >> 7) * 32 + (e & 31)] >> (((e >> 5) & 3) * 2)) & 0x3;
            const int sidx = (e >> 7) * 8 + ((e >> 5) & 3) * 2 + ((e & 31) >> 4);
            const int scale = (int)(int8_t)bb[192 + sidx];
            return d * (double)scale * (double)((low4 | (high2 << 4)) - 32);
        }
        default: abort();
    }
}

/* matmulQ{2..6}KxF32 (tensor.js:304-466): dot += input * weight in doubles, f32 store. */
static void matmul_kq(int type, const uint8_t* w, int64_t in_dim, int64_t out_dim, const float* x, float* y) {
    const int64_t bpc = (in_dim + ORC_QK_K - 1) / ORC_QK_K;
    const int bs = kq_block_bytes(type);
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && out_dim >= 64)
    for (int64_t c = 0; c < out_dim; c++) {
        double dot = 0;
        for (int64_t b = 0; b < bpc; b++) {
            const uint8_t* bb = w + ((size_t)c * bpc + b) * bs;
            const int64_t eb = b * ORC_QK_K;
            const int64_t n = in_dim - eb < ORC_QK_K ? in_dim - eb : ORC_QK_K;
            for (int e = 0; e < n; e++) dot += (double)x[eb + e] * kq_value(type, bb, e);
        }
        y[c] = (float)dot;
    }
}

/* _q{2..6}kColumn (tensor.js:525-664): column c as floats (each value stored into a Float32Array). */
static void kq_column(int type, const uint8_t* w, int64_t out_dim, int64_t c, float* out) {
    const int64_t bpc = (out_dim + ORC_QK_K - 1) / ORC_QK_K;
    const int bs = kq_block_bytes(type);
    for (int64_t b = 0; b < bpc; b++) {
        const uint8_t* bb = w + ((size_t)c * bpc + b) * bs;
        const int64_t eb = b * ORC_QK_K;
        const int64_t n = out_dim - eb < ORC_QK_K ? out_dim - eb : ORC_QK_K;
        for (int e = 0; e < n; e++) out[eb + e] = (float)kq_value(type, bb, e);
    }
}

/* matmulGeneric (tensor.js:485-496): F32, Q8_0 and the k-quants; a 3-D tensor is treated as its
 * first [ne0, ne1] matrix, as a meta object with that shape would be. */
void orc_matmul(const orc_tensor* w, const float* x, float* y) {
    if (w->type == ORC_TYPE_Q8_0) matmul_q8(w->data, w->ne[0], w->ne[1], x, y);
    else if (w->type == ORC_TYPE_F32) matmul_f32(w->data, w->ne[0], w->ne[1], x, y);
    else if (is_kquant(w->type)) matmul_kq(w->type, w->data, w->ne[0], w->ne[1], x, y);
    else abort();
}

/* M independent matmulGeneric calls (the reference has M = 1 only). */
void orc_matmul_rows(const orc_tensor* w, const float* x, int64_t m, float* y) {
    for (int64_t r = 0; r < m; r++) orc_matmul(w, x + r * w->ne[0], y + r * w->ne[1]);
}

/* embeddingLookupQ80 / embeddingLookupGeneric (tensor.js:56-77, 499-523). */
void orc_embedding(const orc_tensor* w, int32_t token, float* out) {
    const int64_t out_dim = w->ne[0];
    if (w->type == ORC_TYPE_F32) {
        const uint8_t* base = w->data + (size_t)token * out_dim * 4;
        for (int64_t i = 0; i < out_dim; i++) out[i] = rd_f32(base + i * 4);
        return;
    }
    if (is_kquant(w->type)) {  /* embeddingLookupGeneric -> _lookupKQuantColumn (tensor.js:511-549) */
        kq_column(w->type, w->data, out_dim, token, out);
        return;
    }
    if (w->type != ORC_TYPE_Q8_0) abort();
    const int64_t bpc = (out_dim + 31) / 32;
    const uint8_t* col = w->data + (size_t)token * bpc * 34;
    for (int64_t b = 0; b < bpc; b++) {
        const uint8_t* blk = col + b * 34;
        const double d = rd_f16(blk);
        const int8_t* qs = (const int8_t*)(blk + 2);
        for (int i = 0; i < 32 && b * 32 + i < out_dim; i++) out[b * 32 + i] = (float)((double)qs[i] * d);
    }
}

/* Full dequantisation of a Q8_0 tensor in storage order, element value q*d as the
 * column readers of tensor.js:56-77 and 80-100 produce it (exact in f32). */
void orc_dequant(const orc_tensor* w, float* out) {
    int64_t n = 1;
    for (int i = 0; i < w->n_dims; i++) n *= w->ne[i];
    if (w->type == ORC_TYPE_F32) { memcpy(out, w->data, (size_t)n * 4); return; }
    if (is_kquant(w->type)) {  /* every column through its column reader, in storage order */
        for (int64_t c = 0; c < n / w->ne[0]; c++) kq_column(w->type, w->data, w->ne[0], c, out + c * w->ne[0]);
        return;
    }
    const int64_t nb = (n + 31) / 32;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = w->data + b * 34;
        const double d = rd_f16(blk);
        const int8_t* qs = (const int8_t*)(blk + 2);
        for (int i = 0; i < 32 && b * 32 + i < n; i++) out[b * 32 + i] = (float)((double)qs[i] * d);
    }
}

/* _readWeightF32 (tensor.js:80-100): element i of a 1-D F32 or Q8_0 weight. */
static double weight_at(const orc_tensor* w, int64_t i) {
    if (w->type == ORC_TYPE_F32) return (double)rd_f32(w->data + i * 4);
    if (w->type == ORC_TYPE_Q8_0) {
        const uint8_t* blk = w->data + (i / 32) * 34;
        /* stored into a Float32Array: q*d rounded to f32 (exact) */
        return (double)(float)((double)((const int8_t*)(blk + 2))[i % 32] * rd_f16(blk));
    }
    abort();
}

/* rmsnorm (tensor.js:103-114), in place. */
void orc_rmsnorm(float* x, int64_t n, const orc_tensor* w, double eps) {
    double ss = 0;
    for (int64_t i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    const double inv = 1.0 / sqrt(ss / (double)n + eps);
    for (int64_t i = 0; i < n; i++) x[i] = (float)((weight_at(w, i) * (double)x[i]) * inv);
}

/* perHeadRMSNorm (tensor.js:117-129). */
void orc_per_head_rmsnorm(float* x, int n_heads, int head_dim, const orc_tensor* w, double eps) {
    for (int h = 0; h < n_heads; h++) {
        float* t = x + (size_t)h * head_dim;
        double ss = 0;
        for (int d = 0; d < head_dim; d++) ss += (double)t[d] * (double)t[d];
        const double inv = 1.0 / sqrt(ss / (double)head_dim + eps);
        for (int d = 0; d < head_dim; d++) t[d] = (float)((weight_at(w, d) * (double)t[d]) * inv);
    }
}

/* applyRoPE, split-half (tensor.js:132-147). */
void orc_rope(float* x, int n_heads, int head_dim, int position, double base) {
    const int half = head_dim >> 1;
    for (int h = 0; h < n_heads; h++) {
        float* t = x + (size_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            const double freq = 1.0 / pow(base, (double)i / (double)half);
            const double theta = (double)position * freq;
            const double c = cos(theta), s = sin(theta);
            const double x0 = t[i], x1 = t[i + half];
            t[i] = (float)(x0 * c - x1 * s);
            t[i + half] = (float)(x0 * s + x1 * c);
        }
    }
}

/* softmaxInPlace (tensor.js:150-164): exp stored to f32 before it is summed. */
void orc_softmax(float* a, int64_t start, int64_t end) {
    float mx = a[start];
    for (int64_t i = start + 1; i < end; i++)
        if (a[i] > mx) mx = a[i];
    double sum = 0;
    for (int64_t i = start; i < end; i++) {
        a[i] = (float)exp((double)a[i] - (double)mx);
        sum += a[i];
    }
    const double inv = 1.0 / sum;
    for (int64_t i = start; i < end; i++) a[i] = (float)((double)a[i] * inv);
}

/* siluInPlace / mulInPlace / addVec (tensor.js:167-185). */
void orc_silu(float* a, int64_t n) {
    for (int64_t i = 0; i < n; i++) a[i] = (float)((double)a[i] * (1.0 / (1.0 + exp(-(double)a[i]))));
}
void orc_mul(float* a, const float* b, int64_t n) {
    for (int64_t i = 0; i < n; i++) a[i] = (float)((double)a[i] * (double)b[i]);
}
void orc_add(float* a, const float* b, int64_t n) {
    for (int64_t i = 0; i < n; i++) a[i] = (float)((double)a[i] + (double)b[i]);
}

/* sampleGreedy (tensor.js:231-237): first maximum wins. */
int32_t orc_sample_greedy(const float* logits, int64_t n) {
    int64_t mi = 0;
    for (int64_t i = 1; i < n; i++)
        if (logits[i] > logits[mi]) mi = i;
    return (int32_t)mi;
}

/* sampleWithThinkControl, mode 'suppress', temperature 0 (tensor.js:244-265). */
int32_t orc_sample_suppress(float* logits, int64_t n, int32_t think_id) {
    if (think_id >= 0 && think_id < n) logits[think_id] = -INFINITY;
    return orc_sample_greedy(logits, n);
}

/* _expertSlice (lfm2-engine.js:490-505, qwen3-engine.js:366-381): expert e of a packed
 * [in, hid, E] Q8_0 tensor viewed as an [in, hid] matrix. */
static orc_tensor expert_slice(const orc_tensor* w, int e) {
    orc_tensor s = *w;
    const int64_t bytes_per_col = ((w->ne[0] + 31) / 32) * 34;
    s.data = w->data + (size_t)e * w->ne[1] * bytes_per_col;
    s.n_dims = 2;
    s.ne[2] = 1;
    return s;
}

/* Lfm2Engine._moEFFN (lfm2-engine.js:413-487) for one token. */
static void lfm2_moe_token(const orc_layer* L, int n_embd, int n_expert, int top_k, const float* normed,
                           float* moe_out, float* routing, const uint8_t* mask, float* logits, float* rw,
                           float* sel, float* g, float* u, float* dn) {
    /* 1. router logits (:418) */
    orc_matmul(&L->t[ORC_ROUTER], normed, logits);
    /* 2. sigmoid stored in a Float32Array (:421-424) */
    for (int e = 0; e < n_expert; e++) rw[e] = (float)(1.0 / (1.0 + exp(-(double)logits[e])));
    /* 3. selection scores = f32 copy + bias (:427-431) */
    for (int e = 0; e < n_expert; e++) sel[e] = rw[e];
    if (L->t[ORC_EXP_BIAS].data)
        for (int e = 0; e < n_expert; e++) sel[e] = (float)((double)sel[e] + weight_at(&L->t[ORC_EXP_BIAS], e));
    /* 4. stable descending sort, take top_k (:434-442): equivalent to repeated first-max selection */
    int top[64];
    double topw[64];
    uint8_t taken[256];
    memset(taken, 0, sizeof(taken));
    for (int k = 0; k < top_k; k++) {
        int best = -1;
        for (int e = 0; e < n_expert; e++) {
            if (taken[e]) continue;
            if (best < 0 || sel[e] > sel[best]) best = e;
        }
        taken[best] = 1;
        top[k] = best;
        topw[k] = rw[best];
    }
    /* 5. normalise with the 1e-6 seed (:445-447) */
    double sum_w = 1e-6;
    for (int k = 0; k < top_k; k++) sum_w += topw[k];
    const double inv = 1.0 / sum_w;
    if (routing) {
        for (int k = 0; k < top_k; k++) {
            routing[k] = (float)top[k];
            routing[top_k + k] = (float)(topw[k] * inv);
        }
        for (int e = 0; e < n_expert; e++) routing[2 * top_k + e] = rw[e];
    }
    /* 6. weighted accumulation in slot order, skipping masked experts without renormalising (:459-484) */
    const int64_t n_ff = L->t[ORC_GATE_EXPS].ne[1];
    for (int64_t i = 0; i < n_embd; i++) moe_out[i] = 0.0f;
    for (int k = 0; k < top_k; k++) {
        const int e = top[k];
        if (mask && mask[e]) continue;
        const double weight = topw[k] * inv;
        orc_tensor gs = expert_slice(&L->t[ORC_GATE_EXPS], e);
        orc_tensor us = expert_slice(&L->t[ORC_UP_EXPS], e);
        orc_tensor ds = expert_slice(&L->t[ORC_DOWN_EXPS], e);
        orc_matmul(&gs, normed, g);
        orc_silu(g, n_ff);
        orc_matmul(&us, normed, u);
        orc_mul(g, u, n_ff);
        orc_matmul(&ds, g, dn);
        for (int64_t i = 0; i < n_embd; i++) moe_out[i] = (float)((double)moe_out[i] + weight * (double)dn[i]);
    }
}

/* Qwen3Engine._moEFFN (qwen3-engine.js:304-362): softmax router, stable top-k of the
 * probabilities, weights renormalised by their sum (no seed, no bias), slot-order accumulation
 * into a Float32Array, masked experts skipped without renormalising. */
static void qwen3_moe_token(const orc_layer* L, int n_embd, int n_expert, int top_k, const float* normed,
                            float* moe_out, float* routing, const uint8_t* mask, float* probs, float* g, float* u,
                            float* dn) {
    /* 1. router logits and softmaxInPlace over them (:306-307) */
    orc_matmul(&L->t[ORC_ROUTER], normed, probs);
    orc_softmax(probs, 0, n_expert);
    /* 2. stable descending sort of (prob, id), first top_k (:310-316) */
    int top[256];
    double topw[256];
    uint8_t taken[256];
    memset(taken, 0, sizeof(taken));
    for (int k = 0; k < top_k; k++) {
        int best = -1;
        for (int e = 0; e < n_expert; e++) {
            if (taken[e]) continue;
            if (best < 0 || probs[e] > probs[best]) best = e;
        }
        taken[best] = 1;
        top[k] = best;
        topw[k] = probs[best];
    }
    /* 3. renormalisation (:318-320) */
    double sum_w = 0;
    for (int k = 0; k < top_k; k++) sum_w += topw[k];
    const double inv = sum_w > 0 ? 1.0 / sum_w : 0.0;
    if (routing) { /* onRouterUpdate record (:323-330): [ids | weights | probs] */
        for (int k = 0; k < top_k; k++) {
            routing[k] = (float)top[k];
            routing[top_k + k] = (float)(topw[k] * inv);
        }
        for (int e = 0; e < n_expert; e++) routing[2 * top_k + e] = probs[e];
    }
    /* 4. experts in slot order (:333-359) */
    const int64_t n_ff = L->t[ORC_GATE_EXPS].ne[1];
    for (int64_t i = 0; i < n_embd; i++) moe_out[i] = 0.0f;
    for (int k = 0; k < top_k; k++) {
        const int e = top[k];
        if (mask && mask[e]) continue;
        const double weight = topw[k] * inv;
        orc_tensor gs = expert_slice(&L->t[ORC_GATE_EXPS], e);
        orc_tensor us = expert_slice(&L->t[ORC_UP_EXPS], e);
        orc_tensor ds = expert_slice(&L->t[ORC_DOWN_EXPS], e);
        orc_matmul(&gs, normed, g);
        orc_silu(g, n_ff);
        orc_matmul(&us, normed, u);
        orc_mul(g, u, n_ff);
        orc_matmul(&ds, g, dn);
        for (int64_t i = 0; i < n_embd; i++) moe_out[i] = (float)((double)moe_out[i] + weight * (double)dn[i]);
    }
}

void orc_lfm2_moe(const orc_layer* layer, int n_embd, int n_expert, int top_k, const float* normed, int64_t T,
                  float* out, float* routing, const uint8_t* mask) {
    const int64_t n_ff = layer->t[ORC_GATE_EXPS].ne[1];
    float* logits = (float*)malloc(sizeof(float) * n_expert * 3);
    float* g = (float*)malloc(sizeof(float) * (n_ff * 2 + n_embd));
    for (int64_t t = 0; t < T; t++) {
        lfm2_moe_token(layer, n_embd, n_expert, top_k, normed + t * n_embd, out + t * n_embd,
                       routing ? routing + t * (2 * top_k + n_expert) : NULL, mask, logits, logits + n_expert,
                       logits + 2 * n_expert, g, g + n_ff, g + 2 * n_ff);
    }
    free(logits);
    free(g);
}

/* ------------------------------------------------------------------------------------ */
/* Engines: Qwen3Engine (qwen3-engine.js:1-301) and Lfm2Engine (lfm2-engine.js:14-505). */

struct orc_model {
    orc_model_desc d;
    orc_layer* layers;
    int* attn_slot;      /* layer -> KV cache slot, -1 for conv layers */
    int* moe_slot;       /* layer -> routing record slot, -1 for dense */
    int n_attn, n_moe, n_ff_max;
    /* KVCache (kv-cache.js:1-53): [slot][kvHead][maxCtx][headDim] */
    float* k_cache;
    float* v_cache;
    float* conv_state;   /* [layer][2][n_embd] (lfm2-engine.js:204-212) */
    float *hidden, *normed, *q, *k, *v, *attn_out, *scores, *ffn, *ffn_tmp, *moe_out, *tmp, *bcx, *bx, *cout, *cy;
    float *r_logits, *r_w, *r_sel, *e_dn;
    uint8_t mask[256];
};

int orc_n_moe_layers(const orc_model* m) { return m->n_moe; }

int orc_model_create(const orc_model_desc* desc, orc_model** out) {
    /* the routers keep their top-k in fixed arrays */
    if (desc->n_expert > 256 || desc->n_expert_used > 64 || desc->n_expert_used > desc->n_expert) return -3;
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    if (!m) return -1;
    m->d = *desc;
    m->layers = (orc_layer*)malloc(sizeof(orc_layer) * desc->n_layers);
    memcpy(m->layers, desc->layers, sizeof(orc_layer) * desc->n_layers);
    m->d.layers = m->layers;
    m->attn_slot = (int*)malloc(sizeof(int) * desc->n_layers);
    m->moe_slot = (int*)malloc(sizeof(int) * desc->n_layers);
    const int E = desc->n_embd;
    int n_ff_max = 0;
    for (int l = 0; l < desc->n_layers; l++) {
        const orc_layer* L = &m->layers[l];
        m->attn_slot[l] = L->is_attn ? m->n_attn++ : -1;
        m->moe_slot[l] = L->is_moe ? m->n_moe++ : -1;
        int64_t f = L->is_moe ? L->t[ORC_GATE_EXPS].ne[1] : (L->t[ORC_FFN_GATE].data ? L->t[ORC_FFN_GATE].ne[1] : 0);
        if (f > n_ff_max) n_ff_max = (int)f;
    }
    m->n_ff_max = n_ff_max;
    const size_t kv = (size_t)(m->n_attn ? m->n_attn : 1) * desc->n_head_kv * desc->max_ctx * desc->head_dim;
    m->k_cache = (float*)calloc(kv, sizeof(float));
    m->v_cache = (float*)calloc(kv, sizeof(float));
    m->conv_state = (float*)calloc((size_t)desc->n_layers * 2 * E, sizeof(float));
    const int nq = desc->n_head * desc->head_dim, nkv = desc->n_head_kv * desc->head_dim;
    const size_t big = (size_t)(E > nq ? E : nq);
    m->hidden = (float*)calloc(big, 4);
    m->normed = (float*)calloc(big, 4);
    m->q = (float*)calloc(nq, 4);
    m->k = (float*)calloc(nkv, 4);
    m->v = (float*)calloc(nkv, 4);
    m->attn_out = (float*)calloc(nq, 4);
    m->scores = (float*)calloc((size_t)desc->n_head * desc->max_ctx, 4);
    m->ffn = (float*)calloc(n_ff_max + 1, 4);
    m->ffn_tmp = (float*)calloc(n_ff_max + 1, 4);
    m->moe_out = (float*)calloc(E, 4);
    m->tmp = (float*)calloc(big, 4);
    m->bcx = (float*)calloc((size_t)3 * E, 4);
    m->bx = (float*)calloc(E, 4);
    m->cout = (float*)calloc(E, 4);
    m->cy = (float*)calloc(E, 4);
    const int ne = desc->n_expert > 0 ? desc->n_expert : 1;
    m->r_logits = (float*)calloc(ne, 4);
    m->r_w = (float*)calloc(ne, 4);
    m->r_sel = (float*)calloc(ne, 4);
    m->e_dn = (float*)calloc(E, 4);
    if (!m->k_cache || !m->v_cache || !m->scores) {
        orc_model_destroy(m);
        return -2;
    }
    *out = m;
    return 0;
}

void orc_model_destroy(orc_model* m) {
    if (!m) return;
    free(m->layers); free(m->attn_slot); free(m->moe_slot);
    free(m->k_cache); free(m->v_cache); free(m->conv_state);
    free(m->hidden); free(m->normed); free(m->q); free(m->k); free(m->v); free(m->attn_out);
    free(m->scores); free(m->ffn); free(m->ffn_tmp); free(m->moe_out); free(m->tmp);
    free(m->bcx); free(m->bx); free(m->cout); free(m->cy);
    free(m->r_logits); free(m->r_w); free(m->r_sel); free(m->e_dn);
    free(m);
}

/* resetState (lfm2-engine.js:216-221); KVCache.reset only rewinds nPast (kv-cache.js:50-52). */
void orc_reset(orc_model* m) {
    memset(m->conv_state, 0, sizeof(float) * (size_t)m->d.n_layers * 2 * m->d.n_embd);
}

int orc_set_expert_mask(orc_model* m, const int32_t* ids, int n) {
    memset(m->mask, 0, sizeof(m->mask));
    for (int i = 0; i < n; i++) {
        if (ids[i] < 0 || ids[i] >= 256) return -1;
        m->mask[ids[i]] = 1;
    }
    return 0;
}

/* KVCache.store (kv-cache.js:16-32) */
static void kv_store(orc_model* m, int slot, int pos, const float* k, const float* v) {
    const int H = m->d.n_head_kv, C = m->d.max_ctx, D = m->d.head_dim;
    for (int h = 0; h < H; h++) {
        const size_t off = (((size_t)slot * H + h) * C + pos) * D;
        memcpy(m->k_cache + off, k + (size_t)h * D, sizeof(float) * D);
        memcpy(m->v_cache + off, v + (size_t)h * D, sizeof(float) * D);
    }
}

/* GQA core: Qwen3Engine._selfAttentionCore (qwen3-engine.js:249-293) which is the same
 * arithmetic as the body of Lfm2Engine._selfAttention (lfm2-engine.js:351-385). */
static void attention_core(orc_model* m, int slot, int position) {
    const int nH = m->d.n_head, nKV = m->d.n_head_kv, D = m->d.head_dim, C = m->d.max_ctx;
    const int seq_len = position + 1;
    const double scale = 1.0 / sqrt((double)D);
    float* scores = m->scores;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int h = 0; h < nH; h++) {
        const int kvh = (int)((double)h * nKV / nH);
        const float* q = m->q + (size_t)h * D;
        float* sc = scores + (size_t)h * seq_len;
        const float* kb = m->k_cache + (((size_t)slot * nKV + kvh) * C) * D;
        for (int p = 0; p < seq_len; p++) {
            double dot = 0;
            for (int d = 0; d < D; d++) dot += (double)q[d] * (double)kb[(size_t)p * D + d];
            sc[p] = (float)(dot * scale);
        }
        orc_softmax(sc, 0, seq_len);
    }
    for (int i = 0; i < nH * D; i++) m->attn_out[i] = 0.0f;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
    for (int h = 0; h < nH; h++) {
        const int kvh = (int)((double)h * nKV / nH);
        float* o = m->attn_out + (size_t)h * D;
        const float* sc = scores + (size_t)h * seq_len;
        const float* vb = m->v_cache + (((size_t)slot * nKV + kvh) * C) * D;
        for (int p = 0; p < seq_len; p++) {
            const float w = sc[p];
            if (w == 0.0f) continue;
            for (int d = 0; d < D; d++) o[d] = (float)((double)o[d] + (double)vb[(size_t)p * D + d] * (double)w);
        }
    }
}

/* Q/K/V projection, QK-norm, RoPE, cache store, attention, wo (qwen3-engine.js:149-179,
 * lfm2-engine.js:329-390).  Result in m->tmp. */
static void self_attention(orc_model* m, const orc_layer* L, int slot, int position) {
    const int nH = m->d.n_head, nKV = m->d.n_head_kv, D = m->d.head_dim;
    orc_matmul(&L->t[ORC_WQ], m->normed, m->q);
    orc_matmul(&L->t[ORC_WK], m->normed, m->k);
    orc_matmul(&L->t[ORC_WV], m->normed, m->v);
    orc_per_head_rmsnorm(m->q, nH, D, &L->t[ORC_Q_NORM], m->d.rms_eps);
    orc_per_head_rmsnorm(m->k, nKV, D, &L->t[ORC_K_NORM], m->d.rms_eps);
    orc_rope(m->q, nH, D, position, m->d.rope_base);
    orc_rope(m->k, nKV, D, position, m->d.rope_base);
    kv_store(m, slot, position, m->k, m->v);
    attention_core(m, slot, position);
    orc_matmul(&L->t[ORC_WO], m->attn_out, m->tmp);
}

/* Lfm2Engine._shortConv (lfm2-engine.js:282-325).  Result in m->tmp. */
static void short_conv(orc_model* m, const orc_layer* L, int layer) {
    const int E = m->d.n_embd;
    float* st = m->conv_state + (size_t)layer * 2 * E;
    const orc_tensor* kt = &L->t[ORC_CONV];
    orc_matmul(&L->t[ORC_IN_PROJ], m->normed, m->bcx);
    for (int d = 0; d < E; d++) m->bx[d] = (float)((double)m->bcx[d] * (double)m->bcx[2 * E + d]);
    for (int d = 0; d < E; d++) {
        const double k0 = weight_at(kt, (int64_t)d * 3 + 0), k1 = weight_at(kt, (int64_t)d * 3 + 1),
                     k2 = weight_at(kt, (int64_t)d * 3 + 2);
        m->cout[d] = (float)(k0 * (double)st[d] + k1 * (double)st[E + d] + k2 * (double)m->bx[d]);
    }
    memmove(st, st + E, sizeof(float) * E);
    memcpy(st + E, m->bx, sizeof(float) * E);
    for (int d = 0; d < E; d++) m->cy[d] = (float)((double)m->bcx[E + d] * (double)m->cout[d]);
    orc_matmul(&L->t[ORC_OUT_PROJ], m->cy, m->tmp);
}

/* Dense SwiGLU (qwen3-engine.js:202-209, lfm2-engine.js:394-403): hidden += down(silu(gate)*up). */
static void dense_ffn(orc_model* m, const orc_layer* L) {
    const int64_t f = L->t[ORC_FFN_GATE].ne[1];
    orc_matmul(&L->t[ORC_FFN_GATE], m->normed, m->ffn);
    orc_silu(m->ffn, f);
    orc_matmul(&L->t[ORC_FFN_UP], m->normed, m->ffn_tmp);
    orc_mul(m->ffn, m->ffn_tmp, f);
    orc_matmul(&L->t[ORC_FFN_DOWN], m->ffn, m->tmp);
    orc_add(m->hidden, m->tmp, m->d.n_embd);
}

/* Qwen3Engine.forward (qwen3-engine.js:115-245) / Lfm2Engine.forward (lfm2-engine.js:228-269). */
int orc_forward(orc_model* m, int32_t token, int32_t position, int skip_logits, float* logits,
                float* hidden_dump, float* routing) {
    const int E = m->d.n_embd;
    if (token < 0 || token >= m->d.n_vocab) return -1;
    if (position < 0 || position >= m->d.max_ctx) return -2; /* the JS would write past the slab */
    orc_embedding(&m->d.tok_embd, token, m->hidden);
    for (int l = 0; l < m->d.n_layers; l++) {
        const orc_layer* L = &m->layers[l];
        memcpy(m->normed, m->hidden, sizeof(float) * E);
        orc_rmsnorm(m->normed, E, &L->t[ORC_ATTN_NORM], m->d.rms_eps);
        if (L->is_attn) self_attention(m, L, m->attn_slot[l], position);
        else short_conv(m, L, l);
        orc_add(m->hidden, m->tmp, E);
        memcpy(m->normed, m->hidden, sizeof(float) * E);
        orc_rmsnorm(m->normed, E, &L->t[ORC_FFN_NORM], m->d.rms_eps);
        if (L->is_moe) {
            const int K = m->d.n_expert_used, NE = m->d.n_expert;
            float* rec = routing ? routing + (size_t)m->moe_slot[l] * (2 * K + NE) : NULL;
            if (m->d.arch == 0) /* Qwen3 family: softmax router (qwen3-engine.js:198-199, 304-362) */
                qwen3_moe_token(L, E, NE, K, m->normed, m->moe_out, rec, m->mask, m->r_w, m->ffn, m->ffn_tmp,
                                m->e_dn);
            else
                lfm2_moe_token(L, E, NE, K, m->normed, m->moe_out, rec, m->mask, m->r_logits, m->r_w, m->r_sel,
                               m->ffn, m->ffn_tmp, m->e_dn);
            orc_add(m->hidden, m->moe_out, E);
        } else {
            dense_ffn(m, L);
        }
        if (hidden_dump) memcpy(hidden_dump + (size_t)l * E, m->hidden, sizeof(float) * E);
    }
    if (!skip_logits) {
        orc_rmsnorm(m->hidden, E, &m->d.output_norm, m->d.rms_eps);
        const orc_tensor* out = m->d.output.data ? &m->d.output : &m->d.tok_embd;
        orc_matmul(out, m->hidden, logits);
    }
    return 0;
}

/* generate() greedy with thinking suppressed (qwen3-engine.js:397-457, lfm2-engine.js:523-583). */
int orc_generate(orc_model* m, const int32_t* prompt, int n_prompt, int max_steps, int32_t think_id,
                 int32_t eos_id, int32_t* out_tokens) {
    if (n_prompt < 1) return -1;
    float* logits = (float*)malloc(sizeof(float) * m->d.n_vocab);
    orc_reset(m);
    int rc = 0;
    for (int i = 0; i < n_prompt - 1 && rc == 0; i++) rc = orc_forward(m, prompt[i], i, 1, NULL, NULL, NULL);
    if (rc == 0) rc = orc_forward(m, prompt[n_prompt - 1], n_prompt - 1, 0, logits, NULL, NULL);
    int n = 0;
    if (rc == 0) {
        int32_t cur = orc_sample_suppress(logits, m->d.n_vocab, think_id);
        for (int step = 0; step < max_steps; step++) {
            if (cur == eos_id) break;
            rc = orc_forward(m, cur, n_prompt + step, 0, logits, NULL, NULL);
            if (rc) break;
            out_tokens[n++] = cur;
            cur = orc_sample_suppress(logits, m->d.n_vocab, think_id);
        }
    }
    free(logits);
    return rc ? rc : n;
}
