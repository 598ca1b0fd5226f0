// kernels_attn_tc.cu -- causal prefill attention on the tensor cores (sm_100a).
//
// _selfAttentionCore of a prompt chunk (qwen3-engine.js:249-293; the LFM2 attention layers are the
// same GQA attention): for every query row (token t at position pos0 + t, head h), softmax over the
// keys 0 .. pos0 + t of q.k / sqrt(hd), times V.  The reference computes it in f32 / f64 scalar
// loops; here a CTA takes 128 query rows of one kv head (128 / G consecutive tokens x its G query
// heads: the UMMA's M) and walks the keys in tiles of 64 (the N of the scores, the K of P.V):
//
//   per tile S = Q.K^T on the tensor cores (TMEM accumulators); two of the 256 threads own a
//            query row (its TMEM lane: warps w and w + 4), one half of its columns each;
//            p = exp(s - mr) against the row's reference maximum mr (0 past the row's position),
//            l += p, the tile's P written to shared memory as the A operand of O += P.V (O in
//            TMEM); at the end o = O / l.
//
// Exact splits keep f32 accuracy on fp16 tensor cores: every operand x is the fp16 pair
// xh = fp16(x), xl = fp16((x - xh) * 2048); S1 = qh.kh and S2 = qh.kl + ql.kh give
// s = S1 + S2 / 2048 (the dropped ql.kl / 2^22 is below f32 rounding), and O1 = ph.vh,
// O2 = ph.vl + pl.vh the same way.  The reference maximum of a row moves only when a tile's
// maximum exceeds it by more than e^8 (then O and l are rescaled in place), so p stays within
// fp16 range and the TMEM accumulator is rescaled a few times per row at most.
//
// Operand tiles in shared memory are K-major with the 128-byte swizzle (`sw128`): Q [128][hd] and
// K [64][hd] (hd / 64 column blocks of 64), V transposed to [hd][64 keys], P [128][64 keys].
#include <cuda_fp16.h>

#include "kernels.h"
#include "pipe.cuh"
#include "tc_sm100.cuh"

namespace qq3 {

namespace {

constexpr int kTcRows = 128;   // query rows per CTA (UMMA M)
constexpr int kTcKeys = 64;    // keys per tile
constexpr int kTcThreads = 256;  // two threads per query row: column halves

template <int HD>
struct AttnTcCfg {
    static constexpr int QPlane = kTcRows * HD * 2;  // bytes of one fp16 plane (hi or lo)
    static constexpr int KPlane = kTcKeys * HD * 2;
    static constexpr int VPlane = HD * kTcKeys * 2;
    static constexpr int PPlane = kTcRows * kTcKeys * 2;
    static constexpr int Smem = 2 * (QPlane + KPlane + VPlane + PPlane) + 1024;
    // tensor memory: S1 | S2 (64 columns each) | O1 | O2 (hd columns each)
    static constexpr uint32_t ColS1 = 0, ColS2 = kTcKeys, ColO1 = 2 * kTcKeys, ColO2 = 2 * kTcKeys + HD;
    static constexpr uint32_t TmemCols = (2 * kTcKeys + 2 * HD) <= 256 ? 256 : 512;
    static constexpr uint32_t IdescS = (1u << 4) | ((uint32_t)(kTcKeys >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
    static constexpr uint32_t IdescO = (1u << 4) | ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
};

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// eight f32 -> the fp16 hi and lo planes of one 16-byte chunk
__device__ __forceinline__ void split8(const float (&v)[8], uint4& hi, uint4& lo) {
    float h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = __half2float(__float2half_rn(v[i]));
    hi = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]), pack_h2(h[6], h[7]));
    lo = make_uint4(pack_h2((v[0] - h[0]) * 2048.f, (v[1] - h[1]) * 2048.f),
                    pack_h2((v[2] - h[2]) * 2048.f, (v[3] - h[3]) * 2048.f),
                    pack_h2((v[4] - h[4]) * 2048.f, (v[5] - h[5]) * 2048.f),
                    pack_h2((v[6] - h[6]) * 2048.f, (v[7] - h[7]) * 2048.f));
}

// 16 consecutive 32-bit tensor-memory columns of this thread's lane
__device__ __forceinline__ void tmem_st16_flat(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// byte offset of 16-byte chunk c (8 fp16 of K) of row r in a K-major tile of `rows` rows
__device__ __forceinline__ uint32_t tile_chunk(int rows, int r, int c) {
    return (uint32_t)(c >> 3) * (uint32_t)rows * 128u + sw128(r, c & 7);
}

template <int HD>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_attn_prefill_tc(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc, int T,
                      int pos0, int n_head, int n_kv, int max_ctx, float* __restrict__ out, int* err) {
    using C = AttnTcCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* Qh = smem;
    uint8_t* Ql = Qh + C::QPlane;
    uint8_t* Kh = Ql + C::QPlane;
    uint8_t* Kl = Kh + C::KPlane;
    uint8_t* Vh = Kl + C::KPlane;
    uint8_t* Vl = Vh + C::VPlane;
    uint8_t* Ph = Vl + C::VPlane;
    uint8_t* Pl = Ph + C::PPlane;
    __shared__ __align__(8) uint64_t mma_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ float row_red[kTcThreads];  // the two halves' row maxima, then sums
    const int t = threadIdx.x, warp = t >> 5;
    const int G = n_head / n_kv, QT = kTcRows / G;
    const int t0 = blockIdx.x * QT, kvh = blockIdx.y;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(C::TmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (t == 0) {
        mbar_init(&mma_bar, 1);
        mbar_fence_init();
    }
    // thread t holds query row t % 128 (token t0 + row / G, head kvh G + row % G), column half t / 128
    const int row = t & (kTcRows - 1), half = t / kTcRows, tok = t0 + row / G, head = kvh * G + row % G;
    const bool live = tok < T;
    {
        const float* qr = q + ((size_t)tok * n_head + head) * HD;
#pragma unroll 2
        for (int c = half * (HD / 16); c < (half + 1) * (HD / 16); c++) {
            float v[8];
            if (live) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(qr + 8 * c));
                const float4 b = __ldg(reinterpret_cast<const float4*>(qr + 8 * c + 4));
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = 0.f;
            }
            uint4 hi, lo;
            split8(v, hi, lo);
            const uint32_t off = tile_chunk(kTcRows, row, c);
            *reinterpret_cast<uint4*>(Qh + off) = hi;
            *reinterpret_cast<uint4*>(Ql + off) = lo;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int t_last = min(T, t0 + QT) - 1;
    const int n_keys = pos0 + t_last + 1;  // keys 0 .. the tile's last position
    const int my_pos = pos0 + tok;         // this row sees keys 0 .. my_pos
    const float* kb = kc + (size_t)kvh * max_ctx * HD;
    const float* vb = vc + (size_t)kvh * max_ctx * HD;
    const float scale = (float)(1.0 / sqrt((double)HD));
    const int n_tiles = (n_keys + kTcKeys - 1) / kTcKeys;
    float l = 0.f;
    uint32_t phase = 0;
    bool ok = true;
    // staging of a key tile: K rows (keys past n_keys are zero) and V transposed; a thread's
    // kTasks tasks of each are 8 elements (K: key j, dims 8c..; V: dim d, keys 8jc..; consecutive
    // threads read consecutive dims of a key row)
    constexpr int kTasks = kTcKeys * (HD / 8) / kTcThreads;
    auto load_k = [&](int k0, float (&v)[kTasks][8]) {
#pragma unroll
        for (int u = 0; u < kTasks; u++) {
            const int f = t + u * kTcThreads;
            const int j = f / (HD / 8), c = f % (HD / 8);
            if (k0 + j < n_keys) {
                const float* kr = kb + (size_t)(k0 + j) * HD + 8 * c;
                const float4 a = __ldg(reinterpret_cast<const float4*>(kr));
                const float4 b = __ldg(reinterpret_cast<const float4*>(kr + 4));
                v[u][0] = a.x; v[u][1] = a.y; v[u][2] = a.z; v[u][3] = a.w;
                v[u][4] = b.x; v[u][5] = b.y; v[u][6] = b.z; v[u][7] = b.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) v[u][i] = 0.f;
            }
        }
    };
    auto store_k = [&](const float (&v)[kTasks][8]) {
#pragma unroll
        for (int u = 0; u < kTasks; u++) {
            const int f = t + u * kTcThreads;
            const int j = f / (HD / 8), c = f % (HD / 8);
            uint4 hi, lo;
            split8(v[u], hi, lo);
            const uint32_t off = tile_chunk(kTcKeys, j, c);
            *reinterpret_cast<uint4*>(Kh + off) = hi;
            *reinterpret_cast<uint4*>(Kl + off) = lo;
        }
    };
    auto load_v = [&](int k0, float (&v)[kTasks][8]) {
#pragma unroll
        for (int u = 0; u < kTasks; u++) {
            const int f = t + u * kTcThreads;
            const int d = f % HD, jc = f / HD;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int j = k0 + 8 * jc + i;
                v[u][i] = j < n_keys ? __ldg(vb + (size_t)j * HD + d) : 0.f;
            }
        }
    };
    auto store_v = [&](const float (&v)[kTasks][8]) {
#pragma unroll
        for (int u = 0; u < kTasks; u++) {
            const int f = t + u * kTcThreads;
            const int d = f % HD, jc = f / HD;
            uint4 hi, lo;
            split8(v[u], hi, lo);
            const uint32_t off = sw128(d, jc);
            *reinterpret_cast<uint4*>(Vh + off) = hi;
            *reinterpret_cast<uint4*>(Vl + off) = lo;
        }
    };
    // One pass over the key tiles, an online softmax against a reference maximum mr of the row
    // (the same in both threads of the row): p = exp(s - mr); mr moves only when a tile's maximum
    // exceeds it by more than kLazy, and then O (in TMEM) and l are rescaled by exp(mr_old -
    // mr_new).  So p <= e^kLazy (an fp16 hi/lo pair holds it) and the accumulator is rarely touched.
    constexpr float kLazy = 8.0f;
    float mr = -INFINITY;
    float kr[kTasks][8], vr[kTasks][8];
    load_k(0, kr);
    load_v(0, vr);
    for (int kt = 0; kt < n_tiles; kt++) {
        const int k0 = kt * kTcKeys;
        store_k(kr);
        store_v(vr);
        fence_async_smem();  // the tiles are read by the tensor cores (async proxy)
        tc_fence_before();
        __syncthreads();
        if (t == 0) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < HD / 16; ks++) {
                const uint32_t qo = (uint32_t)(ks >> 2) * kTcRows * 128u + 32u * (ks & 3);
                const uint32_t ko = (uint32_t)(ks >> 2) * kTcKeys * 128u + 32u * (ks & 3);
                const uint32_t acc = ks ? 1u : 0u;
                const uint64_t qh = umma_desc(smem_u32(Qh + qo)), ql = umma_desc(smem_u32(Ql + qo));
                const uint64_t kh = umma_desc(smem_u32(Kh + ko)), kl = umma_desc(smem_u32(Kl + ko));
                umma_f16(tmem + C::ColS1, qh, kh, C::IdescS, acc);
                umma_f16(tmem + C::ColS2, qh, kl, C::IdescS, acc);
                umma_f16(tmem + C::ColS2, ql, kh, C::IdescS, 1u);
            }
            umma_commit(&mma_bar);
        }
        // the next tile's K and V travel while this tile's MMAs and softmax run
        if (kt + 1 < n_tiles) {
            load_k(k0 + kTcKeys, kr);
            load_v(k0 + kTcKeys, vr);
        }
        if (!mbar_wait(&mma_bar, phase)) {
            set_err(err, kErrFullWait);
            ok = false;
        }
        phase ^= 1u;
        tc_fence_after();
        // this thread's 32 scores of the tile (-inf past the row's position) and their maximum
        float sv[kTcKeys / 2];
        float tmax = -INFINITY;
#pragma unroll
        for (int c = 0; c < kTcKeys / 2; c += 16) {
            const int c0 = half * (kTcKeys / 2) + c;
            uint32_t s1[16], s2[16];
            tmem_ld16(tmem + lane_base + C::ColS1 + (uint32_t)c0, s1);
            tmem_ld16(tmem + lane_base + C::ColS2 + (uint32_t)c0, s2);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int key = k0 + c0 + i;
                const bool valid = live && ok && key <= my_pos;
                const float sc = fmaf(__uint_as_float(s2[i]), 1.0f / 2048.0f, __uint_as_float(s1[i])) * scale;
                sv[c + i] = valid ? sc : -INFINITY;
                tmax = fmaxf(tmax, sv[c + i]);
            }
        }
        // the tile maximum of the row over both halves (row_red is next written after two barriers)
        row_red[t] = tmax;
        __syncthreads();
        tmax = fmaxf(row_red[row], row_red[row + kTcRows]);
        if (tmax > mr + kLazy) {
            if (mr > -INFINITY) {  // rescale this thread's half of the O row and its l
                const float f = expf(mr - tmax);
                l *= f;
#pragma unroll 1
                for (int c0 = half * (HD / 2); c0 < (half + 1) * (HD / 2); c0 += 16) {
                    uint32_t o1[16], o2[16];
                    tmem_ld16(tmem + lane_base + C::ColO1 + (uint32_t)c0, o1);
                    tmem_ld16(tmem + lane_base + C::ColO2 + (uint32_t)c0, o2);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        o1[i] = __float_as_uint(__uint_as_float(o1[i]) * f);
                        o2[i] = __float_as_uint(__uint_as_float(o2[i]) * f);
                    }
                    tmem_st16_flat(tmem + lane_base + C::ColO1 + (uint32_t)c0, o1);
                    tmem_st16_flat(tmem + lane_base + C::ColO2 + (uint32_t)c0, o2);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            mr = tmax;
        }
        // p = exp(s - mr) into this thread's half of the P row
#pragma unroll
        for (int c = 0; c < kTcKeys / 2; c += 8) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                v[i] = sv[c + i] == -INFINITY ? 0.f : expf(sv[c + i] - mr);
                l += v[i];
            }
            uint4 hi, lo;
            split8(v, hi, lo);
            const uint32_t off = sw128(row, (half * (kTcKeys / 2) + c) >> 3);
            *reinterpret_cast<uint4*>(Ph + off) = hi;
            *reinterpret_cast<uint4*>(Pl + off) = lo;
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (t == 0) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < kTcKeys / 16; ks++) {
                const uint32_t acc = (kt > 0 || ks > 0) ? 1u : 0u;
                const uint64_t ph = umma_desc(smem_u32(Ph + 32u * ks)), pl = umma_desc(smem_u32(Pl + 32u * ks));
                const uint64_t vh = umma_desc(smem_u32(Vh + 32u * ks)), vl = umma_desc(smem_u32(Vl + 32u * ks));
                umma_f16(tmem + C::ColO1, ph, vh, C::IdescO, acc);
                umma_f16(tmem + C::ColO2, ph, vl, C::IdescO, acc);
                umma_f16(tmem + C::ColO2, pl, vh, C::IdescO, 1u);
            }
            umma_commit(&mma_bar);
        }
        if (!mbar_wait(&mma_bar, phase)) {
            set_err(err, kErrFullWait);
            ok = false;
        }
        phase ^= 1u;
        tc_fence_after();
    }
    // o = (O1 + O2 / 2048) / l for this row (l summed over both column halves)
    row_red[t] = l;
    __syncthreads();
    l = row_red[row] + row_red[row + kTcRows];
    if (n_tiles > 0) {
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        float* o = out + ((size_t)tok * n_head + head) * HD;
#pragma unroll 1
        for (int c0 = half * (HD / 2); c0 < (half + 1) * (HD / 2); c0 += 16) {
            uint32_t o1[16], o2[16];
            tmem_ld16(tmem + lane_base + C::ColO1 + (uint32_t)c0, o1);
            tmem_ld16(tmem + lane_base + C::ColO2 + (uint32_t)c0, o2);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (live && ok) {
#pragma unroll
                for (int i = 0; i < 16; i += 4) {
                    float4 r;
                    r.x = fmaf(__uint_as_float(o2[i]), 1.0f / 2048.0f, __uint_as_float(o1[i])) * inv;
                    r.y = fmaf(__uint_as_float(o2[i + 1]), 1.0f / 2048.0f, __uint_as_float(o1[i + 1])) * inv;
                    r.z = fmaf(__uint_as_float(o2[i + 2]), 1.0f / 2048.0f, __uint_as_float(o1[i + 2])) * inv;
                    r.w = fmaf(__uint_as_float(o2[i + 3]), 1.0f / 2048.0f, __uint_as_float(o1[i + 3])) * inv;
                    *reinterpret_cast<float4*>(o + c0 + i) = r;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TmemCols));
}

template <int HD>
void launch_tc(const float* q, const float* kc, const float* vc, int T, int pos0, int n_head, int n_kv, int max_ctx,
               float* out, cudaStream_t s) {
    using C = AttnTcCfg<HD>;
    if (first_use_on_device(reinterpret_cast<const void*>(k_attn_prefill_tc<HD>)))
        QQ_CUDA_TRY(cudaFuncSetAttribute(k_attn_prefill_tc<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::Smem));
    const int QT = kTcRows / (n_head / n_kv);
    dim3 grid((unsigned)((T + QT - 1) / QT), (unsigned)n_kv);
    k_attn_prefill_tc<HD><<<grid, kTcThreads, C::Smem, s>>>(q, kc, vc, T, pos0, n_head, n_kv, max_ctx, out,
                                                             kernel_err_ptr());
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace

bool attn_prefill_tc_supported(int n_head, int n_kv, int hd) {
    if (n_kv < 1 || n_head % n_kv) return false;
    const int G = n_head / n_kv;
    return (hd == 64 || hd == 128) && G >= 1 && kTcRows % G == 0;
}

void launch_attn_prefill_tc(const float* q, const float* kc, const float* vc, int T, int pos0, int n_head, int n_kv,
                            int hd, int max_ctx, float* out, cudaStream_t s) {
    QQ_CHECK(attn_prefill_tc_supported(n_head, n_kv, hd), -4, "tensor-core prefill attention: unsupported shape");
    if (T <= 0) return;
    if (hd == 64) launch_tc<64>(q, kc, vc, T, pos0, n_head, n_kv, max_ctx, out, s);
    else launch_tc<128>(q, kc, vc, T, pos0, n_head, n_kv, max_ctx, out, s);
}

}  // namespace qq3
