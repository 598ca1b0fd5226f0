// kernels_gemm.cu -- Q8_0 weights x activations on the 5th-generation tensor cores (sm_100a).
//
// Y[M][N] = X[M][K] . W[N][K]^T for M >= 2 rows (prefill, batched matmul): the M > 1 form of
// matmulQ80xF32 (tensor.js:26-53), which the reference runs as M independent calls.
//
//  * operands: X is converted once to fp16 (k_f32_to_f16).  W tiles are dequantised in shared
//    memory, w = q*d rounded to fp16 (11-bit significand; the product needs up to 18 bits, so
//    each weight carries a relative error <= 2^-12 -- the 1e-2 parity bar holds with margin).
//    Both are written in the K-major 128-byte-swizzled layout the UMMA descriptors name;
//  * tcgen05.mma.cta_group::1.kind::f16 (fp16 x fp16 -> f32), M = 128 rows x N = 256 columns x
//    K = 16 per instruction, issued by one thread; the accumulator lives in tensor memory
//    (256 of its 512 columns); completion is tracked with tcgen05.commit on mbarriers;
//  * a 3-stage shared-memory ring (48 KB per stage) lets the 128 threads convert tile k+1..k+2
//    while the tensor core works on tile k;
//  * epilogue: each warp reads its 32 accumulator lanes (rows) with tcgen05.ld and stores f32.
//
// All waits are bounded (error code in the kernel error word, no hang).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <string>

#include "kernels.h"
#include "pipe.cuh"
#include "tc_sm100.cuh"
#include "qq3.h"

namespace qq3 {

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kStages = 3;
constexpr uint32_t kTmemCols = 256;


__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, int* err) {
    if (mbar_wait(b, parity)) return true;
    set_err(err, kErrFullWait);
    return false;
}

// TMA: 2-D tiled bulk copy global -> shared, completing on an mbarrier (no multicast).
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 4 signed int8 weights -> two fp16 pairs scaled by d (exact int -> fp16 via the 1024 + byte
// bit pattern; RN(q * d) with one HMUL2, the same rounding as converting the exact product).
__device__ __forceinline__ void dq4(uint32_t w, __half2 d2, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;  // b + 128 per byte
    uint32_t a = __byte_perm(u, 0x64646464u, 0x5140), b = __byte_perm(u, 0x64646464u, 0x5342);
    const __half2 bias = __float2half2_rn(1152.0f);
    __half2 ha = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&a), bias), d2);
    __half2 hb = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&b), bias), d2);
    lo = *reinterpret_cast<uint32_t*>(&ha);
    hi = *reinterpret_cast<uint32_t*>(&hb);
}

// Warp roles: 0-7 dequantise B and run the epilogue; 8 issues the TMA loads; 9 allocates
// tensor memory and issues the MMAs.
constexpr int kConvWarps = 8;
constexpr int kThreadsG2 = (kConvWarps + 2) * 32;

// SPLIT = 1: one fp16 product (x and w = q*d rounded to 11-bit significands; ~1e-3 relative).
// SPLIT = 3: x = xh + xl/2048 and w = wh + wl/2048 split into fp16 pairs (w exactly: q*d has at
//   most 18 significant bits), three products xh.wh -> D1 and xh.wl + xl.wh -> D2 in two TMEM
//   accumulators, y = D1 + D2/2048: ~2^-22 relative, the f32 GEMV's accuracy.
template <int SPLIT>
struct Cfg {
    static constexpr int BN = SPLIT == 1 ? 256 : 128;
    static constexpr int NT = SPLIT == 1 ? 1 : 2;     // operand tiles per side (hi, lo)
    static constexpr int ATile = kBM * kBK * 2;       // 16 KB
    static constexpr int BTile = BN * kBK * 2;        // 32 KB / 16 KB
    static constexpr int RawTile = BN * kBK;          // int8
    static constexpr int DTile = BN * 16;             // block scales: 8 fp16 per row (4 K steps)
    static constexpr int Stage = NT * ATile + NT * BTile + RawTile + DTile;
    static constexpr int Smem = kStages * Stage + 1024;
    static constexpr uint32_t Idesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
    static constexpr int RowThreads = 256 / BN;       // converter threads per B row
};


__device__ __forceinline__ uint32_t h2bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// 32 weights of one row (raw[0..1] in K order, block scale dc) -> the exact hi and lo fp16 pairs
// (the SPLIT = 3 conversion above): hw[c][w], lw[c][w] hold weights 8c + 2w and 8c + 2w + 1
__device__ __forceinline__ void split3_words(const uint4 (&raw)[2], __half2 dc, uint32_t (&hw)[4][4],
                                             uint32_t (&lw)[4][4]) {
    const float dfs = __low2float(dc);
    if (fabsf(dfs) < 0.25f) {  // one branch for the four chunks, so their chains interleave
        const __half2 d2s = __low2half2(dc);
        const __half2 d2k = __float2half2_rn(dfs * 2048.0f);
        const __half2 m2k = __float2half2_rn(-2048.0f);
        const __half2 bias = __float2half2_rn(1152.0f);
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 r4 = raw[c >> 1];
            const uint32_t w0 = (c & 1) ? r4.z : r4.x, w1 = (c & 1) ? r4.w : r4.y;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const uint32_t u = (j ? w1 : w0) ^ 0x80808080u;
                uint32_t pa = __byte_perm(u, 0x64646464u, 0x5140), pb = __byte_perm(u, 0x64646464u, 0x5342);
                const __half2 qa = __hsub2(*reinterpret_cast<__half2*>(&pa), bias);
                const __half2 qb = __hsub2(*reinterpret_cast<__half2*>(&pb), bias);
                const __half2 ha = __hmul2(qa, d2s), hb = __hmul2(qb, d2s);
                hw[c][2 * j] = h2bits(ha);
                hw[c][2 * j + 1] = h2bits(hb);
                lw[c][2 * j] = h2bits(__hfma2(qa, d2k, __hmul2(ha, m2k)));
                lw[c][2 * j + 1] = h2bits(__hfma2(qb, d2k, __hmul2(hb, m2k)));
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 r4 = raw[c >> 1];
            const uint32_t w0 = (c & 1) ? r4.z : r4.x, w1 = (c & 1) ? r4.w : r4.y;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t word = j < 2 ? w0 : w1;
                const int sh = 16 * (j & 1);
                const float wa = (float)(int8_t)((word >> sh) & 0xff) * dfs;
                const float wb = (float)(int8_t)((word >> (sh + 8)) & 0xff) * dfs;
                const __half2 h = __floats2half2_rn(wa, wb);
                const float2 hf = __half22float2(h);
                hw[c][j] = h2bits(h);
                lw[c][j] = h2bits(__floats2half2_rn((wa - hf.x) * 2048.f, (wb - hf.y) * 2048.f));
            }
        }
    }
}

// The same conversion stored into the hi and lo planes of the swizzled K-major tiles bh / bl,
// 16-byte chunks c0 .. c0 + 3 of row brow
__device__ __forceinline__ void split3_convert(const uint4 (&raw)[2], __half2 dc, uint8_t* bh, uint8_t* bl, int brow,
                                               int c0) {
    uint32_t hw[4][4], lw[4][4];
    split3_words(raw, dc, hw, lw);
#pragma unroll
    for (int c = 0; c < 4; c++) {
        *reinterpret_cast<uint4*>(bh + sw128(brow, c0 + c)) = make_uint4(hw[c][0], hw[c][1], hw[c][2], hw[c][3]);
        *reinterpret_cast<uint4*>(bl + sw128(brow, c0 + c)) = make_uint4(lw[c][0], lw[c][1], lw[c][2], lw[c][3]);
    }
}


template <int SPLIT>
__global__ void __launch_bounds__(kThreadsG2, 1)
    k_gemm_q8_tma(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmD, int d_tma, int M, int K, const __half* __restrict__ d, int N,
                  float* __restrict__ C, int ldc, const int4* __restrict__ tiles, const int* __restrict__ n_tiles,
                  int* err) {
    using G = Cfg<SPLIT>;
    constexpr int BN = G::BN;
    // Dense: CTA (x, y) computes rows [128x, 128x + 128) x columns [BN y, BN y + BN).
    // Grouped (tiles != null): CTA x takes work item tiles[x] = (group g, first row, rows); its B
    // rows are those of group g (rows g*N .. g*N + N - 1 of W), e.g. one expert of a packed
    // expert tensor.  Items past *n_tiles exit at once.  With SPLIT = 3 the A map holds the hi
    // rows at 0.. and the lo rows at M..
    int grp = 0, m0 = blockIdx.x * kBM, m_rows = M - m0;
    if (tiles) {
        if ((int)blockIdx.x >= *n_tiles) return;
        const int4 ti = tiles[blockIdx.x];
        grp = ti.x;
        m0 = ti.y;
        m_rows = ti.z;
    }
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_a[kStages], full_raw[kStages], raw_free[kStages], conv_done[kStages],
        mma_done[kStages], done_bar;
    __shared__ uint32_t tmem_slot;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int n0 = blockIdx.y * BN;   // M-tiles adjacent: they share the B tile in L2
    const int nb0 = grp * N + n0;     // first B row of the tile in W
    const int nk = (K + kBK - 1) / kBK;
    const int KB = K >> 5;
    // stage layout: A tiles | B tiles | raw int8 B
    auto a_tile = [&](uint8_t* st, int h) { return st + h * G::ATile; };
    auto b_tile = [&](uint8_t* st, int h) { return st + G::NT * G::ATile + h * G::BTile; };
    auto raw_tile = [&](uint8_t* st) { return st + G::NT * (G::ATile + G::BTile); };
    auto d_tile = [&](uint8_t* st) { return reinterpret_cast<const __half*>(raw_tile(st) + G::RawTile); };
    if (warp == kConvWarps + 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (t == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full_a[s], 1);
            mbar_init(&full_raw[s], 1);
            mbar_init(&raw_free[s], kConvWarps);
            mbar_init(&conv_done[s], kConvWarps);
            mbar_init(&mma_done[s], 1);
        }
        mbar_init(&done_bar, 1);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    bool ok = true;
    if (warp == kConvWarps) {
        if (lane == 0) {  // TMA producer
            int issued = 0;
            for (int kt = 0; kt < nk && ok; kt++, issued++) {
                const int s = kt % kStages;
                const uint32_t pu = (uint32_t)((kt / kStages - 1) & 1);
                if (kt >= kStages) ok = bar_wait(&raw_free[s], pu, err) && bar_wait(&mma_done[s], pu, err);
                if (!ok) break;
                uint8_t* st = smem + s * G::Stage;
                mbar_arrive_expect_tx(&full_a[s], (uint32_t)(G::NT * G::ATile));
                tma_2d(a_tile(st, 0), &tmA, kt * kBK, m0, &full_a[s]);
                if (SPLIT == 3) tma_2d(a_tile(st, 1), &tmA, kt * kBK, M + m0, &full_a[s]);
                mbar_arrive_expect_tx(&full_raw[s], (uint32_t)(G::RawTile + (d_tma ? G::DTile : 0)));
                tma_2d(raw_tile(st), &tmB, kt * kBK, nb0, &full_raw[s]);
                // the block scales of this K step ride in the same stage (8 per row from an
                // 8-aligned block index, which holds blocks 2kt and 2kt + 1)
                if (d_tma) tma_2d(raw_tile(st) + G::RawTile, &tmD, (2 * kt) & ~7, nb0, &full_raw[s]);
            }
            // every issued copy lands before the CTA can exit (already true unless a wait failed)
            for (int kt = (issued > kStages ? issued - kStages : 0); kt < issued; kt++) {
                const uint32_t pu = (uint32_t)((kt / kStages) & 1);
                bar_wait(&full_a[kt % kStages], pu, err);
                bar_wait(&full_raw[kt % kStages], pu, err);
            }
        }
    } else if (warp == kConvWarps + 1) {
        if (lane == 0) {  // MMA issuer
            for (int kt = 0; kt < nk && ok; kt++) {
                const int s = kt % kStages;
                const uint32_t pu = (uint32_t)((kt / kStages) & 1);
                ok = bar_wait(&full_a[s], pu, err) && bar_wait(&conv_done[s], pu, err);
                if (!ok) break;
                tc_fence_after();
                uint8_t* st = smem + s * G::Stage;
                const uint32_t ah = smem_u32(a_tile(st, 0)), bh = smem_u32(b_tile(st, 0));
#pragma unroll
                for (int ks = 0; ks < kBK / 16; ks++) {
                    const uint32_t acc = (kt | ks) != 0 ? 1u : 0u;
                    umma_f16(tmem, umma_desc(ah + 32u * ks), umma_desc(bh + 32u * ks), G::Idesc, acc);
                    if (SPLIT == 3) {
                        const uint32_t al = smem_u32(a_tile(st, 1)), bl = smem_u32(b_tile(st, 1));
                        umma_f16(tmem + BN, umma_desc(ah + 32u * ks), umma_desc(bl + 32u * ks), G::Idesc, acc);
                        umma_f16(tmem + BN, umma_desc(al + 32u * ks), umma_desc(bh + 32u * ks), G::Idesc, 1u);
                    }
                }
                umma_commit(&mma_done[s]);
            }
            umma_commit(&done_bar);  // covers every MMA issued
        }
    } else {
        // converters: RowThreads threads per B row, each 64 / RowThreads weights of it
        constexpr int RT = G::RowThreads, WPT = kBK / RT;  // weights per thread: 64 or 32
        const int brow = t / RT, part = t % RT;
        const int n = n0 + brow;                 // column of the output
        const size_t drow = (size_t)(nb0 + brow);  // row of W
        auto load_d = [&](int kt) -> uint32_t {  // block scales of this thread's weights, as a half2
            __half2 v = __float2half2_rn(0.f);
            const int kb = 2 * kt + (RT == 2 ? part : 0);
            if (n < N && kb < KB) {
                const __half* dp = d + drow * KB + kb;
                v = RT == 2 ? __halves2half2(dp[0], dp[0]) : __halves2half2(dp[0], kb + 1 < KB ? dp[1] : __float2half(0.f));
            }
            return h2bits(v);
        };
        uint32_t dnext = d_tma ? 0u : load_d(0);
        for (int kt = 0; kt < nk && ok; kt++) {
            const int s = kt % kStages;
            const uint32_t pu = (uint32_t)((kt / kStages) & 1);
            uint32_t dcur = dnext;
            if (!d_tma && kt + 1 < nk) dnext = load_d(kt + 1);
            uint8_t* st = smem + s * G::Stage;
            ok = __all_sync(0xffffffffu, bar_wait(&full_raw[s], pu, err));  // warp-uniform outcome
            uint4 raw[WPT / 16];
            if (ok) {
                const uint4* rp = reinterpret_cast<const uint4*>(raw_tile(st) + brow * kBK + part * WPT);
#pragma unroll
                for (int j = 0; j < WPT / 16; j++) raw[j] = rp[j];
                if (d_tma) {  // rows past N were zero-filled by the copy
                    const __half* ds = d_tile(st) + brow * 8 + ((2 * kt + (RT == 2 ? part : 0)) & 7);
                    dcur = h2bits(RT == 2 ? __halves2half2(ds[0], ds[0]) : __halves2half2(ds[0], ds[1]));
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_free[s]);
            if (ok && kt >= kStages)
                ok = __all_sync(0xffffffffu, bar_wait(&mma_done[s], (uint32_t)((kt / kStages - 1) & 1), err));
            if (!ok) break;
            const __half2 dc = *reinterpret_cast<const __half2*>(&dcur);
            const int c0 = part * (WPT / 8);  // first 8-weight chunk of this thread in the row
            if constexpr (SPLIT == 3) {
                // exact hi/lo pair (RT == 2: each thread's 32 weights share one block scale)
                split3_convert(*reinterpret_cast<const uint4(*)[2]>(raw), dc, b_tile(st, 0), b_tile(st, 1), brow, c0);
            } else {
#pragma unroll
                for (int c = 0; c < WPT / 8; c++) {
                    const uint4 r4 = raw[c >> 1];
                    const uint32_t w0 = (c & 1) ? r4.z : r4.x, w1 = (c & 1) ? r4.w : r4.y;
                    const __half2 d2 = (c >> 2) ? __high2half2(dc) : __low2half2(dc);
                    uint4 o;
                    dq4(w0, d2, o.x, o.y);
                    dq4(w1, d2, o.z, o.w);
                    *reinterpret_cast<uint4*>(b_tile(st, 0) + sw128(brow, c0 + c)) = o;
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv_done[s]);
        }
        // epilogue: warp w reads TMEM lanes 32 (w % 4) .. (rows), columns BN/2 (w / 4) ..
        if (ok) ok = bar_wait(&done_bar, 0u, err);
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
        if (ok) {
            const int q = warp & 3, half = warp >> 2;
            const int row = q * 32 + lane, m = m0 + row;
            const bool live = row < m_rows;
#pragma unroll 1
            for (int cc = half * (BN / 2); cc < (half + 1) * (BN / 2); cc += 16) {
                uint32_t v[16], v2[16];
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)cc;
                tmem_ld16(taddr, v);
                if (SPLIT == 3) tmem_ld16(taddr + BN, v2);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                float f[16];
#pragma unroll
                for (int j = 0; j < 16; j++)
                    f[j] = SPLIT == 3 ? fmaf(__uint_as_float(v2[j]), 1.0f / 2048.0f, __uint_as_float(v[j]))
                                      : __uint_as_float(v[j]);
                if (live) {
                    float* crow = C + (size_t)m * ldc + n0 + cc;
                    if (n0 + cc + 16 <= N && (ldc & 3) == 0) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            *reinterpret_cast<float4*>(crow + j) = make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            if (n0 + cc + j < N) crow[j] = f[j];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kConvWarps + 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// ---- few-row form (M <= 32 activation rows): weights on the MMA's M side, split-K ---------------
// With a handful of activation rows (a multi-sequence decode step) the 128-row activation tile
// above leaves 7/8 of every MMA empty and the grid holds only ceil(N / 128) CTAs, so the weights
// stream through a few SMs.  Here a work item is 128 weight rows (the UMMA's M operand) against
// all MN (16 or 32) activation rows (its N operand) over one of S splits of the K range, and one
// persistent CTA per SM walks its items:
//   warp 8    streams raw int8 weight stages of 128 rows x 256 K (two 128-byte-wide swizzled TMA
//             boxes, plus the 8 block scales per row of that K range) into a 5-deep ring;
//   warp 10   loads the fp16 activation tiles (hi rows, then lo rows) of each 64-wide K step;
//   warps 0-7 convert: thread (row r, K half h) turns its 32 weights of a K step into the exact
//             fp16 hi/lo pairs and writes them to tensor memory (tcgen05.st, lane r), the MMA's
//             A operand, and go straight on to the next item's K steps;
//   warp 9    issues [hh | hl] += wh.[xh | xl] (N = 2 MN) and lh += wl.xh (N = MN) per 16 of K,
//             with A read from tensor memory, into one of two accumulator pairs (items
//             alternate, so an item's MMAs overlap the previous item's epilogue);
//   warps 11-18 (two per 32 tensor-memory lanes, each half of the activation rows) read an
//             item's accumulators once its MMAs are done and store them, so no converter waits
//             for an item to drain.
// A in tensor memory keeps the converted weights out of shared memory: an N = 16 MMA with A in
// shared memory re-reads its 4 KB A tile for 16 output columns, and those reads, the converted
// stores and the raw stages share one pipe (measured: conversion, MMAs and loads added up).
// With S > 1 each split writes its partial sums to scratch [S][M][N]; the last CTA to finish a row
// tile (arrival ticket) adds them in split order, so the result does not depend on scheduling.
// Exact three-product split only (as SPLIT = 3 above): y = hh + (hl + lh) / 2048.
constexpr int kRowsBM = 128;       // weight rows per item
constexpr int kRowsKR = 256;       // K of one raw weight stage (four 64-wide MMA K steps)
constexpr int kRowsMaxItems = 296; // S * row tiles <= this when S > 1
constexpr int kRowsTickets = 256;  // >= row tiles whenever S > 1
constexpr int kRowsEpiWarp = 11;   // first epilogue warp
constexpr int kRowsEpiWarps = 8;   // two per 32 tensor-memory lanes
constexpr int kRowsWarps = kRowsEpiWarp + kRowsEpiWarps;  // 8 converters, 3 producer / issuer warps, epilogue
constexpr int kRowsThreads = kRowsWarps * 32;

// MN = 16 / 32: all activation rows of a few-row product in one item; MN = 128: the wide form for
// many rows (prefill), items over (weight tile, 128-row activation tile) with one accumulator set
// of 384 columns ([hh | hl] N = 256, lh N = 128), so the MMAs run at N = 256 / 128.
template <int MN>
struct RowsCfg {
    static constexpr bool Wide = MN > 32;
    static constexpr int KPS = Wide ? 1 : 2;            // 64-wide K steps per operand stage (one handshake)
    static constexpr int RawStages = Wide ? 4 : 5;      // 136 / 170 KB of weight reads in flight per SM
    static constexpr int OpStages = MN == 16 ? 3 : 2;   // operand stages in TMEM
    static constexpr int XStages = OpStages;            // released by the same MMA commit
    static constexpr int NumAcc = Wide ? 1 : 2;         // accumulator sets (items alternate)
    static constexpr int XTile = MN * kBK * 2;          // fp16 activations (hi or lo) of one K step
    static constexpr int RawBox = kRowsBM * 128;        // one swizzled 128-byte-wide box: 16 KB
    static constexpr int DTile = kRowsBM * 16;          // block scales: 8 fp16 per row (256 K)
    static constexpr int RawStage = (2 * RawBox + DTile + 1023) & ~1023;
    static constexpr int XStage = KPS * 2 * XTile;      // per K step: hi rows, then lo rows
    static constexpr int Smem = RawStages * RawStage + XStages * XStage + 1024;
    static constexpr uint32_t IdescHL = (1u << 4) | ((uint32_t)((2 * MN) >> 3) << 17) | ((uint32_t)(kRowsBM >> 4) << 24);
    static constexpr uint32_t IdescL = (1u << 4) | ((uint32_t)(MN >> 3) << 17) | ((uint32_t)(kRowsBM >> 4) << 24);
    static constexpr uint32_t AccCols = MN == 16 ? 64 : 3 * MN;  // per set: [hh | hl] at +0, lh at +2 MN
    static constexpr uint32_t OpCols = 64 * KPS;        // per K step: hi (4 x 8 columns) | lo
    static constexpr uint32_t OpBase = NumAcc * AccCols;
    static constexpr uint32_t TmemCols = 512;
    static_assert(OpBase + OpStages * OpCols <= TmemCols, "tensor memory columns");
    static_assert(kRowsKR / kBK % KPS == 0, "operand stages tile a raw stage");
    static_assert(3 * MN <= (int)AccCols && 2 * MN <= 256, "accumulator columns, MMA width");
    static_assert(Smem <= 227 * 1024, "shared memory");
};

// tcgen05.mma with the A operand in tensor memory (kind::f16: fp16 x fp16 -> f32)
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// 16 consecutive 32-bit tensor-memory columns of this thread's lane
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[4][4]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0][0]), "r"(v[0][1]), "r"(v[0][2]), "r"(v[0][3]), "r"(v[1][0]), "r"(v[1][1]), "r"(v[1][2]), "r"(v[1][3]),
        "r"(v[2][0]), "r"(v[2][1]), "r"(v[2][2]), "r"(v[2][3]), "r"(v[3][0]), "r"(v[3][1]), "r"(v[3][2]), "r"(v[3][3])
        : "memory");
}

template <int MN>
__global__ void __launch_bounds__(kRowsThreads, 1)
    k_gemm_q8_rows(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmD, int d_tma, int M, int K,
                   const __half* __restrict__ d, int N, float* __restrict__ C, int ldc, float* __restrict__ part,
                   unsigned int* __restrict__ tickets, int S, int n_items, int* err) {
    using G = RowsCfg<MN>;
    constexpr int KPS = G::KPS, NA = G::NumAcc;
    extern __shared__ uint8_t smem_raw[];
    constexpr int R = G::RawStages, O = G::OpStages, X = G::XStages;
    __shared__ __align__(8) uint64_t full_raw[R], raw_free[R], full_x[X], conv_done[O], op_free[O], acc_full[2],
        acc_free[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int last_flag;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int nk = (K + kBK - 1) / kBK;          // 64-wide MMA K steps
    const int nr = (K + kRowsKR - 1) / kRowsKR;  // 256-wide raw stages
    constexpr int SPR = kRowsKR / kBK / KPS;  // operand stages per raw stage
    const int nks = (nk + KPS - 1) / KPS;     // operand stages of the whole K range
    const int n_at = (M + MN - 1) / MN;       // activation tiles (1 unless wide)
    const int KB = K >> 5;
    // shared memory: raw weight stages | activation stages
    auto raw_stage = [&](int rs) { return smem + rs * G::RawStage; };
    auto x_tile = [&](int xs, int sub, int h) {
        return smem + R * G::RawStage + xs * G::XStage + (2 * sub + h) * G::XTile;
    };
    // item it: tile it / S = (weight row tile, activation tile) = (rows n0.., activation rows
    // a0..), split it % S (raw stages [r0, r1))
    auto item_range = [&](int it, int& n0, int& a0, int& sp, int& r0, int& r1) {
        n0 = (it / S / n_at) * kRowsBM;
        a0 = (it / S % n_at) * MN;
        sp = it % S;
        r0 = (int)(((long long)sp * nr) / S);
        r1 = (int)(((long long)(sp + 1) * nr) / S);
    };
    if (warp == 9) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(G::TmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (t == 0) {
        for (int r = 0; r < R; r++) {
            mbar_init(&full_raw[r], 1);
            mbar_init(&raw_free[r], kConvWarps);
        }
        for (int x = 0; x < X; x++) mbar_init(&full_x[x], 1);
        for (int o = 0; o < O; o++) {
            mbar_init(&conv_done[o], kConvWarps);
            mbar_init(&op_free[o], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_free[a], kRowsEpiWarps);
        }
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    bool ok = true;
    if (warp == 8) {
        if (lane == 0) {  // raw weight producer
            int r = 0;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                int n0, a0, sp, r0, r1;
                item_range(it, n0, a0, sp, r0, r1);
                for (int rt = r0; rt < r1 && ok; rt++, r++) {
                    const int rs = r % R;
                    if (r >= R) ok = bar_wait(&raw_free[rs], (uint32_t)((r / R - 1) & 1), err);
                    if (!ok) break;
                    mbar_arrive_expect_tx(&full_raw[rs], (uint32_t)(2 * G::RawBox + (d_tma ? G::DTile : 0)));
                    // a box past K reads zeros (its K coordinate stays a multiple of 128 bytes)
                    tma_2d(raw_stage(rs), &tmW, rt * kRowsKR, n0, &full_raw[rs]);
                    tma_2d(raw_stage(rs) + G::RawBox, &tmW, rt * kRowsKR + 128, n0, &full_raw[rs]);
                    if (d_tma) tma_2d(raw_stage(rs) + 2 * G::RawBox, &tmD, rt * 8, n0, &full_raw[rs]);
                }
            }
            for (int i = (r > R ? r - R : 0); i < r; i++)  // copies land before exit
                bar_wait(&full_raw[i % R], (uint32_t)((i / R) & 1), err);
        }
    } else if (warp == 10) {
        if (lane == 0) {  // activation producer: hi rows at 0, lo rows at M
            int o = 0;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                int n0, a0, sp, r0, r1;
                item_range(it, n0, a0, sp, r0, r1);
                for (int ks2 = SPR * r0; ks2 < min(SPR * r1, nks) && ok; ks2++, o++) {
                    const int xs = o % X;
                    if (o >= X) ok = bar_wait(&op_free[xs], (uint32_t)((o / X - 1) & 1), err);
                    if (!ok) break;
                    // a K step past K reads zeros (its coordinate stays a multiple of 128 bytes)
                    mbar_arrive_expect_tx(&full_x[xs], (uint32_t)G::XStage);
#pragma unroll
                    for (int sub = 0; sub < KPS; sub++) {
                        const int kt = KPS * ks2 + sub;
                        tma_2d(x_tile(xs, sub, 0), &tmX, kt * kBK, a0, &full_x[xs]);
                        tma_2d(x_tile(xs, sub, 1), &tmX, kt * kBK, M + a0, &full_x[xs]);
                    }
                }
            }
            for (int i = (o > X ? o - X : 0); i < o; i++)
                bar_wait(&full_x[i % X], (uint32_t)((i / X) & 1), err);
        }
    } else if (warp == 9) {
        if (lane == 0) {  // MMA issuer
            int o = 0, j = 0;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, j++) {
                int n0, a0, sp, r0, r1;
                item_range(it, n0, a0, sp, r0, r1);
                const int ab = j % NA;
                if (j >= NA) ok = bar_wait(&acc_free[ab], (uint32_t)((j / NA - 1) & 1), err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t acc_d = tmem + (uint32_t)ab * G::AccCols;
                for (int ks2 = SPR * r0; ks2 < min(SPR * r1, nks) && ok; ks2++, o++) {
                    const int os = o % O, xs = o % X;
                    ok = bar_wait(&full_x[xs], (uint32_t)((o / X) & 1), err) &&
                         bar_wait(&conv_done[os], (uint32_t)((o / O) & 1), err);
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int sub = 0; sub < KPS; sub++) {
                        const int kt = KPS * ks2 + sub;
                        if (kt >= nk) break;  // its operand columns were not written
                        const uint32_t a_hi = tmem + G::OpBase + (uint32_t)os * G::OpCols + 64u * sub, a_lo = a_hi + 32u;
                        const uint32_t xh = smem_u32(x_tile(xs, sub, 0));
#pragma unroll
                        for (int ks = 0; ks < kBK / 16; ks++) {
                            const uint32_t acc = (kt != 4 * r0 || ks != 0) ? 1u : 0u;
                            const uint64_t bx = umma_desc(xh + 32u * ks);
                            umma_f16_tmem_a(acc_d, a_hi + 8u * ks, bx, G::IdescHL, acc);
                            umma_f16_tmem_a(acc_d + 2u * MN, a_lo + 8u * ks, bx, G::IdescL, acc);
                        }
                    }
                    umma_commit(&op_free[os]);  // frees the operand columns and the activation stage
                }
                umma_commit(&acc_full[ab]);  // covers the item's MMAs (also after a failed wait)
            }
        }
    } else if (warp < kConvWarps) {
        // converters: thread t holds weight row t & 127 (its TMEM lane) and K half t >> 7 of each
        // K step
        const int row = t & 127, kh = t >> 7;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        int o = 0, r = 0;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            int n0, a0, sp, r0, r1;
            item_range(it, n0, a0, sp, r0, r1);
            const int n = n0 + row;
            for (int rt = r0; rt < r1 && ok; rt++, r++) {
                const int rs = r % R;
                ok = __all_sync(0xffffffffu, bar_wait(&full_raw[rs], (uint32_t)((r / R) & 1), err));
                if (!ok) break;
                // the row's 8 block scales of this raw stage (rows past N and blocks past K: 0)
                uint4 s8 = make_uint4(0u, 0u, 0u, 0u);
                if (d_tma) {
                    s8 = *reinterpret_cast<const uint4*>(raw_stage(rs) + 2 * G::RawBox + row * 16);
                } else if (n < N) {
                    uint32_t sw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                    for (int b = 0; b < 8; b++) {
                        const int kb = 8 * rt + b;
                        const uint32_t h = kb < KB ? (uint32_t)__half_as_ushort(d[(size_t)n * KB + kb]) : 0u;
                        sw[b >> 1] |= h << (16 * (b & 1));
                    }
                    s8 = make_uint4(sw[0], sw[1], sw[2], sw[3]);
                }
                const uint8_t* rowp = raw_stage(rs) + row * 128;
                for (int js = 0; js < 4 && ok; js++) {
                    const int kt = 4 * rt + js;
                    if (kt >= nk) break;
                    const int os = o % O, sub = js % KPS;
                    // 32 weights at K 64 js + 32 kh of the stage: box js / 2, 16-byte chunks c0 and
                    // c0 + 1 of the row, stored at chunk c ^ (row & 7) (128-byte swizzle)
                    const int c0 = 4 * (js & 1) + 2 * kh;
                    const uint8_t* bp = rowp + (js >> 1) * G::RawBox;
                    uint4 raw[2];
                    raw[0] = *reinterpret_cast<const uint4*>(bp + ((c0 ^ (row & 7)) << 4));
                    raw[1] = *reinterpret_cast<const uint4*>(bp + (((c0 + 1) ^ (row & 7)) << 4));
                    const int b = 2 * js + kh;  // block within the stage
                    const uint32_t sword = (b >> 1) == 0 ? s8.x : ((b >> 1) == 1 ? s8.y : ((b >> 1) == 2 ? s8.z : s8.w));
                    const __half hs = __ushort_as_half((unsigned short)((b & 1) ? (sword >> 16) : (sword & 0xffffu)));
                    if (sub == 0 && o >= O)
                        ok = __all_sync(0xffffffffu, bar_wait(&op_free[os], (uint32_t)((o / O - 1) & 1), err));
                    if (!ok) break;
                    if (sub == 0) tc_fence_after();
                    uint32_t hw[4][4], lw[4][4];
                    split3_words(raw, __halves2half2(hs, hs), hw, lw);
                    const uint32_t col =
                        tmem + lane_base + G::OpBase + (uint32_t)os * G::OpCols + 64u * sub + 16u * kh;
                    tmem_st16(col, hw);
                    tmem_st16(col + 32u, lw);
                    // the operand stage is complete after its last K step (or the last one of K)
                    if (sub == KPS - 1 || kt == nk - 1) {
                        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&conv_done[os]);
                        o++;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_free[rs]);  // the stage's bytes are in registers / TMEM
            }
        }
    } else {
        // epilogue warps: warp w reads tensor-memory lanes 32 (w % 4) .. (weight rows) of item j's
        // accumulator set j % NA and stores activation rows of its half hb, in chunks of 16 (the
        // MN = 16 form: one chunk, stored by the first four warps)
        constexpr int kEpiThreads = kRowsEpiWarps * 32;
        constexpr int kHalf = MN > 16 ? MN / 2 : 16;
        const int q = warp & 3, te = t - kRowsEpiWarp * 32, hb = te >> 7;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        int j = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, j++) {
            int n0, a0, sp, r0, r1;
            item_range(it, n0, a0, sp, r0, r1);
            const int ab = j % NA;
            if (ok) ok = bar_wait(&acc_full[ab], (uint32_t)((j / NA) & 1), err);
            ok = __all_sync(0xffffffffu, ok);
            tc_fence_after();
            const int nn = n0 + q * 32 + lane;
#pragma unroll 1
            for (int c16 = hb * kHalf; c16 < (hb + 1) * kHalf && c16 < MN; c16 += 16) {
                float f[16];
                if (ok) {
                    uint32_t v[16], v2[16], v3[16];
                    const uint32_t taddr = tmem + lane_base + (uint32_t)ab * G::AccCols + (uint32_t)c16;
                    tmem_ld16(taddr, v);                  // hh
                    tmem_ld16(taddr + (uint32_t)MN, v2);  // hl
                    tmem_ld16(taddr + 2u * MN, v3);       // lh
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        f[i] = fmaf(__uint_as_float(v2[i]) + __uint_as_float(v3[i]), 1.0f / 2048.0f, __uint_as_float(v[i]));
                }
                if (ok && nn < N) {
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const int m = a0 + c16 + i;
                        if (m < M) {
                            if (S == 1) C[(size_t)m * ldc + nn] = f[i];
                            else part[((size_t)sp * M + m) * N + nn] = f[i];
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_free[ab]);
            if (S > 1) {  // every item takes a ticket (also after a failed wait, so the tickets reset)
                __threadfence();
                named_bar(1, kEpiThreads);
                if (te == 0) {
                    const int tile = it / S;
                    const unsigned prev = atomicAdd(&tickets[tile], 1u);
                    last_flag = prev == (unsigned)(S - 1);
                    if (last_flag) tickets[tile] = 0u;
                }
                named_bar(1, kEpiThreads);
                if (last_flag) {
                    __threadfence();
                    for (int i = te; i < M * kRowsBM; i += kEpiThreads) {
                        const int m = i / kRowsBM, c = n0 + i % kRowsBM;
                        if (c < N) {
                            float acc = __ldcg(part + (size_t)m * N + c);
                            for (int s2 = 1; s2 < S; s2++) acc += __ldcg(part + ((size_t)s2 * M + m) * N + c);
                            C[(size_t)m * ldc + c] = acc;
                        }
                    }
                }
                named_bar(1, kEpiThreads);  // last_flag is rewritten by the next item
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::TmemCols));
}

// x -> (xh, xl) with xh = fp16(x), xl = fp16((x - xh) * 2048), rows of xl after those of xh
__global__ void k_f32_to_f16_split(const float* __restrict__ x, __half* __restrict__ y, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 2; i += (size_t)gridDim.x * blockDim.x) {
        const float2 v = reinterpret_cast<const float2*>(x)[i];
        const __half2 h = __floats2half2_rn(v.x, v.y);
        const float2 hf = __half22float2(h);
        reinterpret_cast<__half2*>(y)[i] = h;
        reinterpret_cast<__half2*>(y + n)[i] = __floats2half2_rn((v.x - hf.x) * 2048.f, (v.y - hf.y) * 2048.f);
    }
}

__global__ void k_f32_to_f16(const float* __restrict__ x, __half* __restrict__ y, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 2; i += (size_t)gridDim.x * blockDim.x) {
        const float2 v = reinterpret_cast<const float2*>(x)[i];
        reinterpret_cast<__half2*>(y)[i] = __floats2half2_rn(v.x, v.y);
    }
}

}  // namespace

bool gemm_q8_supported(const DTensor& W) { return W.K % 32 == 0 && W.K >= 32 && W.K % 8 == 0; }

bool gemm_exact() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("QQ3_GEMM_FAST");
        v = (e && atoi(e) != 0) ? 0 : 1;
    }
    return v == 1;
}

size_t gemm_q8_scratch_bytes(int64_t M, int64_t K) { return (size_t)M * K * sizeof(__half) * (gemm_exact() ? 2 : 1); }

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        QQ_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        QQ_CHECK(p != nullptr && q == cudaDriverEntryPointSuccess, QQ_ERR_CUDA, "cuTensorMapEncodeTiled not available");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D tensor map over a row-major [rows][cols] matrix; box = box_cols x box_rows.
CUtensorMap tensor_map(void* base, CUtensorMapDataType type, int elem_bytes, uint64_t cols, uint64_t rows,
                       uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * (cuuint64_t)elem_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, type, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    QQ_CHECK(r == CUDA_SUCCESS, QQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return m;
}

// Block scales by TMA when the rows of the scale plane are 16-byte multiples (K % 256 == 0): a
// box of 8 scales x `rows` rows per K step.  Otherwise the converters load them directly.
bool scales_by_tma(const DTensor& W) { return (W.K / 32) % 8 == 0 && ((uintptr_t)W.d & 15u) == 0; }

CUtensorMap scale_map(const DTensor& W, int rows) {
    return tensor_map(W.d, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)(W.K / 32), (uint64_t)W.rows, 8,
                      (uint32_t)rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace

template <int SPLIT>
void launch_split(const DTensor& W, int64_t N, const __half* a16, int M, float* y, int ldc, const GemmGroups* groups,
                  cudaStream_t s) {
    using G = Cfg<SPLIT>;
    const int64_t K = W.K;
    // TMA: the fp16 activations arrive already 128-byte swizzled (hi rows, then lo rows when
    // split); the int8 weights plain
    const CUtensorMap ta = tensor_map(const_cast<__half*>(a16), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)K,
                                      (uint64_t)M * (SPLIT == 3 ? 2 : 1), kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap tb = tensor_map(W.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)W.rows, kBK,
                                      G::BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    const bool d_tma = scales_by_tma(W);
    const CUtensorMap td = d_tma ? scale_map(W, G::BN) : tb;
    if (first_use_on_device(reinterpret_cast<const void*>(k_gemm_q8_tma<SPLIT>)))
        QQ_CUDA_TRY(cudaFuncSetAttribute(k_gemm_q8_tma<SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::Smem));
    QQ_CHECK(N <= (int64_t)65535 * G::BN, QQ_ERR_INVALID, "tensor-core Q8_0 matmul: too many columns");
    const unsigned gx = groups ? (unsigned)groups->max_tiles : (unsigned)((M + kBM - 1) / kBM);
    dim3 grid(gx, (unsigned)((N + G::BN - 1) / G::BN));
    k_gemm_q8_tma<SPLIT><<<grid, kThreadsG2, G::Smem, s>>>(ta, tb, td, d_tma ? 1 : 0, M, (int)K, W.d, (int)N, y, ldc,
                                                           groups ? groups->tiles : nullptr,
                                                           groups ? groups->n_tiles : nullptr, kernel_err_ptr());
    QQ_CUDA_TRY(cudaGetLastError());
}

namespace {

// splits S of the raw K stages per 128-row tile: fewest rounds of one item per SM per unit of work
int rows_splits(int64_t N, int64_t K) {
    const int tiles = (int)((N + kRowsBM - 1) / kRowsBM);
    const int nk = (int)((K + kRowsKR - 1) / kRowsKR);
    const int sms = num_sms();
    int best = 1;
    double best_t = (double)((tiles + sms - 1) / sms);
    for (int S = 2; S <= 16 && 2 * S <= nk && tiles * S <= kRowsMaxItems; S++) {
        const double tt = (double)((tiles * S + sms - 1) / sms) / S;
        if (tt < best_t - 1e-9) {
            best = S;
            best_t = tt;
        }
    }
    return best;
}

template <int MN>
void launch_rows(const DTensor& W, const __half* a16, int M, float* y, int ldc, void* rows_scratch, cudaStream_t s) {
    using G = RowsCfg<MN>;
    const int64_t K = W.K, N = W.rows;
    const CUtensorMap tx = tensor_map(const_cast<__half*>(a16), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)K,
                                      (uint64_t)M * 2, kBK, MN, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap tw = tensor_map(W.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)W.rows, 128,
                                      kRowsBM, CU_TENSOR_MAP_SWIZZLE_128B);
    const bool d_tma = scales_by_tma(W);
    const CUtensorMap td = d_tma ? scale_map(W, kRowsBM) : tw;
    if (first_use_on_device(reinterpret_cast<const void*>(k_gemm_q8_rows<MN>)))
        QQ_CUDA_TRY(cudaFuncSetAttribute(k_gemm_q8_rows<MN>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::Smem));
    // the wide form takes its work from the activation tiles and never splits K
    const int S = G::Wide ? 1 : rows_splits(N, K);
    const int64_t n_at = (M + MN - 1) / MN;
    QQ_CHECK(G::Wide || n_at == 1, QQ_ERR_INVALID, "few-row Q8_0 matmul: more rows than the form takes");
    const int64_t items = ((N + kRowsBM - 1) / kRowsBM) * n_at * S;
    QQ_CHECK(items <= (int64_t)1 << 30, QQ_ERR_INVALID, "few-row Q8_0 matmul: too many rows");
    const unsigned grid = (unsigned)std::min<int64_t>(items, num_sms());
    QQ_CHECK(S == 1 || rows_scratch, QQ_ERR_INVALID, "few-row Q8_0 matmul: split K needs the scratch");
    unsigned int* tickets = static_cast<unsigned int*>(rows_scratch);
    float* part = rows_scratch ? reinterpret_cast<float*>(static_cast<char*>(rows_scratch) +
                                                          kRowsTickets * sizeof(unsigned int))
                               : nullptr;
    k_gemm_q8_rows<MN><<<grid, kRowsThreads, G::Smem, s>>>(tx, tw, td, d_tma ? 1 : 0, M, (int)K, W.d, (int)N, y, ldc,
                                                           part, tickets, S,
                                                           (int)items, kernel_err_ptr());
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace

size_t gemm_rows_scratch_bytes(int M) {
    return kRowsTickets * sizeof(unsigned int) + (size_t)kRowsMaxItems * kRowsBM * (size_t)std::max(M, 1) * 4;
}

void gemm_rows_reset(void* rows_scratch, cudaStream_t s) {
    QQ_CUDA_TRY(cudaMemsetAsync(rows_scratch, 0, kRowsTickets * sizeof(unsigned int), s));
}

void launch_gemm_q8_few(const DTensor& W, const float* x, int M, __half* x16, void* rows_scratch, float* y,
                        cudaStream_t s, bool x16_ready) {
    if (M <= 0 || W.rows <= 0) return;
    if (!rows_scratch || M > kGemmFewMax || !gemm_exact()) {
        launch_gemm_q8(W, x, M, x16, y, s, x16_ready);
        return;
    }
    QQ_CHECK(gemm_q8_supported(W), QQ_ERR_INVALID, "tensor-core Q8_0 matmul: K must be a multiple of 32");
    if (!x16_ready) launch_f32_to_f16(x, x16, (size_t)M * W.K, s);
    if (M <= 16) launch_rows<16>(W, x16, M, y, (int)W.rows, rows_scratch, s);
    else launch_rows<32>(W, x16, M, y, (int)W.rows, rows_scratch, s);
}

void launch_gemm_q8_f16(const DTensor& W, int64_t group_rows, const __half* a16, int M, float* y, int ldc,
                        const GemmGroups* groups, cudaStream_t s) {
    const int64_t N = group_rows;
    QQ_CHECK(gemm_q8_supported(W), QQ_ERR_INVALID, "tensor-core Q8_0 matmul: K must be a multiple of 32");
    QQ_CHECK(N >= 1 && W.rows % N == 0 && M <= 65535 * kBM, QQ_ERR_INVALID, "tensor-core Q8_0 matmul: bad shape");
    if (M <= 0) return;
    // a dense product of more rows with enough (weight tile, 128-row activation tile) items for
    // every SM: the wide tensor-memory form (QQ3_GEMM_WIDE=0 keeps the 128-row activation tile)
    static const bool wide_off = [] {
        const char* e = getenv("QQ3_GEMM_WIDE");
        return e && atoi(e) == 0;
    }();
    if (!groups && gemm_exact() && !wide_off && M > kGemmFewMax && N == W.rows &&
        ((N + kRowsBM - 1) / kRowsBM) * ((M + 127) / 128) >= num_sms()) {
        launch_rows<128>(W, a16, M, y, ldc, nullptr, s);
        return;
    }
    if (gemm_exact()) launch_split<3>(W, N, a16, M, y, ldc, groups, s);
    else launch_split<1>(W, N, a16, M, y, ldc, groups, s);
}

void launch_f32_to_f16(const float* x, __half* y, size_t n, cudaStream_t s) {
    if (n == 0) return;
    const unsigned g = (unsigned)std::min<size_t>((n / 2 + 255) / 256, 148 * 16);
    if (gemm_exact()) k_f32_to_f16_split<<<g, 256, 0, s>>>(x, y, n);
    else k_f32_to_f16<<<g, 256, 0, s>>>(x, y, n);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_gemm_q8(const DTensor& W, const float* x, int M, __half* x16, float* y, cudaStream_t s, bool x16_ready) {
    if (M <= 0 || W.rows <= 0) return;
    if (!x16_ready) launch_f32_to_f16(x, x16, (size_t)M * W.K, s);
    launch_gemm_q8_f16(W, W.rows, x16, M, y, (int)W.rows, nullptr, s);
}

}  // namespace qq3
