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
#include "qq3.h"

namespace qq3 {

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kStages = 3;
constexpr uint32_t kTmemCols = 256;

// K-major, 128-byte swizzle: row r of a tile is 128 B (64 fp16 of K) at r*128; its 16-byte
// chunk c sits at chunk position c ^ (r & 7).  Tiles start on 1024-byte boundaries.
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
    return (uint32_t)row * 128u + (uint32_t)((chunk ^ (row & 7)) << 4);
}

// Shared-memory matrix descriptor (sm100 UMMA): start address >> 4, leading byte offset 1
// (unused for swizzled K-major), stride byte offset 1024 >> 4 between 8-row groups,
// version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

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
    static constexpr int Stage = NT * ATile + NT * BTile + RawTile;
    static constexpr int Smem = kStages * Stage + 1024;
    static constexpr uint32_t Idesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
    static constexpr int RowThreads = 256 / BN;       // converter threads per B row
};

__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    const uint32_t mask[4] = {0u, 0u, 0u, 0u};
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(mask[0]), "r"(mask[1]), "r"(mask[2]), "r"(mask[3]));
}

__device__ __forceinline__ uint32_t h2bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

template <int SPLIT>
__global__ void __launch_bounds__(kThreadsG2, 1)
    k_gemm_q8_tma(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int K,
                  const __half* __restrict__ d, int N, float* __restrict__ C, int ldc, const int4* __restrict__ tiles,
                  const int* __restrict__ n_tiles, int* err) {
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
                mbar_arrive_expect_tx(&full_raw[s], (uint32_t)G::RawTile);
                tma_2d(raw_tile(st), &tmB, kt * kBK, nb0, &full_raw[s]);
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
        uint32_t dnext = load_d(0);
        for (int kt = 0; kt < nk && ok; kt++) {
            const int s = kt % kStages;
            const uint32_t pu = (uint32_t)((kt / kStages) & 1);
            const uint32_t dcur = dnext;
            if (kt + 1 < nk) dnext = load_d(kt + 1);
            uint8_t* st = smem + s * G::Stage;
            ok = __all_sync(0xffffffffu, bar_wait(&full_raw[s], pu, err));  // warp-uniform outcome
            uint4 raw[WPT / 16];
            if (ok) {
                const uint4* rp = reinterpret_cast<const uint4*>(raw_tile(st) + brow * kBK + part * WPT);
#pragma unroll
                for (int j = 0; j < WPT / 16; j++) raw[j] = rp[j];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_free[s]);
            if (ok && kt >= kStages)
                ok = __all_sync(0xffffffffu, bar_wait(&mma_done[s], (uint32_t)((kt / kStages - 1) & 1), err));
            if (!ok) break;
            const __half2 dc = *reinterpret_cast<const __half2*>(&dcur);
            const int c0 = part * (WPT / 8);  // first 8-weight chunk of this thread in the row
            // SPLIT = 3 in half2 arithmetic when |d| < 1/4: then |q d| < 32, so 2048 wh and 2048 d
            // are finite fp16 values (each thread's weights share one block scale here)
            const float dfs = __low2float(dc);
            const bool split_fast = SPLIT == 3 && RT == 2 && fabsf(dfs) < 0.25f;
            const __half2 d2s = __low2half2(dc);
            const __half2 d2k = __float2half2_rn(dfs * 2048.0f);
            const __half2 m2k = __float2half2_rn(-2048.0f);
#pragma unroll
            for (int c = 0; c < WPT / 8; c++) {
                const uint4 r4 = raw[c >> 1];
                const uint32_t w0 = (c & 1) ? r4.z : r4.x, w1 = (c & 1) ? r4.w : r4.y;
                if (SPLIT == 1) {
                    const __half2 d2 = (c >> 2) ? __high2half2(dc) : __low2half2(dc);
                    uint4 o;
                    dq4(w0, d2, o.x, o.y);
                    dq4(w1, d2, o.z, o.w);
                    *reinterpret_cast<uint4*>(b_tile(st, 0) + sw128(brow, c0 + c)) = o;
                } else if (split_fast) {
                    // wh = RN16(q d) (one HMUL2) and wl = RN16((q d - wh) 2048) (one HFMA2 on
                    // d 2048 and -2048 wh, both exact scalings): the same bits as the f32 path
                    // below, at full-rate half2 arithmetic instead of conversions
                    uint32_t hw[4], lw[4];
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const uint32_t u = (j ? w1 : w0) ^ 0x80808080u;  // b + 128 per byte
                        uint32_t pa = __byte_perm(u, 0x64646464u, 0x5140), pb = __byte_perm(u, 0x64646464u, 0x5342);
                        const __half2 bias = __float2half2_rn(1152.0f);
                        const __half2 qa = __hsub2(*reinterpret_cast<__half2*>(&pa), bias);  // exact q pairs
                        const __half2 qb = __hsub2(*reinterpret_cast<__half2*>(&pb), bias);
                        const __half2 ha = __hmul2(qa, d2s), hb = __hmul2(qb, d2s);
                        hw[2 * j] = h2bits(ha);
                        hw[2 * j + 1] = h2bits(hb);
                        lw[2 * j] = h2bits(__hfma2(qa, d2k, __hmul2(ha, m2k)));
                        lw[2 * j + 1] = h2bits(__hfma2(qb, d2k, __hmul2(hb, m2k)));
                    }
                    *reinterpret_cast<uint4*>(b_tile(st, 0) + sw128(brow, c0 + c)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    *reinterpret_cast<uint4*>(b_tile(st, 1) + sw128(brow, c0 + c)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                } else {
                    const float df = __low2float(dc);
                    uint32_t hw[4], lw[4];
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const uint32_t word = j < 2 ? w0 : w1;
                        const int sh = 16 * (j & 1);
                        const float wa = (float)(int8_t)((word >> sh) & 0xff) * df;        // exact
                        const float wb = (float)(int8_t)((word >> (sh + 8)) & 0xff) * df;
                        const __half2 h = __floats2half2_rn(wa, wb);
                        const float2 hf = __half22float2(h);
                        hw[j] = h2bits(h);
                        lw[j] = h2bits(__floats2half2_rn((wa - hf.x) * 2048.f, (wb - hf.y) * 2048.f));  // exact
                    }
                    *reinterpret_cast<uint4*>(b_tile(st, 0) + sw128(brow, c0 + c)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    *reinterpret_cast<uint4*>(b_tile(st, 1) + sw128(brow, c0 + c)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
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
    static bool init = false;
    if (!init) {
        QQ_CUDA_TRY(cudaFuncSetAttribute(k_gemm_q8_tma<SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::Smem));
        init = true;
    }
    QQ_CHECK(N <= (int64_t)65535 * G::BN, QQ_ERR_INVALID, "tensor-core Q8_0 matmul: too many columns");
    const unsigned gx = groups ? (unsigned)groups->max_tiles : (unsigned)((M + kBM - 1) / kBM);
    dim3 grid(gx, (unsigned)((N + G::BN - 1) / G::BN));
    k_gemm_q8_tma<SPLIT><<<grid, kThreadsG2, G::Smem, s>>>(ta, tb, M, (int)K, W.d, (int)N, y, ldc,
                                                           groups ? groups->tiles : nullptr,
                                                           groups ? groups->n_tiles : nullptr, kernel_err_ptr());
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_gemm_q8_f16(const DTensor& W, int64_t group_rows, const __half* a16, int M, float* y, int ldc,
                        const GemmGroups* groups, cudaStream_t s) {
    const int64_t N = group_rows;
    QQ_CHECK(gemm_q8_supported(W), QQ_ERR_INVALID, "tensor-core Q8_0 matmul: K must be a multiple of 32");
    QQ_CHECK(N >= 1 && W.rows % N == 0 && M <= 65535 * kBM, QQ_ERR_INVALID, "tensor-core Q8_0 matmul: bad shape");
    if (M <= 0) return;
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

void launch_gemm_q8(const DTensor& W, const float* x, int M, __half* x16, float* y, cudaStream_t s) {
    if (M <= 0 || W.rows <= 0) return;
    launch_f32_to_f16(x, x16, (size_t)M * W.K, s);
    launch_gemm_q8_f16(W, W.rows, x16, M, y, (int)W.rows, nullptr, s);
}

}  // namespace qq3
