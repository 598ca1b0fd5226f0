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
#include "kernels.h"
#include "pipe.cuh"
#include "qq3.h"

namespace qq3 {

namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 3;
constexpr int kThreadsG = 128;
constexpr int kATile = kBM * kBK * 2;  // 16 KB
constexpr int kBTile = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kATile + kBTile;
constexpr int kGemmSmem = kStages * kStageBytes + 1024;  // + alignment slack
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

// Instruction descriptor: D f32, A/B fp16, both K-major, N = kBN, M = kBM.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    const uint32_t mask[4] = {0u, 0u, 0u, 0u};
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate), "r"(mask[0]), "r"(mask[1]), "r"(mask[2]), "r"(mask[3]));
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

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(kThreadsG, 1)
    k_gemm_q8(const __half* __restrict__ A, int M, int K, const int8_t* __restrict__ qs, const __half* __restrict__ d,
              int N, float* __restrict__ C, int ldc, int* err) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t mma_bar[kStages];
    __shared__ uint32_t tmem_slot;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (t == 0) {
        for (int s = 0; s < kStages; s++) mbar_init(&mma_bar[s], 1);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const int nk = (K + kBK - 1) / kBK;
    const int KB = K >> 5;  // Q8_0 blocks per row
    bool ok = true;
    for (int kt = 0; kt < nk; kt++) {
        const int s = kt % kStages;
        // every thread waits for the tensor core to release this stage; the outcome is made
        // uniform by the barrier below, so all threads leave the loop together on a timeout
        if (kt >= kStages) ok = bar_wait(&mma_bar[s], (uint32_t)((kt / kStages - 1) & 1), err) && ok;
        uint8_t* sa = smem + s * kStageBytes;
        uint8_t* sb = sa + kATile;
        const int k0 = kt * kBK;
        // A: thread t converts row t of the tile (64 fp16 = 8 chunks); zero past M or K
        {
            const int row = t, m = m0 + row;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                const int k = k0 + 8 * c;
                if (m < M && k < K) v = __ldg(reinterpret_cast<const uint4*>(A + (size_t)m * K + k));
                *reinterpret_cast<uint4*>(sa + sw128(row, c)) = v;
            }
        }
        // B: thread t dequantises rows t and t + 128 (64 weights = two Q8_0 blocks each)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int row = t + h * kThreadsG, n = n0 + row;
#pragma unroll
            for (int b = 0; b < 2; b++) {
                const int kb = (k0 >> 5) + b;
                uint4 q0 = make_uint4(0u, 0u, 0u, 0u), q1 = q0;
                float sc = 0.f;
                if (n < N && kb < KB) {
                    const uint4* qp = reinterpret_cast<const uint4*>(qs + (size_t)n * K + (size_t)kb * 32);
                    q0 = __ldg(qp);
                    q1 = __ldg(qp + 1);
                    sc = __half2float(d[(size_t)n * KB + kb]);
                }
                const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int c = 0; c < 4; c++) {  // 8 weights per 16-byte chunk
                    const uint32_t lo = w[2 * c], hi = w[2 * c + 1];
                    uint4 o;
                    o.x = pack_h2((float)(int8_t)(lo & 0xff) * sc, (float)(int8_t)((lo >> 8) & 0xff) * sc);
                    o.y = pack_h2((float)(int8_t)((lo >> 16) & 0xff) * sc, (float)(int8_t)(lo >> 24) * sc);
                    o.z = pack_h2((float)(int8_t)(hi & 0xff) * sc, (float)(int8_t)((hi >> 8) & 0xff) * sc);
                    o.w = pack_h2((float)(int8_t)((hi >> 16) & 0xff) * sc, (float)(int8_t)(hi >> 24) * sc);
                    *reinterpret_cast<uint4*>(sb + sw128(row, 4 * b + c)) = o;
                }
            }
        }
        fence_async_smem();  // generic-proxy stores -> visible to the tensor core (async proxy)
        ok = __syncthreads_and(ok);
        if (!ok) break;
        if (t == 0) {
            tc_fence_after();
            const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb);
#pragma unroll
            for (int ks = 0; ks < kBK / 16; ks++)  // K = 16 fp16 = 32 bytes per instruction
                umma_f16(tmem, umma_desc(a0 + 32u * ks), umma_desc(b0 + 32u * ks), (kt | ks) != 0 ? 1u : 0u);
            umma_commit(&mma_bar[s]);
        }
    }
    // the last commit covers every MMA issued before it
    if (ok && nk > 0) ok = bar_wait(&mma_bar[(nk - 1) % kStages], (uint32_t)(((nk - 1) / kStages) & 1), err);
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (ok) {
        const int row = warp * 32 + lane, m = m0 + row;
#pragma unroll 1
        for (int c0 = 0; c0 < kBN; c0 += 16) {
            uint32_t v[16];
            const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                "[%16];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                  "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (m < M) {
                float* crow = C + (size_t)m * ldc + n0 + c0;
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (n0 + c0 + j < N) crow[j] = __uint_as_float(v[j]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

__global__ void k_f32_to_f16(const float* __restrict__ x, __half* __restrict__ y, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 2; i += (size_t)gridDim.x * blockDim.x) {
        const float2 v = reinterpret_cast<const float2*>(x)[i];
        reinterpret_cast<__half2*>(y)[i] = __floats2half2_rn(v.x, v.y);
    }
}

}  // namespace

bool gemm_q8_supported(const DTensor& W) { return W.K % 32 == 0 && W.K >= 32 && W.K % 8 == 0; }

size_t gemm_q8_scratch_bytes(int64_t M, int64_t K) { return (size_t)M * K * sizeof(__half); }

void launch_gemm_q8(const DTensor& W, const float* x, int M, __half* x16, float* y, cudaStream_t s) {
    const int64_t K = W.K, N = W.rows;
    QQ_CHECK(gemm_q8_supported(W), QQ_ERR_INVALID, "tensor-core Q8_0 matmul: K must be a multiple of 32");
    QQ_CHECK(N <= (int64_t)65535 * kBN && M <= 65535 * kBM, QQ_ERR_INVALID, "tensor-core Q8_0 matmul: too large");
    if (M <= 0 || N <= 0) return;
    const size_t n = (size_t)M * K;
    k_f32_to_f16<<<(unsigned)std::min<size_t>((n / 2 + 255) / 256, 148 * 16), 256, 0, s>>>(x, x16, n);
    QQ_CUDA_TRY(cudaGetLastError());
    static bool init = false;
    if (!init) {
        QQ_CUDA_TRY(cudaFuncSetAttribute(k_gemm_q8, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
        init = true;
    }
    dim3 grid((unsigned)((N + kBN - 1) / kBN), (unsigned)((M + kBM - 1) / kBM));
    k_gemm_q8<<<grid, kThreadsG, kGemmSmem, s>>>(x16, M, (int)K, W.qs, W.d, (int)N, y, (int)N, kernel_err_ptr());
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace qq3
