// common.cuh -- shared device helpers and internal types of libqq3cuda.so (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace qq3 {

// ---------------------------------------------------------------------------------------
// Error plumbing.  Every C-ABI entry point returns an int status and records a
// thread-local message retrievable through qq_last_error().
void set_error(const std::string& msg);

struct Error {
    int code;
    std::string msg;
};

#define QQ_CUDA_TRY(expr)                                                                      \
    do {                                                                                       \
        cudaError_t e_ = (expr);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            throw ::qq3::Error{-2, std::string(#expr) + ": " + cudaGetErrorString(e_)};         \
    } while (0)

#define QQ_CHECK(cond, code, msg)                                                              \
    do {                                                                                       \
        if (!(cond)) throw ::qq3::Error{(code), (msg)};                                        \
    } while (0)

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------------------
// Device-side Q8_0 tensor.  The raw GGUF blocks (fp16 d + 32 x int8, 34 bytes) are uploaded
// as-is and split once on the device into two planes so that every row starts on a 32-byte
// boundary and streams with 128-bit loads:
//   qs: int8  [rows][K]       row r = GGUF column r (output index), K = ne[0]
//   d : fp16  [rows][K/32]
// A packed expert tensor [K, N, E] is rows = N*E with expert e at rows [e*N, (e+1)*N).
// F32 tensors keep their float array in f32.
struct DTensor {
    int type = 0;  // ggml type: 0 F32, 8 Q8_0
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    int64_t K = 0;     // ne[0]
    int64_t rows = 0;  // product of ne[1..]
    int8_t* qs = nullptr;
    __half* d = nullptr;
    float* f32 = nullptr;
    int device = 0;
};

// ---------------------------------------------------------------------------------------
// Device helpers.

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum of the 4 signed bytes of w, each multiplied by the matching lane of x.
__device__ __forceinline__ float dot4_i8(uint32_t w, float4 x) {
    const int32_t v = (int32_t)w;
    float s = x.x * (float)((v << 24) >> 24);
    s = fmaf(x.y, (float)((v << 16) >> 24), s);
    s = fmaf(x.z, (float)((v << 8) >> 24), s);
    s = fmaf(x.w, (float)(v >> 24), s);
    return s;
}

// Ordered-key encoding for a (float value, index) argmax with "first maximum wins"
// (sampleGreedy, tensor.js:231-237): larger value first, then smaller index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}
__device__ __forceinline__ int argmax_key_index(unsigned long long k) {
    return (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
}

}  // namespace qq3
