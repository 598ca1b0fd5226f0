// kernels_misc.cu -- Q8_0 block repack/dequant, embedding gather, standalone RMSNorm,
// decode-loop bookkeeping (sm_100a).
#include "kernels.h"

namespace qq3 {

// Raw GGUF Q8_0 blocks (fp16 d, 32 x int8; 34 bytes, tensor.js:1-2) -> qs/d planes.
// One thread per block; the 34-byte stride keeps only 2-byte alignment so the block is read
// as 17 halfwords, then written as two 16-byte vectors.
__global__ void k_repack_q8(const uint16_t* __restrict__ raw, int64_t n_blocks, int8_t* __restrict__ qs,
                            __half* __restrict__ d) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    const uint16_t* p = raw + b * 17;
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; i++) w[i] = (uint32_t)p[1 + 2 * i] | ((uint32_t)p[2 + 2 * i] << 16);
    uint4* dst = reinterpret_cast<uint4*>(qs + b * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    d[b] = __ushort_as_half(p[0]);
}

// Transpose of n_mat row-major matrices [rows][cols] -> [cols][rows], 32 x 32 tiles through
// shared memory (both sides coalesced).
template <typename T>
__global__ void k_transpose(const T* __restrict__ in, int rows, int cols, T* __restrict__ out) {
    __shared__ T tile[32][33];
    const int64_t m = blockIdx.z;
    const T* src = in + m * rows * (int64_t)cols;
    T* dst = out + m * rows * (int64_t)cols;
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int y = threadIdx.y; y < 32; y += blockDim.y) {
        const int r = r0 + y, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[y][threadIdx.x] = src[(int64_t)r * cols + c];
    }
    __syncthreads();
    for (int y = threadIdx.y; y < 32; y += blockDim.y) {
        const int c = c0 + y, r = r0 + threadIdx.x;
        if (r < rows && c < cols) dst[(int64_t)c * rows + r] = tile[threadIdx.x][y];
    }
}

void launch_transpose_experts(const DTensor& W, int n_expert, int8_t* t_qs, __half* t_d, cudaStream_t s) {
    const int64_t rows = W.rows / n_expert, K = W.K;
    QQ_CHECK(W.type == 8 && W.rows % n_expert == 0 && K % 32 == 0 && rows <= (1 << 20) && K <= (1 << 20), -4,
             "expert transpose: unsupported tensor");
    const dim3 blk(32, 8);
    k_transpose<int8_t><<<dim3((unsigned)((K + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)n_expert), blk, 0, s>>>(
        W.qs, (int)rows, (int)K, t_qs);
    QQ_CUDA_TRY(cudaGetLastError());
    k_transpose<__half><<<dim3((unsigned)((K / 32 + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)n_expert), blk, 0, s>>>(
        W.d, (int)rows, (int)(K / 32), t_d);
    QQ_CUDA_TRY(cudaGetLastError());
}

void launch_repack_q8(const uint8_t* raw, int64_t n_blocks, int8_t* qs, __half* d, cudaStream_t s) {
    if (n_blocks <= 0) return;
    const int t = 256;
    k_repack_q8<<<(unsigned)((n_blocks + t - 1) / t), t, 0, s>>>(reinterpret_cast<const uint16_t*>(raw), n_blocks,
                                                                   qs, d);
    QQ_CUDA_TRY(cudaGetLastError());
}

// Element value q*d in storage order (exact in f32: <= 18 significant bits).
__global__ void k_dequant_q8(const int8_t* __restrict__ qs, const __half* __restrict__ d, int64_t n,
                             float* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (float)qs[i] * __half2float(d[i >> 5]);
}

void launch_dequant_q8(const DTensor& W, float* out, cudaStream_t s) {
    const int64_t n = W.K * W.rows;
    if (n <= 0) return;
    int grid = (int)((n + 255) / 256);
    if (grid > num_sms() * 16) grid = num_sms() * 16;
    k_dequant_q8<<<grid, 256, 0, s>>>(W.qs, W.d, n, out);
    QQ_CUDA_TRY(cudaGetLastError());
}

// embeddingLookupQ80 (tensor.js:56-77) with the token id read from device memory, so the
// whole decode step can be replayed from a CUDA graph.  Also clears the argmax slot.
__global__ void k_embed(const int8_t* __restrict__ qs, const __half* __restrict__ d, int K, int n_vocab,
                        const int* __restrict__ token, float* __restrict__ hidden, unsigned long long* best) {
    int t = *token;
    if (t < 0 || t >= n_vocab) t = 0;  // out-of-range ids are rejected on the host before launch
    const int8_t* q = qs + (int64_t)t * K;
    const __half* dd = d + (int64_t)t * (K >> 5);
    for (int i = threadIdx.x; i < K; i += blockDim.x) hidden[i] = (float)q[i] * __half2float(dd[i >> 5]);
    if (best && threadIdx.x == 0) *best = 0ull;
}

void launch_embed(const DTensor& E, const int* token, float* hidden, unsigned long long* argmax_reset,
                  cudaStream_t s) {
    QQ_CHECK(E.type == 8, -4, "embedding must be Q8_0");
    k_embed<<<1, 512, 0, s>>>(E.qs, E.d, (int)E.K, (int)E.ne[1], token, hidden, argmax_reset);
    QQ_CUDA_TRY(cudaGetLastError());
}

// Row-wise RMSNorm (tensor.js:103-114, per head: 117-129).  y may alias x.
__global__ void k_rmsnorm(const float* __restrict__ x, int n, const float* __restrict__ w, float eps, float* y) {
    __shared__ double red[32];
    const float* xr = x + (int64_t)blockIdx.x * n;
    float* yr = y + (int64_t)blockIdx.x * n;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)xr[i] * xr[i];
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
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = (w[i] * xr[i]) * inv;
}

void launch_rmsnorm(float* x, int64_t n_rows, int n, const float* w, float eps, float* y, cudaStream_t s) {
    if (n_rows <= 0) return;
    // long rows (the hidden state) get more threads: shorter per-thread sums, less latency
    const int threads = n >= 2048 ? 1024 : (n >= 512 ? 256 : 128);
    k_rmsnorm<<<(unsigned)n_rows, threads, 0, s>>>(x, n, w, eps, y);
    QQ_CUDA_TRY(cudaGetLastError());
}

// Decode-loop bookkeeping: next token = argmax, position += 1 (both stay on the device),
// and the token is recorded at its position in the per-sequence trace.
__global__ void k_argmax_finish(const unsigned long long* best, int* ctl, int* trace) {
    const int t = argmax_key_index(*best);
    const int p = ctl[1] + 1;
    ctl[0] = t;
    ctl[1] = p;
    trace[p] = t;
}

void launch_argmax_finish(const unsigned long long* best, int* ctl, int* trace, cudaStream_t s) {
    k_argmax_finish<<<1, 1, 0, s>>>(best, ctl, trace);
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace qq3
