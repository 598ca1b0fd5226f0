// kernels_sample.cu -- next-token sampling on the device (sm_100a).
//
// sampleWithThinkControl (tensor.js:244-265) over the logits of a decode step, so that a
// sampled generate() needs no logits readback:
//   * think control: 'suppress' treats logits[thinkId] as -Infinity; 'shorten' (until the end
//     of thinking was produced) returns endThinkId when fewer than topK logits exceed its logit;
//   * temperature <= 0: sampleGreedy (tensor.js:231-237), the first maximum (NaN never wins);
//   * otherwise sampleTopPTopK (tensor.js:188-228): probabilities exp((l - max) / T) stored as
//     f32, normalised by 1 / (their f64 sum) and stored as f32 again; the topK most probable
//     (ties: lower id first, as the stable sort leaves them); cut after the first prefix whose
//     f64 cumulative sum reaches topP; then the first prefix whose cumulative sum reaches r;
//     when r exceeds the kept mass, the last id of the full sorted order (the least probable,
//     ties: the highest id), as the JS loop falls through to indexed[n - 1].
//
// One CTA of 1024 threads: max, sum and probabilities in three passes over the logits, the
// top-K by an exact MSB radix select on the f32 probability bits (four 8-bit passes over a
// u32 key array), the K candidates bitonic-sorted in shared memory, the final walk by one thread.
// The f64 sum of the probabilities is reassociated (per-thread runs, then a tree); the JS adds
// them in index order.  The two sums differ by a few f64 ulps, which moves a sampled id only
// when r falls within ~1e-15 of a cumulative boundary.  A NaN probability counts as 0.
//
// The uniform draw r is either given, or drawn from (seed, sequence, position) by a counter-based
// generator (splitmix64 finaliser, 53 bits), so that a host can reproduce every draw.
#include <cstdint>

#include "kernels.h"

namespace qq3 {

namespace {

constexpr int kSThreads = 1024;
constexpr int kSWarps = kSThreads / 32;

__device__ __forceinline__ double block_sum_d(double v, double* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    double r = 0.0;
    if (w == 0) {
        r = l < kSWarps ? red[l] : 0.0;
        for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
        if (l == 0) red[0] = r;
    }
    __syncthreads();
    return red[0];
}

__device__ __forceinline__ int block_sum_i(int v, int* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        int r = l < kSWarps ? red[l] : 0;
        for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
        if (l == 0) red[0] = r;
    }
    __syncthreads();
    return red[0];
}

// max over non-NaN values (the JS `if (x > m) m = x` scan from -Infinity)
__device__ __forceinline__ float block_max_f(float v, float* red) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));  // fmaxf drops NaN
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        float r = l < kSWarps ? red[l] : -INFINITY;
        for (int o = 16; o; o >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
        if (l == 0) red[0] = r;
    }
    __syncthreads();
    return red[0];
}

template <bool kMax>
__device__ __forceinline__ unsigned long long block_ext_u64(unsigned long long v, unsigned long long* red) {
    for (int o = 16; o; o >>= 1) {
        const unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
        v = kMax ? (u > v ? u : v) : (u < v ? u : v);
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        unsigned long long r = l < kSWarps ? red[l] : (kMax ? 0ull : ~0ull);
        for (int o = 16; o; o >>= 1) {
            const unsigned long long u = __shfl_xor_sync(0xffffffffu, r, o);
            r = kMax ? (u > r ? u : r) : (u < r ? u : r);
        }
        if (l == 0) red[0] = r;
    }
    __syncthreads();
    return red[0];
}

// probability key -> composite key ordered as the JS sort: higher probability first, then lower id
__device__ __forceinline__ unsigned long long ckey(uint32_t pbits, int i) {
    return ((unsigned long long)pbits << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
}
__device__ __forceinline__ int ckey_id(unsigned long long k) { return (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)); }

__global__ void __launch_bounds__(kSThreads, 1)
    k_sample(const float* __restrict__ logits, int n, const SampleArgs* __restrict__ args, int* think_done, double r_in,
             int seq, int pos_in, int* ctl, int* trace, int* out, uint32_t* __restrict__ pk) {
    __shared__ double red_d[kSWarps];
    __shared__ float red_f[kSWarps];
    __shared__ int red_i[kSWarps];
    __shared__ unsigned long long red_u[kSWarps];
    __shared__ unsigned int hist[256];
    __shared__ unsigned long long cand[kSampleMaxTopK];
    __shared__ unsigned int n_cand, sel_prefix, sel_remaining;
    __shared__ int result_s;
    const int t = threadIdx.x;
    const SampleArgs A = *args;
    const int pos = pos_in >= 0 ? pos_in : (ctl ? ctl[1] - 1 : 0);
    // think ids beyond the vocabulary (LFM2's, against a smaller synthetic vocabulary) disable
    // think control, as a JS typed-array write out of bounds does for 'suppress'
    const int suppress = (A.think_mode == kThinkSuppress && A.think_id >= 0 && A.think_id < n) ? A.think_id : -1;
    const bool done = think_done ? (*think_done != 0) : (A.think_mode == kThinkSuppress);
    if (t == 0) result_s = -1;
    __syncthreads();
    auto logit = [&](int i) -> float { return i == suppress ? -INFINITY : __ldg(logits + i); };

    // 'shorten': force endThinkId while it ranks within the top K
    if (A.think_mode == kThinkShorten && !done && A.end_think_id >= 0 && A.end_think_id < n) {
        const float el = __ldg(logits + A.end_think_id);
        int c = 0;
        for (int i = t; i < n; i += kSThreads) c += __ldg(logits + i) > el ? 1 : 0;
        c = block_sum_i(c, red_i);
        if (t == 0 && c < A.top_k) result_s = A.end_think_id;
        __syncthreads();
    }
    if (result_s < 0 && A.temperature <= 0.0) {
        // sampleGreedy: maxIdx starts at 0 and only a strictly greater value moves it, so a NaN
        // logit 0 wins, and otherwise the first maximum over the non-NaN values
        const float l0 = logit(0);
        unsigned long long best = 0ull;
        for (int i = t; i < n; i += kSThreads) {
            const float v = logit(i);
            if (v != v) continue;
            uint32_t b = __float_as_uint(v);
            b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // order-preserving
            const unsigned long long k = ((unsigned long long)b << 32) | (0xFFFFFFFFu - (uint32_t)i);
            best = k > best ? k : best;
        }
        best = block_ext_u64<true>(best, red_u);
        if (t == 0) result_s = (l0 != l0 || best == 0ull) ? 0 : ckey_id(best);
        __syncthreads();
    } else if (result_s < 0) {
        // max, then e = f32(exp((l - max) / T)) and its f64 sum, then p = f32(e * (1 / sum))
        float mx = -INFINITY;
        for (int i = t; i < n; i += kSThreads) mx = fmaxf(mx, logit(i));
        mx = block_max_f(mx, red_f);
        const int chunk = (n + kSThreads - 1) / kSThreads;
        const int i0 = min(n, t * chunk), i1 = min(n, i0 + chunk);
        double s = 0.0;
        for (int i = i0; i < i1; i++) {
            const float e = (float)exp(((double)logit(i) - (double)mx) / A.temperature);
            pk[i] = __float_as_uint(e);
            s += (double)e;
        }
        const double inv = 1.0 / block_sum_d(s, red_d);
        unsigned long long last = ~0ull;  // the last id of the full sorted order
        for (int i = i0; i < i1; i++) {
            float p = (float)((double)__uint_as_float(pk[i]) * inv);
            if (!(p > 0.f)) p = 0.f;  // NaN and -0 count as 0
            const uint32_t b = __float_as_uint(p);
            pk[i] = b;
            const unsigned long long k = ckey(b, i);
            last = k < last ? k : last;
        }
        last = block_ext_u64<false>(last, red_u);
        // K-th largest probability bits by an MSB radix select, 8 bits a pass
        const int K = min(A.top_k, n);
        if (t == 0) {
            sel_prefix = 0u;
            sel_remaining = (unsigned)K;
        }
        uint32_t mask = 0u;
        for (int shift = 24; shift >= 0; shift -= 8) {
            if (t < 256) hist[t] = 0u;
            __syncthreads();
            const uint32_t prefix = sel_prefix;
            for (int i = i0; i < i1; i++) {
                const uint32_t u = pk[i];
                if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (t == 0) {
                unsigned int cum = 0u, rem = sel_remaining;
                int b = 255;
                for (; b > 0; b--) {
                    if (cum + hist[b] >= rem) break;
                    cum += hist[b];
                }
                sel_prefix = prefix | ((uint32_t)b << shift);
                sel_remaining = rem - cum;
            }
            mask |= 255u << shift;
            __syncthreads();
        }
        // candidates: every probability above the threshold, and the lowest ids equal to it
        const uint32_t thr = sel_prefix;
        const int need_eq = (int)sel_remaining;
        if (t == 0) n_cand = 0u;
        __syncthreads();
        int eq = 0;
        for (int i = i0; i < i1; i++) {
            const uint32_t u = pk[i];
            if (u > thr) cand[atomicAdd(&n_cand, 1u)] = ckey(u, i);
            eq += u == thr ? 1 : 0;
        }
        // exclusive prefix of the equal counts in thread (= id) order
        int incl = eq;
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if ((t & 31) >= o) incl += v;
        }
        __syncthreads();
        if ((t & 31) == 31) red_i[t >> 5] = incl;
        __syncthreads();
        if (t < 32) {
            int v = red_i[t];
            for (int o = 1; o < 32; o <<= 1) {
                const int w = __shfl_up_sync(0xffffffffu, v, o);
                if (t >= o) v += w;
            }
            red_i[t] = v;  // inclusive over warps
        }
        __syncthreads();
        int before = incl - eq + ((t >> 5) ? red_i[(t >> 5) - 1] : 0);
        for (int i = i0; i < i1 && before < need_eq; i++)
            if (pk[i] == thr) {
                cand[atomicAdd(&n_cand, 1u)] = ckey(thr, i);
                before++;
            }
        __syncthreads();
        // bitonic sort of the K candidates, descending (padding keys 0 sort last)
        int P = 1;
        while (P < K) P <<= 1;
        for (int i = t + K; i < P; i += kSThreads) cand[i] = 0ull;
        __syncthreads();
        for (int size = 2; size <= P; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = t; i < P; i += kSThreads) {
                    const int j = i ^ stride;
                    if (j > i) {
                        const bool desc = (i & size) == 0;
                        const unsigned long long a = cand[i], b = cand[j];
                        if (desc ? (a < b) : (a > b)) {
                            cand[i] = b;
                            cand[j] = a;
                        }
                    }
                }
                __syncthreads();
            }
        }
        if (t == 0) {
            // top-p cut, then the walk with r
            const double r = r_in >= 0.0 ? r_in : sample_uniform(A.seed, seq, pos);
            int kept = K;
            double cum = 0.0;
            for (int i = 0; i < K; i++) {
                cum += (double)__uint_as_float((uint32_t)(cand[i] >> 32));
                if (cum >= A.top_p) {
                    kept = i + 1;
                    break;
                }
            }
            int res = ckey_id(last);
            cum = 0.0;
            for (int i = 0; i < kept; i++) {
                cum += (double)__uint_as_float((uint32_t)(cand[i] >> 32));
                if (r <= cum) {
                    res = ckey_id(cand[i]);
                    break;
                }
            }
            result_s = res;
        }
        __syncthreads();
    }
    if (t == 0) {
        const int tok = result_s;
        out[0] = tok;
        if (ctl) {
            ctl[0] = tok;
            if (trace) trace[ctl[1]] = tok;
        }
        if (think_done && tok == A.end_think_id) *think_done = 1;
    }
}

}  // namespace

void launch_sample(const float* logits, int n, const SampleArgs* args_dev, int* think_done, double r, int seq,
                   int pos, int* ctl, int* trace, int* out, uint32_t* scratch, cudaStream_t s) {
    QQ_CHECK(n >= 1, -1, "sampling needs at least one logit");
    k_sample<<<1, kSThreads, 0, s>>>(logits, n, args_dev, think_done, r, seq, pos, ctl, trace, out, scratch);
    QQ_CUDA_TRY(cudaGetLastError());
}

}  // namespace qq3
