// kernels_gemv.cu -- Q8_0 dequant-GEMV family for single-token decode (sm_100a).
//
// Replaces matmulQ80xF32 (tensor.js:26-53) and WGSL_MATMUL_Q8_0 / WGSL_MATMUL_EXPERT_Q80
// (webgpu.js:8-45, 1290-1324), with the elementwise ops that surround each call in the
// engines fused into the same launch (RMSNorm prologue; residual / SwiGLU / short-conv /
// MoE-combine / argmax epilogues).
//
// Work decomposition: a persistent grid of 256-thread CTAs.  Each CTA stages its input
// vector(s) in shared memory once, then every warp takes "items" in a grid-stride loop.
// An item is one output value; it needs S weight rows (S = 1 plain, 2 gate/up, 3 conv
// B/C/x, top_k for the MoE down-combine).  Lane l streams 16-byte chunks c = l, l+32, ...
// of each row with 128-bit non-allocating loads, multiplies by the matching 16 inputs,
// scales each half block by its fp16 d, and the warp reduces with shuffles.
#include "gemv_core.cuh"

namespace qq3 {

template <int S, class Map, class Epi>
__global__ void __launch_bounds__(kGemvThreads) k_gemv(XStage st, Map map, Epi epi, int n_items) {
    extern __shared__ float4 xs[];
    __shared__ double red[kGemvWarps];
    stage_x(st, xs, red);
    const int warp = threadIdx.x >> 5;
    const int nch = st.K >> 4;
    const int K4 = st.K >> 2;
    typename Epi::WarpState ws;
    epi.init(ws);
    for (int item = blockIdx.x * kGemvWarps + warp; item < n_items; item += gridDim.x * kGemvWarps) {
        Rows<S> r;
        map.get(item, r);
        const float4* xv[S];
#pragma unroll
        for (int s = 0; s < S; s++) xv[s] = xs + (size_t)r.xsel[s] * K4;
        float acc[S];
#pragma unroll
        for (int s = 0; s < S; s++) acc[s] = 0.f;
        lane_dots<S>(r.q, r.d, xv, r.on, nch, acc);
#pragma unroll
        for (int s = 0; s < S; s++) acc[s] = warp_sum(acc[s]);
        epi.apply(ws, item, acc, r.on);
    }
    epi.finish(ws);
}

// ---------------------------------------------------------------------------------------
// Maps: item -> weight rows

struct MapRows {  // one tensor, row = row0 + item
    const int8_t* qs;
    const __half* d;
    int64_t K, row0;
    __device__ void get(int item, Rows<1>& r) const {
        const int64_t row = row0 + item;
        r.q[0] = qs + row * K;
        r.d[0] = d + row * (K >> 5);
        r.xsel[0] = 0;
        r.on[0] = true;
    }
};

struct MapConcat3 {  // Q|K|V: items split across three tensors with the same K
    const int8_t* qs[3];
    const __half* d[3];
    int n0, n1;
    int64_t K;
    __device__ void get(int item, Rows<1>& r) const {
        int t = 0, row = item;
        if (item >= n0 + n1) { t = 2; row = item - n0 - n1; }
        else if (item >= n0) { t = 1; row = item - n0; }
        r.q[0] = qs[t] + (int64_t)row * K;
        r.d[0] = d[t] + (int64_t)row * (K >> 5);
        r.xsel[0] = 0;
        r.on[0] = true;
    }
};

struct MapPair {  // gate row j, up row j
    const int8_t* qa; const __half* da;
    const int8_t* qb; const __half* db;
    int64_t K;
    __device__ void get(int item, Rows<2>& r) const {
        r.q[0] = qa + (int64_t)item * K; r.d[0] = da + (int64_t)item * (K >> 5);
        r.q[1] = qb + (int64_t)item * K; r.d[1] = db + (int64_t)item * (K >> 5);
        r.xsel[0] = r.xsel[1] = 0;
        r.on[0] = r.on[1] = true;
    }
};

struct MapStride3 {  // rows j, j+E, j+2E of one tensor (short-conv in_proj B, C, x)
    const int8_t* qs; const __half* d;
    int64_t K, stride;
    __device__ void get(int item, Rows<3>& r) const {
#pragma unroll
        for (int s = 0; s < 3; s++) {
            const int64_t row = item + s * stride;
            r.q[s] = qs + row * K;
            r.d[s] = d + row * (K >> 5);
            r.xsel[s] = 0;
            r.on[s] = true;
        }
    }
};

__device__ __forceinline__ bool masked(const uint32_t* mask, int e) {
    return mask && ((mask[e >> 5] >> (e & 31)) & 1u);
}

struct MapExpertPair {  // item = k*N + j: gate/up row j of expert idx[k]
    const int8_t* qa; const __half* da;
    const int8_t* qb; const __half* db;
    const int* idx; const uint32_t* mask;
    int64_t K; int N;
    __device__ void get(int item, Rows<2>& r) const {
        const int k = item / N, j = item - k * N;
        const int e = idx[k];
        const int64_t row = (int64_t)e * N + j;
        const bool on = !masked(mask, e);
        r.q[0] = qa + row * K; r.d[0] = da + row * (K >> 5);
        r.q[1] = qb + row * K; r.d[1] = db + row * (K >> 5);
        r.xsel[0] = r.xsel[1] = 0;
        r.on[0] = r.on[1] = on;
    }
};

template <int S>
struct MapExpertDown {  // item j: row j of expert idx[s] for every slot s < top_k, input h[s]
    const int8_t* qs; const __half* d;
    const int* idx; const uint32_t* mask;
    int64_t K; int N;
    int top_k = S;  // slots past top_k (a top_k below S) are off
    __device__ void get(int item, Rows<S>& r) const {
#pragma unroll
        for (int s = 0; s < S; s++) {
            const bool live = s < top_k;
            const int e = live ? idx[s] : 0;
            const int64_t row = (int64_t)e * N + item;
            r.q[s] = qs + row * K;
            r.d[s] = d + row * (K >> 5);
            r.xsel[s] = live ? s : 0;
            r.on[s] = live && !masked(mask, e);
        }
    }
};

// ---------------------------------------------------------------------------------------
// Epilogues (applied once per item; all lanes hold the reduced sums, lane 0 writes)

struct NoState {};

struct EpiStore {
    float* y;
    bool residual;
    using WarpState = NoState;
    __device__ void init(WarpState&) const {}
    template <int S>
    __device__ void apply(WarpState&, int item, const float (&acc)[S], const bool (&)[S]) const {
        if ((threadIdx.x & 31) == 0) y[item] = residual ? y[item] + acc[0] : acc[0];
    }
    __device__ void finish(WarpState&) const {}
};

__device__ __forceinline__ float silu_f(float g) { return g * (1.0f / (1.0f + expf(-g))); }

struct EpiSwiGLU {  // siluInPlace(gate); mulInPlace(gate, up)  (tensor.js:167-178)
    float* h;
    using WarpState = NoState;
    __device__ void init(WarpState&) const {}
    __device__ void apply(WarpState&, int item, const float (&acc)[2], const bool (&on)[2]) const {
        if ((threadIdx.x & 31) == 0 && on[0]) h[item] = silu_f(acc[0]) * acc[1];
    }
    __device__ void finish(WarpState&) const {}
};

struct EpiConv {  // lfm2-engine.js:294-321 for element j
    const float* kw;  // [E][3] F32 kernel, element (k, d) at d*3 + k
    float* state;     // [2][E] rolling state, lag 0 = oldest
    float* y;
    int E;
    using WarpState = NoState;
    __device__ void init(WarpState&) const {}
    __device__ void apply(WarpState&, int j, const float (&acc)[3], const bool (&)[3]) const {
        if ((threadIdx.x & 31) != 0) return;
        const float B = acc[0], C = acc[1], X = acc[2];
        const float bx = B * X;
        const float s0 = state[j], s1 = state[E + j];
        const float co = kw[j * 3 + 0] * s0 + kw[j * 3 + 1] * s1 + kw[j * 3 + 2] * bx;
        state[j] = s1;
        state[E + j] = bx;
        y[j] = C * co;
    }
    __device__ void finish(WarpState&) const {}
};

struct EpiArgmax {  // logits store + first-max argmax, reduced per CTA then one atomicMax
    float* logits;
    unsigned long long* best;
    const int* suppress;  // device id excluded from the argmax (< 0: none)
    struct WarpState { unsigned long long k; int skip; };
    __device__ void init(WarpState& s) const {
        s.k = 0ull;
        s.skip = suppress ? *suppress : -1;
    }
    __device__ void apply(WarpState& s, int item, const float (&acc)[1], const bool (&)[1]) const {
        if ((threadIdx.x & 31) == 0) {
            logits[item] = acc[0];
            if (item != s.skip) {
                const unsigned long long k = argmax_key(acc[0], item);
                if (k > s.k) s.k = k;
            }
        }
    }
    __device__ void finish(WarpState& s) const {
        __shared__ unsigned long long keys[kGemvWarps];
        if ((threadIdx.x & 31) == 0) keys[threadIdx.x >> 5] = s.k;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long m = 0ull;
            for (int w = 0; w < kGemvWarps; w++) m = keys[w] > m ? keys[w] : m;
            if (m) atomicMax(best, m);
        }
    }
};

template <int S>
struct EpiMoECombine {  // lfm2-engine.js:459-486: moe = sum_k w_k * down_k (slot order); hidden += moe
    const float* w;
    float* hidden;
    using WarpState = NoState;
    __device__ void init(WarpState&) const {}
    __device__ void apply(WarpState&, int j, const float (&acc)[S], const bool (&on)[S]) const {
        if ((threadIdx.x & 31) != 0) return;
        float moe = 0.f;
#pragma unroll
        for (int s = 0; s < S; s++)
            if (on[s]) moe += w[s] * acc[s];
        hidden[j] += moe;
    }
    __device__ void finish(WarpState&) const {}
};

// ---------------------------------------------------------------------------------------
// Launch helpers

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

constexpr size_t kMaxStageBytes = 160 * 1024;

template <int S, class Map, class Epi>
static void launch(const XStage& st, const Map& map, const Epi& epi, int n_items, cudaStream_t s) {
    QQ_CHECK(st.K % 32 == 0 && st.K > 0, -1, "GEMV inner dimension must be a positive multiple of 32");
    const size_t smem = (size_t)st.nvec * st.K * sizeof(float);
    QQ_CHECK(smem <= kMaxStageBytes, -4, "GEMV input vectors exceed the shared-memory staging limit");
    for (int v = 0; v < st.nvec; v++)
        QQ_CHECK(st.x[v] && ((uintptr_t)st.x[v] & 15u) == 0, -1, "GEMV input must be a 16-byte aligned device pointer");
    QQ_CHECK(((uintptr_t)st.norm_w & 15u) == 0, -1, "norm weight must be 16-byte aligned");
    static int per_sm = 0;  // the same on every B200
    auto kern = k_gemv<S, Map, Epi>;
    if (first_use_on_device(reinterpret_cast<const void*>(kern)))
        QQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxStageBytes));
    if (!per_sm) {
        QQ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGemvThreads, 48 * 1024));
        if (per_sm < 1) per_sm = 1;
    }
    const int want = (n_items + kGemvWarps - 1) / kGemvWarps;
    int grid = num_sms() * per_sm;
    if (grid > want) grid = want;
    if (grid < 1) grid = 1;
    kern<<<grid, kGemvThreads, smem, s>>>(st, map, epi, n_items);
    QQ_CUDA_TRY(cudaGetLastError());
}

static void check_q8(const DTensor& W) {
    QQ_CHECK(W.type == 8 && W.qs && W.d, -1, "weight must be a Q8_0 tensor");
}

static int g_stream_path = 1;
void set_stream_path(int on) { g_stream_path = on; }
int stream_path() { return g_stream_path; }

void launch_gemv_rows(const DTensor& W, int64_t row0, int64_t n, const XStage& st, float* y, bool residual,
                      cudaStream_t s) {
    check_q8(W);
    if (g_stream_path && launch2_rows(W, row0, n, st, y, residual, s)) return;
    QQ_CHECK(st.K == W.K, -1, "GEMV: input length does not match the weight's ne[0]");
    QQ_CHECK(row0 >= 0 && row0 + n <= W.rows, -1, "GEMV: row range outside the tensor");
    MapRows m{W.qs, W.d, W.K, row0};
    launch<1>(st, m, EpiStore{y, residual}, (int)n, s);
}

void launch_gemv_qkv(const DTensor& wq, const DTensor& wk, const DTensor& wv, const XStage& st, float* qkv,
                     cudaStream_t s) {
    check_q8(wq); check_q8(wk); check_q8(wv);
    QQ_CHECK(wq.K == st.K && wk.K == st.K && wv.K == st.K, -1, "QKV: inner dimensions differ");
    if (g_stream_path && launch2_qkv(wq, wk, wv, st, qkv, s)) return;
    MapConcat3 m;
    m.qs[0] = wq.qs; m.qs[1] = wk.qs; m.qs[2] = wv.qs;
    m.d[0] = wq.d; m.d[1] = wk.d; m.d[2] = wv.d;
    m.n0 = (int)wq.rows; m.n1 = (int)wk.rows; m.K = st.K;
    launch<1>(st, m, EpiStore{qkv, false}, (int)(wq.rows + wk.rows + wv.rows), s);
}

void launch_gemv_swiglu(const DTensor& gate, const DTensor& up, const XStage& st, float* h, cudaStream_t s) {
    check_q8(gate); check_q8(up);
    QQ_CHECK(gate.K == st.K && up.K == st.K && gate.rows == up.rows, -1, "SwiGLU: gate/up shapes differ");
    if (g_stream_path && launch2_swiglu(gate, up, st, h, s)) return;
    MapPair m{gate.qs, gate.d, up.qs, up.d, st.K};
    launch<2>(st, m, EpiSwiGLU{h}, (int)gate.rows, s);
}

void launch_gemv_conv(const DTensor& in_proj, const float* conv_w, float* state, const XStage& st, float* y,
                      cudaStream_t s) {
    check_q8(in_proj);
    QQ_CHECK(in_proj.rows % 3 == 0 && in_proj.K == st.K, -1, "short-conv in_proj must be [E, 3E]");
    const int E = (int)(in_proj.rows / 3);
    if (g_stream_path && launch2_conv(in_proj, conv_w, state, st, y, s)) return;
    MapStride3 m{in_proj.qs, in_proj.d, st.K, E};
    launch<3>(st, m, EpiConv{conv_w, state, y, E}, E, s);
}

void launch_gemv_logits_argmax(const DTensor& W, const XStage& st, float* logits, unsigned long long* best,
                               const int* suppress_dev, cudaStream_t s) {
    check_q8(W);
    QQ_CHECK(W.K == st.K, -1, "lm_head: inner dimension mismatch");
    if (g_stream_path && launch2_logits_argmax(W, st, logits, best, suppress_dev, s)) return;
    const int64_t n = W.ne[1];
    MapRows m{W.qs, W.d, W.K, 0};
    launch<1>(st, m, EpiArgmax{logits, best, suppress_dev}, (int)n, s);
}

void launch_moe_gateup(const DTensor& gate_exps, const DTensor& up_exps, const int* idx, const uint32_t* mask,
                       int top_k, const XStage& st, float* h, cudaStream_t s) {
    check_q8(gate_exps); check_q8(up_exps);
    const int N = (int)gate_exps.ne[1];
    if (g_stream_path && launch2_moe_gateup(gate_exps, up_exps, idx, mask, top_k, st, h, s)) return;
    MapExpertPair m{gate_exps.qs, gate_exps.d, up_exps.qs, up_exps.d, idx, mask, st.K, N};
    launch<2>(st, m, EpiSwiGLU{h}, top_k * N, s);
}

void launch_moe_down_combine(const DTensor& down_exps, const int* idx, const float* w, const uint32_t* mask,
                             int top_k, const float* h, float* hidden, cudaStream_t s) {
    check_q8(down_exps);
    QQ_CHECK(top_k >= 1 && top_k <= 8, -4, "MoE down-combine: top_k must be 1..8");
    if (top_k == 4 && g_stream_path && launch2_moe_down_combine(down_exps, idx, w, mask, top_k, h, hidden, s)) return;
    const int K = (int)down_exps.K, N = (int)down_exps.ne[1];
    XStage st;
    st.nvec = top_k;
    st.K = K;
    for (int k = 0; k < top_k; k++) st.x[k] = h + (size_t)k * K;
    if (top_k == 4) {
        MapExpertDown<4> m{down_exps.qs, down_exps.d, idx, mask, K, N};
        launch<4>(st, m, EpiMoECombine<4>{w, hidden}, N, s);
    } else {  // any other top_k (Qwen3-MoE routes 8): up to 8 slots, the unused ones off
        MapExpertDown<8> m{down_exps.qs, down_exps.d, idx, mask, K, N, top_k};
        launch<8>(st, m, EpiMoECombine<8>{w, hidden}, N, s);
    }
}

}  // namespace qq3
