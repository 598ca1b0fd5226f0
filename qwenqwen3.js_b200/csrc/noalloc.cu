// noalloc.cu -- qq_moe_block_noalloc: the LFM2-MoE block without any device allocation.
//
// Some callers cannot let this library call cudaMalloc while they run a layer: a host that owns
// every byte of device memory through its own pool or budget (an embedding runtime such as a
// JS engine's addon, or a serving process that pre-plans its memory), or code that issues the
// block while it is recording its own stream work.  This entry point takes the same inputs and
// outputs as qq_moe_block, but its scratch (routing ids and weights, routing records, expert
// activations) lives in one file-scope device array of fixed size, created when the module is
// loaded on a device and held by every device that loads the library until the process exits.
//
// Limits: T <= QQ_NOALLOC_MAX_TOKENS token rows, expert FFN width <= QQ_NOALLOC_MAX_FF,
// top_k == 4, n_expert <= 32.  Larger requests are rejected with QQ_ERR_INVALID.
// The array is shared by every call on a device and keeps the last call's contents; nothing
// in it has to start at zero (each call writes the ids, weights, records and activations it
// reads).  Calls whose GPU work overlaps (different streams, or host threads without ordering)
// race on the array.
#include <mutex>

#include "api_internal.h"

using namespace qq3api;

namespace {

constexpr int kTopK = 4;
constexpr int kMaxExperts = 32;
constexpr size_t kIdxBytes = (size_t)QQ_NOALLOC_MAX_TOKENS * kTopK * sizeof(int);
constexpr size_t kWBytes = (size_t)QQ_NOALLOC_MAX_TOKENS * kTopK * sizeof(float);
constexpr size_t kRecBytes = (size_t)QQ_NOALLOC_MAX_TOKENS * (2 * kTopK + kMaxExperts) * sizeof(float);
constexpr size_t kHBytes = (size_t)kTopK * QQ_NOALLOC_MAX_FF * sizeof(float);
constexpr size_t kScratchBytes = kIdxBytes + kWBytes + kRecBytes + kHBytes;  // 256 KiB

}  // namespace

// The scratch itself.  In host code this name is only a stand-in for the symbol: the device
// address comes from cudaGetSymbolAddress (below), per device.
static __device__ __align__(256) unsigned char g_moe_noalloc_scratch[kScratchBytes];

namespace {

constexpr int kMaxDevices = 64;

// Device address of the scratch on `dev` (which must be current).  Resolved on the first call
// per device and cached; that first call should come before any stream capture.
unsigned char* scratch_on(int dev) {
    static std::mutex mu;
    static void* addr[kMaxDevices] = {nullptr};
    QQ_CHECK(dev >= 0 && dev < kMaxDevices, QQ_ERR_INVALID, "qq_moe_block_noalloc: device index too large");
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
        QQ_CHECK(e == cudaSuccess && p != nullptr, QQ_ERR_CUDA,
                 std::string("qq_moe_block_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
        addr[dev] = p;
    }
    return static_cast<unsigned char*>(addr[dev]);
}

}  // namespace

extern "C" int qq_moe_block_noalloc(qq_ctx* ctx, const qq_layer_desc* layer, int n_expert, int top_k,
                                    const float* x_dev, int T, float* out_dev, float* routing_dev) {
    return guard([&] {
        need(ctx && layer && x_dev && out_dev && T >= 0, "qq_moe_block_noalloc: bad argument");
        const DTensor* router = dt(layer->t[QQ_ROUTER]);
        const DTensor* gate = dt(layer->t[QQ_GATE_EXPS]);
        const DTensor* up = dt(layer->t[QQ_UP_EXPS]);
        const DTensor* down = dt(layer->t[QQ_DOWN_EXPS]);
        const DTensor* bias = dt(layer->t[QQ_EXP_BIAS]);
        need(router && gate && up && down, "qq_moe_block_noalloc: router and expert tensors are required");
        need(top_k == kTopK && n_expert >= kTopK && n_expert <= kMaxExperts,
             "qq_moe_block_noalloc: routes top-4 of at most 32 experts");
        const int64_t K = router->ne[0], F = gate->ne[1];
        check_shape(router, QQ_TYPE_Q8_0, K, n_expert, 1, "ffn_gate_inp.weight");
        check_shape(gate, QQ_TYPE_Q8_0, K, F, n_expert, "ffn_gate_exps.weight");
        check_shape(up, QQ_TYPE_Q8_0, K, F, n_expert, "ffn_up_exps.weight");
        check_shape(down, QQ_TYPE_Q8_0, F, K, n_expert, "ffn_down_exps.weight");
        if (bias) check_shape(bias, QQ_TYPE_F32, n_expert, 1, 1, "exp_probs_b.bias");
        need(T <= QQ_NOALLOC_MAX_TOKENS, "qq_moe_block_noalloc: T = " + std::to_string(T) + " exceeds the limit of " +
                                             std::to_string(QQ_NOALLOC_MAX_TOKENS) + " token rows");
        need(F <= QQ_NOALLOC_MAX_FF, "qq_moe_block_noalloc: expert FFN width " + std::to_string(F) +
                                         " exceeds the limit of " + std::to_string(QQ_NOALLOC_MAX_FF));
        if (T == 0) return;
        DeviceGuard dg(ctx->device);
        cudaStream_t s = ctx->stream;
        unsigned char* base = scratch_on(ctx->device);
        int* idx = reinterpret_cast<int*>(base);
        float* w = reinterpret_cast<float*>(base + kIdxBytes);
        float* rec = routing_dev ? routing_dev : reinterpret_cast<float*>(base + kIdxBytes + kWBytes);
        float* h = reinterpret_cast<float*>(base + kIdxBytes + kWBytes + kRecBytes);
        qq3::launch_lfm2_router(*router, bias ? bias->f32 : nullptr, x_dev, T, nullptr, 0.f, n_expert, top_k, rec, idx,
                                w, s);
        // the down-combine accumulates into the caller's output rows
        QQ_CUDA_TRY(cudaMemsetAsync(out_dev, 0, sizeof(float) * (size_t)T * K, s));
        for (int t = 0; t < T; t++) {
            qq3::XStage st;
            st.x[0] = x_dev + (size_t)t * K;
            st.K = (int)K;
            qq3::launch_moe_gateup(*gate, *up, idx + (size_t)t * top_k, nullptr, top_k, st, h, s);
            qq3::launch_moe_down_combine(*down, idx + (size_t)t * top_k, w + (size_t)t * top_k, nullptr, top_k, h,
                                         out_dev + (size_t)t * K, s);
        }
    });
}
