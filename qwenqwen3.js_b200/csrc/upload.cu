// upload.cu -- streaming weight upload: GGUF tensor bytes to the device through a pinned ring.
//
// gguf.js hands the engine one ArrayBuffer slice per tensor (GGUFReader.fromFile,
// gguf.js:350-374) and the WebGPU engine copies each raw (GPUDevice.uploadBuffer,
// webgpu.js:370-383).  qq_upload_tensor does the same one tensor at a time, synchronously.  The
// uploader here keeps every stage busy at once for a whole model:
//   host thread : copies the next chunk of the caller's bytes into a free pinned slot (several
//                 threads share a large chunk);
//   copy engine : DMAs the previous slot to the device (cudaMemcpyAsync on the uploader's own
//                 stream);
//   SMs         : split the Q8_0 blocks of the slot before that into the qs / d planes (F32
//                 tensors are DMA'd straight to their destination).
// A slot is reused once the event recorded after its last consumer fires.  Tensors created by
// an uploader may be used once qq_upload_finish has returned.
#include <algorithm>
#include <thread>
#include <vector>

#include "api_internal.h"

using namespace qq3api;

struct qq_uploader {
    qq_ctx* ctx = nullptr;
    cudaStream_t stream = nullptr;
    size_t slot_bytes = 0;
    std::vector<uint8_t*> pinned;
    std::vector<uint8_t*> draw;  // device raw staging of each slot
    std::vector<cudaEvent_t> done;
    size_t next = 0;
    size_t bytes = 0;            // bytes uploaded so far
};

namespace {

constexpr int kUploadSlots = 4;
// a slot holds whole Q8_0 blocks (34 B) and whole floats, 16-byte multiples: 272 = lcm(34, 16)
constexpr size_t kSlotQuantum = 272;

void release(qq_uploader* u) {
    if (u->stream) cudaStreamSynchronize(u->stream);
    for (auto e : u->done)
        if (e) cudaEventDestroy(e);
    for (auto p : u->pinned)
        if (p) cudaFreeHost(p);
    for (auto p : u->draw)
        if (p) cudaFree(p);
    if (u->stream) cudaStreamDestroy(u->stream);
    u->done.clear();
    u->pinned.clear();
    u->draw.clear();
    u->stream = nullptr;
}

// memcpy split over up to 8 host threads (the caller's bytes are pageable, often a file mapping)
void par_copy(uint8_t* dst, const uint8_t* src, size_t n) {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t min_piece = 4u << 20;
    const int P = (int)std::min<size_t>({(size_t)8, (size_t)hw, std::max<size_t>(1, n / min_piece)});
    if (P <= 1) {
        memcpy(dst, src, n);
        return;
    }
    std::vector<std::thread> th;
    const size_t piece = (n + P - 1) / P;
    for (int i = 1; i < P; i++) {
        const size_t a = std::min(n, i * piece), b = std::min(n, a + piece);
        if (a < b) th.emplace_back([=] { memcpy(dst + a, src + a, b - a); });
    }
    memcpy(dst, src, std::min(n, piece));
    for (auto& t : th) t.join();
}

}  // namespace

extern "C" int qq_upload_begin(qq_ctx* ctx, size_t staging_bytes, qq_uploader** out) {
    return guard([&] {
        need(ctx && out, "qq_upload_begin: NULL argument");
        if (staging_bytes == 0) staging_bytes = (size_t)128 << 20;
        DeviceGuard dg(ctx->device);
        qq_uploader* u = new qq_uploader;
        u->ctx = ctx;
        try {
            u->slot_bytes = std::max(kSlotQuantum, (staging_bytes / kUploadSlots) / kSlotQuantum * kSlotQuantum);
            QQ_CUDA_TRY(cudaStreamCreateWithFlags(&u->stream, cudaStreamNonBlocking));
            u->pinned.assign(kUploadSlots, nullptr);
            u->draw.assign(kUploadSlots, nullptr);
            u->done.assign(kUploadSlots, nullptr);
            for (int i = 0; i < kUploadSlots; i++) {
                QQ_CUDA_TRY(cudaMallocHost(&u->pinned[i], u->slot_bytes));
                QQ_CUDA_TRY(cudaMalloc(&u->draw[i], u->slot_bytes));
                QQ_CUDA_TRY(cudaEventCreateWithFlags(&u->done[i], cudaEventDisableTiming));
            }
        } catch (...) {
            release(u);
            delete u;
            throw;
        }
        *out = u;
    });
}

extern "C" int qq_upload_tensor_async(qq_uploader* u, const void* host, size_t nbytes, int ggml_type, const int64_t* ne,
                                      int n_dims, qq_tensor** out) {
    return guard([&] {
        need(u && u->stream && host && ne && out, "qq_upload_tensor_async: NULL argument or finished uploader");
        need(n_dims >= 1 && n_dims <= 4, "qq_upload_tensor_async: n_dims must be 1..4");
        QQ_CHECK(ggml_type == QQ_TYPE_F32 || ggml_type == QQ_TYPE_Q8_0 || qq3::kq_block_bytes(ggml_type) > 0,
                 QQ_ERR_UNSUPPORTED, "qq_upload_tensor_async: F32 (0), Q8_0 (8) and Q2_K..Q6_K (10..14) only");
        DTensor t;
        t.type = ggml_type;
        t.n_dims = n_dims;
        int64_t n = 1;
        for (int i = 0; i < n_dims; i++) {
            need(ne[i] >= 1, "qq_upload_tensor_async: every ne[i] must be >= 1");
            t.ne[i] = ne[i];
            n *= ne[i];
        }
        t.K = t.ne[0];
        t.rows = n / t.ne[0];
        t.device = u->ctx->device;
        DeviceGuard dg(u->ctx->device);
        size_t total;
        const int kbs = qq3::kq_block_bytes(ggml_type);
        if (kbs) {  // k-quant superblocks stay raw: DMA'd straight to their destination
            need(t.ne[0] % 256 == 0, "qq_upload_tensor_async: k-quant tensors need ne[0] % 256 == 0");
            total = (size_t)(n / 256) * kbs;
            need(nbytes >= total, "qq_upload_tensor_async: buffer shorter than the k-quant superblocks");
            QQ_CUDA_TRY(cudaMalloc(&t.qs, total + 256));
        } else if (ggml_type == QQ_TYPE_F32) {
            total = (size_t)n * 4;
            need(nbytes >= total, "qq_upload_tensor_async: buffer shorter than ne0*ne1*... floats");
            QQ_CUDA_TRY(cudaMalloc(&t.f32, total));
        } else {
            need(t.ne[0] % 32 == 0, "qq_upload_tensor_async: Q8_0 needs ne[0] % 32 == 0");
            total = (size_t)(n / 32) * 34;
            need(nbytes >= total, "qq_upload_tensor_async: buffer shorter than the Q8_0 block stream");
            // +256 bytes: the streamed GEMV rounds the last group's scale copy up to 16 bytes
            if (cudaMalloc(&t.qs, (size_t)n + 256) != cudaSuccess || cudaMalloc(&t.d, sizeof(__half) * (n / 32 + 128)) != cudaSuccess) {
                cudaGetLastError();
                if (t.qs) cudaFree(t.qs);
                throw Error{QQ_ERR_OOM, "qq_upload_tensor_async: device allocation failed"};
            }
        }
        const uint8_t* src = static_cast<const uint8_t*>(host);
        try {
            for (size_t off = 0; off < total; off += u->slot_bytes) {
                const size_t len = std::min(u->slot_bytes, total - off);
                const size_t slot = u->next++ % kUploadSlots;
                QQ_CUDA_TRY(cudaEventSynchronize(u->done[slot]));  // the slot's previous chunk is consumed
                par_copy(u->pinned[slot], src + off, len);
                if (ggml_type == QQ_TYPE_F32 || kbs) {
                    uint8_t* dst = kbs ? reinterpret_cast<uint8_t*>(t.qs) : reinterpret_cast<uint8_t*>(t.f32);
                    QQ_CUDA_TRY(cudaMemcpyAsync(dst + off, u->pinned[slot], len, cudaMemcpyHostToDevice, u->stream));
                } else {
                    QQ_CUDA_TRY(cudaMemcpyAsync(u->draw[slot], u->pinned[slot], len, cudaMemcpyHostToDevice, u->stream));
                    const int64_t b0 = (int64_t)(off / 34);
                    qq3::launch_repack_q8(u->draw[slot], (int64_t)(len / 34), t.qs + b0 * 32, t.d + b0, u->stream);
                }
                QQ_CUDA_TRY(cudaEventRecord(u->done[slot], u->stream));
            }
        } catch (...) {
            cudaStreamSynchronize(u->stream);
            if (t.f32) cudaFree(t.f32);
            if (t.qs) cudaFree(t.qs);
            if (t.d) cudaFree(t.d);
            throw;
        }
        u->bytes += total;
        qq_tensor* r = new qq_tensor;
        r->ctx = u->ctx;
        r->t = t;
        *out = r;
    });
}

extern "C" int qq_upload_finish(qq_uploader* u, size_t* bytes_out) {
    return guard([&] {
        need(u != nullptr, "qq_upload_finish: NULL uploader");
        DeviceGuard dg(u->ctx->device);
        const cudaError_t e = u->stream ? cudaStreamSynchronize(u->stream) : cudaSuccess;
        const size_t bytes = u->bytes;
        release(u);
        delete u;
        QQ_CHECK(e == cudaSuccess, QQ_ERR_CUDA, std::string("qq_upload_finish: ") + cudaGetErrorString(e));
        if (bytes_out) *bytes_out = bytes;
    });
}
