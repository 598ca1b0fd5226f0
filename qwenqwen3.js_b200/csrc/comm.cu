// comm.cu -- the library's own NCCL communicator (one per context) for the multi-GPU paths.
//
// The reference has no multi-device code; the build adds expert parallelism for LFM2-MoE and
// tensor parallelism for dense Qwen3, one process per GPU.  Their exchanges (expert dispatch /
// combine, the row-parallel all-reduces) are enqueued by the library itself on the context's
// stream, next to the kernels that produce and consume them, so a layer needs no host round
// trip.  NCCL is opened at run time (dlopen): a process that already loaded it (PyTorch's
// torch.distributed) shares that copy, otherwise the system libnccl.so.2 is used.
//
// Initialisation uses a non-blocking communicator and polls it against a deadline, so a rank
// that never joins turns into an error (and an aborted communicator) instead of a hang; every
// later NCCL call is polled the same way.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "api_internal.h"
#include "comm.h"

using namespace qq3api;

namespace qq3 {

namespace {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    std::string err;
};

const NcclApi& api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy already in the process
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            a.err = std::string("libnccl.so.2 could not be loaded: ") + dlerror();
            return;
        }
        auto sym = [&](const char* n) {
            void* p = dlsym(h, n);
            if (!p && a.err.empty()) a.err = std::string("NCCL symbol missing: ") + n;
            return p;
        };
        a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(sym("ncclGetUniqueId"));
        a.CommInitRankConfig = reinterpret_cast<decltype(a.CommInitRankConfig)>(sym("ncclCommInitRankConfig"));
        a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(sym("ncclCommDestroy"));
        a.CommAbort = reinterpret_cast<decltype(a.CommAbort)>(sym("ncclCommAbort"));
        a.CommGetAsyncError = reinterpret_cast<decltype(a.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
        a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(sym("ncclGetErrorString"));
        a.GroupStart = reinterpret_cast<decltype(a.GroupStart)>(sym("ncclGroupStart"));
        a.GroupEnd = reinterpret_cast<decltype(a.GroupEnd)>(sym("ncclGroupEnd"));
        a.Send = reinterpret_cast<decltype(a.Send)>(sym("ncclSend"));
        a.Recv = reinterpret_cast<decltype(a.Recv)>(sym("ncclRecv"));
        a.AllReduce = reinterpret_cast<decltype(a.AllReduce)>(sym("ncclAllReduce"));
        a.AllGather = reinterpret_cast<decltype(a.AllGather)>(sym("ncclAllGather"));
    });
    QQ_CHECK(a.err.empty(), QQ_ERR_UNSUPPORTED, a.err);
    return a;
}

}  // namespace

ncclComm_t comm_of(qq_ctx* c) {
    QQ_CHECK(c && c->comm, QQ_ERR_INVALID, "this context has no communicator (qq_comm_init)");
    return static_cast<ncclComm_t>(c->comm);
}

// poll a non-blocking communicator until the last call has left the in-progress state
void settle(qq_ctx* c, ncclResult_t r, const char* what) {
    const NcclApi& a = api();
    ncclComm_t comm = comm_of(c);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(c->comm_timeout_ms);
    while (r == ncclInProgress) {
        if (std::chrono::steady_clock::now() > deadline) {
            a.CommAbort(comm);
            c->comm = nullptr;
            throw Error{QQ_ERR_CUDA, std::string(what) + ": timed out; communicator aborted"};
        }
        std::this_thread::yield();
        a.CommGetAsyncError(comm, &r);
    }
    if (r != ncclSuccess) {
        a.CommAbort(comm);
        c->comm = nullptr;
        throw Error{QQ_ERR_CUDA, std::string(what) + ": " + a.GetErrorString(r) + "; communicator aborted"};
    }
}

void comm_group_start() { api().GroupStart(); }

void comm_group_end(qq_ctx* c) { settle(c, api().GroupEnd(), "ncclGroupEnd"); }

void comm_send(qq_ctx* c, const void* buf, size_t bytes, int peer, cudaStream_t s) {
    const ncclResult_t r = api().Send(buf, bytes, ncclUint8, peer, comm_of(c), s);
    if (r != ncclSuccess && r != ncclInProgress) settle(c, r, "ncclSend");
}

void comm_recv(qq_ctx* c, void* buf, size_t bytes, int peer, cudaStream_t s) {
    const ncclResult_t r = api().Recv(buf, bytes, ncclUint8, peer, comm_of(c), s);
    if (r != ncclSuccess && r != ncclInProgress) settle(c, r, "ncclRecv");
}

void comm_allreduce_sum_f32(qq_ctx* c, const float* in, float* out, size_t n, cudaStream_t s) {
    settle(c, api().AllReduce(in, out, n, ncclFloat32, ncclSum, comm_of(c), s), "ncclAllReduce");
}

void comm_allgather(qq_ctx* c, const void* in, void* out, size_t bytes_per_rank, cudaStream_t s) {
    settle(c, api().AllGather(in, out, bytes_per_rank, ncclUint8, comm_of(c), s), "ncclAllGather");
}

void comm_destroy(qq_ctx* c) {
    if (!c || !c->comm) return;
    const NcclApi& a = api();
    ncclComm_t comm = static_cast<ncclComm_t>(c->comm);
    c->comm = nullptr;
    ncclResult_t r = ncclSuccess;
    a.CommGetAsyncError(comm, &r);
    if (r == ncclSuccess) a.CommDestroy(comm);
    else a.CommAbort(comm);
}

}  // namespace qq3

extern "C" int qq_comm_unique_id(void* id_out) {
    return guard([&] {
        need(id_out != nullptr, "qq_comm_unique_id: NULL argument");
        static_assert(sizeof(ncclUniqueId) == QQ_COMM_ID_BYTES, "NCCL unique id size");
        ncclUniqueId id;
        const ncclResult_t r = qq3::api().GetUniqueId(&id);
        QQ_CHECK(r == ncclSuccess, QQ_ERR_CUDA, std::string("ncclGetUniqueId: ") + qq3::api().GetErrorString(r));
        memcpy(id_out, &id, sizeof(id));
    });
}

extern "C" int qq_comm_init(qq_ctx* ctx, const void* id, int rank, int world, int timeout_ms) {
    return guard([&] {
        need(ctx && id, "qq_comm_init: NULL argument");
        need(world >= 1 && rank >= 0 && rank < world, "qq_comm_init: bad rank / world");
        need(ctx->comm == nullptr, "qq_comm_init: the context already has a communicator");
        const auto& a = qq3::api();
        DeviceGuard dg(ctx->device);
        ncclUniqueId uid;
        memcpy(&uid, id, sizeof(uid));
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;  // initialisation and every call are polled against a deadline
        ncclComm_t comm = nullptr;
        ctx->comm_timeout_ms = timeout_ms > 0 ? timeout_ms : 120000;
        ncclResult_t r = a.CommInitRankConfig(&comm, world, uid, rank, &cfg);
        ctx->comm = comm;
        ctx->comm_rank = rank;
        ctx->comm_world = world;
        if (!comm) throw qq3::Error{QQ_ERR_CUDA, std::string("ncclCommInitRankConfig: ") + a.GetErrorString(r)};
        if (r == ncclSuccess || r == ncclInProgress) {
            if (r == ncclInProgress) a.CommGetAsyncError(comm, &r);
            qq3::settle(ctx, r, "ncclCommInitRankConfig");
        } else {
            qq3::settle(ctx, r, "ncclCommInitRankConfig");
        }
    });
}

extern "C" int qq_comm_destroy(qq_ctx* ctx) {
    return guard([&] {
        need(ctx != nullptr, "qq_comm_destroy: NULL context");
        DeviceGuard dg(ctx->device);
        qq3::comm_destroy(ctx);
    });
}
