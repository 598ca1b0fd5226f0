// api_internal.h -- types and helpers shared by the C-ABI translation units of libqq3cuda.so.
#pragma once
#include <cstdlib>
#include <new>
#include <string>

#include "kernels.h"
#include "qq3.h"

namespace qq3 {
const char* last_error_cstr();
}  // namespace qq3

struct qq_ctx {
    int device = 0;
    cudaStream_t own = nullptr;
    cudaStream_t stream = nullptr;
    // scratch arena for op-level calls (grow-only)
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    // NCCL communicator of the multi-GPU paths (comm.cu; an ncclComm_t), or null
    void* comm = nullptr;
    int comm_rank = 0, comm_world = 1;
    int comm_timeout_ms = 120000;
};

struct qq_tensor {
    qq_ctx* ctx = nullptr;
    qq3::DTensor t;
};

namespace qq3api {

using qq3::DTensor;
using qq3::Error;

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) QQ_CUDA_TRY(cudaSetDevice(dev));
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

template <class F>
int guard(F&& f) {
    try {
        f();
        return QQ_OK;
    } catch (const Error& e) {
        qq3::set_error(e.msg);
        return e.code;
    } catch (const std::bad_alloc&) {
        qq3::set_error("host allocation failed");
        return QQ_ERR_OOM;
    } catch (const std::exception& e) {
        qq3::set_error(e.what());
        return QQ_ERR_INVALID;
    }
}

inline const DTensor* dt(const qq_tensor* t) { return t ? &t->t : nullptr; }

inline void need(bool cond, const std::string& msg) { QQ_CHECK(cond, QQ_ERR_INVALID, msg); }

inline void check_shape(const DTensor* t, int type, int64_t ne0, int64_t ne1, int64_t ne2, const char* what) {
    need(t != nullptr, std::string("missing tensor: ") + what);
    need(t->type == type, std::string("wrong ggml type for ") + what);
    need(t->ne[0] == ne0 && t->ne[1] == ne1 && t->ne[2] == ne2,
         std::string("wrong shape for ") + what + ": got [" + std::to_string(t->ne[0]) + ", " +
             std::to_string(t->ne[1]) + ", " + std::to_string(t->ne[2]) + "]");
}

}  // namespace qq3api
