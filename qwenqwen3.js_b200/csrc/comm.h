// comm.h -- the context's NCCL communicator (comm.cu), for the multi-GPU exchanges.
#pragma once
#include "api_internal.h"

namespace qq3 {

// calls enqueue on stream s; a group's sends and receives progress together
void comm_group_start();
void comm_group_end(qq_ctx* c);
void comm_send(qq_ctx* c, const void* buf, size_t bytes, int peer, cudaStream_t s);
void comm_recv(qq_ctx* c, void* buf, size_t bytes, int peer, cudaStream_t s);
void comm_allreduce_sum_f32(qq_ctx* c, const float* in, float* out, size_t n, cudaStream_t s);
void comm_allgather(qq_ctx* c, const void* in, void* out, size_t bytes_per_rank, cudaStream_t s);
void comm_destroy(qq_ctx* c);

}  // namespace qq3
