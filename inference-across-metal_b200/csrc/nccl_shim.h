// NCCL entry points used by the tensor-parallel step, resolved at run time
// from libnccl.so.2 so that single-GPU use never loads NCCL.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace iam {
int nccl_unique_id(void* id128);
// Non-blocking set-up polled against `timeout_ms`: a rank that never joins
// ends in IAM_ETIMEOUT (the half-built communicator is aborted).
int nccl_init(void** comm, const void* id128, int rank, int world, int timeout_ms);
void nccl_destroy(void* comm);
// Aborts a communicator: its kernels in flight return, it is freed.
void nccl_abort(void* comm);
// IAM_OK, or the communicator's asynchronous error (a peer that failed).
int nccl_async_status(void* comm);
int nccl_allreduce_f32(void* comm, float* buf, size_t n, cudaStream_t st);
int nccl_allgather_u64(void* comm, const unsigned long long* send, unsigned long long* recv, size_t n_per_rank,
                       cudaStream_t st);
}  // namespace iam
