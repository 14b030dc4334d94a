// NCCL entry points used by the tensor-parallel step, resolved at run time
// from libnccl.so.2 so that single-GPU use never loads NCCL.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace iam {
int nccl_unique_id(void* id128);
int nccl_init(void** comm, const void* id128, int rank, int world);
void nccl_destroy(void* comm);
int nccl_allreduce_f32(void* comm, float* buf, size_t n, cudaStream_t st);
int nccl_allgather_u64(void* comm, const unsigned long long* send, unsigned long long* recv, size_t n_per_rank,
                       cudaStream_t st);
}  // namespace iam
