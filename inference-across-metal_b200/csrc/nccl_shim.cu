// Run-time binding of the NCCL calls of the tensor-parallel step.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "nccl_shim.h"

namespace iam {
namespace {

struct Nccl {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

Nccl& lib() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      n.why = std::string("dlopen libnccl.so.2: ") + dlerror();
      return;
    }
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_reduce && n.all_gather && n.error_string;
    if (!n.ok) n.why = "libnccl.so.2 lacks an expected symbol";
  });
  return n;
}

int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return IAM_OK;
  return fail(IAM_ENCCL, std::string(what) + ": " + lib().error_string(r));
}

}  // namespace

int nccl_unique_id(void* id128) {
  Nccl& n = lib();
  if (!n.ok) return fail(IAM_ENCCL, n.why);
  ncclUniqueId id;
  const int r = nccl_status(n.get_unique_id(&id), "ncclGetUniqueId");
  if (r == IAM_OK) std::memcpy(id128, &id, sizeof(id));
  return r;
}

int nccl_init(void** comm, const void* id128, int rank, int world) {
  Nccl& n = lib();
  if (!n.ok) return fail(IAM_ENCCL, n.why);
  ncclUniqueId id;
  std::memcpy(&id, id128, sizeof(id));
  ncclComm_t c = nullptr;
  const int r = nccl_status(n.comm_init_rank(&c, world, id, rank), "ncclCommInitRank");
  *comm = c;
  return r;
}

void nccl_destroy(void* comm) {
  if (comm && lib().ok) lib().comm_destroy(static_cast<ncclComm_t>(comm));
}

int nccl_allreduce_f32(void* comm, float* buf, size_t n, cudaStream_t st) {
  return nccl_status(lib().all_reduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st),
                     "ncclAllReduce");
}

int nccl_allgather_u64(void* comm, const unsigned long long* send, unsigned long long* recv, size_t n_per_rank,
                       cudaStream_t st) {
  return nccl_status(lib().all_gather(send, recv, n_per_rank, ncclUint64, static_cast<ncclComm_t>(comm), st),
                     "ncclAllGather");
}

}  // namespace iam
