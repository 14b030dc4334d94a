// Run-time binding of the NCCL calls of the tensor-parallel step.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "common.cuh"
#include "nccl_shim.h"

namespace iam {
namespace {

struct Nccl {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
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
    n.comm_init_rank_config =
        reinterpret_cast<decltype(n.comm_init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.comm_abort = reinterpret_cast<decltype(n.comm_abort)>(dlsym(h, "ncclCommAbort"));
    n.comm_get_async_error =
        reinterpret_cast<decltype(n.comm_get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.get_unique_id && n.comm_init_rank_config && n.comm_destroy && n.comm_abort && n.comm_get_async_error &&
           n.all_reduce && n.all_gather && n.error_string;
    if (!n.ok) n.why = "libnccl.so.2 lacks an expected symbol";
  });
  return n;
}

int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return IAM_OK;
  return fail(IAM_ENCCL, std::string(what) + ": " + lib().error_string(r));
}

// Polls a non-blocking communicator until its pending operation finished,
// failed, or the deadline passed.
int nccl_wait(ncclComm_t c, std::chrono::steady_clock::time_point deadline, const char* what) {
  Nccl& n = lib();
  for (;;) {
    ncclResult_t st = ncclInProgress;
    const ncclResult_t r = n.comm_get_async_error(c, &st);
    if (r != ncclSuccess) return nccl_status(r, "ncclCommGetAsyncError");
    if (st == ncclSuccess) return IAM_OK;
    if (st != ncclInProgress) return nccl_status(st, what);
    if (std::chrono::steady_clock::now() > deadline)
      return fail(IAM_ETIMEOUT, std::string(what) + ": not finished within the communicator timeout");
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

std::chrono::steady_clock::time_point after_ms(int ms) {
  return std::chrono::steady_clock::now() + std::chrono::milliseconds(ms);
}

// A non-blocking communicator may answer ncclInProgress while it enqueues;
// the host then polls until the enqueue finished (bounded like the set-up).
int nccl_enqueued(ncclResult_t r, void* comm, const char* what) {
  if (r == ncclInProgress) return nccl_wait(static_cast<ncclComm_t>(comm), after_ms(60000), what);
  return nccl_status(r, what);
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

int nccl_init(void** comm, const void* id128, int rank, int world, int timeout_ms) {
  Nccl& n = lib();
  *comm = nullptr;
  if (!n.ok) return fail(IAM_ENCCL, n.why);
  ncclUniqueId id;
  std::memcpy(&id, id128, sizeof(id));
  // non-blocking: the host polls the set-up against a deadline, so a rank
  // that never joins ends in an error (and an abort) instead of a hang
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t c = nullptr;
  const ncclResult_t r = n.comm_init_rank_config(&c, world, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (c) n.comm_abort(c);
    return nccl_status(r, "ncclCommInitRankConfig");
  }
  const int w = nccl_wait(c, after_ms(timeout_ms), "ncclCommInitRankConfig");
  if (w != IAM_OK) {
    n.comm_abort(c);
    return w;
  }
  *comm = c;
  return IAM_OK;
}

void nccl_destroy(void* comm) {
  if (comm && lib().ok) lib().comm_destroy(static_cast<ncclComm_t>(comm));
}

void nccl_abort(void* comm) {
  if (comm && lib().ok) lib().comm_abort(static_cast<ncclComm_t>(comm));
}

int nccl_async_status(void* comm) {
  Nccl& n = lib();
  if (!comm || !n.ok) return IAM_OK;
  ncclResult_t st = ncclSuccess;
  const ncclResult_t r = n.comm_get_async_error(static_cast<ncclComm_t>(comm), &st);
  if (r != ncclSuccess) return nccl_status(r, "ncclCommGetAsyncError");
  if (st == ncclSuccess || st == ncclInProgress) return IAM_OK;
  return nccl_status(st, "NCCL asynchronous error");
}

int nccl_allreduce_f32(void* comm, float* buf, size_t n, cudaStream_t st) {
  return nccl_enqueued(lib().all_reduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st), comm,
                       "ncclAllReduce");
}

int nccl_allgather_u64(void* comm, const unsigned long long* send, unsigned long long* recv, size_t n_per_rank,
                       cudaStream_t st) {
  return nccl_enqueued(lib().all_gather(send, recv, n_per_rank, ncclUint64, static_cast<ncclComm_t>(comm), st), comm,
                       "ncclAllGather");
}

}  // namespace iam
