// Error text for the C ABI: one slot per host thread (operator level).
#include <cstdio>
#include <string>

#include "common.cuh"

namespace iam {
namespace {
thread_local std::string g_err;
}

void set_error(const std::string& msg) { g_err = msg; }

int fail(int status, const std::string& msg) {
  g_err = msg;
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  g_err = std::string(what) + ": " + cudaGetErrorString(e);
  return e == cudaErrorMemoryAllocation ? IAM_ENOMEM : IAM_ECUDA;
}

}  // namespace iam

extern "C" const char* iam_last_error(void) { return iam::g_err.c_str(); }

extern "C" const char* iam_status_string(int s) {
  switch (s) {
    case IAM_OK: return "ok";
    case IAM_EINVAL: return "invalid argument";
    case IAM_ECUDA: return "CUDA error";
    case IAM_ENCCL: return "NCCL error";
    case IAM_ETIMEOUT: return "device wait timed out";
    case IAM_ENOMEM: return "out of device memory";
    case IAM_ESTATE: return "invalid engine state";
    default: return "unknown status";
  }
}

extern "C" int iam_version(void) { return 1; }
