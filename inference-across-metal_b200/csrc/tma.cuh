// TMA (cp.async.bulk.tensor) and mbarrier helpers for sm_100a.
//
// Every wait on an mbarrier is bounded: after kMbarSpinLimit polls it records
// an error code in a device flag and gives up, so a missing completion shows
// up as IAM_ETIMEOUT on the host instead of a hung GPU.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace iam {

constexpr uint32_t kMbarSpinLimit = 1u << 22;

// The poll budget of a wait that may give up: a kernel argument of 0 means
// the library default.
__device__ __forceinline__ uint32_t wait_limit(int arg) {
  return arg > 0 ? static_cast<uint32_t>(arg) : kMbarSpinLimit;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Returns false when the phase did not complete within the poll budget, or
// (when `abort` is given) once another thread of the CTA has raised *abort:
// after one wait gave up, the others end promptly instead of each spending
// its own budget.  Waits for copies or MMAs already in flight pass no abort
// flag -- those complete by themselves and must before the CTA exits.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase, const volatile int* abort = nullptr,
                                          uint32_t limit = kMbarSpinLimit) {
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(phase)
        : "memory");
    if (done) return true;
    if (abort && (i & 63) == 63 && *abort) return false;
  }
  return false;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Contiguous global -> shared bulk copy (no multicast) completing on `bar`;
// both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// As mbar_wait, but polls with relaxed semantics and orders the caller's later
// accesses after the barrier with a lightweight acquire fence.  Cheaper per
// poll (about 100 cycles instead of about 400), for threads whose issue rate
// matters (a tensor-core issuer).
__device__ __forceinline__ bool mbar_wait_light(uint32_t bar, uint32_t phase, const volatile int* abort = nullptr,
                                                uint32_t limit = kMbarSpinLimit) {
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.relaxed.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(phase)
        : "memory");
    if (done) {
      asm volatile("fence.acquire.sync_restrict::shared::cluster.cluster;" ::: "memory");
      return true;
    }
    if (abort && (i & 63) == 63 && *abort) return false;
  }
  return false;
}

// Non-blocking: has the phase of parity `phase` completed?
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(phase)
      : "memory");
  return done != 0;
}

// 2D tiled TMA load (no multicast) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Encodes a 2D row-major tensor map [rows, cols] of `esize`-byte elements
// (row pitch `pitch` elements, 0 = cols) with a [box_rows, box_cols] box.
// Elements outside [rows, cols] read as zero.  Returns IAM_OK or IAM_EINVAL /
// IAM_ECUDA.
int tma_encode_2d(CUtensorMap* map, const void* base, int esize, uint64_t rows, uint64_t cols, uint32_t box_rows,
                  uint32_t box_cols, bool swizzle128, uint64_t pitch = 0);

}  // namespace iam
