// The reduction of rms_norm_bf16 (full_forward.swift:59-86) for one row, in
// the reference's summation order: the reference's thread i (of 256) sums
// x[i + 256 j]^2 in j order, then a shared-memory tree adds thread i + s into
// i for s = 128..1.  One warp plays all 256 threads: lane l owns virtual
// threads 8l..8l+7; tree levels s >= 8 are lane shuffles (xor 16..1),
// s = 4, 2, 1 are in-lane.  Shared by the RMSNorm kernel and the matmul
// epilogue that normalises the residual stream it just wrote, so both give
// the same bits.
#pragma once
#include "common.cuh"

namespace iam {

// rms = sqrt(sum(x^2) / dim + eps) of a row of `dim` bf16 values (dim % 256
// == 0), read as 16-byte chunks through chunk(i) (i < dim / 8); every lane of
// the calling warp returns it.
template <typename Chunk>
__device__ __forceinline__ float rms_row_warp(Chunk chunk, int dim, float eps, int lane) {
  float p[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const int nj = dim / 256;
  for (int j = 0; j < nj; ++j) {
    const uint4 v = chunk(32 * j + lane);  // virtual threads 8 lane .. 8 lane + 7, element block j
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a0 = lo_bf(u[i]), a1 = hi_bf(u[i]);
      p[2 * i] += a0 * a0;
      p[2 * i + 1] += a1 * a1;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, p[i], o);
      if (lane < o) p[i] += other;  // lanes >= o only feed lower lanes
    }
  float rms = 0.f;
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] += p[i + 4];
    p[0] += p[2];
    p[1] += p[3];
    p[0] += p[1];
    rms = sqrtf(p[0] / static_cast<float>(dim) + eps);
  }
  return __shfl_sync(0xffffffffu, rms, 0);
}

// out = bf16((x / rms) * w) for the 8 values of one chunk.
__device__ __forceinline__ uint4 rms_apply8(uint4 v, uint4 ww, float rms) {
  const uint32_t xv[4] = {v.x, v.y, v.z, v.w}, wv[4] = {ww.x, ww.y, ww.z, ww.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    o[k] = pack_bf2((lo_bf(xv[k]) / rms) * lo_bf(wv[k]), (hi_bf(xv[k]) / rms) * hi_bf(wv[k]));
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ uint4 ld_cg_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// The rows of the residual stream written by every CTA of a matmul,
// normalised by the one CTA that saw the matmul's last tile arrive: rows
// m < rows of x (ldx, dim bf16 each; rows * dim * 2 bytes must fit in `stage`)
// -> out (ldo).  The CTA's `threads` threads (ids tid, bar_id a named barrier
// over exactly them) copy the rows into shared memory with asynchronous
// 16-byte copies (all in flight at once, read from L2: other CTAs wrote them,
// published by the acquire-release arrival count), each warp reduces its
// rows, then every thread writes normalised chunks.
__device__ __forceinline__ void rms_norm_rows_cta(const uint16_t* x, int ldx, const uint16_t* w, uint16_t* out,
                                                  int ldo, int rows, int dim, float eps, uint4* stage, float* rms_s,
                                                  int tid, int threads, int bar_id) {
  const int nv = dim / 8;
  for (int i = tid; i < rows * nv; i += threads) {
    const int m = i / nv, c = i - m * nv;
    cp_async16(stage + i, x + static_cast<size_t>(m) * ldx + 8 * c);
  }
  cp_async_wait_all();
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(threads) : "memory");
  const int warp = tid >> 5, lane = tid & 31, warps = threads >> 5;
  for (int m = warp; m < rows; m += warps) {
    const uint4* xr = stage + m * nv;
    const float r = rms_row_warp([&](int i) { return xr[i]; }, dim, eps, lane);
    if (lane == 0) rms_s[m] = r;
  }
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(threads) : "memory");
  for (int c = tid; c < nv; c += threads) {
    const uint4 ww = *reinterpret_cast<const uint4*>(w + 8 * c);
    for (int m = 0; m < rows; ++m)
      *reinterpret_cast<uint4*>(out + static_cast<size_t>(m) * ldo + 8 * c) = rms_apply8(stage[m * nv + c], ww, rms_s[m]);
  }
}

}  // namespace iam
