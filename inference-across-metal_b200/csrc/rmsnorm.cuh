// The reduction of rms_norm_bf16 (full_forward.swift:59-86) for one row, in
// the reference's summation order: the reference's thread i (of 256) sums
// x[i + 256 j]^2 in j order, then a shared-memory tree adds thread i + s into
// i for s = 128..1.  One warp plays all 256 threads: lane l owns virtual
// threads 8l..8l+7; tree levels s >= 8 are lane shuffles (xor 16..1),
// s = 4, 2, 1 are in-lane.
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

}  // namespace iam
