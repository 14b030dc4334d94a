// Seeded synthetic tensors generated on the GPU.
//
// Element i of tensor `name` is a function of mix64(stream(seed, name) +
// (i + 1) * golden) only (splitmix64 finalizer), so any sub-block of a tensor
// (a tensor-parallel shard) is generated independently and identically.  The
// float paths use integer sums and correctly rounded fp32 multiplies/adds only,
// so the host restatement produces the same bits.
#include "synth.cuh"

namespace iam {

uint64_t synth_mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t synth_fnv1a(const char* s) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (; *s; ++s) {
    h ^= static_cast<unsigned char>(*s);
    h *= 0x100000001B3ull;
  }
  return h;
}

uint64_t synth_stream(uint64_t seed, const char* name) {
  return synth_mix64(seed * kGolden + synth_fnv1a(name) * 0xD1B54A32D192ED03ull);
}

namespace {

__device__ __forceinline__ uint64_t dmix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Irwin-Hall(4) of 16-bit fields, centred, scaled to unit variance
__device__ __forceinline__ float unit_normal(uint64_t h) {
  const uint32_t s = static_cast<uint32_t>(h & 0xFFFF) + static_cast<uint32_t>((h >> 16) & 0xFFFF) +
                     static_cast<uint32_t>((h >> 32) & 0xFFFF) + static_cast<uint32_t>((h >> 48) & 0xFFFF);
  const float c = static_cast<float>(static_cast<int>(s) - 131070);  // exact
  return __fmul_rn(c, __uint_as_float(0x37DDB3D7u));                  // * fp32(sqrt(3) / 65536)
}

__global__ void synth_kernel(SynthJob j) {
  const uint64_t n = static_cast<uint64_t>(j.rows) * j.width;
  for (uint64_t o = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; o < n;
       o += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t r = o / j.width, c = o % j.width;
    const uint64_t i = (j.row0 + r) * j.full_cols + j.col0 + c;  // index in the full tensor
    const uint64_t h = dmix64(j.stream + (i + 1) * kGolden);
    const uint64_t o_dst = r * (j.dst_ld ? j.dst_ld : j.width) + c;
    switch (j.kind) {
      case SYN_WORDS:
        static_cast<uint32_t*>(j.dst)[o_dst] = static_cast<uint32_t>(h);
        break;
      case SYN_TOKENS:
        static_cast<int32_t*>(j.dst)[o_dst] = static_cast<int32_t>(h % static_cast<uint64_t>(j.modulo));
        break;
      case SYN_NORMAL_F32:
        static_cast<float*>(j.dst)[o_dst] = __fmul_rn(unit_normal(h), j.p0);
        break;
      case SYN_UNIFORM_F32: {
        const float u = __fmul_rn(static_cast<float>(h >> 40), __uint_as_float(0x33800000u));  // * 2^-24
        static_cast<float*>(j.dst)[o_dst] = __fadd_rn(j.p0, __fmul_rn(u, j.p1));
        break;
      }
      default: {
        const float n0 = __fmul_rn(unit_normal(h), j.p0);
        float v;
        if (j.kind == SYN_NORMAL_BF16) v = n0;
        else if (j.kind == SYN_ONE_PLUS_NORMAL_BF16) v = __fadd_rn(1.0f, n0);
        else if (j.kind == SYN_ABSNORMAL_BF16) v = fabsf(n0);
        else v = -8.0f * bf2f(f2bf(fabsf(n0)));  // SYN_NEG8_ABSNORMAL_BF16: bias = -8 * scale
        static_cast<uint16_t*>(j.dst)[o_dst] = f2bf(v);
      }
    }
  }
}

}  // namespace

int synth_fill(const SynthJob& j, cudaStream_t st) {
  const uint64_t n = static_cast<uint64_t>(j.rows) * j.width;
  if (n == 0) return IAM_OK;
  const int grid = static_cast<int>(std::min<uint64_t>((n + 255) / 256, 148ull * 64));
  synth_kernel<<<grid, 256, 0, st>>>(j);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

}  // namespace iam
