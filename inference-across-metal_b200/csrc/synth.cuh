// Seeded synthetic tensor generator (device) — see synth.cu.
#pragma once
#include <algorithm>

#include "common.cuh"

namespace iam {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

enum SynthKind : int {
  SYN_WORDS = 0,                 // uint32 of 8 uniform 4-bit codes
  SYN_NORMAL_BF16 = 1,           // bf16(N(0, p0))
  SYN_ABSNORMAL_BF16 = 2,        // bf16(|N(0, p0)|)            (scales)
  SYN_NEG8_ABSNORMAL_BF16 = 3,   // bf16(-8 * bf16(|N(0, p0)|)) (biases, scale stream)
  SYN_ONE_PLUS_NORMAL_BF16 = 4,  // bf16(1 + N(0, p0))          (norm weights)
  SYN_NORMAL_F32 = 5,            // N(0, p0)
  SYN_UNIFORM_F32 = 6,           // p0 + U[0,1) * p1
  SYN_TOKENS = 7,                // uniform integers mod `modulo`
};

// A sub-block [row0, row0+rows) x [col0, col0+width) of a [*, full_cols]
// tensor, written densely (row-major, `width` per row) to dst.
struct SynthJob {
  void* dst;
  uint64_t stream;
  int kind;
  float p0, p1;
  int64_t modulo;
  uint64_t full_cols;
  uint64_t row0, rows;
  uint64_t col0, width;
  uint64_t dst_ld;  // destination row stride in elements (0: width)
};

uint64_t synth_mix64(uint64_t z);
uint64_t synth_fnv1a(const char* s);
uint64_t synth_stream(uint64_t seed, const char* name);
int synth_fill(const SynthJob& j, cudaStream_t st);

}  // namespace iam
