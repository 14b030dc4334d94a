/* Multi-threaded C helpers for the CPU oracle: TEST INFRASTRUCTURE ONLY.
 *
 * The numpy oracle (oracle/iam_oracle.py, oracle/synth.py) is the statement
 * of the arithmetic; these helpers compute exactly the same bits, faster, so
 * that tests can run the oracle over the full 64-layer model (25.6 G
 * weights) in minutes instead of hours.  tests/test_oracle_fast.py checks
 * every helper against its numpy statement.  The product library never links
 * this file.
 *
 *  - ofast_stream / ofast_words / ofast_absnormal_bf16 / ofast_normal_bf16:
 *    the counter-based generator of oracle/synth.py (splitmix64 finalizer over
 *    (seed, tensor name, element index); "N(0, sigma)" as the Irwin-Hall sum of
 *    four 16-bit uniforms).
 *  - ofast_dequant: MLX affine dequant to bf16 values, bf16(q * scale + bias)
 *    computed in fp32 and rounded to nearest even (iam_oracle.dequant;
 *    reference nibble order full_forward.swift:123-132).
 *
 * Compile with -ffp-contract=off: every product and sum is rounded in fp32
 * exactly where numpy rounds it.
 */
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define GOLDEN 0x9E3779B97F4A7C15ull
#define KEYMUL 0xD1B54A32D192ED03ull

static inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static uint64_t fnv1a64(const char* name) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (const unsigned char* p = (const unsigned char*)name; *p; ++p) {
    h ^= *p;
    h *= 0x100000001B3ull;
  }
  return h;
}

uint64_t ofast_stream(uint64_t seed, const char* name) { return mix64(seed * GOLDEN + fnv1a64(name) * KEYMUL); }

/* element i (0-based, counting from `start`) hashes counter start + i + 1 */
static inline uint64_t hash_at(uint64_t stream, uint64_t idx) { return mix64(stream + (idx + 1) * GOLDEN); }

static inline float ih_normal(uint64_t h, float sigma) {
  const uint64_t m = 0xFFFF;
  const int64_t s = (int64_t)((h & m) + ((h >> 16) & m) + ((h >> 32) & m) + ((h >> 48) & m));
  const float c = (float)(s - 131070);
  uint32_t u = 0x37DDB3D7u; /* float32(sqrt(3) / 65536) */
  float scale;
  memcpy(&scale, &u, 4);
  const float n = c * scale; /* one fp32 rounding, then a second for sigma */
  return n * sigma;
}

static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u); /* NaN stays NaN */
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

void ofast_words(uint64_t stream, uint64_t start, int64_t n, uint32_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = (uint32_t)hash_at(stream, start + (uint64_t)i);
}

void ofast_normal_bf16(uint64_t stream, uint64_t start, int64_t n, float sigma, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(ih_normal(hash_at(stream, start + (uint64_t)i), sigma));
}

void ofast_absnormal_bf16(uint64_t stream, uint64_t start, int64_t n, float sigma, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    float v = ih_normal(hash_at(stream, start + (uint64_t)i), sigma);
    out[i] = f2bf(v < 0.f ? -v : v);
  }
}

/* bias = bf16(scale * -8) for every scale (exact: a power of two) */
void ofast_neg8(const uint16_t* s, int64_t n, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(bf2f(s[i]) * -8.0f);
}

/* rows x K bf16 weights as fp32 values from w [rows, K/8] (nibble i of word j =
 * column 8j + i, low nibble first), s and b [rows, K/64] bf16 */
void ofast_dequant(const uint32_t* w, const uint16_t* s, const uint16_t* b, int64_t rows, int K, float* out) {
  const int KW = K / 8, G = K / 64;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const uint32_t* wr = w + r * KW;
    float* o = out + r * (int64_t)K;
    for (int g = 0; g < G; ++g) {
      const float sc = bf2f(s[r * G + g]), bi = bf2f(b[r * G + g]);
      for (int j = 0; j < 8; ++j) {
        const uint32_t v = wr[g * 8 + j];
        for (int e = 0; e < 8; ++e) {
          const float p = (float)((v >> (4 * e)) & 15u) * sc;
          o[g * 64 + j * 8 + e] = bf2f(f2bf(p + bi));
        }
      }
    }
  }
}
