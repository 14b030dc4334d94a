// W4A16 quantized matmul (MLX affine 4-bit, group 64) for decode / verify widths.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace iam {

// Epilogues fused into the matmul (full_forward.swift:88-110, 169-183).
enum QmmEpi : int {
  EPI_STORE = 0,   // out = bf16(y)
  EPI_RESID = 1,   // out = bf16(resid + bf16(y))            residual_add_bf16
  EPI_SWIGLU = 2,  // out = bf16(silu(bf16(gate)) * bf16(up)) silu_multiply_bf16
  EPI_ARGMAX = 3,  // per-CTA (max bf16(y), first index) keys  argmax_bf16 (partial)
  EPI_F32 = 4,     // out32 = y (fp32 partial sums, reduced across GPUs next)
};

struct QmmSeg {
  const unsigned char* packed;  // tile-packed weights (qmm_pack_*); used instead of w/s/b when set
  const uint32_t* w;   // [rows, K/8] MLX packing
  const uint16_t* s;   // [rows, K/64] bf16
  const uint16_t* b;   // [rows, K/64] bf16
  const uint32_t* w2;  // EPI_SWIGLU: the up matrix (w is gate)
  const uint16_t* s2;
  const uint16_t* b2;
  uint16_t* out;       // out[tok * ldo + col]
  const uint16_t* resid;
  unsigned long long* keys;  // EPI_ARGMAX: keys[cta * key_ld + tok], packed (value, index)
  float* out32;              // EPI_F32
  int ldo, ldr, key_ld;
  int rows;       // output columns of this segment (SWIGLU: features)
  int mode;
  int cta_begin;  // first blockIdx.x of this segment
  int col_base;   // EPI_ARGMAX: global column index of local column 0
};

constexpr int kQmmMaxSeg = 4;
constexpr int kQmmMaxPeers = 8;

struct QmmArgs {
  const uint16_t* x;  // x[tok * ldx + k], bf16
  int ldx;
  int M;  // tokens
  int K;  // reduction length, multiple of 64
  int nseg;
  int total_ctas;
  int chunk;      // 64-groups per staged x chunk
  int xrows;      // token rows of a staged x chunk
  int ws_blocks;  // row blocks (CTAs along x) of the split-K workspace
  float* ws;      // split-K partial sums (zero between launches)
  int* counters;  // split-K arrival counters (zero between launches)
  int* err;       // device error word (a bounded wait that gave up writes IAM_ETIMEOUT)
  // Poll budget of every wait that may give up (0: the library default).
  // Waits for copies or MMAs already in flight always get the full budget.
  int wait_limit;
  // Fault injection for tests: the producer issues no copies at all, so the
  // consumers' first wait is on a phase that nothing completes and must run
  // out (nothing is in flight when the CTA exits).
  int starve;
  // Row-parallel matmul across GPUs (packed weights, one EPI_F32 segment):
  // each tile's final fp32 values go to push[r] + tok * ldo + col for every
  // rank r (this GPU's own slot and the peers' receive slots, by plain stores
  // over NVLink), then one release add of 1 at system scope to push_ctr[r][tile]
  // tells rank r that this rank's tile of the pass has landed.  npush = 0: the
  // values go to out32.
  int npush;
  float* push[kQmmMaxPeers];
  int* push_ctr[kQmmMaxPeers];
  // RMSNorm fused ahead of the matmul (GEMV passes of at most
  // kGemvNormMaxM tokens): x holds the raw rows and the matmul's input is
  // bf16((x / rms) * norm_w) with rms over each whole row, computed in the
  // reference's summation order (rms_norm_bf16).  Null: x is the input.
  const uint16_t* norm_w;
  float norm_eps;
  QmmSeg seg[kQmmMaxSeg];
};
constexpr int kGemvNormMaxM = 2;

// Passes the packed-weight matmul makes over M tokens (64 tokens at most each).
inline int qmm_packed_passes(int M) { return (M + 63) / 64; }

// After a tile's values went out (all epilogue threads past a barrier): one
// thread orders them before the arrivals at system scope and adds the
// arrivals (cumulative through the barrier, so it publishes every thread's
// stores to the peers).
__device__ __forceinline__ void qmm_push_arrive(const QmmArgs& A, int tile) {
  __threadfence_system();
#pragma unroll
  for (int r = 0; r < kQmmMaxPeers; ++r) {
    if (r >= A.npush) break;
    asm volatile("red.release.sys.global.add.s32 [%0], 1;" ::"l"(A.push_ctr[r] + tile) : "memory");
  }
}

// Tile configuration chosen by the host for a given shape.
struct QmmConfig {
  int nt;     // n8 token tiles per pass (1, 2 or 4): tokens per pass = 8*nt
  int rt;     // 16-row tiles per CTA (one warp each)
  int ks;     // CTAs splitting K (partials summed in an fp32 workspace)
  int kp;     // weight groups in flight per warp
  int chunk;  // 64-groups per staged x chunk
  bool tma;   // weights through the TMA ring (else register loads)
};
// Split-K workspace needed by a plan: floats and counters.
size_t qmm_ws_floats(const QmmArgs& a, const QmmConfig& c);
size_t qmm_ws_counters(const QmmArgs& a, const QmmConfig& c);
constexpr int kQmmMaxSmem = 200 * 1024;

// Tensor maps of one segment for the TMA variant: packed codes [rows, K/2]
// uint8 (box 16 or 8 rows x 128 bytes, 128B swizzle), scales and biases
// [rows, K/64] uint16 (box 16 or 8 rows x 8 groups).  SwiGLU segments use
// 8-row boxes of the gate (w, s, b) and up (w2, s2, b2) matrices.
struct QmmTmaMaps {
  CUtensorMap w, s, b, w2, s2, b2;
};
struct QmmTmaArgs {
  QmmArgs a;
  QmmTmaMaps maps[kQmmMaxSeg];
};

// Rows of output handled by one CTA of a segment for a config.
inline int qmm_rows_per_cta(int mode, int rt) { return (mode == EPI_SWIGLU ? 8 : 16) * rt; }

// Fills cta_begin of each segment and total_ctas; picks the config.
QmmConfig qmm_plan(QmmArgs& a);
int qmm_launch(const QmmArgs& a, const QmmConfig& c, cudaStream_t st, bool pdl);

// ---- tile-packed weights for the tensor-core and GEMV kernels (qmm_tc.cu,
// qmm_gemv.cu)
//
// A matrix of `rows` x K becomes ceil(rows / 128) tiles (SwiGLU pairs: 64
// features a tile, gate rows 0-63 and up rows 64-127) of ceil(K / 256)
// blocks of kQpBlockBytes, tile-major:
//   block (t, kb) at (t * KB + kb) * kQpBlockBytes;
//   codes: row r at r * 128, its 32-k chunk c (4 words) at ((c ^ qp_swz(r)) * 16);
//     each word holds 8 consecutive k with nibble s = k 2s, nibble s+4 = k 2s+1
//     (so (w >> 4s) & 0x000F000F is the natural pair (k 2s, k 2s+1));
//   (scale, bias) of row r, group g (0..3) at kQpCodeBytes + r * 16 + g * 4
//     (scale in the low half);
// then one byte a tile: 1 when every scale of the tile is below 0.5 in
// magnitude, in which case the tile's scales are stored multiplied by 2^129
// (exact: a power of two, and the product stays below the bf16 maximum).
// Such tiles are converted with the code in bits 4-7 of each 16-bit half: as
// a bf16 bit pattern that is q * 2^-129 (subnormal for q < 8, the smallest
// normal binade for q >= 8 -- one linear scale across both), so one packed
// FMA, fma(q * 2^-129, s * 2^129, b) = bf16(q * s + b) with the product exact
// and one rounding -- the same bits as the general form in fewer instructions.
// Padding rows and k read as zero codes with zero scale and bias.
//
// The chunk swizzle qp_swz(r) is a bijection of r % 8 that keeps both readers
// free of shared-memory bank conflicts: the tensor-core kernel's 16-byte
// loads of one chunk by 8 consecutive rows, and the GEMV kernel's 8-byte
// loads of word pairs by 4 consecutive rows x 4 lanes.
__host__ __device__ __forceinline__ int qp_swz(int r) { return ((r & 3) << 1) | ((r >> 2) & 1); }

// The four code pairs of a packed word in bits 4-7 of each half (the fast
// conversion's operand): pair s = (k 2s, k 2s+1) in v[s].
__device__ __forceinline__ void qp_codes_hi(uint32_t w, uint32_t (&v)[4]) {
  v[0] = (w << 4) & 0x00F000F0u;
  v[1] = w & 0x00F000F0u;
  v[2] = (w >> 4) & 0x00F000F0u;
  v[3] = (w >> 8) & 0x00F000F0u;
}

constexpr int kQpRows = 128;
constexpr int kQpBlockK = 256;
constexpr int kQpCodeBytes = kQpRows * kQpBlockK / 2;   // 16384
constexpr int kQpBlockBytes = kQpCodeBytes + kQpRows * 16;  // 18432
inline int qp_kblocks(int K) { return (K + kQpBlockK - 1) / kQpBlockK; }
inline size_t qp_blocks_bytes(int tiles, int K) {
  return static_cast<size_t>(tiles) * qp_kblocks(K) * kQpBlockBytes;
}
inline size_t qp_bytes(int tiles, int K) { return qp_blocks_bytes(tiles, K) + (static_cast<size_t>(tiles) + 255) / 256 * 256; }
inline int qp_tiles(int rows, bool swiglu) { return (rows + (swiglu ? 63 : 127)) / (swiglu ? 64 : 128); }

// Packing, in three stream-ordered steps per packed matrix `dst` of `tiles`
// tiles: qmm_pack_begin sets every tile flag; qmm_pack_scan clears the flag
// of each tile holding a scale >= 0.5 in magnitude (or not finite) among
// the rows of one source; qmm_pack then writes the rows of one source.  A
// source's row r goes to tile r / per_tile, tile row row_off + r % per_tile
// (per_tile 128 with row_off 0, or 64 with row_off 0 / 64 for the gate / up
// half of SwiGLU pairs).  Scan every source of the matrix before packing any.
int qmm_pack_begin(unsigned char* dst, int tiles, int K, cudaStream_t st);
int qmm_pack_scan(const uint16_t* s, int rows, int K, unsigned char* dst, int tiles, int per_tile, cudaStream_t st);
int qmm_pack(const uint32_t* w, const uint16_t* s, const uint16_t* b, int rows, int K, unsigned char* dst,
             int tiles, int per_tile, int row_off, cudaStream_t st);

// Tensor-core matmul over packed segments (every segment has `packed`; M <= 64).
// A null a.ws selects the library's own split-K workspace.
int qmm_tc_run(QmmArgs a, cudaStream_t st, bool pdl, size_t ws_floats_cap, size_t ws_ctr_cap);
// Register-dequant matmul over packed segments for narrow passes (M <= 16):
// mma.sync on weights converted in registers, no tensor memory.
constexpr int kGemvMaxM = 16;
constexpr int kGemvDefaultMaxM = 8;
int qmm_gemv_run(QmmArgs a, cudaStream_t st, bool pdl, size_t ws_floats_cap, size_t ws_ctr_cap);
// Widest pass that qmm_run sends to the GEMV kernel (IAM_QMM_GEMV_MAX_M
// overrides: 0 sends every pass to the tensor-core kernel).
int qmm_gemv_max_m();
// The library's split-K workspace for operator-level calls (grown on demand,
// zeroed when grown): kind 0 for the mma.sync kernels (which keep it zero),
// kind 1 for the tensor-core kernel (which keeps only its counters zero).
int qmm_op_workspace(int kind, size_t floats, size_t ctrs, cudaStream_t st, float** ws, int** ctr);

// Order-preserving key: larger float -> larger key; ties -> smaller index wins.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | static_cast<unsigned long long>(0xffffffffu - idx);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) {
  return 0xffffffffu - static_cast<uint32_t>(k & 0xffffffffull);
}

}  // namespace iam
