// Kernel launchers shared between the operator ABI and the engine.
#pragma once
#include <algorithm>

#include "common.cuh"
#include "qmm.cuh"

namespace iam {

constexpr int kMaxRowsFinalize = 256;

// Launch with an optional programmatic-dependent-launch attribute.
template <typename... KArgs, typename... Args>
int launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return cuda_status(e, "cudaLaunchKernelEx");
  return IAM_OK;
}

// a.ws == nullptr: use the library's split-K workspace; else a.ws/a.counters
// hold at least ws_floats_cap floats / ws_ctr_cap counters, all zero.
int qmm_run(QmmArgs a, cudaStream_t st, bool pdl, size_t ws_floats_cap = 0, size_t ws_ctr_cap = 0);

int launch_rms_norm(const uint16_t* x, int ldx, const uint16_t* w, uint16_t* out, int ldo, int rows, int dim,
                    float eps, cudaStream_t st, bool pdl);
int launch_embed_bf16(const uint16_t* table, const int32_t* tokens, uint16_t* out, int rows, int hidden, int vocab,
                      int* err, cudaStream_t st, bool pdl);
// keys[part * key_ld + row]: argmax_out[row] = index of the best key over parts;
// *accept = greedy accept length of `tokens` against argmax_out.
int launch_finalize(const unsigned long long* keys, int nparts, int key_ld, int M, const int32_t* tokens,
                    int32_t* argmax_out, int32_t* accept, cudaStream_t st, bool pdl);
// best[row] = the best key over parts (tensor-parallel partial of finalize)
int launch_best_keys(const unsigned long long* keys, int nparts, int key_ld, int M, unsigned long long* best,
                     cudaStream_t st, bool pdl);
// Several sequences of seq_rows rows each: per-row argmax (one CTA a row),
// then each sequence's accept length.
int launch_finalize_batch(const unsigned long long* keys, int nparts, int key_ld, int n_seq, int seq_rows,
                          const int32_t* tokens, int32_t* argmax_out, int32_t* accept, cudaStream_t st, bool pdl);
// Per-row best key over nparts partial keys, one CTA a row (multi-sequence TP).
int launch_best_rows(const unsigned long long* keys, int nparts, int key_ld, int M, unsigned long long* best,
                     cudaStream_t st, bool pdl);

// GatedDeltaNet fused step (gdn.cu)
struct GdnArgs {
  const uint16_t* in;  // [rows, ld_in]: q | k | v at 0 / key_dim / 2*key_dim; z, a, b at their columns
  int ld_in, z_col, a_col, b_col;
  const uint16_t* conv_w;   // [conv_dim, 4]
  const uint16_t* conv_in;  // [3, conv_dim]
  uint16_t* conv_out;       // [3, conv_dim]
  const float* A_log;
  const uint16_t* dt_bias;
  const uint16_t* norm_w;  // [dv]
  float* S;                // [n_v_heads, dv, dk]
  float* S_alt;            // optional second state buffer: the state is read from S and written
                           // here (the two swap when *parity_dev == 1); null = in place
  uint16_t* out;           // [rows, ld_out]
  int ld_out;
  int n_k_heads, n_v_heads;  // heads handled by this launch (shard-local)
  int key_dim, conv_dim;     // shard-local widths of the qkv block
  int rows;                  // tokens of one sequence
  float eps;
  // Several sequences in one launch (grid.y = n_seq; 0 or 1: one): sequence
  // q reads input rows [q * rows, (q + 1) * rows) of `in`, writes the same rows
  // of `out`, and its state, conv windows and parity word sit seq_S floats,
  // seq_conv elements and q ints past those of sequence 0.
  int n_seq;
  size_t seq_S, seq_conv;
  const int* parity_dev;  // optional: when *parity_dev == 1, conv_in/conv_out (and S/S_alt) swap roles;
                          // read before the grid-dependency wait, so only a kernel launched without
                          // programmatic overlap may have written it
};
int launch_gdn(const GdnArgs& a, cudaStream_t st, bool pdl);

// Attention (attn.cu)
struct AttnArgs {
  const uint16_t* qkv;  // [rows, ld_qkv]: per head [q | gate] x n_heads, then k, v
  int ld_qkv, k_col, v_col;
  const uint16_t* q_norm_w;
  const uint16_t* k_norm_w;
  uint16_t* k_cache;  // [max_ctx, n_kv_heads, head_dim]
  uint16_t* v_cache;
  uint16_t* q_buf;    // [rows, n_heads, head_dim] normed + roped queries
  float* part_o;      // [rows, n_heads, nchunk, head_dim] partial outputs
  float* part_ml;     // [rows, n_heads, nchunk, 2] (max, sum)
  uint16_t* out;      // [rows, ld_out] gated attention output
  int ld_out;
  int n_heads, n_kv_heads, head_dim, rotary_dim;
  const float* rope_cs;  // [max_ctx, rotary/2, 2] cos/sin
  int max_ctx;
  int rows;             // all rows of the launch
  int pos;              // position of row 0 (ignored when pos_dev is set)
  const int* pos_dev;   // device position (graph replay); one per sequence when n_seq > 1
  // Several sequences in one launch (0 or 1: one): rows [q * seq_rows,
  // (q + 1) * seq_rows) belong to sequence q, whose caches sit q * seq_kv
  // elements past k_cache / v_cache and whose position is pos_dev[q].
  int n_seq, seq_rows;
  size_t seq_kv;
  int chunk;            // context tokens per split
  int nsplit;           // context splits (partials per query head)
  float eps;
};
int gdn_init_attrs();
int attn_init_attrs();
int launch_attn_prep(const AttnArgs& a, cudaStream_t st, bool pdl);
int launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl);
int launch_attn_combine(const AttnArgs& a, cudaStream_t st, bool pdl);

}  // namespace iam
