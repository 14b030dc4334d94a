/*
 * iam.h — C ABI of libiamcuda.so: the per-layer decode and K-token verify
 * forward of Qwen3.5-27B-shape hybrid models (GatedDeltaNet + full attention,
 * MLX affine 4-bit weights) on NVIDIA B200 (sm_100a).
 *
 * Plain C: pointers, sizes, int status codes; no C++ or CUDA types.  Streams
 * are passed as `void*` (a cudaStream_t, or NULL for the legacy default stream).
 * Every bf16 tensor is `uint16_t` bit patterns.  All device pointers must be
 * 16-byte aligned.
 *
 * Two levels, mirroring the reference (inference-across-metal):
 *  - operator level: one call per reference kernel, on caller-owned device
 *    buffers (the reference's Metal argument slots, full_forward.swift:55-445,
 *    711-728); the only device memory the library allocates at this level is
 *    its own split-K and attention scratch, grown on demand (see
 *    iam_qmm_affine4_noalloc for a variant that allocates nothing);
 *  - engine level: weights, recurrent state and KV cache owned by the library
 *    and resident in HBM, a whole token step captured as one CUDA graph
 *    (replaces forwardPass, full_forward.swift:1198-1308, and the M-row
 *    verify of batch_verify_27b.swift:141-274).
 */
#ifndef IAM_H_
#define IAM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (the reference only checks command-buffer status,
 *      full_forward.swift:1242-1245; here every call returns one) ---------- */
#define IAM_OK 0
#define IAM_EINVAL 1    /* bad shape, alignment or argument */
#define IAM_ECUDA 2     /* a CUDA runtime error */
#define IAM_ENCCL 3     /* an NCCL error */
#define IAM_ETIMEOUT 4  /* a bounded device-side wait gave up */
#define IAM_ENOMEM 5    /* device memory exhausted */
#define IAM_ESTATE 6    /* call not valid in the engine's current state */

/* Text of the last error on this host thread (operator level) or engine. */
const char* iam_last_error(void);
const char* iam_status_string(int status);
int iam_version(void);

/* ======================================================================
 * Operator level.  y/out are written; nothing else is modified unless
 * stated.  `rows` is the number of tokens (verify width) processed.
 * ====================================================================== */

/* MLX affine 4-bit quantized matmul, group size 64, transpose=True:
 *   y[m, n] = bf16( sum_k x[m, k] * bf16(q[n,k] * s[n,k/64] + b[n,k/64]) )
 * w: uint32 [N, K/8], nibble i of word j = column 8j+i (low nibble first);
 * s, b: bf16 [N, K/64]; x: bf16 [M, K]; y: bf16 [M, N].
 * Requires K % 64 == 0, N % 8 == 0, 1 <= M.
 * Split-K scratch: one library workspace per (device, stream), grown on
 * demand; calls on one stream are ordered, calls on different streams never
 * share a workspace.  The same holds for iam_qmm_affine4_packed.
 * Replaces dispatchQMatmul (full_forward.swift:711-728) / encodeQMM
 * (batch_verify_27b.swift:100-119), which bind MLX's
 * affine_qmm_t_nax_bfloat16_t_gs_64_b_4 kernel with args (w,s,b,x,y,K,N,M). */
int iam_qmm_affine4(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x,
                    uint16_t* y, int M, int N, int K, int group_size, void* stream);

/* iam_qmm_affine4 for callers that cannot allocate device memory while they
 * run it (they manage all device memory themselves, or run inside a section
 * where an allocation would synchronise the device).  No counterpart in the
 * reference.  Same arguments, kernel and results; the split-K scratch is a
 * fixed array inside the library (1 Mi floats, 16 Ki counters) instead of a
 * workspace grown on demand, and a shape whose plan needs more is rejected
 * with IAM_EINVAL (iam_qmm_affine4_plan tells a caller in advance).  Every
 * call looks the scratch's device address up (cudaGetSymbolAddress); the
 * first call on a device also clears it with cudaMemsetAsync on the call's
 * stream, so make that first call outside any stream capture.  The scratch is
 * shared by all calls on a device: calls must not overlap (one stream, or
 * ordered), and a call that failed part-way may leave it dirty. */
int iam_qmm_affine4_noalloc(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x,
                            uint16_t* y, int M, int N, int K, int group_size, void* stream);

/* The plan iam_qmm_affine4 and iam_qmm_affine4_noalloc run for an [M, K] x
 * [N, K]^T shape on the current device: the largest number of CTAs that
 * split K in one pass (1: no split-K scratch is used), and the split-K
 * scratch it needs (floats, counters; 0 when nothing is split).  No
 * counterpart in the reference. */
int iam_qmm_affine4_plan(int M, int N, int K, int* splits, size_t* scratch_floats, size_t* scratch_counters);

/* The same matmul on the tensor cores (tcgen05, bf16 weights dequantized into
 * tensor memory) over weights re-packed once into 128-row x 256-k blocks.
 * No counterpart in the reference, whose qmm reads the MLX layout on every
 * call; these three replace the same dispatchQMatmul / encodeQMM call when
 * the caller can keep a packed copy.  The engine packs its own weights.
 *   iam_qmm_packed_bytes: size of the packed form of an [N, K] matrix (0 for
 *     invalid sizes);
 *   iam_qmm_pack_affine4: w, s, b as for iam_qmm_affine4 -> packed (device
 *     memory of that size, 16-byte aligned), stream-ordered;
 *   iam_qmm_affine4_packed: y = x . W^T, any M >= 1 (passes of 64 tokens). */
size_t iam_qmm_packed_bytes(int N, int K);
int iam_qmm_pack_affine4(const uint32_t* w, const uint16_t* s, const uint16_t* b, void* packed, int N, int K,
                         void* stream);
int iam_qmm_affine4_packed(const void* packed, const uint16_t* x, uint16_t* y, int M, int N, int K,
                           void* stream);

/* iam_qmm_affine4_packed run synchronously with its device-side waits
 * checked: every wait inside the kernel that may give up polls at most
 * `wait_limit` times (0: the library default, about a second), and a wait
 * that gave up makes the call return IAM_ETIMEOUT after the kernel has
 * drained its copies and exited (the context stays usable; y is then not
 * written).  `starve` != 0 is fault injection for tests: the kernel issues
 * none of its copies, so its first wait is on a phase that nothing completes.
 * No counterpart in the reference, whose only check is the command-buffer
 * status after waitUntilCompleted (full_forward.swift:1242-1245). */
int iam_qmm_affine4_packed_checked(const void* packed, const uint16_t* x, uint16_t* y, int M, int N, int K,
                                   int wait_limit, int starve, void* stream);

/* rms_norm_bf16 (full_forward.swift:59-86), applied to each of `rows` rows. */
int iam_rms_norm_bf16(const uint16_t* x, const uint16_t* weight, uint16_t* out, int rows, int dim,
                      float eps, void* stream);

/* silu_multiply_bf16 (full_forward.swift:88-99): out = bf16(silu(gate) * up). */
int iam_silu_multiply_bf16(const uint16_t* gate, const uint16_t* up, uint16_t* out, int count,
                           void* stream);

/* residual_add_bf16 (full_forward.swift:101-110): out = bf16(a + b). */
int iam_residual_add_bf16(const uint16_t* a, const uint16_t* b, uint16_t* out, int count, void* stream);

/* embed_lookup_bf16 (full_forward.swift:112-133): dequantize rows of a 4-bit
 * table for `rows` token ids (device int32).  out: bf16 [rows, hidden]. */
int iam_embed_lookup_q4(const uint32_t* w, const uint16_t* s, const uint16_t* b, const int32_t* tokens,
                        uint16_t* out, int rows, int hidden, int group_size, void* stream);

/* The same lookup on a bf16 table [vocab, hidden] (the benchmark's table). */
int iam_embed_lookup_bf16(const uint16_t* table, const int32_t* tokens, uint16_t* out, int rows,
                          int hidden, int vocab, void* stream);

/* sigmoid_gate_bf16 = sigmoid_multiply_bf16 (full_forward.swift:135-146):
 * out = bf16(a * sigmoid(gate)). */
int iam_sigmoid_gate_bf16(const uint16_t* a, const uint16_t* gate, uint16_t* out, int count, void* stream);

/* rope_bf16 + precomputeRoPE (full_forward.swift:148-167, 734-743): rotate
 * adjacent pairs (2i, 2i+1), i < rotary_dim/2, of every head of x in place;
 * x: bf16 [rows, num_heads, head_dim]; row r is at position pos + r. */
int iam_rope_bf16(uint16_t* x, int rows, int num_heads, int head_dim, int rotary_dim, float theta, int pos,
                  void* stream);

/* argmax_bf16 (full_forward.swift:169-183): first index of the maximum of
 * each of `rows` rows of length `count`; out: int32 [rows]. */
int iam_argmax_bf16(const uint16_t* x, int32_t* out, int rows, int count, void* stream);

/* per_head_rms_norm_bf16 (full_forward.swift:185-207) on [rows*num_heads, head_dim]. */
int iam_per_head_rms_norm_bf16(const uint16_t* x, const uint16_t* weight, uint16_t* out, int rows,
                               int num_heads, int head_dim, float eps, void* stream);

/* depthwise_conv1d_step = depthwise_conv1d_m1_bf16 (full_forward.swift:240-263)
 * over `rows` consecutive tokens: state_in bf16 [3, channels] (the last three
 * inputs), x bf16 [rows, channels], w bf16 [channels, 4] -> out bf16
 * [rows, channels] (no bias, not activated), state_out bf16 [3, channels].
 * state_out must not alias state_in (the reference double-buffers it,
 * full_forward.swift:657-658). */
int iam_depthwise_conv1d_step(const uint16_t* state_in, const uint16_t* x, const uint16_t* w, uint16_t* out,
                              uint16_t* state_out, int channels, int rows, void* stream);

/* compute_g_beta_bf16 (full_forward.swift:299-319) for `rows` tokens:
 * a, b bf16 [rows, n_v_heads]; A_log fp32 [n_v_heads]; dt_bias bf16 [n_v_heads]
 * -> g, beta bf16 [rows, n_v_heads]. */
int iam_compute_g_beta(const uint16_t* a, const uint16_t* b, const float* A_log, const uint16_t* dt_bias,
                       uint16_t* g, uint16_t* beta, int rows, int n_v_heads, void* stream);

/* gated_delta_step = gated_delta_step_bf16 (full_forward.swift:321-355) with
 * the K-head expansion of expand_kv_heads_bf16 (209-222) folded in, for
 * `rows` sequential tokens: q, k bf16 [rows, n_k_heads, dk] (already
 * normalised), v bf16 [rows, n_v_heads, dv], g, beta bf16 [rows, n_v_heads],
 * S fp32 [n_v_heads, dv, dk] updated in place, y bf16 [rows, n_v_heads, dv].
 * V-head h reads K-head h / (n_v_heads / n_k_heads).  Requires dk == dv == 128. */
int iam_gated_delta_step(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* g,
                         const uint16_t* beta, float* S, uint16_t* y, int n_v_heads, int n_k_heads, int dk,
                         int dv, int rows, void* stream);

/* rms_norm_gated_bf16 (full_forward.swift:357-381): per head of dim
 * head_dim: out = bf16(silu(z) * (y / rms(y)) * w); y, z, out bf16
 * [rows, num_heads, head_dim]; w bf16 [head_dim]. */
int iam_rms_norm_gated_bf16(const uint16_t* y, const uint16_t* z, const uint16_t* w, uint16_t* out, int rows,
                            int num_heads, int head_dim, float eps, void* stream);

/* The fused GatedDeltaNet step of one layer for `rows` sequential tokens
 * (full_forward.swift:1025-1123 in one kernel): conv1d step + SiLU + q/k
 * scaled norms + g/beta + gated delta rule + gated RMSNorm.
 * qkv bf16 [rows, ld_in] with q at column 0, k at key_dim, v at 2*key_dim;
 * z/a/b bf16 [rows, ld_in] at the given column offsets; conv_w bf16
 * [conv_dim, 4]; conv_in/conv_out bf16 [3, conv_dim] (must differ); A_log
 * fp32, dt_bias bf16 [n_v_heads]; norm_w bf16 [dv]; S fp32
 * [n_v_heads, dv, dk] in place; out bf16 [rows, ld_out] (n_v_heads*dv cols). */
int iam_gdn_step_fused(const uint16_t* qkvzab, int ld_in, int z_col, int a_col, int b_col,
                       const uint16_t* conv_w, const uint16_t* conv_in, uint16_t* conv_out, const float* A_log,
                       const uint16_t* dt_bias, const uint16_t* norm_w, float* S, uint16_t* out, int ld_out,
                       int n_k_heads, int n_v_heads, int rows, float eps, void* stream);

/* GQA SDPA decode with KV-cache append: copy_bf16 x2 + sdpa_decode_bf16
 * (full_forward.swift:384-444, dispatched 909-938), for `rows` tokens at
 * positions pos..pos+rows-1, causal within the block.  q bf16
 * [rows, n_q_heads, head_dim] (normed + roped); k_new (normed + roped) and
 * v_new bf16 [rows, n_kv_heads, head_dim] are appended to k_cache / v_cache
 * bf16 [max_ctx, n_kv_heads, head_dim] at pos..; out bf16
 * [rows, n_q_heads, head_dim].  No 1024-token cap (the reference's limit,
 * full_forward.swift:415); requires pos + rows <= max_ctx. */
int iam_sdpa_decode_append(const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new, uint16_t* k_cache,
                           uint16_t* v_cache, uint16_t* out, int rows, int pos, int n_q_heads, int n_kv_heads,
                           int head_dim, int max_ctx, void* stream);

/* ======================================================================
 * Engine level
 * ====================================================================== */

typedef struct iam_dims {
  int hidden;            /* 5120 */
  int intermediate;      /* 17408 */
  int vocab;             /* 248320 */
  int n_layers;          /* 64; layer i is attention iff (i+1) % full_attn_interval == 0 */
  int full_attn_interval;/* 4 */
  int n_heads;           /* 24 query heads */
  int n_kv_heads;        /* 4 */
  int head_dim;          /* 256 */
  int rotary_dim;        /* 64 */
  float rope_theta;      /* 1e7 */
  int gdn_k_heads;       /* 16 */
  int gdn_v_heads;       /* 48 */
  int gdn_dk;            /* 128 */
  int gdn_dv;            /* 128 */
  int conv_kernel;       /* 4 */
  int group_size;        /* 64 */
  float eps;             /* 1e-6 */
  int max_ctx;           /* KV-cache capacity in tokens */
  int max_rows;          /* largest verify width (tokens per step, all sequences) */
  int max_seqs;          /* sequence slots for iam_verify_batch (1: one sequence) */
  int comm_timeout_ms;   /* world > 1: bound on the communicator set-up and on each synchronous
                            step's wait for its collectives (0: 120000); past it the communicator
                            is aborted and the call returns IAM_ETIMEOUT */
  long long resident_weight_bytes; /* HBM budget for the layers' 4-bit matrices, as loaded plus
                            tile-packed (0: all resident).  Layers are kept resident in order
                            while they fit; the 4-bit matrices of the rest live in pinned host
                            memory and each step copies them, one layer ahead of its use, into
                            two device slots on a second stream (the role of prefetchLayer,
                            warm_forward.swift:556-650).  Outputs are bit-identical. */
} iam_dims;

/* Qwen3.5-27B defaults (full_forward.swift:18-49). */
void iam_dims_qwen35_27b(iam_dims* d);

/* The tensor-parallel shard that rank `rank` of `world` holds; host only, no
 * GPU needed.  No counterpart in the reference (it runs on one device); the
 * engine builds its tensor list from exactly this plan.  Each pair is
 * [first, first + count) in the unsharded numbering:
 *   GDN        V heads split evenly; the K heads they read follow them;
 *   attention  query heads split evenly; KV heads split up to n_kv_heads
 *              ways and are replicated beyond (rank r then holds KV head
 *              r / (world / n_kv_heads));
 *   MLP        intermediate columns (gate/up rows, down_proj input features);
 *   lm_head    vocab rows.
 * out_proj, o_proj and down_proj take the input-feature slice that matches
 * and their fp32 partial products are summed over the ranks.  Returns
 * IAM_EINVAL when the dims do not split over `world`. */
typedef struct iam_tp_shard {
  int gdn_k_head0, gdn_k_heads;
  int gdn_v_head0, gdn_v_heads;
  int q_head0, q_heads;
  int kv_head0, kv_heads;
  int inter0, inter;
  int vocab0, vocab;
} iam_tp_shard;
int iam_tp_shard_of(const iam_dims* dims, int rank, int world, iam_tp_shard* out);

typedef struct iam_engine iam_engine;

/* Create an engine on `device` (one process per GPU).  For tensor
 * parallelism over `world` GPUs, rank r passes the same 128-byte NCCL unique
 * id obtained by rank 0 from iam_nccl_unique_id(); world == 1 uses no NCCL. */
int iam_create(const iam_dims* dims, int device, int rank, int world, const void* nccl_id, iam_engine** out);
int iam_nccl_unique_id(void* id128);
void iam_destroy(iam_engine* e);
const char* iam_engine_error(const iam_engine* e);

/* Copy one tensor from host memory, by the reference's tensor name
 * (full_forward.swift:756-820), e.g. "model.layers.3.self_attn.q_proj.weight",
 * "model.layers.0.linear_attn.A_log", "model.embed_tokens.weight", "lm_head.scales".
 * `bytes` must equal the full (unsharded) tensor size; each rank keeps its shard. */
int iam_load_tensor(iam_engine* e, const char* name, const void* host_ptr, size_t bytes);

/* Load every weight from the safetensors files of an MLX 4-bit checkpoint
 * (its shards, in any order).  Replaces the reference's weight index + mmap +
 * loadTensorToBuffer (full_forward.swift:451-472, 555-595), the per-layer
 * tensor names (:749-822) and the lm_head load (:1279-1283).  Files are
 * memory-mapped; each rank copies its shard through pinned staging buffers.
 * Names may carry the "language_model." prefixes of multimodal exports;
 * non-decoder tensors are ignored.  A 4-bit embedding (weight U32, scales
 * and biases BF16) is dequantized once into the bf16 table with the
 * reference's embed_lookup_bf16 arithmetic (:112-133); without lm_head.* the
 * 4-bit embedding also serves as lm_head (tied).  Every engine tensor must be
 * present with its dtype and size (A_log may be BF16), and no decoder tensor
 * may be left over; otherwise IAM_EINVAL names the mismatches and nothing is
 * loaded. */
int iam_load_safetensors(iam_engine* e, const char* const* paths, int n_paths);

/* The same matching without a GPU: checks that the files hold exactly the
 * model `dims` describes and writes a summary (tensor count, bytes,
 * embedding and lm_head forms, then one line per problem) into report. */
int iam_check_safetensors(const iam_dims* dims, const char* const* paths, int n_paths, char* report,
                          size_t report_len);

/* Fill every weight with the seeded synthetic distributions of the benchmark
 * (generated on the GPU; bit-identical to oracle/synth.py). */
int iam_init_synthetic(iam_engine* e, uint64_t seed);

/* Seeded recurrent state: conv state N(0,1), S N(0,0.01) and `ctx` prior KV
 * tokens N(0,1) in every sequence slot (each slot its own streams); or zero
 * state (the reference's resetAllState) when seed == 0 and ctx == 0. */
int iam_state_init(iam_engine* e, uint64_t seed, int ctx);
int iam_state_reset(iam_engine* e);

/* The K-token verify step (K = 1 is a decode step): tokens[0] is the token
 * being decoded at position pos, tokens[1..K-1] are draft tokens.  Writes
 * argmax_out[K] (the greedy prediction after each position) and *accept_len,
 * the largest j with tokens[i+1] == argmax_out[i] for all i < j.  State,
 * conv window and KV cache advance by all K tokens. */
int iam_verify(iam_engine* e, const int32_t* tokens, int K, int pos, int32_t* argmax_out, int* accept_len);
int iam_decode_step(iam_engine* e, int32_t token, int pos, int32_t* next_token);

/* Speculative-decode rollback: keep the recurrent state after the first
 * n_keep tokens of the last verify block (1 <= n_keep <= its K), as if only
 * those tokens had been verified.  After a verify that returned accept_len
 * j, tokens[0..j] are the accepted ones: call iam_rollback(e, j + 1, ...) and
 * start the next block at pos + j + 1 with argmax_out[j].  Every step keeps
 * the state it started from; the GDN recurrence of the kept rows is re-run
 * from it (conv windows included) and the device position moves back to
 * pos + n_keep.  KV-cache rows of rejected tokens need no undo (the next
 * block writes them before any query reads them).  n_keep == K re-runs the
 * block and leaves the state as the step left it.  Enqueued on `stream`
 * (NULL: the engine's own stream), which must be the stream the verify ran
 * on; IAM_ESTATE when no verify ran since the state was last set.  Tensor
 * parallel engines: every rank calls it with the same n_keep (no collective).
 * No counterpart in the reference: its verify loop (batch_verify_27b.swift:
 * 141-274) never commits a partial block, and the GDN conv state flips
 * (full_forward.swift:1196, 1259) are the only state it swaps. */
int iam_rollback(iam_engine* e, int n_keep, void* stream);

/* Greedy generation (runTest, test_context.swift:1216-1270; forwardPass per
 * token, full_forward.swift:1198-1308): resets the state, runs the prompt at
 * positions 0..n_prompt-1 in verify blocks of up to max_rows tokens (the same
 * result as one token at a time), takes the last position's argmax as the
 * first generated token, then decodes one token at a time until max_new
 * tokens are out or one of the n_eos stop ids (Qwen3.5: 248046 <|im_end|>,
 * 248044 <|endoftext|>, warm_forward.swift:1254-1256) was emitted; the stop
 * id is kept.  out: int32 [max_new]; *n_out: tokens written.  Requires
 * n_prompt + max_new - 1 <= max_ctx. */
int iam_generate(iam_engine* e, const int32_t* prompt, int n_prompt, int max_new, const int32_t* eos, int n_eos,
                 int32_t* out, int* n_out);

/* Multi-sequence batch verify: n_seq independent sequences (slots
 * 0..n_seq-1, each with its own GDN state, conv window and KV cache) verify K
 * tokens each in one step; the weights are streamed once for all n_seq * K
 * rows.  tokens int32 [n_seq][K] (row 0 of each is the token being decoded),
 * pos int32 [n_seq] (each sequence's position), argmax_out int32 [n_seq][K],
 * accept_len int32 [n_seq] (per sequence, as iam_verify).  Slots from n_seq
 * on are untouched.  Requires n_seq <= max_seqs, n_seq * K <= max_rows and
 * pos[s] + K <= max_ctx.  iam_rollback applies to single-sequence verifies
 * only.  Follows batch_verify_27b.swift:141-274 (the M-row loop) with the M
 * rows split into sequences; the reference has no multi-sequence state. */
int iam_verify_batch(iam_engine* e, const int32_t* tokens, int n_seq, int K, const int32_t* pos,
                     int32_t* argmax_out, int32_t* accept_len);
/* Device-resident variant (benchmarking): d_tokens int32 [n_seq * K]; d_pos
 * int32 [n_seq] or NULL to continue from the positions the previous batch
 * step left; d_argmax int32 [n_seq * K] and d_accept int32 [n_seq] may be
 * NULL.  Nothing is synchronised. */
int iam_verify_batch_device(iam_engine* e, const int32_t* d_tokens, int n_seq, int K, const int32_t* d_pos,
                            int32_t* d_argmax, int32_t* d_accept, void* stream);

/* Device-resident variant for benchmarking: tokens/outputs stay on the GPU
 * (d_tokens int32 [K], d_argmax int32 [K]) and nothing is synchronised. */
int iam_verify_device(iam_engine* e, const int32_t* d_tokens, int K, int pos, int32_t* d_argmax, void* stream);

/* The device-side status of the engine's steps so far, for the variants that
 * do not synchronise: waits for `stream` (NULL: the engine's) and the engine
 * stream, then returns IAM_OK, IAM_ETIMEOUT (a bounded wait inside a kernel
 * gave up), IAM_EINVAL (a token id out of range reached the embedding) or,
 * across GPUs, the communicator's failure (IAM_ENCCL / IAM_ETIMEOUT past
 * comm_timeout_ms, with the communicator aborted).  The word is cleared.
 * iam_verify and iam_verify_batch return the same statuses by themselves.
 * No counterpart in the reference (full_forward.swift:1242-1245 checks the
 * command-buffer status only). */
int iam_engine_status(iam_engine* e, void* stream);

/* Read back device copies of internal tensors for tests (host buffers).
 * State tensors ("state.S.<layer>", "state.conv.<layer>",
 * "state.k_cache.<layer>", "state.v_cache.<layer>") hold every sequence
 * slot, slot after slot. */
int iam_read_tensor(iam_engine* e, const char* name, void* host_ptr, size_t bytes);
/* Final normed hidden [K, hidden] of the last step (bf16). */
int iam_read_hidden(iam_engine* e, uint16_t* host_ptr, int K);

/* Per-kernel-kind timing of one eager (non-graph) step with CUDA events:
 * kinds[i] names, ms[i] total time, bytes[i] algorithmic bytes, launches[i];
 * returns the number of kinds written (<= cap). */
int iam_profile_step(iam_engine* e, int K, int pos, int cap, const char** kinds, double* ms, double* bytes,
                     int* launches);
/* Device time of each decoder layer in one eager step of width K at pos
 * (CUDA events around every launch, summed per layer): ms[i] for its
 * attention or GDN block (input norm to the residual add), mlp_ms[i] for its
 * MLP block, is_attn[i], for i < n_layers; returns n_layers (or minus a
 * status). */
int iam_profile_layers(iam_engine* e, int K, int pos, double* ms, double* mlp_ms, int* is_attn);
/* Number of kernel launches in one graph step of width K. */
int iam_step_launches(iam_engine* e, int K);
/* Layers whose 4-bit matrices stream from pinned host memory each step
 * (dims.resident_weight_bytes), 0 when every layer is resident. */
int iam_streamed_layers(const iam_engine* e);
/* Algorithmic HBM bytes of one step of width K at position pos (weights +
 * state read/write + KV read), per GPU. */
double iam_step_bytes(iam_engine* e, int K, int pos);
/* The same for a multi-sequence step: weights once, per-sequence bytes
 * n_seq times (every sequence at position pos). */
double iam_step_bytes_batch(iam_engine* e, int n_seq, int K, int pos);

#ifdef __cplusplus
}
#endif
#endif /* IAM_H_ */
