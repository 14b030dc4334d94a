// The engine behind iam_create / iam_verify: the whole 64-layer decode or
// K-token verify step of a Qwen3.5-27B-shape model on one GPU (or one
// tensor-parallel shard), with weights, recurrent state and KV cache resident
// in HBM and the step captured as one CUDA graph per verify width.
//
// Replaces forwardPass (full_forward.swift:1198-1308), which re-reads each
// layer's weights from mmap and waits on the GPU once per layer, and the
// MLP-only M-row loop of batch_verify_27b.swift:141-274.
//
// Per GDN layer (dispatchGDNLayer, full_forward.swift:993-1161): input RMSNorm,
// one matmul launch for in_proj_qkv|z|b|a, the fused recurrent kernel, out_proj
// with the residual add fused, post-norm, gate|up with SwiGLU fused, down with
// the residual add fused.  Per attention layer (dispatchAttnLayer, 828-987):
// RMSNorm, q|k|v matmul, q/k-norm + RoPE + KV append, split flash decode,
// combine + sigmoid gate, o_proj + residual, MLP.  Then final norm, lm_head with
// an argmax epilogue and the accept-length finalisation.
#include <dlfcn.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "kernels.cuh"
#include "nccl_shim.h"
#include "safetensors.h"
#include "synth.cuh"

namespace iam {

int attn_chunk_tokens();

namespace {

constexpr int kNSplit = 32;     // attention context splits
constexpr size_t kAlign = 256;  // tensor alignment in the pool

enum class Kind { kQ4Words, kQ4Scales, kQ4Biases, kBf16, kF32 };

// A shard of a tensor: row ranges (concatenated) x one column range, of a
// [full_rows, full_cols] element grid.
struct Shard {
  std::vector<std::pair<int64_t, int64_t>> rows;  // [begin, end)
  int64_t col0 = 0, col1 = 0;
  int64_t local_rows() const {
    int64_t n = 0;
    for (auto& r : rows) n += r.second - r.first;
    return n;
  }
};

struct TensorRec {
  std::string name;      // reference tensor name
  std::string gen_name;  // name of the generator stream
  Kind kind;
  int esize;
  int64_t full_rows, full_cols;  // in stored elements (words for packed codes)
  Shard shard;
  void* ptr = nullptr;
  int syn_kind;
  float p0 = 0.f, p1 = 0.f;
  int layer = -1;     // decoder layer the tensor belongs to (-1: embedding, final norm, lm_head)
  bool host = false;  // in pinned host memory (a 4-bit matrix of a streamed layer)
  size_t bytes() const { return static_cast<size_t>(shard.local_rows()) * (shard.col1 - shard.col0) * esize; }
};

struct QW {
  uint32_t* w = nullptr;  // MLX layout (as loaded)
  uint16_t* s = nullptr;
  uint16_t* b = nullptr;
  unsigned char* packed = nullptr;  // tile-packed copy the tensor-core matmul reads
  int rows = 0, cols = 0;           // local output rows, local K
};

struct Layer {
  bool attn = false;
  int idx = 0;  // index among GDN or among attention layers
  // Streamed layers (beyond the resident budget): index among them (-1:
  // resident), and where their packed matrices sit in the pinned host copy;
  // the QW::packed pointers of a streamed layer point into device slot
  // stream_j % 2.
  int stream_j = -1;
  size_t hp_off = 0, hp_bytes = 0;
  uint16_t* in_norm = nullptr;
  uint16_t* post_norm = nullptr;
  QW gate, up, down;
  unsigned char* gateup = nullptr;  // gate and up packed as SwiGLU pairs
  // GDN
  QW qkv, z, bproj, aproj, out;
  uint16_t* conv_w = nullptr;
  float* A_log = nullptr;
  uint16_t* dt_bias = nullptr;
  uint16_t* norm_w = nullptr;
  // attention
  QW q, k, v, o;
  uint16_t* q_norm = nullptr;
  uint16_t* k_norm = nullptr;
};

struct StepIn {  // device copy of the step inputs
  int32_t pos;
  int32_t tokens[1];  // [max_rows]
};

struct ProfEntry {
  std::string kind;
  double bytes;
  int part;  // 2 * layer + (0: attention or GDN block, 1: MLP); -1: embedding, final norm, lm_head, finish
  cudaEvent_t a, b;
};

}  // namespace

struct EngineImpl {
  iam_dims d{};
  int device = 0, rank = 0, world = 1;
  cudaStream_t stream = nullptr;
  void* comm = nullptr;  // ncclComm_t
  std::string err;

  // shard-local dimensions
  int gk_l = 0, gv_l = 0, k0 = 0, v0 = 0;            // GDN heads
  int hq_l = 0, hkv_l = 0, h0 = 0, kv0 = 0;          // attention heads
  int inter_l = 0, i0 = 0, vocab_l = 0, voff = 0;     // MLP / lm_head
  int key_l = 0, conv_l = 0, vd_l = 0;
  int n_gdn = 0, n_attn = 0;

  std::vector<TensorRec> tensors;
  std::map<std::string, int> by_name;
  char* pool = nullptr;
  size_t pool_bytes = 0;
  // Tile-packed weights (qmm.cuh), rebuilt from the pool whenever a 4-bit
  // tensor was loaded or generated since the last pack.
  char* ppool = nullptr;
  size_t ppool_bytes = 0;
  // Layers past dims.resident_weight_bytes: their 4-bit matrices as loaded
  // (hpool) and tile-packed (hpacked) in pinned, device-mapped host memory;
  // two device slots take turns holding one streamed layer's packed matrices,
  // filled one layer ahead by copies on pf_stream (pf_ready[s]: slot s holds
  // its next layer; pf_free[s]: the layer in slot s has finished).
  char* hpool = nullptr;
  char* hpacked = nullptr;
  size_t hpool_bytes = 0, hpacked_bytes = 0;
  char* slot[2] = {nullptr, nullptr};
  size_t slot_bytes = 0;
  int n_streamed = 0;
  std::vector<int> streamed;  // layer index of each streamed layer, in order
  cudaStream_t pf_stream = nullptr;
  cudaEvent_t pf_ready[2] = {nullptr, nullptr}, pf_free[2] = {nullptr, nullptr}, pf_start = nullptr;
  int reg_layer = -1;  // the layer build_registry is adding tensors for
  bool packed_dirty = true;

  std::vector<Layer> layers;
  uint16_t* embed = nullptr;
  uint16_t* final_norm = nullptr;
  QW lm;

  // state, per layer one block of max_seqs sequence slots (slot 0: the
  // single-sequence entry points); S holds two copies of every slot's state
  // (s_half floats apart) and conv two windows, swapped each step by the
  // slot's parity word d_parity[slot]: a step reads the state before it and
  // leaves that copy intact, which is what iam_rollback replays the accepted
  // rows from
  int max_seqs = 1;
  size_t s_per = 0;  // floats of one slot's state in one layer
  float* S = nullptr;
  size_t s_half = 0;
  uint16_t* conv[2] = {nullptr, nullptr};
  uint16_t* kc = nullptr;
  uint16_t* vc = nullptr;
  int* d_parity = nullptr;  // [max_seqs]
  int parity = 0;
  int last_K = 0;  // rows of the last verify block since the state was set (0: none to roll back)

  // activations / workspace
  int ld_in = 0, ld_attn = 0;
  uint16_t *hidden = nullptr, *resid = nullptr, *normed = nullptr, *inproj = nullptr, *mid = nullptr,
           *mlp_h = nullptr, *q_buf = nullptr;
  uint16_t* gin = nullptr;  // [n_gdn][max_rows][ld_in]: each GDN layer's projections of the last block
  float *part_o = nullptr, *part_ml = nullptr, *red32 = nullptr;
  float* qws = nullptr;  // split-K workspace of the matmuls (zero between launches)
  int* qctr = nullptr;
  size_t qws_floats = 0, qctr_n = 0;
  unsigned long long* keys = nullptr;
  unsigned long long* best = nullptr;      // [world][max_rows] (TP)
  // Row-parallel sums over peer memory (world > 1): this rank's receive area,
  // [2 alternating buffers][world slots][max_rows][hidden] fp32 partials and
  // then [2][hidden / 128] arrival counters; every rank's area mapped here
  // through CUDA IPC (tp_peer[rank] is this rank's own).  Off (tp_p2p false):
  // NCCL all-reduce of the partials and a residual kernel.
  char* tp_area = nullptr;
  char* tp_peer[kQmmMaxPeers] = {};
  size_t tp_ctr_off = 0;
  int tp_tiles = 0;
  bool tp_p2p = false;
  int rp_idx = 0;  // row-parallel matmuls enqueued so far in the current step
  int lm_ctas = 0;
  float* rope_cs = nullptr;
  StepIn* d_in = nullptr;
  int32_t* d_out = nullptr;  // [0] accept, [1..] argmax
  int* d_err = nullptr;
  StepIn* h_in = nullptr;
  int32_t* h_out = nullptr;
  int* h_err = nullptr;  // pinned mirror of d_err, read with every synchronous step

  // multi-sequence steps: positions [max_seqs] then tokens [max_rows] (d_bin,
  // pinned mirror h_bin); accept lengths [max_seqs] then argmax [max_rows]
  // (d_bout, h_bout)
  int32_t* d_bin = nullptr;
  int32_t* h_bin = nullptr;
  int32_t* d_bout = nullptr;
  int32_t* h_bout = nullptr;

  std::map<int, cudaGraphExec_t> graphs;
  std::map<std::pair<int, int>, cudaGraphExec_t> bgraphs;  // by (n_seq, K)
  int cur_rows = 0;  // rows of the step being enqueued (all sequences)
  int cur_seqs = 0;  // sequences of a multi-sequence step being enqueued (0: the single-sequence step)
  int cur_k = 0;     // rows per sequence of that step
  int host_pos = 0;  // the position the next device-driven step starts at
  bool pdl = true;
  std::vector<ProfEntry>* prof = nullptr;
  int launches = 0;
  int cur_part = -1;  // 2 * layer + block that enqueue_step is enqueuing (profiling tags)

  int setf(int st, const std::string& m) {
    err = m;
    set_error(m);
    return st;
  }
};

namespace {

// ------------------------------------------------------------------ helpers
int ceil_div(int a, int b) { return (a + b - 1) / b; }

int check(EngineImpl& e, int r) {
  if (r != IAM_OK) e.err = iam_last_error();
  return r;
}

#define E_CUDA(call)                                                          \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess) return e.setf(e_ == cudaErrorMemoryAllocation ? IAM_ENOMEM : IAM_ECUDA, \
                                         std::string(#call) + ": " + cudaGetErrorString(e_));   \
  } while (0)

#define E_RUN(call)                      \
  do {                                   \
    int r_ = (call);                     \
    if (r_ != IAM_OK) return check(e, r_); \
  } while (0)

// Registers one stored tensor.
void add(EngineImpl& e, const std::string& name, const std::string& gen, Kind kind, int64_t full_rows,
         int64_t full_cols, Shard sh, int syn, float p0 = 0.f, float p1 = 0.f) {
  TensorRec t;
  t.name = name;
  t.gen_name = gen;
  t.kind = kind;
  t.esize = (kind == Kind::kQ4Words || kind == Kind::kF32) ? 4 : 2;
  t.full_rows = full_rows;
  t.full_cols = full_cols;
  if (sh.rows.empty()) sh.rows.push_back({0, full_rows});
  if (sh.col1 == 0) {
    sh.col0 = 0;
    sh.col1 = full_cols;
  }
  t.shard = sh;
  t.syn_kind = syn;
  t.p0 = p0;
  t.p1 = p1;
  t.layer = e.reg_layer;
  e.by_name[name] = static_cast<int>(e.tensors.size());
  e.tensors.push_back(t);
}

// A 4-bit matrix [rows, K]: row shard (output features) or K shard (columns).
void add_q4(EngineImpl& e, const std::string& base, int64_t rows, int64_t K, const Shard& row_shard, int64_t kc0,
            int64_t kc1) {
  const int g = e.d.group_size;
  Shard sw = row_shard, ss = row_shard;
  if (kc1 > kc0) {
    sw.col0 = kc0 / 8;
    sw.col1 = kc1 / 8;
    ss.col0 = kc0 / g;
    ss.col1 = kc1 / g;
  }
  add(e, base + ".weight", base + ".weight", Kind::kQ4Words, rows, K / 8, sw, SYN_WORDS);
  add(e, base + ".scales", base + ".scales", Kind::kQ4Scales, rows, K / g, ss, SYN_ABSNORMAL_BF16, 0.02f);
  add(e, base + ".biases", base + ".scales", Kind::kQ4Biases, rows, K / g, ss, SYN_NEG8_ABSNORMAL_BF16, 0.02f);
}

Shard rows_of(int64_t b, int64_t en) {
  Shard s;
  s.rows.push_back({b, en});
  return s;
}

void* tptr(EngineImpl& e, const std::string& name) { return e.tensors[e.by_name.at(name)].ptr; }

QW qw(EngineImpl& e, const std::string& base, int rows, int cols) {
  QW q;
  q.w = static_cast<uint32_t*>(tptr(e, base + ".weight"));
  q.s = static_cast<uint16_t*>(tptr(e, base + ".scales"));
  q.b = static_cast<uint16_t*>(tptr(e, base + ".biases"));
  q.rows = rows;
  q.cols = cols;
  return q;
}

int build_registry(EngineImpl& e) {
  const iam_dims& d = e.d;
  const int W = e.world, r = e.rank;
  const int H = d.hidden, I = d.intermediate;
  const int hd = d.head_dim, gd = d.gdn_dk;
  const int key_dim = d.gdn_k_heads * gd, vdim = d.gdn_v_heads * d.gdn_dv;
  const int conv_dim = 2 * key_dim + vdim;
  iam_tp_shard sp;
  E_RUN(iam_tp_shard_of(&d, r, W, &sp));
  e.gk_l = sp.gdn_k_heads;
  e.gv_l = sp.gdn_v_heads;
  e.k0 = sp.gdn_k_head0;
  e.v0 = sp.gdn_v_head0;
  e.key_l = e.gk_l * gd;
  e.vd_l = e.gv_l * d.gdn_dv;
  e.conv_l = 2 * e.key_l + e.vd_l;
  e.hq_l = sp.q_heads;
  e.h0 = sp.q_head0;
  e.hkv_l = sp.kv_heads;
  e.kv0 = sp.kv_head0;
  e.inter_l = sp.inter;
  e.i0 = sp.inter0;
  e.vocab_l = sp.vocab;
  e.voff = sp.vocab0;

  Shard qkv_rows;  // q heads, k heads, v heads of this shard
  qkv_rows.rows.push_back({e.k0 * gd, (e.k0 + e.gk_l) * gd});
  qkv_rows.rows.push_back({key_dim + e.k0 * gd, key_dim + (e.k0 + e.gk_l) * gd});
  qkv_rows.rows.push_back({2 * key_dim + e.v0 * d.gdn_dv, 2 * key_dim + (e.v0 + e.gv_l) * d.gdn_dv});
  const Shard all;

  add(e, "model.embed_tokens.weight", "model.embed_tokens.weight", Kind::kBf16, d.vocab, H, all, SYN_NORMAL_BF16,
      0.02f);
  add(e, "model.norm.weight", "model.norm.weight", Kind::kBf16, 1, H, all, SYN_ONE_PLUS_NORMAL_BF16, 0.02f);
  add_q4(e, "lm_head", d.vocab, H, rows_of(e.voff, e.voff + e.vocab_l), 0, 0);

  for (int li = 0; li < d.n_layers; ++li) {
    const std::string p = "model.layers." + std::to_string(li) + ".";
    const bool attn = (li + 1) % d.full_attn_interval == 0;
    e.reg_layer = li;
    add(e, p + "input_layernorm.weight", p + "input_layernorm.weight", Kind::kBf16, 1, H, all,
        SYN_ONE_PLUS_NORMAL_BF16, 0.02f);
    if (attn) {
      add_q4(e, p + "self_attn.q_proj", 2 * d.n_heads * hd, H, rows_of(2 * e.h0 * hd, 2 * (e.h0 + e.hq_l) * hd), 0, 0);
      add_q4(e, p + "self_attn.k_proj", d.n_kv_heads * hd, H, rows_of(e.kv0 * hd, (e.kv0 + e.hkv_l) * hd), 0, 0);
      add_q4(e, p + "self_attn.v_proj", d.n_kv_heads * hd, H, rows_of(e.kv0 * hd, (e.kv0 + e.hkv_l) * hd), 0, 0);
      add_q4(e, p + "self_attn.o_proj", H, d.n_heads * hd, all, e.h0 * hd, (e.h0 + e.hq_l) * hd);
      add(e, p + "self_attn.q_norm.weight", p + "self_attn.q_norm.weight", Kind::kBf16, 1, hd, all,
          SYN_ONE_PLUS_NORMAL_BF16, 0.02f);
      add(e, p + "self_attn.k_norm.weight", p + "self_attn.k_norm.weight", Kind::kBf16, 1, hd, all,
          SYN_ONE_PLUS_NORMAL_BF16, 0.02f);
    } else {
      add_q4(e, p + "linear_attn.in_proj_qkv", conv_dim, H, qkv_rows, 0, 0);
      add_q4(e, p + "linear_attn.in_proj_z", vdim, H, rows_of(e.v0 * d.gdn_dv, (e.v0 + e.gv_l) * d.gdn_dv), 0, 0);
      add_q4(e, p + "linear_attn.in_proj_b", d.gdn_v_heads, H, rows_of(e.v0, e.v0 + e.gv_l), 0, 0);
      add_q4(e, p + "linear_attn.in_proj_a", d.gdn_v_heads, H, rows_of(e.v0, e.v0 + e.gv_l), 0, 0);
      add(e, p + "linear_attn.conv1d.weight", p + "linear_attn.conv1d.weight", Kind::kBf16, conv_dim, d.conv_kernel,
          qkv_rows, SYN_NORMAL_BF16, 0.1f);
      add(e, p + "linear_attn.A_log", p + "linear_attn.A_log", Kind::kF32, d.gdn_v_heads, 1,
          rows_of(e.v0, e.v0 + e.gv_l), SYN_UNIFORM_F32, -1.0f, 2.0f);
      add(e, p + "linear_attn.dt_bias", p + "linear_attn.dt_bias", Kind::kBf16, d.gdn_v_heads, 1,
          rows_of(e.v0, e.v0 + e.gv_l), SYN_NORMAL_BF16, 0.1f);
      add(e, p + "linear_attn.norm.weight", p + "linear_attn.norm.weight", Kind::kBf16, 1, d.gdn_dv, all,
          SYN_ONE_PLUS_NORMAL_BF16, 0.02f);
      add_q4(e, p + "linear_attn.out_proj", H, vdim, all, e.v0 * d.gdn_dv, (e.v0 + e.gv_l) * d.gdn_dv);
    }
    add(e, p + "post_attention_layernorm.weight", p + "post_attention_layernorm.weight", Kind::kBf16, 1, H, all,
        SYN_ONE_PLUS_NORMAL_BF16, 0.02f);
    add_q4(e, p + "mlp.gate_proj", I, H, rows_of(e.i0, e.i0 + e.inter_l), 0, 0);
    add_q4(e, p + "mlp.up_proj", I, H, rows_of(e.i0, e.i0 + e.inter_l), 0, 0);
    add_q4(e, p + "mlp.down_proj", H, I, all, e.i0, e.i0 + e.inter_l);
  }
  e.reg_layer = -1;
  return IAM_OK;
}

bool is_q4(const TensorRec& t) {
  return t.kind == Kind::kQ4Words || t.kind == Kind::kQ4Scales || t.kind == Kind::kQ4Biases;
}
size_t aligned(size_t b) { return (b + kAlign - 1) / kAlign * kAlign; }

// Output rows and K of every 4-bit matrix of layer li (pointers come later).
void shape_layer(EngineImpl& e, Layer& L, int li) {
  const iam_dims& d = e.d;
  const int H = d.hidden;
  L.attn = (li + 1) % d.full_attn_interval == 0;
  auto sh = [](QW& q, int rows, int cols) {
    q.rows = rows;
    q.cols = cols;
  };
  sh(L.gate, e.inter_l, H);
  sh(L.up, e.inter_l, H);
  sh(L.down, H, e.inter_l);
  if (L.attn) {
    sh(L.q, 2 * e.hq_l * d.head_dim, H);
    sh(L.k, e.hkv_l * d.head_dim, H);
    sh(L.v, e.hkv_l * d.head_dim, H);
    sh(L.o, H, e.hq_l * d.head_dim);
  } else {
    sh(L.qkv, e.conv_l, H);
    sh(L.z, e.vd_l, H);
    sh(L.bproj, e.gv_l, H);
    sh(L.aproj, e.gv_l, H);
    sh(L.out, H, e.vd_l);
  }
}

// The packed matrices of a layer with their sizes, in their order inside the
// packed pool (or inside a slot, for a streamed layer).
std::vector<std::pair<unsigned char**, size_t>> layer_packed(EngineImpl& e, Layer& L) {
  std::vector<std::pair<unsigned char**, size_t>> v;
  auto need = [&](unsigned char** dst, int rows, int K, bool swiglu) {
    v.push_back({dst, aligned(qp_bytes(qp_tiles(rows, swiglu), K))});
  };
  need(&L.gateup, e.inter_l, e.d.hidden, true);
  need(&L.down.packed, L.down.rows, L.down.cols, false);
  for (QW* q : {&L.q, &L.k, &L.v, &L.o, &L.qkv, &L.z, &L.bproj, &L.aproj, &L.out})
    if (q->rows > 0) need(&q->packed, q->rows, q->cols, false);
  return v;
}

// Which layers stream: in order, each stays resident while its 4-bit
// matrices (as loaded and packed) fit in what is left of the budget.
void plan_streaming(EngineImpl& e) {
  const long long budget = e.d.resident_weight_bytes;
  std::vector<size_t> bytes(e.layers.size(), 0);
  for (const TensorRec& t : e.tensors)
    if (t.layer >= 0 && is_q4(t)) bytes[t.layer] += aligned(t.bytes());
  for (size_t li = 0; li < e.layers.size(); ++li)
    for (auto& m : layer_packed(e, e.layers[li])) bytes[li] += m.second;
  size_t used = 0;
  bool streaming = false;
  for (size_t li = 0; li < e.layers.size(); ++li) {
    Layer& L = e.layers[li];
    if (budget > 0 && (streaming || used + bytes[li] > static_cast<size_t>(budget))) {
      streaming = true;
      L.stream_j = e.n_streamed++;
      e.streamed.push_back(static_cast<int>(li));
    } else {
      used += bytes[li];
    }
  }
  for (TensorRec& t : e.tensors) t.host = t.layer >= 0 && is_q4(t) && e.layers[t.layer].stream_j >= 0;
}

// Packed copies: the resident layers' matrices and the lm_head in one device
// pool, every matrix at a 256-byte boundary with zero padding; a streamed
// layer's matrices at the same offsets inside device slot stream_j % 2, and
// layer after layer in the pinned host copy.
int alloc_packed(EngineImpl& e) {
  std::vector<std::pair<unsigned char**, size_t>> want;
  for (Layer& L : e.layers) {
    auto v = layer_packed(e, L);
    if (L.stream_j < 0) {
      want.insert(want.end(), v.begin(), v.end());
      continue;
    }
    size_t tot = 0;
    for (auto& m : v) tot += m.second;
    L.hp_off = e.hpacked_bytes;
    L.hp_bytes = tot;
    e.hpacked_bytes += tot;
    e.slot_bytes = std::max(e.slot_bytes, tot);
  }
  want.push_back({&e.lm.packed, aligned(qp_bytes(qp_tiles(e.lm.rows, false), e.lm.cols))});
  size_t tot = 0;
  for (auto& w : want) tot += w.second;
  E_CUDA(cudaMalloc(&e.ppool, std::max<size_t>(tot, 256)));
  E_CUDA(cudaMemset(e.ppool, 0, std::max<size_t>(tot, 256)));
  e.ppool_bytes = tot;
  size_t off = 0;
  for (auto& w : want) {
    *w.first = reinterpret_cast<unsigned char*>(e.ppool + off);
    off += w.second;
  }
  if (e.n_streamed == 0) return IAM_OK;
  for (int s = 0; s < 2; ++s) {
    E_CUDA(cudaMalloc(&e.slot[s], e.slot_bytes));
    E_CUDA(cudaMemset(e.slot[s], 0, e.slot_bytes));
    E_CUDA(cudaEventCreateWithFlags(&e.pf_ready[s], cudaEventDisableTiming));
    E_CUDA(cudaEventCreateWithFlags(&e.pf_free[s], cudaEventDisableTiming));
  }
  E_CUDA(cudaEventCreateWithFlags(&e.pf_start, cudaEventDisableTiming));
  E_CUDA(cudaHostAlloc(&e.hpacked, e.hpacked_bytes, cudaHostAllocPortable));
  E_CUDA(cudaStreamCreateWithFlags(&e.pf_stream, cudaStreamNonBlocking));
  for (Layer& L : e.layers) {
    if (L.stream_j < 0) continue;
    size_t o = 0;
    for (auto& m : layer_packed(e, L)) {
      *m.first = reinterpret_cast<unsigned char*>(e.slot[L.stream_j % 2] + o);
      o += m.second;
    }
  }
  return IAM_OK;
}

int alloc_all(EngineImpl& e) {
  const iam_dims& d = e.d;
  e.layers.resize(d.n_layers);
  for (int li = 0; li < d.n_layers; ++li) shape_layer(e, e.layers[li], li);
  plan_streaming(e);
  size_t dev_total = 0, host_total = 0;
  for (auto& t : e.tensors) (t.host ? host_total : dev_total) += aligned(t.bytes());
  e.pool_bytes = dev_total;
  E_CUDA(cudaMalloc(&e.pool, std::max<size_t>(dev_total, 256)));
  if (host_total) {
    // pinned and mapped: the generator and pack kernels read and write it in
    // place, through the same address (unified addressing)
    E_CUDA(cudaHostAlloc(&e.hpool, host_total, cudaHostAllocMapped | cudaHostAllocPortable));
    e.hpool_bytes = host_total;
    void* dp = nullptr;
    E_CUDA(cudaHostGetDevicePointer(&dp, e.hpool, 0));
    if (dp != e.hpool) return e.setf(IAM_ECUDA, "streamed weights need unified addressing of pinned host memory");
  }
  size_t off = 0, hoff = 0;
  for (auto& t : e.tensors) {
    if (t.host) {
      t.ptr = e.hpool + hoff;
      hoff += aligned(t.bytes());
    } else {
      t.ptr = e.pool + off;
      off += aligned(t.bytes());
    }
  }
  // layers
  const int H = d.hidden;
  for (int li = 0; li < d.n_layers; ++li) {
    const std::string p = "model.layers." + std::to_string(li) + ".";
    Layer& L = e.layers[li];
    L.idx = L.attn ? e.n_attn++ : e.n_gdn++;
    L.in_norm = static_cast<uint16_t*>(tptr(e, p + "input_layernorm.weight"));
    L.post_norm = static_cast<uint16_t*>(tptr(e, p + "post_attention_layernorm.weight"));
    L.gate = qw(e, p + "mlp.gate_proj", e.inter_l, H);
    L.up = qw(e, p + "mlp.up_proj", e.inter_l, H);
    L.down = qw(e, p + "mlp.down_proj", H, e.inter_l);
    if (L.attn) {
      L.q = qw(e, p + "self_attn.q_proj", 2 * e.hq_l * d.head_dim, H);
      L.k = qw(e, p + "self_attn.k_proj", e.hkv_l * d.head_dim, H);
      L.v = qw(e, p + "self_attn.v_proj", e.hkv_l * d.head_dim, H);
      L.o = qw(e, p + "self_attn.o_proj", H, e.hq_l * d.head_dim);
      L.q_norm = static_cast<uint16_t*>(tptr(e, p + "self_attn.q_norm.weight"));
      L.k_norm = static_cast<uint16_t*>(tptr(e, p + "self_attn.k_norm.weight"));
    } else {
      L.qkv = qw(e, p + "linear_attn.in_proj_qkv", e.conv_l, H);
      L.z = qw(e, p + "linear_attn.in_proj_z", e.vd_l, H);
      L.bproj = qw(e, p + "linear_attn.in_proj_b", e.gv_l, H);
      L.aproj = qw(e, p + "linear_attn.in_proj_a", e.gv_l, H);
      L.out = qw(e, p + "linear_attn.out_proj", H, e.vd_l);
      L.conv_w = static_cast<uint16_t*>(tptr(e, p + "linear_attn.conv1d.weight"));
      L.A_log = static_cast<float*>(tptr(e, p + "linear_attn.A_log"));
      L.dt_bias = static_cast<uint16_t*>(tptr(e, p + "linear_attn.dt_bias"));
      L.norm_w = static_cast<uint16_t*>(tptr(e, p + "linear_attn.norm.weight"));
    }
  }
  e.embed = static_cast<uint16_t*>(tptr(e, "model.embed_tokens.weight"));
  e.final_norm = static_cast<uint16_t*>(tptr(e, "model.norm.weight"));
  e.lm = qw(e, "lm_head", e.vocab_l, H);
  E_RUN(alloc_packed(e));
  // state
  e.max_seqs = d.max_seqs;
  const size_t slots = static_cast<size_t>(e.max_seqs);
  e.s_per = static_cast<size_t>(e.gv_l) * d.gdn_dk * d.gdn_dv;
  e.s_half = static_cast<size_t>(e.n_gdn) * slots * e.s_per;
  E_CUDA(cudaMalloc(&e.S, std::max<size_t>(1, 2 * e.s_half) * sizeof(float)));
  for (int i = 0; i < 2; ++i)
    E_CUDA(cudaMalloc(&e.conv[i], std::max<size_t>(1, static_cast<size_t>(e.n_gdn) * slots * 3 * e.conv_l) * 2));
  const size_t kv = static_cast<size_t>(e.n_attn) * slots * d.max_ctx * e.hkv_l * d.head_dim;
  E_CUDA(cudaMalloc(&e.kc, std::max<size_t>(1, kv) * 2));
  E_CUDA(cudaMalloc(&e.vc, std::max<size_t>(1, kv) * 2));
  E_CUDA(cudaMalloc(&e.d_parity, slots * sizeof(int)));
  E_CUDA(cudaMemset(e.d_parity, 0, slots * sizeof(int)));

  // activations
  const int R = d.max_rows;
  e.ld_in = (e.conv_l + e.vd_l + 2 * e.gv_l + 7) / 8 * 8;
  e.ld_attn = 2 * e.hq_l * d.head_dim + 2 * e.hkv_l * d.head_dim;
  const int ld_big = std::max(e.ld_in, e.ld_attn);
  const int ld_mid = std::max(e.vd_l, e.hq_l * d.head_dim);
  E_CUDA(cudaMalloc(&e.hidden, static_cast<size_t>(R) * H * 2));
  E_CUDA(cudaMalloc(&e.resid, static_cast<size_t>(R) * H * 2));
  E_CUDA(cudaMalloc(&e.normed, static_cast<size_t>(R) * H * 2));
  E_CUDA(cudaMalloc(&e.inproj, static_cast<size_t>(R) * ld_big * 2));
  E_CUDA(cudaMalloc(&e.gin, std::max<size_t>(1, static_cast<size_t>(e.n_gdn) * R * e.ld_in) * 2));
  E_CUDA(cudaMalloc(&e.mid, static_cast<size_t>(R) * ld_mid * 2));
  E_CUDA(cudaMalloc(&e.mlp_h, static_cast<size_t>(R) * e.inter_l * 2));
  E_CUDA(cudaMalloc(&e.q_buf, static_cast<size_t>(R) * e.hq_l * d.head_dim * 2));
  E_CUDA(cudaMalloc(&e.part_o, static_cast<size_t>(R) * e.hq_l * kNSplit * d.head_dim * 4));
  E_CUDA(cudaMalloc(&e.part_ml, static_cast<size_t>(R) * e.hq_l * kNSplit * 2 * 4));
  if (e.world > 1) E_CUDA(cudaMalloc(&e.red32, static_cast<size_t>(R) * H * 4));
  e.lm_ctas = ceil_div(e.vocab_l, 16);  // at least 16 rows per CTA in every config
  E_CUDA(cudaMalloc(&e.keys, static_cast<size_t>(e.lm_ctas) * R * 8));
  // split-K workspace: (rows / 16) tiles x 512 floats for the widest matrix
  // (lm_head or the fused projections); a plan that would need more runs
  // with a smaller split (qmm_tc_run caps it by the workspace)
  {
    const size_t widest = std::max<size_t>({static_cast<size_t>(e.vocab_l), static_cast<size_t>(2 * e.inter_l),
                                            static_cast<size_t>(e.ld_in), static_cast<size_t>(e.ld_attn),
                                            static_cast<size_t>(H)});
    e.qctr_n = (widest / 16 + 64) * 1;
    e.qws_floats = (widest / 16 + 64) * 4 * 128;
    E_CUDA(cudaMalloc(&e.qws, e.qws_floats * sizeof(float)));
    E_CUDA(cudaMalloc(&e.qctr, e.qctr_n * sizeof(int)));
    E_CUDA(cudaMemset(e.qws, 0, e.qws_floats * sizeof(float)));
    E_CUDA(cudaMemset(e.qctr, 0, e.qctr_n * sizeof(int)));
  }
  E_CUDA(cudaMalloc(&e.best, static_cast<size_t>(e.world) * R * 8));
  E_CUDA(cudaMalloc(&e.d_in, sizeof(int32_t) * (1 + R)));
  E_CUDA(cudaMalloc(&e.d_out, sizeof(int32_t) * (1 + R)));
  E_CUDA(cudaMalloc(&e.d_err, sizeof(int)));
  E_CUDA(cudaMemset(e.d_err, 0, sizeof(int)));
  E_CUDA(cudaMallocHost(&e.h_in, sizeof(int32_t) * (1 + R)));
  E_CUDA(cudaMallocHost(&e.h_out, sizeof(int32_t) * (1 + R)));
  E_CUDA(cudaMallocHost(&e.h_err, sizeof(int)));
  *e.h_err = 0;
  E_CUDA(cudaMalloc(&e.d_bin, sizeof(int32_t) * (slots + R)));
  E_CUDA(cudaMemset(e.d_bin, 0, sizeof(int32_t) * (slots + R)));
  E_CUDA(cudaMalloc(&e.d_bout, sizeof(int32_t) * (slots + R)));
  E_CUDA(cudaMallocHost(&e.h_bin, sizeof(int32_t) * (slots + R)));
  E_CUDA(cudaMallocHost(&e.h_bout, sizeof(int32_t) * (slots + R)));

  // RoPE table [max_ctx][rotary/2] (cos, sin): precomputeRoPE in double
  // (full_forward.swift:734-743)
  std::vector<float> cs(static_cast<size_t>(d.max_ctx) * d.rotary_dim);
  for (int pos = 0; pos < d.max_ctx; ++pos)
    for (int i = 0; i < d.rotary_dim / 2; ++i) {
      const double freq = 1.0 / std::pow(static_cast<double>(d.rope_theta), static_cast<double>(2 * i) / d.rotary_dim);
      const double ang = static_cast<double>(pos) * freq;
      cs[static_cast<size_t>(pos) * d.rotary_dim + 2 * i] = static_cast<float>(std::cos(ang));
      cs[static_cast<size_t>(pos) * d.rotary_dim + 2 * i + 1] = static_cast<float>(std::sin(ang));
    }
  E_CUDA(cudaMalloc(&e.rope_cs, cs.size() * 4));
  E_CUDA(cudaMemcpy(e.rope_cs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  return IAM_OK;
}

// ------------------------------------------------------------------ step
struct Recorder {
  EngineImpl& e;
  const char* kind;
  double bytes;
  ProfEntry ent;
  Recorder(EngineImpl& en, const char* k, double b) : e(en), kind(k), bytes(b) {
    e.launches++;
    if (e.prof) {
      ent.kind = k;
      ent.part = e.cur_part;
      ent.bytes = b;
      cudaEventCreate(&ent.a);
      cudaEventCreate(&ent.b);
      cudaEventRecord(ent.a, e.stream);
    }
  }
  ~Recorder() {
    if (e.prof) {
      cudaEventRecord(ent.b, e.stream);
      e.prof->push_back(ent);
    }
  }
};

double qbytes(const QW& q) { return static_cast<double>(q.rows) * q.cols * (0.5 + 4.0 / 64.0); }

void seg_of(QmmSeg& s, const QW& q, int mode) {
  s = QmmSeg{};
  s.packed = q.packed;
  s.w = q.w;
  s.s = q.s;
  s.b = q.b;
  s.rows = q.rows;
  s.mode = mode;
}

// Rebuilds the packed weights from the loaded ones (never during capture).
int ensure_packed(EngineImpl& e) {
  if (!e.packed_dirty) return IAM_OK;
  auto pk = [&](const QW& q) {
    const int tiles = qp_tiles(q.rows, false);
    int r = qmm_pack_begin(q.packed, tiles, q.cols, e.stream);
    if (r == IAM_OK) r = qmm_pack_scan(q.s, q.rows, q.cols, q.packed, tiles, 128, e.stream);
    if (r == IAM_OK) r = qmm_pack(q.w, q.s, q.b, q.rows, q.cols, q.packed, tiles, 128, 0, e.stream);
    return r;
  };
  for (const Layer& L : e.layers) {
    // a streamed layer is packed in its slot (cleared first: the slot held
    // other matrices) and copied out to the pinned host copy
    if (L.stream_j >= 0) E_CUDA(cudaMemsetAsync(e.slot[L.stream_j % 2], 0, L.hp_bytes, e.stream));
    const int gt = qp_tiles(e.inter_l, true);
    E_RUN(qmm_pack_begin(L.gateup, gt, L.gate.cols, e.stream));
    E_RUN(qmm_pack_scan(L.gate.s, L.gate.rows, L.gate.cols, L.gateup, gt, 64, e.stream));
    E_RUN(qmm_pack_scan(L.up.s, L.up.rows, L.up.cols, L.gateup, gt, 64, e.stream));
    E_RUN(qmm_pack(L.gate.w, L.gate.s, L.gate.b, L.gate.rows, L.gate.cols, L.gateup, gt, 64, 0, e.stream));
    E_RUN(qmm_pack(L.up.w, L.up.s, L.up.b, L.up.rows, L.up.cols, L.gateup, gt, 64, 64, e.stream));
    E_RUN(pk(L.down));
    for (const QW* q : {&L.q, &L.k, &L.v, &L.o, &L.qkv, &L.z, &L.bproj, &L.aproj, &L.out})
      if (q->w) E_RUN(pk(*q));
    if (L.stream_j >= 0)
      E_CUDA(cudaMemcpyAsync(e.hpacked + L.hp_off, e.slot[L.stream_j % 2], L.hp_bytes, cudaMemcpyDeviceToHost,
                             e.stream));
  }
  E_RUN(pk(e.lm));
  E_CUDA(cudaStreamSynchronize(e.stream));
  e.packed_dirty = false;
  return IAM_OK;
}

int run_qmm(EngineImpl& e, QmmArgs& a, const char* kind, double bytes) {
  Recorder rec(e, kind, bytes);
  a.ws = e.qws;
  a.counters = e.qctr;
  a.err = e.d_err;
  return qmm_run(a, e.stream, e.pdl, e.qws_floats, e.qctr_n);
}

// Row-parallel matmul (K sharded) followed by the residual add: fused on one
// GPU; fp32 partials + NCCL all-reduce + residual kernel across GPUs.
int row_parallel_resid(EngineImpl& e, const QW& q, const uint16_t* x, int ldx, const uint16_t* resid, uint16_t* out);

// The GDN kernel's arguments for layer L over the first `rows` rows of each
// of n_seq sequences (slots 0..n_seq-1; sequence q's rows follow the q * rows
// before them) of the layer's projections of the current block (e.gin); the
// state buffers and conv windows of each slot are picked on the device by its
// parity word.
GdnArgs gdn_args(EngineImpl& e, const Layer& L, int rows, int n_seq) {
  const iam_dims& d = e.d;
  GdnArgs g = {};
  g.in = e.gin + static_cast<size_t>(L.idx) * d.max_rows * e.ld_in;
  g.ld_in = e.ld_in;
  g.z_col = e.conv_l;
  g.b_col = e.conv_l + e.vd_l;
  g.a_col = e.conv_l + e.vd_l + e.gv_l;
  g.conv_w = L.conv_w;
  const size_t coff = static_cast<size_t>(L.idx) * e.max_seqs * 3 * e.conv_l;
  g.conv_in = e.conv[0] + coff;
  g.conv_out = e.conv[1] + coff;
  g.parity_dev = e.d_parity;
  g.A_log = L.A_log;
  g.dt_bias = L.dt_bias;
  g.norm_w = L.norm_w;
  g.S = e.S + static_cast<size_t>(L.idx) * e.max_seqs * e.s_per;
  g.S_alt = g.S + e.s_half;
  g.n_seq = n_seq;
  g.seq_S = e.s_per;
  g.seq_conv = static_cast<size_t>(3) * e.conv_l;
  g.out = e.mid;
  g.ld_out = e.vd_l;
  g.n_k_heads = e.gk_l;
  g.n_v_heads = e.gv_l;
  g.key_dim = e.key_l;
  g.conv_dim = e.conv_l;
  g.rows = rows;
  g.eps = d.eps;
  return g;
}

// The RMSNorm ahead of a matmul over the residual stream: fused into the
// matmul (its CTAs normalise the rows they read) when the step has at most
// kGemvNormMaxM rows and runs on the GEMV path, which removes the norm
// kernel's launch and its serialisation; else the norm kernel writes
// e.normed.  Sets the matmul's input either way.  IAM_FUSED_NORM=0 keeps the
// norm kernel.
int norm_into(EngineImpl& e, QmmArgs& a, const uint16_t* x, const uint16_t* w, int K) {
  const iam_dims& d = e.d;
  const int H = d.hidden;
  const char* env = std::getenv("IAM_FUSED_NORM");
  const bool fuse = K <= kGemvNormMaxM && K <= qmm_gemv_max_m() && !(env && env[0] == '0');
  a.ldx = H;
  if (fuse) {
    a.x = x;
    a.norm_w = w;
    a.norm_eps = d.eps;
    return IAM_OK;
  }
  Recorder rec(e, "rmsnorm", 4.0 * K * H);
  E_RUN(launch_rms_norm(x, H, w, e.normed, H, K, H, d.eps, e.stream, e.pdl));
  a.x = e.normed;
  return IAM_OK;
}

int enqueue_gdn(EngineImpl& e, const Layer& L, int K) {
  const iam_dims& d = e.d;
  const int H = d.hidden;
  uint16_t* const in = e.gin + static_cast<size_t>(L.idx) * d.max_rows * e.ld_in;
  QmmArgs a = {};
  E_RUN(norm_into(e, a, e.hidden, L.in_norm, K));
  a.M = K;
  a.K = H;
  a.nseg = 4;
  seg_of(a.seg[0], L.qkv, EPI_STORE);
  a.seg[0].out = in;
  seg_of(a.seg[1], L.z, EPI_STORE);
  a.seg[1].out = in + e.conv_l;
  seg_of(a.seg[2], L.bproj, EPI_STORE);
  a.seg[2].out = in + e.conv_l + e.vd_l;
  seg_of(a.seg[3], L.aproj, EPI_STORE);
  a.seg[3].out = in + e.conv_l + e.vd_l + e.gv_l;
  for (int i = 0; i < 4; ++i) a.seg[i].ldo = e.ld_in;
  E_RUN(run_qmm(e, a, "qmm", qbytes(L.qkv) + qbytes(L.z) + qbytes(L.bproj) + qbytes(L.aproj)));

  const GdnArgs g = gdn_args(e, L, e.cur_seqs ? e.cur_k : K, std::max(1, e.cur_seqs));
  {
    Recorder rec(e, "gdn", 2.0 * e.gv_l * d.gdn_dk * d.gdn_dv * 4 + 2.0 * 3 * e.conv_l * 2);
    E_RUN(launch_gdn(g, e.stream, e.pdl));
  }
  E_RUN(row_parallel_resid(e, L.out, e.mid, e.vd_l, e.hidden, e.resid));
  return IAM_OK;
}

int enqueue_attn(EngineImpl& e, const Layer& L, int K) {
  const iam_dims& d = e.d;
  const int H = d.hidden, hd = d.head_dim;
  QmmArgs a = {};
  E_RUN(norm_into(e, a, e.hidden, L.in_norm, K));
  a.M = K;
  a.K = H;
  a.nseg = 3;
  seg_of(a.seg[0], L.q, EPI_STORE);
  a.seg[0].out = e.inproj;
  seg_of(a.seg[1], L.k, EPI_STORE);
  a.seg[1].out = e.inproj + 2 * e.hq_l * hd;
  seg_of(a.seg[2], L.v, EPI_STORE);
  a.seg[2].out = e.inproj + 2 * e.hq_l * hd + e.hkv_l * hd;
  for (int i = 0; i < 3; ++i) a.seg[i].ldo = e.ld_attn;
  E_RUN(run_qmm(e, a, "qmm", qbytes(L.q) + qbytes(L.k) + qbytes(L.v)));

  AttnArgs t = {};
  t.qkv = e.inproj;
  t.ld_qkv = e.ld_attn;
  t.k_col = 2 * e.hq_l * hd;
  t.v_col = 2 * e.hq_l * hd + e.hkv_l * hd;
  t.q_norm_w = L.q_norm;
  t.k_norm_w = L.k_norm;
  const size_t seq_kv = static_cast<size_t>(d.max_ctx) * e.hkv_l * hd;
  const size_t kvoff = static_cast<size_t>(L.idx) * e.max_seqs * seq_kv;
  t.k_cache = e.kc + kvoff;
  t.v_cache = e.vc + kvoff;
  t.q_buf = e.q_buf;
  t.part_o = e.part_o;
  t.part_ml = e.part_ml;
  t.out = e.mid;
  t.ld_out = e.hq_l * hd;
  t.n_heads = e.hq_l;
  t.n_kv_heads = e.hkv_l;
  t.head_dim = hd;
  t.rotary_dim = d.rotary_dim;
  t.rope_cs = e.rope_cs;
  t.max_ctx = d.max_ctx;
  t.rows = K;
  t.pos_dev = &e.d_in->pos;
  if (e.cur_seqs) {
    t.n_seq = e.cur_seqs;
    t.seq_rows = e.cur_k;
    t.seq_kv = seq_kv;
    t.pos_dev = e.d_bin;
  }
  t.chunk = attn_chunk_tokens();
  t.nsplit = kNSplit;
  t.eps = d.eps;
  {
    Recorder rec(e, "attn_prep", 2.0 * K * e.ld_attn);
    E_RUN(launch_attn_prep(t, e.stream, e.pdl));
  }
  {
    Recorder rec(e, "attn_decode", 0.0);
    E_RUN(launch_attn_decode(t, e.stream, e.pdl));
  }
  {
    Recorder rec(e, "attn_combine", 4.0 * K * e.hq_l * kNSplit * hd);
    E_RUN(launch_attn_combine(t, e.stream, e.pdl));
  }
  E_RUN(row_parallel_resid(e, L.o, e.mid, e.hq_l * hd, e.hidden, e.resid));
  return IAM_OK;
}

int enqueue_mlp(EngineImpl& e, const Layer& L, int K) {
  const iam_dims& d = e.d;
  const int H = d.hidden;
  QmmArgs a = {};
  E_RUN(norm_into(e, a, e.resid, L.post_norm, K));
  a.M = K;
  a.K = H;
  a.nseg = 1;
  seg_of(a.seg[0], L.gate, EPI_SWIGLU);
  a.seg[0].packed = L.gateup;
  a.seg[0].w2 = L.up.w;
  a.seg[0].s2 = L.up.s;
  a.seg[0].b2 = L.up.b;
  a.seg[0].out = e.mlp_h;
  a.seg[0].ldo = e.inter_l;
  E_RUN(run_qmm(e, a, "qmm", qbytes(L.gate) + qbytes(L.up)));
  E_RUN(row_parallel_resid(e, L.down, e.mlp_h, e.inter_l, e.resid, e.hidden));
  return IAM_OK;
}

__global__ void resid_from_f32_kernel(const float* y, const uint16_t* resid, uint16_t* out, int n) {
  pdl_wait();
  pdl_trigger();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = f2bf(bf2f(resid[i]) + round_bf(y[i]));
}

// The row-parallel sum across GPUs plus the residual, one CTA per 128-column
// tile: waits (bounded, on the GPU's global timer) until every rank's every
// pass of the tile has arrived in this rank's receive slots, re-arms the
// counter, then out = bf16(resid + bf16(sum of the ranks' partials in rank
// order)) -- every rank computes the same bits.
__global__ void __launch_bounds__(512) tp_reduce_resid_kernel(const float* __restrict__ recv, int* ctr, int world,
                                                              size_t slot, int expect, int M, int H,
                                                              const uint16_t* __restrict__ resid,
                                                              uint16_t* __restrict__ out, int* err,
                                                              unsigned long long limit_ns) {
  pdl_wait();
  pdl_trigger();
  __shared__ int ok;
  const int tile = blockIdx.x;
  if (threadIdx.x == 0) {
    unsigned long long t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    int v = 0;
    // after one wait gave up (a peer is gone), the rest of the step does not
    // wait again: the step returns the error and the engine refuses further
    // steps
    bool failed = *reinterpret_cast<volatile int*>(err) == IAM_ETIMEOUT;
    for (uint32_t n = 0; !failed; ++n) {
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(ctr + tile) : "memory");
      if (v >= expect) break;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > limit_ns) failed = true;
      if ((n & 255) == 255 && *reinterpret_cast<volatile int*>(err) == IAM_ETIMEOUT) failed = true;
      __nanosleep(128);
    }
    ok = !failed && v >= expect;
    if (ok) ctr[tile] = 0;
    else atomicCAS(err, 0, IAM_ETIMEOUT);
  }
  __syncthreads();
  if (!ok) return;
  const int c0 = tile * 128;
  for (int i = threadIdx.x; i < M * 128; i += blockDim.x) {
    const int c = c0 + (i & 127);
    if (c >= H) continue;
    const size_t o = static_cast<size_t>(i >> 7) * H + c;
    float sum = __ldcg(recv + o);
    for (int r = 1; r < world; ++r) sum += __ldcg(recv + r * slot + o);
    out[o] = f2bf(bf2f(resid[o]) + round_bf(sum));
  }
}

__global__ void advance_kernel(StepIn* in, int* parity, int K) {
  in->pos += K;
  *parity ^= 1;
}

// Undoes advance_kernel: the state copies the last step read become the
// current ones again and the device position returns to the block's start.
__global__ void rewind_kernel(StepIn* in, int* parity, int K) {
  in->pos -= K;
  *parity ^= 1;
}

// Re-runs the GDN recurrence of every GDN layer over the first n_keep rows of
// the last block, from the state copies that block read, into the copies it
// wrote; the device position ends n_keep past the block's start.  The
// attention layers need nothing: the KV-cache rows of rejected tokens lie past
// the new position, and the next block overwrites them before any query
// reaches them (a query at position p reads rows <= p).
int enqueue_rollback(EngineImpl& e, int K, int n_keep, cudaStream_t st) {
  rewind_kernel<<<1, 1, 0, st>>>(e.d_in, e.d_parity, K);
  E_CUDA(cudaGetLastError());
  for (const Layer& L : e.layers)
    if (!L.attn) E_RUN(launch_gdn(gdn_args(e, L, n_keep, 1), st, false));
  advance_kernel<<<1, 1, 0, st>>>(e.d_in, e.d_parity, n_keep);
  E_CUDA(cudaGetLastError());
  return IAM_OK;
}


int row_parallel_resid(EngineImpl& e, const QW& q, const uint16_t* x, int ldx, const uint16_t* resid, uint16_t* out) {
  const int H = e.d.hidden, M = e.cur_rows;
  QmmArgs a = {};
  a.x = x;
  a.ldx = ldx;
  a.M = M;
  a.K = q.cols;
  a.nseg = 1;
  if (e.world == 1) {
    seg_of(a.seg[0], q, EPI_RESID);
    a.seg[0].out = out;
    a.seg[0].ldo = H;
    a.seg[0].resid = resid;
    a.seg[0].ldr = H;
    return run_qmm(e, a, "qmm", qbytes(q));
  }
  seg_of(a.seg[0], q, EPI_F32);
  a.seg[0].ldo = H;
  if (e.tp_p2p) {
    // alternating buffers: a rank writes buffer b again only after its own sum
    // over the other buffer, which waited for every peer's partial of that
    // matmul -- pushed after the peer's sum over buffer b had finished
    const int b = e.rp_idx++ & 1;
    const size_t slot = static_cast<size_t>(e.d.max_rows) * H;
    auto data = [&](char* area) {
      return reinterpret_cast<float*>(area) + static_cast<size_t>(b) * e.world * slot;
    };
    auto ctr = [&](char* area) { return reinterpret_cast<int*>(area + e.tp_ctr_off) + b * e.tp_tiles; };
    a.npush = e.world;
    for (int i = 0; i < e.world; ++i) {  // this rank's own slot first, then the peers in ring order
      const int r = (e.rank + i) % e.world;
      a.push[i] = data(e.tp_peer[r]) + static_cast<size_t>(e.rank) * slot;
      a.push_ctr[i] = ctr(e.tp_peer[r]);
    }
    E_RUN(run_qmm(e, a, "qmm", qbytes(q)));
    Recorder rec(e, "tp_reduce", 4.0 * M * H * e.world + 4.0 * M * H);
    const unsigned long long limit_ns = 1000000ull * static_cast<unsigned long long>(e.d.comm_timeout_ms > 0 ? e.d.comm_timeout_ms : 120000);
    return launch_k(tp_reduce_resid_kernel, dim3(e.tp_tiles), dim3(512), 0, e.stream, e.pdl,
                    static_cast<const float*>(data(e.tp_area)), ctr(e.tp_area), e.world, slot,
                    e.world * qmm_packed_passes(M), M, H, resid, out, e.d_err, limit_ns);
  }
  a.seg[0].out32 = e.red32;
  E_RUN(run_qmm(e, a, "qmm", qbytes(q)));
  {
    Recorder rec(e, "allreduce", 4.0 * M * H);
    E_RUN(nccl_allreduce_f32(e.comm, e.red32, static_cast<size_t>(M) * H, e.stream));
  }
  Recorder rec(e, "resid", 8.0 * M * H);
  const int n = M * H;
  return launch_k(resid_from_f32_kernel, dim3(std::min(ceil_div(n, 256), 1184)), dim3(256), 0, e.stream, e.pdl, e.red32,
                  resid, out, n);
}

__global__ void advance_seqs_kernel(int32_t* pos, int* parity, int n_seq, int K) {
  for (int q = threadIdx.x; q < n_seq; q += blockDim.x) {
    pos[q] += K;
    parity[q] ^= 1;
  }
}

// The multi-sequence step's end: per-row argmax (lm_head keys reduced one CTA
// a row, across ranks through an all-gather of the rows' best keys), each
// sequence's accept length, and the slots' positions and parities advanced.
int enqueue_finish_seqs(EngineImpl& e, int nparts, int n_seq, int Kseq) {
  const int rows = n_seq * Kseq;
  const int32_t* tokens = e.d_bin + e.max_seqs;
  int32_t* argmax = e.d_bout + e.max_seqs;
  if (e.world == 1) {
    Recorder rec(e, "finalize", 8.0 * nparts * rows);
    E_RUN(launch_finalize_batch(e.keys, nparts, e.d.max_rows, n_seq, Kseq, tokens, argmax, e.d_bout, e.stream,
                                e.pdl));
  } else {
    unsigned long long* mine = e.best + static_cast<size_t>(e.rank) * rows;
    {
      Recorder rec(e, "finalize", 8.0 * nparts * rows);
      E_RUN(launch_best_rows(e.keys, nparts, e.d.max_rows, rows, mine, e.stream, e.pdl));
    }
    {
      Recorder rec(e, "allgather", 8.0 * e.world * rows);
      E_RUN(nccl_allgather_u64(e.comm, mine, e.best, static_cast<size_t>(rows), e.stream));
    }
    Recorder rec(e, "finalize", 8.0 * e.world * rows);
    E_RUN(launch_finalize_batch(e.best, e.world, rows, n_seq, Kseq, tokens, argmax, e.d_bout, e.stream, false));
  }
  Recorder rec(e, "advance", 8.0 * n_seq);
  advance_seqs_kernel<<<1, 256, 0, e.stream>>>(e.d_bin, e.d_parity, n_seq, Kseq);
  E_CUDA(cudaGetLastError());
  return IAM_OK;
}

// Copies streamed layer j's packed matrices into slot j % 2 on the prefetch
// stream, once the layer that held the slot before it (j - 2) has finished.
int prefetch_layer(EngineImpl& e, int j) {
  const Layer& L = e.layers[e.streamed[j]];
  const int s = j % 2;
  if (j >= 2) E_CUDA(cudaStreamWaitEvent(e.pf_stream, e.pf_free[s], 0));
  E_CUDA(cudaMemcpyAsync(e.slot[s], e.hpacked + L.hp_off, L.hp_bytes, cudaMemcpyHostToDevice, e.pf_stream));
  E_CUDA(cudaEventRecord(e.pf_ready[s], e.pf_stream));
  return IAM_OK;
}

// One step of the whole model: K rows of the single sequence (n_seq = 0), or
// K rows of each of the sequences in slots 0..n_seq-1 (n_seq >= 1, the
// multi-sequence step: inputs and outputs in d_bin / d_bout).
int enqueue_step(EngineImpl& e, int n_seq, int Kseq) {
  const iam_dims& d = e.d;
  const int K = n_seq ? n_seq * Kseq : Kseq;  // rows of the step
  e.cur_rows = K;
  e.cur_seqs = n_seq;
  e.cur_k = Kseq;
  e.rp_idx = 0;  // two row-parallel matmuls a layer: every step starts on buffer 0
  const int32_t* tokens = n_seq ? e.d_bin + e.max_seqs : e.d_in->tokens;
  {
    Recorder rec(e, "embed", 4.0 * K * d.hidden);
    E_RUN(launch_embed_bf16(e.embed, tokens, e.hidden, K, d.hidden, d.vocab, e.d_err, e.stream, false));
  }
  if (e.n_streamed) {
    // the prefetch stream forks from the step's start (the slots are free:
    // the previous step precedes it on the engine stream)
    E_CUDA(cudaEventRecord(e.pf_start, e.stream));
    E_CUDA(cudaStreamWaitEvent(e.pf_stream, e.pf_start, 0));
    for (int j = 0; j < std::min(2, e.n_streamed); ++j) E_RUN(prefetch_layer(e, j));
  }
  for (const Layer& L : e.layers) {
    const int j = L.stream_j;
    e.cur_part = 2 * static_cast<int>(&L - e.layers.data());
    if (j >= 0) E_CUDA(cudaStreamWaitEvent(e.stream, e.pf_ready[j % 2], 0));
    if (L.attn) E_RUN(enqueue_attn(e, L, K));
    else E_RUN(enqueue_gdn(e, L, K));
    e.cur_part += 1;
    E_RUN(enqueue_mlp(e, L, K));
    if (j >= 0) {
      E_CUDA(cudaEventRecord(e.pf_free[j % 2], e.stream));
      if (j + 2 < e.n_streamed) E_RUN(prefetch_layer(e, j + 2));
    }
  }
  e.cur_part = -1;
  {
    Recorder rec(e, "rmsnorm", 4.0 * K * d.hidden);
    E_RUN(launch_rms_norm(e.hidden, d.hidden, e.final_norm, e.normed, d.hidden, K, d.hidden, d.eps, e.stream, e.pdl));
  }
  QmmArgs a = {};
  a.x = e.normed;
  a.ldx = d.hidden;
  a.M = K;
  a.K = d.hidden;
  a.nseg = 1;
  seg_of(a.seg[0], e.lm, EPI_ARGMAX);
  a.seg[0].keys = e.keys;
  a.seg[0].key_ld = d.max_rows;
  a.seg[0].col_base = e.voff;
  E_RUN(run_qmm(e, a, "qmm", qbytes(e.lm)));
  // one key row per 128-row lm_head tile
  const int nparts = qp_tiles(e.lm.rows, false);
  if (n_seq) return enqueue_finish_seqs(e, nparts, n_seq, Kseq);
  if (e.world == 1) {
    Recorder rec(e, "finalize", 8.0 * nparts * K);
    E_RUN(launch_finalize(e.keys, nparts, d.max_rows, K, e.d_in->tokens, e.d_out + 1, e.d_out, e.stream, e.pdl));
  } else {
    {
      Recorder rec(e, "finalize", 8.0 * nparts * K);
      E_RUN(launch_best_keys(e.keys, nparts, d.max_rows, K, e.best + static_cast<size_t>(e.rank) * K, e.stream, e.pdl));
    }
    {
      Recorder rec(e, "allgather", 8.0 * e.world * K);
      E_RUN(nccl_allgather_u64(e.comm, e.best + static_cast<size_t>(e.rank) * K, e.best, static_cast<size_t>(K),
                               e.stream));
    }
    Recorder rec(e, "finalize", 8.0 * e.world * K);
    E_RUN(launch_finalize(e.best, e.world, K, K, e.d_in->tokens, e.d_out + 1, e.d_out, e.stream, false));
  }
  {
    Recorder rec(e, "advance", 8.0);
    advance_kernel<<<1, 1, 0, e.stream>>>(e.d_in, e.d_parity, K);
    E_CUDA(cudaGetLastError());
  }
  return IAM_OK;
}

int get_graph(EngineImpl& e, int K, cudaGraphExec_t* out) {
  auto it = e.graphs.find(K);
  if (it != e.graphs.end()) {
    *out = it->second;
    return IAM_OK;
  }
  cudaGraph_t g = nullptr;
  E_CUDA(cudaStreamBeginCapture(e.stream, cudaStreamCaptureModeThreadLocal));
  const int r = enqueue_step(e, 0, K);
  cudaGraph_t gg = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(e.stream, &gg);
  if (r != IAM_OK) {
    if (gg) cudaGraphDestroy(gg);
    return r;
  }
  E_CUDA(ce);
  g = gg;
  cudaGraphExec_t ex = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  E_CUDA(ie);
  e.graphs[K] = ex;
  *out = ex;
  return IAM_OK;
}

int get_batch_graph(EngineImpl& e, int n_seq, int K, cudaGraphExec_t* out) {
  const auto key = std::make_pair(n_seq, K);
  auto it = e.bgraphs.find(key);
  if (it != e.bgraphs.end()) {
    *out = it->second;
    return IAM_OK;
  }
  E_CUDA(cudaStreamBeginCapture(e.stream, cudaStreamCaptureModeThreadLocal));
  const int r = enqueue_step(e, n_seq, K);
  cudaGraph_t gg = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(e.stream, &gg);
  if (r != IAM_OK) {
    if (gg) cudaGraphDestroy(gg);
    return r;
  }
  E_CUDA(ce);
  cudaGraphExec_t ex = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&ex, gg, 0);
  cudaGraphDestroy(gg);
  E_CUDA(ie);
  e.bgraphs[key] = ex;
  *out = ex;
  return IAM_OK;
}

int synth_tensor(EngineImpl& e, const TensorRec& t, uint64_t seed) {
  SynthJob j = {};
  j.stream = synth_stream(seed, t.gen_name.c_str());
  j.kind = t.syn_kind;
  j.p0 = t.p0;
  j.p1 = t.p1;
  j.full_cols = static_cast<uint64_t>(t.full_cols);
  j.col0 = static_cast<uint64_t>(t.shard.col0);
  j.width = static_cast<uint64_t>(t.shard.col1 - t.shard.col0);
  char* dst = static_cast<char*>(t.ptr);
  for (auto& rr : t.shard.rows) {
    j.dst = dst;
    j.row0 = static_cast<uint64_t>(rr.first);
    j.rows = static_cast<uint64_t>(rr.second - rr.first);
    E_RUN(synth_fill(j, e.stream));
    dst += static_cast<size_t>(j.rows) * j.width * t.esize;
  }
  return IAM_OK;
}

}  // namespace
}  // namespace iam

// ====================================================================== C ABI
using iam::EngineImpl;

struct iam_engine {
  EngineImpl impl;
};

extern "C" void iam_dims_qwen35_27b(iam_dims* d) {
  d->hidden = 5120;
  d->intermediate = 17408;
  d->vocab = 248320;
  d->n_layers = 64;
  d->full_attn_interval = 4;
  d->n_heads = 24;
  d->n_kv_heads = 4;
  d->head_dim = 256;
  d->rotary_dim = 64;
  d->rope_theta = 1.0e7f;
  d->gdn_k_heads = 16;
  d->gdn_v_heads = 48;
  d->gdn_dk = 128;
  d->gdn_dv = 128;
  d->conv_kernel = 4;
  d->group_size = 64;
  d->eps = 1e-6f;
  d->max_ctx = 4608;
  d->max_rows = 128;
  d->max_seqs = 1;
  d->comm_timeout_ms = 0;
  d->resident_weight_bytes = 0;
}

static int validate_dims(const iam_dims& d, int world) {
  using iam::fail;
  IAM_CHECK(d.hidden > 0 && d.hidden % 64 == 0, "dims: hidden must be a multiple of 64");
  IAM_CHECK(d.group_size == 64 && d.conv_kernel == 4, "dims: group_size 64 and conv_kernel 4 required");
  IAM_CHECK(d.gdn_dk == 128 && d.gdn_dv == 128 && d.head_dim == 256, "dims: GDN head 128 and attention head 256 required");
  IAM_CHECK(d.rotary_dim % 8 == 0 && d.rotary_dim <= d.head_dim, "dims: rotary_dim must be a multiple of 8");
  IAM_CHECK(d.full_attn_interval >= 1 && d.n_layers >= 1, "dims: layers");
  IAM_CHECK(world >= 1 && d.gdn_k_heads % world == 0 && d.gdn_v_heads % world == 0 &&
                d.gdn_v_heads % d.gdn_k_heads == 0,
            "dims: GDN heads must split evenly over the GPUs");
  IAM_CHECK(d.n_heads % world == 0 && d.n_heads % d.n_kv_heads == 0, "dims: query heads must split evenly");
  IAM_CHECK(world <= d.n_kv_heads ? d.n_kv_heads % world == 0 : world % d.n_kv_heads == 0,
            "dims: KV heads split or replicate evenly");
  IAM_CHECK((d.n_heads / world) / std::max(1, world <= d.n_kv_heads ? d.n_kv_heads / world : 1) <= 8,
            "dims: at most 8 query heads per KV head per GPU");
  IAM_CHECK(d.intermediate % (64 * world) == 0, "dims: intermediate / world must be a multiple of 64");
  IAM_CHECK(d.vocab % (16 * world) == 0, "dims: vocab / world must be a multiple of 16");
  IAM_CHECK(d.max_rows >= 1 && d.max_rows <= 4096, "dims: max_rows in 1..4096");
  IAM_CHECK(d.max_seqs >= 1 && d.max_seqs <= d.max_rows && d.max_seqs <= 65535, "dims: max_seqs in 1..max_rows");
  IAM_CHECK(d.max_ctx >= d.max_rows, "dims: max_ctx");
  return IAM_OK;
}

extern "C" int iam_tp_shard_of(const iam_dims* dims, int rank, int world, iam_tp_shard* out) {
  IAM_CHECK(dims && out, "iam_tp_shard_of: null argument");
  const int r = validate_dims(*dims, world);
  if (r != IAM_OK) return r;
  IAM_CHECK(rank >= 0 && rank < world, "iam_tp_shard_of: rank out of range");
  const iam_dims& d = *dims;
  iam_tp_shard s;
  s.gdn_k_heads = d.gdn_k_heads / world;
  s.gdn_k_head0 = rank * s.gdn_k_heads;
  s.gdn_v_heads = d.gdn_v_heads / world;
  s.gdn_v_head0 = rank * s.gdn_v_heads;
  s.q_heads = d.n_heads / world;
  s.q_head0 = rank * s.q_heads;
  if (world <= d.n_kv_heads) {
    s.kv_heads = d.n_kv_heads / world;
    s.kv_head0 = rank * s.kv_heads;
  } else {
    s.kv_heads = 1;
    s.kv_head0 = rank / (world / d.n_kv_heads);
  }
  s.inter = d.intermediate / world;
  s.inter0 = rank * s.inter;
  s.vocab = d.vocab / world;
  s.vocab0 = rank * s.vocab;
  *out = s;
  return IAM_OK;
}

extern "C" int iam_nccl_unique_id(void* id128) { return iam::nccl_unique_id(id128); }

static int comm_timeout_ms(const iam::EngineImpl& e) { return e.d.comm_timeout_ms > 0 ? e.d.comm_timeout_ms : 120000; }
static int sync_step(iam::EngineImpl& e, const char* what);

// Maps every rank's receive area for the row-parallel sums into every rank
// (CUDA IPC; the handles travel through the communicator, and so do the
// verdicts: either every rank could map every peer and all use the
// peer-memory sums, or none does and the NCCL all-reduce stays).
// IAM_TP_P2P=0 keeps the NCCL all-reduce.
static int tp_p2p_init(iam::EngineImpl& e) {
  using namespace iam;
  const char* env = std::getenv("IAM_TP_P2P");
  const bool want = !(env && env[0] == '0') && e.world <= kQmmMaxPeers;
  const size_t R = static_cast<size_t>(e.d.max_rows), H = static_cast<size_t>(e.d.hidden);
  e.tp_tiles = ceil_div(e.d.hidden, kQpRows);
  e.tp_ctr_off = (2 * static_cast<size_t>(e.world) * R * H * sizeof(float) + 255) / 256 * 256;
  const size_t bytes = e.tp_ctr_off + 2 * static_cast<size_t>(e.tp_tiles) * sizeof(int);
  constexpr int kW = 9;  // a rank's words: its 64-byte handle and a verdict
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  bool ok = want;
  cudaIpcMemHandle_t h{};
  if (ok && (cudaMalloc(&e.tp_area, bytes) != cudaSuccess || cudaMemsetAsync(e.tp_area, 0, bytes, e.stream) != cudaSuccess ||
             cudaIpcGetMemHandle(&h, e.tp_area) != cudaSuccess)) {
    cudaGetLastError();
    ok = false;
  }
  std::vector<unsigned long long> hx(static_cast<size_t>(e.world) * kW, 0ull);
  std::memcpy(&hx[static_cast<size_t>(e.rank) * kW], &h, sizeof(h));
  hx[static_cast<size_t>(e.rank) * kW + 8] = ok ? 1ull : 0ull;
  unsigned long long* dx = nullptr;
  E_CUDA(cudaMalloc(&dx, hx.size() * sizeof(unsigned long long)));
  auto gather = [&]() -> int {
    E_CUDA(cudaMemcpyAsync(dx, hx.data(), hx.size() * 8, cudaMemcpyHostToDevice, e.stream));
    unsigned long long* mine = dx + static_cast<size_t>(e.rank) * kW;
    E_RUN(nccl_allgather_u64(e.comm, mine, dx, kW, e.stream));
    E_RUN(sync_step(e, "iam_create: exchanging peer-memory handles"));
    E_CUDA(cudaMemcpy(hx.data(), dx, hx.size() * 8, cudaMemcpyDeviceToHost));
    return IAM_OK;
  };
  int r = gather();
  bool all = r == IAM_OK;
  for (int q = 0; all && q < e.world; ++q) all = hx[static_cast<size_t>(q) * kW + 8] == 1ull;
  if (all) {
    for (int q = 0; q < e.world; ++q) {
      if (q == e.rank) {
        e.tp_peer[q] = e.tp_area;
        continue;
      }
      cudaIpcMemHandle_t ph;
      std::memcpy(&ph, &hx[static_cast<size_t>(q) * kW], sizeof(ph));
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, ph, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        ok = false;
        break;
      }
      e.tp_peer[q] = static_cast<char*>(p);
    }
    hx[static_cast<size_t>(e.rank) * kW + 8] = ok ? 1ull : 0ull;
    r = gather();
    for (int q = 0; r == IAM_OK && q < e.world; ++q) all = all && hx[static_cast<size_t>(q) * kW + 8] == 1ull;
    all = all && r == IAM_OK;
  }
  cudaFree(dx);
  if (!all) {
    for (int q = 0; q < e.world; ++q)
      if (q != e.rank && e.tp_peer[q]) cudaIpcCloseMemHandle(e.tp_peer[q]);
    for (char*& p : e.tp_peer) p = nullptr;
    if (e.tp_area) cudaFree(e.tp_area);
    e.tp_area = nullptr;
  }
  e.tp_p2p = all;
  return r;
}

extern "C" int iam_create(const iam_dims* dims, int device, int rank, int world, const void* nccl_id,
                          iam_engine** out) {
  using namespace iam;
  IAM_CHECK(dims && out, "iam_create: null argument");
  *out = nullptr;
  int r = validate_dims(*dims, world);
  if (r != IAM_OK) return r;
  IAM_CHECK(rank >= 0 && rank < world, "iam_create: rank out of range");
  IAM_CHECK(world == 1 || nccl_id, "iam_create: an NCCL id is required for world > 1");
  IAM_CUDA(cudaSetDevice(device));
  auto* eng = new iam_engine();
  EngineImpl& e = eng->impl;
  e.d = *dims;
  e.device = device;
  e.rank = rank;
  e.world = world;
  const char* pdl = std::getenv("IAM_PDL");
  e.pdl = !(pdl && pdl[0] == '0');
  cudaError_t ce = cudaStreamCreateWithFlags(&e.stream, cudaStreamNonBlocking);
  if (ce != cudaSuccess) {
    delete eng;
    return cuda_status(ce, "cudaStreamCreate");
  }
  r = build_registry(e);
  if (r == IAM_OK) r = gdn_init_attrs();  // kernel attributes before any graph capture
  if (r == IAM_OK) r = attn_init_attrs();
  if (r == IAM_OK) r = alloc_all(e);
  if (r == IAM_OK && world > 1) r = nccl_init(&e.comm, nccl_id, rank, world, comm_timeout_ms(e));
  if (r == IAM_OK && world > 1) r = tp_p2p_init(e);
  if (r != IAM_OK) {
    iam_destroy(eng);
    return r;
  }
  *out = eng;
  return IAM_OK;
}

extern "C" void iam_destroy(iam_engine* eng) {
  if (!eng) return;
  EngineImpl& e = eng->impl;
  cudaSetDevice(e.device);
  if (e.stream) cudaStreamSynchronize(e.stream);
  for (auto& kv : e.graphs) cudaGraphExecDestroy(kv.second);
  e.graphs.clear();
  for (auto& kv : e.bgraphs) cudaGraphExecDestroy(kv.second);
  e.bgraphs.clear();
  if (e.comm) iam::nccl_destroy(e.comm);
  for (int q = 0; q < e.world && q < iam::kQmmMaxPeers; ++q)
    if (q != e.rank && e.tp_peer[q]) cudaIpcCloseMemHandle(e.tp_peer[q]);
  if (e.tp_area) cudaFree(e.tp_area);
  if (e.pf_stream) cudaStreamSynchronize(e.pf_stream);
  for (int s = 0; s < 2; ++s) {
    if (e.slot[s]) cudaFree(e.slot[s]);
    if (e.pf_ready[s]) cudaEventDestroy(e.pf_ready[s]);
    if (e.pf_free[s]) cudaEventDestroy(e.pf_free[s]);
  }
  if (e.pf_start) cudaEventDestroy(e.pf_start);
  if (e.pf_stream) cudaStreamDestroy(e.pf_stream);
  if (e.hpool) cudaFreeHost(e.hpool);
  if (e.hpacked) cudaFreeHost(e.hpacked);
  void* bufs[] = {e.pool, e.ppool, e.S, e.conv[0], e.conv[1], e.kc, e.vc, e.d_parity, e.hidden, e.resid, e.normed, e.inproj,
                  e.mid, e.mlp_h, e.q_buf, e.part_o, e.part_ml, e.red32, e.keys, e.best, e.rope_cs, e.d_in, e.d_out,
                  e.d_err, e.qws, e.qctr, e.gin, e.d_bin, e.d_bout};
  for (void* p : bufs)
    if (p) cudaFree(p);
  for (void* p : {static_cast<void*>(e.h_in), static_cast<void*>(e.h_out), static_cast<void*>(e.h_bin),
                  static_cast<void*>(e.h_bout), static_cast<void*>(e.h_err)})
    if (p) cudaFreeHost(p);
  if (e.stream) cudaStreamDestroy(e.stream);
  delete eng;
}

extern "C" const char* iam_engine_error(const iam_engine* eng) { return eng ? eng->impl.err.c_str() : ""; }

extern "C" int iam_load_tensor(iam_engine* eng, const char* name, const void* host_ptr, size_t bytes) {
  using namespace iam;
  IAM_CHECK(eng && name && host_ptr, "iam_load_tensor: null argument");
  EngineImpl& e = eng->impl;
  auto it = e.by_name.find(name);
  if (it == e.by_name.end()) return e.setf(IAM_EINVAL, std::string("iam_load_tensor: unknown tensor ") + name);
  const TensorRec& t = e.tensors[it->second];
  const size_t full = static_cast<size_t>(t.full_rows) * t.full_cols * t.esize;
  if (bytes != full)
    return e.setf(IAM_EINVAL, std::string("iam_load_tensor: ") + name + " expects " + std::to_string(full) + " bytes");
  E_CUDA(cudaSetDevice(e.device));
  const char* src = static_cast<const char*>(host_ptr);
  char* dst = static_cast<char*>(t.ptr);
  const size_t width = static_cast<size_t>(t.shard.col1 - t.shard.col0) * t.esize;
  const size_t pitch = static_cast<size_t>(t.full_cols) * t.esize;
  for (auto& rr : t.shard.rows) {
    const size_t nrows = static_cast<size_t>(rr.second - rr.first);
    E_CUDA(cudaMemcpy2DAsync(dst, width, src + rr.first * pitch + t.shard.col0 * t.esize, pitch, width, nrows,
                             cudaMemcpyDefault, e.stream));  // dst: device, or pinned host for a streamed layer
    dst += nrows * width;
  }
  E_CUDA(cudaStreamSynchronize(e.stream));
  if (t.kind == Kind::kQ4Words || t.kind == Kind::kQ4Scales || t.kind == Kind::kQ4Biases) e.packed_dirty = true;
  return IAM_OK;
}

// ---------------------------------------------------------------- checkpoints
namespace iam {
namespace {

const char* kind_dtype(Kind k) {
  switch (k) {
    case Kind::kQ4Words: return "U32";
    case Kind::kF32: return "F32";
    default: return "BF16";
  }
}

// Where each of the engine's tensors comes from in a checkpoint.
struct CkptPlan {
  struct Item {
    const TensorRec* t;
    const StTensor* src;
    bool to_f32;  // a bf16 tensor read into an fp32 one (A_log stored as bf16)
  };
  std::vector<Item> items;
  bool embed_q4 = false;  // 4-bit embedding: dequantized into the bf16 table at load
  const StTensor *ew = nullptr, *es = nullptr, *eb = nullptr;
  bool tied = false;  // lm_head read from the 4-bit embedding
  size_t bytes = 0;
  std::vector<std::string> problems;
};

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

void plan_checkpoint(const EngineImpl& e, const StCheckpoint& ck, CkptPlan& plan) {
  auto find = [&](const std::string& n) -> const StTensor* {
    auto it = ck.tensors.find(n);
    return it == ck.tensors.end() ? nullptr : &it->second;
  };
  // embedding: a bf16 table, or the reference's 4-bit one (embed_lookup_bf16,
  // full_forward.swift:112-133) dequantized once into the table
  const int64_t V = e.d.vocab, H = e.d.hidden, G = H / e.d.group_size;
  if (const StTensor* w = find("model.embed_tokens.weight")) {
    if (w->dtype == "U32") {
      plan.ew = w;
      plan.es = find("model.embed_tokens.scales");
      plan.eb = find("model.embed_tokens.biases");
      const size_t wb = static_cast<size_t>(V * H / 2), sb = static_cast<size_t>(V * G * 2);
      if (w->bytes() != wb || !plan.es || !plan.eb || plan.es->dtype != "BF16" || plan.eb->dtype != "BF16" ||
          plan.es->bytes() != sb || plan.eb->bytes() != sb)
        plan.problems.push_back("model.embed_tokens: a 4-bit embedding needs weight U32 [" + std::to_string(V) + ", " +
                                std::to_string(H / 8) + "] with BF16 scales and biases [" + std::to_string(V) + ", " +
                                std::to_string(G) + "]");
      else
        plan.embed_q4 = true;
    }
  }
  for (const TensorRec& t : e.tensors) {
    const size_t full = static_cast<size_t>(t.full_rows) * t.full_cols * t.esize;
    if (t.name == "model.embed_tokens.weight" && plan.embed_q4) {
      plan.bytes += plan.ew->bytes() + plan.es->bytes() + plan.eb->bytes();
      continue;
    }
    const StTensor* src = find(t.name);
    if (!src && t.name.compare(0, 8, "lm_head.") == 0 && plan.embed_q4) {
      src = find("model.embed_tokens." + t.name.substr(8));  // tied output embedding
      if (src) plan.tied = true;
    }
    if (!src) {
      plan.problems.push_back("missing " + t.name);
      continue;
    }
    bool to_f32 = false;
    if (src->dtype != kind_dtype(t.kind)) {
      if (t.kind == Kind::kF32 && src->dtype == "BF16" && src->bytes() * 2 == full) {
        to_f32 = true;
      } else {
        plan.problems.push_back(t.name + ": dtype " + src->dtype + ", expected " + kind_dtype(t.kind));
        continue;
      }
    }
    if (!to_f32 && src->bytes() != full) {
      plan.problems.push_back(t.name + ": shape " + shape_str(src->shape) + " " + src->dtype + " (" +
                              std::to_string(src->bytes()) + " bytes), expected [" + std::to_string(t.full_rows) +
                              ", " + std::to_string(t.full_cols) + "] (" + std::to_string(full) + " bytes)");
      continue;
    }
    if (t.full_rows > 1 && src->shape.size() >= 2 && src->shape[0] != t.full_rows) {
      plan.problems.push_back(t.name + ": shape " + shape_str(src->shape) + ", expected " +
                              std::to_string(t.full_rows) + " rows");
      continue;
    }
    plan.items.push_back({&t, src, to_f32});
    plan.bytes += src->bytes();
  }
  // decoder tensors the engine has no place for: a different architecture
  for (const auto& kv : ck.tensors) {
    if (e.by_name.count(kv.first)) continue;
    if (plan.embed_q4 && (kv.first == "model.embed_tokens.scales" || kv.first == "model.embed_tokens.biases")) continue;
    plan.problems.push_back("unused tensor " + kv.second.name);
  }
}

// Host -> device copies staged through two pinned buffers: the gather from
// the mapped file into one overlaps the DMA out of the other.
struct Staging {
  static constexpr size_t kBytes = 32u << 20;
  unsigned char* buf[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool used[2] = {false, false};
  int next = 0;
  cudaStream_t st = nullptr;
  ~Staging() {
    if (st) cudaStreamSynchronize(st);
    for (int i = 0; i < 2; ++i) {
      if (buf[i]) cudaFreeHost(buf[i]);
      if (ev[i]) cudaEventDestroy(ev[i]);
    }
  }
  cudaError_t init(cudaStream_t s) {
    st = s;
    for (int i = 0; i < 2; ++i) {
      cudaError_t r = cudaHostAlloc(reinterpret_cast<void**>(&buf[i]), kBytes, cudaHostAllocDefault);
      if (r != cudaSuccess) return r;
      r = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
      if (r != cudaSuccess) return r;
    }
    return cudaSuccess;
  }
  // the next free buffer
  cudaError_t take(unsigned char** out) {
    const int b = next;
    next ^= 1;
    if (used[b]) {
      const cudaError_t r = cudaEventSynchronize(ev[b]);
      if (r != cudaSuccess) return r;
    }
    used[b] = true;
    *out = buf[b];
    cur = b;
    return cudaSuccess;
  }
  cudaError_t send(void* dst, size_t n) {
    cudaError_t r = cudaMemcpyAsync(dst, buf[cur], n, cudaMemcpyDefault, st);  // dst may be pinned host memory
    if (r == cudaSuccess) r = cudaEventRecord(ev[cur], st);
    return r;
  }
  int cur = 0;
};

// rows [r0, r1) x columns [c0, c1) (bytes) of a row-major host matrix with
// `pitch` bytes a row, to contiguous device memory at dst
int stage_rows(EngineImpl& e, Staging& sg, const unsigned char* src, size_t pitch, int64_t r0, int64_t r1, size_t c0,
               size_t width, unsigned char* dst) {
  const int64_t per = std::max<int64_t>(1, static_cast<int64_t>(Staging::kBytes / width));
  for (int64_t r = r0; r < r1; r += per) {
    const int64_t n = std::min(per, r1 - r);
    unsigned char* b = nullptr;
    E_CUDA(sg.take(&b));
    if (width == pitch) {
      std::memcpy(b, src + r * pitch, static_cast<size_t>(n) * pitch);
    } else {
      for (int64_t i = 0; i < n; ++i) std::memcpy(b + i * width, src + (r + i) * pitch + c0, width);
    }
    E_CUDA(sg.send(dst, static_cast<size_t>(n) * width));
    dst += static_cast<size_t>(n) * width;
  }
  return IAM_OK;
}

// one tensor's shard, as iam_load_tensor places it
int stage_tensor(EngineImpl& e, Staging& sg, const TensorRec& t, const unsigned char* src) {
  unsigned char* dst = static_cast<unsigned char*>(t.ptr);
  const size_t width = static_cast<size_t>(t.shard.col1 - t.shard.col0) * t.esize;
  const size_t pitch = static_cast<size_t>(t.full_cols) * t.esize;
  for (auto& rr : t.shard.rows) {
    E_RUN(stage_rows(e, sg, src, pitch, rr.first, rr.second, static_cast<size_t>(t.shard.col0) * t.esize, width, dst));
    dst += static_cast<size_t>(rr.second - rr.first) * width;
  }
  return IAM_OK;
}

int load_checkpoint(EngineImpl& e, const StCheckpoint& ck, const CkptPlan& plan) {
  E_CUDA(cudaSetDevice(e.device));
  Staging sg;
  E_CUDA(sg.init(e.stream));
  for (const auto& it : plan.items) {
    const unsigned char* src = static_cast<const unsigned char*>(ck.data(*it.src));
    if (!it.to_f32) {
      E_RUN(stage_tensor(e, sg, *it.t, src));
      continue;
    }
    const size_t n = it.src->bytes() / 2;
    std::vector<float> f(n);
    for (size_t i = 0; i < n; ++i) {
      uint16_t h;
      std::memcpy(&h, src + 2 * i, 2);
      const uint32_t u = static_cast<uint32_t>(h) << 16;
      std::memcpy(&f[i], &u, 4);
    }
    E_RUN(stage_tensor(e, sg, *it.t, reinterpret_cast<const unsigned char*>(f.data())));
    E_CUDA(cudaStreamSynchronize(e.stream));  // f is released below
  }
  if (plan.embed_q4) {
    // the 4-bit table through device scratch, a block of rows at a time,
    // dequantized by the reference's embed_lookup_bf16 arithmetic
    const int64_t V = e.d.vocab, H = e.d.hidden, G = H / e.d.group_size;
    const int64_t rows = 8192;
    struct Tmp {
      void* p[4] = {nullptr, nullptr, nullptr, nullptr};
      ~Tmp() {
        for (void* q : p)
          if (q) cudaFree(q);
      }
    } tmp;
    E_CUDA(cudaMalloc(&tmp.p[0], static_cast<size_t>(rows * H / 2)));
    E_CUDA(cudaMalloc(&tmp.p[1], static_cast<size_t>(rows * G * 2)));
    E_CUDA(cudaMalloc(&tmp.p[2], static_cast<size_t>(rows * G * 2)));
    E_CUDA(cudaMalloc(&tmp.p[3], static_cast<size_t>(rows * 4)));
    std::vector<int32_t> ids(static_cast<size_t>(rows));
    for (int64_t i = 0; i < rows; ++i) ids[static_cast<size_t>(i)] = static_cast<int32_t>(i);
    E_CUDA(cudaMemcpy(tmp.p[3], ids.data(), ids.size() * 4, cudaMemcpyHostToDevice));
    const unsigned char* w = static_cast<const unsigned char*>(ck.data(*plan.ew));
    const unsigned char* sc = static_cast<const unsigned char*>(ck.data(*plan.es));
    const unsigned char* bi = static_cast<const unsigned char*>(ck.data(*plan.eb));
    for (int64_t r = 0; r < V; r += rows) {
      const int64_t n = std::min(rows, V - r);
      E_RUN(stage_rows(e, sg, w, H / 2, r, r + n, 0, H / 2, static_cast<unsigned char*>(tmp.p[0])));
      E_RUN(stage_rows(e, sg, sc, G * 2, r, r + n, 0, G * 2, static_cast<unsigned char*>(tmp.p[1])));
      E_RUN(stage_rows(e, sg, bi, G * 2, r, r + n, 0, G * 2, static_cast<unsigned char*>(tmp.p[2])));
      const int rc = iam_embed_lookup_q4(static_cast<const uint32_t*>(tmp.p[0]), static_cast<const uint16_t*>(tmp.p[1]),
                                         static_cast<const uint16_t*>(tmp.p[2]), static_cast<const int32_t*>(tmp.p[3]),
                                         e.embed + static_cast<size_t>(r) * H, static_cast<int>(n), static_cast<int>(H),
                                         e.d.group_size, e.stream);
      if (rc != IAM_OK) return e.setf(rc, iam_last_error());
      E_CUDA(cudaStreamSynchronize(e.stream));  // the scratch is reused by the next block
    }
  }
  E_CUDA(cudaStreamSynchronize(e.stream));
  e.packed_dirty = true;
  return IAM_OK;
}

std::vector<std::string> path_list(const char* const* paths, int n) {
  std::vector<std::string> v;
  for (int i = 0; i < n; ++i) v.push_back(paths[i] ? paths[i] : "");
  return v;
}

std::string plan_summary(const CkptPlan& plan, const StCheckpoint& ck) {
  std::string r = std::to_string(plan.items.size() + (plan.embed_q4 ? 1 : 0)) + " tensors, " +
                  std::to_string(plan.bytes) + " bytes from " + std::to_string(ck.files.size()) + " file(s); embedding " +
                  (plan.embed_q4 ? "4-bit (dequantized at load)" : "bf16") + "; lm_head " +
                  (plan.tied ? "tied to the embedding" : "own") + "; " + std::to_string(ck.ignored.size()) +
                  " non-decoder tensors ignored";
  for (const auto& p : plan.problems) r += "\n" + p;
  return r;
}

}  // namespace
}  // namespace iam

extern "C" int iam_check_safetensors(const iam_dims* dims, const char* const* paths, int n_paths, char* report,
                                     size_t report_len) {
  using namespace iam;
  IAM_CHECK(dims && paths && n_paths > 0, "iam_check_safetensors: bad arguments");
  int r = validate_dims(*dims, 1);
  if (r != IAM_OK) return r;
  EngineImpl e;
  e.d = *dims;
  r = build_registry(e);
  if (r != IAM_OK) return fail(r, e.err);
  StCheckpoint ck;
  std::string err;
  std::string text;
  CkptPlan plan;
  if (!st_open(path_list(paths, n_paths), ck, err)) {
    text = err;
    r = fail(IAM_EINVAL, err);
  } else {
    plan_checkpoint(e, ck, plan);
    text = plan_summary(plan, ck);
    r = plan.problems.empty() ? IAM_OK : fail(IAM_EINVAL, "checkpoint: " + plan.problems.front());
  }
  if (report && report_len) {
    std::strncpy(report, text.c_str(), report_len - 1);
    report[report_len - 1] = '\0';
  }
  return r;
}

extern "C" int iam_load_safetensors(iam_engine* eng, const char* const* paths, int n_paths) {
  using namespace iam;
  IAM_CHECK(eng && paths && n_paths > 0, "iam_load_safetensors: bad arguments");
  EngineImpl& e = eng->impl;
  StCheckpoint ck;
  std::string err;
  if (!st_open(path_list(paths, n_paths), ck, err)) return e.setf(IAM_EINVAL, err);
  CkptPlan plan;
  plan_checkpoint(e, ck, plan);
  if (!plan.problems.empty()) {
    std::string m = "checkpoint does not match the model (" + std::to_string(plan.problems.size()) + " problems):";
    for (size_t i = 0; i < plan.problems.size() && i < 8; ++i) m += "\n  " + plan.problems[i];
    return e.setf(IAM_EINVAL, m);
  }
  return load_checkpoint(e, ck, plan);
}

extern "C" int iam_read_tensor(iam_engine* eng, const char* name, void* host_ptr, size_t bytes) {
  using namespace iam;
  IAM_CHECK(eng && name && host_ptr, "iam_read_tensor: null argument");
  EngineImpl& e = eng->impl;
  E_CUDA(cudaSetDevice(e.device));
  E_CUDA(cudaStreamSynchronize(e.stream));
  const std::string n(name);
  auto it = e.by_name.find(n);
  if (it != e.by_name.end()) {
    if (bytes > e.tensors[it->second].bytes())
      return e.setf(IAM_EINVAL, "iam_read_tensor: more bytes requested than the tensor holds");
    E_CUDA(cudaMemcpy(host_ptr, e.tensors[it->second].ptr, bytes, cudaMemcpyDefault));
    return IAM_OK;
  }
  const bool isS = n.rfind("state.S.", 0) == 0, isC = n.rfind("state.conv.", 0) == 0;
  const bool isK = n.rfind("state.k_cache.", 0) == 0, isV = n.rfind("state.v_cache.", 0) == 0;
  if (!(isS || isC || isK || isV)) return e.setf(IAM_EINVAL, std::string("iam_read_tensor: unknown tensor ") + n);
  const int li = std::atoi(n.substr(n.rfind('.') + 1).c_str());
  if (li < 0 || li >= e.d.n_layers) return e.setf(IAM_EINVAL, "iam_read_tensor: layer out of range");
  const Layer& L = e.layers[li];
  if ((isS || isC) == L.attn) return e.setf(IAM_EINVAL, std::string("iam_read_tensor: layer has no ") + n);
  // every slot, slot after slot; the GDN state and conv window of a slot from
  // the copy its parity word names
  size_t per = 0;
  std::vector<int> par(static_cast<size_t>(e.max_seqs), 0);
  if (isS || isC) E_CUDA(cudaMemcpy(par.data(), e.d_parity, sizeof(int) * e.max_seqs, cudaMemcpyDeviceToHost));
  if (isS) per = e.s_per * 4;
  else if (isC) per = static_cast<size_t>(3) * e.conv_l * 2;
  else per = static_cast<size_t>(e.d.max_ctx) * e.hkv_l * e.d.head_dim * 2;
  if (bytes > per * e.max_seqs) return e.setf(IAM_EINVAL, "iam_read_tensor: more bytes requested than the tensor holds");
  char* dst = static_cast<char*>(host_ptr);
  for (int q = 0; q < e.max_seqs && bytes > 0; ++q) {
    const char* src = nullptr;
    if (isS)
      src = reinterpret_cast<const char*>(e.S + (par[q] ? e.s_half : 0) +
                                          (static_cast<size_t>(L.idx) * e.max_seqs + q) * e.s_per);
    else if (isC)
      src = reinterpret_cast<const char*>(e.conv[par[q]] +
                                          (static_cast<size_t>(L.idx) * e.max_seqs + q) * 3 * e.conv_l);
    else
      src = reinterpret_cast<const char*>((isK ? e.kc : e.vc) +
                                          (static_cast<size_t>(L.idx) * e.max_seqs + q) * e.d.max_ctx * e.hkv_l *
                                              e.d.head_dim);
    const size_t nb = std::min(bytes, per);
    E_CUDA(cudaMemcpy(dst, src, nb, cudaMemcpyDeviceToHost));
    dst += nb;
    bytes -= nb;
  }
  return IAM_OK;
}

extern "C" int iam_init_synthetic(iam_engine* eng, uint64_t seed) {
  using namespace iam;
  IAM_CHECK(eng, "iam_init_synthetic: null engine");
  EngineImpl& e = eng->impl;
  E_CUDA(cudaSetDevice(e.device));
  for (const TensorRec& t : e.tensors) E_RUN(synth_tensor(e, t, seed));
  E_CUDA(cudaStreamSynchronize(e.stream));
  e.packed_dirty = true;
  return IAM_OK;
}

extern "C" int iam_state_reset(iam_engine* eng) {
  using namespace iam;
  IAM_CHECK(eng, "iam_state_reset: null engine");
  EngineImpl& e = eng->impl;
  E_CUDA(cudaSetDevice(e.device));
  const size_t slots = static_cast<size_t>(e.max_seqs);
  if (e.s_half) E_CUDA(cudaMemsetAsync(e.S, 0, 2 * e.s_half * sizeof(float), e.stream));
  for (int i = 0; i < 2; ++i)
    if (e.n_gdn)
      E_CUDA(cudaMemsetAsync(e.conv[i], 0, static_cast<size_t>(e.n_gdn) * slots * 3 * e.conv_l * 2, e.stream));
  const size_t kv = static_cast<size_t>(e.n_attn) * slots * e.d.max_ctx * e.hkv_l * e.d.head_dim * 2;
  if (kv) {
    E_CUDA(cudaMemsetAsync(e.kc, 0, kv, e.stream));
    E_CUDA(cudaMemsetAsync(e.vc, 0, kv, e.stream));
  }
  E_CUDA(cudaMemsetAsync(e.d_parity, 0, slots * sizeof(int), e.stream));
  E_CUDA(cudaMemsetAsync(e.d_bin, 0, slots * sizeof(int32_t), e.stream));
  E_CUDA(cudaStreamSynchronize(e.stream));
  e.last_K = 0;
  return IAM_OK;
}

// Synthetic-stream name of a state tensor of sequence slot q: slot 0 keeps
// the single-sequence names, slot q > 0 appends ".s<q>".
static std::string state_name(const std::string& base, int q) {
  return q ? base + ".s" + std::to_string(q) : base;
}

extern "C" int iam_state_init(iam_engine* eng, uint64_t seed, int ctx) {
  using namespace iam;
  IAM_CHECK(eng, "iam_state_init: null engine");
  EngineImpl& e = eng->impl;
  IAM_CHECK(ctx >= 0 && ctx <= e.d.max_ctx, "iam_state_init: ctx out of range");
  int r = iam_state_reset(eng);
  if (r != IAM_OK || seed == 0) return r;
  const iam_dims& d = e.d;
  const int gd = d.gdn_dk;
  const int key_dim = d.gdn_k_heads * gd;
  const int conv_dim = 2 * key_dim + d.gdn_v_heads * d.gdn_dv;
  const std::pair<int, int> cr[3] = {{e.k0 * gd, e.gk_l * gd},
                                     {key_dim + e.k0 * gd, e.gk_l * gd},
                                     {2 * key_dim + e.v0 * d.gdn_dv, e.gv_l * d.gdn_dv}};
  for (const Layer& L : e.layers) {
    const int li = static_cast<int>(&L - e.layers.data());
    const std::string ls = std::to_string(li);
    for (int q = 0; q < e.max_seqs; ++q) {
      const size_t slot = static_cast<size_t>(L.idx) * e.max_seqs + q;
      if (L.attn) {
        if (ctx == 0) continue;
        for (int kvsel = 0; kvsel < 2; ++kvsel) {
          SynthJob j = {};
          j.stream = synth_stream(seed, state_name(std::string(kvsel ? "state.v_cache." : "state.k_cache.") + ls, q).c_str());
          j.kind = SYN_NORMAL_BF16;
          j.p0 = 1.0f;
          j.full_cols = static_cast<uint64_t>(d.n_kv_heads) * d.head_dim;
          j.row0 = 0;
          j.rows = static_cast<uint64_t>(ctx);
          j.col0 = static_cast<uint64_t>(e.kv0) * d.head_dim;
          j.width = static_cast<uint64_t>(e.hkv_l) * d.head_dim;
          j.dst = (kvsel ? e.vc : e.kc) + slot * d.max_ctx * e.hkv_l * d.head_dim;
          E_RUN(synth_fill(j, e.stream));
        }
      } else {
        SynthJob j = {};
        j.stream = synth_stream(seed, state_name("state.conv." + ls, q).c_str());
        j.kind = SYN_NORMAL_BF16;
        j.p0 = 1.0f;
        j.full_cols = static_cast<uint64_t>(conv_dim);
        j.row0 = 0;
        j.rows = 3;
        j.dst_ld = static_cast<uint64_t>(e.conv_l);
        int local = 0;
        for (auto& c : cr) {
          j.col0 = static_cast<uint64_t>(c.first);
          j.width = static_cast<uint64_t>(c.second);
          j.dst = e.conv[0] + slot * 3 * e.conv_l + local;
          E_RUN(synth_fill(j, e.stream));
          local += c.second;
        }
        SynthJob sj = {};
        sj.stream = synth_stream(seed, state_name("state.S." + ls, q).c_str());
        sj.kind = SYN_NORMAL_F32;
        sj.p0 = 0.01f;
        sj.full_cols = static_cast<uint64_t>(d.gdn_dk) * d.gdn_dv;
        sj.row0 = static_cast<uint64_t>(e.v0);
        sj.rows = static_cast<uint64_t>(e.gv_l);
        sj.col0 = 0;
        sj.width = sj.full_cols;
        sj.dst = e.S + slot * e.s_per;
        E_RUN(synth_fill(sj, e.stream));
      }
    }
  }
  E_CUDA(cudaStreamSynchronize(e.stream));
  return IAM_OK;
}

// After a synchronous step: the device error word (a bounded wait that gave
// up, a token id out of range) becomes the call's status; the word is
// cleared for the next step.  h_err was filled by a copy enqueued after the
// step and before the synchronisation.
static int device_status(iam::EngineImpl& e, const char* what) {
  using namespace iam;
  const int st = *e.h_err;
  if (st == IAM_OK) return IAM_OK;
  *e.h_err = 0;
  E_CUDA(cudaMemsetAsync(e.d_err, 0, sizeof(int), e.stream));
  E_CUDA(cudaStreamSynchronize(e.stream));
  if (st == IAM_ETIMEOUT && e.world > 1 && e.comm) {
    // a peer-memory sum gave up: the ranks' arrival counters no longer agree,
    // so the engine refuses further steps (like an aborted communicator)
    nccl_abort(e.comm);
    e.comm = nullptr;
  }
  return e.setf(st, std::string(what) + ": device-side error " + iam_status_string(st) +
                        (st == IAM_ETIMEOUT ? " (a bounded wait inside a kernel gave up)" : ""));
}

// Waits for the engine stream.  With one GPU a plain synchronisation; across
// GPUs the host polls the stream, the communicator's asynchronous error and a
// deadline (comm_timeout_ms): a peer that failed or left makes the call end
// in IAM_ENCCL / IAM_ETIMEOUT, with the communicator aborted (its kernels in
// flight return) instead of a hang.  After that the engine refuses steps.
static int sync_step(iam::EngineImpl& e, const char* what) {
  using namespace iam;
  if (e.world == 1 || !e.comm) {
    E_CUDA(cudaStreamSynchronize(e.stream));
    return IAM_OK;
  }
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(comm_timeout_ms(e));
  for (;;) {
    const cudaError_t q = cudaStreamQuery(e.stream);
    if (q == cudaSuccess) return IAM_OK;
    if (q != cudaErrorNotReady) E_CUDA(q);
    int st = nccl_async_status(e.comm);
    if (st == IAM_OK && std::chrono::steady_clock::now() > deadline) st = IAM_ETIMEOUT;
    if (st != IAM_OK) {
      nccl_abort(e.comm);
      e.comm = nullptr;
      cudaStreamSynchronize(e.stream);  // the aborted collectives return
      return e.setf(st, std::string(what) + (st == IAM_ETIMEOUT ? ": the step's collectives did not finish within "
                                                                  "comm_timeout_ms; communicator aborted"
                                                                : ": communicator failed and was aborted"));
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

static int verify_common(iam_engine* eng, int K, int pos) {
  using namespace iam;
  IAM_CHECK(eng, "iam_verify: null engine");
  EngineImpl& e = eng->impl;
  IAM_CHECK(K >= 1 && K <= e.d.max_rows && K <= kMaxRowsFinalize, "iam_verify: K out of range (1..max_rows, <= 256)");
  IAM_CHECK(pos >= 0 && pos + K <= e.d.max_ctx, "iam_verify: pos + K exceeds max_ctx");
  if (e.world > 1 && !e.comm) return e.setf(IAM_ESTATE, "iam_verify: the communicator was aborted");
  E_CUDA(cudaSetDevice(e.device));
  E_RUN(ensure_packed(e));
  return IAM_OK;
}

extern "C" int iam_verify(iam_engine* eng, const int32_t* tokens, int K, int pos, int32_t* argmax_out,
                          int* accept_len) {
  using namespace iam;
  int r = verify_common(eng, K, pos);
  if (r != IAM_OK) return r;
  IAM_CHECK(tokens && argmax_out, "iam_verify: null buffer");
  EngineImpl& e = eng->impl;
  for (int i = 0; i < K; ++i)
    if (tokens[i] < 0 || tokens[i] >= e.d.vocab) return e.setf(IAM_EINVAL, "iam_verify: token id out of range");
  E_CUDA(cudaSetDevice(e.device));
  cudaGraphExec_t g = nullptr;
  E_RUN(get_graph(e, K, &g));
  e.h_in->pos = pos;
  e.host_pos = pos + K;
  std::memcpy(e.h_in->tokens, tokens, sizeof(int32_t) * K);
  E_CUDA(cudaMemcpyAsync(e.d_in, e.h_in, sizeof(int32_t) * (1 + K), cudaMemcpyHostToDevice, e.stream));
  E_CUDA(cudaGraphLaunch(g, e.stream));
  e.last_K = K;
  E_CUDA(cudaMemcpyAsync(e.h_out, e.d_out, sizeof(int32_t) * (1 + K), cudaMemcpyDeviceToHost, e.stream));
  E_CUDA(cudaMemcpyAsync(e.h_err, e.d_err, sizeof(int), cudaMemcpyDeviceToHost, e.stream));
  E_RUN(sync_step(e, "iam_verify"));
  E_RUN(device_status(e, "iam_verify"));
  std::memcpy(argmax_out, e.h_out + 1, sizeof(int32_t) * K);
  if (accept_len) *accept_len = e.h_out[0];
  return IAM_OK;
}

extern "C" int iam_decode_step(iam_engine* eng, int32_t token, int pos, int32_t* next_token) {
  int acc = 0;
  return iam_verify(eng, &token, 1, pos, next_token, &acc);
}

extern "C" int iam_generate(iam_engine* eng, const int32_t* prompt, int n_prompt, int max_new, const int32_t* eos,
                            int n_eos, int32_t* out, int* n_out) {
  using namespace iam;
  IAM_CHECK(eng && prompt && out && n_out && n_prompt > 0 && max_new > 0 && n_eos >= 0 && (eos || n_eos == 0),
            "iam_generate: bad arguments");
  EngineImpl& e = eng->impl;
  *n_out = 0;
  if (n_prompt + max_new - 1 > e.d.max_ctx)
    return e.setf(IAM_EINVAL, "iam_generate: prompt + max_new - 1 exceeds max_ctx");
  auto is_eos = [&](int32_t t) {
    for (int i = 0; i < n_eos; ++i)
      if (eos[i] == t) return true;
    return false;
  };
  // runTest (test_context.swift:1216-1270): reset, prefill, then greedy steps
  int r = iam_state_reset(eng);
  if (r != IAM_OK) return r;
  std::vector<int32_t> am(static_cast<size_t>(e.d.max_rows));
  int32_t next = -1;
  for (int p0 = 0; p0 < n_prompt; p0 += e.d.max_rows) {  // prefill in verify blocks
    const int k = std::min(e.d.max_rows, n_prompt - p0);
    r = iam_verify(eng, prompt + p0, k, p0, am.data(), nullptr);
    if (r != IAM_OK) return r;
    next = am[static_cast<size_t>(k - 1)];
  }
  int pos = n_prompt;
  out[(*n_out)++] = next;
  while (*n_out < max_new && !is_eos(next)) {
    r = iam_decode_step(eng, next, pos++, &next);
    if (r != IAM_OK) return r;
    out[(*n_out)++] = next;
  }
  return IAM_OK;
}

extern "C" int iam_verify_device(iam_engine* eng, const int32_t* d_tokens, int K, int pos, int32_t* d_argmax,
                                 void* stream) {
  using namespace iam;
  IAM_CHECK(eng, "iam_verify_device: null engine");
  EngineImpl& e = eng->impl;
  if (K < 1 || K > e.d.max_rows || K > kMaxRowsFinalize)
    return e.setf(IAM_EINVAL, "iam_verify_device: K out of range (1..max_rows, <= 256)");
  if (e.world > 1 && !e.comm) return e.setf(IAM_ESTATE, "iam_verify_device: the communicator was aborted");
  cudaStream_t st = stream ? as_stream(stream) : e.stream;
  E_CUDA(cudaSetDevice(e.device));
  E_RUN(ensure_packed(e));  // weights loaded or generated since the last step: pack them first
  cudaGraphExec_t g = nullptr;
  E_RUN(get_graph(e, K, &g));
  // pos < 0 keeps the device position (advanced by the previous step); the
  // host mirror keeps every step inside the KV cache
  const int start = pos >= 0 ? pos : e.host_pos;
  if (start < 0 || start + K > e.d.max_ctx) return e.setf(IAM_EINVAL, "iam_verify_device: pos + K exceeds max_ctx");
  e.host_pos = start + K;
  if (pos >= 0) {
    e.h_in->pos = pos;
    E_CUDA(cudaMemcpyAsync(&e.d_in->pos, &e.h_in->pos, sizeof(int32_t), cudaMemcpyHostToDevice, st));
  }
  if (d_tokens) E_CUDA(cudaMemcpyAsync(e.d_in->tokens, d_tokens, sizeof(int32_t) * K, cudaMemcpyDeviceToDevice, st));
  E_CUDA(cudaGraphLaunch(g, st));
  e.last_K = K;
  if (d_argmax) E_CUDA(cudaMemcpyAsync(d_argmax, e.d_out + 1, sizeof(int32_t) * K, cudaMemcpyDeviceToDevice, st));
  return IAM_OK;
}

extern "C" int iam_rollback(iam_engine* eng, int n_keep, void* stream) {
  using namespace iam;
  IAM_CHECK(eng, "iam_rollback: null engine");
  EngineImpl& e = eng->impl;
  if (e.last_K == 0)
    return e.setf(IAM_ESTATE, "iam_rollback: no verify block since the state was reset or initialised");
  if (n_keep < 1 || n_keep > e.last_K)
    return e.setf(IAM_EINVAL, "iam_rollback: n_keep out of range (1..rows of the last verify)");
  E_CUDA(cudaSetDevice(e.device));
  const int K = e.last_K;
  E_RUN(enqueue_rollback(e, K, n_keep, stream ? as_stream(stream) : e.stream));
  e.host_pos += n_keep - K;
  e.last_K = n_keep;
  return IAM_OK;
}

static int batch_common(iam_engine* eng, int n_seq, int K) {
  using namespace iam;
  IAM_CHECK(eng, "iam_verify_batch: null engine");
  EngineImpl& e = eng->impl;
  if (n_seq < 1 || n_seq > e.max_seqs) return e.setf(IAM_EINVAL, "iam_verify_batch: n_seq out of range (1..max_seqs)");
  if (K < 1 || static_cast<long long>(n_seq) * K > e.d.max_rows)
    return e.setf(IAM_EINVAL, "iam_verify_batch: n_seq * K exceeds max_rows");
  if (e.world > 1 && !e.comm) return e.setf(IAM_ESTATE, "iam_verify_batch: the communicator was aborted");
  E_CUDA(cudaSetDevice(e.device));
  E_RUN(ensure_packed(e));
  return IAM_OK;
}

extern "C" int iam_verify_batch(iam_engine* eng, const int32_t* tokens, int n_seq, int K, const int32_t* pos,
                                int32_t* argmax_out, int32_t* accept_len) {
  using namespace iam;
  int r = batch_common(eng, n_seq, K);
  if (r != IAM_OK) return r;
  EngineImpl& e = eng->impl;
  IAM_CHECK(tokens && pos && argmax_out, "iam_verify_batch: null buffer");
  const int rows = n_seq * K;
  for (int q = 0; q < n_seq; ++q)
    if (pos[q] < 0 || pos[q] + K > e.d.max_ctx) return e.setf(IAM_EINVAL, "iam_verify_batch: pos + K exceeds max_ctx");
  for (int i = 0; i < rows; ++i)
    if (tokens[i] < 0 || tokens[i] >= e.d.vocab) return e.setf(IAM_EINVAL, "iam_verify_batch: token id out of range");
  cudaGraphExec_t g = nullptr;
  E_RUN(get_batch_graph(e, n_seq, K, &g));
  // positions of slots 0..n_seq-1, then the tokens right after the slot table
  std::memcpy(e.h_bin, pos, sizeof(int32_t) * n_seq);
  std::memcpy(e.h_bin + e.max_seqs, tokens, sizeof(int32_t) * rows);
  E_CUDA(cudaMemcpyAsync(e.d_bin, e.h_bin, sizeof(int32_t) * n_seq, cudaMemcpyHostToDevice, e.stream));
  E_CUDA(cudaMemcpyAsync(e.d_bin + e.max_seqs, e.h_bin + e.max_seqs, sizeof(int32_t) * rows, cudaMemcpyHostToDevice,
                         e.stream));
  E_CUDA(cudaGraphLaunch(g, e.stream));
  e.last_K = 0;  // slot 0 advanced outside the single-sequence path: nothing to roll back
  E_CUDA(cudaMemcpyAsync(e.h_bout, e.d_bout, sizeof(int32_t) * n_seq, cudaMemcpyDeviceToHost, e.stream));
  E_CUDA(cudaMemcpyAsync(e.h_bout + e.max_seqs, e.d_bout + e.max_seqs, sizeof(int32_t) * rows,
                         cudaMemcpyDeviceToHost, e.stream));
  E_CUDA(cudaMemcpyAsync(e.h_err, e.d_err, sizeof(int), cudaMemcpyDeviceToHost, e.stream));
  E_RUN(sync_step(e, "iam_verify_batch"));
  E_RUN(device_status(e, "iam_verify_batch"));
  std::memcpy(argmax_out, e.h_bout + e.max_seqs, sizeof(int32_t) * rows);
  if (accept_len) std::memcpy(accept_len, e.h_bout, sizeof(int32_t) * n_seq);
  return IAM_OK;
}

extern "C" int iam_verify_batch_device(iam_engine* eng, const int32_t* d_tokens, int n_seq, int K,
                                       const int32_t* d_pos, int32_t* d_argmax, int32_t* d_accept, void* stream) {
  using namespace iam;
  int r = batch_common(eng, n_seq, K);
  if (r != IAM_OK) return r;
  EngineImpl& e = eng->impl;
  cudaStream_t st = stream ? as_stream(stream) : e.stream;
  cudaGraphExec_t g = nullptr;
  E_RUN(get_batch_graph(e, n_seq, K, &g));
  const int rows = n_seq * K;
  if (d_pos) E_CUDA(cudaMemcpyAsync(e.d_bin, d_pos, sizeof(int32_t) * n_seq, cudaMemcpyDeviceToDevice, st));
  if (d_tokens)
    E_CUDA(cudaMemcpyAsync(e.d_bin + e.max_seqs, d_tokens, sizeof(int32_t) * rows, cudaMemcpyDeviceToDevice, st));
  E_CUDA(cudaGraphLaunch(g, st));
  e.last_K = 0;
  if (d_argmax)
    E_CUDA(cudaMemcpyAsync(d_argmax, e.d_bout + e.max_seqs, sizeof(int32_t) * rows, cudaMemcpyDeviceToDevice, st));
  if (d_accept) E_CUDA(cudaMemcpyAsync(d_accept, e.d_bout, sizeof(int32_t) * n_seq, cudaMemcpyDeviceToDevice, st));
  return IAM_OK;
}

extern "C" int iam_engine_status(iam_engine* eng, void* stream) {
  using namespace iam;
  IAM_CHECK(eng, "iam_engine_status: null engine");
  EngineImpl& e = eng->impl;
  E_CUDA(cudaSetDevice(e.device));
  const cudaStream_t st = stream ? as_stream(stream) : e.stream;
  if (st != e.stream) {  // order the engine stream after the caller's
    cudaEvent_t ev = nullptr;
    E_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    const cudaError_t a = cudaEventRecord(ev, st);
    const cudaError_t b = a == cudaSuccess ? cudaStreamWaitEvent(e.stream, ev, 0) : a;
    cudaEventDestroy(ev);
    E_CUDA(b);
  }
  E_CUDA(cudaMemcpyAsync(e.h_err, e.d_err, sizeof(int), cudaMemcpyDeviceToHost, e.stream));
  E_RUN(sync_step(e, "iam_engine_status"));
  return device_status(e, "iam_engine_status");
}

extern "C" int iam_read_hidden(iam_engine* eng, uint16_t* host_ptr, int K) {
  using namespace iam;
  IAM_CHECK(eng && host_ptr && K >= 1, "iam_read_hidden: bad argument");
  EngineImpl& e = eng->impl;
  E_CUDA(cudaStreamSynchronize(e.stream));
  E_CUDA(cudaMemcpy(host_ptr, e.normed, static_cast<size_t>(K) * e.d.hidden * 2, cudaMemcpyDeviceToHost));
  return IAM_OK;
}

extern "C" int iam_streamed_layers(const iam_engine* eng) { return eng ? eng->impl.n_streamed : -1; }

extern "C" int iam_step_launches(iam_engine* eng, int K) {
  if (!eng) return -1;
  EngineImpl& e = eng->impl;
  // count launches by enqueueing into a throw-away capture
  if (cudaSetDevice(e.device) != cudaSuccess || iam::ensure_packed(e) != IAM_OK) return -1;
  cudaGraphExec_t g = nullptr;
  const int before = e.launches;
  if (e.graphs.count(K)) {
    cudaGraphExecDestroy(e.graphs[K]);
    e.graphs.erase(K);
  }
  if (iam::get_graph(e, K, &g) != IAM_OK) return -1;
  return e.launches - before;
}

// Weights once, plus per sequence its K embedding rows, state read + write
// and KV read.
static double step_bytes(const iam::EngineImpl& e, int n_seq, int K, int pos) {
  const iam_dims& d = e.d;
  double w = 0.0;
  for (const auto& t : e.tensors) {
    if (t.name == "model.embed_tokens.weight") continue;
    w += static_cast<double>(t.bytes());
  }
  double q = static_cast<double>(K) * d.hidden * 2;                                      // embedding rows
  q += 2.0 * e.n_gdn * e.gv_l * d.gdn_dk * d.gdn_dv * 4;                                 // S read + write
  q += 2.0 * e.n_gdn * 3 * e.conv_l * 2;                                                 // conv state
  q += 2.0 * e.n_attn * static_cast<double>(pos + K) * e.hkv_l * d.head_dim * 2;         // KV read
  return w + n_seq * q;
}

extern "C" double iam_step_bytes(iam_engine* eng, int K, int pos) {
  return eng ? step_bytes(eng->impl, 1, K, pos) : 0.0;
}

extern "C" double iam_step_bytes_batch(iam_engine* eng, int n_seq, int K, int pos) {
  return eng ? step_bytes(eng->impl, n_seq, K, pos) : 0.0;
}

// One eager (non-graph) step at width K with CUDA events around every launch.
static int profile_run(iam_engine* eng, int K, int pos, std::vector<iam::ProfEntry>& ents) {
  using namespace iam;
  int r = verify_common(eng, K, pos);
  if (r != IAM_OK) return r;
  EngineImpl& e = eng->impl;
  e.h_in->pos = pos;
  E_CUDA(cudaMemcpyAsync(&e.d_in->pos, &e.h_in->pos, 4, cudaMemcpyHostToDevice, e.stream));
  e.prof = &ents;
  r = enqueue_step(e, 0, K);
  e.prof = nullptr;
  if (r != IAM_OK) return r;
  E_CUDA(cudaStreamSynchronize(e.stream));
  return IAM_OK;
}

static float prof_ms(iam::ProfEntry& en) {
  float x = 0.f;
  cudaEventElapsedTime(&x, en.a, en.b);
  cudaEventDestroy(en.a);
  cudaEventDestroy(en.b);
  return x;
}

extern "C" int iam_profile_step(iam_engine* eng, int K, int pos, int cap, const char** kinds, double* ms,
                                double* bytes, int* launches) {
  using namespace iam;
  std::vector<ProfEntry> ents;
  const int r = profile_run(eng, K, pos, ents);
  if (r != IAM_OK) return -r;
  static std::vector<std::string> names;
  std::vector<std::string> order;
  std::map<std::string, double> tms, tby;
  std::map<std::string, int> tn;
  for (auto& en : ents) {
    if (!tn.count(en.kind)) order.push_back(en.kind);
    tms[en.kind] += prof_ms(en);
    tby[en.kind] += en.bytes;
    tn[en.kind] += 1;
  }
  names = order;
  int n = 0;
  for (auto& k : names) {
    if (n >= cap) break;
    kinds[n] = k.c_str();
    ms[n] = tms[k];
    bytes[n] = tby[k];
    launches[n] = tn[k];
    ++n;
  }
  return n;
}

extern "C" int iam_profile_layers(iam_engine* eng, int K, int pos, double* ms, double* mlp_ms, int* is_attn) {
  using namespace iam;
  std::vector<ProfEntry> ents;
  const int r = profile_run(eng, K, pos, ents);
  if (r != IAM_OK) return -r;
  EngineImpl& e = eng->impl;
  const int n = e.d.n_layers;
  for (int i = 0; i < n; ++i) {
    ms[i] = mlp_ms[i] = 0.0;
    is_attn[i] = e.layers[i].attn ? 1 : 0;
  }
  for (auto& en : ents) {
    const float x = prof_ms(en);
    if (en.part >= 0 && en.part < 2 * n) (en.part & 1 ? mlp_ms : ms)[en.part >> 1] += x;
  }
  return n;
}
