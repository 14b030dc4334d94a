// Host launcher for the reference's Metal compute kernels (test infrastructure).
//
// The kernel source is the reference's own full_forward.swift:55-445, extracted
// unchanged at build time into oracle/_ref/ (see extract_msl.py, Makefile).  Each
// extern "C" wrapper below runs one kernel over the grid that the reference's
// Swift dispatch code uses (full_forward.swift:828-1308), one grid position at a
// time; rms_norm_bf16, the one kernel with threadgroup memory and barriers, runs
// its 256-thread group as 256 host threads.
#include <metal_stdlib>
#include "ref_kernels.metal"
#undef kernel
#undef device
#undef constant
#undef threadgroup

#include <thread>
#include <vector>

static thread_local std::barrier<>* g_bar = nullptr;
void threadgroup_barrier(metal::mem_flags) { g_bar->arrive_and_wait(); }

template <class F>
static void run_group(unsigned n, F f) {
  std::barrier<> bar(n);
  std::vector<std::thread> ts;
  ts.reserve(n);
  for (unsigned i = 0; i < n; ++i) ts.emplace_back([&, i] { g_bar = &bar; f(i); });
  for (auto& t : ts) t.join();
}

typedef uint16_t u16;
#define B(p) reinterpret_cast<bfloat*>(p)
#define CB(p) reinterpret_cast<const bfloat*>(p)

extern "C" {

// rms_norm_bf16: dispatchThreads(256) with threadgroup 256 (full_forward.swift:1005-1013)
void ref_rms_norm_bf16(const u16* x, const u16* w, u16* out, uint rows, uint dim, float eps) {
  for (uint r = 0; r < rows; ++r) {
    uint d = dim; float e = eps;
    run_group(256, [&](uint tid) { rms_norm_bf16(CB(x + r * dim), CB(w), B(out + r * dim), d, e, tid, 256); });
  }
}

void ref_silu_multiply_bf16(const u16* g, const u16* u, u16* out, uint count) {
  for (uint t = 0; t < count; ++t) silu_multiply_bf16(CB(g), CB(u), B(out), count, t);
}

void ref_residual_add_bf16(const u16* a, const u16* b, u16* out, uint count) {
  for (uint t = 0; t < count; ++t) residual_add_bf16(CB(a), CB(b), B(out), count, t);
}

void ref_embed_lookup_bf16(const uint32_t* w, const u16* s, const u16* b, u16* out, uint token,
                           uint hidden, uint group) {
  for (uint t = 0; t < hidden; ++t)
    embed_lookup_bf16(reinterpret_cast<const uint*>(w), CB(s), CB(b), B(out), token, hidden, group, t);
}

void ref_sigmoid_multiply_bf16(const u16* a, const u16* b, u16* out, uint count) {
  for (uint t = 0; t < count; ++t) sigmoid_multiply_bf16(CB(a), CB(b), B(out), count, t);
}

void ref_rope_bf16(u16* x, float* cosv, float* sinv, uint heads, uint head_dim, uint rotary) {
  for (uint h = 0; h < heads; ++h)
    for (uint p = 0; p < rotary / 2; ++p) rope_bf16(B(x), cosv, sinv, heads, head_dim, rotary, uint2{p, h});
}

void ref_argmax_bf16(const u16* x, uint32_t* result, uint count) {
  argmax_bf16(CB(x), reinterpret_cast<uint*>(result), count, 0);
}

void ref_per_head_rms_norm_bf16(const u16* x, const u16* w, u16* out, uint heads, uint head_dim, float eps) {
  for (uint h = 0; h < heads; ++h)
    for (uint e = 0; e < head_dim; ++e) per_head_rms_norm_bf16(CB(x), CB(w), B(out), heads, head_dim, eps, uint2{e, h});
}

void ref_expand_kv_heads_bf16(const u16* kv, u16* out, uint heads, uint kv_heads, uint head_dim) {
  for (uint h = 0; h < heads; ++h)
    for (uint e = 0; e < head_dim; ++e) expand_kv_heads_bf16(CB(kv), B(out), heads, kv_heads, head_dim, uint2{e, h});
}

void ref_split_q_gate_bf16(const u16* qg, u16* q, u16* gate, uint heads, uint head_dim) {
  for (uint h = 0; h < heads; ++h)
    for (uint e = 0; e < head_dim; ++e) split_q_gate_bf16(CB(qg), B(q), B(gate), heads, head_dim, uint2{e, h});
}

void ref_depthwise_conv1d_m1_bf16(const u16* state, const u16* x, const u16* w, u16* out, u16* new_state,
                                  uint conv_dim) {
  for (uint t = 0; t < conv_dim; ++t)
    depthwise_conv1d_m1_bf16(CB(state), CB(x), CB(w), B(out), B(new_state), conv_dim, t);
}

void ref_silu_bf16(const u16* x, u16* out, uint count) {
  for (uint t = 0; t < count; ++t) silu_bf16(CB(x), B(out), count, t);
}

void ref_per_head_rms_norm_scaled_bf16(const u16* x, u16* out, uint heads, uint head_dim, float eps, float scale) {
  for (uint h = 0; h < heads; ++h)
    for (uint e = 0; e < head_dim; ++e)
      per_head_rms_norm_scaled_bf16(CB(x), B(out), heads, head_dim, eps, scale, uint2{e, h});
}

void ref_compute_g_beta_bf16(const u16* a, const u16* b, const float* A_log, const u16* dt_bias, u16* g,
                             u16* beta, uint heads) {
  for (uint t = 0; t < heads; ++t) compute_g_beta_bf16(CB(a), CB(b), A_log, CB(dt_bias), B(g), B(beta), heads, t);
}

void ref_gated_delta_step_bf16(const u16* q, const u16* k, const u16* v, const u16* g, const u16* beta,
                               float* state, u16* y, uint v_heads, uint dv, uint dk) {
  for (uint h = 0; h < v_heads; ++h)
    for (uint r = 0; r < dv; ++r)
      gated_delta_step_bf16(CB(q), CB(k), CB(v), CB(g), CB(beta), state, B(y), v_heads, dv, dk, uint2{r, h});
}

void ref_rms_norm_gated_bf16(const u16* x, const u16* z, const u16* w, u16* out, uint heads, uint head_dim,
                             float eps) {
  for (uint h = 0; h < heads; ++h)
    for (uint e = 0; e < head_dim; ++e) rms_norm_gated_bf16(CB(x), CB(z), CB(w), B(out), heads, head_dim, eps, uint2{e, h});
}

void ref_copy_bf16(const u16* src, u16* dst, uint count) {
  for (uint t = 0; t < count; ++t) copy_bf16(CB(src), B(dst), count, t);
}

void ref_sdpa_decode_bf16(const u16* q, const u16* kc, const u16* vc, u16* out, uint heads, uint kv_heads,
                          uint head_dim, uint seq_len) {
  for (uint h = 0; h < heads; ++h) sdpa_decode_bf16(CB(q), CB(kc), CB(vc), B(out), heads, kv_heads, head_dim, seq_len, h);
}

}  // extern "C"
