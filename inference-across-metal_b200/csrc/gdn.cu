// GatedDeltaNet recurrent step for K sequential tokens, one CTA per V-head.
//
// Fuses, per layer (dispatchGDNLayer, full_forward.swift:1025-1123):
//   depthwise_conv1d_m1_bf16 -> silu_bf16 -> per_head_rms_norm_scaled_bf16 (q, k)
//   -> expand_kv_heads_bf16 (index math) -> compute_g_beta_bf16
//   -> gated_delta_step_bf16 -> rms_norm_gated_bf16
// with the reference's bf16 rounding points (conv out, SiLU out, q^/k^, g,
// beta, y, gated-norm out) and its fp32 state.
//
// Layout: the head's 128x128 fp32 state lives in registers for the whole
// verify block (warp w owns rows dv = 8w..8w+7, lane l owns dk = 4l..4l+3);
// it is read once and written once per step.  Rows of S evolve independently,
// so the per-token chain needs no block-wide barrier: two 8-row transposed
// warp reductions (9 shuffles each) and an 8-value broadcast per token.
// Conv outputs, q^, k^, v, g, beta of a chunk of tokens are prepared in
// parallel in shared memory before the sequential part; the gated norm runs
// after it, again in parallel over tokens.
#include <cstdlib>

#include "kernels.cuh"

namespace iam {
namespace {

constexpr int kHD = 128;      // dk == dv
constexpr int kThreads = 512; // 16 warps x 8 rows
constexpr int kChunk = 32;    // tokens prepared per pass
constexpr int kConvSeqRows = 8;  // blocks of this many tokens or more: conv one channel a thread

struct GdnSmem {
  float q[kChunk][kHD];
  float k[kChunk][kHD];
  float v[kChunk][kHD];
  float y[kChunk][kHD];
  float g[kChunk];
  float beta[kChunk];
  float ssx[2][kChunk];  // partial sums of y^2 of this CTA's rows (cluster exchange), by chunk parity
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// a float in the shared memory of CTA `rank` of the cluster, at this CTA's address of p
__device__ __forceinline__ float ld_peer(const float* p, uint32_t rank) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p)), ra;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

// Sum v[0..V-1] (V/2 "a" partials, then V/2 "b" partials) over the warp in
// five dependent exchange steps.  Lane l ends with the sum of a[row] (bit 4
// of l clear) or b[row] (set); the row is made of the next log2(V/2) bits of
// l below bit 4, most significant first, and the remaining low bits select
// lanes holding the same sum.
template <int V>
__device__ __forceinline__ float xreduce(float (&v)[V], int lane) {
  int n = V;
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    if (n > 1) {
      const bool up = lane & m;
      const int h = n / 2;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < h) {
          const float send = up ? v[i] : v[i + h];
          const float keep = up ? v[i + h] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
      }
      n = h;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
    }
  }
  return v[0];
}
template <int RPW>
struct RowMap {
  static constexpr int kLog = RPW == 8 ? 3 : RPW == 4 ? 2 : RPW == 2 ? 1 : 0;
  static constexpr int kShift = 4 - kLog;  // lane bits below the row bits
  __device__ static int row(int lane) { return (lane >> kShift) & (RPW - 1); }
  __device__ static int lane_of(int r) { return r << kShift; }
  __device__ static bool writer(int lane) { return (lane & ((1 << kShift) - 1)) == 0; }
};

// gated_delta_step_bf16 (full_forward.swift:321-355) for tokens [0, n) of the
// chunk in shared memory: S = g*S; kv = S.k; delta = beta*(v - kv);
// S = S + k*delta; y = bf16(S.q).  The warp holds RPW rows of S:
// S[r][i] = state[dv = row0 + RPW*w + r][dk = 4l + i].  Per token one warp
// reduction carries both y_t = S_t.q_t and the next token's S_t.k_{t+1}
// (kv_{t+1} = g_{t+1} * S_t.k_{t+1}, the same product in another order), so
// the serial chain holds one reduction a token, not two.
template <int RPW>
__device__ __forceinline__ void delta_chunk(float (&S)[RPW][4], const GdnSmem& sm, float (*ys)[kHD], int n,
                                            int row0, int lane) {
  using RM = RowMap<RPW>;
  const int rr = RM::row(lane);
  const bool is_y = lane & 16;
  float v[2 * RPW];
  {
    const float4 k4 = *reinterpret_cast<const float4*>(&sm.k[0][4 * lane]);
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      v[r] = fmaf(S[r][3], k4.w, fmaf(S[r][2], k4.z, fmaf(S[r][1], k4.y, S[r][0] * k4.x)));
      v[RPW + r] = 0.f;
    }
  }
  float red = xreduce<2 * RPW>(v, lane);  // lanes without bit 4: S.k_0 of row rr
  for (int t = 0; t < n; ++t) {
    const float gv = sm.g[t], bv = sm.beta[t];
    const float4 k4 = *reinterpret_cast<const float4*>(&sm.k[t][4 * lane]);
    const float4 q4 = *reinterpret_cast<const float4*>(&sm.q[t][4 * lane]);
    const float4 kn = t + 1 < n ? *reinterpret_cast<const float4*>(&sm.k[t + 1][4 * lane]) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float dmine = (sm.v[t][row0 + rr] - gv * red) * bv;  // meaningful in the lanes holding S.k
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const float d = __shfl_sync(0xffffffffu, dmine, RM::lane_of(r));
      S[r][0] = fmaf(S[r][0], gv, k4.x * d);
      S[r][1] = fmaf(S[r][1], gv, k4.y * d);
      S[r][2] = fmaf(S[r][2], gv, k4.z * d);
      S[r][3] = fmaf(S[r][3], gv, k4.w * d);
      v[RPW + r] = fmaf(S[r][3], q4.w, fmaf(S[r][2], q4.z, fmaf(S[r][1], q4.y, S[r][0] * q4.x)));
      v[r] = fmaf(S[r][3], kn.w, fmaf(S[r][2], kn.z, fmaf(S[r][1], kn.y, S[r][0] * kn.x)));
    }
    red = xreduce<2 * RPW>(v, lane);
    if (is_y && RM::writer(lane)) ys[t][row0 + rr] = round_bf(red);
  }
}

template <int RPW>
__device__ __forceinline__ void load_state(float (&S)[RPW][4], const float* Sh, int row0, int lane) {
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const float4 v = *reinterpret_cast<const float4*>(Sh + (row0 + r) * kHD + 4 * lane);
    S[r][0] = v.x;
    S[r][1] = v.y;
    S[r][2] = v.z;
    S[r][3] = v.w;
  }
}
template <int RPW>
__device__ __forceinline__ void store_state(const float (&S)[RPW][4], float* Sh, int row0, int lane) {
#pragma unroll
  for (int r = 0; r < RPW; ++r)
    *reinterpret_cast<float4*>(Sh + (row0 + r) * kHD + 4 * lane) = make_float4(S[r][0], S[r][1], S[r][2], S[r][3]);
}

// One V-head over a cluster of C CTAs: CTA j of the cluster holds state rows
// dv = 128j/C .. 128(j+1)/C - 1 (rows evolve independently), prepares the
// head's q^, k^ and its own v rows, runs the recurrence on its rows, and the
// gated norm's sum of squares over dv is exchanged through distributed
// shared memory (summed in rank order).  C = 1 is the one-CTA-a-head kernel.
// kSeq: one launch over several sequences, grid.y = sequence (GdnArgs n_seq).
template <int C, bool kSeq, bool kSpread>
__global__ void __launch_bounds__(kThreads, 1) gdn_fused_kernel(const GdnArgs a) {
  constexpr int R = kHD / C, RPW = R / (kThreads / 32);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  GdnSmem& sm = *reinterpret_cast<GdnSmem*>(smem_raw);
  const int h = blockIdx.x / C;
  const int jr = C == 1 ? 0 : static_cast<int>(cluster_rank());
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rep = a.n_v_heads / a.n_k_heads;
  const int kh = h / rep;
  const int sq = kSeq ? static_cast<int>(blockIdx.y) : 0;
  const uint16_t* in = a.in;
  uint16_t* out = a.out;
  size_t soff = 0, coff = 0;
  if constexpr (kSeq) {
    in += static_cast<size_t>(sq) * a.rows * a.ld_in;
    out += static_cast<size_t>(sq) * a.rows * a.ld_out;
    soff = static_cast<size_t>(sq) * a.seq_S;
    coff = static_cast<size_t>(sq) * a.seq_conv;
  }
  const bool swap = a.parity_dev && __ldcg(a.parity_dev + sq);
  float* S_rd = a.S + soff;
  float* S_wr = (a.S_alt ? a.S_alt : a.S) + soff;
  if (swap && a.S_alt) {
    S_rd = a.S_alt + soff;
    S_wr = a.S + soff;
  }
  const size_t hoff = static_cast<size_t>(h) * kHD * kHD;
  const int row0 = jr * R + warp * RPW;  // this warp's first state row

  // The state, the conv window, the conv and norm weights do not depend on
  // the preceding kernel (the window and state were written by the previous
  // step): load them before waiting for it.
  float S[RPW][4];
  load_state<RPW>(S, S_rd + hoff, row0, lane);
  const uint16_t* conv_in = (swap ? a.conv_out : a.conv_in) + coff;
  uint16_t* conv_out = (swap ? const_cast<uint16_t*>(a.conv_in) : a.conv_out) + coff;

  // The head's conv channels: 0..127 q (K-head kh), 128..255 k, then this
  // CTA's R v rows (V-head h).  Global column of channel ci:
  const int nch = 256 + R;
  auto chan_col = [&](int ci) {
    return ci < 128 ? kh * kHD + ci : ci < 256 ? a.key_dim + kh * kHD + (ci - 128) : 2 * a.key_dim + h * kHD + jr * R + (ci - 256);
  };
  // the conv input of global token u (u < 0: the window of the previous step)
  auto conv_x = [&](int u, int col) -> uint16_t {
    return u >= 0 ? in[static_cast<size_t>(u) * a.ld_in + col] : conv_in[static_cast<size_t>(3 + u) * a.conv_dim + col];
  };
  // Two schedules for conv + SiLU, the same arithmetic: blocks of at least
  // kConvSeqRows tokens give thread ci < nch channel ci for every token, its
  // inputs loaded once and the window kept in registers (weights and window
  // fetched before the grid-dependency wait); shorter blocks spread the
  // (token, channel) pairs over all threads.  Measured on the 27B step: the
  // first is 0.17 ms faster at K = 32, the second 0.08 ms faster at K = 1.
  constexpr bool seq_conv = !kSpread;  // one kernel a schedule (each allocates its own registers)
  const int ct = threadIdx.x;
  const int my_col = ct < nch ? chan_col(ct) : -1;
  float k0 = 0.f, k1 = 0.f, k2 = 0.f, k3 = 0.f;
  uint16_t w0 = 0, w1 = 0, w2 = 0;  // window: the last three inputs (bf16)
  if (seq_conv && my_col >= 0) {
    const uint2 cw = *reinterpret_cast<const uint2*>(a.conv_w + static_cast<size_t>(my_col) * 4);
    k0 = lo_bf(cw.x);
    k1 = hi_bf(cw.x);
    k2 = lo_bf(cw.y);
    k3 = hi_bf(cw.y);
    w0 = conv_in[my_col];
    w1 = conv_in[a.conv_dim + my_col];
    w2 = conv_in[2 * a.conv_dim + my_col];
  }
  // this lane's four gated-norm weights (phase D: lanes < R / 4)
  uint2 ww = make_uint2(0u, 0u);
  if (lane < R / 4) ww = *reinterpret_cast<const uint2*>(a.norm_w + jr * R + 4 * lane);
  pdl_wait();
  pdl_trigger();

  int chunk = 0;
  for (int t0 = 0; t0 < a.rows; t0 += kChunk, ++chunk) {
    const int n = min(kChunk, a.rows - t0);
    // ---- A: conv + SiLU for the chunk (depthwise_conv1d_m1_bf16, silu_bf16),
    // every (token, channel) pair independent: spread over all threads, each
    // reading its four inputs (the tokens before the block from the window)
    if (seq_conv) {
      if (my_col >= 0) {
        float* dst = ct < 128 ? &sm.q[0][ct] : ct < 256 ? &sm.k[0][ct - 128] : &sm.v[0][jr * R + (ct - 256)];
        uint16_t xin[kChunk];
#pragma unroll
        for (int t = 0; t < kChunk; ++t)
          xin[t] = t < n ? in[static_cast<size_t>(t0 + t) * a.ld_in + my_col] : uint16_t(0);
#pragma unroll
        for (int t = 0; t < kChunk; ++t) {
          if (t < n) {
            const uint16_t xi = xin[t];
            float sum = 0.f;
            sum = __fadd_rn(sum, __fmul_rn(bf2f(w0), k0));
            sum = __fadd_rn(sum, __fmul_rn(bf2f(w1), k1));
            sum = __fadd_rn(sum, __fmul_rn(bf2f(w2), k2));
            sum = __fadd_rn(sum, __fmul_rn(bf2f(xi), k3));
            dst[t * kHD] = round_bf(silu_f(round_bf(sum)));
            w0 = w1;
            w1 = w2;
            w2 = xi;
          }
        }
      } else if (ct >= 384 && ct - 384 < n) {
        // g, beta per token (compute_g_beta_bf16)
        const int t = ct - 384;
        const size_t row = static_cast<size_t>(t0 + t) * a.ld_in;
        float gv, bv;
        g_beta(bf2f(in[row + a.a_col + h]), bf2f(in[row + a.b_col + h]), a.A_log[h], bf2f(a.dt_bias[h]), gv, bv);
        sm.g[t] = gv;
        sm.beta[t] = bv;
      }
    } else if (threadIdx.x < n) {
      // g, beta per token (compute_g_beta_bf16)
      const int t = threadIdx.x;
      const size_t row = static_cast<size_t>(t0 + t) * a.ld_in;
      float gv, bv;
      g_beta(bf2f(in[row + a.a_col + h]), bf2f(in[row + a.b_col + h]), a.A_log[h], bf2f(a.dt_bias[h]), gv, bv);
      sm.g[t] = gv;
      sm.beta[t] = bv;
    }
#pragma unroll 2
    for (int idx = threadIdx.x; !seq_conv && idx < n * nch; idx += kThreads) {
      const int t = idx / nch, ci = idx - t * nch;
      const int col = chan_col(ci);
      const uint2 cw = *reinterpret_cast<const uint2*>(a.conv_w + static_cast<size_t>(col) * 4);
      const int u = t0 + t;
      const uint16_t x0 = conv_x(u - 3, col), x1 = conv_x(u - 2, col), x2 = conv_x(u - 1, col), x3 = conv_x(u, col);
      float sum = 0.f;
      sum = __fadd_rn(sum, __fmul_rn(bf2f(x0), lo_bf(cw.x)));
      sum = __fadd_rn(sum, __fmul_rn(bf2f(x1), hi_bf(cw.x)));
      sum = __fadd_rn(sum, __fmul_rn(bf2f(x2), lo_bf(cw.y)));
      sum = __fadd_rn(sum, __fmul_rn(bf2f(x3), hi_bf(cw.y)));
      float* dst = ci < 128 ? &sm.q[t][ci] : ci < 256 ? &sm.k[t][ci - 128] : &sm.v[t][jr * R + (ci - 256)];
      *dst = round_bf(silu_f(round_bf(sum)));
    }
    __syncthreads();
    // ---- B: q^ = bf16(q_scale * (q / rms)), k^ likewise (per_head_rms_norm_scaled_bf16)
    for (int t = warp; t < n; t += kThreads / 32) {
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        float* row = which == 0 ? sm.q[t] : sm.k[t];
        // GDN_INV_SCALE = Float(0.08838834764) and its fp32 square (full_forward.swift:41, 1056, 1064)
        const float scale = which == 0 ? __uint_as_float(0x3bffffffu) : __uint_as_float(0x3db504f3u);
        float4 v = *reinterpret_cast<float4*>(row + 4 * lane);
        const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
        const float rms = sqrtf(ss / 128.f + 1e-6f);
        v.x = round_bf(scale * (v.x / rms));
        v.y = round_bf(scale * (v.y / rms));
        v.z = round_bf(scale * (v.z / rms));
        v.w = round_bf(scale * (v.w / rms));
        *reinterpret_cast<float4*>(row + 4 * lane) = v;
      }
    }
    __syncthreads();
    // ---- C: the recurrence on this CTA's rows
    delta_chunk<RPW>(S, sm, sm.y, n, row0, lane);
    __syncthreads();
    // ---- D: gated RMSNorm (rms_norm_gated_bf16) and store; lanes < R / 4
    // hold four of this CTA's rows each
    constexpr int kLanes = R / 4;
    float* ssx = sm.ssx[chunk & 1];
    for (int t = warp; t < n; t += kThreads / 32) {
      float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
      if (lane < kLanes) y = *reinterpret_cast<const float4*>(&sm.y[t][jr * R + 4 * lane]);
      const float part = warp_sum(y.x * y.x + y.y * y.y + y.z * y.z + y.w * y.w);
      if (lane == 0) ssx[t] = part;
    }
    if constexpr (C > 1) cluster_sync_all();  // every CTA's partial sums are in place
    else __syncthreads();
    for (int t = warp; t < n; t += kThreads / 32) {
      float ss = ssx[t];
      if constexpr (C > 1) {
        ss = 0.f;
#pragma unroll
        for (int j = 0; j < C; ++j) ss += ld_peer(&ssx[t], static_cast<uint32_t>(j));
      }
      if (lane < kLanes) {
        const float4 y = *reinterpret_cast<const float4*>(&sm.y[t][jr * R + 4 * lane]);
        const float rms = sqrtf(ss / 128.f + a.eps);
        const size_t row = static_cast<size_t>(t0 + t);
        const int d0 = jr * R + 4 * lane;
        const uint2 zz = *reinterpret_cast<const uint2*>(in + row * a.ld_in + a.z_col + h * kHD + d0);
        const float o0 = silu_f(lo_bf(zz.x)) * ((y.x / rms) * lo_bf(ww.x));
        const float o1 = silu_f(hi_bf(zz.x)) * ((y.y / rms) * hi_bf(ww.x));
        const float o2 = silu_f(lo_bf(zz.y)) * ((y.z / rms) * lo_bf(ww.y));
        const float o3 = silu_f(hi_bf(zz.y)) * ((y.w / rms) * hi_bf(ww.y));
        *reinterpret_cast<uint2*>(out + row * a.ld_out + h * kHD + d0) =
            make_uint2(pack_bf2(o0, o1), pack_bf2(o2, o3));
      }
    }
    __syncthreads();
  }
  store_state<RPW>(S, S_wr + hoff, row0, lane);
  // new conv state = the last three inputs; q/k channels are shared by the
  // `rep` V-heads of a K-head, the first CTA of the first of them writes them
  if (threadIdx.x < nch && (threadIdx.x >= 256 || (h % rep == 0 && jr == 0))) {
    const int col = chan_col(threadIdx.x);
#pragma unroll
    for (int j = 0; j < 3; ++j) conv_out[static_cast<size_t>(j) * a.conv_dim + col] = conv_x(a.rows - 3 + j, col);
  }
  if constexpr (C > 1) cluster_sync_all();  // no CTA leaves while a peer may read its shared memory
}

// The operator-level gated_delta_step: q^, k^ (K-head layout), v, g, beta given.
__global__ void __launch_bounds__(kThreads, 1) gated_delta_kernel(const uint16_t* q, const uint16_t* k,
                                                                  const uint16_t* v, const uint16_t* g,
                                                                  const uint16_t* beta, float* Sg, uint16_t* y,
                                                                  int n_v, int n_k, int rows) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  GdnSmem& sm = *reinterpret_cast<GdnSmem*>(smem_raw);
  const int h = blockIdx.x, kh = h / (n_v / n_k);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* Sh = Sg + static_cast<size_t>(h) * kHD * kHD;
  float S[8][4];
  load_state<8>(S, Sh, 8 * warp, lane);
  for (int t0 = 0; t0 < rows; t0 += kChunk) {
    const int n = min(kChunk, rows - t0);
    for (int i = threadIdx.x; i < n * kHD; i += kThreads) {
      const int t = i / kHD, e = i % kHD;
      const size_t tr = static_cast<size_t>(t0 + t);
      sm.q[t][e] = bf2f(q[(tr * n_k + kh) * kHD + e]);
      sm.k[t][e] = bf2f(k[(tr * n_k + kh) * kHD + e]);
      sm.v[t][e] = bf2f(v[(tr * n_v + h) * kHD + e]);
    }
    if (threadIdx.x < n) {
      sm.g[threadIdx.x] = bf2f(g[static_cast<size_t>(t0 + threadIdx.x) * n_v + h]);
      sm.beta[threadIdx.x] = bf2f(beta[static_cast<size_t>(t0 + threadIdx.x) * n_v + h]);
    }
    __syncthreads();
    delta_chunk<8>(S, sm, sm.y, n, 8 * warp, lane);
    __syncthreads();
    for (int i = threadIdx.x; i < n * kHD; i += kThreads) {
      const int t = i / kHD, e = i % kHD;
      y[(static_cast<size_t>(t0 + t) * n_v + h) * kHD + e] = f2bf(sm.y[t][e]);
    }
    __syncthreads();
  }
  store_state<8>(S, Sh, 8 * warp, lane);
}

bool g_attr_done = false;
int g_sms = 148;
}  // namespace

int gdn_init_attrs();
namespace {
int ensure_attrs() { return gdn_init_attrs(); }
}  // namespace

int gdn_init_attrs() {
  if (g_attr_done) return IAM_OK;
  for (auto* k : {gdn_fused_kernel<1, false, false>, gdn_fused_kernel<2, false, false>,
                  gdn_fused_kernel<4, false, false>, gdn_fused_kernel<8, false, false>,
                  gdn_fused_kernel<1, true, false>, gdn_fused_kernel<2, true, false>,
                  gdn_fused_kernel<4, true, false>, gdn_fused_kernel<8, true, false>,
                  gdn_fused_kernel<1, false, true>, gdn_fused_kernel<2, false, true>,
                  gdn_fused_kernel<4, false, true>, gdn_fused_kernel<8, false, true>,
                  gdn_fused_kernel<1, true, true>, gdn_fused_kernel<2, true, true>,
                  gdn_fused_kernel<4, true, true>, gdn_fused_kernel<8, true, true>})
    IAM_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(GdnSmem)));
  int dev = 0;
  IAM_CUDA(cudaGetDevice(&dev));
  IAM_CUDA(cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev));
  IAM_CUDA(cudaFuncSetAttribute(gated_delta_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(GdnSmem)));
  g_attr_done = true;
  return IAM_OK;
}

template <int C, bool kSeq>
int launch_gdn_c(const GdnArgs& a, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_v_heads * C, kSeq ? a.n_seq : 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sizeof(GdnSmem);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (C > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = C;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  if (a.rows >= kConvSeqRows) {
    IAM_CUDA(cudaLaunchKernelEx(&cfg, gdn_fused_kernel<C, kSeq, false>, a));
  } else {
    IAM_CUDA(cudaLaunchKernelEx(&cfg, gdn_fused_kernel<C, kSeq, true>, a));
  }
  return IAM_OK;
}

// CTAs a head: the largest cluster (up to 8) that keeps every CTA of the
// launch in one wave on the SMs; one CTA a head for a single token, where the
// recurrence is one step and the split would only duplicate the q/k work.
// IAM_GDN_SPLIT forces 1, 2, 4 or 8, for experiments.
int gdn_split(int heads, int rows) {
  if (const char* v = std::getenv("IAM_GDN_SPLIT")) {
    const int c = std::atoi(v);
    if (c == 1 || c == 2 || c == 4 || c == 8) return c;
  }
  if (rows < 4) return 1;
  for (int c = 8; c > 1; c >>= 1)
    if (heads * c <= g_sms) return c;
  return 1;
}

int launch_gdn(const GdnArgs& a, cudaStream_t st, bool pdl) {
  IAM_CHECK(a.n_k_heads > 0 && a.n_v_heads % a.n_k_heads == 0, "gdn: n_v_heads must be a multiple of n_k_heads");
  IAM_CHECK(a.rows > 0, "gdn: rows must be positive");
  IAM_CHECK(a.conv_in != a.conv_out, "gdn: conv state in/out must differ");
  IAM_CHECK(a.ld_in % 4 == 0 && a.z_col % 4 == 0 && a.ld_out % 4 == 0 && aligned16(a.S) && aligned16(a.in) &&
                (!a.S_alt || aligned16(a.S_alt)),
            "gdn: 8-byte aligned rows required");
  IAM_CHECK(a.S_alt != a.S, "gdn: the second state buffer must differ from the first");
  IAM_CHECK(a.n_seq <= 1 || (a.seq_S % 4 == 0 && a.seq_conv > 0 && a.n_seq <= 65535),
            "gdn: sequence strides (state 16-byte aligned) and 1..65535 sequences required");
  const int r = ensure_attrs();
  if (r != IAM_OK) return r;
  if (a.n_seq > 1) {
    switch (gdn_split(a.n_v_heads * a.n_seq, a.rows)) {
      case 8:
        return launch_gdn_c<8, true>(a, st, pdl);
      case 4:
        return launch_gdn_c<4, true>(a, st, pdl);
      case 2:
        return launch_gdn_c<2, true>(a, st, pdl);
      default:
        return launch_gdn_c<1, true>(a, st, pdl);
    }
  }
  switch (gdn_split(a.n_v_heads, a.rows)) {
    case 8:
      return launch_gdn_c<8, false>(a, st, pdl);
    case 4:
      return launch_gdn_c<4, false>(a, st, pdl);
    case 2:
      return launch_gdn_c<2, false>(a, st, pdl);
    default:
      return launch_gdn_c<1, false>(a, st, pdl);
  }
}

}  // namespace iam

using namespace iam;

extern "C" int iam_gdn_step_fused(const uint16_t* qkvzab, int ld_in, int z_col, int a_col, int b_col,
                                  const uint16_t* conv_w, const uint16_t* conv_in, uint16_t* conv_out,
                                  const float* A_log, const uint16_t* dt_bias, const uint16_t* norm_w, float* S,
                                  uint16_t* out, int ld_out, int n_k_heads, int n_v_heads, int rows, float eps,
                                  void* stream) {
  IAM_CHECK(qkvzab && conv_w && conv_in && conv_out && A_log && dt_bias && norm_w && S && out,
            "iam_gdn_step_fused: null pointer");
  GdnArgs a = {};
  a.in = qkvzab;
  a.ld_in = ld_in;
  a.z_col = z_col;
  a.a_col = a_col;
  a.b_col = b_col;
  a.conv_w = conv_w;
  a.conv_in = conv_in;
  a.conv_out = conv_out;
  a.A_log = A_log;
  a.dt_bias = dt_bias;
  a.norm_w = norm_w;
  a.S = S;
  a.out = out;
  a.ld_out = ld_out;
  a.n_k_heads = n_k_heads;
  a.n_v_heads = n_v_heads;
  a.key_dim = n_k_heads * kHD;
  a.conv_dim = 2 * n_k_heads * kHD + n_v_heads * kHD;
  a.rows = rows;
  a.eps = eps;
  return launch_gdn(a, as_stream(stream), false);
}

extern "C" int iam_gated_delta_step(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* g,
                                    const uint16_t* beta, float* S, uint16_t* y, int n_v_heads, int n_k_heads, int dk,
                                    int dv, int rows, void* stream) {
  IAM_CHECK(q && k && v && g && beta && S && y, "iam_gated_delta_step: null pointer");
  IAM_CHECK(dk == kHD && dv == kHD, "iam_gated_delta_step: dk == dv == 128 required");
  IAM_CHECK(n_k_heads > 0 && n_v_heads % n_k_heads == 0 && rows > 0, "iam_gated_delta_step: bad head counts");
  IAM_CHECK(aligned16(S), "iam_gated_delta_step: S must be 16-byte aligned");
  const int r = ensure_attrs();
  if (r != IAM_OK) return r;
  return launch_k(gated_delta_kernel, dim3(n_v_heads), dim3(kThreads), sizeof(GdnSmem), as_stream(stream), false,
                  q, k, v, g, beta, S, y, n_v_heads, n_k_heads, rows);
}
