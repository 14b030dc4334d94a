// Full-attention block of the decode / verify step (dispatchAttnLayer,
// full_forward.swift:828-987), in three kernels:
//  1. attn_prep: per-head RMSNorm of q and k (per_head_rms_norm_bf16), partial
//     RoPE on adjacent pairs (rope_bf16), KV-cache append of roped k and raw
//     v (copy_bf16) — one warp per (token, head);
//  2. attn_decode: split-context flash decode (sdpa_decode_bf16 without its
//     1024-token cap) — one CTA per (context split, KV head, token) walking
//     its 32-key chunks with an online softmax, one warp per query head of the
//     GQA group; a lane owns one key for the scores and 8 output dims for
//     P.V; causal inside the verify block;
//  3. attn_combine: merges the chunks' (max, sum, o) and applies the sigmoid
//     output gate (sigmoid_multiply_bf16, full_forward.swift:940-948).
#include <cmath>

#include "kernels.cuh"
#include "tma.cuh"

namespace iam {
namespace {

constexpr int kHeadDim = 256;
constexpr int kChunkTok = 32;
constexpr int kKvStride = kHeadDim + 8;  // padded smem row (bf16 elements)

// Position of row 0 of sequence sq (one sequence: sq = 0).
__device__ __forceinline__ int cur_pos(const AttnArgs& a, int sq = 0) { return a.pos_dev ? a.pos_dev[sq] : a.pos; }

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  f[0] = lo_bf(v.x); f[1] = hi_bf(v.x); f[2] = lo_bf(v.y); f[3] = hi_bf(v.y);
  f[4] = lo_bf(v.z); f[5] = hi_bf(v.z); f[6] = lo_bf(v.w); f[7] = hi_bf(v.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf2(f[0], f[1]), pack_bf2(f[2], f[3]), pack_bf2(f[4], f[5]), pack_bf2(f[6], f[7]));
}

// ---------------------------------------------------------------- prep
// kSeq: rows of several sequences (AttnArgs n_seq); row t belongs to sequence
// t / seq_rows, whose own position and caches it uses.
template <bool kSeq>
__global__ void __launch_bounds__(256) attn_prep_kernel(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y * 8 + warp;
  if (head >= a.n_heads + a.n_kv_heads) return;
  const bool is_q = head < a.n_heads;
  const int kvh = head - a.n_heads;
  int sq = 0, tt = t;
  if constexpr (kSeq) {
    sq = t / a.seq_rows;
    tt = t - sq * a.seq_rows;
  }
  const int pos = cur_pos(a, sq) + tt;
  if (pos < 0 || pos >= a.max_ctx) return;  // the host keeps pos + rows <= max_ctx
  const uint16_t* row = a.qkv + static_cast<size_t>(t) * a.ld_qkv;
  const uint16_t* src = is_q ? row + static_cast<size_t>(head) * 2 * kHeadDim : row + a.k_col + kvh * kHeadDim;
  float x[8];
  unpack8(*reinterpret_cast<const uint4*>(src + 8 * lane), x);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
  ss = warp_sum(ss);
  const float rms = sqrtf(ss / static_cast<float>(kHeadDim) + a.eps);
  float w[8];
  unpack8(*reinterpret_cast<const uint4*>((is_q ? a.q_norm_w : a.k_norm_w) + 8 * lane), w);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = round_bf((x[i] / rms) * w[i]);
  // RoPE on pairs (2i, 2i+1) with i < rotary/2: lane owns pairs 4*lane .. 4*lane+3
  if (8 * lane < a.rotary_dim) {
    const float* cs = a.rope_cs + static_cast<size_t>(pos) * a.rotary_dim;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int pi = 4 * lane + j;
      const float c = cs[2 * pi], s = cs[2 * pi + 1];
      const float x0 = x[2 * j], x1 = x[2 * j + 1];
      x[2 * j] = round_bf(x0 * c - x1 * s);
      x[2 * j + 1] = round_bf(x0 * s + x1 * c);
    }
  }
  if (is_q) {
    *reinterpret_cast<uint4*>(a.q_buf + (static_cast<size_t>(t) * a.n_heads + head) * kHeadDim + 8 * lane) = pack8(x);
  } else {
    size_t off = (static_cast<size_t>(pos) * a.n_kv_heads + kvh) * kHeadDim + 8 * lane;
    if constexpr (kSeq) off += static_cast<size_t>(sq) * a.seq_kv;
    *reinterpret_cast<uint4*>(a.k_cache + off) = pack8(x);
    *reinterpret_cast<uint4*>(a.v_cache + off) =
        *reinterpret_cast<const uint4*>(row + a.v_col + kvh * kHeadDim + 8 * lane);
  }
}

// ---------------------------------------------------------------- decode
// One CTA per (context split, KV head, block of kRowBlock verify rows): the
// split's 32-key chunks are staged once in shared memory and serve every
// (row, query head) pair of the block; warp w owns pairs w, w + 8, ...
constexpr int kRowBlock = 8;
constexpr int kMaxPairs = 8;  // pairs per warp: kRowBlock * 8 query heads / 8 warps

struct DecodeSmem {
  uint16_t k[kChunkTok][kKvStride];
  uint16_t v[kChunkTok][kKvStride];
  uint16_t q[kRowBlock * 8][kHeadDim];
};

// kSeq: grid.z = sequence x row block of the sequence (AttnArgs n_seq).
template <bool kSeq>
__global__ void __launch_bounds__(256) attn_decode_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(smem_raw);
  pdl_wait();
  pdl_trigger();
  int sq = 0, zb = blockIdx.z, srows = a.rows, rbase = 0;
  const uint16_t* kc = a.k_cache;
  const uint16_t* vc = a.v_cache;
  if constexpr (kSeq) {
    const int bps = (a.seq_rows + kRowBlock - 1) / kRowBlock;
    sq = blockIdx.z / bps;
    zb = blockIdx.z - sq * bps;
    srows = a.seq_rows;
    rbase = sq * a.seq_rows;
    kc += static_cast<size_t>(sq) * a.seq_kv;
    vc += static_cast<size_t>(sq) * a.seq_kv;
  }
  const int split = blockIdx.x, kvh = blockIdx.y, t0 = zb * kRowBlock;  // t0: row within the sequence
  const int rep = a.n_heads / a.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nrows = min(kRowBlock, srows - t0);
  const int npairs = nrows * rep;
  const int pos0 = cur_pos(a, sq);
  // the block's longest context decides its chunk range; shorter rows mask
  const int last_max = min(pos0 + t0 + nrows - 1, a.max_ctx - 1);
  const int nch = last_max / kChunkTok + 1;
  const int c_begin = static_cast<int>((static_cast<long long>(split) * nch) / a.nsplit);
  const int c_end = static_cast<int>((static_cast<long long>(split + 1) * nch) / a.nsplit);
  for (int i = threadIdx.x; i < npairs * (kHeadDim / 8); i += blockDim.x) {
    const int pr = i / (kHeadDim / 8), d8 = (i % (kHeadDim / 8)) * 8;
    const int t = rbase + t0 + pr / rep, h = kvh * rep + pr % rep;
    *reinterpret_cast<uint4*>(&sm.q[pr][d8]) =
        *reinterpret_cast<const uint4*>(a.q_buf + (static_cast<size_t>(t) * a.n_heads + h) * kHeadDim + d8);
  }
  float m_run[kMaxPairs], l_run[kMaxPairs], o[kMaxPairs][8];
#pragma unroll
  for (int pp = 0; pp < kMaxPairs; ++pp) {
    m_run[pp] = -INFINITY;
    l_run[pp] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[pp][i] = 0.f;
  }
  for (int c = c_begin; c < c_end; ++c) {
    const int p0 = c * kChunkTok;
    const int nstage = min(kChunkTok, last_max - p0 + 1);
    __syncthreads();  // previous chunk consumed (and q staged on the first pass)
    for (int i = threadIdx.x; i < kChunkTok * (kHeadDim / 8); i += blockDim.x) {
      const int r = i / (kHeadDim / 8), d8 = (i % (kHeadDim / 8)) * 8;
      uint4 kk = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (r < nstage) {
        const size_t off = (static_cast<size_t>(p0 + r) * a.n_kv_heads + kvh) * kHeadDim + d8;
        kk = *reinterpret_cast<const uint4*>(kc + off);
        vv = *reinterpret_cast<const uint4*>(vc + off);
      }
      *reinterpret_cast<uint4*>(&sm.k[r][d8]) = kk;
      *reinterpret_cast<uint4*>(&sm.v[r][d8]) = vv;
    }
    __syncthreads();
#pragma unroll
    for (int pp = 0; pp < kMaxPairs; ++pp) {
      const int pr = warp + 8 * pp;
      if (pr < npairs) {
        const int t = t0 + pr / rep;
        const int nvalid = min(kChunkTok, min(pos0 + t, a.max_ctx - 1) - p0 + 1);  // causal
        if (nvalid > 0) {
          float s = 0.f;  // lane = key
          for (int d = 0; d < kHeadDim; d += 8) {
            float kf[8], qf[8];
            unpack8(*reinterpret_cast<const uint4*>(&sm.k[lane][d]), kf);
            unpack8(*reinterpret_cast<const uint4*>(&sm.q[pr][d]), qf);
#pragma unroll
            for (int i = 0; i < 8; ++i) s = fmaf(qf[i], kf[i], s);
          }
          s *= 0.0625f;  // 1/sqrt(256)
          float mc = lane < nvalid ? s : -INFINITY;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
          const float m_new = fmaxf(m_run[pp], mc);
          const float keep = expf(m_run[pp] - m_new);  // 0 on the first chunk
          const float p = lane < nvalid ? expf(s - m_new) : 0.f;
          l_run[pp] = l_run[pp] * keep + warp_sum(p);
#pragma unroll
          for (int i = 0; i < 8; ++i) o[pp][i] *= keep;
          for (int j = 0; j < nvalid; ++j) {
            const float pj = __shfl_sync(0xffffffffu, p, j);
            float vf[8];
            unpack8(*reinterpret_cast<const uint4*>(&sm.v[j][8 * lane]), vf);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[pp][i] = fmaf(pj, vf[i], o[pp][i]);
          }
          m_run[pp] = m_new;
        }
      }
    }
  }
#pragma unroll
  for (int pp = 0; pp < kMaxPairs; ++pp) {
    const int pr = warp + 8 * pp;
    if (pr < npairs) {
      const int t = rbase + t0 + pr / rep, h = kvh * rep + pr % rep;
      const size_t part = (static_cast<size_t>(t) * a.n_heads + h) * a.nsplit + split;
      float4* po = reinterpret_cast<float4*>(a.part_o + part * kHeadDim + 8 * lane);
      po[0] = make_float4(o[pp][0], o[pp][1], o[pp][2], o[pp][3]);
      po[1] = make_float4(o[pp][4], o[pp][5], o[pp][6], o[pp][7]);
      if (lane == 0) {
        a.part_ml[2 * part] = m_run[pp];  // -inf when the split saw no key of this row
        a.part_ml[2 * part + 1] = l_run[pp];
      }
    }
  }
}

// ---------------------------------------------------------------- decode on tensor cores
// The same split-context decode for wide verify blocks, on mma.sync
// m16n8k16 (bf16 in, fp32 accumulate).  The (token, query head) pairs of a KV
// head form the rows of a small attention problem; one CTA takes 64 of them
// (four warps of 16) against the 64-key chunks of its context split:
// S = Q K^T and O += P V run on the tensor cores from padded shared memory
// (ldmatrix), the online softmax in registers; P is rounded to bf16 for the
// P V product, the row sums l use the unrounded p.  Partials go to the same
// (max, sum, o) slots as attn_decode_kernel and attn_combine_kernel merges them.
constexpr int kTcPairs = 64;              // query (token, head) rows a CTA
constexpr int kTcKeys = 64;               // keys a staged chunk
constexpr int kTcStride = kHeadDim + 8;   // padded smem row: ldmatrix without bank conflicts
constexpr size_t kTcSmem = static_cast<size_t>(3) * 64 * kTcStride * 2;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// kSeq: grid.z = sequence x 64-pair tile of the sequence (AttnArgs n_seq).
template <bool kSeq>
__global__ void __launch_bounds__(128, 1) attn_decode_tc_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint16_t* sq = reinterpret_cast<uint16_t*>(smem_raw);
  uint16_t* sk = sq + kTcPairs * kTcStride;
  uint16_t* sv = sk + kTcKeys * kTcStride;
  pdl_wait();
  pdl_trigger();
  const int rep = a.n_heads / a.n_kv_heads;
  int seq = 0, zb = blockIdx.z, srows = a.rows, rbase = 0;
  const uint16_t* kc = a.k_cache;
  const uint16_t* vc = a.v_cache;
  if constexpr (kSeq) {
    const int tps = (a.seq_rows * rep + kTcPairs - 1) / kTcPairs;
    seq = blockIdx.z / tps;
    zb = blockIdx.z - seq * tps;
    srows = a.seq_rows;
    rbase = seq * a.seq_rows;
    kc += static_cast<size_t>(seq) * a.seq_kv;
    vc += static_cast<size_t>(seq) * a.seq_kv;
  }
  const int split = blockIdx.x, kvh = blockIdx.y, p0 = zb * kTcPairs;  // pairs within the sequence
  const int npairs = srows * rep;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int pos0 = cur_pos(a, seq);
  const int t_hi = (min(p0 + kTcPairs, npairs) - 1) / rep;
  const int nkeys = min(pos0 + t_hi, a.max_ctx - 1) + 1;
  const int nch = (nkeys + kTcKeys - 1) / kTcKeys;
  const int c_begin = static_cast<int>((static_cast<long long>(split) * nch) / a.nsplit);
  const int c_end = static_cast<int>((static_cast<long long>(split + 1) * nch) / a.nsplit);
  // this lane's two rows (pairs) and their query positions (-1: no such row)
  const int r_lo = warp * 16 + g, r_hi = r_lo + 8;
  const int pl = p0 + r_lo, ph = p0 + r_hi;
  const int qpos_lo = pl < npairs ? min(pos0 + pl / rep, a.max_ctx - 1) : -1;
  const int qpos_hi = ph < npairs ? min(pos0 + ph / rep, a.max_ctx - 1) : -1;
  auto part_of = [&](int p) {
    const int t = rbase + p / rep, h = kvh * rep + p % rep;
    return (static_cast<size_t>(t) * a.n_heads + h) * a.nsplit + split;
  };
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  float o[32][4];
#pragma unroll
  for (int nd = 0; nd < 32; ++nd)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[nd][e] = 0.f;

  if (c_begin < c_end) {
    for (int i = threadIdx.x; i < kTcPairs * (kHeadDim / 8); i += blockDim.x) {
      const int r = i / (kHeadDim / 8), d8 = (i % (kHeadDim / 8)) * 8;
      const int p = p0 + r;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (p < npairs) {
        const int t = rbase + p / rep, h = kvh * rep + p % rep;
        v = *reinterpret_cast<const uint4*>(a.q_buf + (static_cast<size_t>(t) * a.n_heads + h) * kHeadDim + d8);
      }
      *reinterpret_cast<uint4*>(sq + r * kTcStride + d8) = v;
    }
    const uint32_t sq_a = smem_addr(sq), sk_a = smem_addr(sk), sv_a = smem_addr(sv);
    const int lr = lane & 7, lj = lane >> 3;  // ldmatrix: row in matrix, matrix index
    for (int c = c_begin; c < c_end; ++c) {
      const int kbase = c * kTcKeys;
      __syncthreads();  // previous chunk consumed (and q staged on the first pass)
      for (int i = threadIdx.x; i < kTcKeys * (kHeadDim / 8); i += blockDim.x) {
        const int r = i / (kHeadDim / 8), d8 = (i % (kHeadDim / 8)) * 8;
        uint4 kk = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (kbase + r < nkeys) {
          const size_t off = (static_cast<size_t>(kbase + r) * a.n_kv_heads + kvh) * kHeadDim + d8;
          kk = *reinterpret_cast<const uint4*>(kc + off);
          vv = *reinterpret_cast<const uint4*>(vc + off);
        }
        *reinterpret_cast<uint4*>(sk + r * kTcStride + d8) = kk;
        *reinterpret_cast<uint4*>(sv + r * kTcStride + d8) = vv;
      }
      __syncthreads();
      // S = Q K^T for the warp's 16 rows x 64 keys
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] = 0.f;
#pragma unroll 4
      for (int kk = 0; kk < kHeadDim / 16; ++kk) {
        uint32_t af[4];
        ldsm_x4(sq_a + 2 * ((warp * 16 + (lj & 1) * 8 + lr) * kTcStride + 16 * kk + (lj >> 1) * 8), af);
#pragma unroll
        for (int n2 = 0; n2 < 4; ++n2) {
          uint32_t bf[4];
          ldsm_x4(sk_a + 2 * ((16 * n2 + (lj >> 1) * 8 + lr) * kTcStride + 16 * kk + (lj & 1) * 8), bf);
          mma16816(sc[2 * n2], af, bf[0], bf[1]);
          mma16816(sc[2 * n2 + 1], af, bf[2], bf[3]);
        }
      }
      // scale, causal mask, online softmax (a row lives in the 4 lanes of a quad)
      float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = kbase + nt * 8 + 2 * tq + (e & 1);
          const int qp = e < 2 ? qpos_lo : qpos_hi;
          const float v = key <= qp ? sc[nt][e] * 0.0625f : -INFINITY;  // 1/sqrt(256)
          sc[nt][e] = v;
          if (e < 2) mx_lo = fmaxf(mx_lo, v);
          else mx_hi = fmaxf(mx_hi, v);
        }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
        mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
      }
      const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
      const float keep_lo = m_lo == -INFINITY ? 0.f : expf(m_lo - mn_lo);
      const float keep_hi = m_hi == -INFINITY ? 0.f : expf(m_hi - mn_hi);
      float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mref = e < 2 ? mn_lo : mn_hi;
          const float p = sc[nt][e] == -INFINITY ? 0.f : expf(sc[nt][e] - mref);
          sc[nt][e] = p;
          if (e < 2) sum_lo += p;
          else sum_hi += p;
        }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        sum_lo += __shfl_xor_sync(0xffffffffu, sum_lo, off);
        sum_hi += __shfl_xor_sync(0xffffffffu, sum_hi, off);
      }
      l_lo = l_lo * keep_lo + sum_lo;
      l_hi = l_hi * keep_hi + sum_hi;
      m_lo = mn_lo;
      m_hi = mn_hi;
#pragma unroll
      for (int nd = 0; nd < 32; ++nd) {
        o[nd][0] *= keep_lo;
        o[nd][1] *= keep_lo;
        o[nd][2] *= keep_hi;
        o[nd][3] *= keep_hi;
      }
      // O += P V: P (16 x 64, bf16) straight from the score registers
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t pa[4];
        pa[0] = pack_bf2(sc[2 * ks][0], sc[2 * ks][1]);
        pa[1] = pack_bf2(sc[2 * ks][2], sc[2 * ks][3]);
        pa[2] = pack_bf2(sc[2 * ks + 1][0], sc[2 * ks + 1][1]);
        pa[3] = pack_bf2(sc[2 * ks + 1][2], sc[2 * ks + 1][3]);
#pragma unroll
        for (int nd2 = 0; nd2 < 16; ++nd2) {
          uint32_t bf[4];
          ldsm_x4_t(sv_a + 2 * ((16 * ks + (lj & 1) * 8 + lr) * kTcStride + 16 * nd2 + (lj >> 1) * 8), bf);
          mma16816(o[2 * nd2], pa, bf[0], bf[1]);
          mma16816(o[2 * nd2 + 1], pa, bf[2], bf[3]);
        }
      }
    }
  }
  // partials: (max, sum) and the unnormalised output of each of the lane's rows
#pragma unroll
  for (int hl = 0; hl < 2; ++hl) {
    const int p = hl == 0 ? pl : ph;
    if (p >= npairs) continue;
    const size_t part = part_of(p);
    if (c_begin < c_end) {
      float* po = a.part_o + part * kHeadDim + 2 * tq;
#pragma unroll
      for (int nd = 0; nd < 32; ++nd)
        *reinterpret_cast<float2*>(po + nd * 8) = make_float2(o[nd][2 * hl], o[nd][2 * hl + 1]);
    }
    if (tq == 0) {
      a.part_ml[2 * part] = hl == 0 ? m_lo : m_hi;  // -inf when the split saw no key of this row
      a.part_ml[2 * part + 1] = hl == 0 ? l_lo : l_hi;
    }
  }
}

// ---------------------------------------------------------------- combine + gate
// One CTA per (row, query head): warp w merges the splits w, w + 8, ... of
// the head's partial outputs (each split's weight exp(m_i - max), from the
// partial maxima every warp reads), the eight warps' sums meet in shared
// memory and are added in warp order, then each thread finishes one of the
// head's 256 dimensions with the attention output gate.
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float part[8][kHeadDim];
  const int t = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = a.nsplit;  // <= 64
  const size_t base = (static_cast<size_t>(t) * a.n_heads + h) * ns;
  // lane i holds split i and i + 32: max, then each split's weight exp(m_i - max)
  const float m0 = lane < ns ? a.part_ml[2 * (base + lane)] : -INFINITY;
  const float m1 = lane + 32 < ns ? a.part_ml[2 * (base + lane + 32)] : -INFINITY;
  float mx = fmaxf(m0, m1);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float sc0 = m0 == -INFINITY ? 0.f : expf(m0 - mx);
  const float sc1 = m1 == -INFINITY ? 0.f : expf(m1 - mx);
  float l = (lane < ns ? a.part_ml[2 * (base + lane) + 1] * sc0 : 0.f) +
            (lane + 32 < ns ? a.part_ml[2 * (base + lane + 32) + 1] * sc1 : 0.f);
  l = warp_sum(l);
  float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int c = warp; c < ns; c += 8) {
    const float sc = __shfl_sync(0xffffffffu, c < 32 ? sc0 : sc1, c & 31);
    if (sc == 0.f) continue;
    const float4* po = reinterpret_cast<const float4*>(a.part_o + (base + c) * kHeadDim + 8 * lane);
    const float4 x0 = po[0], x1 = po[1];
    o[0] = fmaf(x0.x, sc, o[0]); o[1] = fmaf(x0.y, sc, o[1]); o[2] = fmaf(x0.z, sc, o[2]); o[3] = fmaf(x0.w, sc, o[3]);
    o[4] = fmaf(x1.x, sc, o[4]); o[5] = fmaf(x1.y, sc, o[5]); o[6] = fmaf(x1.z, sc, o[6]); o[7] = fmaf(x1.w, sc, o[7]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) part[warp][8 * lane + i] = o[i];
  __syncthreads();
  const int dim = threadIdx.x;  // 0 .. 255
  float acc = part[0][dim];
#pragma unroll
  for (int w = 1; w < 8; ++w) acc += part[w][dim];
  float r;
  if (a.qkv) {  // attention output gate: the second half of each head's q_proj row
    const float gate = bf2f(a.qkv[static_cast<size_t>(t) * a.ld_qkv + static_cast<size_t>(h) * 2 * kHeadDim + kHeadDim +
                                  dim]);
    r = round_bf(acc / l) * sigmoid_f(gate);
  } else {
    r = acc / l;
  }
  a.out[static_cast<size_t>(t) * a.ld_out + h * kHeadDim + dim] = f2bf(r);
}

// copy_bf16 x2 (full_forward.swift:384-392, 909-924): append rows of k and v.
__global__ void attn_append_kernel(const uint16_t* k_new, const uint16_t* v_new, uint16_t* kc, uint16_t* vc,
                                   int n_kv, int pos) {
  const int t = blockIdx.x;
  const size_t n = static_cast<size_t>(n_kv) * kHeadDim / 8;
  const uint4* ks = reinterpret_cast<const uint4*>(k_new + static_cast<size_t>(t) * n_kv * kHeadDim);
  const uint4* vs = reinterpret_cast<const uint4*>(v_new + static_cast<size_t>(t) * n_kv * kHeadDim);
  uint4* kd = reinterpret_cast<uint4*>(kc + static_cast<size_t>(pos + t) * n_kv * kHeadDim);
  uint4* vd = reinterpret_cast<uint4*>(vc + static_cast<size_t>(pos + t) * n_kv * kHeadDim);
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
    kd[i] = ks[i];
    vd[i] = vs[i];
  }
}

bool g_attn_attr = false;

// Split-context partials of the operator-level entry point: library-owned,
// grown on demand, one set per device.
struct OpScratch {
  float* o = nullptr;
  float* ml = nullptr;
  size_t parts = 0;
};
OpScratch g_scratch[64];

}  // namespace

int launch_attn_prep(const AttnArgs& a, cudaStream_t st, bool pdl) {
  IAM_CHECK(a.head_dim == kHeadDim, "attention: head_dim 256 required");
  IAM_CHECK(a.rotary_dim % 8 == 0 && a.rotary_dim <= kHeadDim, "attention: rotary_dim % 8 == 0 required");
  const dim3 grid(a.rows, (a.n_heads + a.n_kv_heads + 7) / 8);
  if (a.n_seq > 1) {
    IAM_CHECK(a.seq_rows >= 1 && a.rows == a.n_seq * a.seq_rows && a.pos_dev, "attention: sequence rows / positions");
    return launch_k(attn_prep_kernel<true>, grid, dim3(256), 0, st, pdl, a);
  }
  return launch_k(attn_prep_kernel<false>, grid, dim3(256), 0, st, pdl, a);
}

int attn_init_attrs() {
  if (!g_attn_attr) {
    for (auto* k : {attn_decode_kernel<false>, attn_decode_kernel<true>})
      IAM_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(DecodeSmem)));
    for (auto* k : {attn_decode_tc_kernel<false>, attn_decode_tc_kernel<true>})
      IAM_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTcSmem)));
    g_attn_attr = true;
  }
  return IAM_OK;
}

// Verify blocks with at least kTcMinPairs (token, query head) pairs per KV
// head take the tensor-core decode; narrower ones the warp-per-pair kernel.
constexpr int kTcMinPairs = 32;

int launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl) {
  IAM_CHECK(a.n_heads % a.n_kv_heads == 0 && a.n_heads / a.n_kv_heads <= 8, "attention: GQA group of at most 8");
  const int r = attn_init_attrs();
  if (r != IAM_OK) return r;
  IAM_CHECK(a.nsplit >= 1 && a.nsplit <= 64, "attention: 1..64 context splits");
  const int rep = a.n_heads / a.n_kv_heads;
  if (a.n_seq > 1) {  // pairs of one sequence per CTA
    IAM_CHECK(a.seq_rows >= 1 && a.rows == a.n_seq * a.seq_rows && a.pos_dev, "attention: sequence rows / positions");
    const int sp = a.seq_rows * rep;
    if (sp >= kTcMinPairs)
      return launch_k(attn_decode_tc_kernel<true>,
                      dim3(a.nsplit, a.n_kv_heads, a.n_seq * ((sp + kTcPairs - 1) / kTcPairs)), dim3(128), kTcSmem,
                      st, pdl, a);
    return launch_k(attn_decode_kernel<true>,
                    dim3(a.nsplit, a.n_kv_heads, a.n_seq * ((a.seq_rows + kRowBlock - 1) / kRowBlock)), dim3(256),
                    sizeof(DecodeSmem), st, pdl, a);
  }
  const int npairs = a.rows * rep;
  if (npairs >= kTcMinPairs)
    return launch_k(attn_decode_tc_kernel<false>, dim3(a.nsplit, a.n_kv_heads, (npairs + kTcPairs - 1) / kTcPairs),
                    dim3(128), kTcSmem, st, pdl, a);
  return launch_k(attn_decode_kernel<false>, dim3(a.nsplit, a.n_kv_heads, (a.rows + kRowBlock - 1) / kRowBlock),
                  dim3(256), sizeof(DecodeSmem), st, pdl, a);
}

int launch_attn_combine(const AttnArgs& a, cudaStream_t st, bool pdl) {
  IAM_CHECK(a.head_dim == kHeadDim, "attention combine: head_dim 256");
  return launch_k(attn_combine_kernel, dim3(a.rows, a.n_heads), dim3(256), 0, st, pdl, a);
}

int attn_chunk_tokens() { return kChunkTok; }

}  // namespace iam

using namespace iam;

extern "C" int iam_sdpa_decode_append(const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new,
                                      uint16_t* k_cache, uint16_t* v_cache, uint16_t* out, int rows, int pos,
                                      int n_q_heads, int n_kv_heads, int head_dim, int max_ctx, void* stream) {
  IAM_CHECK(q && k_new && v_new && k_cache && v_cache && out, "iam_sdpa_decode_append: null pointer");
  IAM_CHECK(head_dim == kHeadDim, "iam_sdpa_decode_append: head_dim 256 required");
  IAM_CHECK(rows > 0 && pos >= 0 && pos + rows <= max_ctx, "iam_sdpa_decode_append: pos + rows exceeds max_ctx");
  IAM_CHECK(n_kv_heads > 0 && n_q_heads % n_kv_heads == 0 && n_q_heads / n_kv_heads <= 8,
            "iam_sdpa_decode_append: GQA group of at most 8 query heads per KV head");
  IAM_CHECK(aligned16(q) && aligned16(k_new) && aligned16(v_new) && aligned16(k_cache) && aligned16(v_cache) &&
                aligned16(out),
            "iam_sdpa_decode_append: pointers must be 16-byte aligned");
  int dev = 0;
  IAM_CUDA(cudaGetDevice(&dev));
  IAM_CHECK(dev >= 0 && dev < 64, "iam_sdpa_decode_append: device index out of range");
  const int nchunk = std::min(64, (pos + rows + kChunkTok - 1) / kChunkTok);  // context splits
  const size_t parts = static_cast<size_t>(rows) * n_q_heads * nchunk;
  OpScratch& sc = g_scratch[dev];
  if (sc.parts < parts) {
    cudaStream_t st = as_stream(stream);
    IAM_CUDA(cudaStreamSynchronize(st));
    cudaFree(sc.o);
    cudaFree(sc.ml);
    sc.o = nullptr;
    sc.ml = nullptr;
    sc.parts = 0;
    IAM_CUDA(cudaMalloc(&sc.o, parts * kHeadDim * sizeof(float)));
    IAM_CUDA(cudaMalloc(&sc.ml, parts * 2 * sizeof(float)));
    sc.parts = parts;
  }
  cudaStream_t st = as_stream(stream);
  attn_append_kernel<<<rows, 256, 0, st>>>(k_new, v_new, k_cache, v_cache, n_kv_heads, pos);
  IAM_CUDA(cudaGetLastError());
  AttnArgs a = {};
  a.q_buf = const_cast<uint16_t*>(q);
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.part_o = sc.o;
  a.part_ml = sc.ml;
  a.out = out;
  a.ld_out = n_q_heads * kHeadDim;
  a.n_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.max_ctx = max_ctx;
  a.rows = rows;
  a.pos = pos;
  a.chunk = kChunkTok;
  a.nsplit = nchunk;
  int r = launch_attn_decode(a, st, false);
  if (r != IAM_OK) return r;
  return launch_attn_combine(a, st, false);
}
