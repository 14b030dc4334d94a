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

namespace iam {
namespace {

constexpr int kHeadDim = 256;
constexpr int kChunkTok = 32;
constexpr int kKvStride = kHeadDim + 8;  // padded smem row (bf16 elements)

__device__ __forceinline__ int cur_pos(const AttnArgs& a) { return a.pos_dev ? *a.pos_dev : a.pos; }

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  f[0] = lo_bf(v.x); f[1] = hi_bf(v.x); f[2] = lo_bf(v.y); f[3] = hi_bf(v.y);
  f[4] = lo_bf(v.z); f[5] = hi_bf(v.z); f[6] = lo_bf(v.w); f[7] = hi_bf(v.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf2(f[0], f[1]), pack_bf2(f[2], f[3]), pack_bf2(f[4], f[5]), pack_bf2(f[6], f[7]));
}

// ---------------------------------------------------------------- prep
__global__ void __launch_bounds__(256) attn_prep_kernel(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y * 8 + warp;
  if (head >= a.n_heads + a.n_kv_heads) return;
  const bool is_q = head < a.n_heads;
  const int kvh = head - a.n_heads;
  const int pos = cur_pos(a) + t;
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
    const size_t off = (static_cast<size_t>(pos) * a.n_kv_heads + kvh) * kHeadDim + 8 * lane;
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

__global__ void __launch_bounds__(256) attn_decode_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(smem_raw);
  pdl_wait();
  pdl_trigger();
  const int split = blockIdx.x, kvh = blockIdx.y, t0 = blockIdx.z * kRowBlock;
  const int rep = a.n_heads / a.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nrows = min(kRowBlock, a.rows - t0);
  const int npairs = nrows * rep;
  const int pos0 = cur_pos(a);
  // the block's longest context decides its chunk range; shorter rows mask
  const int last_max = min(pos0 + t0 + nrows - 1, a.max_ctx - 1);
  const int nch = last_max / kChunkTok + 1;
  const int c_begin = static_cast<int>((static_cast<long long>(split) * nch) / a.nsplit);
  const int c_end = static_cast<int>((static_cast<long long>(split + 1) * nch) / a.nsplit);
  for (int i = threadIdx.x; i < npairs * (kHeadDim / 8); i += blockDim.x) {
    const int pr = i / (kHeadDim / 8), d8 = (i % (kHeadDim / 8)) * 8;
    const int t = t0 + pr / rep, h = kvh * rep + pr % rep;
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
        kk = *reinterpret_cast<const uint4*>(a.k_cache + off);
        vv = *reinterpret_cast<const uint4*>(a.v_cache + off);
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
      const int t = t0 + pr / rep, h = kvh * rep + pr % rep;
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

// ---------------------------------------------------------------- combine + gate
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 8 + warp;
  if (h >= a.n_heads) return;
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
#pragma unroll 8
  for (int c = 0; c < ns; ++c) {
    const float sc = __shfl_sync(0xffffffffu, c < 32 ? sc0 : sc1, c & 31);
    if (sc == 0.f) continue;
    const float4* po = reinterpret_cast<const float4*>(a.part_o + (base + c) * kHeadDim + 8 * lane);
    const float4 x0 = po[0], x1 = po[1];
    o[0] = fmaf(x0.x, sc, o[0]); o[1] = fmaf(x0.y, sc, o[1]); o[2] = fmaf(x0.z, sc, o[2]); o[3] = fmaf(x0.w, sc, o[3]);
    o[4] = fmaf(x1.x, sc, o[4]); o[5] = fmaf(x1.y, sc, o[5]); o[6] = fmaf(x1.z, sc, o[6]); o[7] = fmaf(x1.w, sc, o[7]);
  }
  float r[8];
  if (a.qkv) {  // attention output gate: the second half of each head's q_proj row
    float gate[8];
    unpack8(*reinterpret_cast<const uint4*>(a.qkv + static_cast<size_t>(t) * a.ld_qkv +
                                            static_cast<size_t>(h) * 2 * kHeadDim + kHeadDim + 8 * lane),
            gate);
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = round_bf(o[i] / l) * sigmoid_f(gate[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = o[i] / l;
  }
  *reinterpret_cast<uint4*>(a.out + static_cast<size_t>(t) * a.ld_out + h * kHeadDim + 8 * lane) = pack8(r);
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
  return launch_k(attn_prep_kernel, dim3(a.rows, (a.n_heads + a.n_kv_heads + 7) / 8), dim3(256), 0, st, pdl, a);
}

int attn_init_attrs() {
  if (!g_attn_attr) {
    IAM_CUDA(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(DecodeSmem)));
    g_attn_attr = true;
  }
  return IAM_OK;
}

int launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl) {
  IAM_CHECK(a.n_heads % a.n_kv_heads == 0 && a.n_heads / a.n_kv_heads <= 8, "attention: GQA group of at most 8");
  const int r = attn_init_attrs();
  if (r != IAM_OK) return r;
  IAM_CHECK(a.nsplit >= 1 && a.nsplit <= 64, "attention: 1..64 context splits");
  return launch_k(attn_decode_kernel, dim3(a.nsplit, a.n_kv_heads, (a.rows + kRowBlock - 1) / kRowBlock), dim3(256),
                  sizeof(DecodeSmem), st, pdl, a);
}

int launch_attn_combine(const AttnArgs& a, cudaStream_t st, bool pdl) {
  return launch_k(attn_combine_kernel, dim3(a.rows, (a.n_heads + 7) / 8), dim3(256), 0, st, pdl, a);
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
