// W4A16 matmul for decode and verify widths on sm_100a.
//
// y[m, n] = sum_k x[m, k] * (q[n, k] * s[n, k/64] + b[n, k/64]) on MLX-packed
// weights (uint32 [N, K/8], low nibble first; bf16 scales/biases [N, K/64]),
// the operation of MLX's affine_qmm_t kernel as the reference dispatches it
// (full_forward.swift:711-728, batch_verify_27b.swift:100-119).
//
// Design (HBM-bound at verify widths <= 32):
//  * each warp owns 16 weight rows and a contiguous range of 64-wide groups;
//    thread (g, t) of the warp streams words 2t, 2t+1 of rows g and g+8 of
//    every group (8-byte loads, L1 bypassed, 256-byte L2 prefetch), four
//    groups in flight;
//  * dequantisation in registers, three instructions per pair of codes:
//    (w >> 4s) & 0x000F000F | 0x43004300 is the bf16 pair (128 + q_s,
//    128 + q_{s+4}); a packed bf16 FMA removes the 128 exactly and a second one
//    gives bf16(q * scale + bias) with a single rounding — the bf16 weight that
//    mx.dequantize (and so the reference's qmm) multiplies with;
//  * the tensor core (mma.sync m16n8k16, bf16 in, fp32 accumulate) consumes
//    the pairs straight from registers.  The code pairs (s, s+4) of a word fill
//    one A register, so the k order inside a group is permuted; the B fragments
//    are built with the same permutation (PRMT of 16 contiguous activations per
//    thread), which leaves the sum unchanged;
//  * warps splitting K reduce through shared memory; the epilogue applies
//    residual add, SwiGLU or an argmax partial in registers.
#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>

#include "kernels.cuh"
#include "tma.cuh"

namespace iam {
namespace {

constexpr uint32_t kMagic = 0x43004300u;    // bf16 pair (128, 128)
constexpr uint32_t kNibMask = 0x000F000Fu;  // codes s and s+4 of a word after >> 4s
constexpr uint32_t kOne = 0x3F803F80u;      // bf16 pair (1, 1)
constexpr uint32_t kNeg128 = 0xC300C300u;   // bf16 pair (-128, -128)

__device__ __forceinline__ uint32_t fma_bf2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Codes s and s+4 of a (pre-shifted) word -> the bf16 pair bf16(q*scale + bias):
// (w & 0x000F000F) | 0x43004300 is (128+q0, 128+q1) exactly; subtracting 128 is
// exact; one fused multiply-add rounds q*scale + bias to bf16 once, the value
// mx.dequantize produces.
__device__ __forceinline__ uint32_t dequant2(uint32_t w, uint32_t s2, uint32_t b2) {
  const uint32_t v = lop3_and_or(w, kNibMask, kMagic);
  return fma_bf2(fma_bf2(v, kOne, kNeg128), s2, b2);
}

struct WSlot {
  uint2 a;      // row g: words 2t, 2t+1 of the group
  uint2 b;      // row g+8 (SwiGLU: the up row of the same feature)
  uint32_t sa;  // row g: scale | bias << 16
  uint32_t sb;  // row g+8
};

__device__ __forceinline__ uint32_t ld_u16(const uint16_t* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}


// x chunk in shared memory: for each staged token, for each 64-group of the
// chunk, 32 words in B-fragment order [t][s][h]: word (t, s, h) holds the bf16
// pair (x[16t + 8h + s], x[16t + 8h + s + 4]) of the group.
constexpr int kUnitsPerThread = 4;  // 32-byte x units a thread stages per chunk (register budget)

struct XStage {
  uint4 v[kUnitsPerThread][2];
};

__device__ __forceinline__ void x_load(const QmmArgs& A, XStage& st, int tok0, int mt, int g0, int cg, int nthreads) {
  const int units = mt * cg * 4;
#pragma unroll
  for (int u = 0; u < kUnitsPerThread; ++u) {
    const int i = threadIdx.x + u * nthreads;
    if (i < units) {
      const int tok = i / (cg * 4), rem = i - tok * (cg * 4);
      const int gl = rem >> 2, tt = rem & 3;
      const uint16_t* src = A.x + static_cast<size_t>(tok0 + tok) * A.ldx + (g0 + gl) * 64 + 16 * tt;
      st.v[u][0] = ld_nc_u4(src);
      st.v[u][1] = ld_nc_u4(src + 8);
    }
  }
}

__device__ __forceinline__ void x_store(const XStage& st, unsigned char* buf, int mt, int cg, int tstride,
                                        int nthreads) {
  const int units = mt * cg * 4;
#pragma unroll
  for (int u = 0; u < kUnitsPerThread; ++u) {
    const int i = threadIdx.x + u * nthreads;
    if (i < units) {
      const int tok = i / (cg * 4), rem = i - tok * (cg * 4);
      const int gl = rem >> 2, tt = rem & 3;
      const uint4 v0 = st.v[u][0], v1 = st.v[u][1];
      uint4 o0, o1;
      o0.x = prmt(v0.x, v0.z, 0x5410u);  // s=0, h=0
      o0.y = prmt(v1.x, v1.z, 0x5410u);  // s=0, h=1
      o0.z = prmt(v0.x, v0.z, 0x7632u);  // s=1
      o0.w = prmt(v1.x, v1.z, 0x7632u);
      o1.x = prmt(v0.y, v0.w, 0x5410u);  // s=2
      o1.y = prmt(v1.y, v1.w, 0x5410u);
      o1.z = prmt(v0.y, v0.w, 0x7632u);  // s=3
      o1.w = prmt(v1.y, v1.w, 0x7632u);
      uint4* dst = reinterpret_cast<uint4*>(buf + static_cast<size_t>(tok) * tstride + gl * 128 + tt * 32);
      dst[0] = o0;
      dst[1] = o1;
    }
  }
}

// Stages a whole chunk, any number of units (used for the first chunk).
__device__ __forceinline__ void x_stage_all(const QmmArgs& A, unsigned char* buf, int tok0, int mt, int g0, int cg,
                                            int tstride, int nthreads) {
  for (int i = threadIdx.x; i < mt * cg * 4; i += nthreads) {
    const int tok = i / (cg * 4), rem = i - tok * (cg * 4);
    const int gl = rem >> 2, tt = rem & 3;
    const uint16_t* src = A.x + static_cast<size_t>(tok0 + tok) * A.ldx + (g0 + gl) * 64 + 16 * tt;
    const uint4 v0 = ld_nc_u4(src), v1 = ld_nc_u4(src + 8);
    uint4 o0, o1;
    o0.x = prmt(v0.x, v0.z, 0x5410u);
    o0.y = prmt(v1.x, v1.z, 0x5410u);
    o0.z = prmt(v0.x, v0.z, 0x7632u);
    o0.w = prmt(v1.x, v1.z, 0x7632u);
    o1.x = prmt(v0.y, v0.w, 0x5410u);
    o1.y = prmt(v1.y, v1.w, 0x5410u);
    o1.z = prmt(v0.y, v0.w, 0x7632u);
    o1.w = prmt(v1.y, v1.w, 0x7632u);
    uint4* dst = reinterpret_cast<uint4*>(buf + static_cast<size_t>(tok) * tstride + gl * 128 + tt * 32);
    dst[0] = o0;
    dst[1] = o1;
  }
}

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
__device__ __forceinline__ float4 ld_cg_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
  return r;
}

// Split-K reduction (partial sums meet in an fp32 workspace; the last CTA of
// a row block applies the epilogue and leaves the workspace zeroed again) and
// the fused epilogue.  Every thread of the CTA must call it.
template <int NT, int RT>
__device__ __forceinline__ void qmm_finish(const QmmArgs& A, const QmmSeg& S, float (&acc)[NT][4], int mode, int r0,
                                           int r1, int rt, int lane, int g, int t, int tok0, int cta_local) {
  const int KS = gridDim.z;
  const int bx = blockIdx.x;
  if (KS > 1) {
    float* wsp = A.ws + (static_cast<size_t>(blockIdx.y) * A.ws_blocks + bx) * (RT * NT * 128) +
                 static_cast<size_t>(rt) * (NT * 128) + lane * 4;
#pragma unroll
    for (int j = 0; j < NT; ++j) red_add_v4(wsp + j * 128, acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) {
      int* ctr = A.counters + static_cast<size_t>(blockIdx.y) * A.ws_blocks + bx;
      last = atomicAdd(ctr, 1) == KS - 1;
      if (last) *ctr = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const float4 v = ld_cg_f4(wsp + j * 128);
      acc[j][0] = v.x;
      acc[j][1] = v.y;
      acc[j][2] = v.z;
      acc[j][3] = v.w;
      *reinterpret_cast<float4*>(wsp + j * 128) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  // ---- epilogue
  if (mode == EPI_ARGMAX) {
    __shared__ unsigned long long kbuf[RT][8 * NT];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        unsigned long long k = 0ull;
        if (r0 < S.rows) k = argmax_key(round_bf(acc[j][e]), static_cast<uint32_t>(S.col_base + r0));
        if (r1 < S.rows) {
          const unsigned long long k1 = argmax_key(round_bf(acc[j][2 + e]), static_cast<uint32_t>(S.col_base + r1));
          k = k1 > k ? k1 : k;
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
          k = other > k ? other : k;
        }
        if (g == 0) kbuf[rt][8 * j + 2 * t + e] = k;
      }
    __syncthreads();
    if (threadIdx.x < 8 * NT) {
      const int tok = tok0 + threadIdx.x;
      if (tok < A.M) {
        unsigned long long k = kbuf[0][threadIdx.x];
#pragma unroll
        for (int q = 1; q < RT; ++q) k = kbuf[q][threadIdx.x] > k ? kbuf[q][threadIdx.x] : k;
        S.keys[static_cast<size_t>(cta_local) * S.key_ld + tok] = k;
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int tok = tok0 + 8 * j + 2 * t + e;
      if (tok >= A.M) continue;
      const float v0 = acc[j][e], v1 = acc[j][2 + e];
      if (mode == EPI_F32) {
        float* frow = S.out32 + static_cast<size_t>(tok) * S.ldo;
        if (r0 < S.rows) frow[r0] = v0;
        if (r1 < S.rows) frow[r1] = v1;
        continue;
      }
      uint16_t* orow = S.out + static_cast<size_t>(tok) * S.ldo;
      if (mode == EPI_SWIGLU) {
        if (r0 < S.rows) orow[r0] = f2bf(silu_f(round_bf(v0)) * round_bf(v1));
      } else if (mode == EPI_RESID) {
        const uint16_t* rrow = S.resid + static_cast<size_t>(tok) * S.ldr;
        if (r0 < S.rows) orow[r0] = f2bf(bf2f(rrow[r0]) + round_bf(v0));
        if (r1 < S.rows) orow[r1] = f2bf(bf2f(rrow[r1]) + round_bf(v1));
      } else {
        if (r0 < S.rows) orow[r0] = f2bf(v0);
        if (r1 < S.rows) orow[r1] = f2bf(v1);
      }
    }
}

template <int NT, int RT, int KP>
__global__ void __launch_bounds__(32 * RT) qmm_w4a16_kernel(const __grid_constant__ QmmArgs A) {
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr int kThreads = 32 * RT;
  const int bx = blockIdx.x;
  int si = 0;
#pragma unroll
  for (int i = 1; i < kQmmMaxSeg; ++i)
    if (i < A.nseg && bx >= A.seg[i].cta_begin) si = i;
  const QmmSeg& S = A.seg[si];
  const int mode = S.mode;

  const int rt = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int cta_local = bx - S.cta_begin;
  const int tile = cta_local * RT + rt;
  const int K = A.K, G = K >> 6, KWORDS = K >> 3;
  const int tok0 = blockIdx.y * (8 * NT);
  const int mt = min(8 * NT, A.M - tok0);
  const int KS = gridDim.z, ks = blockIdx.z;
  const int gb = (ks * G) / KS, ge = ((ks + 1) * G) / KS, ng = ge - gb;
  const int cgmax = A.chunk;  // groups per staged x chunk
  const int tstride = cgmax * 128 + 16;
  const size_t xbuf_bytes = static_cast<size_t>(A.xrows) * tstride;

  // ---- the two weight rows this thread streams
  int r0, r1;
  const uint32_t *w0, *w1;
  const uint16_t *s0p, *b0p, *s1p, *b1p;
  if (mode == EPI_SWIGLU) {
    r0 = r1 = tile * 8 + g;
    const size_t fc = static_cast<size_t>(min(r0, S.rows - 1));
    w0 = S.w + fc * KWORDS;
    w1 = S.w2 + fc * KWORDS;
    s0p = S.s + fc * G;
    b0p = S.b + fc * G;
    s1p = S.s2 + fc * G;
    b1p = S.b2 + fc * G;
  } else {
    r0 = tile * 16 + g;
    r1 = r0 + 8;
    const size_t c0 = static_cast<size_t>(min(r0, S.rows - 1));
    const size_t c1 = static_cast<size_t>(min(r1, S.rows - 1));
    w0 = S.w + c0 * KWORDS;
    w1 = S.w + c1 * KWORDS;
    s0p = S.s + c0 * G;
    b0p = S.b + c0 * G;
    s1p = S.s + c1 * G;
    b1p = S.b + c1 * G;
  }
  w0 += 2 * t;
  w1 += 2 * t;

  auto load_slot = [&](int gi) {
    WSlot s;
    s.a = ld_stream_u2(w0 + gi * 8);
    s.b = ld_stream_u2(w1 + gi * 8);
    s.sa = ld_u16(s0p + gi) | (ld_u16(b0p + gi) << 16);
    s.sb = ld_u16(s1p + gi) | (ld_u16(b1p + gi) << 16);
    return s;
  };

  // Weights do not depend on the preceding kernel: start streaming them
  // before waiting for it.
  WSlot ws[KP];
#pragma unroll
  for (int p = 0; p < KP; ++p)
    if (p < ng) ws[p] = load_slot(gb + p);
  pdl_wait();
  pdl_trigger();

  const int nchunks = (ng + cgmax - 1) / cgmax;
  // later chunks are staged through registers while the previous one is
  // consumed; the host keeps their size within kUnitsPerThread units a thread
  // (for NT == 1 the host keeps the whole k range in one chunk)
  constexpr bool kPipeX = NT > 1;
  XStage xst;
  x_stage_all(A, smem, tok0, mt, gb, min(cgmax, ng), tstride, kThreads);
  if (kPipeX && nchunks > 1) x_load(A, xst, tok0, mt, gb + cgmax, min(cgmax, ng - cgmax), kThreads);
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;
  bool xok[NT];
  int xoff[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    xok[j] = 8 * j + g < mt;
    xoff[j] = (xok[j] ? 8 * j + g : 0) * tstride + t * 32;
  }

  int gl = 0;  // group index inside the CTA's k range
  for (int c = 0; c < nchunks; ++c) {
    const unsigned char* xb = smem + (c & 1) * xbuf_bytes;
    const int cend = min(ng, (c + 1) * cgmax);
    for (; gl < cend; gl += KP) {
#pragma unroll
      for (int p = 0; p < KP; ++p) {
        const int gg = gl + p;
        if (gg < cend) {
          // chunks start on multiples of KP, so group gg lives in slot p
          const WSlot cur = ws[p];
          if (gg + KP < ng) ws[p] = load_slot(gb + gg + KP);
          const int cl = gg - c * cgmax;
          uint4 xb0[NT], xb1[NT];
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            if (xok[j]) {
              const uint4* q = reinterpret_cast<const uint4*>(xb + xoff[j] + cl * 128);
              xb0[j] = q[0];
              xb1[j] = q[1];
            } else {
              xb0[j] = make_uint4(0, 0, 0, 0);
              xb1[j] = make_uint4(0, 0, 0, 0);
            }
          }
          // (scale, scale) and (bias, bias) bf16 pairs of rows g and g+8
          const uint32_t s2a = prmt(cur.sa, cur.sa, 0x1010u), b2a = prmt(cur.sa, cur.sa, 0x3232u);
          const uint32_t s2b = prmt(cur.sb, cur.sb, 0x1010u), b2b = prmt(cur.sb, cur.sb, 0x3232u);
#pragma unroll
          for (int sb = 0; sb < 4; ++sb) {
            uint32_t a[4];
            a[0] = dequant2(cur.a.x >> (4 * sb), s2a, b2a);  // row g,   k 2t..2t+1
            a[1] = dequant2(cur.b.x >> (4 * sb), s2b, b2b);  // row g+8, k 2t..2t+1
            a[2] = dequant2(cur.a.y >> (4 * sb), s2a, b2a);  // row g,   k 2t+8..
            a[3] = dequant2(cur.b.y >> (4 * sb), s2b, b2b);  // row g+8, k 2t+8..
#pragma unroll
            for (int j = 0; j < NT; ++j) {
              const uint4& q = sb < 2 ? xb0[j] : xb1[j];
              mma_bf16_16816(acc[j], a, (sb & 1) ? q.z : q.x, (sb & 1) ? q.w : q.y, acc[j]);
            }
          }
        }
      }
    }
    gl = cend;
    if (kPipeX && c + 1 < nchunks) {
      // chunk c+1 was loaded into registers during chunk c; chunk c+2 goes next
      const int c1 = c + 1;
      x_store(xst, smem + (c1 & 1) * xbuf_bytes, mt, min(cgmax, ng - c1 * cgmax), tstride, kThreads);
      if (c1 + 1 < nchunks)
        x_load(A, xst, tok0, mt, gb + (c1 + 1) * cgmax, min(cgmax, ng - (c1 + 1) * cgmax), kThreads);
      __syncthreads();
    }
  }

  qmm_finish<NT, RT>(A, S, acc, mode, r0, r1, rt, lane, g, t, tok0, cta_local);
}

// ============================================================================
// TMA variant: each warp streams its 16 weight rows through a private ring of
// shared-memory stages.  A stage is 8 groups: two 16x128-byte boxes of packed
// codes (128B swizzle, so the fragment reads below are bank-conflict free) and
// 16x8 scales and biases, loaded by 2D tensor-map copies that complete on the
// stage's mbarrier.  Lane 0 re-arms a stage as soon as the warp has consumed
// it; the other lanes only dequantize and issue MMAs.
// ============================================================================
constexpr int kTmaStages = 2;
constexpr int kStageBytes = 5120;  // 4096 codes + 256 scales + 256 biases, padded to 1 KiB
constexpr uint32_t kStageTx = 4608;  // bytes a stage's copies deliver

template <int NT, int RT>
__global__ void __launch_bounds__(32 * RT) qmm_tma_kernel(const __grid_constant__ QmmTmaArgs T) {
  const QmmArgs& A = T.a;
  extern __shared__ __align__(16) unsigned char smem_tma[];
  // the 128B-swizzled boxes need 1 KiB-aligned destinations
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_tma) + 1023) & ~uintptr_t(1023));
  constexpr int kThreads = 32 * RT;
  const int bx = blockIdx.x;
  int si = 0;
#pragma unroll
  for (int i = 1; i < kQmmMaxSeg; ++i)
    if (i < A.nseg && bx >= A.seg[i].cta_begin) si = i;
  const QmmSeg& S = A.seg[si];
  const QmmTmaMaps& MP = T.maps[si];
  const int mode = S.mode;
  const bool swiglu = mode == EPI_SWIGLU;

  const int rt = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int cta_local = bx - S.cta_begin;
  const int tile = cta_local * RT + rt;
  const int r0 = swiglu ? tile * 8 + g : tile * 16 + g;
  const int r1 = swiglu ? r0 : r0 + 8;
  const int row_base = swiglu ? tile * 8 : tile * 16;  // first matrix row of this warp's boxes

  const int G = A.K >> 6, GB = G >> 3;
  const int tok0 = blockIdx.y * (8 * NT);
  const int mt = min(8 * NT, A.M - tok0);
  const int KS = gridDim.z, ks = blockIdx.z;
  const int bb = (ks * GB) / KS, nb = ((ks + 1) * GB) / KS - bb;  // 8-group blocks of this CTA
  const int gb = bb * 8, ng = nb * 8;

  unsigned char* ring = smem + rt * kTmaStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + RT * kTmaStages * kStageBytes) + rt * kTmaStages;
  unsigned char* xs = smem + RT * kTmaStages * kStageBytes + ((RT * kTmaStages * 8 + 127) / 128) * 128;

  auto issue = [&](int blk, int st) {  // lane 0 only
    const uint32_t bar = smem_addr(&bars[st]);
    const uint32_t dst = smem_addr(ring + st * kStageBytes);
    const int xw = (gb + blk * 8) * 32;  // byte column of the packed codes
    const int xg = gb + blk * 8;         // group column of scales / biases
    mbar_expect_tx(bar, kStageTx);
    if (swiglu) {
      tma_load_2d(dst, &MP.w, xw, row_base, bar);
      tma_load_2d(dst + 1024, &MP.w2, xw, row_base, bar);
      tma_load_2d(dst + 2048, &MP.w, xw + 128, row_base, bar);
      tma_load_2d(dst + 3072, &MP.w2, xw + 128, row_base, bar);
      tma_load_2d(dst + 4096, &MP.s, xg, row_base, bar);
      tma_load_2d(dst + 4096 + 128, &MP.s2, xg, row_base, bar);
      tma_load_2d(dst + 4352, &MP.b, xg, row_base, bar);
      tma_load_2d(dst + 4352 + 128, &MP.b2, xg, row_base, bar);
    } else {
      tma_load_2d(dst, &MP.w, xw, row_base, bar);
      tma_load_2d(dst + 2048, &MP.w, xw + 128, row_base, bar);
      tma_load_2d(dst + 4096, &MP.s, xg, row_base, bar);
      tma_load_2d(dst + 4352, &MP.b, xg, row_base, bar);
    }
  };

  // The weights do not depend on the preceding kernel: start the copies first.
  if (lane == 0) {
#pragma unroll
    for (int st = 0; st < kTmaStages; ++st) mbar_init(smem_addr(&bars[st]), 1);
    fence_mbar_init();
    for (int st = 0; st < kTmaStages && st < nb; ++st) issue(st, st);
  }
  __syncwarp();
  pdl_wait();
  pdl_trigger();  // the next kernel may start streaming its weights

  const int cgmax = A.chunk;
  const int tstride = cgmax * 128 + 16;
  const size_t xbuf_bytes = static_cast<size_t>(A.xrows) * tstride;
  const int nchunks = (ng + cgmax - 1) / cgmax;
  constexpr bool kPipeX = NT > 1;
  XStage xst;
  x_stage_all(A, xs, tok0, mt, gb, min(cgmax, ng), tstride, kThreads);
  if (kPipeX && nchunks > 1) x_load(A, xst, tok0, mt, gb + cgmax, min(cgmax, ng - cgmax), kThreads);
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;
  // fragment addresses inside a stage (128B swizzle: 16-byte chunk ^= row & 7):
  // group q of the stage sits in box q >> 2, chunk 2 (q & 3) + (t >> 1)
  int wofs[4];
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) wofs[q4] = g * 128 + (((2 * q4 + (t >> 1)) ^ (g & 7)) << 4) + (t & 1) * 8;
  // token rows past M read row 0: their MMA columns are never stored
  int xoff[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) xoff[j] = (8 * j + g < mt ? 8 * j + g : 0) * tstride + t * 32;
  const int sofs0 = 4096 + g * 16, sofs1 = 4096 + (g + 8) * 16;
  bool ok = true;

  int blk = 0;
  for (int c = 0; c < nchunks; ++c) {
    const unsigned char* xb = xs + (c & 1) * xbuf_bytes;
    const int bend = min(nb, ((c + 1) * cgmax) / 8);
    for (; blk < bend; ++blk) {
      const int st = blk % kTmaStages;
      if (ok && !mbar_wait(smem_addr(&bars[st]), (blk / kTmaStages) & 1)) {
        ok = false;
        if (A.err && lane == 0) atomicExch(A.err, IAM_ETIMEOUT);
      }
      __syncwarp();
      if (ok) {
        const unsigned char* sp = ring + st * kStageBytes;
        const unsigned char* xq = xb + (blk * 8 - c * cgmax) * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const unsigned char* wb = sp + (q >> 2) * 2048 + wofs[q & 3];
          const uint2 wa = *reinterpret_cast<const uint2*>(wb);         // row g:   words 2t, 2t+1
          const uint2 wc = *reinterpret_cast<const uint2*>(wb + 1024);  // row g+8
          const uint32_t sg = *reinterpret_cast<const uint16_t*>(sp + sofs0 + q * 2);
          const uint32_t bg = *reinterpret_cast<const uint16_t*>(sp + sofs0 + 256 + q * 2);
          const uint32_t sh = *reinterpret_cast<const uint16_t*>(sp + sofs1 + q * 2);
          const uint32_t bh = *reinterpret_cast<const uint16_t*>(sp + sofs1 + 256 + q * 2);
          // (s, s), (s/16, s/16) exact, (b, b) for rows g and g+8
          const uint32_t s2a = sg * 0x10001u, b2a = bg * 0x10001u;  // (s, s), (b, b) of row g
          const uint32_t s2b = sh * 0x10001u, b2b = bh * 0x10001u;  // row g+8
          uint4 xlo[NT], xhi[NT];
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const uint4* qx = reinterpret_cast<const uint4*>(xq + xoff[j] + q * 128);
            xlo[j] = qx[0];
            xhi[j] = qx[1];
          }
          // code pair (sb, sb+4) of each word after >> 4 sb
          uint32_t a[4][4];
#pragma unroll
          for (int sb = 0; sb < 4; ++sb) {
            a[sb][0] = dequant2(wa.x >> (4 * sb), s2a, b2a);  // row g,   k 2t..2t+1
            a[sb][1] = dequant2(wc.x >> (4 * sb), s2b, b2b);  // row g+8
            a[sb][2] = dequant2(wa.y >> (4 * sb), s2a, b2a);  // row g,   k 2t+8..
            a[sb][3] = dequant2(wc.y >> (4 * sb), s2b, b2b);  // row g+8
          }
#pragma unroll
          for (int sb = 0; sb < 4; ++sb)
#pragma unroll
            for (int j = 0; j < NT; ++j) {
              const uint4& qx = sb < 2 ? xlo[j] : xhi[j];
              mma_bf16_16816(acc[j], a[sb], (sb & 1) ? qx.z : qx.x, (sb & 1) ? qx.w : qx.y, acc[j]);
            }
        }
      }
      __syncwarp();  // every lane has read the stage before it is refilled
      if (ok && lane == 0 && blk + kTmaStages < nb) issue(blk + kTmaStages, st);
    }
    if (kPipeX && c + 1 < nchunks) {
      const int c1 = c + 1;
      x_store(xst, xs + (c1 & 1) * xbuf_bytes, mt, min(cgmax, ng - c1 * cgmax), tstride, kThreads);
      if (c1 + 1 < nchunks)
        x_load(A, xst, tok0, mt, gb + (c1 + 1) * cgmax, min(cgmax, ng - (c1 + 1) * cgmax), kThreads);
      __syncthreads();
    }
  }
  qmm_finish<NT, RT>(A, S, acc, mode, r0, r1, rt, lane, g, t, tok0, cta_local);
}

size_t qmm_tma_smem_bytes(const QmmArgs& a, const QmmConfig& c) {
  const int GB = a.K / 512;
  const int nb = (GB + c.ks - 1) / c.ks;
  const int ng = nb * 8;
  const int bufs = ng > c.chunk ? 2 : 1;
  return 1024 + static_cast<size_t>(c.rt) * kTmaStages * kStageBytes + ((c.rt * kTmaStages * 8 + 127) / 128) * 128 +
         static_cast<size_t>(bufs) * std::min(a.M, 8 * c.nt) * (c.chunk * 128 + 16);
}

template <int NT, int RT>
int launch_tma(const QmmTmaArgs& ta, const QmmConfig& c, cudaStream_t st, bool pdl) {
  const size_t smem = qmm_tma_smem_bytes(ta.a, c);
  if (smem > static_cast<size_t>(kQmmMaxSmem)) return fail(IAM_EINVAL, "qmm: TMA tile exceeds shared memory");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ta.a.total_ctas, (ta.a.M + 8 * NT - 1) / (8 * NT), c.ks);
  cfg.blockDim = dim3(32 * RT, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  IAM_CUDA(cudaLaunchKernelEx(&cfg, qmm_tma_kernel<NT, RT>, ta));
  return IAM_OK;
}

size_t qmm_smem_bytes(const QmmArgs& a, const QmmConfig& c) {
  const int G = a.K / 64;
  const int ng = (G + c.ks - 1) / c.ks;
  const int bufs = ng > c.chunk ? 2 : 1;
  return static_cast<size_t>(bufs) * std::min(a.M, 8 * c.nt) * (c.chunk * 128 + 16);
}

// groups per staged chunk: the whole k range when it fits one buffer,
// else chunks a thread stages in kUnitsPerThread 32-byte units (multiples of kp)
int qmm_chunk(int M, int nt, int rt, int kp, int ng) {
  const int rows = std::min(M, 8 * nt);
  if (static_cast<size_t>(rows) * (ng * 128 + 16) <= (nt == 1 ? 96 : 64) * 1024) return ng;
  // later chunks go through registers: at most kUnitsPerThread 32-byte units a thread
  int ch = (kUnitsPerThread * 32 * rt) / (rows * 4);
  ch = std::min(ch, 16) / kp * kp;
  return ch >= kp ? ch : -1;  // -1: this tile shape cannot stage x in chunks
}
template <int NT, int RT, int KP>
int launch_cfg(const QmmArgs& a, const QmmConfig& c, cudaStream_t st, bool pdl) {
  const size_t smem = qmm_smem_bytes(a, c);
  if (smem > static_cast<size_t>(kQmmMaxSmem)) return fail(IAM_EINVAL, "qmm: x chunk exceeds shared memory");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.total_ctas, (a.M + 8 * NT - 1) / (8 * NT), c.ks);
  cfg.blockDim = dim3(32 * RT, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  IAM_CUDA(cudaLaunchKernelEx(&cfg, qmm_w4a16_kernel<NT, RT, KP>, a));
  return IAM_OK;
}

// The kernel instances: (nt, rt, kp, tma)
struct Inst {
  int nt, rt, kp;
  bool tma;
  void* fn;
  int (*launch)(const QmmArgs&, const QmmConfig&, cudaStream_t, bool);
  int (*launch_t)(const QmmTmaArgs&, const QmmConfig&, cudaStream_t, bool);
};
#define IAM_QMM_INST(NT, RT, KP) \
  {NT, RT, KP, false, reinterpret_cast<void*>(qmm_w4a16_kernel<NT, RT, KP>), launch_cfg<NT, RT, KP>, nullptr}
#define IAM_QMM_TMA(NT, RT) \
  {NT, RT, 0, true, reinterpret_cast<void*>(qmm_tma_kernel<NT, RT>), nullptr, launch_tma<NT, RT>}
Inst g_inst[] = {
    IAM_QMM_INST(1, 4, 8), IAM_QMM_INST(1, 8, 8), IAM_QMM_INST(2, 4, 8), IAM_QMM_INST(2, 8, 8),
    IAM_QMM_INST(4, 4, 4), IAM_QMM_INST(4, 8, 4), IAM_QMM_TMA(1, 4),     IAM_QMM_TMA(1, 8),
    IAM_QMM_TMA(2, 4),     IAM_QMM_TMA(2, 8),     IAM_QMM_TMA(4, 4),     IAM_QMM_TMA(4, 8),
};
#undef IAM_QMM_INST
#undef IAM_QMM_TMA
bool g_attr_set[sizeof(g_inst) / sizeof(g_inst[0])] = {};

Inst* find_inst(int nt, int rt, bool tma) {
  for (auto& i : g_inst)
    if (i.nt == nt && i.rt == rt && i.tma == tma) return &i;
  return nullptr;
}

int g_num_sms = 0;

// Resident CTAs per SM of an instance with `smem` dynamic shared memory.
int occupancy(Inst& in, size_t smem) {
  const size_t idx = &in - g_inst;
  if (!g_attr_set[idx]) {
    cudaFuncSetAttribute(in.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kQmmMaxSmem);
    g_attr_set[idx] = true;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, in.fn, 32 * in.rt, smem) != cudaSuccess) n = 1;
  return std::max(1, n);
}

// IAM_QMM_CFG="rt,ks" or "rt,ks@K" (only for that K) overrides the plan.
bool env_override(QmmConfig& c, int K) {
  const char* v = std::getenv("IAM_QMM_CFG");
  if (!v) return false;
  int rt = 0, ks = 0, k = 0;
  const int n = std::sscanf(v, "%d,%d@%d", &rt, &ks, &k);
  if (n < 2 || (n == 3 && k != K)) return false;
  c.rt = rt;
  c.ks = ks;
  return true;
}

}  // namespace

// TMA needs 8-group blocks (K % 512) and 16-byte aligned operand bases.
bool tma_ok(const QmmArgs& a) {
  if (a.K % 512 != 0 || std::getenv("IAM_QMM_NO_TMA")) return false;
  for (int i = 0; i < a.nseg; ++i) {
    const QmmSeg& s = a.seg[i];
    if (!aligned16(s.w) || !aligned16(s.s) || !aligned16(s.b)) return false;
    if (s.mode == EPI_SWIGLU && (!aligned16(s.w2) || !aligned16(s.s2) || !aligned16(s.b2))) return false;
  }
  return true;
}

QmmConfig qmm_plan(QmmArgs& a) {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  QmmConfig c;
  c.nt = a.M <= 8 ? 1 : (a.M <= 16 ? 2 : 4);
  c.kp = c.nt == 4 ? 4 : 8;
  c.tma = tma_ok(a);
  const int G = a.K / 64;
  auto blocks = [&](int rt) {
    int n = 0;
    for (int i = 0; i < a.nseg; ++i) n += (a.seg[i].rows + qmm_rows_per_cta(a.seg[i].mode, rt) - 1) /
                                          qmm_rows_per_cta(a.seg[i].mode, rt);
    return n;
  };
  const int unit = c.tma ? 8 : 1;  // k splits fall on multiples of `unit` groups
  const int GU = G / unit;
  double best = 1e30;
  c.rt = 8;
  c.ks = 1;
  c.chunk = G;
  for (int rt : {4, 8}) {
    Inst* in = find_inst(c.nt, rt, c.tma);
    for (int ks = 1; ks <= 16; ++ks) {
      const int ng = ((GU + ks - 1) / ks) * unit;
      if (ks > 1 && ng < 4) break;
      const int chunk = qmm_chunk(a.M, c.nt, rt, c.tma ? 8 : c.kp, ng);
      if (chunk < 0) continue;
      if (c.nt == 1 && chunk < ng) continue;  // the narrow kernels stage their whole k range
      QmmConfig t{c.nt, rt, ks, c.kp, chunk, c.tma};
      const size_t smem = c.tma ? qmm_tma_smem_bytes(a, t) : qmm_smem_bytes(a, t);
      if (smem > static_cast<size_t>(kQmmMaxSmem)) continue;
      const int occ = occupancy(*in, smem);
      const long ctas = static_cast<long>(blocks(rt)) * ks * ((a.M + 8 * c.nt - 1) / (8 * c.nt));
      const long slots = static_cast<long>(g_num_sms) * occ;
      const long waves = (ctas + slots - 1) / slots;
      // Memory-bound: an SM streams ~75 group-warps per microsecond at the HBM
      // roofline once it holds enough loads in flight; each wave of CTAs also
      // pays a fixed prologue/epilogue latency (more with a split-K reduction).
      const double per_sm = std::ceil(static_cast<double>(std::min<long>(ctas, slots)) / g_num_sms);
      const double warps_sat = c.tma ? 12.0 : 48.0 * 1024 / (c.kp * 512.0);
      const double rate = std::min(1.0, per_sm * rt / warps_sat);
      const double per_group_us = (c.nt == 4 ? 1.6 : 1.0) / 75.0;  // wide tiles are issue-heavier
      const double cost = static_cast<double>(waves) * (per_sm * rt * ng * per_group_us / rate + 2.0 + (ks > 1 ? 1.5 : 0.0));
      if (cost < best - 1e-9) {
        best = cost;
        c.rt = rt;
        c.ks = ks;
        c.chunk = chunk;
      }
    }
  }
  if (env_override(c, a.K)) {
    const int ng = ((GU + c.ks - 1) / c.ks) * unit;
    c.chunk = qmm_chunk(a.M, c.nt, c.rt, c.tma ? 8 : c.kp, ng);
    if (c.chunk < 0) c.chunk = 0;  // rejected at launch
  }
  int cta = 0;
  for (int i = 0; i < a.nseg; ++i) {
    a.seg[i].cta_begin = cta;
    cta += (a.seg[i].rows + qmm_rows_per_cta(a.seg[i].mode, c.rt) - 1) / qmm_rows_per_cta(a.seg[i].mode, c.rt);
  }
  a.total_ctas = cta;
  a.chunk = c.chunk;
  a.xrows = std::min(a.M, 8 * c.nt);
  a.ws_blocks = cta;
  return c;
}

int qmm_launch(const QmmArgs& a, const QmmConfig& c, cudaStream_t st, bool pdl) {
  Inst* in = find_inst(c.nt, c.rt, c.tma);
  if (!in) return fail(IAM_EINVAL, "qmm: unsupported tile config");
  {
    const int G = a.K / 64, unit = c.tma ? 8 : 1;
    const int ng = ((G / unit + c.ks - 1) / c.ks) * unit;
    const int rows = std::min(a.M, 8 * c.nt);
    const bool piped = c.chunk < ng;
    if (c.chunk <= 0 || (piped && (c.nt == 1 || rows * c.chunk * 4 > kUnitsPerThread * 32 * c.rt ||
                                   c.chunk % (c.tma ? 8 : c.kp) != 0)))
      return fail(IAM_EINVAL, "qmm: x chunk does not fit the tile");
  }
  if (c.ks > 1 && (!a.ws || !a.counters)) return fail(IAM_EINVAL, "qmm: split-K needs a workspace");
  if (!c.tma) return in->launch(a, c, st, pdl);
  QmmTmaArgs ta;
  std::memset(&ta, 0, sizeof(ta));
  ta.a = a;
  const uint64_t K = static_cast<uint64_t>(a.K), G = K / 64;
  for (int i = 0; i < a.nseg; ++i) {
    const QmmSeg& s = a.seg[i];
    QmmTmaMaps& m = ta.maps[i];
    const uint32_t br = s.mode == EPI_SWIGLU ? 8 : 16;
    const uint64_t rows = static_cast<uint64_t>(s.rows);
    int r = tma_encode_2d(&m.w, s.w, 1, rows, K / 2, br, 128, true);
    if (r == IAM_OK) r = tma_encode_2d(&m.s, s.s, 2, rows, G, br, 8, false);
    if (r == IAM_OK) r = tma_encode_2d(&m.b, s.b, 2, rows, G, br, 8, false);
    if (r == IAM_OK && s.mode == EPI_SWIGLU) {
      r = tma_encode_2d(&m.w2, s.w2, 1, rows, K / 2, br, 128, true);
      if (r == IAM_OK) r = tma_encode_2d(&m.s2, s.s2, 2, rows, G, br, 8, false);
      if (r == IAM_OK) r = tma_encode_2d(&m.b2, s.b2, 2, rows, G, br, 8, false);
    }
    if (r != IAM_OK) return r;
  }
  return in->launch_t(ta, c, st, pdl);
}

size_t qmm_ws_floats(const QmmArgs& a, const QmmConfig& c) {
  return static_cast<size_t>((a.M + 8 * c.nt - 1) / (8 * c.nt)) * a.total_ctas * c.rt * c.nt * 128;
}
size_t qmm_ws_counters(const QmmArgs& a, const QmmConfig& c) {
  return static_cast<size_t>((a.M + 8 * c.nt - 1) / (8 * c.nt)) * a.total_ctas;
}

namespace {
// Split-K workspace of the operator-level entry points: library-owned, zeroed,
// grown on demand, one per (device, stream, kind), so calls on different
// streams never share one.  (The engine passes its own.)
struct OpWs {
  float* ws = nullptr;
  int* ctr = nullptr;
  size_t floats = 0, ctrs = 0;
};
// kind: the mma.sync kernels sum partials into a workspace they keep zeroed;
// the tensor-core kernel stores partials without clearing them, so the two
// never share one.
struct OpWsKey {
  int dev;
  cudaStream_t st;
  int kind;
  bool operator<(const OpWsKey& o) const {
    if (dev != o.dev) return dev < o.dev;
    if (st != o.st) return std::less<cudaStream_t>()(st, o.st);
    return kind < o.kind;
  }
};
std::mutex g_opws_mu;
std::map<OpWsKey, OpWs> g_opws;

}  // namespace

int qmm_op_workspace(int kind, size_t floats, size_t ctrs, cudaStream_t st, float** ws, int** ctr) {
  int dev = 0;
  IAM_CUDA(cudaGetDevice(&dev));
  IAM_CHECK(kind == 0 || kind == 1, "qmm: workspace kind");
  std::lock_guard<std::mutex> lock(g_opws_mu);
  OpWs& w = g_opws[OpWsKey{dev, st, kind}];
  if (w.floats < floats || w.ctrs < ctrs) {
    // the stream's earlier calls may still read the old workspace
    IAM_CUDA(cudaStreamSynchronize(st));
    cudaFree(w.ws);
    cudaFree(w.ctr);
    w = OpWs{};
    IAM_CUDA(cudaMalloc(&w.ws, floats * sizeof(float)));
    IAM_CUDA(cudaMalloc(&w.ctr, ctrs * sizeof(int)));
    IAM_CUDA(cudaMemsetAsync(w.ws, 0, floats * sizeof(float), st));
    IAM_CUDA(cudaMemsetAsync(w.ctr, 0, ctrs * sizeof(int), st));
    w.floats = floats;
    w.ctrs = ctrs;
  }
  *ws = w.ws;
  *ctr = w.ctr;
  return IAM_OK;
}

// Validates one matmul and launches it in passes of at most 64 tokens (packed
// weights, tensor cores) or 32 (MLX layout, mma.sync).  A null
// a.ws selects the library's own split-K workspace.
int qmm_run(QmmArgs a, cudaStream_t st, bool pdl, size_t ws_floats_cap, size_t ws_ctr_cap) {
  IAM_CHECK(a.K > 0 && a.K % 64 == 0, "qmm: K must be a positive multiple of 64");
  IAM_CHECK(a.M >= 1, "qmm: M must be >= 1");
  if (a.norm_w)
    IAM_CHECK(a.seg[0].packed && a.M <= kGemvNormMaxM && a.M <= qmm_gemv_max_m() && aligned16(a.norm_w) &&
                  a.K % 256 == 0 && a.ldx % 8 == 0,
              "qmm: the fused RMSNorm needs packed weights and at most two tokens on the GEMV path");
  IAM_CHECK(a.nseg >= 1 && a.nseg <= kQmmMaxSeg, "qmm: 1..4 segments");
  IAM_CHECK(aligned16(a.x) && a.ldx % 8 == 0, "qmm: x must be 16-byte aligned with ldx % 8 == 0");
  bool packed = a.seg[0].packed != nullptr;
  for (int i = 1; i < a.nseg; ++i)
    IAM_CHECK((a.seg[i].packed != nullptr) == packed, "qmm: segments mix packed and MLX-layout weights");
  IAM_CHECK(a.npush >= 0 && a.npush <= kQmmMaxPeers, "qmm: 0..8 receive slots");
  if (a.npush > 0)
    IAM_CHECK(packed && a.nseg == 1 && a.seg[0].mode == EPI_F32, "qmm: pushing to peers needs one fp32 segment of packed weights");
  if (packed) {
    const int total_m = a.M;
    const uint16_t* x0 = a.x;
    for (int m0 = 0; m0 < total_m; m0 += 64) {  // the tensor-core kernel's widest token tile
      QmmArgs p = a;
      p.M = std::min(64, total_m - m0);
      p.x = x0 + static_cast<size_t>(m0) * a.ldx;
      for (int i = 0; i < p.nseg; ++i) {
        QmmSeg& s = p.seg[i];
        if (s.out) s.out += static_cast<size_t>(m0) * s.ldo;
        if (s.out32) s.out32 += static_cast<size_t>(m0) * s.ldo;
        if (s.resid) s.resid += static_cast<size_t>(m0) * s.ldr;
        if (s.keys) s.keys += m0;
      }
      for (int r = 0; r < p.npush; ++r) p.push[r] += static_cast<size_t>(m0) * a.seg[0].ldo;
      // narrow passes convert the weights in registers (mma.sync); wider ones
      // on the tensor cores
      const int r = p.M <= qmm_gemv_max_m() ? qmm_gemv_run(p, st, pdl, ws_floats_cap, ws_ctr_cap)
                                            : qmm_tc_run(p, st, pdl, ws_floats_cap, ws_ctr_cap);
      if (r != IAM_OK) return r;
    }
    return IAM_OK;
  }
  for (int i = 0; i < a.nseg; ++i) {
    const QmmSeg& s = a.seg[i];
    IAM_CHECK(s.rows > 0 && s.w && s.s && s.b, "qmm: segment without weights");
    IAM_CHECK(aligned16(s.w), "qmm: w must be 16-byte aligned");
    if (s.mode == EPI_SWIGLU) IAM_CHECK(s.w2 && s.s2 && s.b2 && aligned16(s.w2), "qmm: SwiGLU needs the up matrix");
    if (s.mode == EPI_ARGMAX) IAM_CHECK(s.keys != nullptr && s.key_ld >= 1, "qmm: argmax needs a key buffer");
    else if (s.mode == EPI_F32) IAM_CHECK(s.out32 != nullptr || a.npush > 0, "qmm: no fp32 output");
    else IAM_CHECK(s.out != nullptr, "qmm: no output");
    if (s.mode == EPI_RESID) IAM_CHECK(s.resid != nullptr, "qmm: residual input missing");
  }
  const int total_m = a.M;
  const uint16_t* x0 = a.x;
  for (int m0 = 0; m0 < total_m; m0 += 32) {
    QmmArgs p = a;
    p.M = std::min(32, total_m - m0);
    p.x = x0 + static_cast<size_t>(m0) * a.ldx;
    for (int i = 0; i < p.nseg; ++i) {
      QmmSeg& s = p.seg[i];
      if (s.out) s.out += static_cast<size_t>(m0) * s.ldo;
      if (s.out32) s.out32 += static_cast<size_t>(m0) * s.ldo;
      if (s.resid) s.resid += static_cast<size_t>(m0) * s.ldr;
      if (s.keys) s.keys += m0;
    }
    const QmmConfig c = qmm_plan(p);
    if (c.ks > 1) {
      const size_t nf = qmm_ws_floats(p, c), nc = qmm_ws_counters(p, c);
      if (!a.ws) {
        const int r = qmm_op_workspace(0, nf, nc, st, &p.ws, &p.counters);
        if (r != IAM_OK) return r;
      } else {
        IAM_CHECK(nf <= ws_floats_cap && nc <= ws_ctr_cap, "qmm: split-K workspace too small");
      }
    }
    const int r = qmm_launch(p, c, st, pdl);
    if (r != IAM_OK) return r;
  }
  return IAM_OK;
}

}  // namespace iam

extern "C" int iam_qmm_affine4(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x,
                               uint16_t* y, int M, int N, int K, int group_size, void* stream) {
  using namespace iam;
  IAM_CHECK(group_size == 64, "iam_qmm_affine4: group_size must be 64");
  IAM_CHECK(N > 0 && N % 8 == 0, "iam_qmm_affine4: N must be a positive multiple of 8");
  IAM_CHECK(w && s && b && x && y, "iam_qmm_affine4: null pointer");
  QmmArgs a = {};
  a.x = x;
  a.ldx = K;
  a.M = M;
  a.K = K;
  a.nseg = 1;
  a.seg[0].w = w;
  a.seg[0].s = s;
  a.seg[0].b = b;
  a.seg[0].out = y;
  a.seg[0].ldo = N;
  a.seg[0].rows = N;
  a.seg[0].mode = EPI_STORE;
  return qmm_run(a, as_stream(stream), false);
}

// ---------------------------------------------------------------- fixed scratch
// A variant of iam_qmm_affine4 for callers that cannot allocate device memory
// while they run it: a caller that manages all device memory itself (its own
// pool, nothing left to hand to cudaMalloc), or one inside a section where an
// allocation would synchronise the device or fail.  The split-K scratch is a
// fixed array inside the library image instead of the library's grown-on-demand
// workspace.
namespace iam {
namespace {
constexpr size_t kNoAllocFloats = static_cast<size_t>(1) << 20;  // 4 MiB of fp32 partial sums
constexpr size_t kNoAllocCounters = 16384;                        // one arrival counter a row block
// Both must be zero when a call starts.  They are zero when the module loads
// (static storage), the first call on a device clears them again, ordered on
// the caller's stream, and every call that completes leaves them zero (the
// last CTA of a row block clears what it summed).
__device__ __align__(256) float g_noalloc_ws[kNoAllocFloats];
__device__ __align__(256) int g_noalloc_ctr[kNoAllocCounters];
std::mutex g_noalloc_mu;
bool g_noalloc_cleared[64] = {};  // per device: the first call's clear was enqueued
}  // namespace
}  // namespace iam

extern "C" int iam_qmm_affine4_noalloc(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x,
                                       uint16_t* y, int M, int N, int K, int group_size, void* stream) {
  using namespace iam;
  IAM_CHECK(group_size == 64, "iam_qmm_affine4_noalloc: group_size must be 64");
  IAM_CHECK(N > 0 && N % 8 == 0, "iam_qmm_affine4_noalloc: N must be a positive multiple of 8");
  IAM_CHECK(M >= 1 && K > 0 && K % 64 == 0, "iam_qmm_affine4_noalloc: M >= 1 and K a positive multiple of 64");
  IAM_CHECK(w && s && b && x && y, "iam_qmm_affine4_noalloc: null pointer");
  int dev = 0;
  IAM_CUDA(cudaGetDevice(&dev));
  IAM_CHECK(dev >= 0 && dev < 64, "iam_qmm_affine4_noalloc: device index out of range");
  const cudaStream_t st = as_stream(stream);
  // The arrays' device addresses, looked up on every call: a host-side
  // lookup, and never stale after the device's context was re-created.
  float* ws = nullptr;
  int* ctr = nullptr;
  IAM_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&ws), g_noalloc_ws));
  IAM_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&ctr), g_noalloc_ctr));
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_cleared[dev]) {  // first call on this device: a stream-ordered clear, no allocation
      IAM_CUDA(cudaMemsetAsync(ws, 0, kNoAllocFloats * sizeof(float), st));
      IAM_CUDA(cudaMemsetAsync(ctr, 0, kNoAllocCounters * sizeof(int), st));
      g_noalloc_cleared[dev] = true;
    }
  }
  QmmArgs a = {};
  a.x = x;
  a.ldx = K;
  a.M = M;
  a.K = K;
  a.nseg = 1;
  a.seg[0].w = w;
  a.seg[0].s = s;
  a.seg[0].b = b;
  a.seg[0].out = y;
  a.seg[0].ldo = N;
  a.seg[0].rows = N;
  a.seg[0].mode = EPI_STORE;
  // the passes are of 32 tokens and a remainder: check both plans' scratch
  for (int pm : {std::min(M, 32), M % 32}) {
    if (pm == 0) continue;
    QmmArgs probe = a;
    probe.M = pm;
    const QmmConfig c = qmm_plan(probe);
    if (c.ks < 2) continue;
    const size_t nf = qmm_ws_floats(probe, c), nc = qmm_ws_counters(probe, c);
    if (nf > kNoAllocFloats || nc > kNoAllocCounters)
      return fail(IAM_EINVAL, "iam_qmm_affine4_noalloc: this shape needs " + std::to_string(nf) + " floats and " +
                                  std::to_string(nc) + " counters of split-K scratch; the fixed scratch holds " +
                                  std::to_string(kNoAllocFloats) + " and " + std::to_string(kNoAllocCounters));
  }
  a.ws = ws;
  a.counters = ctr;
  return qmm_run(a, st, false, kNoAllocFloats, kNoAllocCounters);
}

extern "C" int iam_qmm_affine4_plan(int M, int N, int K, int* splits, size_t* scratch_floats,
                                    size_t* scratch_counters) {
  using namespace iam;
  IAM_CHECK(N > 0 && N % 8 == 0 && M >= 1 && K > 0 && K % 64 == 0, "iam_qmm_affine4_plan: bad shape");
  IAM_CHECK(splits && scratch_floats && scratch_counters, "iam_qmm_affine4_plan: null output");
  QmmArgs a = {};
  a.ldx = K;
  a.K = K;
  a.nseg = 1;
  a.seg[0].rows = N;
  a.seg[0].mode = EPI_STORE;
  *splits = 1;
  *scratch_floats = 0;
  *scratch_counters = 0;
  // passes of 32 tokens and a remainder, as iam_qmm_affine4 runs them
  for (int pm : {std::min(M, 32), M % 32}) {
    if (pm == 0) continue;
    QmmArgs probe = a;
    probe.M = pm;
    const QmmConfig c = qmm_plan(probe);
    *splits = std::max(*splits, c.ks);
    if (c.ks < 2) continue;
    *scratch_floats = std::max(*scratch_floats, qmm_ws_floats(probe, c));
    *scratch_counters = std::max(*scratch_counters, qmm_ws_counters(probe, c));
  }
  return IAM_OK;
}
