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
//  * dequantisation is one LOP3 per pair of codes: (w >> 4s) & 0x000F000F |
//    0x43004300 is the bf16 pair (128 + q_s, 128 + q_{s+4}), exact;
//  * the tensor core (mma.sync m16n8k16, fp32 accumulate) forms, per group,
//    R = sum_k x_k (128 + q_k) and, with an all-ones A operand, Sx = sum_k x_k;
//    the group's contribution is s * R + (b - 128 s) * Sx in fp32.  The code
//    pairs (s, s+4) of a word fill one A register, so the k order inside a
//    group is permuted; the B fragments are built with the same permutation
//    (PRMT of 16 contiguous activations per thread), which leaves the sum
//    unchanged;
//  * warps splitting K reduce through shared memory; the epilogue applies
//    residual add, SwiGLU or an argmax partial in registers.
#include <algorithm>
#include <cstdlib>
#include <cstdio>

#include "qmm.cuh"

namespace iam {
namespace {

constexpr uint32_t kMagic = 0x43004300u;    // bf16 pair (128, 128)
constexpr uint32_t kNibMask = 0x000F000Fu;  // codes s and s+4 of a word after >> 4s
constexpr uint32_t kOnes = 0x3F803F80u;     // bf16 pair (1, 1)
constexpr int kPipe = 4;                    // weight groups in flight per warp

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

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

template <int NT, int RT, int KW>
__global__ void __launch_bounds__(32 * RT * KW) qmm_w4a16_kernel(const __grid_constant__ QmmArgs A) {
  pdl_wait();
  const int bx = blockIdx.x;
  int si = 0;
#pragma unroll
  for (int i = 1; i < kQmmMaxSeg; ++i)
    if (i < A.nseg && bx >= A.seg[i].cta_begin) si = i;
  const QmmSeg& S = A.seg[si];
  const int mode = S.mode;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rt = warp % RT, kw = warp / RT;
  const int g = lane >> 2, t = lane & 3;
  const int cta_local = bx - S.cta_begin;
  const int tile = cta_local * RT + rt;
  const int K = A.K, G = K >> 6, KWORDS = K >> 3;
  const int tok0 = blockIdx.y * (8 * NT);

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

  const int gb = (kw * G) / KW, ge = ((kw + 1) * G) / KW;

  // ---- activation rows: token tok0 + 8j + g feeds B fragments of n-tile j
  const uint16_t* xr[NT];
  bool xok[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int tok = tok0 + 8 * j + g;
    xok[j] = tok < A.M;
    xr[j] = A.x + static_cast<size_t>(xok[j] ? tok : 0) * A.ldx + 16 * t;
  }

  auto load_slot = [&](int gi) {
    WSlot s;
    s.a = ld_stream_u2(w0 + gi * 8);
    s.b = ld_stream_u2(w1 + gi * 8);
    s.sa = ld_u16(s0p + gi) | (ld_u16(b0p + gi) << 16);
    s.sb = ld_u16(s1p + gi) | (ld_u16(b1p + gi) << 16);
    return s;
  };

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;

  WSlot ws[kPipe];
#pragma unroll
  for (int p = 0; p < kPipe; ++p)
    if (gb + p < ge) ws[p] = load_slot(gb + p);

  uint4 xa[NT], xb[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    xa[j] = make_uint4(0, 0, 0, 0);
    xb[j] = make_uint4(0, 0, 0, 0);
    if (xok[j] && gb < ge) {
      xa[j] = ld_nc_u4(xr[j] + gb * 64);
      xb[j] = ld_nc_u4(xr[j] + gb * 64 + 8);
    }
  }

  const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};

  for (int base = gb; base < ge; base += kPipe) {
#pragma unroll
    for (int p = 0; p < kPipe; ++p) {
      const int gi = base + p;
      if (gi < ge) {
        uint4 cxa[NT], cxb[NT];
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          cxa[j] = xa[j];
          cxb[j] = xb[j];
          if (xok[j] && gi + 1 < ge) {
            xa[j] = ld_nc_u4(xr[j] + (gi + 1) * 64);
            xb[j] = ld_nc_u4(xr[j] + (gi + 1) * 64 + 8);
          }
        }
        const WSlot cur = ws[p];
        if (gi + kPipe < ge) ws[p] = load_slot(gi + kPipe);

        float R[NT][4], SX[NT][4];
#pragma unroll
        for (int sb = 0; sb < 4; ++sb) {
          uint32_t a[4];
          a[0] = lop3_and_or(cur.a.x >> (4 * sb), kNibMask, kMagic);  // row g,   k 2t..2t+1
          a[1] = lop3_and_or(cur.b.x >> (4 * sb), kNibMask, kMagic);  // row g+8, k 2t..2t+1
          a[2] = lop3_and_or(cur.a.y >> (4 * sb), kNibMask, kMagic);  // row g,   k 2t+8..
          a[3] = lop3_and_or(cur.b.y >> (4 * sb), kNibMask, kMagic);  // row g+8, k 2t+8..
          const uint32_t sel = (sb & 1) ? 0x7632u : 0x5410u;
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const uint32_t bq0 = prmt(word_of(cxa[j], sb >> 1), word_of(cxa[j], (sb >> 1) + 2), sel);
            const uint32_t bq1 = prmt(word_of(cxb[j], sb >> 1), word_of(cxb[j], (sb >> 1) + 2), sel);
            if (sb == 0) {
              mma_bf16_16816(R[j], a, bq0, bq1, zero4);
              mma_bf16_16816(SX[j], ones, bq0, bq1, zero4);
            } else {
              mma_bf16_16816(R[j], a, bq0, bq1, R[j]);
              mma_bf16_16816(SX[j], ones, bq0, bq1, SX[j]);
            }
          }
        }
        const float sc0 = bf2f(cur.sa & 0xffffu), bi0 = bf2f(cur.sa >> 16);
        const float sc1 = bf2f(cur.sb & 0xffffu), bi1 = bf2f(cur.sb >> 16);
        const float bp0 = fmaf(-128.f, sc0, bi0), bp1 = fmaf(-128.f, sc1, bi1);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          acc[j][0] = fmaf(sc0, R[j][0], fmaf(bp0, SX[j][0], acc[j][0]));
          acc[j][1] = fmaf(sc0, R[j][1], fmaf(bp0, SX[j][1], acc[j][1]));
          acc[j][2] = fmaf(sc1, R[j][2], fmaf(bp1, SX[j][2], acc[j][2]));
          acc[j][3] = fmaf(sc1, R[j][3], fmaf(bp1, SX[j][3], acc[j][3]));
        }
      }
    }
  }

  // ---- reduce the K-split warps
  if constexpr (KW > 1) {
    __shared__ float red[KW - 1][RT][NT * 4][32];
    if (kw > 0) {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[kw - 1][rt][j * 4 + i][lane] = acc[j][i];
    }
    __syncthreads();
    if (kw == 0) {
#pragma unroll
      for (int q = 0; q < KW - 1; ++q)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[j][i] += red[q][rt][j * 4 + i][lane];
    }
  }
  pdl_trigger();

  // ---- epilogue (warps with kw == 0 hold the sums)
  if (mode == EPI_ARGMAX) {
    __shared__ unsigned long long kbuf[RT][8 * NT];
    if (kw == 0) {
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
  if (kw != 0) return;
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

template <int NT, int RT, int KW>
int launch_cfg(const QmmArgs& a, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.total_ctas, (a.M + 8 * NT - 1) / (8 * NT), 1);
  cfg.blockDim = dim3(32 * RT * KW, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  IAM_CUDA(cudaLaunchKernelEx(&cfg, qmm_w4a16_kernel<NT, RT, KW>, a));
  return IAM_OK;
}

template <int NT>
int launch_nt(const QmmArgs& a, const QmmConfig& c, cudaStream_t st, bool pdl) {
  if (c.rt == 1 && c.kw == 4) return launch_cfg<NT, 1, 4>(a, st, pdl);
  if (c.rt == 2 && c.kw == 4) return launch_cfg<NT, 2, 4>(a, st, pdl);
  if (c.rt == 4 && c.kw == 2) return launch_cfg<NT, 4, 2>(a, st, pdl);
  if (c.rt == 1 && c.kw == 8) return launch_cfg<NT, 1, 8>(a, st, pdl);
  if (c.rt == 2 && c.kw == 2) return launch_cfg<NT, 2, 2>(a, st, pdl);
  if (c.rt == 4 && c.kw == 1) return launch_cfg<NT, 4, 1>(a, st, pdl);
  return fail(IAM_EINVAL, "qmm: unsupported tile config");
}

bool env_override(QmmConfig& c, int K) {
  const char* v = std::getenv("IAM_QMM_CFG");  // "rt,kw" or "rt,kw@K" applied to one K only
  if (!v) return false;
  int rt = 0, kw = 0, k = 0;
  const int n = std::sscanf(v, "%d,%d@%d", &rt, &kw, &k);
  if (n < 2 || (n == 3 && k != K)) return false;
  c.rt = rt;
  c.kw = kw;
  return true;
}

}  // namespace

QmmConfig qmm_plan(QmmArgs& a) {
  QmmConfig c;
  c.nt = a.M <= 8 ? 1 : (a.M <= 16 ? 2 : 4);
  int tiles = 0;
  for (int i = 0; i < a.nseg; ++i) {
    const int tr = a.seg[i].mode == EPI_SWIGLU ? 8 : 16;
    tiles += (a.seg[i].rows + tr - 1) / tr;
  }
  if (a.K >= 12288) {
    c.rt = 1;
    c.kw = 8;
  } else if (tiles >= 2048) {
    c.rt = 2;
    c.kw = 4;
  } else {
    c.rt = 1;
    c.kw = 4;
  }
  env_override(c, a.K);
  int cta = 0;
  for (int i = 0; i < a.nseg; ++i) {
    a.seg[i].cta_begin = cta;
    cta += (a.seg[i].rows + qmm_rows_per_cta(a.seg[i].mode, c.rt) - 1) / qmm_rows_per_cta(a.seg[i].mode, c.rt);
  }
  a.total_ctas = cta;
  return c;
}

int qmm_launch(const QmmArgs& a, const QmmConfig& c, cudaStream_t st, bool pdl) {
  if (c.nt == 1) return launch_nt<1>(a, c, st, pdl);
  if (c.nt == 2) return launch_nt<2>(a, c, st, pdl);
  if (c.nt == 4) return launch_nt<4>(a, c, st, pdl);
  return fail(IAM_EINVAL, "qmm: unsupported token tile");
}

// Validates one matmul and launches it in passes of at most 32 tokens.
int qmm_run(QmmArgs a, cudaStream_t st, bool pdl) {
  IAM_CHECK(a.K > 0 && a.K % 64 == 0, "qmm: K must be a positive multiple of 64");
  IAM_CHECK(a.M >= 1, "qmm: M must be >= 1");
  IAM_CHECK(a.nseg >= 1 && a.nseg <= kQmmMaxSeg, "qmm: 1..4 segments");
  IAM_CHECK(aligned16(a.x) && a.ldx % 8 == 0, "qmm: x must be 16-byte aligned with ldx % 8 == 0");
  for (int i = 0; i < a.nseg; ++i) {
    const QmmSeg& s = a.seg[i];
    IAM_CHECK(s.rows > 0 && s.w && s.s && s.b, "qmm: segment without weights");
    IAM_CHECK(aligned16(s.w), "qmm: w must be 16-byte aligned");
    if (s.mode == EPI_SWIGLU) IAM_CHECK(s.w2 && s.s2 && s.b2 && aligned16(s.w2), "qmm: SwiGLU needs the up matrix");
    if (s.mode == EPI_ARGMAX) IAM_CHECK(s.keys != nullptr && s.key_ld >= 1, "qmm: argmax needs a key buffer");
    else if (s.mode == EPI_F32) IAM_CHECK(s.out32 != nullptr, "qmm: no fp32 output");
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
