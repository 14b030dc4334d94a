// Register-dequant W4A16 matmul for narrow passes (decode and narrow verify
// blocks, up to 16 tokens) on the tile-packed weights of qmm.cuh.
//
// y[m, n] = sum_k x[m, k] * bf16(q[n, k] * s[n, k/64] + b[n, k/64]) -- the MLX
// affine 4-bit matmul the reference dispatches (full_forward.swift:711-728,
// batch_verify_27b.swift:100-119) -- with every weight converted exactly
// once, in registers, and fed straight into mma.sync.m16n8k16 (fp32
// accumulation): no tensor memory, no MMA issuer thread, no conversion
// stores.  At these widths the work is the weight stream; the conversion is
// about 1.4 instructions a weight and the tensor core does the rest.
//
// One CTA (8 consumer warps + 1 producer warp; two CTAs per SM) takes one
// 128-row tile of y^T for all tokens of the pass over a range of 256-k blocks:
//  * one producer thread streams each block through a 4-stage shared-memory
//    ring: the 18 KiB weight block in one contiguous bulk copy (issued for the
//    first stages before the grid-dependency wait: weights never depend on the
//    preceding kernel) plus the block's activations as four 2D tensor-map
//    copies of [8 or 16 tokens x 64 k] in the 128-byte swizzle (tokens >= M
//    read as zero);
//  * consumer warp w takes rows 32 (w/2) .. +31 (two m16 tiles) and k half
//    w%2 of every block.  Lane (g, t) = (lane/4, lane%4) reads, per 64-k group
//    b of its half and per row, the word pair k 64b + 16t .. +15 (one 8-byte
//    load, bank-conflict free under the packed chunk swizzle) and the
//    matching 16 bytes of x (bank-conflict free under the 128-byte swizzle),
//    and runs two MMAs per word.  The MMA's k order is permuted consistently
//    in A and B (lane t's physical pairs take its fragment slots 2t and
//    2t+8), which leaves the sums unchanged;
//  * the two k halves are added through shared memory; with the k range split
//    over CTAs each stores its fp32 partial and the last CTA of the tile (one
//    acquire-release counter) sums them in split order -- bitwise
//    reproducible; then the fused epilogue (store, residual, SwiGLU, argmax
//    keys, fp32 partials).
// Every mbarrier wait is bounded; a wait that gives up records IAM_ETIMEOUT,
// and the producer drains its copies before the CTA exits.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "kernels.cuh"
#include "rmsnorm.cuh"
#include "tc.cuh"
#include "tma.cuh"

namespace iam {
namespace {

constexpr int kGvStages = 4;
// Resident CTAs an SM.  (Three, with a 3-stage ring at 72 registers, measured
// slower on every shape: 248320 x 5120 at one token 170.9 against 152.7 us.)
__host__ __device__ constexpr int gv_min_ctas(int) { return 2; }
// QW: the number of consumer warps sharing one 32-row pair of a block, each
// taking 4 / QW of its four 64-k groups; 4 QW consumer warps + 1 producer.
__host__ __device__ constexpr int gv_warps(int QW) { return 4 * QW; }
__host__ __device__ constexpr int gv_threads(int QW) { return 32 * (gv_warps(QW) + 1); }

template <int NT, int QW = 4>
struct GvLayout {
  static_assert(NT == 1 || NT == 2, "8 or 16 tokens a pass");
  static_assert(QW == 2 || QW == 4, "2 or 4 warps on a row pair");
  static constexpr int kTok = 8 * NT;
  static constexpr int kXBox = kTok * 128;                 // one [kTok x 64 k] box
  static constexpr int kXBytes = 4 * kXBox;                // the block's 256 k of activations
  static constexpr int kStage = kXBytes + kQpBlockBytes;   // activations (1 KiB aligned), then weights
  static_assert(kStage % 1024 == 0, "stages keep the activation boxes 1 KiB aligned");
  static constexpr int kBarOff = kGvStages * kStage;
  static constexpr int kNumBars = 2 * kGvStages;           // full[S], empty[S]
  // barriers, then abort / last flags (64 bytes), then this CTA's segment
  static constexpr int kSmem = kBarOff + kNumBars * 8 + 64 + 128 + 1024;  // + alignment slack
  // the input rows the consumers build for a fused RMSNorm (runtime size, after the tail)
  static constexpr int kNxOff = (kBarOff + kNumBars * 8 + 64 + 128 + 15) / 16 * 16;
  // after the block loop the ring holds the k parts' partials [QW][128][kTok]
  // fp32, the tile's sums [128][kTok] and the argmax keys [4][kTok]
  static constexpr int kRedBytes = 128 * kTok * 4;
  static constexpr int kPartOff = kRedBytes + 4 * kTok * 8;
  static_assert(kPartOff + QW * kRedBytes <= kBarOff, "epilogue buffers fit in the ring");
  static_assert(gv_min_ctas(NT) * (kSmem + 1024) <= 228 * 1024, "resident CTAs per SM");
  static_assert(sizeof(QmmSeg) <= 128, "segment copy");
};

__device__ __forceinline__ uint32_t fma_bf2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// bf16(q * s + b) for the four code pairs of a packed word (pair s in v[s]):
// the fast form for tiles whose scales were stored times 2^129, the general
// form (q from (128 + q) - 128, then one rounded FMA) otherwise.
template <bool kFast>
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t s2, uint32_t b2, uint32_t (&v)[4]) {
  if constexpr (kFast) {
    qp_codes_hi(w, v);
#pragma unroll
    for (int s = 0; s < 4; ++s) v[s] = fma_bf2(v[s], s2, b2);
  } else {
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t q = lop3_and_or(w >> (4 * s), 0x000F000Fu, 0x43004300u);
      v[s] = fma_bf2(fma_bf2(q, 0x3F803F80u, 0xC300C300u), s2, b2);
    }
  }
}

__device__ __forceinline__ uint2 lds64(const unsigned char* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint4 lds128(const unsigned char* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ float4 ld_cg_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
  return r;
}

struct QmmGvArgs {
  CUtensorMap xmap;  // x [M, K] bf16, box [8 NT tokens x 64 k], 128B swizzle
  QmmArgs a;
};

template <int NT, int QW>
__global__ void __launch_bounds__(gv_threads(QW), gv_min_ctas(NT)) qmm_gemv_kernel(const __grid_constant__ QmmGvArgs T) {
  using L = GvLayout<NT, QW>;
  constexpr int S = kGvStages, TOK = L::kTok;
  constexpr int kGvWarps = gv_warps(QW);
  constexpr int GPW = 4 / QW;  // 64-k groups of a block a warp converts
  const QmmArgs& A = T.a;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar0 = sbase + L::kBarOff;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (S + s); };
  unsigned char* tail = smem + L::kBarOff + L::kNumBars * 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tail);
  int* last_flag = reinterpret_cast<int*>(tail + 8);
  QmmSeg* seg_copy = reinterpret_cast<QmmSeg*>(tail + 64);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bx = blockIdx.x;
  int si = 0;
#pragma unroll
  for (int i = 1; i < kQmmMaxSeg; ++i)
    if (i < A.nseg && bx >= A.seg[i].cta_begin) si = i;
  int tile = bx;
#pragma unroll
  for (int i = 0; i < kQmmMaxSeg; ++i)
    if (i == si) tile = bx - A.seg[i].cta_begin;
  const int KB = (A.K + kQpBlockK - 1) / kQpBlockK;
  const int KS = gridDim.z, ks = blockIdx.z;
  const int kb0 = (ks * KB) / KS, kb1 = ((ks + 1) * KB) / KS, nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), kGvWarps);
    }
    *abort_flag = 0;
    // a copy with constant indices: a parameter struct indexed at run time is
    // read through the slow generic path
#pragma unroll
    for (int i = 0; i < kQmmMaxSeg; ++i)
      if (i == si) *seg_copy = A.seg[i];
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  const QmmSeg& SG = *seg_copy;

  auto give_up = [&]() {
    *abort_flag = 1;
    if (A.err) atomicExch(A.err, IAM_ETIMEOUT);
  };
  // budget of the waits that may give up; waits for copies in flight get the full one
  const uint32_t lim = wait_limit(A.wait_limit);

  if (warp == kGvWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const unsigned char* wsrc = SG.packed + (static_cast<size_t>(tile) * KB + kb0) * kQpBlockBytes;
      const bool own_x = A.norm_w == nullptr;  // fused norm: the consumers build x themselves
      auto load_w = [&](int i) {
        const int s = i % S;
        mbar_expect_tx(full(s), kQpBlockBytes + (own_x ? L::kXBytes : 0));
        bulk_load(sbase + s * L::kStage + L::kXBytes, wsrc + static_cast<size_t>(i) * kQpBlockBytes, kQpBlockBytes,
                  full(s));
      };
      auto load_x = [&](int i) {
        if (!own_x) return;
        const int s = i % S;
#pragma unroll
        for (int b = 0; b < 4; ++b)
          tma_load_2d(sbase + s * L::kStage + b * L::kXBox, &T.xmap, (kb0 + i) * kQpBlockK + 64 * b, 0, full(s));
      };
      // (a starved launch, a test's fault injection, issues nothing: the
      // consumers' first wait can only run out)
      const int first = A.starve ? 0 : min(nkb, S);
      for (int i = 0; i < first; ++i) load_w(i);  // weights do not depend on the preceding kernel
      pdl_wait();
      for (int i = 0; i < first; ++i) load_x(i);
      int issued = first;
      for (; !A.starve && issued < nkb; ++issued) {
        const int s = issued % S;
        if (!mbar_wait(empty(s), ((issued / S) - 1) & 1, abort_flag, lim)) {
          give_up();
          break;
        }
        load_w(issued);
        load_x(issued);
      }
      // copies still in flight must land before the CTA exits
      for (int i = max(0, issued - S); i < issued; ++i)
        if (!mbar_wait(full(i % S), (i / S) & 1)) give_up();
    }
    return;  // the producer takes no part in the epilogue
  }

  // -------------------------------------------------------------- consumers
  const int rp = warp / QW, qp = warp % QW;  // row pair, k part (groups GPW qp .. +GPW-1)
  const int g = lane >> 2, t = lane & 3;
  const int M = A.M;
  const bool sw = SG.mode == EPI_SWIGLU;
  const int seg_tiles = (SG.rows + (sw ? 63 : 127)) / (sw ? 64 : 128);
  const bool fast = SG.packed[static_cast<size_t>(seg_tiles) * KB * kQpBlockBytes + tile] != 0;
  const int swz = qp_swz(g);  // rows 32 rp + 16 mt + g (+8) all share it
  // Stage offsets as a per-thread base plus compile-time terms (few live
  // registers): row R = 32 rp + g + 16 mt + 8 h holds its word pair
  // (k 64b + 16t ..) of group b = GPW qp + bb in chunk (2b + t/2) ^ swz, and
  // its (scale, bias) of that group at 16 R + 4 b.
  const int cbase = L::kXBytes + (32 * rp + g) * 128 + (t & 1) * 8;
  int cch[GPW];
#pragma unroll
  for (int bb = 0; bb < GPW; ++bb) cch[bb] = ((2 * (GPW * qp + bb) + (t >> 1)) ^ swz) << 4;
  const int sbbase = L::kXBytes + kQpCodeBytes + (32 * rp + g) * 16 + GPW * qp * 4;
  // x: token row nt*8 + g, its 8 k at 64b + 16t + 8 delta in chunk (2t + delta) ^ g
  const int xbase = GPW * qp * L::kXBox + g * 128;
  int xch[2];
#pragma unroll
  for (int d = 0; d < 2; ++d) xch[d] = ((2 * t + d) ^ g) << 4;
  bool xon[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) xon[nt] = nt * 8 + g < M;

  // Fused RMSNorm (rms_norm_bf16, full_forward.swift:59-86) ahead of the
  // matmul: x holds the raw rows.  Warp t sums row t in the reference's order;
  // then the consumers write bf16((x / rms) * w) for this CTA's blocks into
  // shared memory in the layout the copies would have had (rows < M only,
  // the boxes M rows apart), and the block loop reads it from there.
  const bool norm = A.norm_w != nullptr;
  unsigned char* const nx = smem + L::kNxOff;
  const int nxbox = M * 128;
  const int nxrow = GPW * qp * nxbox + g * 128;
  if (norm) {
    pdl_wait();  // the rows come from the preceding kernel
    float* rms_s = reinterpret_cast<float*>(tail + 16);
    if (warp < M) {
      const uint4* xrow = reinterpret_cast<const uint4*>(A.x + static_cast<size_t>(warp) * A.ldx);
      const float rms = rms_row_warp([&](int i) { return xrow[i]; }, A.K, A.norm_eps, lane);
      if (lane == 0) rms_s[warp] = rms;
    }
    named_bar_sync(1, 32 * kGvWarps);
    const int nchunk = nkb * 32;  // 8-element chunks of a row over this CTA's blocks
    for (int idx = threadIdx.x; idx < M * nchunk; idx += 32 * kGvWarps) {
      const int tr = idx / nchunk, kc = idx - tr * nchunk;
      const int k = (kb0 * 32 + kc) * 8;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (k < A.K)
        v = rms_apply8(*reinterpret_cast<const uint4*>(A.x + static_cast<size_t>(tr) * A.ldx + k),
                       *reinterpret_cast<const uint4*>(A.norm_w + k), rms_s[tr]);
      const int blk = kc >> 5, box = (kc >> 3) & 3, c = kc & 7;
      *reinterpret_cast<uint4*>(nx + (blk * 4 + box) * nxbox + tr * 128 + ((c ^ (tr & 7)) << 4)) = v;
    }
    named_bar_sync(1, 32 * kGvWarps);
  }

  // one accumulator set per 64-k group of the warp: independent MMA chains
  float acc[2][GPW][NT][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int bb = 0; bb < GPW; ++bb)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][bb][nt][e] = 0.f;

  // the block loop, compiled once per conversion form (a tile's scales pick it)
  auto blocks = [&](auto fast_tag) -> bool {
    constexpr bool kFast = decltype(fast_tag)::value;
    uint32_t phase = 0;
    int s = 0;
    for (int i = 0; i < nkb; ++i) {
      if (!__all_sync(0xffffffffu, !*abort_flag && mbar_wait_light(full(s), phase, abort_flag, lim))) return false;
      const unsigned char* stg = smem + s * L::kStage;
      uint4 xr[GPW][2][NT];
#pragma unroll
      for (int bb = 0; bb < GPW; ++bb)
#pragma unroll
        for (int d = 0; d < 2; ++d)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            xr[bb][d][nt] = !xon[nt] ? make_uint4(0u, 0u, 0u, 0u)
                            : norm   ? lds128(nx + i * 4 * nxbox + nxrow + bb * nxbox + xch[d])
                                     : lds128(stg + xbase + bb * L::kXBox + nt * 1024 + xch[d]);
      uint2 cw[2][2][GPW];
      uint32_t sb[2][2][GPW];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int bb = 0; bb < GPW; ++bb) cw[mt][h][bb] = lds64(stg + cbase + mt * 2048 + h * 1024 + cch[bb]);
          if constexpr (GPW == 2) {
            const uint2 p = lds64(stg + sbbase + mt * 256 + h * 128);
            sb[mt][h][0] = p.x;
            sb[mt][h][GPW - 1] = p.y;
          } else {
            sb[mt][h][0] = *reinterpret_cast<const uint32_t*>(stg + sbbase + mt * 256 + h * 128);
          }
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty(s));
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int bb = 0; bb < GPW; ++bb) {
          const uint32_t sb0 = sb[mt][0][bb], sb1 = sb[mt][1][bb];
          const uint32_t s20 = prmt(sb0, sb0, 0x1010u), b20 = prmt(sb0, sb0, 0x3232u);
          const uint32_t s21 = prmt(sb1, sb1, 0x1010u), b21 = prmt(sb1, sb1, 0x3232u);
#pragma unroll
          for (int d = 0; d < 2; ++d) {
            uint32_t v0[4], v1[4];
            dequant_word<kFast>(d ? cw[mt][0][bb].y : cw[mt][0][bb].x, s20, b20, v0);
            dequant_word<kFast>(d ? cw[mt][1][bb].y : cw[mt][1][bb].x, s21, b21, v1);
            const uint32_t a01[4] = {v0[0], v1[0], v0[1], v1[1]};
            const uint32_t a23[4] = {v0[2], v1[2], v0[3], v1[3]};
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              mma_bf16_16816(acc[mt][bb][nt], a01, xr[bb][d][nt].x, xr[bb][d][nt].y, acc[mt][bb][nt]);
              mma_bf16_16816(acc[mt][bb][nt], a23, xr[bb][d][nt].z, xr[bb][d][nt].w, acc[mt][bb][nt]);
            }
          }
        }
      if (++s == S) {
        s = 0;
        phase ^= 1u;
      }
    }
    return true;
  };
  const bool ok = fast ? blocks(std::true_type{}) : blocks(std::false_type{});
  if (!ok) give_up();

  // ------------------------------------------------------------ epilogue
  constexpr int kEpi = 32 * kGvWarps;
  const int ct = threadIdx.x;  // 0 .. kEpi - 1
  float* red = reinterpret_cast<float*>(smem);  // [128][TOK], over the idle ring
  unsigned long long* kbuf = reinterpret_cast<unsigned long long*>(smem + L::kRedBytes);  // [4][TOK]
  float* part = reinterpret_cast<float*>(smem + L::kPartOff);  // [QW][128][TOK]
  named_bar_sync(1, kEpi);  // every consumer is done with the ring
  // each warp's partial (its groups in k order), then the k parts summed in order
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float a = acc[mt][0][nt][e];
#pragma unroll
        for (int bb = 1; bb < GPW; ++bb) a += acc[mt][bb][nt][e];
        const int row = 32 * rp + 16 * mt + g + 8 * (e >> 1);
        const int tok = nt * 8 + 2 * t + (e & 1);
        part[(qp * 128 + row) * TOK + tok] = a;
      }
  pdl_wait();  // outputs, residuals and the workspace follow the preceding kernel
  const bool good = !named_bar_or(1, kEpi, !ok || *abort_flag);
  // thread ct: row ct & 127, tokens (ct >> 7) + QW j
  const int row = ct & 127, tpar = ct >> 7;
  constexpr int TPT = TOK / QW;  // tokens a thread
  float v[TPT];
#pragma unroll
  for (int j = 0; j < TPT; ++j) {
    const int tok = tpar + QW * j;
    float a = part[row * TOK + tok];
#pragma unroll
    for (int q = 1; q < QW; ++q) a += part[(q * 128 + row) * TOK + tok];
    v[j] = a;
  }
  bool last = true;
  if (KS > 1) {
    float* base = A.ws + static_cast<size_t>(bx) * KS * kQpRows * TOK + static_cast<size_t>(row) * TOK;
    if (good) {
      float* mine = base + static_cast<size_t>(ks) * kQpRows * TOK;
#pragma unroll
      for (int j = 0; j < TPT; ++j) mine[tpar + QW * j] = v[j];
    }
    named_bar_sync(1, kEpi);
    if (ct == 0) {
      int* ctr = A.counters + bx;
      int prev;
      asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(prev) : "l"(ctr) : "memory");
      const int l = prev == KS - 1;
      if (l) *ctr = 0;
      *last_flag = l;
    }
    named_bar_sync(1, kEpi);
    last = *last_flag != 0;
    if (last) {
      // every split's partial, in split order (reproducible bits)
#pragma unroll
      for (int j = 0; j < TPT; ++j) v[j] = 0.f;
      for (int q = 0; q < KS; ++q) {
        const float* p = base + static_cast<size_t>(q) * kQpRows * TOK;
        // the row's TOK floats; this thread's are tokens tpar, tpar + QW, ...
#pragma unroll
        for (int c4 = 0; c4 < TOK / 4; ++c4) {
          const float4 f = ld_cg_f4(p + 4 * c4);
          const float fv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if ((4 * c4 + e) % QW == tpar) v[(4 * c4 + e) / QW] += fv[e];
        }
      }
    }
  }
  if (last && good) {
    const int mode = SG.mode;
    if (mode == EPI_SWIGLU || mode == EPI_ARGMAX) {
      named_bar_sync(2, kEpi);  // every thread has read red
#pragma unroll
      for (int j = 0; j < TPT; ++j) red[row * TOK + tpar + QW * j] = v[j];
      named_bar_sync(2, kEpi);
    }
    if (mode == EPI_SWIGLU) {
      // rows 0-63 gate, 64-127 up of features tile*64 + (row & 63)
      const int f = tile * 64 + row;
      uint16_t* const out = SG.out;
      const size_t ldo = static_cast<size_t>(SG.ldo);
      if (row < 64 && f < SG.rows) {
#pragma unroll
        for (int j = 0; j < TPT; ++j) {
          const int tok = tpar + QW * j;
          if (tok < M) out[tok * ldo + f] = f2bf(silu_f(round_bf(v[j])) * round_bf(red[(row + 64) * TOK + tok]));
        }
      }
    } else if (mode == EPI_ARGMAX) {
      // per token: the best (value, first index) key over the tile's rows;
      // warp w holds rows 32 (w & 3) .. +31 of tokens (w >> 2) + QW j
      const int grow = tile * kQpRows + row;
#pragma unroll
      for (int j = 0; j < TPT; ++j) {
        unsigned long long k = 0ull;
        if (grow < SG.rows) k = argmax_key(round_bf(v[j]), static_cast<uint32_t>(SG.col_base + grow));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
          k = other > k ? other : k;
        }
        if (lane == 0) kbuf[(warp & 3) * TOK + tpar + QW * j] = k;
      }
      named_bar_sync(2, kEpi);
      if (ct < TOK && ct < M) {
        unsigned long long k = kbuf[ct];
#pragma unroll
        for (int qq = 1; qq < 4; ++qq) k = kbuf[qq * TOK + ct] > k ? kbuf[qq * TOK + ct] : k;
        SG.keys[static_cast<size_t>(tile) * SG.key_ld + ct] = k;
      }
    } else if (mode == EPI_F32 && A.npush > 0) {
      // this rank's values of the tile into every rank's receive slot
      const int grow = tile * kQpRows + row;
      const size_t ldo = static_cast<size_t>(SG.ldo);
      if (grow < SG.rows) {
#pragma unroll
        for (int r = 0; r < kQmmMaxPeers; ++r) {  // constant indices: the pointers straight from the parameters
          if (r >= A.npush) break;
          float* const dst = A.push[r];
#pragma unroll
          for (int j = 0; j < TPT; ++j) {
            const int tok = tpar + QW * j;
            if (tok < M) dst[tok * ldo + grow] = v[j];
          }
        }
      }
      named_bar_sync(2, kEpi);
      if (ct == 0) qmm_push_arrive(A, tile);
    } else {
      const int grow = tile * kQpRows + row;
      uint16_t* const out = SG.out;
      float* const out32 = SG.out32;
      const uint16_t* const resid = SG.resid;
      const size_t ldo = static_cast<size_t>(SG.ldo), ldr = static_cast<size_t>(SG.ldr);
      if (grow < SG.rows) {
#pragma unroll
        for (int j = 0; j < TPT; ++j) {
          const int tok = tpar + QW * j;
          if (tok >= M) continue;
          const size_t o = tok * ldo + grow;
          if (mode == EPI_F32) {
            out32[o] = v[j];
          } else if (mode == EPI_RESID) {
            out[o] = f2bf(bf2f(resid[tok * ldr + grow]) + round_bf(v[j]));
          } else {
            out[o] = f2bf(v[j]);
          }
        }
      }
    }
  }
}

int g_gv_sms = 0;
// shared memory a launch may add for the rows of a fused RMSNorm
constexpr int kGvNormSmem = 24 * 1024;
bool g_gv_attr[2][2] = {{false, false}, {false, false}};

template <int NT, int QW>
int gv_set_attr() {
  if (!g_gv_attr[NT - 1][QW / 4]) {
    IAM_CUDA(cudaFuncSetAttribute(qmm_gemv_kernel<NT, QW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  GvLayout<NT, QW>::kSmem + kGvNormSmem));
    g_gv_attr[NT - 1][QW / 4] = true;
  }
  return IAM_OK;
}

// Split-K factor.  A CTA streams its blocks at a rate bounded by latency
// (about one 18 KiB block a microsecond), so the plan fills the GPU with two
// resident CTAs an SM where the tile count allows: the smallest split that
// gives about 1.8 CTAs an SM without a second wave, and never CTAs of fewer
// than two blocks.  Matrices with at least 1.8 tiles an SM are not split.
int gv_plan_ks(int tiles, int KB) {
  if (const char* v = std::getenv("IAM_QMM_GEMV_KS")) {
    const int k = std::atoi(v);
    if (k >= 1) return std::min(k, KB);
  }
  double per_sm = 1.8;  // target resident CTAs an SM (IAM_QMM_GEMV_CTAS overrides, for measurements)
  if (const char* v = std::getenv("IAM_QMM_GEMV_CTAS")) per_sm = std::max(0.1, std::min(2.0, std::atof(v)));
  const int slots = 2 * g_gv_sms;
  int ks = (static_cast<int>(per_sm * g_gv_sms) + tiles - 1) / tiles;
  if (static_cast<long>(tiles) * ks > slots) ks = slots / tiles;
  ks = std::min(ks, std::max(1, KB / 2));
  return std::max(ks, 1);
}

template <int NT, int QW>
int gv_launch(const QmmGvArgs& ga, int ks, cudaStream_t st, bool pdl) {
  const int r = gv_set_attr<NT, QW>();
  if (r != IAM_OK) return r;
  // fused RMSNorm: the CTA's input rows, 4 boxes of M rows x 128 bytes a block
  size_t extra = 0;
  if (ga.a.norm_w) {
    const int nkb = (qp_kblocks(ga.a.K) + ks - 1) / ks;
    extra = 16 + static_cast<size_t>(nkb) * 4 * ga.a.M * 128;
    IAM_CHECK(extra <= static_cast<size_t>(kGvNormSmem), "qmm: the fused RMSNorm's rows do not fit");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ga.a.total_ctas, 1, ks);
  cfg.blockDim = dim3(gv_threads(QW), 1, 1);
  cfg.dynamicSmemBytes = GvLayout<NT, QW>::kSmem + extra;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  IAM_CUDA(cudaLaunchKernelEx(&cfg, qmm_gemv_kernel<NT, QW>, ga));
  return IAM_OK;
}

}  // namespace

int qmm_gemv_max_m() {
  // read on every call (host side, once per matmul launch or graph capture)
  if (const char* e = std::getenv("IAM_QMM_GEMV_MAX_M")) return std::max(0, std::min(std::atoi(e), kGemvMaxM));
  return kGemvDefaultMaxM;
}

int qmm_gemv_run(QmmArgs a, cudaStream_t st, bool pdl, size_t ws_floats_cap, size_t ws_ctr_cap) {
  IAM_CHECK(a.K > 0 && a.K % 64 == 0, "qmm: K must be a positive multiple of 64");
  IAM_CHECK(a.M >= 1 && a.M <= kGemvMaxM, "qmm: the GEMV path takes 1..16 tokens a pass");
  IAM_CHECK(a.nseg >= 1 && a.nseg <= kQmmMaxSeg, "qmm: 1..4 segments");
  IAM_CHECK(aligned16(a.x) && a.ldx % 8 == 0 && a.ldx >= a.K, "qmm: x must be 16-byte aligned with ldx % 8 == 0");
  if (g_gv_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_gv_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_gv_sms <= 0) g_gv_sms = 148;
  }
  int cta = 0;
  for (int i = 0; i < a.nseg; ++i) {
    QmmSeg& s = a.seg[i];
    IAM_CHECK(s.rows > 0 && s.packed && aligned16(s.packed), "qmm: segment without packed weights");
    if (s.mode == EPI_ARGMAX) IAM_CHECK(s.keys != nullptr && s.key_ld >= 1, "qmm: argmax needs a key buffer");
    else if (s.mode == EPI_F32) IAM_CHECK(s.out32 != nullptr || a.npush > 0, "qmm: no fp32 output");
    else IAM_CHECK(s.out != nullptr, "qmm: no output");
    if (s.mode == EPI_RESID) IAM_CHECK(s.resid != nullptr, "qmm: residual input missing");
    s.cta_begin = cta;
    cta += qp_tiles(s.rows, s.mode == EPI_SWIGLU);
  }
  a.total_ctas = cta;
  const int NT = a.M <= 8 ? 1 : 2;
  const int TOK = 8 * NT;
  const int KB = qp_kblocks(a.K);
  int ks = gv_plan_ks(cta, KB);
  if (ks > 1 && a.ws) {  // a caller's workspace bounds the split
    const size_t per = static_cast<size_t>(cta) * kQpRows * TOK;
    ks = static_cast<int>(std::min<size_t>(ks, ws_floats_cap / per));
    if (static_cast<size_t>(cta) > ws_ctr_cap) ks = 1;
    ks = std::max(ks, 1);
  }
  if (ks > 1) {
    const size_t nf = static_cast<size_t>(cta) * ks * kQpRows * TOK, nc = static_cast<size_t>(cta);
    if (!a.ws) {
      const int r = qmm_op_workspace(1, nf, nc, st, &a.ws, &a.counters);
      if (r != IAM_OK) return r;
    } else {
      IAM_CHECK(nf <= ws_floats_cap && nc <= ws_ctr_cap, "qmm: split-K workspace too small");
    }
  }
  QmmGvArgs ga;
  std::memset(&ga, 0, sizeof(ga));
  ga.a = a;
  const int r = tma_encode_2d(&ga.xmap, a.x, 2, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.K), TOK, 64,
                              true, static_cast<uint64_t>(a.ldx));
  if (r != IAM_OK) return r;
  // 8 consumer warps (each converts two 64-k groups of a block) by default:
  // measured faster than 16 (one group each), whose per-block overheads are
  // spread over half the weights; IAM_QMM_GEMV_WARPS=16 selects 16
  const char* wv = std::getenv("IAM_QMM_GEMV_WARPS");
  const bool w16 = wv && std::atoi(wv) == 16;
  if (NT == 1) return w16 ? gv_launch<1, 4>(ga, ks, st, pdl) : gv_launch<1, 2>(ga, ks, st, pdl);
  return w16 ? gv_launch<2, 4>(ga, ks, st, pdl) : gv_launch<2, 2>(ga, ks, st, pdl);
}

}  // namespace iam
