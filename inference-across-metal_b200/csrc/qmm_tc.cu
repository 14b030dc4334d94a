// Tensor-core W4A16 matmul for sm_100a: tcgen05.mma with the dequantized
// weights in tensor memory.
//
// y[m, n] = sum_k x[m, k] * bf16(q[n, k] * s[n, k/64] + b[n, k/64]) -- the MLX
// affine 4-bit matmul the reference dispatches (full_forward.swift:711-728,
// batch_verify_27b.swift:100-119), computed on weights re-packed once at load
// into 128-row x 256-k blocks (qmm.cuh).
//
// One CTA per SM owns a 128-row tile of y^T for all tokens of the pass (<= 64)
// over a range of k blocks:
//  * one thread of warp 0 feeds two shared-memory rings: weight blocks (codes
//    and (scale, bias) pairs, one contiguous 18 KiB bulk copy a block, freed
//    as soon as the dequantizers hold them in registers) and activations (four
//    2D tensor-map copies of [N tokens x 64 k] a block in the 128-byte swizzle
//    the MMA reads, freed when the MMAs complete; tokens >= M and k >= K read
//    as zero);
//  * sixteen dequantizer warps, one thread per weight row (warp % 4 is the
//    TMEM lane quadrant its sub-partition may access, (warp - 2) / 4 the 64-k
//    group of each block it converts), turn codes into bf16 weights --
//    (w >> 4s) & 0x000F000F | 0x43004300 is the bf16 pair (128 + q, 128 + q'),
//    a packed FMA removes the 128 exactly and a second one rounds
//    q * scale + bias to bf16 once, the value mx.dequantize produces -- and
//    store them into a 3-block ring of A operands in tensor memory
//    (tcgen05.st): the MMA's A operand never passes through shared memory;
//  * one thread of warp 1 issues tcgen05.mma kind::f16 (M = 128, N = 16, 32
//    or 64, K = 16; A from tensor memory, B from shared memory) into an fp32
//    accumulator in tensor memory; tcgen05.commit hands A slots and
//    activation stages back.  The tensor core takes about 19 cycles an MMA
//    at these shapes but a barrier check stalls the issuing thread for 100+,
//    so the issuer synchronises once per block (16 MMAs);
//  * the dequantizer warps then read the accumulators (tcgen05.ld); with the k
//    range split over CTAs each stores its fp32 partial and the last CTA of
//    the tile sums them in split order (bitwise reproducible); then the fused
//    epilogue.
// Every mbarrier wait is bounded; a wait that gives up records IAM_ETIMEOUT,
// and the CTA drains its copies and MMAs before freeing tensor memory.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "kernels.cuh"
#include "tc.cuh"
#include "tma.cuh"

namespace iam {
namespace {

// One CTA per SM (it holds all 512 TMEM columns): a producer warp, an MMA warp
// and 16 dequantizer warps -- warp w works on TMEM lane quadrant w % 4 (the
// quadrant its SM sub-partition may access) and on 64-k group (w - 2) / 4 of
// every 256-k block.
constexpr int kTcDqWarps = 16;
constexpr int kTcThreads = 32 * (3 + kTcDqWarps);  // + a watcher warp (the last)
constexpr int kTcEarly = 2;                           // weight blocks issued before the CTA barrier
constexpr int kTcASlots = 3;                         // TMEM A slots of one 256-k block (128 columns)
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kTcDCol = 128 * kTcASlots;        // accumulator: NN (<= 64) columns

constexpr uint32_t kMagic = 0x43004300u;
constexpr uint32_t kNibMask = 0x000F000Fu;
constexpr uint32_t kOne = 0x3F803F80u;
constexpr uint32_t kNeg128 = 0xC300C300u;

__device__ __forceinline__ uint32_t fma_bf2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t dequant2(uint32_t w, uint32_t s2, uint32_t b2) {
  const uint32_t v = lop3_and_or(w, kNibMask, kMagic);
  return fma_bf2(fma_bf2(v, kOne, kNeg128), s2, b2);
}

// One 64-k group of a row (two 16-byte code chunks) -> 32 TMEM columns of bf16 pairs.
__device__ __forceinline__ void dequant_group(const uint4& c0, const uint4& c1, uint32_t sb, uint32_t (&r)[32]) {
  const uint32_t s2 = prmt(sb, sb, 0x1010u), b2 = prmt(sb, sb, 0x3232u);
  const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int s = 0; s < 4; ++s) r[4 * j + s] = dequant2(w[j] >> (4 * s), s2, b2);
}

// The same for a tile whose scales were stored times 2^129 (qmm.cuh).
__device__ __forceinline__ void dequant_group_fast(const uint4& c0, const uint4& c1, uint32_t sb, uint32_t (&r)[32]) {
  const uint32_t s2 = prmt(sb, sb, 0x1010u), b2 = prmt(sb, sb, 0x3232u);
  const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint32_t v[4];
    qp_codes_hi(w[j], v);
#pragma unroll
    for (int s = 0; s < 4; ++s) r[4 * j + s] = fma_bf2(v[s], s2, b2);
  }
}

__device__ __forceinline__ float4 ld_cg_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
  return r;
}

// Cursor over an N-stage ring: stage index and the parity of its current lap
// (no divisions in the hot loops).
template <int N>
struct Ring {
  int idx = 0;
  uint32_t phase = 0;
  bool first_lap = true;
  __device__ __forceinline__ void next() {
    if (++idx == N) {
      idx = 0;
      phase ^= 1u;
      first_lap = false;
    }
  }
  // positioned at element i, stepping two elements at a time (N > 2)
  __device__ __forceinline__ void start(int i) {
    idx = i % N;
    phase = static_cast<uint32_t>(i / N) & 1u;
    first_lap = i < N;
  }
  __device__ __forceinline__ void next2() {
    idx += 2;
    if (idx >= N) {
      idx -= N;
      phase ^= 1u;
      first_lap = false;
    }
  }
};

struct QmmTcArgs {
  CUtensorMap xmap;  // x [M, K] bf16, box [NN tokens x 64 k], 128B swizzle
  QmmArgs a;
};

template <int NN>
struct TcLayout {
  static_assert(NN == 16 || NN == 32 || NN == 64, "token tile");
  static_assert(kTcDCol + NN <= kTcTmemCols, "TMEM budget");
  static constexpr int kWS = NN == 16 ? 8 : 7;                        // weight ring stages
  static constexpr int kXS = NN == 16 ? 8 : NN == 32 ? 6 : 3;         // activation ring stages (L2 latency ~1 us)
  static constexpr int kXBox = NN * 128;                   // one [NN x 64 k] box
  static constexpr int kXBytes = 4 * kXBox;                // 256 k of activations
  static constexpr int kWOff = kXS * kXBytes;              // weight ring after the (1 KiB aligned) x ring
  static constexpr int kBarOff = kWOff + kWS * kQpBlockBytes;
  // wfull, wempty [kWS]; xfull, xempty [kXS]; afull, aempty [kTcASlots];
  // dfull; then the TMEM base and flags (64 bytes) and this CTA's segment
  static constexpr int kNumBars = 2 * kWS + 2 * kXS + 2 * kTcASlots + 1;
  static constexpr int kSmem = kBarOff + kNumBars * 8 + 64 + 128 + 1024;  // + alignment slack
  static_assert(sizeof(QmmSeg) <= 128, "segment copy");
  static_assert(kXBytes % 1024 == 0, "x stages must keep 1 KiB alignment");
  // more than half an SM's shared memory: one CTA (512 TMEM columns) per SM
  static_assert(kSmem > 116 * 1024 && kSmem <= 227 * 1024, "one CTA per SM");
};

template <int NN>
__global__ void __launch_bounds__(kTcThreads, 1) qmm_tc_kernel(const __grid_constant__ QmmTcArgs T) {
  using L = TcLayout<NN>;
  constexpr int WS = L::kWS, XS = L::kXS;
  const QmmArgs& A = T.a;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar0 = sbase + L::kBarOff;
  auto wfull = [&](int s) { return bar0 + 8u * s; };
  auto wempty = [&](int s) { return bar0 + 8u * (WS + s); };
  auto xfull = [&](int s) { return bar0 + 8u * (2 * WS + s); };
  auto xempty = [&](int s) { return bar0 + 8u * (2 * WS + XS + s); };
  auto afull = [&](int s) { return bar0 + 8u * (2 * WS + 2 * XS + s); };
  auto aempty = [&](int s) { return bar0 + 8u * (2 * WS + 2 * XS + kTcASlots + s); };
  const uint32_t dfull = bar0 + 8u * (L::kNumBars - 1);
  unsigned char* tail = smem + L::kBarOff + L::kNumBars * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tail);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tail + 8);
  int* last_flag = reinterpret_cast<int*>(tail + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bx = blockIdx.x;
  int si = 0;
#pragma unroll
  for (int i = 1; i < kQmmMaxSeg; ++i)
    if (i < A.nseg && bx >= A.seg[i].cta_begin) si = i;
  // The CTA's segment is read from a shared-memory copy: a parameter struct
  // indexed at run time is read through the generic path, hundreds of cycles
  // a field while the weight stream fills the memory system.
  QmmSeg* seg_copy = reinterpret_cast<QmmSeg*>(tail + 64);
  int tile = bx;
#pragma unroll
  for (int i = 0; i < kQmmMaxSeg; ++i)
    if (i == si) tile = bx - A.seg[i].cta_begin;
  const int KB = (A.K + kQpBlockK - 1) / kQpBlockK;
  const int KS = gridDim.z, ks = blockIdx.z;
  const int kb0 = (ks * KB) / KS, kb1 = ((ks + 1) * KB) / KS, nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WS; ++s) {
      mbar_init(wfull(s), 1);
      mbar_init(wempty(s), kTcDqWarps / 2);  // the team that converts the block
    }
    for (int s = 0; s < XS; ++s) {
      mbar_init(xfull(s), 1);
      mbar_init(xempty(s), 1);
    }
    for (int s = 0; s < kTcASlots; ++s) {
      mbar_init(afull(s), kTcDqWarps / 2);
      mbar_init(aempty(s), 1);
    }
    mbar_init(dfull, 1);
    *abort_flag = 0;
#pragma unroll
    for (int i = 0; i < kQmmMaxSeg; ++i)  // constant indices: constant-bank loads
      if (i == si) *seg_copy = A.seg[i];
    fence_mbar_init();
    // the first weight blocks go out now, before the tensor-memory allocation
    // and the CTA barrier (this thread is also the producer below)
    if (!A.starve) {
      const unsigned char* wsrc = seg_copy->packed + (static_cast<size_t>(tile) * KB + kb0) * kQpBlockBytes;
      for (int i = 0; i < min(nkb, kTcEarly); ++i) {
        mbar_expect_tx(wfull(i), kQpBlockBytes);
        bulk_load(sbase + L::kWOff + i * kQpBlockBytes, wsrc + static_cast<size_t>(i) * kQpBlockBytes, kQpBlockBytes,
                  wfull(i));
      }
    }
  }
  if (warp == 0) {
    __syncwarp();
    tmem_alloc(smem_addr(tmem_slot), kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const QmmSeg& S = *seg_copy;
  pdl_trigger();

  auto give_up = [&]() {
    *abort_flag = 1;
    if (A.err) atomicExch(A.err, IAM_ETIMEOUT);
  };
  // budget of the waits that may give up; waits for work in flight get the full one
  const uint32_t lim = wait_limit(A.wait_limit);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One thread feeds both rings, issuing whichever stage frees first.
    if (lane == 0) {
      const unsigned char* wsrc = S.packed + (static_cast<size_t>(tile) * KB + kb0) * kQpBlockBytes;
      auto load_w = [&](int i) {
        const int s = i % WS;
        mbar_expect_tx(wfull(s), kQpBlockBytes);
        bulk_load(sbase + L::kWOff + s * kQpBlockBytes, wsrc + static_cast<size_t>(i) * kQpBlockBytes,
                  kQpBlockBytes, wfull(s));
      };
      auto load_x = [&](int i) {
        const int s = i % XS;
        const uint32_t xs = sbase + s * L::kXBytes;
        mbar_expect_tx(xfull(s), L::kXBytes);
#pragma unroll
        for (int b = 0; b < 4; ++b)
          tma_load_2d(xs + b * L::kXBox, &T.xmap, (kb0 + i) * kQpBlockK + 64 * b, 0, xfull(s));
      };
      // (a starved launch, a test's fault injection, issues nothing: the
      // consumers' first waits can only run out)
      // (the first min(nkb, WS) weight blocks went out at the start: weights
      // do not depend on the preceding kernel)
      int iw = A.starve ? 0 : min(nkb, kTcEarly), ix = A.starve ? 0 : min(nkb, XS);
      // the rest of the ring's first lap: behind the first blocks, so those
      // arrive first when every CTA of the launch starts at once
      if (!A.starve)
        for (; iw < min(nkb, WS); ++iw) load_w(iw);
      pdl_wait();
      for (int i = 0; i < ix; ++i) load_x(i);
      uint32_t idle = 0;
      while (!A.starve && (iw < nkb || ix < nkb)) {
        bool progress = false;
        if (iw < nkb && mbar_test(wempty(iw % WS), ((iw / WS) - 1) & 1)) {
          load_w(iw++);
          progress = true;
        }
        if (ix < nkb && mbar_test(xempty(ix % XS), ((ix / XS) - 1) & 1)) {
          load_x(ix++);
          progress = true;
        }
        if (progress) {
          idle = 0;
        } else {
          if (++idle > lim || *abort_flag) {
            give_up();
            break;
          }
          __nanosleep(20);
        }
      }
      // copies still in flight must land before the CTA exits
      for (int i = max(0, iw - WS); i < iw; ++i)
        if (!mbar_wait(wfull(i % WS), (i / WS) & 1)) give_up();
      for (int i = max(0, ix - XS); i < ix; ++i)
        if (!mbar_wait(xfull(i % XS), (i / XS) & 1)) give_up();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The warp runs the loop converged and one elected lane issues.  It never
    // polls an mbarrier itself: the watcher warp waits for each block's A slot
    // (the dequantizer warp converting the block's first rows of its first
    // half also waited for the block's activations before arriving on it) and
    // hands the block over through a named barrier.  (Barrier checks by the
    // issuing warp cost about 400 cycles each even on a completed phase, as
    // much as a block's 16 MMAs.)
    constexpr uint32_t idesc = umma_idesc_bf16(128, NN);
    const uint32_t dt = tmem + kTcDCol;
    bool ok = true;
    Ring<kTcASlots> ar;
    Ring<XS> xr;
    for (int i = 0; i < nkb; ++i, ar.next(), xr.next()) {
      const int slot = ar.idx, xsl = xr.idx;
      // with the watcher: block i is ready, or (the OR of the barrier) the CTA
      // gave up -- no shared-memory read on this path
      if (named_bar_or(3, 64, false)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (elect_one()) {
        const uint32_t xs = sbase + xsl * L::kXBytes;
#pragma unroll
        for (int h = 0; h < 4; ++h)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            umma_bf16_ts(dt, tmem + slot * 128 + h * 32 + 8 * j, umma_sdesc_sw128(xs + h * L::kXBox + j * 32),
                         idesc, (i | h | j) != 0);
        umma_commit(aempty(slot));
        umma_commit(xempty(xsl));
      }
      __syncwarp();
    }
    if (!ok) give_up();
    if (elect_one()) umma_commit(dfull);
    __syncwarp();
    // every MMA of this CTA has completed once dfull flips
    if (!__all_sync(0xffffffffu, mbar_wait(dfull, 0))) give_up();
  } else if (warp == 2 + kTcDqWarps) {
    // ------------------------------------------------------------ watcher
    // Block by block: wait for the A slot, then meet the issuer (both sides
    // meet once per block until one of them gives up).
    Ring<kTcASlots> ar;
    for (int i = 0; i < nkb; ++i, ar.next()) {
      const bool got = __all_sync(0xffffffffu, !*abort_flag && mbar_wait_light(afull(ar.idx), ar.phase, abort_flag, lim));
      if (!got && lane == 0) give_up();
      named_bar_or(3, 64, !got);
      if (!got) break;
    }
  } else {
    // ------------------------------------------------------------ dequantizers
    const int q = warp & 3, h = (warp - 2) >> 2;  // h: 64-k group of each block
    const int row = 32 * q + lane;
    const uint32_t lane_base = tmem + ((32u * q) << 16);
    const bool sw = S.mode == EPI_SWIGLU;
    const int seg_tiles = (S.rows + (sw ? 63 : 127)) / (sw ? 64 : 128);
    const bool fast = S.packed[static_cast<size_t>(seg_tiles) * KB * kQpBlockBytes + tile] != 0;
    // Two teams of eight warps take alternate blocks; a warp converts two
    // 64-k groups (gp: groups 2gp, 2gp+1) of its quadrant's rows per visit.
    // The teams drift apart by half a block, so one team's barrier waits and
    // store latencies overlap the other team's conversion on every SM
    // sub-partition.
    const int team = (warp - 2) >> 3, gp = ((warp - 2) >> 2) & 1;
    Ring<WS> wr;
    Ring<kTcASlots> ar;
    wr.start(team);
    ar.start(team);
    for (int i = team; i < nkb; i += 2, wr.next2(), ar.next2()) {
      const int s = wr.idx;
      // every branch below is warp-uniform: tcgen05.st/ld need the whole warp
      if (!__all_sync(0xffffffffu, !*abort_flag && mbar_wait_light(wfull(s), wr.phase, abort_flag, lim))) {
        give_up();
        break;
      }
      const unsigned char* blk = smem + L::kWOff + s * kQpBlockBytes;
      uint4 c[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        c[j] = *reinterpret_cast<const uint4*>(blk + row * 128 + (((4 * gp + j) ^ qp_swz(row)) << 4));
      const uint2 sb = *reinterpret_cast<const uint2*>(blk + kQpCodeBytes + row * 16 + gp * 8);
      __syncwarp();
      if (lane == 0) mbar_arrive(wempty(s));
      const int slot = ar.idx;
      if (!__all_sync(0xffffffffu, ar.first_lap || mbar_wait_light(aempty(slot), ar.phase ^ 1u, abort_flag, lim))) {
        give_up();
        break;
      }
      tc_fence_after();
      uint32_t r[32];
      if (fast) {
        dequant_group_fast(c[0], c[1], sb.x, r);
      } else {
        dequant_group(c[0], c[1], sb.x, r);
      }
      tmem_st8x4(lane_base + slot * 128 + (2 * gp) * 32, r);
      if (fast) {
        dequant_group_fast(c[2], c[3], sb.y, r);
      } else {
        dequant_group(c[2], c[3], sb.y, r);
      }
      tmem_st8x4(lane_base + slot * 128 + (2 * gp + 1) * 32, r);
      tmem_wait_st();
      tc_fence_before();
      // one warp of the team also vouches for the block's activations (the
      // MMA issuer waits on the A slot alone)
      if (q == 0 && gp == 0 &&
          !__all_sync(0xffffffffu, mbar_wait_light(xfull(i % XS), static_cast<uint32_t>(i / XS) & 1u, abort_flag, lim))) {
        give_up();
        break;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(afull(slot));
    }

    // ------------------------------------------------------------ epilogue
    constexpr int EC = NN / 4;  // accumulator columns (tokens) per warp
    float v[EC];
    const bool have = __all_sync(0xffffffffu, mbar_wait_light(dfull, 0));
    if (!have) give_up();
    tc_fence_after();
    if constexpr (EC == 16) {
      tmem_ld16(lane_base + kTcDCol + h * EC, v);
    } else if constexpr (EC == 8) {
      tmem_ld8(lane_base + kTcDCol + h * EC, v);
    } else {
      tmem_ld4(lane_base + kTcDCol + h * EC, v);
    }
    tmem_wait_ld();
    tc_fence_before();
    const int tok0 = h * EC;
    pdl_wait();
    // one verdict for all epilogue threads (their named barriers below)
    const bool ok = !named_bar_or(1, 32 * kTcDqWarps, !have || *abort_flag);
    bool last = true;
    if (KS > 1) {
      // split-K: each CTA stores its partial in its own slice [ks][row][token];
      // the last CTA of the tile sums the slices in ks order (reproducible bits)
      float* base = A.ws + static_cast<size_t>(bx) * KS * kQpRows * NN + static_cast<size_t>(row) * NN + tok0;
      if (ok) {
        float* mine = base + static_cast<size_t>(ks) * kQpRows * NN;
#pragma unroll
        for (int c4 = 0; c4 < EC / 4; ++c4)
          *reinterpret_cast<float4*>(mine + 4 * c4) = make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
      }
      // The barrier orders every thread's partial before one GPU-scope
      // acquire-release arrival (cumulative, so it publishes the whole CTA's
      // partial and, for the last arrival, acquires the others').
      named_bar_sync(1, 32 * kTcDqWarps);
      if (threadIdx.x == 64) {
        int* ctr = A.counters + bx;
        int prev;
        asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(prev) : "l"(ctr) : "memory");
        const int l = prev == KS - 1;
        if (l) *ctr = 0;
        *last_flag = l;
      }
      named_bar_sync(1, 32 * kTcDqWarps);
      last = *last_flag != 0;
      if (last) {
#pragma unroll
        for (int e = 0; e < EC; ++e) v[e] = 0.f;
        for (int j = 0; j < KS; ++j) {
          const float* p = base + static_cast<size_t>(j) * kQpRows * NN;
#pragma unroll
          for (int c4 = 0; c4 < EC / 4; ++c4) {
            const float4 t = ld_cg_f4(p + 4 * c4);
            v[4 * c4] += t.x;
            v[4 * c4 + 1] += t.y;
            v[4 * c4 + 2] += t.z;
            v[4 * c4 + 3] += t.w;
          }
        }
      }
    }
    if (last && ok) {
      const int mode = S.mode;
      if (mode == EPI_SWIGLU) {
        // rows 0-63 gate, 64-127 up of features tile*64 + (row & 63)
        float* ubuf = reinterpret_cast<float*>(smem);  // the x ring is idle now
        if (row >= 64) {
#pragma unroll
          for (int e = 0; e < EC; ++e) ubuf[(row - 64) * NN + tok0 + e] = v[e];
        }
        named_bar_sync(1, 32 * kTcDqWarps);
        const int f = tile * 64 + row;
        uint16_t* const out = S.out;
        const size_t ldo = static_cast<size_t>(S.ldo);
        const int M = A.M;
        if (row < 64 && f < S.rows) {
#pragma unroll
          for (int e = 0; e < EC; ++e) {
            const int tok = tok0 + e;
            if (tok < M) out[tok * ldo + f] = f2bf(silu_f(round_bf(v[e])) * round_bf(ubuf[row * NN + tok]));
          }
        }
      } else if (mode == EPI_ARGMAX) {
        unsigned long long* kbuf = reinterpret_cast<unsigned long long*>(smem);  // [4][NN]
        const int grow = tile * kQpRows + row;
#pragma unroll
        for (int e = 0; e < EC; ++e) {
          unsigned long long k = 0ull;
          if (grow < S.rows) k = argmax_key(round_bf(v[e]), static_cast<uint32_t>(S.col_base + grow));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
            k = other > k ? other : k;
          }
          if (lane == 0) kbuf[q * NN + tok0 + e] = k;
        }
        named_bar_sync(1, 32 * kTcDqWarps);
        const int t = threadIdx.x - 64;
        if (t < NN && t < A.M) {
          unsigned long long k = kbuf[t];
#pragma unroll
          for (int qq = 1; qq < 4; ++qq) k = kbuf[qq * NN + t] > k ? kbuf[qq * NN + t] : k;
          S.keys[static_cast<size_t>(tile) * S.key_ld + t] = k;
        }
      } else if (mode == EPI_F32 && A.npush > 0) {
        // this rank's values of the tile into every rank's receive slot
        const int grow = tile * kQpRows + row;
        const size_t ldo = static_cast<size_t>(S.ldo);
        const int M = A.M;
        if (grow < S.rows) {
#pragma unroll
          for (int r = 0; r < kQmmMaxPeers; ++r) {  // constant indices: the pointers straight from the parameters
            if (r >= A.npush) break;
            float* const dst = A.push[r];
#pragma unroll
            for (int e = 0; e < EC; ++e) {
              const int tok = tok0 + e;
              if (tok < M) dst[tok * ldo + grow] = v[e];
            }
          }
        }
        named_bar_sync(1, 32 * kTcDqWarps);
        if (threadIdx.x == 64) qmm_push_arrive(A, tile);
      } else {
        const int grow = tile * kQpRows + row;
        // the fields in registers: the stores would make the compiler re-read
        // them every token otherwise
        uint16_t* const out = S.out;
        float* const out32 = S.out32;
        const uint16_t* const resid = S.resid;
        const size_t ldo = static_cast<size_t>(S.ldo), ldr = static_cast<size_t>(S.ldr);
        const int M = A.M;
        if (grow < S.rows) {
#pragma unroll
          for (int e = 0; e < EC; ++e) {
            const int tok = tok0 + e;
            if (tok >= M) continue;
            const size_t o = tok * ldo + grow;
            if (mode == EPI_F32) {
              out32[o] = v[e];
            } else if (mode == EPI_RESID) {
              out[o] = f2bf(bf2f(resid[tok * ldr + grow]) + round_bf(v[e]));
            } else {
              out[o] = f2bf(v[e]);
            }
          }
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
}

// ---------------------------------------------------------------- packing
// Clears the flag of every tile holding a scale that is not below 0.5 in
// magnitude (bf16 exponent field >= 126, non-finite values included).
__global__ void qmm_pack_scan_kernel(const uint16_t* __restrict__ s, int rows, int G, unsigned char* __restrict__ flags,
                                     int per_tile) {
  const long long total = static_cast<long long>(rows) * G;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    if (((s[idx] >> 7) & 0xFF) >= 126) flags[(idx / G) / per_tile] = 0;
  }
}

// One thread per (tile, k block, row): 8 chunks of codes and 4 (scale, bias) pairs.
__global__ void qmm_pack_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                const uint16_t* __restrict__ b, int rows, int K, unsigned char* __restrict__ dst,
                                const unsigned char* __restrict__ flags, int per_tile, int row_off) {
  const int KB = (K + kQpBlockK - 1) / kQpBlockK;
  const int G = K / 64, KW = K / 8;
  const long long total = static_cast<long long>(rows) * KB;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(idx / KB), kb = static_cast<int>(idx - static_cast<long long>(r) * KB);
    const int t = r / per_tile, tr = row_off + r % per_tile;
    unsigned char* blk = dst + (static_cast<size_t>(t) * KB + kb) * kQpBlockBytes;
    const uint32_t* wr = w + static_cast<size_t>(r) * KW;
    for (int c = 0; c < 8; ++c) {
      uint32_t o[4];
      for (int j = 0; j < 4; ++j) {
        const int kw = kb * 32 + 4 * c + j;
        const uint32_t v = kw < KW ? wr[kw] : 0u;
        uint32_t p = 0;
        for (int e = 0; e < 8; ++e) {
          const int pos = (e & 1) ? 4 + (e >> 1) : (e >> 1);
          p |= ((v >> (4 * e)) & 15u) << (4 * pos);
        }
        o[j] = p;
      }
      *reinterpret_cast<uint4*>(blk + tr * 128 + ((c ^ qp_swz(tr)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    const bool fast = flags[t] != 0;
    uint32_t sbv[4];
    for (int g = 0; g < 4; ++g) {
      const int gg = kb * 4 + g;
      uint32_t sc = 0, bi = 0;
      if (gg < G) {
        sc = s[static_cast<size_t>(r) * G + gg];
        bi = b[static_cast<size_t>(r) * G + gg];
        // exact: |scale| < 0.5, so scale * 2^129 is a finite bf16 with the same digits
        if (fast) sc = f2bf(ldexpf(bf2f(static_cast<uint16_t>(sc)), 129));
      }
      sbv[g] = sc | (bi << 16);
    }
    *reinterpret_cast<uint4*>(blk + kQpCodeBytes + tr * 16) = make_uint4(sbv[0], sbv[1], sbv[2], sbv[3]);
  }
}

int g_tc_sms = 0;
bool g_tc_attr[3] = {false, false, false};

template <int NN>
void* tc_fn() {
  return reinterpret_cast<void*>(qmm_tc_kernel<NN>);
}

template <int NN>
int tc_occupancy() {
  const int idx = NN == 16 ? 0 : NN == 32 ? 1 : 2;
  if (!g_tc_attr[idx]) {
    cudaFuncSetAttribute(qmm_tc_kernel<NN>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcLayout<NN>::kSmem);
    g_tc_attr[idx] = true;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qmm_tc_kernel<NN>, kTcThreads, TcLayout<NN>::kSmem) !=
      cudaSuccess)
    n = 1;
  return std::max(1, std::min(n, 1));
}

// Split-K factor: spread tiles x k blocks over the CTA slots.  An SM streams
// about 2.6 blocks/us at the HBM roofline.
int tc_plan_ks(int tiles, int KB, int occ) {
  if (const char* v = std::getenv("IAM_QMM_TC_KS")) {
    const int k = std::atoi(v);
    if (k >= 1) return std::min(k, KB);
  }
  const double r_sm = 2.6, r_cta = 2.6, c0 = 2.0, c1 = 1.0;
  const long slots = static_cast<long>(g_tc_sms) * occ;
  double best = 1e30;
  int bk = 1;
  for (int ksp = 1; ksp <= std::min(KB, 32); ++ksp) {
    const long ctas = static_cast<long>(tiles) * ksp;
    const long waves = (ctas + slots - 1) / slots;
    const double per_sm = std::ceil(static_cast<double>(std::min(ctas, slots)) / g_tc_sms);
    const double blocks = std::ceil(static_cast<double>(KB) / ksp);
    const double t = waves * (blocks * per_sm / std::min(r_sm, per_sm * r_cta) + c0 + (ksp > 1 ? c1 : 0.0));
    if (t < best - 1e-9) {
      best = t;
      bk = ksp;
    }
  }
  return bk;
}

}  // namespace

int qmm_pack_begin(unsigned char* dst, int tiles, int K, cudaStream_t st) {
  IAM_CHECK(dst && tiles > 0 && K > 0, "qmm_pack_begin: bad arguments");
  IAM_CUDA(cudaMemsetAsync(dst + qp_blocks_bytes(tiles, K), 1, static_cast<size_t>(tiles), st));
  return IAM_OK;
}

int qmm_pack_scan(const uint16_t* s, int rows, int K, unsigned char* dst, int tiles, int per_tile, cudaStream_t st) {
  IAM_CHECK(s && dst && rows > 0 && K > 0 && K % 64 == 0 && (per_tile == 128 || per_tile == 64),
            "qmm_pack_scan: bad arguments");
  IAM_CHECK((rows + per_tile - 1) / per_tile <= tiles, "qmm_pack_scan: rows exceed the packed tiles");
  const long long total = static_cast<long long>(rows) * (K / 64);
  const int threads = 256;
  const int blocks = static_cast<int>(std::min<long long>((total + threads - 1) / threads, 148LL * 32));
  qmm_pack_scan_kernel<<<blocks, threads, 0, st>>>(s, rows, K / 64, dst + qp_blocks_bytes(tiles, K), per_tile);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

int qmm_pack(const uint32_t* w, const uint16_t* s, const uint16_t* b, int rows, int K, unsigned char* dst,
             int tiles, int per_tile, int row_off, cudaStream_t st) {
  IAM_CHECK(w && s && b && dst && rows > 0 && K > 0 && K % 64 == 0, "qmm_pack: bad arguments");
  IAM_CHECK((per_tile == 128 && row_off == 0) || (per_tile == 64 && (row_off == 0 || row_off == 64)),
            "qmm_pack: bad tile split");
  IAM_CHECK((rows + per_tile - 1) / per_tile <= tiles, "qmm_pack: rows exceed the packed tiles");
  IAM_CHECK(aligned16(dst), "qmm_pack: destination must be 16-byte aligned");
  const long long total = static_cast<long long>(rows) * qp_kblocks(K);
  const int threads = 128;
  const int blocks = static_cast<int>(std::min<long long>((total + threads - 1) / threads, 148LL * 64));
  qmm_pack_kernel<<<blocks, threads, 0, st>>>(w, s, b, rows, K, dst, dst + qp_blocks_bytes(tiles, K), per_tile,
                                              row_off);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

template <int NN>
static int tc_launch(const QmmTcArgs& ta, int ks, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ta.a.total_ctas, 1, ks);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = TcLayout<NN>::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  IAM_CUDA(cudaLaunchKernelEx(&cfg, qmm_tc_kernel<NN>, ta));
  return IAM_OK;
}

int qmm_tc_run(QmmArgs a, cudaStream_t st, bool pdl, size_t ws_floats_cap, size_t ws_ctr_cap) {
  IAM_CHECK(a.K > 0 && a.K % 64 == 0, "qmm: K must be a positive multiple of 64");
  IAM_CHECK(a.M >= 1 && a.M <= 64, "qmm: the tensor-core path takes 1..64 tokens a pass");
  IAM_CHECK(!a.norm_w, "qmm: the fused RMSNorm runs on the GEMV path only");
  IAM_CHECK(a.nseg >= 1 && a.nseg <= kQmmMaxSeg, "qmm: 1..4 segments");
  IAM_CHECK(aligned16(a.x) && a.ldx % 8 == 0 && a.ldx >= a.K, "qmm: x must be 16-byte aligned with ldx % 8 == 0");
  if (g_tc_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_tc_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_tc_sms <= 0) g_tc_sms = 148;
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
  const int NN = a.M <= 16 ? 16 : a.M <= 32 ? 32 : 64;
  const int KB = qp_kblocks(a.K);
  const int occ = NN == 16 ? tc_occupancy<16>() : NN == 32 ? tc_occupancy<32>() : tc_occupancy<64>();
  int ks = tc_plan_ks(cta, KB, occ);
  if (ks > 1 && a.ws) {  // a caller's workspace bounds the split
    const size_t per = static_cast<size_t>(cta) * kQpRows * NN;
    ks = static_cast<int>(std::min<size_t>(ks, ws_floats_cap / per));
    if (static_cast<size_t>(cta) > ws_ctr_cap) ks = 1;
    ks = std::max(ks, 1);
  }
  if (ks > 1) {
    const size_t nf = static_cast<size_t>(cta) * ks * kQpRows * NN, nc = static_cast<size_t>(cta);
    if (!a.ws) {
      const int r = qmm_op_workspace(1, nf, nc, st, &a.ws, &a.counters);
      if (r != IAM_OK) return r;
    } else {
      IAM_CHECK(nf <= ws_floats_cap && nc <= ws_ctr_cap, "qmm: split-K workspace too small");
    }
  }
  QmmTcArgs ta;
  std::memset(&ta, 0, sizeof(ta));
  ta.a = a;
  const int r = tma_encode_2d(&ta.xmap, a.x, 2, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.K), NN, 64, true,
                              static_cast<uint64_t>(a.ldx));
  if (r != IAM_OK) return r;
  if (NN == 16) return tc_launch<16>(ta, ks, st, pdl);
  return NN == 32 ? tc_launch<32>(ta, ks, st, pdl) : tc_launch<64>(ta, ks, st, pdl);
}

}  // namespace iam

extern "C" size_t iam_qmm_packed_bytes(int N, int K) {
  using namespace iam;
  if (N <= 0 || K <= 0 || K % 64 != 0) return 0;
  return qp_bytes(qp_tiles(N, false), K);
}

extern "C" int iam_qmm_pack_affine4(const uint32_t* w, const uint16_t* s, const uint16_t* b, void* packed, int N,
                                    int K, void* stream) {
  using namespace iam;
  IAM_CHECK(N > 0 && K > 0 && K % 64 == 0, "iam_qmm_pack_affine4: N > 0 and K a positive multiple of 64");
  IAM_CHECK(w && s && b && packed, "iam_qmm_pack_affine4: null pointer");
  const cudaStream_t st = as_stream(stream);
  const int tiles = qp_tiles(N, false);
  unsigned char* dst = static_cast<unsigned char*>(packed);
  IAM_CUDA(cudaMemsetAsync(packed, 0, qp_bytes(tiles, K), st));
  int r = qmm_pack_begin(dst, tiles, K, st);
  if (r == IAM_OK) r = qmm_pack_scan(s, N, K, dst, tiles, 128, st);
  if (r == IAM_OK) r = qmm_pack(w, s, b, N, K, dst, tiles, 128, 0, st);
  return r;
}

extern "C" int iam_qmm_affine4_packed(const void* packed, const uint16_t* x, uint16_t* y, int M, int N, int K,
                                      void* stream) {
  using namespace iam;
  IAM_CHECK(N > 0 && N % 8 == 0, "iam_qmm_affine4_packed: N must be a positive multiple of 8");
  IAM_CHECK(packed && x && y, "iam_qmm_affine4_packed: null pointer");
  QmmArgs a = {};
  a.x = x;
  a.ldx = K;
  a.M = M;
  a.K = K;
  a.nseg = 1;
  a.seg[0].packed = static_cast<const unsigned char*>(packed);
  a.seg[0].out = y;
  a.seg[0].ldo = N;
  a.seg[0].rows = N;
  a.seg[0].mode = EPI_STORE;
  return qmm_run(a, as_stream(stream), false);
}

extern "C" int iam_qmm_affine4_packed_checked(const void* packed, const uint16_t* x, uint16_t* y, int M, int N,
                                              int K, int wait_limit, int starve, void* stream) {
  using namespace iam;
  IAM_CHECK(N > 0 && N % 8 == 0, "iam_qmm_affine4_packed_checked: N must be a positive multiple of 8");
  IAM_CHECK(packed && x && y, "iam_qmm_affine4_packed_checked: null pointer");
  IAM_CHECK(wait_limit >= 0, "iam_qmm_affine4_packed_checked: wait_limit must be >= 0");
  const cudaStream_t st = as_stream(stream);
  int* d_status = nullptr;
  IAM_CUDA(cudaMalloc(&d_status, sizeof(int)));
  int h_status = 0;
  int r = IAM_OK;
  cudaError_t ce = cudaMemsetAsync(d_status, 0, sizeof(int), st);
  if (ce == cudaSuccess) {
    QmmArgs a = {};
    a.x = x;
    a.ldx = K;
    a.M = M;
    a.K = K;
    a.nseg = 1;
    a.err = d_status;
    a.wait_limit = wait_limit;
    a.starve = starve ? 1 : 0;
    a.seg[0].packed = static_cast<const unsigned char*>(packed);
    a.seg[0].out = y;
    a.seg[0].ldo = N;
    a.seg[0].rows = N;
    a.seg[0].mode = EPI_STORE;
    r = qmm_run(a, st, false);
    if (r == IAM_OK) {
      ce = cudaMemcpyAsync(&h_status, d_status, sizeof(int), cudaMemcpyDeviceToHost, st);
      if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
    }
  }
  cudaFree(d_status);
  if (r != IAM_OK) return r;
  IAM_CUDA(ce);
  if (h_status != IAM_OK)
    return fail(h_status, "iam_qmm_affine4_packed_checked: a bounded wait inside the matmul gave up");
  return IAM_OK;
}
