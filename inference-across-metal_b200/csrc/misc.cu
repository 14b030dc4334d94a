// Small kernels of the decode path: norms, element-wise ops, embedding,
// RoPE, argmax and the verify-block finalisation (operator level + engine).
#include <cmath>

#include "kernels.cuh"
#include "rmsnorm.cuh"

namespace iam {

// ---------------------------------------------------------------- RMSNorm
// rms_norm_bf16 (full_forward.swift:59-86), bit-exact with the reference's
// summation order (rmsnorm.cuh): the CTA stages the row in shared memory with
// one round of 16-byte loads, warp 0 reduces it, then the whole CTA writes
// out = bf16((x / rms) * w) with 16-byte accesses.  Requires dim % 256 == 0.
__global__ void __launch_bounds__(512) rms_norm_kernel(const uint16_t* __restrict__ x, int ldx,
                                                       const uint16_t* __restrict__ w, uint16_t* __restrict__ out,
                                                       int ldo, int dim, float eps) {
  extern __shared__ __align__(16) uint4 xs[];  // the row, staged in one round of loads
  const int row = blockIdx.x, tid = threadIdx.x;
  const int nv = dim / 8;
  // the norm weights do not depend on the preceding kernel: fetch them first
  // (dim <= 16384 and 512 threads: at most four 8-element chunks a thread)
  uint4 wreg[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = tid + r * static_cast<int>(blockDim.x);
    if (i < nv) wreg[r] = *reinterpret_cast<const uint4*>(w + 8 * i);
  }
  pdl_wait();
  pdl_trigger();
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * ldx);
  for (int i = tid; i < nv; i += blockDim.x) xs[i] = xr[i];
  __syncthreads();
  __shared__ float rms_s;
  if (tid < 32) {
    const float r = rms_row_warp([&](int i) { return xs[i]; }, dim, eps, tid);
    if (tid == 0) rms_s = r;
  }
  __syncthreads();
  const float rms = rms_s;
  uint16_t* orow = out + static_cast<size_t>(row) * ldo;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = tid + r * static_cast<int>(blockDim.x);
    if (i >= nv) break;
    *reinterpret_cast<uint4*>(orow + 8 * i) = rms_apply8(xs[i], wreg[r], rms);
  }
}

// The same for rows of exactly 256 * NJ elements, small enough (256
// threads, 1 KiB of shared memory, the row in registers) to become resident
// next to a matmul CTA that holds most of an SM, so that under programmatic
// dependent launch it starts early and runs the moment its input is written:
// thread t is the reference's thread t (it sums x[t + 256 j]^2 in j order) and
// the reference's tree (partial[t] += partial[t + s], s = 128 .. 1) runs
// through shared memory for s >= 32 and lane shuffles below.
template <int NJ>
__global__ void __launch_bounds__(256) rms_norm_row_kernel(const uint16_t* __restrict__ x, int ldx,
                                                           const uint16_t* __restrict__ w,
                                                           uint16_t* __restrict__ out, int ldo, float eps) {
  __shared__ float part[256];
  const int row = blockIdx.x, t = threadIdx.x;
  uint16_t wv[NJ], xv[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) wv[j] = w[t + 256 * j];  // before the wait: weights only
  pdl_wait();
  pdl_trigger();
  const uint16_t* xr = x + static_cast<size_t>(row) * ldx;
#pragma unroll
  for (int j = 0; j < NJ; ++j) xv[j] = xr[t + 256 * j];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const float v = bf2f(xv[j]);
    sum += v * v;
  }
  part[t] = sum;
  __syncthreads();
  if (t < 128) part[t] += part[t + 128];
  __syncthreads();
  if (t < 64) part[t] += part[t + 64];
  __syncthreads();
  if (t < 32) {
    float v = part[t] + part[t + 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_down_sync(0xffffffffu, v, o);
      if (t < o) v += u;
    }
    if (t == 0) part[0] = sqrtf(v / static_cast<float>(256 * NJ) + eps);
  }
  __syncthreads();
  const float rms = part[0];
  uint16_t* orow = out + static_cast<size_t>(row) * ldo;
#pragma unroll
  for (int j = 0; j < NJ; ++j) orow[t + 256 * j] = f2bf((bf2f(xv[j]) / rms) * bf2f(wv[j]));
}

int launch_rms_norm(const uint16_t* x, int ldx, const uint16_t* w, uint16_t* out, int ldo, int rows, int dim,
                    float eps, cudaStream_t st, bool pdl) {
  IAM_CHECK(dim % 256 == 0 && dim <= 16384, "rms_norm: dim must be a multiple of 256, at most 16384");
  IAM_CHECK(aligned16(x) && aligned16(w) && aligned16(out) && ldx % 8 == 0 && ldo % 8 == 0,
            "rms_norm: 16-byte aligned rows required");
  if (dim == 5120)  // the 27B hidden size
    return launch_k(rms_norm_row_kernel<20>, dim3(rows), dim3(256), 0, st, pdl, x, ldx, w, out, ldo, eps);
  return launch_k(rms_norm_kernel, dim3(rows), dim3(std::min(512, std::max(32, dim / 8))),
                  static_cast<size_t>(dim) * 2, st, pdl, x, ldx, w, out, ldo, dim, eps);
}

// ---------------------------------------------------------------- element-wise
__global__ void silu_multiply_kernel(const uint16_t* g, const uint16_t* u, uint16_t* out, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = f2bf(silu_f(bf2f(g[i])) * bf2f(u[i]));
}
__global__ void residual_add_kernel(const uint16_t* a, const uint16_t* b, uint16_t* out, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = f2bf(bf2f(a[i]) + bf2f(b[i]));
}
__global__ void sigmoid_gate_kernel(const uint16_t* a, const uint16_t* g, uint16_t* out, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = f2bf(bf2f(a[i]) * sigmoid_f(bf2f(g[i])));
}

static dim3 ew_grid(int n) { return dim3(std::min((n + 255) / 256, 148 * 16)); }

// ---------------------------------------------------------------- embedding
__global__ void embed_bf16_kernel(const uint16_t* __restrict__ table, const int32_t* __restrict__ tokens,
                                  uint16_t* __restrict__ out, int hidden, int vocab, int* err) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  int tok = tokens[r];
  if (tok < 0 || tok >= vocab) {  // never read outside the table; report when asked
    if (err && threadIdx.x == 0) atomicExch(err, 1);
    tok = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(tok) * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(r) * hidden);
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) dst[i] = src[i];
}

// embed_lookup_bf16 (full_forward.swift:112-133): bf16(float(q) * scale + bias)
__global__ void embed_q4_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                                const uint16_t* __restrict__ b, const int32_t* __restrict__ tokens,
                                uint16_t* __restrict__ out, int hidden, int group) {
  const int r = blockIdx.x;
  const size_t tok = static_cast<size_t>(tokens[r]);
  const int gpr = hidden / group;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const uint32_t word = w[tok * (hidden / 8) + i / 8];
    const float q = static_cast<float>((word >> (4 * (i % 8))) & 0xFu);
    out[static_cast<size_t>(r) * hidden + i] =
        f2bf(q * bf2f(s[tok * gpr + i / group]) + bf2f(b[tok * gpr + i / group]));
  }
}

// ---------------------------------------------------------------- RoPE
// rope_bf16 + precomputeRoPE (full_forward.swift:148-167, 734-743): angles in
// double, cos/sin stored fp32, adjacent pairs (2i, 2i+1) rotated in fp32.
__device__ __forceinline__ void rope_cs(int pos, int i, int rotary, float theta, float& c, float& s) {
  const double freq = 1.0 / pow(static_cast<double>(theta), static_cast<double>(2 * i) / static_cast<double>(rotary));
  const double ang = static_cast<double>(pos) * freq;
  c = static_cast<float>(cos(ang));
  s = static_cast<float>(sin(ang));
}

__global__ void rope_kernel(uint16_t* x, int heads, int head_dim, int rotary, float theta, int pos) {
  const int r = blockIdx.x, h = blockIdx.y, i = threadIdx.x;
  if (i >= rotary / 2) return;
  float c, s;
  rope_cs(pos + r, i, rotary, theta, c, s);
  uint16_t* p = x + (static_cast<size_t>(r) * heads + h) * head_dim + 2 * i;
  const float x0 = bf2f(p[0]), x1 = bf2f(p[1]);
  p[0] = f2bf(x0 * c - x1 * s);
  p[1] = f2bf(x0 * s + x1 * c);
}

// ---------------------------------------------------------------- per-head norms
// per_head_rms_norm_bf16 (full_forward.swift:185-207); the sum runs in index
// order like the reference's per-thread loop.
__global__ void per_head_rms_norm_kernel(const uint16_t* x, const uint16_t* w, uint16_t* out, int head_dim,
                                         float eps) {
  const size_t base = static_cast<size_t>(blockIdx.x) * head_dim;
  __shared__ float rms;
  if (threadIdx.x == 0) {
    float ss = 0.f;
    for (int i = 0; i < head_dim; ++i) {
      const float v = bf2f(x[base + i]);
      ss += v * v;
    }
    rms = sqrtf(ss / static_cast<float>(head_dim) + eps);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < head_dim; e += blockDim.x)
    out[base + e] = f2bf((bf2f(x[base + e]) / rms) * bf2f(w[e]));
}

// rms_norm_gated_bf16 (full_forward.swift:357-381)
__global__ void rms_norm_gated_kernel(const uint16_t* y, const uint16_t* z, const uint16_t* w, uint16_t* out,
                                      int head_dim, float eps) {
  const size_t base = static_cast<size_t>(blockIdx.x) * head_dim;
  __shared__ float rms;
  if (threadIdx.x == 0) {
    float ss = 0.f;
    for (int i = 0; i < head_dim; ++i) {
      const float v = bf2f(y[base + i]);
      ss += v * v;
    }
    rms = sqrtf(ss / static_cast<float>(head_dim) + eps);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < head_dim; e += blockDim.x) {
    const float xn = (bf2f(y[base + e]) / rms) * bf2f(w[e]);
    out[base + e] = f2bf(silu_f(bf2f(z[base + e])) * xn);
  }
}

__global__ void g_beta_kernel(const uint16_t* a, const uint16_t* b, const float* A_log, const uint16_t* dt,
                              uint16_t* g, uint16_t* beta, int rows, int heads) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * heads) return;
  const int h = i % heads;
  float gv, bv;
  g_beta(bf2f(a[i]), bf2f(b[i]), A_log[h], bf2f(dt[h]), gv, bv);
  g[i] = f2bf(gv);
  beta[i] = f2bf(bv);
}

// depthwise_conv1d_m1_bf16 (full_forward.swift:240-263) over `rows` tokens:
// window [s0, s1, s2, x_t] slides one token at a time.
__global__ void conv1d_step_kernel(const uint16_t* st_in, const uint16_t* x, const uint16_t* w, uint16_t* out,
                                   uint16_t* st_out, int C, int rows) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  uint16_t w0 = st_in[c], w1 = st_in[C + c], w2 = st_in[2 * C + c];
  const float k0 = bf2f(w[4 * c]), k1 = bf2f(w[4 * c + 1]), k2 = bf2f(w[4 * c + 2]), k3 = bf2f(w[4 * c + 3]);
  for (int r = 0; r < rows; ++r) {
    const uint16_t xi = x[static_cast<size_t>(r) * C + c];
    float sum = 0.f;
    sum += bf2f(w0) * k0;
    sum += bf2f(w1) * k1;
    sum += bf2f(w2) * k2;
    sum += bf2f(xi) * k3;
    out[static_cast<size_t>(r) * C + c] = f2bf(sum);
    w0 = w1;
    w1 = w2;
    w2 = xi;
  }
  st_out[c] = w0;
  st_out[C + c] = w1;
  st_out[2 * C + c] = w2;
}

// ---------------------------------------------------------------- argmax
// argmax_bf16 (full_forward.swift:169-183): first index of the maximum.
__global__ void argmax_rows_kernel(const uint16_t* x, int32_t* out, int count) {
  const uint16_t* row = x + static_cast<size_t>(blockIdx.x) * count;
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const unsigned long long k = argmax_key(bf2f(row[i]), static_cast<uint32_t>(i));
    best = k > best ? k : best;
  }
  __shared__ unsigned long long sh[32];
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
    best = v > best ? v : best;
  }
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    best = threadIdx.x < blockDim.x / 32 ? sh[threadIdx.x] : 0ull;
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
      best = v > best ? v : best;
    }
    if (threadIdx.x == 0) out[blockIdx.x] = static_cast<int32_t>(argmax_key_index(best));
  }
}

__device__ __forceinline__ unsigned long long best_key_of_row(const unsigned long long* __restrict__ keys, int nparts,
                                                             int key_ld, int r, unsigned long long* sh) {
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
    const unsigned long long k = keys[static_cast<size_t>(i) * key_ld + r];
    best = k > best ? k : best;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
    best = v > best ? v : best;
  }
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = best;
  __syncthreads();
  best = (threadIdx.x & 31) < blockDim.x / 32 ? sh[threadIdx.x & 31] : 0ull;
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
    best = v > best ? v : best;
  }
  __syncthreads();
  return best;
}

// The best key of row r over the parts, by one warp (lane 0's result; the
// maximum does not depend on the order).
__device__ __forceinline__ unsigned long long best_key_of_row_warp(const unsigned long long* __restrict__ keys,
                                                                  int nparts, int key_ld, int r, int lane) {
  unsigned long long best = 0ull;
  for (int i = lane; i < nparts; i += 32) {
    const unsigned long long k = keys[static_cast<size_t>(i) * key_ld + r];
    best = k > best ? k : best;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
    best = v > best ? v : best;
  }
  return best;
}

// Verify-block finalisation: reduce the lm_head's per-CTA keys of every row,
// then the greedy accept length (largest j with tokens[j+1] == argmax[j] for
// every smaller j; tokens[0] is the token being decoded).
__global__ void __launch_bounds__(1024) finalize_kernel(const unsigned long long* __restrict__ keys, int nparts,
                                                        int key_ld, int M, const int32_t* __restrict__ tokens,
                                                        int32_t* __restrict__ argmax_out, int32_t* accept) {
  pdl_wait();
  pdl_trigger();
  __shared__ int32_t am[kMaxRowsFinalize];
  // one warp a row, the rows in parallel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < M; r += blockDim.x >> 5) {
    const unsigned long long best = best_key_of_row_warp(keys, nparts, key_ld, r, lane);
    if (lane == 0) {
      am[r] = static_cast<int32_t>(argmax_key_index(best));
      argmax_out[r] = am[r];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && accept) {
    int j = 0;
    while (j + 1 < M && tokens[j + 1] == am[j]) ++j;
    *accept = j;
  }
}

__global__ void __launch_bounds__(1024) best_keys_kernel(const unsigned long long* __restrict__ keys, int nparts,
                                                         int key_ld, int M, unsigned long long* best_out) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < M; r += blockDim.x >> 5) {
    const unsigned long long best = best_key_of_row_warp(keys, nparts, key_ld, r, lane);
    if (lane == 0) best_out[r] = best;
  }
}

// Multi-sequence finalisation, one CTA a row: the row's best key over the
// nparts partial keys (lm_head tiles, or ranks) -> argmax index, or (best_out)
// the key itself for the cross-rank reduction.
__global__ void __launch_bounds__(256) finalize_rows_kernel(const unsigned long long* __restrict__ keys, int nparts,
                                                            int key_ld, int32_t* argmax_out,
                                                            unsigned long long* best_out) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned long long sh[32];
  const unsigned long long best = best_key_of_row(keys, nparts, key_ld, blockIdx.x, sh);
  if (threadIdx.x == 0) {
    if (best_out) best_out[blockIdx.x] = best;
    else argmax_out[blockIdx.x] = static_cast<int32_t>(argmax_key_index(best));
  }
}

// Each sequence's greedy accept length over its seq_rows rows (the rule of
// finalize_kernel).
__global__ void accept_kernel(const int32_t* __restrict__ tokens, const int32_t* __restrict__ argmax, int n_seq,
                              int seq_rows, int32_t* accept) {
  pdl_wait();
  pdl_trigger();
  for (int q = threadIdx.x; q < n_seq; q += blockDim.x) {
    const int32_t* tk = tokens + static_cast<size_t>(q) * seq_rows;
    const int32_t* am = argmax + static_cast<size_t>(q) * seq_rows;
    int j = 0;
    while (j + 1 < seq_rows && tk[j + 1] == am[j]) ++j;
    accept[q] = j;
  }
}

int launch_finalize_batch(const unsigned long long* keys, int nparts, int key_ld, int n_seq, int seq_rows,
                          const int32_t* tokens, int32_t* argmax_out, int32_t* accept, cudaStream_t st, bool pdl) {
  IAM_CHECK(n_seq >= 1 && seq_rows >= 1 && n_seq * seq_rows <= key_ld, "finalize: bad sequence shape");
  const int r = launch_k(finalize_rows_kernel, dim3(n_seq * seq_rows), dim3(256), 0, st, pdl, keys, nparts, key_ld,
                         argmax_out, static_cast<unsigned long long*>(nullptr));
  if (r != IAM_OK) return r;
  return launch_k(accept_kernel, dim3(1), dim3(256), 0, st, pdl, tokens, static_cast<const int32_t*>(argmax_out),
                  n_seq, seq_rows, accept);
}

int launch_best_rows(const unsigned long long* keys, int nparts, int key_ld, int M, unsigned long long* best,
                     cudaStream_t st, bool pdl) {
  return launch_k(finalize_rows_kernel, dim3(M), dim3(256), 0, st, pdl, keys, nparts, key_ld,
                  static_cast<int32_t*>(nullptr), best);
}

int launch_finalize(const unsigned long long* keys, int nparts, int key_ld, int M, const int32_t* tokens,
                    int32_t* argmax_out, int32_t* accept, cudaStream_t st, bool pdl) {
  IAM_CHECK(M <= kMaxRowsFinalize, "finalize: too many rows");
  return launch_k(finalize_kernel, dim3(1), dim3(1024), 0, st, pdl, keys, nparts, key_ld, M, tokens, argmax_out,
                  accept);
}

int launch_best_keys(const unsigned long long* keys, int nparts, int key_ld, int M, unsigned long long* best,
                     cudaStream_t st, bool pdl) {
  return launch_k(best_keys_kernel, dim3(1), dim3(1024), 0, st, pdl, keys, nparts, key_ld, M, best);
}

int launch_embed_bf16(const uint16_t* table, const int32_t* tokens, uint16_t* out, int rows, int hidden, int vocab,
                      int* err, cudaStream_t st, bool pdl) {
  return launch_k(embed_bf16_kernel, dim3(rows), dim3(256), 0, st, pdl, table, tokens, out, hidden, vocab, err);
}

}  // namespace iam

// ====================================================================== C ABI
using namespace iam;

extern "C" int iam_rms_norm_bf16(const uint16_t* x, const uint16_t* weight, uint16_t* out, int rows, int dim,
                                 float eps, void* stream) {
  IAM_CHECK(x && weight && out && rows > 0 && dim > 0, "iam_rms_norm_bf16: bad arguments");
  return launch_rms_norm(x, dim, weight, out, dim, rows, dim, eps, as_stream(stream), false);
}

extern "C" int iam_silu_multiply_bf16(const uint16_t* gate, const uint16_t* up, uint16_t* out, int count,
                                      void* stream) {
  IAM_CHECK(gate && up && out && count > 0, "iam_silu_multiply_bf16: bad arguments");
  silu_multiply_kernel<<<ew_grid(count), 256, 0, as_stream(stream)>>>(gate, up, out, count);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

extern "C" int iam_residual_add_bf16(const uint16_t* a, const uint16_t* b, uint16_t* out, int count, void* stream) {
  IAM_CHECK(a && b && out && count > 0, "iam_residual_add_bf16: bad arguments");
  residual_add_kernel<<<ew_grid(count), 256, 0, as_stream(stream)>>>(a, b, out, count);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

extern "C" int iam_sigmoid_gate_bf16(const uint16_t* a, const uint16_t* gate, uint16_t* out, int count,
                                     void* stream) {
  IAM_CHECK(a && gate && out && count > 0, "iam_sigmoid_gate_bf16: bad arguments");
  sigmoid_gate_kernel<<<ew_grid(count), 256, 0, as_stream(stream)>>>(a, gate, out, count);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

extern "C" int iam_embed_lookup_q4(const uint32_t* w, const uint16_t* s, const uint16_t* b, const int32_t* tokens,
                                   uint16_t* out, int rows, int hidden, int group_size, void* stream) {
  IAM_CHECK(w && s && b && tokens && out && rows > 0, "iam_embed_lookup_q4: bad arguments");
  IAM_CHECK(hidden % 64 == 0 && group_size == 64, "iam_embed_lookup_q4: hidden % 64 and group 64 required");
  embed_q4_kernel<<<rows, 256, 0, as_stream(stream)>>>(w, s, b, tokens, out, hidden, group_size);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

extern "C" int iam_embed_lookup_bf16(const uint16_t* table, const int32_t* tokens, uint16_t* out, int rows,
                                     int hidden, int vocab, void* stream) {
  IAM_CHECK(table && tokens && out && rows > 0 && hidden % 8 == 0, "iam_embed_lookup_bf16: bad arguments");
  IAM_CHECK(aligned16(table) && aligned16(out), "iam_embed_lookup_bf16: pointers must be 16-byte aligned");
  return launch_embed_bf16(table, tokens, out, rows, hidden, vocab, nullptr, as_stream(stream), false);
}

extern "C" int iam_rope_bf16(uint16_t* x, int rows, int num_heads, int head_dim, int rotary_dim, float theta, int pos,
                             void* stream) {
  IAM_CHECK(x && rows > 0 && num_heads > 0 && rotary_dim % 2 == 0 && rotary_dim <= head_dim && rotary_dim <= 2048,
            "iam_rope_bf16: bad arguments");
  rope_kernel<<<dim3(rows, num_heads), std::max(32, rotary_dim / 2), 0, as_stream(stream)>>>(x, num_heads, head_dim,
                                                                                          rotary_dim, theta, pos);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

extern "C" int iam_argmax_bf16(const uint16_t* x, int32_t* out, int rows, int count, void* stream) {
  IAM_CHECK(x && out && rows > 0 && count > 0, "iam_argmax_bf16: bad arguments");
  argmax_rows_kernel<<<rows, 1024, 0, as_stream(stream)>>>(x, out, count);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

extern "C" int iam_per_head_rms_norm_bf16(const uint16_t* x, const uint16_t* weight, uint16_t* out, int rows,
                                          int num_heads, int head_dim, float eps, void* stream) {
  IAM_CHECK(x && weight && out && rows > 0 && num_heads > 0 && head_dim > 0, "iam_per_head_rms_norm_bf16: bad args");
  per_head_rms_norm_kernel<<<rows * num_heads, 256, 0, as_stream(stream)>>>(x, weight, out, head_dim, eps);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

extern "C" int iam_rms_norm_gated_bf16(const uint16_t* y, const uint16_t* z, const uint16_t* w, uint16_t* out,
                                       int rows, int num_heads, int head_dim, float eps, void* stream) {
  IAM_CHECK(y && z && w && out && rows > 0 && num_heads > 0 && head_dim > 0, "iam_rms_norm_gated_bf16: bad args");
  rms_norm_gated_kernel<<<rows * num_heads, 128, 0, as_stream(stream)>>>(y, z, w, out, head_dim, eps);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

extern "C" int iam_compute_g_beta(const uint16_t* a, const uint16_t* b, const float* A_log, const uint16_t* dt_bias,
                                  uint16_t* g, uint16_t* beta, int rows, int n_v_heads, void* stream) {
  IAM_CHECK(a && b && A_log && dt_bias && g && beta && rows > 0 && n_v_heads > 0, "iam_compute_g_beta: bad args");
  const int n = rows * n_v_heads;
  g_beta_kernel<<<(n + 127) / 128, 128, 0, as_stream(stream)>>>(a, b, A_log, dt_bias, g, beta, rows, n_v_heads);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}

extern "C" int iam_depthwise_conv1d_step(const uint16_t* state_in, const uint16_t* x, const uint16_t* w,
                                         uint16_t* out, uint16_t* state_out, int channels, int rows, void* stream) {
  IAM_CHECK(state_in && x && w && out && state_out && channels > 0 && rows > 0, "iam_depthwise_conv1d_step: bad args");
  IAM_CHECK(state_in != state_out, "iam_depthwise_conv1d_step: state_out must not alias state_in");
  conv1d_step_kernel<<<(channels + 255) / 256, 256, 0, as_stream(stream)>>>(state_in, x, w, out, state_out, channels,
                                                                             rows);
  IAM_CUDA(cudaGetLastError());
  return IAM_OK;
}
