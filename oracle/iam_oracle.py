"""CPU oracle for the Qwen3.5-27B-shape decode / K-token verify path.

TEST INFRASTRUCTURE ONLY: the tests, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may call this module, and only to check or to
time the reference arithmetic.  The product path (libiamcuda.so) never calls
it and has no CPU fallback.

Every function restates one kernel of the reference, in numpy float32, with the
bf16 rounding at exactly the points where the reference stores a bf16 result.
Citations are file:line in the reference project (inference-across-metal).
The reference's own Metal kernels are additionally compiled for the host from
their source (oracle/ref_msl) and tests check this restatement against them
(tests/test_oracle_pin.py), so the restatement is pinned for every kernel the
reference ships as source.  The quantized matmul is MLX 0.31.1's binary
``affine_qmm_t_nax_bfloat16_t_gs_64_b_4`` kernel (absent, not inspected); it is
restated from the MLX API semantics the reference itself verified against:
``mx.dequantize -> matmul`` (kernel_dispatch.swift:6-14, RESULTS.md:28-33), with
the dequant formula pinned by the reference's embed_lookup_bf16 kernel.

Arrays hold bf16 *values* as float32 unless stated; ``bf16()`` rounds
(round-to-nearest-even, the rounding of Metal's float->bfloat conversion).
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np
import ml_dtypes

BF16 = ml_dtypes.bfloat16


def bf16(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(BF16).astype(np.float32)


def to_u16(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(BF16).view(np.uint16)


def from_u16(u) -> np.ndarray:
    return np.asarray(u, dtype=np.uint16).view(BF16).astype(np.float32)


# --------------------------------------------------------------------------
# model dimensions (full_forward.swift:18-49)
# --------------------------------------------------------------------------

@dataclasses.dataclass(frozen=True)
class Dims:
    hidden: int = 5120
    intermediate: int = 17408
    vocab: int = 248320
    n_layers: int = 64
    full_attn_interval: int = 4
    n_heads: int = 24
    n_kv_heads: int = 4
    head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 1.0e7
    gdn_k_heads: int = 16
    gdn_v_heads: int = 48
    gdn_dk: int = 128
    gdn_dv: int = 128
    conv_kernel: int = 4
    group: int = 64
    eps: float = 1e-6

    @property
    def key_dim(self) -> int:
        return self.gdn_k_heads * self.gdn_dk

    @property
    def value_dim(self) -> int:
        return self.gdn_v_heads * self.gdn_dv

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    def is_full_attn(self, layer: int) -> bool:
        # isFullAttn, full_forward.swift:47-49
        return (layer + 1) % self.full_attn_interval == 0


QWEN35_27B = Dims()
# A small member of the same family for fast parity tests: same head sizes,
# fewer heads/layers.  GQA ratios (3:1 GDN, 2:1 attention) are kept non-trivial.
TINY = Dims(hidden=512, intermediate=1024, vocab=4096, n_layers=4, n_heads=4, n_kv_heads=2,
            gdn_k_heads=2, gdn_v_heads=6)

# GDN_INV_SCALE is a Swift Float literal; q uses its square computed in fp32
# (full_forward.swift:41, 1056, 1064).
GDN_INV_SCALE = np.float32(0.08838834764)
GDN_Q_SCALE = np.float32(GDN_INV_SCALE * GDN_INV_SCALE)
GDN_K_SCALE = GDN_INV_SCALE


# --------------------------------------------------------------------------
# kernels
# --------------------------------------------------------------------------

def unpack_codes(w: np.ndarray) -> np.ndarray:
    """uint32 [N, K/8] -> uint8 codes [N, K]; nibble i of word j is column 8j+i,
    low nibble first (embed_lookup_bf16, full_forward.swift:123-128)."""
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    q = (w[..., None] >> shifts) & np.uint32(0xF)
    return q.reshape(*w.shape[:-1], w.shape[-1] * 8).astype(np.uint8)


# Diagnostic switch for tests: keep the dequantised weight in fp32 instead of
# rounding it to bf16 as mx.dequantize does.
EXACT_DEQUANT = False


# An implementation computing the same bits faster (oracle/fast.py, checked
# against this function by tests/test_oracle_fast.py), or None.
_DEQUANT_IMPL = None


def set_dequant_impl(fn):
    """Routes dequant() through ``fn`` (None: this module's numpy statement);
    returns the previous setting."""
    global _DEQUANT_IMPL
    prev, _DEQUANT_IMPL = _DEQUANT_IMPL, fn
    return prev


def dequant(w, s, b, group: int = 64) -> np.ndarray:
    """MLX affine dequant to bf16: w = bf16(q * scale + bias), computed in fp32
    (float(nibble) * scale + bias, full_forward.swift:129-132)."""
    if _DEQUANT_IMPL is not None and not EXACT_DEQUANT:
        return _DEQUANT_IMPL(w, s, b, group)
    q = unpack_codes(w).astype(np.float32)
    sc = np.repeat(np.asarray(s, np.float32), group, axis=-1)
    bi = np.repeat(np.asarray(b, np.float32), group, axis=-1)
    v = (q * sc + bi).astype(np.float32)
    return v if EXACT_DEQUANT else bf16(v)


_DEQ_CACHE: dict = {}


def cache_dequant(enable: bool = True):
    """Memoise dequant() per weight array (for tests that step a layer many times)."""
    global _DEQ_ON
    _DEQ_ON = enable
    _DEQ_CACHE.clear()


_DEQ_ON = False


def _dequant_rows(w, s, b, r0, r1, group):
    if not _DEQ_ON:
        return dequant(w[r0:r1], s[r0:r1], b[r0:r1], group)
    key = (id(w), r0, r1)
    hit = _DEQ_CACHE.get(key)
    if hit is None or hit[0] is not w:
        hit = (w, dequant(w[r0:r1], s[r0:r1], b[r0:r1], group))
        _DEQ_CACHE[key] = hit
    return hit[1]


def qmm_affine4(x, w, s, b, group: int = 64, row_chunk: int = 8192, round_out: bool = True) -> np.ndarray:
    """y[M, N] = bf16(x[M, K] . dequant(W)[N, K]^T), fp32 accumulation.

    The MLX qmm as dispatched by dispatchQMatmul (full_forward.swift:711-728) and
    encodeQMM (batch_verify_27b.swift:100-119); semantics = mx.dequantize ->
    matmul (kernel_dispatch.swift:6-14).  ``round_out=False`` keeps the fp32
    accumulator (a tensor-parallel partial product before its all-reduce)."""
    x = np.asarray(x, np.float32)
    squeeze = x.ndim == 1
    x2 = x.reshape(1, -1) if squeeze else x
    n = w.shape[0]
    y = np.empty((x2.shape[0], n), np.float32)
    for r0 in range(0, n, row_chunk):
        r1 = min(n, r0 + row_chunk)
        wd = _dequant_rows(w, s, b, r0, r1, group)
        y[:, r0:r1] = x2 @ wd.T
    if round_out:
        y = bf16(y)
    return y[0] if squeeze else y


def rms_norm(x, w, eps: float = 1e-6) -> np.ndarray:
    """rms_norm_bf16 (full_forward.swift:59-86): rms = sqrt(sum(x^2)/dim + eps);
    out = bf16((x / rms) * w).  Rows are independent."""
    x = np.asarray(x, np.float32)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=np.float32)
    rms = np.sqrt(ss / np.float32(x.shape[-1]) + np.float32(eps)).astype(np.float32)
    return bf16((x / rms) * np.asarray(w, np.float32))


def silu_f32(v) -> np.ndarray:
    v = np.asarray(v, np.float32)
    return (v / (np.float32(1.0) + np.exp(-v))).astype(np.float32)


def silu_multiply(g, u) -> np.ndarray:
    """silu_multiply_bf16 (full_forward.swift:88-99)."""
    return bf16(silu_f32(g) * np.asarray(u, np.float32))


def residual_add(a, b) -> np.ndarray:
    """residual_add_bf16 (full_forward.swift:101-110)."""
    return bf16(np.asarray(a, np.float32) + np.asarray(b, np.float32))


def embed_lookup_4bit(w, s, b, token: int, group: int = 64) -> np.ndarray:
    """embed_lookup_bf16 (full_forward.swift:112-133): dequant one row."""
    q = unpack_codes(w[token]).astype(np.float32)
    sc = np.repeat(np.asarray(s[token], np.float32), group)
    bi = np.repeat(np.asarray(b[token], np.float32), group)
    return bf16(q * sc + bi)


def embed_lookup_bf16_table(table, tokens) -> np.ndarray:
    """bf16 embedding table (the benchmark's variant of full_forward.swift:112-133)."""
    return np.asarray(table, np.float32)[np.asarray(tokens)]


def sigmoid_multiply(a, b) -> np.ndarray:
    """sigmoid_multiply_bf16 (full_forward.swift:135-146): bf16(a * sigmoid(b))."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return bf16(a * (np.float32(1.0) / (np.float32(1.0) + np.exp(-b))))


def rope_tables(position: int, rotary_dim: int = 64, theta: float = 1.0e7):
    """precomputeRoPE (full_forward.swift:734-743): angles in double, stored fp32."""
    i = np.arange(rotary_dim // 2, dtype=np.float64)
    freq = 1.0 / np.power(np.float64(np.float32(theta)), (2.0 * i) / rotary_dim)
    ang = float(position) * freq
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope(x, position: int, rotary_dim: int = 64, theta: float = 1.0e7) -> np.ndarray:
    """rope_bf16 (full_forward.swift:148-167): adjacent pairs (2i, 2i+1), i < rotary/2,
    rotated in fp32 and stored bf16; dims >= rotary_dim untouched.  x: [heads, head_dim]."""
    x = np.array(x, np.float32, copy=True)
    c, s = rope_tables(position, rotary_dim, theta)
    x0 = x[:, 0:rotary_dim:2].copy()
    x1 = x[:, 1:rotary_dim:2].copy()
    x[:, 0:rotary_dim:2] = bf16(x0 * c - x1 * s)
    x[:, 1:rotary_dim:2] = bf16(x0 * s + x1 * c)
    return x


def argmax_first(x) -> np.ndarray:
    """argmax_bf16 (full_forward.swift:169-183): strict '>' scan, ties -> first index."""
    return np.argmax(np.asarray(x, np.float32), axis=-1)


def per_head_rms_norm(x, w, eps: float = 1e-6) -> np.ndarray:
    """per_head_rms_norm_bf16 (full_forward.swift:185-207). x: [heads, d]."""
    return rms_norm(x, w, eps)


def depthwise_conv1d_step(state, x, w):
    """depthwise_conv1d_m1_bf16 (full_forward.swift:240-263).
    state bf16 [3, C], x bf16 [C], w bf16 [C, 4] -> (out bf16 [C], new_state [3, C]).
    sum = ((0 + s0*w0) + s1*w1) + s2*w2 + x*w3 in fp32 (no bias)."""
    state = np.asarray(state, np.float32)
    x = np.asarray(x, np.float32)
    w = np.asarray(w, np.float32)
    acc = np.zeros_like(x)
    win = [state[0], state[1], state[2], x]
    for i in range(4):
        acc = (acc + (win[i] * w[:, i]).astype(np.float32)).astype(np.float32)
    new_state = np.stack([state[1], state[2], x])
    return bf16(acc), new_state


def silu(x) -> np.ndarray:
    """silu_bf16 (full_forward.swift:265-274)."""
    return bf16(silu_f32(x))


def per_head_rms_norm_scaled(x, scale, eps: float = 1e-6) -> np.ndarray:
    """per_head_rms_norm_scaled_bf16 (full_forward.swift:276-297):
    out = bf16(scale * (x / sqrt(mean(x^2) + eps))).  x: [heads, d]."""
    x = np.asarray(x, np.float32)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=np.float32)
    rms = np.sqrt(ss / np.float32(x.shape[-1]) + np.float32(eps)).astype(np.float32)
    return bf16(np.float32(scale) * (x / rms))


def compute_g_beta(a, b, A_log, dt_bias):
    """compute_g_beta_bf16 (full_forward.swift:299-319):
    g = bf16(exp(-exp(A_log) * softplus(a + dt_bias))) with softplus(x) = x for x > 20;
    beta = bf16(sigmoid(b))."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    sp_in = (a + np.asarray(dt_bias, np.float32)).astype(np.float32)
    with np.errstate(over="ignore"):
        sp = np.where(sp_in > np.float32(20.0), sp_in,
                      np.log(np.float32(1.0) + np.exp(sp_in)).astype(np.float32))
    g = np.exp(-np.exp(np.asarray(A_log, np.float32)) * sp).astype(np.float32)
    beta = (np.float32(1.0) / (np.float32(1.0) + np.exp(-b))).astype(np.float32)
    return bf16(g), bf16(beta)


def expand_heads(x, n_out: int) -> np.ndarray:
    """expand_kv_heads_bf16 (full_forward.swift:209-222): out[h] = in[h / (n_out / n_in)]."""
    rep = n_out // x.shape[0]
    return np.repeat(np.asarray(x, np.float32), rep, axis=0)


def gated_delta_step(q, k, v, g, beta, S):
    """gated_delta_step_bf16 (full_forward.swift:321-355), one token.

    q, k: [Hv, dk] (already expanded), v: [Hv, dv], g, beta: [Hv], S: fp32 [Hv, dv, dk]
    updated in place.  Per row dv of head h:
      s = S*g; kv = s . k; delta = (v - kv) * beta; S = s + k*delta; y = S . q
    Returns y bf16 [Hv, dv]."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    g = np.asarray(g, np.float32)
    beta = np.asarray(beta, np.float32)
    S *= g[:, None, None]
    kv = np.einsum("hvk,hk->hv", S, k, dtype=np.float32)
    delta = ((np.asarray(v, np.float32) - kv) * beta[:, None]).astype(np.float32)
    S += (k[:, None, :] * delta[:, :, None]).astype(np.float32)
    y = np.einsum("hvk,hk->hv", S, q, dtype=np.float32)
    return bf16(y)


def rms_norm_gated(x, z, w, eps: float = 1e-6) -> np.ndarray:
    """rms_norm_gated_bf16 (full_forward.swift:357-381), per head of x: [H, d]:
    out = bf16(silu(z) * ((x / rms) * w)).  The gate is SiLU(z) in the reference."""
    x = np.asarray(x, np.float32)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=np.float32)
    rms = np.sqrt(ss / np.float32(x.shape[-1]) + np.float32(eps)).astype(np.float32)
    xn = ((x / rms) * np.asarray(w, np.float32)).astype(np.float32)
    return bf16(silu_f32(z) * xn)


def sdpa_decode(q, k_cache, v_cache, seq_len: int) -> np.ndarray:
    """sdpa_decode_bf16 (full_forward.swift:396-444) without its 1024-token cap.
    q: [Hq, d]; caches: [T, Hkv, d]; attends to t < seq_len; scale 1/sqrt(d);
    max-subtracted softmax in fp32; out bf16 [Hq, d]."""
    q = np.asarray(q, np.float32)
    hq, d = q.shape
    hkv = k_cache.shape[1]
    rep = hq // hkv
    kc = np.asarray(k_cache[:seq_len], np.float32)
    vc = np.asarray(v_cache[:seq_len], np.float32)
    out = np.empty((hq, d), np.float32)
    scale = np.float32(1.0) / np.sqrt(np.float32(d))
    for h in range(hq):
        kvh = h // rep
        sc = (kc[:, kvh, :] @ q[h]).astype(np.float32) * scale
        e = np.exp(sc - sc.max()).astype(np.float32)
        p = (e / e.sum(dtype=np.float32)).astype(np.float32)
        out[h] = p @ vc[:, kvh, :]
    return bf16(out)


# --------------------------------------------------------------------------
# layers and the model step
# --------------------------------------------------------------------------

def mlp(normed, W, prefix, rowpar=qmm_affine4):
    """dispatchMLP (full_forward.swift:1167-1190).  ``rowpar`` is the down_proj
    matmul (the tensor-parallel variant sums partial products over ranks)."""
    gate = qmm_affine4(normed, *W[prefix + "mlp.gate_proj"])
    up = qmm_affine4(normed, *W[prefix + "mlp.up_proj"])
    return rowpar(silu_multiply(gate, up), *W[prefix + "mlp.down_proj"])


def gdn_block(hidden, W, prefix, conv_state, S, dims: Dims, rowpar=qmm_affine4):
    """dispatchGDNLayer (full_forward.swift:993-1161) for M tokens run as M sequential
    decode steps.  hidden [M, H] bf16; conv_state [3, C] bf16 and S [Hv, dv, dk] fp32
    are updated in place.  Returns the new hidden [M, H].  ``rowpar`` is the
    out_proj / down_proj matmul."""
    d = dims
    normed = rms_norm(hidden, W[prefix + "input_layernorm.weight"], d.eps)
    qkv = qmm_affine4(normed, *W[prefix + "linear_attn.in_proj_qkv"])
    z = qmm_affine4(normed, *W[prefix + "linear_attn.in_proj_z"])
    bproj = qmm_affine4(normed, *W[prefix + "linear_attn.in_proj_b"])
    aproj = qmm_affine4(normed, *W[prefix + "linear_attn.in_proj_a"])
    convw = W[prefix + "linear_attn.conv1d.weight"]
    A_log = W[prefix + "linear_attn.A_log"]
    dt_bias = W[prefix + "linear_attn.dt_bias"]
    normw = W[prefix + "linear_attn.norm.weight"]
    gn = np.empty((hidden.shape[0], d.value_dim), np.float32)
    for t in range(hidden.shape[0]):
        co, ns = depthwise_conv1d_step(conv_state, qkv[t], convw)
        conv_state[...] = ns
        cs = silu(co)
        q = cs[: d.key_dim].reshape(d.gdn_k_heads, d.gdn_dk)
        k = cs[d.key_dim: 2 * d.key_dim].reshape(d.gdn_k_heads, d.gdn_dk)
        v = cs[2 * d.key_dim:].reshape(d.gdn_v_heads, d.gdn_dv)
        qn = expand_heads(per_head_rms_norm_scaled(q, GDN_Q_SCALE, 1e-6), d.gdn_v_heads)
        kn = expand_heads(per_head_rms_norm_scaled(k, GDN_K_SCALE, 1e-6), d.gdn_v_heads)
        g, beta = compute_g_beta(aproj[t], bproj[t], A_log, dt_bias)
        y = gated_delta_step(qn, kn, v, g, beta, S)
        gn[t] = rms_norm_gated(y, z[t].reshape(d.gdn_v_heads, d.gdn_dv), normw, d.eps).reshape(-1)
    out = rowpar(gn, *W[prefix + "linear_attn.out_proj"])
    resid = residual_add(hidden, out)
    normed2 = rms_norm(resid, W[prefix + "post_attention_layernorm.weight"], d.eps)
    return residual_add(resid, mlp(normed2, W, prefix, rowpar))


def attn_block(hidden, W, prefix, k_cache, v_cache, pos: int, dims: Dims, rowpar=qmm_affine4):
    """dispatchAttnLayer (full_forward.swift:828-987) for M tokens at positions
    pos..pos+M-1 (causal inside the block).  Caches [T, Hkv, d] bf16 are appended
    in place: k is normed+roped, v raw (full_forward.swift:909-924).  ``rowpar``
    is the o_proj / down_proj matmul."""
    d = dims
    m = hidden.shape[0]
    normed = rms_norm(hidden, W[prefix + "input_layernorm.weight"], d.eps)
    qg = qmm_affine4(normed, *W[prefix + "self_attn.q_proj"])
    kp = qmm_affine4(normed, *W[prefix + "self_attn.k_proj"])
    vp = qmm_affine4(normed, *W[prefix + "self_attn.v_proj"])
    qnw = W[prefix + "self_attn.q_norm.weight"]
    knw = W[prefix + "self_attn.k_norm.weight"]
    gated = np.empty((m, d.n_heads * d.head_dim), np.float32)
    qs = []
    for t in range(m):
        # split_q_gate_bf16 (full_forward.swift:224-238): per head [q | gate]
        qgh = qg[t].reshape(d.n_heads, 2 * d.head_dim)
        q = qgh[:, : d.head_dim]
        qn = rope(per_head_rms_norm(q, qnw, d.eps), pos + t, d.rotary_dim, d.rope_theta)
        kn = rope(per_head_rms_norm(kp[t].reshape(d.n_kv_heads, d.head_dim), knw, d.eps),
                  pos + t, d.rotary_dim, d.rope_theta)
        k_cache[pos + t] = kn
        v_cache[pos + t] = vp[t].reshape(d.n_kv_heads, d.head_dim)
        qs.append((qn, qgh[:, d.head_dim:]))
    for t in range(m):
        qn, gate = qs[t]
        att = sdpa_decode(qn, k_cache, v_cache, pos + t + 1)
        gated[t] = sigmoid_multiply(att.reshape(-1), gate.reshape(-1))
    o = rowpar(gated, *W[prefix + "self_attn.o_proj"])
    resid = residual_add(hidden, o)
    normed2 = rms_norm(resid, W[prefix + "post_attention_layernorm.weight"], d.eps)
    return residual_add(resid, mlp(normed2, W, prefix, rowpar))


def accept_length(tokens, argmax) -> int:
    """Greedy accept length of a verify block: the largest j such that
    tokens[i+1] == argmax[i] for every i < j (tokens[0] is the token being decoded)."""
    j = 0
    while j + 1 < len(tokens) and int(tokens[j + 1]) == int(argmax[j]):
        j += 1
    return j


@dataclasses.dataclass
class State:
    conv: dict      # gdn layer index -> bf16 values [3, C] (float32 array)
    S: dict         # gdn layer index -> fp32 [Hv, dv, dk]
    k_cache: dict   # attention layer index -> [T, Hkv, d]
    v_cache: dict


def model_step(tokens, pos: int, W, state: State, dims: Dims, return_hidden: bool = False,
               rowpar=qmm_affine4, lm_argmax=argmax_first):
    """forwardPass (full_forward.swift:1198-1308) for a verify block of K tokens at
    positions pos..pos+K-1: embedding, 64-layer loop, final norm, lm_head, argmax.
    Returns (argmax [K], accept_len[, final normed hidden, logits]).  ``rowpar``
    and ``lm_argmax`` are the hooks the tensor-parallel restatement
    (oracle/tp.py) replaces."""
    d = dims
    hidden = embed_lookup_bf16_table(W["model.embed_tokens.weight"], tokens)
    for li in range(d.n_layers):
        prefix = f"model.layers.{li}."
        if d.is_full_attn(li):
            hidden = attn_block(hidden, W, prefix, state.k_cache[li], state.v_cache[li], pos, d, rowpar)
        else:
            hidden = gdn_block(hidden, W, prefix, state.conv[li], state.S[li], d, rowpar)
    normed = rms_norm(hidden, W["model.norm.weight"], d.eps)
    logits = qmm_affine4(normed, *W["lm_head"])
    am = lm_argmax(logits)
    out = (am, accept_length(tokens, am))
    if return_hidden:
        out = out + (normed, logits)
    return out
