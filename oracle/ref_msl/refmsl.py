"""ctypes access to oracle/_ref/libref_msl.so: the reference's Metal kernels
compiled for the host (test infrastructure only).

Arrays are numpy: bf16 tensors as uint16, fp32 as float32, codes as uint32.
Every function returns new arrays and leaves inputs untouched (except the ones
the reference kernel updates in place, which are copied first).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_LIB = None
LIB_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_ref", "libref_msl.so")


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _LIB
    if _LIB is None:
        _LIB = C.CDLL(LIB_PATH)
    return _LIB


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _u16(a):
    return np.ascontiguousarray(a, dtype=np.uint16)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def rms_norm(x, w, eps=1e-6):
    x = _u16(x).reshape(-1, np.shape(x)[-1])
    out = np.empty_like(x)
    lib().ref_rms_norm_bf16(_p(x), _p(_u16(w)), _p(out), C.c_uint(x.shape[0]), C.c_uint(x.shape[1]), C.c_float(eps))
    return out


def silu_multiply(g, u):
    g, u = _u16(g), _u16(u)
    out = np.empty_like(g)
    lib().ref_silu_multiply_bf16(_p(g), _p(u), _p(out), C.c_uint(g.size))
    return out


def residual_add(a, b):
    a, b = _u16(a), _u16(b)
    out = np.empty_like(a)
    lib().ref_residual_add_bf16(_p(a), _p(b), _p(out), C.c_uint(a.size))
    return out


def embed_lookup(w, s, b, token, group=64):
    w = np.ascontiguousarray(w, np.uint32)
    s, b = _u16(s), _u16(b)
    hidden = w.shape[1] * 8
    out = np.empty(hidden, np.uint16)
    lib().ref_embed_lookup_bf16(_p(w), _p(s), _p(b), _p(out), C.c_uint(token), C.c_uint(hidden), C.c_uint(group))
    return out


def sigmoid_multiply(a, b):
    a, b = _u16(a), _u16(b)
    out = np.empty_like(a)
    lib().ref_sigmoid_multiply_bf16(_p(a), _p(b), _p(out), C.c_uint(a.size))
    return out


def rope(x, cosv, sinv, rotary):
    x = _u16(x).copy()
    heads, hd = x.shape
    lib().ref_rope_bf16(_p(x), _p(_f32(cosv)), _p(_f32(sinv)), C.c_uint(heads), C.c_uint(hd), C.c_uint(rotary))
    return x


def argmax(x):
    x = _u16(x)
    r = np.zeros(1, np.uint32)
    lib().ref_argmax_bf16(_p(x), _p(r), C.c_uint(x.size))
    return int(r[0])


def per_head_rms_norm(x, w, eps=1e-6):
    x = _u16(x)
    out = np.empty_like(x)
    lib().ref_per_head_rms_norm_bf16(_p(x), _p(_u16(w)), _p(out), C.c_uint(x.shape[0]), C.c_uint(x.shape[1]),
                                     C.c_float(eps))
    return out


def expand_kv_heads(kv, heads):
    kv = _u16(kv)
    out = np.empty((heads, kv.shape[1]), np.uint16)
    lib().ref_expand_kv_heads_bf16(_p(kv), _p(out), C.c_uint(heads), C.c_uint(kv.shape[0]), C.c_uint(kv.shape[1]))
    return out


def split_q_gate(qg, heads, head_dim):
    qg = _u16(qg)
    q = np.empty((heads, head_dim), np.uint16)
    g = np.empty((heads, head_dim), np.uint16)
    lib().ref_split_q_gate_bf16(_p(qg), _p(q), _p(g), C.c_uint(heads), C.c_uint(head_dim))
    return q, g


def depthwise_conv1d(state, x, w):
    state, x, w = _u16(state), _u16(x), _u16(w)
    out = np.empty_like(x)
    ns = np.empty_like(state)
    lib().ref_depthwise_conv1d_m1_bf16(_p(state), _p(x), _p(w), _p(out), _p(ns), C.c_uint(x.size))
    return out, ns


def silu(x):
    x = _u16(x)
    out = np.empty_like(x)
    lib().ref_silu_bf16(_p(x), _p(out), C.c_uint(x.size))
    return out


def per_head_rms_norm_scaled(x, eps, scale):
    x = _u16(x)
    out = np.empty_like(x)
    lib().ref_per_head_rms_norm_scaled_bf16(_p(x), _p(out), C.c_uint(x.shape[0]), C.c_uint(x.shape[1]),
                                            C.c_float(eps), C.c_float(scale))
    return out


def compute_g_beta(a, b, A_log, dt_bias):
    a, b, dt = _u16(a), _u16(b), _u16(dt_bias)
    g = np.empty_like(a)
    beta = np.empty_like(a)
    lib().ref_compute_g_beta_bf16(_p(a), _p(b), _p(_f32(A_log)), _p(dt), _p(g), _p(beta), C.c_uint(a.size))
    return g, beta


def gated_delta_step(q, k, v, g, beta, state):
    q, k, v, g, beta = (_u16(t) for t in (q, k, v, g, beta))
    st = _f32(state).copy()
    vh, dv, dk = st.shape
    y = np.empty((vh, dv), np.uint16)
    lib().ref_gated_delta_step_bf16(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(st), _p(y), C.c_uint(vh),
                                    C.c_uint(dv), C.c_uint(dk))
    return y, st


def rms_norm_gated(x, z, w, eps=1e-6):
    x, z = _u16(x), _u16(z)
    out = np.empty_like(x)
    lib().ref_rms_norm_gated_bf16(_p(x), _p(z), _p(_u16(w)), _p(out), C.c_uint(x.shape[0]), C.c_uint(x.shape[1]),
                                  C.c_float(eps))
    return out


def sdpa_decode(q, kc, vc, seq_len):
    q, kc, vc = _u16(q), _u16(kc), _u16(vc)
    heads, hd = q.shape
    out = np.empty_like(q)
    lib().ref_sdpa_decode_bf16(_p(q), _p(kc), _p(vc), _p(out), C.c_uint(heads), C.c_uint(kc.shape[1]), C.c_uint(hd),
                               C.c_uint(seq_len))
    return out
