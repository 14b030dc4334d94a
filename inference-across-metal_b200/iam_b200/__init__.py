"""ctypes binding of libiamcuda.so (include/iam.h).

The host side mirrors the reference's operator surface (the Metal kernels of
full_forward.swift:55-445 and the qmm dispatch of full_forward.swift:711-728)
and its model entry points (forwardPass, full_forward.swift:1198-1308; the
M-row verify of batch_verify_27b.swift:141-274).  Operator calls take device
pointers as integers (e.g. ``tensor.data_ptr()``) and an optional CUDA stream
handle; every call raises IamError on a non-zero status.

There is no CPU path: importing works anywhere the shared library exists, and
every compute call needs a CUDA device.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libiamcuda.so")

IAM_OK, IAM_EINVAL, IAM_ECUDA, IAM_ENCCL, IAM_ETIMEOUT, IAM_ENOMEM, IAM_ESTATE = range(7)

# every entry point of include/iam.h with (restype, argtypes)
_vp, _i, _f, _u64, _sz, _cp = C.c_void_p, C.c_int, C.c_float, C.c_uint64, C.c_size_t, C.c_char_p
_SIGS = {
    "iam_last_error": (C.c_char_p, []),
    "iam_status_string": (C.c_char_p, [_i]),
    "iam_version": (_i, []),
    "iam_qmm_affine4": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "iam_qmm_affine4_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "iam_qmm_affine4_packed_checked": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "iam_engine_status": (_i, [_vp, _vp]),
    "iam_qmm_affine4_plan": (_i, [_i, _i, _i, C.POINTER(C.c_int), C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "iam_qmm_packed_bytes": (_sz, [_i, _i]),
    "iam_qmm_pack_affine4": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "iam_qmm_affine4_packed": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "iam_rms_norm_bf16": (_i, [_vp, _vp, _vp, _i, _i, _f, _vp]),
    "iam_silu_multiply_bf16": (_i, [_vp, _vp, _vp, _i, _vp]),
    "iam_residual_add_bf16": (_i, [_vp, _vp, _vp, _i, _vp]),
    "iam_embed_lookup_q4": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "iam_embed_lookup_bf16": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "iam_sigmoid_gate_bf16": (_i, [_vp, _vp, _vp, _i, _vp]),
    "iam_rope_bf16": (_i, [_vp, _i, _i, _i, _i, _f, _i, _vp]),
    "iam_argmax_bf16": (_i, [_vp, _vp, _i, _i, _vp]),
    "iam_per_head_rms_norm_bf16": (_i, [_vp, _vp, _vp, _i, _i, _i, _f, _vp]),
    "iam_depthwise_conv1d_step": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _vp]),
    "iam_compute_g_beta": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp]),
    "iam_gated_delta_step": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "iam_rms_norm_gated_bf16": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _f, _vp]),
    "iam_gdn_step_fused": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f,
                                _vp]),
    "iam_sdpa_decode_append": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "iam_dims_qwen35_27b": (None, [_vp]),
    "iam_tp_shard_of": (_i, [_vp, _i, _i, _vp]),
    "iam_create": (_i, [_vp, _i, _i, _i, _vp, _vp]),
    "iam_nccl_unique_id": (_i, [_vp]),
    "iam_destroy": (None, [_vp]),
    "iam_engine_error": (C.c_char_p, [_vp]),
    "iam_load_tensor": (_i, [_vp, _cp, _vp, _sz]),
    "iam_load_safetensors": (_i, [_vp, _vp, _i]),
    "iam_check_safetensors": (_i, [_vp, _vp, _i, _vp, _sz]),
    "iam_init_synthetic": (_i, [_vp, _u64]),
    "iam_state_init": (_i, [_vp, _u64, _i]),
    "iam_state_reset": (_i, [_vp]),
    "iam_verify": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "iam_decode_step": (_i, [_vp, C.c_int32, _i, _vp]),
    "iam_generate": (_i, [_vp, _vp, _i, _i, _vp, _i, _vp, _vp]),
    "iam_verify_device": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "iam_rollback": (_i, [_vp, _i, _vp]),
    "iam_read_tensor": (_i, [_vp, _cp, _vp, _sz]),
    "iam_read_hidden": (_i, [_vp, _vp, _i]),
    "iam_profile_step": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "iam_step_launches": (_i, [_vp, _i]),
    "iam_streamed_layers": (_i, [_vp]),
    "iam_profile_layers": (_i, [_vp, _i, _i, _vp, _vp, _vp]),
    "iam_step_bytes": (C.c_double, [_vp, _i, _i]),
    "iam_step_bytes_batch": (C.c_double, [_vp, _i, _i, _i]),
    "iam_verify_batch": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp]),
    "iam_verify_batch_device": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp, _vp]),
}

_LIB = None


class IamError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{msg} (status {status})")
        self.status = status


def lib():
    """Load libiamcuda.so; raises if it was not built (no fallback exists)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise IamError(IAM_ESTATE, f"{LIB_PATH} is missing: build it with `make -C inference-across-metal_b200`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def exported_symbols():
    return list(_SIGS)


def _check(status: int, engine=None):
    if status != IAM_OK:
        msg = lib().iam_engine_error(engine).decode() if engine is not None else ""
        if not msg:
            msg = lib().iam_last_error().decode()
        raise IamError(status, msg)


def _s(stream):
    return None if stream is None else C.c_void_p(stream if isinstance(stream, int) else int(stream))


# ------------------------------------------------------------ operator level
def qmm_affine4(w, s, b, x, y, M, N, K, group_size=64, stream=None):
    _check(lib().iam_qmm_affine4(w, s, b, x, y, M, N, K, group_size, _s(stream)))


def qmm_affine4_noalloc(w, s, b, x, y, M, N, K, group_size=64, stream=None):
    _check(lib().iam_qmm_affine4_noalloc(w, s, b, x, y, M, N, K, group_size, _s(stream)))


def qmm_affine4_plan(M, N, K):
    """(splits, scratch floats, scratch counters) of the matmul plan for a shape."""
    ks, nf, nc = C.c_int(0), C.c_size_t(0), C.c_size_t(0)
    _check(lib().iam_qmm_affine4_plan(M, N, K, C.byref(ks), C.byref(nf), C.byref(nc)))
    return ks.value, nf.value, nc.value


def qmm_affine4_packed_checked(packed, x, y, M, N, K, wait_limit=0, starve=False, stream=None):
    _check(lib().iam_qmm_affine4_packed_checked(packed, x, y, M, N, K, wait_limit, int(bool(starve)), _s(stream)))


def qmm_packed_bytes(N, K) -> int:
    return int(lib().iam_qmm_packed_bytes(N, K))


def qmm_pack_affine4(w, s, b, packed, N, K, stream=None):
    _check(lib().iam_qmm_pack_affine4(w, s, b, packed, N, K, _s(stream)))


def qmm_affine4_packed(packed, x, y, M, N, K, stream=None):
    _check(lib().iam_qmm_affine4_packed(packed, x, y, M, N, K, _s(stream)))


def rms_norm_bf16(x, weight, out, rows, dim, eps=1e-6, stream=None):
    _check(lib().iam_rms_norm_bf16(x, weight, out, rows, dim, eps, _s(stream)))


def silu_multiply_bf16(gate, up, out, count, stream=None):
    _check(lib().iam_silu_multiply_bf16(gate, up, out, count, _s(stream)))


def residual_add_bf16(a, b, out, count, stream=None):
    _check(lib().iam_residual_add_bf16(a, b, out, count, _s(stream)))


def embed_lookup_q4(w, s, b, tokens, out, rows, hidden, group_size=64, stream=None):
    _check(lib().iam_embed_lookup_q4(w, s, b, tokens, out, rows, hidden, group_size, _s(stream)))


def embed_lookup_bf16(table, tokens, out, rows, hidden, vocab, stream=None):
    _check(lib().iam_embed_lookup_bf16(table, tokens, out, rows, hidden, vocab, _s(stream)))


def sigmoid_gate_bf16(a, gate, out, count, stream=None):
    _check(lib().iam_sigmoid_gate_bf16(a, gate, out, count, _s(stream)))


def rope_bf16(x, rows, num_heads, head_dim, rotary_dim, theta, pos, stream=None):
    _check(lib().iam_rope_bf16(x, rows, num_heads, head_dim, rotary_dim, theta, pos, _s(stream)))


def argmax_bf16(x, out, rows, count, stream=None):
    _check(lib().iam_argmax_bf16(x, out, rows, count, _s(stream)))


def per_head_rms_norm_bf16(x, weight, out, rows, num_heads, head_dim, eps=1e-6, stream=None):
    _check(lib().iam_per_head_rms_norm_bf16(x, weight, out, rows, num_heads, head_dim, eps, _s(stream)))


def depthwise_conv1d_step(state_in, x, w, out, state_out, channels, rows, stream=None):
    _check(lib().iam_depthwise_conv1d_step(state_in, x, w, out, state_out, channels, rows, _s(stream)))


def compute_g_beta(a, b, A_log, dt_bias, g, beta, rows, n_v_heads, stream=None):
    _check(lib().iam_compute_g_beta(a, b, A_log, dt_bias, g, beta, rows, n_v_heads, _s(stream)))


def gated_delta_step(q, k, v, g, beta, S, y, n_v_heads, n_k_heads, dk, dv, rows, stream=None):
    _check(lib().iam_gated_delta_step(q, k, v, g, beta, S, y, n_v_heads, n_k_heads, dk, dv, rows, _s(stream)))


def rms_norm_gated_bf16(y, z, w, out, rows, num_heads, head_dim, eps=1e-6, stream=None):
    _check(lib().iam_rms_norm_gated_bf16(y, z, w, out, rows, num_heads, head_dim, eps, _s(stream)))


def gdn_step_fused(qkvzab, ld_in, z_col, a_col, b_col, conv_w, conv_in, conv_out, A_log, dt_bias, norm_w, S, out,
                   ld_out, n_k_heads, n_v_heads, rows, eps=1e-6, stream=None):
    _check(lib().iam_gdn_step_fused(qkvzab, ld_in, z_col, a_col, b_col, conv_w, conv_in, conv_out, A_log, dt_bias,
                                    norm_w, S, out, ld_out, n_k_heads, n_v_heads, rows, eps, _s(stream)))


def sdpa_decode_append(q, k_new, v_new, k_cache, v_cache, out, rows, pos, n_q_heads, n_kv_heads, head_dim, max_ctx,
                       stream=None):
    _check(lib().iam_sdpa_decode_append(q, k_new, v_new, k_cache, v_cache, out, rows, pos, n_q_heads, n_kv_heads,
                                        head_dim, max_ctx, _s(stream)))


# ------------------------------------------------------------ engine level
class Dims(C.Structure):
    _fields_ = [(n, C.c_float if n in ("rope_theta", "eps") else C.c_int) for n in (
        "hidden", "intermediate", "vocab", "n_layers", "full_attn_interval", "n_heads", "n_kv_heads", "head_dim",
        "rotary_dim", "rope_theta", "gdn_k_heads", "gdn_v_heads", "gdn_dk", "gdn_dv", "conv_kernel", "group_size",
        "eps", "max_ctx", "max_rows", "max_seqs", "comm_timeout_ms")] + [("resident_weight_bytes", C.c_longlong)]

    @classmethod
    def qwen35_27b(cls, **over):
        d = cls()
        lib().iam_dims_qwen35_27b(C.byref(d))
        for k, v in over.items():
            setattr(d, k, v)
        return d


class TpShard(C.Structure):
    """iam_tp_shard: [first, first + count) ranges of one tensor-parallel rank."""
    _fields_ = [(n, C.c_int) for n in (
        "gdn_k_head0", "gdn_k_heads", "gdn_v_head0", "gdn_v_heads", "q_head0", "q_heads", "kv_head0", "kv_heads",
        "inter0", "inter", "vocab0", "vocab")]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


def tp_shard_of(dims: Dims, rank: int, world: int) -> TpShard:
    """The shard the engine of `rank` holds when the model is split over `world`
    GPUs (host only; needs no GPU)."""
    out = TpShard()
    _check(lib().iam_tp_shard_of(C.byref(dims), rank, world, C.byref(out)))
    return out


def check_safetensors(dims: Dims, paths):
    """(status, report): do the files hold exactly the model `dims` describes? (host only)"""
    arr = (C.c_char_p * len(paths))(*[os.fsencode(p) for p in paths])
    buf = C.create_string_buffer(1 << 16)
    st = lib().iam_check_safetensors(C.byref(dims), arr, len(paths), buf, len(buf))
    return st, buf.value.decode()


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    _check(lib().iam_nccl_unique_id(buf))
    return buf.raw


class Engine:
    """One GPU (or one tensor-parallel shard) holding a Qwen3.5-shape model."""

    def __init__(self, dims: Dims, device: int = 0, rank: int = 0, world: int = 1, nccl_id: bytes | None = None):
        self.dims = dims
        h = C.c_void_p()
        idbuf = C.create_string_buffer(nccl_id, 128) if nccl_id else None
        _check(lib().iam_create(C.byref(dims), device, rank, world, idbuf, C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().iam_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _c(self, status):
        _check(status, self._h)

    def load_tensor(self, name: str, host_array):
        import numpy as np
        a = np.ascontiguousarray(host_array)
        self._c(lib().iam_load_tensor(self._h, name.encode(), a.ctypes.data_as(C.c_void_p), a.nbytes))

    def load_safetensors(self, paths):
        """Load every weight from the safetensors files of an MLX 4-bit checkpoint."""
        arr = (C.c_char_p * len(paths))(*[os.fsencode(p) for p in paths])
        self._c(lib().iam_load_safetensors(self._h, arr, len(paths)))

    def init_synthetic(self, seed: int):
        self._c(lib().iam_init_synthetic(self._h, seed))

    def state_init(self, seed: int, ctx: int):
        self._c(lib().iam_state_init(self._h, seed, ctx))

    def state_reset(self):
        self._c(lib().iam_state_reset(self._h))

    def verify(self, tokens, pos: int):
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(len(t), np.int32)
        acc = C.c_int(0)
        self._c(lib().iam_verify(self._h, t.ctypes.data_as(C.c_void_p), len(t), pos,
                                 out.ctypes.data_as(C.c_void_p), C.byref(acc)))
        return out, acc.value

    def rollback(self, n_keep: int, stream=None):
        """Keep the state after the first n_keep tokens of the last verify block
        (accept_len + 1 after a greedy verify)."""
        self._c(lib().iam_rollback(self._h, n_keep, _s(stream)))

    def generate(self, prompt, max_new: int, eos=(248046, 248044)):
        """Greedy generation from a reset state; returns the generated token ids."""
        import numpy as np
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        e = np.ascontiguousarray(list(eos), dtype=np.int32)
        out = np.zeros(max_new, np.int32)
        n = C.c_int(0)
        self._c(lib().iam_generate(self._h, p.ctypes.data_as(C.c_void_p), len(p), max_new,
                                   e.ctypes.data_as(C.c_void_p), len(e), out.ctypes.data_as(C.c_void_p),
                                   C.byref(n)))
        return out[:n.value]

    def verify_device(self, d_tokens, K: int, pos: int, d_argmax=None, stream=None):
        self._c(lib().iam_verify_device(self._h, d_tokens, K, pos, d_argmax, _s(stream)))

    def verify_batch(self, tokens, pos):
        """tokens [n_seq, K] (row 0 of each: the token being decoded), pos [n_seq]
        -> (argmax [n_seq, K], accept_len [n_seq]); sequence q uses slot q."""
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        n, K = t.shape
        p = np.ascontiguousarray(pos, dtype=np.int32)
        am = np.zeros((n, K), np.int32)
        acc = np.zeros(n, np.int32)
        self._c(lib().iam_verify_batch(self._h, t.ctypes.data_as(C.c_void_p), n, K, p.ctypes.data_as(C.c_void_p),
                                       am.ctypes.data_as(C.c_void_p), acc.ctypes.data_as(C.c_void_p)))
        return am, acc

    def verify_batch_device(self, d_tokens, n_seq: int, K: int, d_pos=None, d_argmax=None, d_accept=None,
                            stream=None):
        self._c(lib().iam_verify_batch_device(self._h, d_tokens, n_seq, K, d_pos, d_argmax, d_accept, _s(stream)))

    def step_bytes_batch(self, n_seq: int, K: int, pos: int) -> float:
        return lib().iam_step_bytes_batch(self._h, n_seq, K, pos)

    def read_tensor(self, name: str, nbytes: int):
        import numpy as np
        buf = np.empty(nbytes, np.uint8)
        self._c(lib().iam_read_tensor(self._h, name.encode(), buf.ctypes.data_as(C.c_void_p), nbytes))
        return buf

    def status(self, stream=None):
        """iam_engine_status: raises IamError for a device-side failure so far."""
        self._c(lib().iam_engine_status(self._h, _s(stream)))

    def read_hidden(self, K: int):
        import numpy as np
        out = np.empty((K, self.dims.hidden), np.uint16)
        self._c(lib().iam_read_hidden(self._h, out.ctypes.data_as(C.c_void_p), K))
        return out

    def profile_step(self, K: int, pos: int, cap: int = 32):
        kinds = (C.c_char_p * cap)()
        ms = (C.c_double * cap)()
        by = (C.c_double * cap)()
        n = (C.c_int * cap)()
        got = lib().iam_profile_step(self._h, K, pos, cap, kinds, ms, by, n)
        if got < 0:
            self._c(-got)
        return {kinds[i].decode(): {"ms": ms[i], "bytes": by[i], "launches": n[i]} for i in range(got)}

    def profile_layers(self, K: int, pos: int):
        """[(is_attention, block ms, MLP ms)] per decoder layer of one eager step
        (CUDA events around every launch)."""
        n = self.dims.n_layers
        ms = (C.c_double * n)()
        mm = (C.c_double * n)()
        at = (C.c_int * n)()
        got = lib().iam_profile_layers(self._h, K, pos, ms, mm, at)
        if got < 0:
            self._c(-got)
        return [(bool(at[i]), ms[i], mm[i]) for i in range(got)]

    def streamed_layers(self) -> int:
        """Layers whose 4-bit matrices stream from pinned host memory each step."""
        return lib().iam_streamed_layers(self._h)

    def step_launches(self, K: int) -> int:
        return lib().iam_step_launches(self._h, K)

    def step_bytes(self, K: int, pos: int) -> float:
        return lib().iam_step_bytes(self._h, K, pos)
