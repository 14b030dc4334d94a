"""Tensor-parallel restatement of the verify step: TEST INFRASTRUCTURE ONLY.

The reference runs on one device; the tensor-parallel split is this project's
(include/iam.h, iam_tp_shard_of).  This module restates what each rank of the
engine computes, in the oracle's arithmetic, so a multi-process test can check
that the ranks' partial products summed over the ranks reproduce the
unsharded oracle step:

* column-parallel matmuls (in_proj_*, q/k/v_proj, gate/up_proj, lm_head) keep
  the rows of the rank's heads / columns, and the per-head kernels run on the
  rank's heads only;
* row-parallel matmuls (out_proj, o_proj, down_proj) keep the matching input
  features; each rank forms its fp32 partial product, the partials are summed
  over the ranks (all-reduce), and the residual add rounds the sum to bf16
  first: out = bf16(resid + bf16(sum)), the engine's resid_from_f32 step;
* lm_head: each rank takes the (bf16 value, first index) maximum over its
  vocab rows; the ranks' pairs are gathered and the largest value wins, the
  smaller global index on a tie, which is the first-index rule of argmax_bf16
  (full_forward.swift:169-183) over the whole vocabulary.

``shard`` is a dict with the fields of iam_tp_shard.
"""
from __future__ import annotations

import dataclasses

import numpy as np

from .iam_oracle import Dims, State, bf16, model_step, qmm_affine4


def local_dims(d: Dims, shard: dict) -> Dims:
    """The dims one rank's per-head kernels see."""
    return dataclasses.replace(
        d, gdn_k_heads=shard["gdn_k_heads"], gdn_v_heads=shard["gdn_v_heads"], n_heads=shard["q_heads"],
        n_kv_heads=shard["kv_heads"], intermediate=shard["inter"], vocab=shard["vocab"])


def qkv_channels(d: Dims, shard: dict) -> np.ndarray:
    """in_proj_qkv rows / conv channels of the rank: its q heads, k heads, v heads."""
    gd, dv = d.gdn_dk, d.gdn_dv
    k0, nk = shard["gdn_k_head0"], shard["gdn_k_heads"]
    v0, nv = shard["gdn_v_head0"], shard["gdn_v_heads"]
    return np.concatenate([
        np.arange(k0 * gd, (k0 + nk) * gd),
        d.key_dim + np.arange(k0 * gd, (k0 + nk) * gd),
        2 * d.key_dim + np.arange(v0 * dv, (v0 + nv) * dv),
    ])


def _rows(q, idx):
    w, s, b = q
    return (w[idx], s[idx], b[idx])


def _cols(q, c0: int, c1: int, group: int):
    """Input features [c0, c1) of a 4-bit matrix (8 codes per word, one scale per group)."""
    assert c0 % group == 0 and c1 % group == 0
    w, s, b = q
    return (w[:, c0 // 8: c1 // 8], s[:, c0 // group: c1 // group], b[:, c0 // group: c1 // group])


def shard_weights(W: dict, d: Dims, shard: dict) -> dict:
    """The tensors rank ``shard`` holds, by the engine's split (csrc/engine.cu, build_registry)."""
    g, hd, dv = d.group, d.head_dim, d.gdn_dv
    v0, nv = shard["gdn_v_head0"], shard["gdn_v_heads"]
    h0, nq = shard["q_head0"], shard["q_heads"]
    kv0, nkv = shard["kv_head0"], shard["kv_heads"]
    i0, ni = shard["inter0"], shard["inter"]
    voc0, nvoc = shard["vocab0"], shard["vocab"]
    qkv = qkv_channels(d, shard)
    out = {}
    for name, t in W.items():
        if name == "lm_head":
            out[name] = _rows(t, slice(voc0, voc0 + nvoc))
        elif name.endswith("self_attn.q_proj"):
            out[name] = _rows(t, slice(2 * h0 * hd, 2 * (h0 + nq) * hd))
        elif name.endswith("self_attn.k_proj") or name.endswith("self_attn.v_proj"):
            out[name] = _rows(t, slice(kv0 * hd, (kv0 + nkv) * hd))
        elif name.endswith("self_attn.o_proj"):
            out[name] = _cols(t, h0 * hd, (h0 + nq) * hd, g)
        elif name.endswith("linear_attn.in_proj_qkv"):
            out[name] = _rows(t, qkv)
        elif name.endswith("linear_attn.conv1d.weight"):
            out[name] = t[qkv]
        elif name.endswith("linear_attn.in_proj_z"):
            out[name] = _rows(t, slice(v0 * dv, (v0 + nv) * dv))
        elif name.endswith("linear_attn.in_proj_b") or name.endswith("linear_attn.in_proj_a"):
            out[name] = _rows(t, slice(v0, v0 + nv))
        elif name.endswith("linear_attn.A_log") or name.endswith("linear_attn.dt_bias"):
            out[name] = t[v0: v0 + nv]
        elif name.endswith("linear_attn.out_proj"):
            out[name] = _cols(t, v0 * dv, (v0 + nv) * dv, g)
        elif name.endswith("mlp.gate_proj") or name.endswith("mlp.up_proj"):
            out[name] = _rows(t, slice(i0, i0 + ni))
        elif name.endswith("mlp.down_proj"):
            out[name] = _cols(t, i0, i0 + ni, g)
        else:  # embedding, norms: replicated
            out[name] = t
    return out


def shard_state(state: State, d: Dims, shard: dict) -> State:
    """Rank ``shard``'s recurrent state: conv channels and S of its GDN heads, KV
    cache of its KV heads (a copy; the rank updates it in place)."""
    qkv = qkv_channels(d, shard)
    v0, nv = shard["gdn_v_head0"], shard["gdn_v_heads"]
    kv0, nkv = shard["kv_head0"], shard["kv_heads"]
    return State(
        conv={li: c[:, qkv].copy() for li, c in state.conv.items()},
        S={li: s[v0: v0 + nv].copy() for li, s in state.S.items()},
        k_cache={li: k[:, kv0: kv0 + nkv].copy() for li, k in state.k_cache.items()},
        v_cache={li: v[:, kv0: kv0 + nkv].copy() for li, v in state.v_cache.items()},
    )


def model_step_tp(tokens, pos: int, W_local: dict, state_local: State, d: Dims, shard: dict, all_reduce,
                  all_gather, return_hidden: bool = False):
    """One rank's verify step.  ``all_reduce(x fp32 [M, H]) -> sum over ranks``;
    ``all_gather(x fp32 [M, 2]) -> list of every rank's x, in rank order``."""

    def rowpar(x, w, s, b):
        part = qmm_affine4(x, w, s, b, round_out=False)
        return bf16(all_reduce(np.ascontiguousarray(part, np.float32)))

    def lm_argmax(logits):
        lg = bf16(logits)
        loc = np.argmax(lg, axis=-1)
        val = lg[np.arange(lg.shape[0]), loc]
        mine = np.stack([val, (loc + shard["vocab0"]).astype(np.float32)], axis=-1).astype(np.float32)
        best_v = np.full(lg.shape[0], -np.inf, np.float32)
        best_i = np.zeros(lg.shape[0], np.int64)
        for part in all_gather(mine):
            v, i = part[:, 0], part[:, 1].astype(np.int64)
            take = (v > best_v) | ((v == best_v) & (i < best_i))
            best_v = np.where(take, v, best_v)
            best_i = np.where(take, i, best_i)
        return best_i

    return model_step(tokens, pos, W_local, state_local, local_dims(d, shard), return_hidden, rowpar=rowpar,
                      lm_argmax=lm_argmax)
