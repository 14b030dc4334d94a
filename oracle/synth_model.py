"""Synthetic Qwen3.5-shape model and state, as the oracle sees them.

TEST INFRASTRUCTURE ONLY (see oracle/iam_oracle.py).  The tensor list mirrors
the reference's per-layer tensor names (full_forward.swift:756-820) and the
engine's device-side generator (csrc/engine.cu, kTensorTable); tests check the
two produce the same bits.
"""
from __future__ import annotations

import numpy as np

from . import synth
from .iam_oracle import Dims, State


def layer_specs(d: Dims, li: int):
    """(name, kind, shape, param) for every tensor of layer li."""
    p = f"model.layers.{li}."
    H, I = d.hidden, d.intermediate
    specs = [(p + "input_layernorm.weight", "one_plus_normal_bf16", (H,), 0.02)]
    if d.is_full_attn(li):
        specs += [
            (p + "self_attn.q_proj", "q4", (2 * d.n_heads * d.head_dim, H), None),
            (p + "self_attn.k_proj", "q4", (d.n_kv_heads * d.head_dim, H), None),
            (p + "self_attn.v_proj", "q4", (d.n_kv_heads * d.head_dim, H), None),
            (p + "self_attn.o_proj", "q4", (H, d.n_heads * d.head_dim), None),
            (p + "self_attn.q_norm.weight", "one_plus_normal_bf16", (d.head_dim,), 0.02),
            (p + "self_attn.k_norm.weight", "one_plus_normal_bf16", (d.head_dim,), 0.02),
        ]
    else:
        specs += [
            (p + "linear_attn.in_proj_qkv", "q4", (d.conv_dim, H), None),
            (p + "linear_attn.in_proj_z", "q4", (d.value_dim, H), None),
            (p + "linear_attn.in_proj_b", "q4", (d.gdn_v_heads, H), None),
            (p + "linear_attn.in_proj_a", "q4", (d.gdn_v_heads, H), None),
            (p + "linear_attn.conv1d.weight", "normal_bf16", (d.conv_dim, d.conv_kernel), 0.1),
            (p + "linear_attn.A_log", "uniform_f32", (d.gdn_v_heads,), (-1.0, 1.0)),
            (p + "linear_attn.dt_bias", "normal_bf16", (d.gdn_v_heads,), 0.1),
            (p + "linear_attn.norm.weight", "one_plus_normal_bf16", (d.gdn_dv,), 0.02),
            (p + "linear_attn.out_proj", "q4", (H, d.value_dim), None),
        ]
    specs += [
        (p + "post_attention_layernorm.weight", "one_plus_normal_bf16", (H,), 0.02),
        (p + "mlp.gate_proj", "q4", (I, H), None),
        (p + "mlp.up_proj", "q4", (I, H), None),
        (p + "mlp.down_proj", "q4", (H, I), None),
    ]
    return specs


def global_specs(d: Dims):
    return [
        ("model.embed_tokens.weight", "normal_bf16", (d.vocab, d.hidden), 0.02),
        ("model.norm.weight", "one_plus_normal_bf16", (d.hidden,), 0.02),
        ("lm_head", "q4", (d.vocab, d.hidden), None),
    ]


def make_tensor(seed: int, name: str, kind: str, shape, param, group: int = 64):
    n = int(np.prod(shape))
    if kind == "q4":
        w, s, b = synth.gen_qweight(seed, name, shape[0], shape[1], group)
        return (w, s.astype(np.float32), b.astype(np.float32))
    if kind == "one_plus_normal_bf16":
        return synth.gen_one_plus_normal_bf16(seed, name, n, param).astype(np.float32).reshape(shape)
    if kind == "normal_bf16":
        return synth.gen_normal_bf16(seed, name, n, param).astype(np.float32).reshape(shape)
    if kind == "uniform_f32":
        return synth.gen_uniform_f32(seed, name, n, *param).reshape(shape)
    if kind == "normal_f32":
        return synth.gen_normal_f32(seed, name, n, param).reshape(shape)
    raise ValueError(kind)


def make_layer(seed: int, d: Dims, li: int) -> dict:
    return {name: make_tensor(seed, name, kind, shape, param, d.group)
            for name, kind, shape, param in layer_specs(d, li)}


def make_weights(seed: int, d: Dims, layers=None) -> dict:
    W = {}
    for name, kind, shape, param in global_specs(d):
        W[name] = make_tensor(seed, name, kind, shape, param, d.group)
    for li in (range(d.n_layers) if layers is None else layers):
        W.update(make_layer(seed, d, li))
    return W


def state_name(kind: str, li: int, slot: int = 0) -> str:
    """Synthetic-stream name of a state tensor; sequence slot s > 0 of a
    multi-sequence engine appends ".s<s>" (slot 0 is the single sequence)."""
    return f"state.{kind}.{li}" + (f".s{slot}" if slot else "")


def make_state(seed: int, d: Dims, ctx: int, max_ctx: int, layers=None, slot: int = 0) -> State:
    """Seeded recurrent state and KV cache for a context of ``ctx`` prior tokens:
    conv state N(0,1) bf16 [3, C]; S N(0, 0.01) fp32 [Hv, dv, dk];
    KV cache N(0,1) bf16 in positions [0, ctx) of a [max_ctx, Hkv, d] buffer.
    ``slot`` selects the sequence slot of a multi-sequence engine."""
    conv, S, kc, vc = {}, {}, {}, {}
    for li in (range(d.n_layers) if layers is None else layers):
        if d.is_full_attn(li):
            n = ctx * d.n_kv_heads * d.head_dim
            for store, tag in ((kc, "k_cache"), (vc, "v_cache")):
                buf = np.zeros((max_ctx, d.n_kv_heads, d.head_dim), np.float32)
                if n:
                    buf[:ctx] = synth.gen_normal_bf16(seed, state_name(tag, li, slot), n, 1.0) \
                        .astype(np.float32).reshape(ctx, d.n_kv_heads, d.head_dim)
                store[li] = buf
        else:
            conv[li] = synth.gen_normal_bf16(seed, state_name("conv", li, slot), (d.conv_kernel - 1) * d.conv_dim,
                                             1.0).astype(np.float32).reshape(d.conv_kernel - 1, d.conv_dim)
            S[li] = synth.gen_normal_f32(seed, state_name("S", li, slot), d.gdn_v_heads * d.gdn_dv * d.gdn_dk, 0.01) \
                .reshape(d.gdn_v_heads, d.gdn_dv, d.gdn_dk).copy()
    return State(conv=conv, S=S, k_cache=kc, v_cache=vc)


def draft_tokens(seed: int, d: Dims, k: int, tag: str = "draft") -> np.ndarray:
    return synth.gen_tokens(seed, f"input.{tag}", k, d.vocab)


def hidden_input(seed: int, d: Dims, m: int, tag: str = "x") -> np.ndarray:
    return synth.gen_normal_bf16(seed, f"input.{tag}", m * d.hidden, 1.0).astype(np.float32).reshape(m, d.hidden)
