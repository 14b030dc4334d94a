"""The oracle restatement against the reference's own kernels.

Golden vectors in tests/golden/ref_kernels.npz come from the reference's Metal
kernels compiled for the host (tests/golden/make_golden.py).  Element-wise
kernels must agree bit for bit; kernels whose fp32 sums the oracle orders
differently (delta step, SDPA) may differ by one bf16 ulp on a few elements.
"""
import numpy as np

from oracle import iam_oracle as O

f = O.from_u16
u = O.to_u16


def exact(a, b):
    assert a.shape == b.shape
    assert np.array_equal(np.asarray(a), np.asarray(b)), f"{np.sum(np.asarray(a) != np.asarray(b))} mismatches"


def near_ulp(a_u16, b_u16, max_frac=0.01):
    a, b = f(a_u16), f(b_u16)
    diff = np.abs(a - b)
    ulp = np.abs(b) * 2.0 ** -7 + 1e-30
    assert np.all(diff <= ulp + 1e-8), diff.max()
    assert np.mean(a_u16 != b_u16) <= max_frac


def test_rms_norm(golden):
    exact(u(O.rms_norm(f(golden["rms_norm.x"]), f(golden["rms_norm.w"]))), golden["rms_norm.out"])


def test_elementwise(golden):
    a, b = f(golden["ew.a"]), f(golden["ew.b"])
    exact(u(O.silu_multiply(a, b)), golden["silu_multiply.out"])
    exact(u(O.residual_add(a, b)), golden["residual_add.out"])
    exact(u(O.sigmoid_multiply(a, b)), golden["sigmoid_multiply.out"])
    exact(u(O.silu(a)), golden["silu.out"])


def test_embed_lookup_pins_dequant(golden):
    s = f(golden["embed.s"]); b = f(golden["embed.b"])
    for i, t in enumerate(golden["embed.tokens"]):
        exact(u(O.embed_lookup_4bit(golden["embed.w"], s, b, int(t))), golden["embed.out"][i])
    # the qmm dequant is the same formula: row t of dequant() == embed lookup of t
    W = O.dequant(golden["embed.w"], s, b)
    exact(u(W[golden["embed.tokens"]]), golden["embed.out"])


def test_rope(golden):
    x = f(golden["rope.x"])
    for i, p in enumerate(golden["rope.pos"]):
        exact(u(O.rope(x, int(p))), golden["rope.out"][i])
    # position 0 is the identity (attn_forward.swift:488)
    exact(u(O.rope(x, 0)), golden["rope.x"])


def test_argmax_first_index(golden):
    assert int(O.argmax_first(f(golden["argmax.x"]))) == int(golden["argmax.out"][0]) == 777


def test_per_head_norms(golden):
    exact(u(O.per_head_rms_norm(f(golden["rope.x"]), f(golden["phnorm.w"]))), golden["phnorm.out"])
    x = f(golden["snorm.x"])
    exact(u(O.per_head_rms_norm_scaled(x, O.GDN_Q_SCALE)), golden["snorm.q_out"])
    exact(u(O.per_head_rms_norm_scaled(x, O.GDN_K_SCALE)), golden["snorm.k_out"])


def test_conv1d(golden):
    out, ns = O.depthwise_conv1d_step(f(golden["conv.state"]), f(golden["conv.x"]), f(golden["conv.w"]))
    exact(u(out), golden["conv.out"])
    exact(u(ns), golden["conv.new_state"])


def test_g_beta(golden):
    g, b = O.compute_g_beta(f(golden["gb.a"]), f(golden["gb.b"]), golden["gb.A_log"], f(golden["gb.dt_bias"]))
    exact(u(g), golden["gb.g"])
    exact(u(b), golden["gb.beta"])


def test_gated_delta_sequence(golden):
    S = golden["delta.S0"].copy()
    for t in range(golden["delta.q"].shape[0]):
        y = O.gated_delta_step(f(golden["delta.q"][t]), f(golden["delta.k"][t]), f(golden["delta.v"][t]),
                               f(golden["delta.g"][t]), f(golden["delta.beta"][t]), S)
        near_ulp(u(y), golden["delta.y"][t])
    ref = golden["delta.S"]
    assert np.max(np.abs(S - ref)) / np.max(np.abs(ref)) < 1e-5


def test_gated_norm(golden):
    exact(u(O.rms_norm_gated(f(golden["gnorm.y"]), f(golden["gnorm.z"]), f(golden["gnorm.w"]))),
          golden["gnorm.out"])


def test_sdpa(golden):
    for i, n in enumerate(golden["sdpa.seq"]):
        out = O.sdpa_decode(f(golden["sdpa.q"]), f(golden["sdpa.k"]), f(golden["sdpa.v"]), int(n))
        near_ulp(u(out), golden["sdpa.out"][i])
    # one cached token: the output is that token's V (attn_forward.swift:638-648)
    out1 = O.sdpa_decode(f(golden["sdpa.q"]), f(golden["sdpa.k"]), f(golden["sdpa.v"]), 1)
    v0 = f(golden["sdpa.v"])[0]
    assert np.array_equal(out1, np.repeat(v0, 6, axis=0))


def test_split_q_gate(golden):
    qg = golden["split.qg"].reshape(24, 512)
    exact(qg[:, :256], golden["split.q"])
    exact(qg[:, 256:], golden["split.gate"])
