"""Engine-level parity on the GPU (the K-token verify entry point).

* device-generated synthetic weights and state == the oracle's, bit for bit;
* one full-size GDN layer (27B dims) and one full-size attention + MLP layer
  against the oracle's layer restatement at K = 1 and K > 1;
* a small model of the same family, K-token verify vs the oracle's model step;
* K-token verify == K sequential decode steps on the GPU;
* the GDN recurrence's fp32 state after 256 steps within 1e-4 relative.
Hidden states within 1e-2 relative / cosine >= 0.9999; argmax identical to the
oracle's on every row (the top-1 minus top-2 margins are printed, and a row
within one bf16 ulp of a tie is named in the failure message).
"""
import dataclasses

import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth_model as SM

from gpu_util import assert_close_bf16, check_argmax_identical, cosine, dev, empty_u16, host_u16, ptr, rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402

SEED = 20261201


def cdims(d: O.Dims, max_ctx: int, max_rows: int) -> I.Dims:
    c = I.Dims.qwen35_27b()
    for f in dataclasses.fields(d):
        name = {"group": "group_size"}.get(f.name, f.name)
        setattr(c, name, getattr(d, f.name))
    c.max_ctx = max_ctx
    c.max_rows = max_rows
    return c


def check_argmax(got, logits_ref):
    check_argmax_identical(got, logits_ref)


def run_engine(d: O.Dims, tokens, pos, ctx, max_ctx=None, max_rows=32):
    e = I.Engine(cdims(d, max(max_ctx or (pos + len(tokens) + 8), max_rows), max_rows))
    e.init_synthetic(SEED)
    e.state_init(SEED, ctx)
    am, acc = e.verify(tokens, pos)
    hid = e.read_hidden(len(tokens))
    return e, am, acc, hid


def oracle_step(d: O.Dims, tokens, pos, ctx, max_ctx):
    W = SM.make_weights(SEED, d)
    st = SM.make_state(SEED, d, ctx, max_ctx)
    am, acc, normed, logits = O.model_step(np.asarray(tokens), pos, W, st, d, return_hidden=True)
    return W, st, am, acc, normed, logits


# ---------------------------------------------------------------- generator
def test_synthetic_weights_bit_exact():
    d = O.TINY
    e = I.Engine(cdims(d, 64, 8))
    e.init_synthetic(SEED)
    for li in (0, 3):
        for name, kind, shape, param in SM.layer_specs(d, li):
            ref = SM.make_tensor(SEED, name, kind, shape, param)
            if kind == "q4":
                w, s, b = ref
                got_w = e.read_tensor(name + ".weight", w.nbytes).view(np.uint32).reshape(w.shape)
                got_s = e.read_tensor(name + ".scales", s.size * 2).view(np.uint16)
                got_b = e.read_tensor(name + ".biases", b.size * 2).view(np.uint16)
                assert np.array_equal(got_w, w), name
                assert np.array_equal(got_s, O.to_u16(s).ravel()), name
                assert np.array_equal(got_b, O.to_u16(b).ravel()), name
            elif kind == "uniform_f32":
                got = e.read_tensor(name, ref.size * 4).view(np.float32)
                assert np.array_equal(got, ref.ravel()), name
            else:
                got = e.read_tensor(name, ref.size * 2).view(np.uint16)
                assert np.array_equal(got, O.to_u16(ref).ravel()), name
    e.close()


def test_seeded_state_bit_exact():
    d = O.TINY
    e = I.Engine(cdims(d, 64, 8))
    e.init_synthetic(SEED)
    e.state_init(SEED, 20)
    st = SM.make_state(SEED, d, 20, 64)
    S0 = e.read_tensor("state.S.0", st.S[0].nbytes).view(np.float32).reshape(st.S[0].shape)
    assert np.array_equal(S0, st.S[0])
    c0 = e.read_tensor("state.conv.0", st.conv[0].size * 2).view(np.uint16).reshape(st.conv[0].shape)
    assert np.array_equal(c0, O.to_u16(st.conv[0]))
    k3 = e.read_tensor("state.k_cache.3", st.k_cache[3].size * 2).view(np.uint16).reshape(st.k_cache[3].shape)
    assert np.array_equal(k3, O.to_u16(st.k_cache[3]))
    e.close()


# ---------------------------------------------------------------- one full-size layer
GDN1 = O.Dims(n_layers=1, vocab=4096)
ATTN1 = O.Dims(n_layers=1, full_attn_interval=1, vocab=4096)


@pytest.mark.parametrize("K", [1, 8, 32])
def test_one_gdn_layer_27b(K):
    tokens = SM.draft_tokens(SEED, GDN1, K)
    e, am, acc, hid = run_engine(GDN1, tokens, 0, 0)
    W, st, am_ref, acc_ref, normed, logits = oracle_step(GDN1, tokens, 0, 0, 16 + K)
    assert_close_bf16(hid, normed)
    check_argmax(am, logits)
    S = e.read_tensor("state.S.0", st.S[0].nbytes).view(np.float32).reshape(st.S[0].shape)
    # the state carries the 1-ulp bf16 differences of the projections feeding it;
    # the recurrence alone is held to 1e-4 by test_gdn_state_256_steps
    assert rel_err(S, st.S[0]) < 1e-2 and cosine(S, st.S[0]) > 0.9999
    e.close()


@pytest.mark.parametrize("K,pos", [(1, 1023), (4, 1023), (32, 1023)])
def test_one_attention_layer_27b(K, pos):
    tokens = SM.draft_tokens(SEED, ATTN1, K)
    max_ctx = pos + K + 8
    e, am, acc, hid = run_engine(ATTN1, tokens, pos, pos, max_ctx)
    W, st, am_ref, acc_ref, normed, logits = oracle_step(ATTN1, tokens, pos, pos, max_ctx)
    assert_close_bf16(hid, normed)
    check_argmax(am, logits)
    kc = e.read_tensor("state.k_cache.0", max_ctx * 4 * 256 * 2).view(np.uint16).reshape(max_ctx, 4, 256)
    # appended k is normed + roped; it inherits the k projection's bf16 ulps
    assert_close_bf16(kc[pos:pos + K], st.k_cache[0][pos:pos + K])
    assert np.array_equal(kc[:pos], O.to_u16(st.k_cache[0][:pos]))
    e.close()


# ---------------------------------------------------------------- small model, whole step
@pytest.mark.parametrize("K", [1, 5, 16])
def test_tiny_model_verify(K):
    d = O.TINY
    tokens = SM.draft_tokens(SEED, d, K, tag=f"tiny{K}")
    pos = 20
    e, am, acc, hid = run_engine(d, tokens, pos, pos, 64)
    W, st, am_ref, acc_ref, normed, logits = oracle_step(d, tokens, pos, pos, 64)
    assert_close_bf16(hid, normed)
    check_argmax(am, logits)
    if np.array_equal(am, am_ref):
        assert acc == acc_ref
    e.close()


@pytest.mark.parametrize("K", [1, 5, 48])
def test_device_resident_step_on_fresh_weights(K):
    """iam_verify_device straight after the weights were generated (no host
    step before it): the step packs the weights first, so its argmax, accept
    length and hidden state equal the host-driven step's, bit for bit."""
    d = O.TINY
    tokens = SM.draft_tokens(SEED, d, K, tag=f"dev{K}")
    pos = 20
    got = []
    for how in ("device", "host"):
        e = I.Engine(cdims(d, 96, 64))
        e.init_synthetic(SEED)
        e.state_init(SEED, pos)
        if how == "device":
            dt = torch.tensor(np.asarray(tokens, np.int32), device="cuda")
            out = torch.zeros(K, dtype=torch.int32, device="cuda")
            e.verify_device(dt.data_ptr(), K, pos, out.data_ptr())
            e.status()
            am = out.cpu().numpy().tolist()
        else:
            am, _ = e.verify(tokens, pos)
            am = list(am)
        got.append((am, e.read_hidden(K).copy()))
        e.close()
    assert got[0][0] == got[1][0]
    assert np.array_equal(got[0][1], got[1][1])
    W, st, am_ref, acc_ref, normed, logits = oracle_step(d, tokens, pos, pos, 96)
    check_argmax(got[0][0], logits)


@pytest.mark.parametrize("K", [1, 2])
def test_fused_rmsnorm_bit_identical(K, monkeypatch):
    """Steps of at most two rows fuse the RMSNorm ahead of each matmul into
    the matmul (its CTAs normalise the rows they read); the outputs must be
    bit-identical to the separate norm kernel's (IAM_FUSED_NORM=0)."""
    d = O.TINY
    tokens = SM.draft_tokens(SEED, d, K, tag=f"fn{K}")
    got = []
    for fused in ("1", "0"):
        monkeypatch.setenv("IAM_FUSED_NORM", fused)
        e = I.Engine(cdims(d, 64, 8))
        e.init_synthetic(SEED)
        e.state_init(SEED, 20)
        am, acc = e.verify(tokens, 20)
        am2, _ = e.verify(tokens[:1], 20 + K)
        got.append((list(am), acc, e.read_hidden(1).copy(), list(am2)))
        prof = e.profile_step(K, 20 + K + 1)
        assert ("rmsnorm" in prof and prof["rmsnorm"]["launches"] == (1 if fused == "1" else 2 * d.n_layers + 1)), prof
        e.close()
    assert got[0][0] == got[1][0] and got[0][1] == got[1][1] and got[0][3] == got[1][3]
    assert np.array_equal(got[0][2], got[1][2])


def test_tiny_model_verify_wide_block():
    """K = 48: every matmul of the step (fused projections, SwiGLU, residual,
    lm_head argmax) on the tensor-core kernel's 64-token tile."""
    d = O.TINY
    K, pos = 48, 20
    tokens = SM.draft_tokens(SEED, d, K, tag="tiny_wide")
    e, am, acc, hid = run_engine(d, tokens, pos, pos, 96, max_rows=64)
    W, st, am_ref, acc_ref, normed, logits = oracle_step(d, tokens, pos, pos, 96)
    assert_close_bf16(hid, normed)
    check_argmax(am, logits)
    e.close()


def test_accept_length_counts_matching_drafts():
    d = O.TINY
    e = I.Engine(cdims(d, 64, 8))
    e.init_synthetic(SEED)
    e.state_init(SEED, 10)
    t0 = np.array([7], np.int32)
    am1, _ = e.verify(t0, 10)  # greedy next token
    e.state_init(SEED, 10)
    toks = np.array([7, am1[0], 3, 3], np.int32)
    am, acc = e.verify(toks, 10)
    assert am[0] == am1[0]
    assert acc >= 1
    e.close()


def test_verify_equals_sequential_decode():
    d = O.TINY
    K, pos = 6, 12
    tokens = SM.draft_tokens(SEED, d, K, tag="seq")
    e = I.Engine(cdims(d, 64, 8))
    e.init_synthetic(SEED)
    e.state_init(SEED, pos)
    am_block, _ = e.verify(tokens, pos)
    S_block = e.read_tensor("state.S.0", 6 * 128 * 128 * 4).view(np.float32).copy()
    e.state_init(SEED, pos)
    am_seq = []
    for i in range(K):
        a, _ = e.verify(tokens[i:i + 1], pos + i)
        am_seq.append(int(a[0]))
    S_seq = e.read_tensor("state.S.0", 6 * 128 * 128 * 4).view(np.float32)
    assert list(am_block) == am_seq
    assert rel_err(S_block, S_seq) < 1e-5
    e.close()


# ---------------------------------------------------------------- recurrence drift
@pytest.mark.parametrize("split", [None, "1", "2", "4", "8"])
def test_gdn_state_256_steps(split, monkeypatch):
    """The fused GDN kernel over 256 tokens (8 verify blocks of 32) against the
    oracle's per-token chain: fp32 state within 1e-4 relative, outputs to the
    parity bar, the conv window bit for bit; with the heads' state rows split
    over 1, 2, 4 or 8 CTAs of a cluster (None: the library's choice)."""
    if split is not None:
        monkeypatch.setenv("IAM_GDN_SPLIT", split)
    d = O.QWEN35_27B
    rng = np.random.default_rng(256)
    C, HV, HK, VD = d.conv_dim, d.gdn_v_heads, d.gdn_k_heads, d.value_dim
    ld = C + VD + 2 * HV
    steps = 256
    inp = O.bf16(rng.standard_normal((steps, ld)) * 0.5)
    conv_w = O.bf16(0.1 * rng.standard_normal((C, 4)))
    A_log = rng.uniform(-1, 1, HV).astype(np.float32)
    dt_bias = O.bf16(0.1 * rng.standard_normal(HV))
    norm_w = O.bf16(1 + 0.02 * rng.standard_normal(128))
    conv0 = O.bf16(rng.standard_normal((3, C)))
    S0 = (0.01 * rng.standard_normal((HV, 128, 128))).astype(np.float32)
    # oracle
    conv = conv0.copy()
    S = S0.copy()
    outs = []
    for t in range(steps):
        co, conv = O.depthwise_conv1d_step(conv, inp[t, :C], conv_w)
        cs = O.silu(co)
        q = O.expand_heads(O.per_head_rms_norm_scaled(cs[:2048].reshape(HK, 128), O.GDN_Q_SCALE), HV)
        k = O.expand_heads(O.per_head_rms_norm_scaled(cs[2048:4096].reshape(HK, 128), O.GDN_K_SCALE), HV)
        v = cs[4096:].reshape(HV, 128)
        g, beta = O.compute_g_beta(inp[t, C + VD + HV:], inp[t, C + VD:C + VD + HV], A_log, dt_bias)
        y = O.gated_delta_step(q, k, v, g, beta, S)
        outs.append(O.rms_norm_gated(y, inp[t, C:C + VD].reshape(HV, 128), norm_w).reshape(-1))
    # GPU, 8 verify blocks of 32 tokens
    dS = dev(S0.copy(), torch)
    ca, cb = dev(O.to_u16(conv0), torch), empty_u16(torch, 3, C)
    out = empty_u16(torch, steps, VD)
    di = dev(O.to_u16(inp), torch)
    dcw, dal, ddt, dnw = (dev(O.to_u16(conv_w), torch), dev(A_log, torch), dev(O.to_u16(dt_bias), torch),
                          dev(O.to_u16(norm_w), torch))
    for blk in range(8):
        src, dst = (ca, cb) if blk % 2 == 0 else (cb, ca)
        I.gdn_step_fused(ptr(di) + blk * 32 * ld * 2, ld, C, C + VD + HV, C + VD, ptr(dcw), ptr(src), ptr(dst),
                         ptr(dal), ptr(ddt), ptr(dnw), ptr(dS), ptr(out) + blk * 32 * VD * 2, VD, HK, HV, 32)
    torch.cuda.synchronize()
    Sg = dS.cpu().numpy()
    assert rel_err(Sg, S) < 1e-4, rel_err(Sg, S)
    go = O.from_u16(host_u16(out))
    assert cosine(go, np.stack(outs)) > 0.9999
    # the last block (7, odd) read cb and wrote the new window into ca
    assert np.array_equal(host_u16(ca), O.to_u16(conv))
