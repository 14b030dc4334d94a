"""Generate tests/golden/ref_kernels.npz from the reference's own kernels.

Runs the reference's Metal kernels compiled for the host (oracle/_ref/libref_msl.so,
built by oracle/ref_msl/Makefile from the reference's full_forward.swift:55-445)
on seeded inputs and stores inputs and outputs.  The fixtures let tests on
machines without the reference check the oracle and the CUDA kernels against
the reference's arithmetic.

usage: python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import iam_oracle as O  # noqa: E402
from oracle import synth  # noqa: E402
from oracle.ref_msl import refmsl as R  # noqa: E402


def main():
    rng = np.random.default_rng(20261201)
    u = O.to_u16
    G = {}

    x = O.bf16(rng.standard_normal((2, 5120)))
    w = O.bf16(1 + 0.02 * rng.standard_normal(5120))
    G["rms_norm.x"], G["rms_norm.w"], G["rms_norm.out"] = u(x), u(w), R.rms_norm(u(x), u(w))

    g = O.bf16(3 * rng.standard_normal(4096))
    up = O.bf16(rng.standard_normal(4096))
    G["ew.a"], G["ew.b"] = u(g), u(up)
    G["silu_multiply.out"] = R.silu_multiply(u(g), u(up))
    G["residual_add.out"] = R.residual_add(u(g), u(up))
    G["sigmoid_multiply.out"] = R.sigmoid_multiply(u(g), u(up))
    G["silu.out"] = R.silu(u(g))

    wq, s, b = synth.gen_qweight(7, "golden.embed", 16, 5120)
    G["embed.w"], G["embed.s"], G["embed.b"] = wq, s.view(np.uint16), b.view(np.uint16)
    G["embed.tokens"] = np.array([0, 5, 15], np.int32)
    G["embed.out"] = np.stack([R.embed_lookup(wq, s.view(np.uint16), b.view(np.uint16), t)
                               for t in G["embed.tokens"]])

    q = O.bf16(rng.standard_normal((24, 256)))
    G["rope.x"] = u(q)
    G["rope.pos"] = np.array([0, 1, 1023, 4099], np.int32)
    G["rope.out"] = np.stack([R.rope(u(q), *O.rope_tables(int(p)), 64) for p in G["rope.pos"]])

    lg = O.bf16(rng.standard_normal(65536))
    lg[777] = lg[40000] = 8.0  # tie: the first index wins
    G["argmax.x"], G["argmax.out"] = u(lg), np.array([R.argmax(u(lg))], np.int32)

    qw = O.bf16(1 + 0.02 * rng.standard_normal(256))
    G["phnorm.w"], G["phnorm.out"] = u(qw), R.per_head_rms_norm(u(q), u(qw))

    C = 2048
    st = O.bf16(rng.standard_normal((3, C)))
    xx = O.bf16(rng.standard_normal(C))
    cw = O.bf16(0.1 * rng.standard_normal((C, 4)))
    G["conv.state"], G["conv.x"], G["conv.w"] = u(st), u(xx), u(cw)
    G["conv.out"], G["conv.new_state"] = R.depthwise_conv1d(u(st), u(xx), u(cw))

    qk = O.bf16(rng.standard_normal((16, 128)))
    G["snorm.x"] = u(qk)
    G["snorm.q_out"] = R.per_head_rms_norm_scaled(u(qk), 1e-6, float(O.GDN_Q_SCALE))
    G["snorm.k_out"] = R.per_head_rms_norm_scaled(u(qk), 1e-6, float(O.GDN_K_SCALE))

    a = O.bf16(5 * rng.standard_normal(48))
    a[3] = 24.0  # softplus threshold branch
    bb = O.bf16(rng.standard_normal(48))
    A = rng.uniform(-1, 1, 48).astype(np.float32)
    dt = O.bf16(0.1 * rng.standard_normal(48))
    G["gb.a"], G["gb.b"], G["gb.A_log"], G["gb.dt_bias"] = u(a), u(bb), A, u(dt)
    G["gb.g"], G["gb.beta"] = R.compute_g_beta(u(a), u(bb), A, u(dt))

    # a sequence of gated-delta steps on 3 V-heads sharing one K-head
    T, HV = 8, 3
    S = (0.01 * rng.standard_normal((HV, 128, 128))).astype(np.float32)
    G["delta.S0"] = S
    qs, ks, vs, gs, bs, ys = [], [], [], [], [], []
    for t in range(T):
        qh = O.expand_heads(O.per_head_rms_norm_scaled(O.bf16(rng.standard_normal((1, 128))), O.GDN_Q_SCALE), HV)
        kh = O.expand_heads(O.per_head_rms_norm_scaled(O.bf16(rng.standard_normal((1, 128))), O.GDN_K_SCALE), HV)
        vh = O.bf16(rng.standard_normal((HV, 128)))
        gg, be = O.compute_g_beta(O.bf16(rng.standard_normal(HV)), O.bf16(rng.standard_normal(HV)),
                                  rng.uniform(-1, 1, HV).astype(np.float32), O.bf16(0.1 * rng.standard_normal(HV)))
        y, S = R.gated_delta_step(u(qh), u(kh), u(vh), u(gg), u(be), S)
        qs.append(u(qh)); ks.append(u(kh)); vs.append(u(vh)); gs.append(u(gg)); bs.append(u(be)); ys.append(y)
    G["delta.q"], G["delta.k"], G["delta.v"] = np.stack(qs), np.stack(ks), np.stack(vs)
    G["delta.g"], G["delta.beta"], G["delta.y"], G["delta.S"] = np.stack(gs), np.stack(bs), np.stack(ys), S

    y = O.bf16(rng.standard_normal((48, 128)))
    z = O.bf16(rng.standard_normal((48, 128)))
    nw = O.bf16(1 + 0.02 * rng.standard_normal(128))
    G["gnorm.y"], G["gnorm.z"], G["gnorm.w"] = u(y), u(z), u(nw)
    G["gnorm.out"] = R.rms_norm_gated(u(y), u(z), u(nw))

    T = 40
    kc = O.bf16(rng.standard_normal((T, 4, 256)))
    vc = O.bf16(rng.standard_normal((T, 4, 256)))
    qa = O.bf16(rng.standard_normal((24, 256)) / 16)
    G["sdpa.q"], G["sdpa.k"], G["sdpa.v"] = u(qa), u(kc), u(vc)
    G["sdpa.seq"] = np.array([1, 7, 40], np.int32)
    G["sdpa.out"] = np.stack([R.sdpa_decode(u(qa), u(kc), u(vc), int(n)) for n in G["sdpa.seq"]])

    qg = O.bf16(rng.standard_normal(24 * 512))
    G["split.qg"] = u(qg)
    G["split.q"], G["split.gate"] = R.split_q_gate(u(qg), 24, 256)

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_kernels.npz")
    np.savez_compressed(path, **G)
    print(f"wrote {path}: {os.path.getsize(path) / 1024:.0f} KiB, {len(G)} arrays")


if __name__ == "__main__":
    main()
