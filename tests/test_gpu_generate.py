"""Greedy generation through the C ABI (iam_generate) against the oracle:
reset state, a prompt longer than one verify block (prefilled in blocks),
then one token at a time; the stop ids end generation after they are
emitted.  Tokens must match the oracle's greedy sequence; the two may part
only where the oracle's top two logits are within one bf16 ulp."""
import dataclasses

import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth_model as SM

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402

D = O.TINY
SEED = 20261204
MAX_CTX = 40


def cdims():
    c = I.Dims.qwen35_27b()
    for f in dataclasses.fields(D):
        setattr(c, {"group": "group_size"}.get(f.name, f.name), getattr(D, f.name))
    c.max_ctx, c.max_rows = MAX_CTX, 8
    return c


def zero_state():
    conv, S, kc, vc = {}, {}, {}, {}
    for li in range(D.n_layers):
        if D.is_full_attn(li):
            kc[li] = np.zeros((MAX_CTX, D.n_kv_heads, D.head_dim), np.float32)
            vc[li] = np.zeros((MAX_CTX, D.n_kv_heads, D.head_dim), np.float32)
        else:
            conv[li] = np.zeros((D.conv_kernel - 1, D.conv_dim), np.float32)
            S[li] = np.zeros((D.gdn_v_heads, D.gdn_dv, D.gdn_dk), np.float32)
    return O.State(conv=conv, S=S, k_cache=kc, v_cache=vc)


def oracle_generate(W, prompt, max_new):
    """The oracle's greedy tokens and, per token, the logits row it came from."""
    st = zero_state()
    am, _, _, logits = O.model_step(np.asarray(prompt), 0, W, st, D, return_hidden=True)
    toks, rows = [int(am[-1])], [logits[-1]]
    pos = len(prompt)
    while len(toks) < max_new:
        am, _, _, logits = O.model_step(np.asarray([toks[-1]]), pos, W, st, D, return_hidden=True)
        toks.append(int(am[0]))
        rows.append(logits[0])
        pos += 1
    return toks, rows


def assert_same_until_tie(got, want, rows):
    """The greedy sequences are identical token for token (each step's top-1
    minus top-2 margin is printed)."""
    marg = [float(np.partition(np.asarray(r, np.float32), -2)[-1] - np.partition(np.asarray(r, np.float32), -2)[-2])
            for r in rows]
    print(f"greedy margins: min {min(marg):.4g}")
    assert list(got) == list(want), f"generated {list(got)} vs oracle {list(want)}"


def test_generate_matches_oracle():
    prompt = SM.draft_tokens(SEED, D, 11, tag="prompt")  # two prefill blocks of max_rows = 8
    e = I.Engine(cdims())
    e.init_synthetic(SEED)
    got = [int(t) for t in e.generate(prompt, 6, eos=())]
    W = SM.make_weights(SEED, D)
    want, rows = oracle_generate(W, prompt, 6)
    assert_same_until_tie(got, want, rows)

    # a stop id ends generation right after it is emitted
    stop = got[2]
    cut = got[:got.index(stop) + 1]
    assert [int(t) for t in e.generate(prompt, 6, eos=(stop, 248046))] == cut
    # generation starts from a reset state each time
    assert [int(t) for t in e.generate(prompt, 6, eos=())] == got
    with pytest.raises(I.IamError):
        e.generate(prompt, MAX_CTX, eos=())
    e.close()
