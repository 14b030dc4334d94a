"""Speculative-decode rollback on the GPU (iam_rollback): after a K-token
verify, keep only the state after its first n tokens.

* the GDN states and conv windows after verify(K) + rollback(n) match the
  oracle run over the first n tokens (the parity bar of the engine tests), and
  match the GPU's own verify of those n tokens to 1e-5; the next block then
  matches the oracle (argmax, hidden), KV-cache rows of rejected tokens
  included;
* rollback(K) leaves the state bit for bit as the step left it, and repeating
  a rollback gives the same bits (it replays from the state the block read);
* greedy speculative decoding with partly wrong drafts, rolled back after
  every block, emits the oracle's greedy tokens;
* calls out of order are errors.
"""
import dataclasses

import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth_model as SM

from gpu_util import assert_close_bf16, cosine, rel_err, check_argmax_identical

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402

D = O.TINY
SEED = 20261205
MAX_CTX = 64
GDN_LAYERS = [li for li in range(D.n_layers) if not D.is_full_attn(li)]


def cdims(max_rows=8):
    c = I.Dims.qwen35_27b()
    for f in dataclasses.fields(D):
        setattr(c, {"group": "group_size"}.get(f.name, f.name), getattr(D, f.name))
    c.max_ctx, c.max_rows = MAX_CTX, max_rows
    return c


def read_states(e):
    S_shape = (D.gdn_v_heads, D.gdn_dv, D.gdn_dk)
    out = {}
    for li in GDN_LAYERS:
        S = e.read_tensor(f"state.S.{li}", int(np.prod(S_shape)) * 4).view(np.float32).reshape(S_shape).copy()
        conv = e.read_tensor(f"state.conv.{li}", 3 * D.conv_dim * 2).view(np.uint16).reshape(3, D.conv_dim).copy()
        out[li] = (S, conv)
    return out


def check_argmax(got, logits):
    check_argmax_identical(got, logits)


@pytest.fixture(scope="module")
def weights():
    return SM.make_weights(SEED, D)


@pytest.mark.parametrize("n", [1, 3, 5])
def test_rollback_matches_oracle(weights, n):
    K, pos = 6, 10
    tokens = SM.draft_tokens(SEED, D, K, tag="rb")
    nxt = SM.draft_tokens(SEED, D, 4, tag="rb_next")
    e = I.Engine(cdims())
    e.init_synthetic(SEED)

    e.state_init(SEED, pos)
    e.verify(tokens[:n], pos)
    plain = read_states(e)

    e.state_init(SEED, pos)
    e.verify(tokens, pos)
    e.rollback(n)
    got = read_states(e)
    am2, _ = e.verify(nxt, pos + n)
    hid2 = e.read_hidden(len(nxt))
    e.close()

    st = SM.make_state(SEED, D, pos, MAX_CTX)
    O.model_step(np.asarray(tokens[:n]), pos, weights, st, D)
    for li in GDN_LAYERS:
        S, conv = got[li]
        # the state carries the 1-ulp bf16 differences of the projections feeding it
        assert rel_err(S, st.S[li]) < 1e-2 and cosine(S, st.S[li]) > 0.9999, li
        assert_close_bf16(conv, st.conv[li])
        assert rel_err(S, plain[li][0]) < 1e-5, li
        assert_close_bf16(conv, O.from_u16(plain[li][1]))
    _, _, normed, logits = O.model_step(np.asarray(nxt), pos + n, weights, st, D, return_hidden=True)
    assert_close_bf16(hid2, normed)
    check_argmax(am2, logits)


def test_rollback_full_block_and_repeat_are_exact():
    K, pos = 6, 10
    tokens = SM.draft_tokens(SEED, D, K, tag="rb")
    e = I.Engine(cdims())
    e.init_synthetic(SEED)
    e.state_init(SEED, pos)
    e.verify(tokens, pos)
    stepped = read_states(e)
    e.rollback(K)
    again = read_states(e)
    e.rollback(2)
    two = read_states(e)
    e.rollback(2)
    two_again = read_states(e)
    e.close()
    for li in GDN_LAYERS:
        for a, b in ((stepped[li], again[li]), (two[li], two_again[li])):
            assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]), li
        assert not np.array_equal(stepped[li][0], two[li][0])


def test_rollback_errors():
    e = I.Engine(cdims())
    e.init_synthetic(SEED)
    e.state_init(SEED, 4)
    with pytest.raises(I.IamError) as err:
        e.rollback(1)
    assert err.value.status == I.IAM_ESTATE
    e.verify(SM.draft_tokens(SEED, D, 4, tag="rb_err"), 4)
    for bad in (0, 5):
        with pytest.raises(I.IamError) as err:
            e.rollback(bad)
        assert err.value.status == I.IAM_EINVAL
    e.rollback(2)
    with pytest.raises(I.IamError):
        e.rollback(3)  # only rows of the kept prefix remain
    e.state_reset()
    with pytest.raises(I.IamError):
        e.rollback(1)
    e.close()


def oracle_greedy(weights, prompt, n):
    """The oracle's greedy tokens after the prompt and the logits row of each."""
    st = SM.make_state(SEED, D, 0, MAX_CTX)
    for li in st.S:
        st.S[li][:] = 0
        st.conv[li][:] = 0
    am, _, _, logits = O.model_step(np.asarray(prompt), 0, weights, st, D, return_hidden=True)
    toks, rows = [int(am[-1])], [logits[-1]]
    pos = len(prompt)
    while len(toks) < n:
        am, _, _, logits = O.model_step(np.asarray([toks[-1]]), pos, weights, st, D, return_hidden=True)
        toks.append(int(am[0]))
        rows.append(logits[0])
        pos += 1
    return toks, rows


def test_speculative_greedy_equals_greedy(weights):
    """Draft K-1 tokens from the greedy continuation with every fifth one wrong,
    verify, keep accept_len + 1 rows, repeat: the emitted tokens are the greedy
    ones (up to a one-ulp tie of the oracle's top two logits)."""
    K, N = 4, 14
    prompt = SM.draft_tokens(SEED, D, 9, tag="rb_prompt")
    want, rows = oracle_greedy(weights, prompt, N + K)
    e = I.Engine(cdims())
    e.init_synthetic(SEED)
    e.state_reset()
    am, _ = e.verify(prompt[:8], 0)
    am, _ = e.verify(prompt[8:], 8)
    out, pos, accepted = [int(am[-1])], len(prompt), []
    while len(out) < N:
        drafts = [want[i] if i % 5 != 3 else (want[i] + 1) % D.vocab for i in range(len(out), len(out) + K - 1)]
        blk = np.array([out[-1]] + drafts, np.int32)
        am, acc = e.verify(blk, pos)
        e.rollback(acc + 1)
        accepted.append(int(acc))
        out += [int(t) for t in blk[1:acc + 1]] + [int(am[acc])]
        pos += acc + 1
    e.close()
    out = out[:N]
    assert min(accepted) < K - 1 and max(accepted) > 0  # partial and full blocks both occurred
    assert out == list(want[:N]), f"speculative greedy {out} vs oracle {list(want[:N])}"
