"""Multi-sequence batch verify on the GPU (iam_verify_batch): n_seq sequences,
each in its own slot (GDN state, conv window, KV cache, position), verify K
tokens each in one step.

* every sequence's argmax, accept length, final hidden and state match the
  oracle run on that sequence alone (parity bar of the engine tests), with
  the shapes that take each kernel variant: GDN state rows split over a
  cluster or one CTA a head, attention on the warp or the tensor-core decode;
* slots past n_seq are left bit for bit as they were;
* two batch steps in a row continue each sequence;
* a one-sequence batch equals the single-sequence verify;
* bad shapes are errors, and rollback does not apply after a batch step.
"""
import dataclasses

import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth_model as SM

from gpu_util import assert_close_bf16, check_argmax_identical, cosine, rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402

D = O.TINY
SEED = 20261206
MAX_CTX = 96
CTX = 10
GDN_LAYERS = [li for li in range(D.n_layers) if not D.is_full_attn(li)]
ATTN_LAYERS = [li for li in range(D.n_layers) if D.is_full_attn(li)]


def cdims(max_seqs, max_rows):
    c = I.Dims.qwen35_27b()
    for f in dataclasses.fields(D):
        setattr(c, {"group": "group_size"}.get(f.name, f.name), getattr(D, f.name))
    c.max_ctx, c.max_rows, c.max_seqs = MAX_CTX, max_rows, max_seqs
    return c


@pytest.fixture(scope="module")
def weights():
    return SM.make_weights(SEED, D)


def engine(max_seqs, max_rows):
    e = I.Engine(cdims(max_seqs, max_rows))
    e.init_synthetic(SEED)
    e.state_init(SEED, CTX)
    return e


def read_slots(e, max_seqs):
    out = {}
    S_shape = (D.gdn_v_heads, D.gdn_dv, D.gdn_dk)
    nS = int(np.prod(S_shape))
    for li in GDN_LAYERS:
        S = e.read_tensor(f"state.S.{li}", max_seqs * nS * 4).view(np.float32).reshape((max_seqs,) + S_shape).copy()
        c = e.read_tensor(f"state.conv.{li}", max_seqs * 3 * D.conv_dim * 2).view(np.uint16) \
            .reshape(max_seqs, 3, D.conv_dim).copy()
        out[li] = (S, c)
    for li in ATTN_LAYERS:
        n = MAX_CTX * D.n_kv_heads * D.head_dim
        k = e.read_tensor(f"state.k_cache.{li}", max_seqs * n * 2).view(np.uint16) \
            .reshape(max_seqs, MAX_CTX, D.n_kv_heads, D.head_dim).copy()
        out[li] = (k,)
    return out


def check_rows(am, logits):
    check_argmax_identical(am, logits)


def oracle_seq(weights, q, tokens, pos, state=None):
    st = state if state is not None else SM.make_state(SEED, D, CTX, MAX_CTX, slot=q)
    am, acc, normed, logits = O.model_step(np.asarray(tokens), pos, weights, st, D, return_hidden=True)
    return st, am, acc, normed, logits


# (n_seq, K): GDN cluster split 8 + warp decode; one CTA a head (K < 4) + warp
# decode; tensor-core decode (K x 2 query heads per KV head >= 32 pairs)
@pytest.mark.parametrize("n_seq,K", [(3, 5), (8, 2), (2, 16)])
def test_batch_matches_oracle_per_sequence(weights, n_seq, K):
    max_seqs = n_seq + 1  # one slot left out of the step
    e = engine(max_seqs, n_seq * K)
    before = read_slots(e, max_seqs)
    tokens = np.stack([SM.draft_tokens(SEED, D, K, tag=f"batch{q}") for q in range(n_seq)])
    pos = np.array([CTX + 3 * q for q in range(n_seq)], np.int32)
    am, acc = e.verify_batch(tokens, pos)
    hid = e.read_hidden(n_seq * K).reshape(n_seq, K, D.hidden)
    after = read_slots(e, max_seqs)
    e.close()
    for q in range(n_seq):
        st, am_r, acc_r, normed, logits = oracle_seq(weights, q, tokens[q], int(pos[q]))
        assert_close_bf16(hid[q], normed)
        check_rows(am[q], logits)
        assert acc[q] == acc_r
        for li in GDN_LAYERS:
            S, c = after[li][0][q], after[li][1][q]
            assert rel_err(S, st.S[li]) < 1e-2 and cosine(S, st.S[li]) > 0.9999, (q, li)
            assert_close_bf16(c, st.conv[li])
        for li in ATTN_LAYERS:
            kc = after[li][0][q]
            p = int(pos[q])
            assert_close_bf16(kc[p:p + K], st.k_cache[li][p:p + K])
            assert np.array_equal(kc[:p], O.to_u16(st.k_cache[li][:p]))
    last = max_seqs - 1
    for li in GDN_LAYERS + ATTN_LAYERS:
        for a, b in zip(before[li], after[li]):
            assert np.array_equal(a[last], b[last]), li


def test_two_batch_steps_continue_each_sequence(weights):
    n_seq, K = 3, 4
    e = engine(n_seq, n_seq * K)
    t1 = np.stack([SM.draft_tokens(SEED, D, K, tag=f"b1_{q}") for q in range(n_seq)])
    t2 = np.stack([SM.draft_tokens(SEED, D, K, tag=f"b2_{q}") for q in range(n_seq)])
    pos = np.array([CTX, CTX + 1, CTX + 5], np.int32)
    e.verify_batch(t1, pos)
    am, acc = e.verify_batch(t2, pos + K)
    hid = e.read_hidden(n_seq * K).reshape(n_seq, K, D.hidden)
    e.close()
    for q in range(n_seq):
        st, *_ = oracle_seq(weights, q, t1[q], int(pos[q]))
        _, am_r, acc_r, normed, logits = oracle_seq(weights, q, t2[q], int(pos[q]) + K, state=st)
        assert_close_bf16(hid[q], normed)
        check_rows(am[q], logits)


def test_one_sequence_batch_equals_single_verify():
    K = 6
    tokens = SM.draft_tokens(SEED, D, K, tag="single")
    e = engine(2, 8)
    am1, acc1 = e.verify(tokens, CTX)
    h1 = e.read_hidden(K)
    s1 = read_slots(e, 2)
    e.state_init(SEED, CTX)
    am2, acc2 = e.verify_batch(tokens[None, :], np.array([CTX], np.int32))
    h2 = e.read_hidden(K)
    s2 = read_slots(e, 2)
    e.close()
    assert np.array_equal(am1, am2[0]) and acc1 == acc2[0]
    assert_close_bf16(h2, O.from_u16(h1))
    for li in GDN_LAYERS:
        assert rel_err(s2[li][0][0], s1[li][0][0]) < 1e-5


def test_batch_errors():
    e = engine(2, 8)
    tok = np.zeros((3, 2), np.int32)
    for t, p in ((tok, np.array([CTX] * 3, np.int32)),                          # n_seq > max_seqs
                 (np.zeros((2, 5), np.int32), np.array([CTX, CTX], np.int32)),  # 10 rows > max_rows
                 (np.zeros((2, 2), np.int32), np.array([CTX, MAX_CTX - 1], np.int32))):  # past max_ctx
        with pytest.raises(I.IamError) as err:
            e.verify_batch(t, p)
        assert err.value.status == I.IAM_EINVAL
    e.verify_batch(np.zeros((2, 2), np.int32), np.array([CTX, CTX], np.int32))
    with pytest.raises(I.IamError) as err:
        e.rollback(1)
    assert err.value.status == I.IAM_ESTATE
    e.close()
