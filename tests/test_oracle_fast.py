"""The oracle's C helpers (oracle/fast) against their numpy statements: the
same bits for the synthetic generator, the dequant and a streamed model step."""
import numpy as np

from oracle import fast as F
from oracle import iam_oracle as O
from oracle import synth
from oracle import synth_model as SM

SEED = 20261201


def test_words_and_normals_match_numpy():
    for name in ("a", "model.layers.3.mlp.gate_proj.weight", "lm_head.scales"):
        assert np.array_equal(F.words(SEED, name, 4099), synth.gen_words(SEED, name, 4099))
        ref = synth.gen_normal_bf16(SEED, name, 5000, 0.02).view(np.uint16)
        assert np.array_equal(F.normal_bf16_u16(SEED, name, 5000, 0.02), ref)
        ref = synth.gen_absnormal_bf16(SEED, name, 5000, 0.02).view(np.uint16)
        assert np.array_equal(F.absnormal_bf16_u16(SEED, name, 5000, 0.02), ref)
    # an offset window of the stream (embedding rows)
    full = synth.gen_normal_bf16(SEED, "e", 3 * 256, 0.02).view(np.uint16)
    assert np.array_equal(F.normal_bf16_u16(SEED, "e", 256, 0.02, start=512), full[512:])


def test_qweight_matches_numpy():
    w, s, b = synth.gen_qweight(SEED, "m.q", 96, 512)
    q = F.gen_qweight(SEED, "m.q", 96, 512)
    assert np.array_equal(q[0], w)
    assert np.array_equal(q.s_u16, s.view(np.uint16))
    assert np.array_equal(q.b_u16, b.view(np.uint16))


def test_dequant_matches_numpy():
    rng = np.random.default_rng(1)
    w = rng.integers(0, 2**32, (64, 40), dtype=np.uint64).astype(np.uint32)
    s = O.bf16(np.abs(rng.standard_normal((64, 5))) * 0.3)  # scales above and below 0.25
    b = O.bf16(-8 * s + rng.standard_normal((64, 5)) * 0.01)
    assert np.array_equal(F.dequant(w, s, b).view(np.uint32), O.dequant(w, s, b).view(np.uint32))


def test_streamed_step_matches_model_step():
    d = O.TINY
    toks = SM.draft_tokens(SEED, d, 3, tag="fast")
    W = SM.make_weights(SEED, d)
    st = SM.make_state(SEED, d, 9, 16)
    am, acc, normed, logits = O.model_step(toks, 9, W, st, d, return_hidden=True)
    am2, acc2, normed2, logits2 = F.model_step_streaming(toks, 9, SEED, d, 9, 16, return_hidden=True)
    assert np.array_equal(am, am2) and acc == acc2
    assert np.array_equal(normed.view(np.uint32), normed2.view(np.uint32))
    assert np.array_equal(logits.view(np.uint32), logits2.view(np.uint32))


def test_make_weights_matches_numpy():
    d = O.TINY
    W = SM.make_weights(SEED, d)
    W2 = F.make_weights(SEED, d)
    assert W.keys() == W2.keys()
    for k, v in W.items():
        if isinstance(v, tuple):
            for a, b in zip(v, W2[k]):
                assert np.array_equal(a, b), k
        else:
            assert np.array_equal(v, W2[k]), k
