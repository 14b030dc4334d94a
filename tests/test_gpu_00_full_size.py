"""Full-size parity of the benchmarked configurations (collected before the
other GPU tests, so a stopped run has checked these first).

* the 64-layer Qwen3.5-27B-shape step (48 GDN + 16 attention layers, vocab
  248320, bf16 embedding, 4-bit lm_head, seeded state and a KV cache of 1024
  prior tokens): K = 32 verify and K = 1 decode against the oracle's streamed
  model step -- per-position argmax identical, accept length identical, final
  normed hidden within 1e-2 relative / cosine 0.9999;
* the 248320-row lm_head with its argmax epilogue behind one full-size GDN
  layer, at K = 1 and K = 32;
* 64 sequences x K = 8 in one multi-sequence verify step (512 token rows:
  eight 64-row matmul passes) at context 1024 on a 4-layer full-width model,
  every sequence against the oracle run on that sequence alone.
"""
import dataclasses

import numpy as np
import pytest

from oracle import fast as F
from oracle import iam_oracle as O
from oracle import synth_model as SM

from gpu_util import assert_close_bf16, check_argmax_identical

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402

SEED = 20261201
CTX = 1024


def cdims(d: O.Dims, max_ctx: int, max_rows: int, max_seqs: int = 1) -> I.Dims:
    c = I.Dims.qwen35_27b()
    for f in dataclasses.fields(d):
        setattr(c, {"group": "group_size"}.get(f.name, f.name), getattr(d, f.name))
    c.max_ctx, c.max_rows, c.max_seqs = max_ctx, max_rows, max_seqs
    return c


def test_27b_step_k32_and_k1():
    d = O.QWEN35_27B
    K = 32
    tokens = SM.draft_tokens(SEED, d, K, tag="full27b")
    max_ctx = CTX + K + 8
    am_ref, acc_ref, normed, logits = F.model_step_streaming(tokens, CTX, SEED, d, CTX, max_ctx, return_hidden=True)
    e = I.Engine(cdims(d, max_ctx, K))
    e.init_synthetic(SEED)
    e.state_init(SEED, CTX)
    am, acc = e.verify(tokens, CTX)
    hid = e.read_hidden(K)
    # K = 1: the first position of the block is the decode step of tokens[0]
    e.state_init(SEED, CTX)
    am1, _ = e.verify(tokens[:1], CTX)
    hid1 = e.read_hidden(1)
    e.close()
    assert_close_bf16(hid, normed)
    assert_close_bf16(hid1, normed[:1])
    check_argmax_identical(am, logits, "27B K=32")
    assert acc == acc_ref
    check_argmax_identical(am1, logits[:1], "27B K=1")


@pytest.mark.parametrize("K", [1, 32])
def test_lm_head_full_vocab(K):
    d = O.Dims(n_layers=1)
    tokens = SM.draft_tokens(SEED, d, K, tag=f"lmhead{K}")
    max_ctx = 64
    am_ref, acc_ref, normed, logits = F.model_step_streaming(tokens, 0, SEED, d, 0, max_ctx, return_hidden=True)
    e = I.Engine(cdims(d, max_ctx, max(K, 8)))
    e.init_synthetic(SEED)
    e.state_init(SEED, 0)
    am, acc = e.verify(tokens, 0)
    hid = e.read_hidden(K)
    e.close()
    assert_close_bf16(hid, normed)
    check_argmax_identical(am, logits, f"lm_head K={K}")
    assert acc == acc_ref


def test_batch_64_sequences_k8_ctx1024():
    d = O.Dims(n_layers=4, vocab=32768)
    n_seq, K = 64, 8
    max_ctx = CTX + K + 8
    tokens = np.stack([SM.draft_tokens(SEED, d, K, tag=f"b64_{q}") for q in range(n_seq)])
    pos = np.full(n_seq, CTX, np.int32)
    e = I.Engine(cdims(d, max_ctx, n_seq * K, n_seq))
    e.init_synthetic(SEED)
    e.state_init(SEED, CTX)  # every slot q seeded from its own streams

    am, acc = e.verify_batch(tokens, pos)
    hid = e.read_hidden(n_seq * K).reshape(n_seq, K, d.hidden)
    e.close()
    W = F.make_weights(SEED, d)
    O.cache_dequant(True)  # one dequantized copy of each weight for all 64 sequences
    try:
        with F.fast_dequant():
            for q in range(n_seq):
                st = SM.make_state(SEED, d, CTX, max_ctx, slot=q)
                am_r, acc_r, normed, logits = O.model_step(tokens[q], CTX, W, st, d, return_hidden=True)
                assert_close_bf16(hid[q], normed)
                check_argmax_identical(am[q], logits, f"sequence {q}")
                assert acc[q] == acc_r, q
    finally:
        O.cache_dequant(False)
