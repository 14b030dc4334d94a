"""Loading MLX-format safetensors checkpoints into the engine on the GPU
(iam_load_safetensors):

* a checkpoint written from the synthetic generator's weights gives the same
  tensors and the same verify outputs, bit for bit, as iam_init_synthetic;
* a checkpoint with a 4-bit embedding, no lm_head (tied) and the prefixes of
  a multimodal export: the embedding is dequantized into the bf16 table bit
  for bit as embed_lookup_bf16 does, and the K-token verify matches the
  oracle step run on the same weights (parity bar of the engine tests).
"""
import dataclasses

import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth_model as SM

from ckpt_util import quantized_embedding, tensors_of, write_checkpoint
from gpu_util import assert_close_bf16, check_argmax_identical

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402

D = O.TINY
SEED = 20261203


def cdims(max_ctx=64, max_rows=8):
    c = I.Dims.qwen35_27b()
    for f in dataclasses.fields(D):
        setattr(c, {"group": "group_size"}.get(f.name, f.name), getattr(D, f.name))
    c.max_ctx, c.max_rows = max_ctx, max_rows
    return c


def test_checkpoint_equals_synthetic(tmp_path):
    paths = write_checkpoint(tmp_path, tensors_of(SM.make_weights(SEED, D)), shards=3)
    tokens = SM.draft_tokens(SEED, D, 5)
    outs = []
    for how in ("synthetic", "checkpoint"):
        e = I.Engine(cdims())
        if how == "synthetic":
            e.init_synthetic(SEED)
        else:
            e.load_safetensors(paths)
        e.state_init(SEED, 7)
        am, acc = e.verify(tokens, 7)
        hid = e.read_hidden(len(tokens))
        w = e.read_tensor("model.layers.3.mlp.down_proj.weight", D.hidden * D.intermediate // 2)
        outs.append((am, acc, hid, w))
        e.close()
    (am0, acc0, h0, w0), (am1, acc1, h1, w1) = outs
    assert np.array_equal(w0, w1)
    assert np.array_equal(am0, am1) and acc0 == acc1
    assert np.array_equal(h0, h1)


def test_quantized_tied_embedding(tmp_path):
    W = SM.make_weights(SEED, D)
    q, table = quantized_embedding(SEED, D)
    t = {k: v for k, v in tensors_of(W).items() if not k.startswith("lm_head.") and k != "model.embed_tokens.weight"}
    t["model.embed_tokens.weight"] = ("U32", q[0])
    t["model.embed_tokens.scales"] = ("BF16", O.to_u16(q[1]))
    t["model.embed_tokens.biases"] = ("BF16", O.to_u16(q[2]))
    t = {("language_model." + k): v for k, v in t.items()}
    paths = write_checkpoint(tmp_path, t, shards=2)

    e = I.Engine(cdims())
    e.load_safetensors(paths)
    got = e.read_tensor("model.embed_tokens.weight", D.vocab * D.hidden * 2).view(np.uint16).reshape(D.vocab, D.hidden)
    assert np.array_equal(got, O.to_u16(table))
    lm = e.read_tensor("lm_head.weight", q[0].nbytes).view(np.uint32).reshape(q[0].shape)
    assert np.array_equal(lm, q[0])

    ctx, K = 6, 4
    tokens = SM.draft_tokens(SEED, D, K)
    e.state_init(SEED, ctx)
    am, acc = e.verify(tokens, ctx)
    hid = e.read_hidden(K)
    e.close()
    W["model.embed_tokens.weight"] = table
    W["lm_head"] = q
    st = SM.make_state(SEED, D, ctx, 64)
    am_ref, acc_ref, normed, logits = O.model_step(np.asarray(tokens), ctx, W, st, D, return_hidden=True)
    assert_close_bf16(hid, normed)
    check_argmax_identical(am, logits)
    assert acc == acc_ref


def test_mismatch_loads_nothing(tmp_path):
    t = tensors_of(SM.make_weights(SEED, D))
    del t["model.norm.weight"]
    paths = write_checkpoint(tmp_path, t)
    e = I.Engine(cdims())
    with pytest.raises(I.IamError) as err:
        e.load_safetensors(paths)
    assert err.value.status == I.IAM_EINVAL and "missing model.norm.weight" in str(err.value)
    e.close()
