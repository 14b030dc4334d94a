"""Weights beyond a resident budget stream from pinned host memory.

dims.resident_weight_bytes keeps the layers resident in order while their
4-bit matrices (as loaded plus tile-packed) fit; the matrices of the rest live
in pinned host memory, and every step copies each streamed layer's packed
matrices into one of two device slots on a second stream, one layer ahead of
its use (the role of prefetchLayer / MADV_WILLNEED, warm_forward.swift:556-650).
The outputs must be bit-identical to the engine with every layer resident:
a K-token verify, a 1-token step and a second block (both graph widths, the
slots turning over within and across steps), from synthetic weights and from
a safetensors checkpoint loaded straight into the pinned copies.
"""
import dataclasses

import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth_model as SM

from ckpt_util import tensors_of, write_checkpoint
from gpu_util import check_argmax_identical

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402

D = O.TINY
SEED = 20261205
CTX = 9


def cdims(budget):
    c = I.Dims.qwen35_27b()
    for f in dataclasses.fields(D):
        setattr(c, {"group": "group_size"}.get(f.name, f.name), getattr(D, f.name))
    c.max_ctx, c.max_rows = 64, 8
    c.resident_weight_bytes = budget
    return c


def _al(n):
    return (n + 255) // 256 * 256


def layer_bytes(li):
    """A layer's 4-bit matrices as loaded (words, scales, biases) plus packed."""
    d = D
    H, I_ = d.hidden, d.intermediate
    mats = [(I_, H), (I_, H), (H, I_)]
    if (li + 1) % d.full_attn_interval == 0:
        hd = d.head_dim
        mats += [(2 * d.n_heads * hd, H), (d.n_kv_heads * hd, H), (d.n_kv_heads * hd, H), (H, d.n_heads * hd)]
    else:
        conv = 2 * d.gdn_k_heads * 128 + d.gdn_v_heads * 128
        mats += [(conv, H), (d.gdn_v_heads * 128, H), (d.gdn_v_heads, H), (d.gdn_v_heads, H),
                 (H, d.gdn_v_heads * 128)]
    loaded = sum(_al(r * k // 2) + 2 * _al(r * k // 64 * 2) for r, k in mats)
    packed = _al(I.qmm_packed_bytes(2 * I_, H)) + sum(_al(I.qmm_packed_bytes(r, k)) for r, k in mats[2:])
    return loaded + packed


def _run(e, blocks):
    e.state_init(SEED, CTX)
    out, pos = [], CTX
    for toks in blocks:
        am, acc = e.verify(toks, pos)
        out.append((list(am), acc, e.read_hidden(len(toks)).copy()))
        pos += len(toks)
    return out


def _blocks():
    return [SM.draft_tokens(SEED, D, 5, tag="pf0"), SM.draft_tokens(SEED, D, 1, tag="pf1"),
            SM.draft_tokens(SEED, D, 4, tag="pf2")]


@pytest.fixture(scope="module")
def resident():
    e = I.Engine(cdims(0))
    e.init_synthetic(SEED)
    assert e.streamed_layers() == 0
    got = _run(e, _blocks())
    e.close()
    W = SM.make_weights(SEED, D)
    st = SM.make_state(SEED, D, CTX, 64)
    _, _, _, logits = O.model_step(_blocks()[0], CTX, W, st, D, return_hidden=True)
    check_argmax_identical(got[0][0], logits)
    return got


@pytest.mark.parametrize("keep", [0, 1, 2])
def test_streamed_layers_bit_identical(resident, keep):
    budget = sum(layer_bytes(li) for li in range(keep)) + 1
    e = I.Engine(cdims(budget))
    try:
        assert e.streamed_layers() == D.n_layers - keep
        e.init_synthetic(SEED)
        got = _run(e, _blocks())
    finally:
        e.close()
    for (am, acc, hid), (am0, acc0, hid0) in zip(got, resident):
        assert am == am0 and acc == acc0
        assert np.array_equal(hid, hid0)


def test_streamed_layers_from_checkpoint(resident, tmp_path):
    paths = write_checkpoint(tmp_path, tensors_of(SM.make_weights(SEED, D)), shards=2)
    e = I.Engine(cdims(1))
    try:
        assert e.streamed_layers() == D.n_layers
        e.load_safetensors(paths)
        w = e.read_tensor("model.layers.2.mlp.down_proj.weight", D.hidden * D.intermediate // 2)
        got = _run(e, _blocks())
    finally:
        e.close()
    r = I.Engine(cdims(0))
    try:
        r.init_synthetic(SEED)
        w0 = r.read_tensor("model.layers.2.mlp.down_proj.weight", D.hidden * D.intermediate // 2)
    finally:
        r.close()
    assert np.array_equal(w, w0)
    for (am, acc, hid), (am0, acc0, hid0) in zip(got, resident):
        assert am == am0 and acc == acc0
        assert np.array_equal(hid, hid0)
