"""Checkpoint matching without a GPU (iam_check_safetensors): safetensors
files of a small model of the family are indexed and matched against the
tensors the engine holds -- names (with the prefixes multimodal exports
carry), dtypes, sizes -- and every kind of mismatch is reported by name."""
import dataclasses
import struct

import numpy as np
import pytest

import iam_b200 as I
from oracle import iam_oracle as O
from oracle import synth_model as SM

from ckpt_util import quantized_embedding, tensors_of, write_checkpoint, write_safetensors

D = O.TINY
SEED = 77


def dims():
    c = I.Dims.qwen35_27b()
    for f in dataclasses.fields(D):
        setattr(c, {"group": "group_size"}.get(f.name, f.name), getattr(D, f.name))
    c.max_ctx, c.max_rows = 64, 8
    return c


@pytest.fixture(scope="module")
def base():
    return tensors_of(SM.make_weights(SEED, D))


def check(paths):
    return I.check_safetensors(dims(), paths)


def test_bf16_embedding_own_lm_head(base, tmp_path):
    st, rep = check(write_checkpoint(tmp_path, base, shards=3))
    assert st == I.IAM_OK, rep
    n_engine = len(base)
    assert rep.startswith(f"{n_engine} tensors")
    assert "embedding bf16" in rep and "lm_head own" in rep and "from 3 file(s)" in rep


def test_quantized_tied_embedding_and_prefixes(base, tmp_path):
    t = {k: v for k, v in base.items() if not k.startswith("lm_head.") and k != "model.embed_tokens.weight"}
    (w, s, b), _ = quantized_embedding(SEED, D)
    t["model.embed_tokens.weight"] = ("U32", w)
    t["model.embed_tokens.scales"] = ("BF16", O.to_u16(s))
    t["model.embed_tokens.biases"] = ("BF16", O.to_u16(b))
    # a multimodal export: decoder under language_model., another tower beside it
    t = {("language_model." + k): v for k, v in t.items()}
    t["vision_tower.patch_embed.weight"] = ("BF16", np.zeros((4, 4), np.uint16))
    st, rep = check(write_checkpoint(tmp_path, t))
    assert st == I.IAM_OK, rep
    assert "embedding 4-bit (dequantized at load)" in rep and "lm_head tied to the embedding" in rep
    assert "1 non-decoder tensors ignored" in rep


def test_a_log_as_bf16(base, tmp_path):
    t = dict(base)
    name = "model.layers.0.linear_attn.A_log"
    t[name] = ("BF16", O.to_u16(base[name][1]))
    st, rep = check(write_checkpoint(tmp_path, t))
    assert st == I.IAM_OK, rep


@pytest.mark.parametrize("case", ["missing", "dtype", "transposed", "extra", "short"])
def test_mismatches_are_named(base, tmp_path, case):
    t = dict(base)
    q = "model.layers.1.mlp.down_proj"
    if case == "missing":
        del t["model.layers.2.linear_attn.conv1d.weight"]
        want = "missing model.layers.2.linear_attn.conv1d.weight"
    elif case == "dtype":
        t[q + ".scales"] = ("F32", O.from_u16(base[q + ".scales"][1]))
        want = q + ".scales: dtype F32, expected BF16"
    elif case == "transposed":
        w = base[q + ".weight"][1]
        t[q + ".weight"] = ("U32", np.ascontiguousarray(w.reshape(w.shape[1], w.shape[0])))
        want = q + ".weight: shape"
    elif case == "extra":
        t["model.layers.0.mlp.extra_proj.weight"] = ("BF16", np.zeros((8, 8), np.uint16))
        want = "unused tensor model.layers.0.mlp.extra_proj.weight"
    else:
        w = base[q + ".weight"][1]
        t[q + ".weight"] = ("U32", np.ascontiguousarray(w[:-1]))
        want = q + ".weight: shape"
    st, rep = check(write_checkpoint(tmp_path, t))
    assert st == I.IAM_EINVAL
    assert want in rep, rep


def test_duplicate_across_files(base, tmp_path):
    paths = write_checkpoint(tmp_path, base, shards=2)
    extra = str(tmp_path / "dup.safetensors")
    write_safetensors(extra, {"model.norm.weight": base["model.norm.weight"]})
    st, rep = check(paths + [extra])
    assert st == I.IAM_EINVAL and "appears twice" in rep


@pytest.mark.parametrize("bad", ["truncated", "header_length", "json", "offsets", "no_file"])
def test_malformed_files(base, tmp_path, bad):
    paths = write_checkpoint(tmp_path, base, shards=2)
    p = paths[0]
    raw = open(p, "rb").read()
    hlen = struct.unpack("<Q", raw[:8])[0]
    if bad == "truncated":
        raw = raw[:-16]
        msg = "beyond the end of the file"
    elif bad == "header_length":
        raw = struct.pack("<Q", len(raw)) + raw[8:]
        msg = "header length beyond the file"
    elif bad == "json":
        raw = raw[:8] + b"{" + b"x" * (hlen - 1) + raw[8 + hlen:]
        msg = "header"
    elif bad == "offsets":
        raw = raw[:8] + raw[8:8 + hlen].replace(b'"data_offsets": [0,', b'"data_offsets": [9,', 1) + raw[8 + hlen:]
        msg = "bytes for"
    else:
        p = str(tmp_path / "absent.safetensors")
        paths[0] = p
        msg = "cannot open"
    if bad != "no_file":
        open(p, "wb").write(raw)
    st, rep = check(paths)
    assert st == I.IAM_EINVAL and msg in rep, rep
