"""Writes small MLX-format safetensors checkpoints for the loader tests.

A checkpoint holds the decoder tensors under the reference's names
(full_forward.swift:749-822): 4-bit matrices as `<name>.weight` (U32 packed
codes), `.scales` and `.biases` (BF16); norms, conv weights and dt_bias BF16;
A_log F32.  The safetensors layout: an 8-byte little-endian header length, a
JSON header {name: {dtype, shape, data_offsets}} padded with spaces to 8
bytes, then the data.
"""
import json
import struct

import numpy as np

from oracle import iam_oracle as O
from oracle import synth


def tensors_of(W):
    """The oracle's weight dict as {name: (dtype, array)} in checkpoint form."""
    out = {}
    for name, v in W.items():
        if isinstance(v, tuple):
            w, s, b = v
            out[name + ".weight"] = ("U32", np.ascontiguousarray(w, np.uint32))
            out[name + ".scales"] = ("BF16", O.to_u16(s))
            out[name + ".biases"] = ("BF16", O.to_u16(b))
        elif name.endswith("A_log"):
            out[name] = ("F32", np.ascontiguousarray(v, np.float32))
        else:
            out[name] = ("BF16", O.to_u16(v))
    return out


def quantized_embedding(seed, d):
    """A 4-bit embedding table and the bf16 table the engine should make of it."""
    w, s, b = synth.gen_qweight(seed, "ckpt.embed_tokens", d.vocab, d.hidden)
    table = O.dequant(w, s.astype(np.float32), b.astype(np.float32))
    return (w, s.astype(np.float32), b.astype(np.float32)), table


def write_safetensors(path, tensors):
    """tensors: {name: (dtype, array)}; arrays are written as their raw bytes."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        dtype, a = tensors[name]
        raw = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    header["__metadata__"] = {"format": "mlx"}
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for raw in blobs:
            f.write(raw)


def write_checkpoint(tmpdir, tensors, shards=2):
    """Split tensors over `shards` files (round robin by sorted name); returns the paths."""
    names = sorted(tensors)
    paths = []
    for i in range(shards):
        p = str(tmpdir / f"model-{i + 1:05d}-of-{shards:05d}.safetensors")
        write_safetensors(p, {n: tensors[n] for n in names[i::shards]})
        paths.append(p)
    return paths
