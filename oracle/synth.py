"""Seeded synthetic tensors, restated in numpy bit-for-bit with the CUDA generator.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module; the
product generates its synthetic weights on the GPU (csrc/synth.cu) and the tests
use this restatement to check that the device generator produced exactly these
bits, and to build oracle inputs of small sizes without a GPU.

The reference loads real MLX-4bit checkpoints (full_forward.swift:555-595); no
checkpoint is available here, so every tensor is a counter-based hash of
(seed, tensor name, element index).  Distributions follow the benchmark
workload description:

* 4-bit codes uniform in 0..15, packed 8 per uint32, low nibble first
  (nibble order of embed_lookup_bf16, full_forward.swift:123-128);
* scale = bf16(|N(0, 0.02)|), bias = bf16(-8 * scale);
* "N(0, sigma)" is the Irwin-Hall sum of four 16-bit uniforms rescaled to unit
  variance (support +-3.46 sigma).  It uses only integer adds and two
  correctly rounded fp32 multiplies, so numpy and CUDA agree to the bit;
* U(lo, hi) from the top 24 bits of the hash.

All arithmetic is modulo 2**64 on uint64.
"""
from __future__ import annotations

import numpy as np
import ml_dtypes

BF16 = ml_dtypes.bfloat16
GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)
KEYMUL = np.uint64(0xD1B54A32D192ED03)
# float32(sqrt(3) / 65536): maps the centred 4x16-bit sum to unit variance.
IH_SCALE = np.uint32(0x37DDB3D7).view(np.float32)
BASE_SEED = 20261201


def _u64(x) -> np.uint64:
    return np.uint64(int(x) & 0xFFFFFFFFFFFFFFFF)


def mix64(z: np.ndarray) -> np.ndarray:
    """splitmix64 finalizer on a uint64 array (wrapping arithmetic)."""
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        return z ^ (z >> np.uint64(31))


def fnv1a64(name: str) -> int:
    h = 0xCBF29CE484222325
    for byte in name.encode():
        h ^= byte
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def stream_of(seed: int, name: str) -> np.uint64:
    with np.errstate(over="ignore"):
        z = np.array([_u64(seed) * GOLDEN + _u64(fnv1a64(name)) * KEYMUL], dtype=np.uint64)
    return mix64(z)[0]


def hashes(seed: int, name: str, n: int, start: int = 0) -> np.ndarray:
    s = stream_of(seed, name)
    i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return mix64(s + i * GOLDEN)


def normal_f32(h: np.ndarray, sigma: float) -> np.ndarray:
    m = np.uint64(0xFFFF)
    s = (h & m) + ((h >> np.uint64(16)) & m) + ((h >> np.uint64(32)) & m) + ((h >> np.uint64(48)) & m)
    c = (s.astype(np.int64) - 131070).astype(np.float32)
    n = (c * IH_SCALE).astype(np.float32)
    return (n * np.float32(sigma)).astype(np.float32)


def uniform_f32(h: np.ndarray, lo: float, hi: float) -> np.ndarray:
    # u = top 24 bits * 2^-24 in [0, 1); value = lo + u * (hi - lo), each op rounded in fp32
    u = (h >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -24)
    return (np.float32(lo) + (u * np.float32(hi - lo)).astype(np.float32)).astype(np.float32)


# ---- typed tensors (what the device generator writes) ----------------------

def gen_words(seed: int, name: str, n: int) -> np.ndarray:
    """uint32 words of 8 packed uniform 4-bit codes."""
    return (hashes(seed, name, n) & np.uint64(0xFFFFFFFF)).astype(np.uint32)


def gen_normal_bf16(seed: int, name: str, n: int, sigma: float) -> np.ndarray:
    return normal_f32(hashes(seed, name, n), sigma).astype(BF16)


def gen_absnormal_bf16(seed: int, name: str, n: int, sigma: float) -> np.ndarray:
    return np.abs(normal_f32(hashes(seed, name, n), sigma)).astype(BF16)


def gen_one_plus_normal_bf16(seed: int, name: str, n: int, sigma: float) -> np.ndarray:
    return (np.float32(1.0) + normal_f32(hashes(seed, name, n), sigma)).astype(np.float32).astype(BF16)


def gen_normal_f32(seed: int, name: str, n: int, sigma: float) -> np.ndarray:
    return normal_f32(hashes(seed, name, n), sigma)


def gen_uniform_f32(seed: int, name: str, n: int, lo: float, hi: float) -> np.ndarray:
    return uniform_f32(hashes(seed, name, n), lo, hi)


def gen_tokens(seed: int, name: str, n: int, vocab: int) -> np.ndarray:
    return (hashes(seed, name, n) % np.uint64(vocab)).astype(np.int32)


def gen_qweight(seed: int, name: str, rows: int, cols: int, group: int = 64):
    """MLX affine 4-bit weight triple for a [rows, cols] matrix:
    w uint32 [rows, cols/8], scales bf16 [rows, cols/group], biases = -8 * scales."""
    w = gen_words(seed, name + ".weight", rows * cols // 8).reshape(rows, cols // 8)
    s = gen_absnormal_bf16(seed, name + ".scales", rows * cols // group, 0.02).reshape(rows, cols // group)
    b = (s.astype(np.float32) * np.float32(-8.0)).astype(BF16)
    return w, s, b
