"""The seeded generator (restated bit-for-bit by csrc/synth.cu)."""
import numpy as np

from oracle import synth


def test_mix64_known_answer():
    # splitmix64 finalizer of 1 (a published test value of the splitmix64 mixer)
    z = synth.mix64(np.array([np.uint64(0x9E3779B97F4A7C15)], np.uint64))[0]
    assert int(z) == 0xE220A8397B1DCDAF


def test_fnv1a_known_answer():
    assert synth.fnv1a64("") == 0xCBF29CE484222325
    assert synth.fnv1a64("a") == 0xAF63DC4C8601EC8C


def test_normal_moments():
    x = synth.gen_normal_f32(1, "t", 200000, 1.0)
    assert abs(float(x.mean())) < 0.01
    assert abs(float(x.std()) - 1.0) < 0.01
    assert float(np.abs(x).max()) <= 3.4642


def test_codes_uniform_and_scales_positive():
    w, s, b = synth.gen_qweight(1, "m", 64, 1024)
    q = (w[..., None] >> (np.arange(8, dtype=np.uint32) * 4)) & 0xF
    counts = np.bincount(q.reshape(-1), minlength=16)
    assert counts.min() > 0.9 * counts.mean()
    assert np.all(s.astype(np.float32) >= 0)
    assert np.array_equal(b.astype(np.float32), -8 * s.astype(np.float32))


def test_prefix_consistency():
    a = synth.hashes(3, "x", 100)
    b = synth.hashes(3, "x", 40, start=60)
    assert np.array_equal(a[60:], b)
