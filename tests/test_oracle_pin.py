"""Fresh random cases: oracle vs the reference kernels compiled for the host.

Runs where oracle/_ref/libref_msl.so exists (built by build() from the
reference's source); elsewhere the committed golden vectors cover the same
kernels (test_oracle_golden.py).
"""
import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle.ref_msl import refmsl as R

pytestmark = pytest.mark.skipif(not R.available(), reason="reference kernels not built on this machine")
u, f = O.to_u16, O.from_u16


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_gdn_chain_matches_reference(seed):
    rng = np.random.default_rng(seed)
    C, HK, HV = 10240, 16, 48
    st = O.bf16(rng.standard_normal((3, C)))
    x = O.bf16(rng.standard_normal(C))
    w = O.bf16(0.1 * rng.standard_normal((C, 4)))
    ro, rs = R.depthwise_conv1d(u(st), u(x), u(w))
    oo, os_ = O.depthwise_conv1d_step(st, x, w)
    assert np.array_equal(ro, u(oo)) and np.array_equal(rs, u(os_))
    cs = u(O.silu(oo))
    assert np.array_equal(R.silu(ro), cs)
    q = f(cs[:2048]).reshape(HK, 128)
    k = f(cs[2048:4096]).reshape(HK, 128)
    assert np.array_equal(R.per_head_rms_norm_scaled(u(q), 1e-6, float(O.GDN_Q_SCALE)),
                          u(O.per_head_rms_norm_scaled(q, O.GDN_Q_SCALE)))
    assert np.array_equal(R.per_head_rms_norm_scaled(u(k), 1e-6, float(O.GDN_K_SCALE)),
                          u(O.per_head_rms_norm_scaled(k, O.GDN_K_SCALE)))


def test_rms_norm_many_rows():
    rng = np.random.default_rng(5)
    x = O.bf16(rng.standard_normal((4, 5120)) * 3)
    w = O.bf16(1 + 0.02 * rng.standard_normal(5120))
    assert np.array_equal(R.rms_norm(u(x), u(w)), u(O.rms_norm(x, w)))


def test_sdpa_long_context_within_cap():
    rng = np.random.default_rng(9)
    kc = O.bf16(rng.standard_normal((1024, 4, 256)))
    vc = O.bf16(rng.standard_normal((1024, 4, 256)))
    q = O.bf16(rng.standard_normal((24, 256)) / 16)
    r = f(R.sdpa_decode(u(q), u(kc), u(vc), 1024))
    o = O.sdpa_decode(q, kc, vc, 1024)
    assert np.max(np.abs(r - o)) <= 2.0 ** -7 * np.max(np.abs(o))
