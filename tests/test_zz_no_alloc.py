"""iam_qmm_affine4_noalloc (fixed split-K scratch inside the library) against
iam_qmm_affine4 through the C ABI: two calls in a row on shapes whose plans
split K (so the scratch is used and must be left zeroed by each call), plus
the argument and size checks.  Both entry points run the same kernels with the
same plan; split-K partials meet through fp32 atomics whose order varies, so
the outputs are compared with the matmul tolerance and must agree bit for bit
on almost every element."""
import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth

from gpu_util import assert_close_bf16, dev, empty_u16, host_u16, ptr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402


@pytest.mark.parametrize("N,K,M", [(1024, 5120, 8), (5120, 17408, 4), (48, 5120, 40)])
def test_noalloc_matches_qmm_affine4_twice(N, K, M):
    ks, nf, nc = I.qmm_affine4_plan(M, N, K)
    assert ks > 1 and 0 < nf <= 1 << 20 and 0 < nc <= 16384, (ks, nf, nc)  # the fixed scratch is in use
    w, s, b = synth.gen_qweight(71, f"t.noalloc.{N}x{K}", N, K)
    x = synth.gen_normal_bf16(72, f"t.noalloc.x.{M}x{K}", M * K, 1.0).reshape(M, K)
    keep = [dev(w, torch), dev(s.view(np.uint16), torch), dev(b.view(np.uint16), torch), dev(x.view(np.uint16), torch)]
    ref = empty_u16(torch, M, N)
    I.qmm_affine4(*[ptr(t) for t in keep], ptr(ref), M, N, K)
    torch.cuda.synchronize()
    want = host_u16(ref)
    oracle = O.qmm_affine4(x.astype(np.float32), w, s.astype(np.float32), b.astype(np.float32))
    for _ in range(2):
        y = empty_u16(torch, M, N)
        I.qmm_affine4_noalloc(*[ptr(t) for t in keep], ptr(y), M, N, K)
        torch.cuda.synchronize()
        got = host_u16(y)
        assert_close_bf16(got, O.from_u16(want).astype(np.float32), rel=1e-3, cos=0.999999)
        assert np.mean(got != want) < 0.01
        assert_close_bf16(got, oracle)


def test_noalloc_rejects_shapes_beyond_its_scratch(monkeypatch):
    """A plan whose split-K scratch exceeds the fixed array is an IAM_EINVAL,
    reported before anything is launched (the pointers are never read).  The
    library's own planner splits K only for matrices too narrow to fill the
    GPU, whose scratch fits; a plan forced to split K four ways over 65536
    rows of 32 tokens (IAM_QMM_CFG, the planner override) needs 2 Mi floats."""
    monkeypatch.setenv("IAM_QMM_CFG", "8,4")
    N, K, M = 65536, 5120, 32
    ks, nf, nc = I.qmm_affine4_plan(M, N, K)
    assert ks == 4 and nf > 1 << 20, (ks, nf, nc)
    with pytest.raises(I.IamError) as err:
        I.qmm_affine4_noalloc(16, 16, 16, 16, 16, M, N, K)
    assert err.value.status == I.IAM_EINVAL


def test_noalloc_rejects_bad_arguments():
    with pytest.raises(I.IamError):
        I.qmm_affine4_noalloc(0, 0, 0, 0, 0, 1, 16, 64, 64)  # null pointers
    with pytest.raises(I.IamError):
        I.qmm_affine4_noalloc(1, 1, 1, 1, 1, 1, 16, 100, 64)  # K not a multiple of 64
    with pytest.raises(I.IamError):
        I.qmm_affine4_noalloc(1, 1, 1, 1, 1, 1, 16, 64, 32)  # group size
