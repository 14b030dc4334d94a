"""Failure detection, tested without faulting, trapping or hanging a GPU.

* A bounded wait inside the matmul runs out: with fault injection the kernel
  issues none of its copies, so its first wait is on a phase that nothing
  completes; under a short poll budget the checked call returns IAM_ETIMEOUT
  promptly, nothing is left in flight, and the next calls on the same context
  are correct.  Both packed-weight kernels (the GEMV at 1 token, the tensor
  cores at 32).
* With its copies issued the checked call succeeds under a modest budget.
* A device-resident engine step whose token id is out of range: the
  embedding reads nothing outside the table and flags it; iam_engine_status
  reports IAM_EINVAL and clears it, and the engine stays usable.
* A tensor-parallel engine whose peer rank never joins: the communicator
  set-up (non-blocking, polled against comm_timeout_ms) ends in IAM_ETIMEOUT
  and is aborted; no kernel runs (one GPU is enough).
"""
import time

import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth
from oracle import synth_model as SM

from gpu_util import assert_close_bf16, dev, empty_u16, host_u16, ptr

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import iam_b200 as I  # noqa: E402


def _packed_case(N, K, M, seed):
    w, s, b = synth.gen_qweight(seed, f"t.fail.{N}x{K}", N, K)
    x = synth.gen_normal_bf16(seed + 1, f"t.fail.x.{M}", M * K, 1.0).astype(np.float32).reshape(M, K)
    ref = O.qmm_affine4(x, w, s.astype(np.float32), b.astype(np.float32))
    packed = torch.empty(I.qmm_packed_bytes(N, K), dtype=torch.uint8, device="cuda")
    keep = [dev(w, torch), dev(s.view(np.uint16), torch), dev(b.view(np.uint16), torch)]
    I.qmm_pack_affine4(*[ptr(t) for t in keep], ptr(packed), N, K)
    torch.cuda.synchronize()
    return packed, dev(O.to_u16(x), torch), ref


@pytest.mark.parametrize("M", [1, 32])
def test_starved_matmul_times_out_and_context_stays_usable(M):
    N, K = 1024, 5120
    packed, dx, ref = _packed_case(N, K, M, 91)
    y = empty_u16(torch, M, N)
    t0 = time.perf_counter()
    with pytest.raises(I.IamError) as err:
        I.qmm_affine4_packed_checked(ptr(packed), ptr(dx), ptr(y), M, N, K, wait_limit=2000, starve=True)
    elapsed = time.perf_counter() - t0
    assert err.value.status == I.IAM_ETIMEOUT
    assert elapsed < 10.0, elapsed
    # the same context, straight after: a checked call and a plain one
    for _ in range(2):
        y = empty_u16(torch, M, N)
        I.qmm_affine4_packed_checked(ptr(packed), ptr(dx), ptr(y), M, N, K, wait_limit=1 << 20)
        assert_close_bf16(host_u16(y), ref)
    y = empty_u16(torch, M, N)
    I.qmm_affine4_packed(ptr(packed), ptr(dx), ptr(y), M, N, K)
    torch.cuda.synchronize()
    assert_close_bf16(host_u16(y), ref)


def test_engine_reports_device_side_token_error():
    d = O.TINY
    c = I.Dims.qwen35_27b(hidden=d.hidden, intermediate=d.intermediate, vocab=d.vocab, n_layers=d.n_layers,
                          n_heads=d.n_heads, n_kv_heads=d.n_kv_heads, gdn_k_heads=d.gdn_k_heads,
                          gdn_v_heads=d.gdn_v_heads, max_ctx=64, max_rows=8)
    e = I.Engine(c)
    e.init_synthetic(5)
    e.state_init(5, 10)
    bad = torch.tensor([3, d.vocab + 7], dtype=torch.int32, device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    e.verify_device(bad.data_ptr(), 2, 10, out.data_ptr())
    with pytest.raises(I.IamError) as err:
        e.status()
    assert err.value.status == I.IAM_EINVAL
    e.status()  # cleared
    # still usable: a host-driven step against the oracle
    e.state_init(5, 10)
    toks = SM.draft_tokens(5, d, 3, tag="after_err")
    am, acc = e.verify(toks, 10)
    W = SM.make_weights(5, d)
    st = SM.make_state(5, d, 10, 64)
    am_ref, acc_ref = O.model_step(toks, 10, W, st, d)
    assert list(am) == list(am_ref) and acc == acc_ref
    e.close()


def test_peer_that_never_joins_times_out():
    d = O.TINY
    c = I.Dims.qwen35_27b(hidden=d.hidden, intermediate=d.intermediate, vocab=d.vocab, n_layers=d.n_layers,
                          n_heads=d.n_heads, n_kv_heads=d.n_kv_heads, gdn_k_heads=d.gdn_k_heads,
                          gdn_v_heads=d.gdn_v_heads, max_ctx=64, max_rows=8, comm_timeout_ms=3000)
    uid = I.nccl_unique_id()
    t0 = time.perf_counter()
    with pytest.raises(I.IamError) as err:
        I.Engine(c, device=0, rank=0, world=2, nccl_id=uid)  # rank 1 is never created
    elapsed = time.perf_counter() - t0
    assert err.value.status == I.IAM_ETIMEOUT, err.value
    assert 2.5 < elapsed < 30.0, elapsed
