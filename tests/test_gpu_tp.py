"""Tensor-parallel verify on 2 GPUs (skipped with fewer).

Two processes, one per GPU, each build their engine shard (iam_create with
world 2 and a shared NCCL id); the row-parallel matmuls push their fp32
partials into every rank's receive slots over NVLink (or all-reduce them over
NCCL with IAM_TP_P2P=0) and the lm_head maxima are all-gathered.  Both ranks must
return the oracle's argmax (up to a one-ulp tie of the oracle's top two
logits) and a final hidden within the parity bar, for a model whose KV heads
split over the ranks and one whose single KV head both ranks replicate; a
K-token verify followed by a 1-token decode exercises both graph widths.
NVLS is off (NCCL_NVLS_ENABLE=0) so no rank binds a multicast object.
"""
import dataclasses
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from oracle import iam_oracle as O
from oracle import synth_model as SM

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SEED = 20261202
CASES = [("tiny", O.TINY, 6, 4), ("tiny_kv1", dataclasses.replace(O.TINY, n_kv_heads=1), 3, 5)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    import iam_b200 as I
    from gpu_util import cosine, rel_err
    from test_gpu_engine import cdims, check_argmax

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        for name, d, ctx, k in CASES:
            W = SM.make_weights(SEED, d)
            st = SM.make_state(SEED, d, ctx, ctx + 32)
            tokens = SM.draft_tokens(SEED, d, k)
            nxt = SM.draft_tokens(SEED, d, 1, tag="next")
            am_ref, acc_ref, normed_ref, logits_ref = O.model_step(tokens, ctx, W, st, d, return_hidden=True)
            am2_ref, _, normed2_ref, logits2_ref = O.model_step(nxt, ctx + k, W, st, d, return_hidden=True)

            obj = [I.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            dims = cdims(d, ctx + 32, 8)
            dims.comm_timeout_ms = 30000
            e = I.Engine(dims, device=rank, rank=rank, world=world, nccl_id=obj[0])
            try:
                e.init_synthetic(SEED)
                e.state_init(SEED, ctx)
                dist.barrier()  # every rank is set up before the first collective
                am, acc = e.verify(tokens, ctx)
                hid = O.from_u16(e.read_hidden(k)).reshape(k, d.hidden)
                check_argmax(am, logits_ref)
                assert rel_err(hid, normed_ref) <= 1e-2 and cosine(hid, normed_ref) >= 0.9999, name
                if np.array_equal(am, am_ref):
                    assert acc == acc_ref
                am2, _ = e.verify(nxt, ctx + k)
                hid2 = O.from_u16(e.read_hidden(1)).reshape(1, d.hidden)
                check_argmax(am2, logits2_ref)
                assert rel_err(hid2, normed2_ref) <= 1e-2 and cosine(hid2, normed2_ref) >= 0.9999, name
                dist.barrier()
            finally:
                e.close()
    finally:
        dist.destroy_process_group()


def _rank_batch(rank, world, port):
    """Multi-sequence verify on 2 ranks: per-row lm_head keys all-gathered,
    argmax and accept length per sequence, each sequence against the oracle."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    import iam_b200 as I
    from gpu_util import cosine, rel_err
    from test_gpu_engine import cdims, check_argmax

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        d, ctx, n, K = O.TINY, 6, 3, 4
        W = SM.make_weights(SEED, d)
        tokens = np.stack([SM.draft_tokens(SEED, d, K, tag=f"tpb{q}") for q in range(n)])
        pos = np.array([ctx, ctx + 2, ctx + 5], np.int32)
        obj = [I.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        dims = cdims(d, ctx + 32, n * K)
        dims.max_seqs = n
        dims.comm_timeout_ms = 30000
        e = I.Engine(dims, device=rank, rank=rank, world=world, nccl_id=obj[0])
        try:
            e.init_synthetic(SEED)
            e.state_init(SEED, ctx)
            dist.barrier()
            am, acc = e.verify_batch(tokens, pos)
            hid = O.from_u16(e.read_hidden(n * K)).reshape(n, K, d.hidden)
            for q in range(n):
                st = SM.make_state(SEED, d, ctx, ctx + 32, slot=q)
                am_r, acc_r, normed, logits = O.model_step(tokens[q], int(pos[q]), W, st, d, return_hidden=True)
                check_argmax(am[q], logits)
                assert rel_err(hid[q], normed) <= 1e-2 and cosine(hid[q], normed) >= 0.9999, q
                if np.array_equal(am[q], am_r):
                    assert acc[q] == acc_r
            dist.barrier()
        finally:
            e.close()
    finally:
        dist.destroy_process_group()


def _rank_p2p(rank, world, port):
    """Row-parallel sums over peer memory against the NCCL all-reduce: the
    engine maps the peers' receive areas (CUDA IPC) by default; IAM_TP_P2P=0
    keeps the NCCL all-reduce.  With two ranks both sum the two partials the
    same way, so the normed hidden states must agree bit for bit, for a
    K = 70 block (two matmul passes arrive per tile) and a 1-token step."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    import iam_b200 as I
    from test_gpu_engine import cdims, check_argmax

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        d, ctx, k = O.TINY, 5, 70
        W = SM.make_weights(SEED, d)
        st = SM.make_state(SEED, d, ctx, ctx + 80)
        tokens = SM.draft_tokens(SEED, d, k, tag="p2p")
        nxt = SM.draft_tokens(SEED, d, 1, tag="p2p_next")
        _, _, _, logits_ref = O.model_step(tokens, ctx, W, st, d, return_hidden=True)
        got = {}
        for mode in ("p2p", "nccl"):
            if mode == "nccl":
                os.environ["IAM_TP_P2P"] = "0"
            obj = [I.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            dims = cdims(d, ctx + 80, k)
            dims.comm_timeout_ms = 30000
            e = I.Engine(dims, device=rank, rank=rank, world=world, nccl_id=obj[0])
            try:
                e.init_synthetic(SEED)
                e.state_init(SEED, ctx)
                dist.barrier()
                am, acc = e.verify(tokens, ctx)
                check_argmax(am, logits_ref)
                hid = e.read_hidden(k).copy()
                am1, _ = e.verify(nxt, ctx + k)
                hid1 = e.read_hidden(1).copy()
                kinds = e.profile_step(1, ctx + k + 1)
                assert ("tp_reduce" in kinds) == (mode == "p2p"), sorted(kinds)
                assert ("allreduce" in kinds) == (mode == "nccl"), sorted(kinds)
                got[mode] = (list(am), acc, hid, list(am1), hid1)
                dist.barrier()
            finally:
                e.close()
        os.environ.pop("IAM_TP_P2P", None)
        a, b = got["p2p"], got["nccl"]
        assert a[0] == b[0] and a[1] == b[1] and a[3] == b[3]
        assert np.array_equal(a[2], b[2]) and np.array_equal(a[4], b[4])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_peer_memory_sums_match_nccl():
    import torch.multiprocessing as mp

    mp.spawn(_rank_p2p, args=(2, _free_port()), nprocs=2, join=True)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_batch_matches_oracle():
    import torch.multiprocessing as mp

    mp.spawn(_rank_batch, args=(2, _free_port()), nprocs=2, join=True)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_verify_matches_oracle():
    import torch.multiprocessing as mp

    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)
