"""Tensor parallelism without a GPU.

* The engine's shard plan (iam_tp_shard_of, the function build_registry uses)
  for the 27B shape at 1/2/4/8 ranks: GDN by V head with the K heads
  following, attention by query head with KV heads split up to 4 ways and
  replicated beyond, MLP by intermediate column, lm_head by vocab row.
* Two gloo ranks on 127.0.0.1 each run their shard of a small model of the
  same family through the oracle (oracle/tp.py), with the row-parallel
  partial products all-reduced and the lm_head maxima all-gathered over gloo:
  the argmax must equal the unsharded oracle step's, the final hidden must
  agree to cos >= 0.9999, and the state shards gathered from both ranks must
  reassemble the unsharded state.
"""
import dataclasses
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

import iam_b200 as I
from oracle import iam_oracle as O
from oracle import synth_model as SM
from oracle import tp as TP

# GQA 2:1 attention, so 2 ranks split the KV heads
TINY = O.TINY
# one KV head, so 2 ranks replicate it (the 8-way case of the 27B model)
TINY_KV1 = dataclasses.replace(O.TINY, n_kv_heads=1)


def iam_dims(d: O.Dims, max_ctx=64, max_rows=8):
    return I.Dims.qwen35_27b(
        hidden=d.hidden, intermediate=d.intermediate, vocab=d.vocab, n_layers=d.n_layers,
        full_attn_interval=d.full_attn_interval, n_heads=d.n_heads, n_kv_heads=d.n_kv_heads, head_dim=d.head_dim,
        rotary_dim=d.rotary_dim, gdn_k_heads=d.gdn_k_heads, gdn_v_heads=d.gdn_v_heads, gdn_dk=d.gdn_dk,
        gdn_dv=d.gdn_dv, max_ctx=max_ctx, max_rows=max_rows)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_27b(world):
    d = I.Dims.qwen35_27b()
    seen_kv = []
    for r in range(world):
        s = I.tp_shard_of(d, r, world)
        assert (s.gdn_k_heads, s.gdn_v_heads) == (16 // world, 48 // world)
        assert (s.gdn_k_head0, s.gdn_v_head0) == (r * 16 // world, r * 48 // world)
        # the 3 V heads that read one K head stay on the same rank
        assert s.gdn_v_head0 // 3 == s.gdn_k_head0 and s.gdn_v_heads == 3 * s.gdn_k_heads
        assert (s.q_heads, s.q_head0) == (24 // world, r * 24 // world)
        assert s.kv_heads == max(1, 4 // world)
        # every query head's KV head (h // 6) is held by the same rank
        for h in range(s.q_head0, s.q_head0 + s.q_heads):
            assert s.kv_head0 <= h // 6 < s.kv_head0 + s.kv_heads
        assert (s.inter, s.inter0) == (17408 // world, r * 17408 // world)
        assert s.inter % 64 == 0
        assert (s.vocab, s.vocab0) == (248320 // world, r * 248320 // world)
        seen_kv.append(s.kv_head0)
    if world == 8:
        assert seen_kv == [0, 0, 1, 1, 2, 2, 3, 3]


@pytest.mark.parametrize("world,rank", [(3, 0), (16, 0), (2, 2), (2, -1), (0, 0)])
def test_plan_rejects(world, rank):
    with pytest.raises(I.IamError) as e:
        I.tp_shard_of(I.Dims.qwen35_27b(), rank, world)
    assert e.value.status == I.IAM_EINVAL


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cos(a, b):
    a, b = a.ravel().astype(np.float64), b.ravel().astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def _rank_main(rank, world, port, cases):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        def all_reduce(x):
            t = torch.from_numpy(np.array(x, np.float32, copy=True))
            dist.all_reduce(t)
            return t.numpy()

        def all_gather(x):
            t = torch.from_numpy(np.array(x, np.float32, copy=True))
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            return [p.numpy() for p in parts]

        for name, d, seed, ctx, k in cases:
            W = SM.make_weights(seed, d)
            st0 = SM.make_state(seed, d, ctx, ctx + 16)
            tokens = SM.draft_tokens(seed, d, k)
            ref_state = SM.make_state(seed, d, ctx, ctx + 16)
            am, acc, normed, _ = O.model_step(tokens, ctx, W, ref_state, d, return_hidden=True)

            shard = I.tp_shard_of(iam_dims(d, ctx + 16), rank, world).as_dict()
            Wl = TP.shard_weights(W, d, shard)
            stl = TP.shard_state(st0, d, shard)
            am_tp, acc_tp, normed_tp, _ = TP.model_step_tp(tokens, ctx, Wl, stl, d, shard, all_reduce, all_gather,
                                                          return_hidden=True)
            assert np.array_equal(am_tp, am), (name, rank, am_tp, am)
            assert acc_tp == acc
            c = _cos(normed_tp, normed)
            assert c >= 0.9999, (name, rank, c)

            # the ranks' state shards reassemble the unsharded state
            for li, S in ref_state.S.items():
                got = np.concatenate(all_gather(stl.S[li]), axis=0)
                rel = np.abs(got - S).max() / np.abs(S).max()
                assert rel <= 1e-3, (name, li, rel)
            for li, conv in ref_state.conv.items():
                parts = all_gather(stl.conv[li])
                got = np.zeros_like(conv)
                for r, p in enumerate(parts):
                    sh = I.tp_shard_of(iam_dims(d, ctx + 16), r, world).as_dict()
                    got[:, TP.qkv_channels(d, sh)] = p
                assert _cos(got, conv) >= 0.9999, (name, li)
                if li == 0:  # layer 0 reads the embedding: same inputs, same bits
                    assert np.array_equal(got, conv), name
            for li, kc in ref_state.k_cache.items():
                parts = all_gather(stl.k_cache[li])
                for r, p in enumerate(parts):
                    sh = I.tp_shard_of(iam_dims(d, ctx + 16), r, world).as_dict()
                    want = kc[:, sh["kv_head0"]: sh["kv_head0"] + sh["kv_heads"]]
                    assert _cos(p, want) >= 0.9999, (name, li, r)
                    assert np.array_equal(p[:ctx], want[:ctx])
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_tp2_gloo_shard_sum_equals_unsharded():
    import torch.multiprocessing as mp

    cases = [("tiny", TINY, 11, 5, 4), ("tiny_kv1", TINY_KV1, 12, 3, 3)]
    mp.spawn(_rank_main, args=(2, _free_port(), cases), nprocs=2, join=True)


def test_tp_oracle_single_rank_is_the_oracle():
    """World 1 through the tensor-parallel code path: bit-identical to the plain step
    (the all-reduce is the identity and bf16(fp32 partial) is the plain matmul)."""
    d = TINY
    W = SM.make_weights(5, d)
    tokens = SM.draft_tokens(5, d, 3)
    s1 = SM.make_state(5, d, 4, 20)
    s2 = SM.make_state(5, d, 4, 20)
    am, acc, normed, _ = O.model_step(tokens, 4, W, s1, d, return_hidden=True)
    shard = I.tp_shard_of(iam_dims(d, 20), 0, 1).as_dict()
    sl = TP.shard_state(s2, d, shard)
    am1, acc1, normed1, _ = TP.model_step_tp(tokens, 4, TP.shard_weights(W, d, shard), sl, d, shard, lambda x: x,
                                             lambda x: [x], return_hidden=True)
    assert np.array_equal(am, am1) and acc == acc1
    assert np.array_equal(normed, normed1)
    for li in s1.S:
        assert np.array_equal(s1.S[li], sl.S[li])
        assert np.array_equal(s1.conv[li], sl.conv[li])
    for li in s1.k_cache:
        assert np.array_equal(s1.k_cache[li], sl.k_cache[li])
