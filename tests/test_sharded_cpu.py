"""Sequence-sharded decode, host side, on CPU: the shard plan, the packed-partial all-gather over
torch.distributed (gloo, world size 2 and 3 as separate processes), and the log-sum-exp merge,
with the oracle standing in for the GPU partial / combine kernels."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from brimkern_b200.sharded import ShardPlan, gather_partials, packed_partial_floats
from oracle import oracle as O


def test_plan_covers_context_once():
    for context in (1, 5, 131072, 1000):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for r in range(world):
                p = ShardPlan(context, world, r)
                assert 0 <= p.lo <= p.hi <= context
                covered.extend(range(p.lo, p.hi))
            assert covered == list(range(context)), (context, world)


def test_plan_owner_and_capacity():
    p = ShardPlan(131072, 8, 7)
    assert p.owner(131071) == 7 and p.owner(131072) == 7 and p.owner(0) == 0 and p.owner(16384) == 1
    assert p.capacity(extra=1) == 16384 + 1
    assert ShardPlan(131072, 8, 3).capacity(extra=1) == 16384
    empty = ShardPlan(5, 4, 3)  # shard 2: ranks own [0,2) [2,4) [4,5) and nothing
    assert empty.lo == empty.hi == 5


def _pack(m, l, o):
    rows = m.size
    buf = np.empty(rows * 2 + o.size, np.float32)
    buf[0:rows * 2:2] = m
    buf[1:rows * 2:2] = l
    buf[rows * 2:] = o
    return buf


def _unpack(buf, rows, D):
    return buf[0:rows * 2:2].astype(np.float64), buf[1:rows * 2:2].astype(np.float64), buf[rows * 2:].astype(np.float64)


def _inputs(L, nH, nKv, D, seed=3):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(nH * D).astype(np.float32)
    k = rng.standard_normal(L * nKv * D).astype(np.float32)
    v = rng.standard_normal(L * nKv * D).astype(np.float32)
    return q, k, v


def _worker(rank, world, port, L, nH, nKv, D, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = _inputs(L, nH, nKv, D)
        plan = ShardPlan(L, world, rank)
        m, l, o = O.attention_partial(q, k, v, 1, nH, nKv, D, L - 1, plan.lo, plan.hi)
        part = torch.from_numpy(_pack(m, l, o))
        assert part.numel() == packed_partial_floats(nH, D)
        gathered = gather_partials(part, world).numpy()
        ms, ls, os_ = zip(*[_unpack(gathered[r], nH, D) for r in range(world)])
        out = O.combine(np.concatenate(ms), np.concatenate(ls), np.concatenate(os_), world, nH, D)
        if rank == 0:
            np.save(result_path, out)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_sharded_partials_match_full_attention(tmp_path, world):
    L, nH, nKv, D = 1000, 8, 2, 16
    path = str(tmp_path / "out.npy")
    mp.start_processes(_worker, args=(world, _free_port(), L, nH, nKv, D, path), nprocs=world, start_method="spawn")
    got = np.load(path)
    q, k, v = _inputs(L, nH, nKv, D)
    ref = O.attention(q, k, v, 1, nH, nKv, D, L - 1)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_empty_shard_carries_no_weight():
    """A rank with no key (m = -inf, l = 0) contributes nothing to the merge."""
    L, nH, nKv, D = 5, 4, 2, 8
    q, k, v = _inputs(L, nH, nKv, D, seed=9)
    parts = [O.attention_partial(q, k, v, 1, nH, nKv, D, L - 1, ShardPlan(L, 4, r).lo, ShardPlan(L, 4, r).hi)
             for r in range(4)]
    assert np.all(np.isneginf(parts[3][0])) and np.all(parts[3][1] == 0)
    out = O.combine(np.concatenate([p[0] for p in parts]), np.concatenate([p[1] for p in parts]),
                    np.concatenate([p[2] for p in parts]), 4, nH, D)
    np.testing.assert_allclose(out, O.attention(q, k, v, 1, nH, nKv, D, L - 1), rtol=1e-5, atol=1e-6)
