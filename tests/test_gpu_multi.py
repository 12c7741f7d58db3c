"""Sequence-sharded decode on 2+ GPUs: each rank holds a slice of the KV positions and decodes it
to partials, which reach every rank either through an NCCL all-gather or, fused, through the
decode kernel's own stores into the other ranks' exchange areas (CUDA IPC over NVLink); every
rank merges them.  The result must match the oracle over the whole context (north-star
tolerance).  Skipped with fewer than 2 visible GPUs."""
import os
import socket

import numpy as np
import pytest

from tests.util import assert_close, f16_round

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(context, B, Hq, Hkv, D):
    rng = np.random.default_rng(123)
    k = rng.standard_normal((B, context + 1, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((B, context + 1, Hkv, D), dtype=np.float32)
    q = rng.standard_normal((B, 1, Hq, D), dtype=np.float32)
    return q, k, v


def _rank(rank, world, port, context, B, Hq, Hkv, D, path, fused):
    import datetime

    import torch
    import torch.distributed as dist

    from brimkern_b200.engine import AttentionEngine, AttnConfig
    from brimkern_b200.sharded import ShardedDecoder, ShardPlan
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        q, k, v = _inputs(context, B, Hq, Hkv, D)
        eng = AttentionEngine(rank)
        plan = ShardPlan(context, world, rank)
        dec = ShardedDecoder(eng, plan, 1, B, Hkv, D, extra=1, fused=fused, max_rows=B * Hq)
        for b in range(B):
            dec.kv.write_rows(0, b, 0, torch.from_numpy(k[b, plan.lo:plan.hi]).to(dev),
                              torch.from_numpy(v[b, plan.lo:plan.hi]).to(dev))
        cfg = AttnConfig(Hq, Hkv, D)
        q_work = torch.empty((B, 1, Hq, D), dtype=torch.float32, device=dev)
        out = torch.empty((B, 1, Hq, D), dtype=torch.float32, device=dev)
        # The new token (position `context`) brings its own K/V; no rope table: q passes through.
        # Two steps over the same token: the second one uses the other parity of the areas.
        for _ in range(2):
            dec.step(0, cfg, torch.from_numpy(q).to(dev), torch.from_numpy(k[:, context:context + 1]).contiguous().to(dev),
                     torch.from_numpy(v[:, context:context + 1]).contiguous().to(dev), context, q_work, out)
        eng.ctx.check()
        if rank == 0:
            np.save(path, out.cpu().numpy())
        dec.close()
        eng.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_sequence_sharded_decode(tmp_path, world, fused):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    from oracle import oracle as O
    context, B, Hq, Hkv, D = 4095, 2, 8, 2, 64
    path = str(tmp_path / "out.npy")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_rank, args=(world, _free_port(), context, B, Hq, Hkv, D, path, fused), nprocs=world,
                       start_method="spawn")
    got = np.load(path)
    q, k, v = _inputs(context, B, Hq, Hkv, D)
    for b in range(B):
        ref = O.attention(q[b].ravel(), f16_round(k[b]).ravel(), f16_round(v[b]).ravel(), 1, Hq, Hkv, D, context)
        assert_close(got[b].ravel(), ref, what=f"sharded seq {b}")
