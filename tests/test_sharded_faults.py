"""Failure detection of the sequence-sharded exchange, on the host (gloo ranks on CPU; no GPU is
faulted): a rank that dies before the exchange, or never joins the group, makes every other rank
end with an error within the process group's timeout instead of hanging."""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from brimkern_b200.sharded import gather_partials, packed_partial_floats


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, failing, mode, result_dir):
    import datetime
    status = "ok"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if rank == failing and mode == "never_joins":
        np.save(os.path.join(result_dir, f"r{rank}.npy"), np.array(["absent"]))
        return
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
        if rank == failing and mode == "dies":
            np.save(os.path.join(result_dir, f"r{rank}.npy"), np.array(["died"]))
            os._exit(0)  # leaves without joining the exchange or shutting the group down
        part = torch.zeros(packed_partial_floats(4, 8))
        gather_partials(part, world)
    except Exception as exc:  # the error every surviving rank must see
        status = "error: " + type(exc).__name__
    np.save(os.path.join(result_dir, f"r{rank}.npy"), np.array([status]))
    if dist.is_initialized() and status == "ok":
        dist.destroy_process_group()
    os._exit(0)  # do not wait on a group whose peer is gone


@pytest.mark.parametrize("mode", ["dies", "never_joins"])
def test_failed_rank_is_reported_not_hung(tmp_path, mode):
    world, failing = 3, 2
    t0 = time.monotonic()
    ctx = mp.start_processes(_worker, args=(world, _free_port(), failing, mode, str(tmp_path)), nprocs=world,
                             start_method="spawn", join=False)
    deadline = time.monotonic() + 60
    while not ctx.join(timeout=1):
        assert time.monotonic() < deadline, "ranks did not finish within 60 s"
    elapsed = time.monotonic() - t0
    for r in range(world):
        status = str(np.load(tmp_path / f"r{r}.npy")[0])
        if r == failing:
            assert status in ("died", "absent")
        else:
            assert status.startswith("error"), f"rank {r}: {status}"
    assert elapsed < 60
