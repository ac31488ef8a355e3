"""Scenario-range sharding across ranks, on CPU with gloo (world size 2).

The multi-GPU path splits [offset, offset + total) into contiguous shards
(nt_shard_range, the C ABI's own arithmetic) and all-reduces the sums vector
once.  Here each rank replays its shard with the CPU oracle and the sums are
all-reduced over gloo: the result must equal the single-process replay of
the whole range.  A second case makes one rank fail before the collective
(it raises and exits); the survivor's collective must end with an error
within the process-group timeout instead of hanging -- failure detection on
the host, no GPU involved.
"""
import os
import socket
import sys

import numpy as np
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ATM = [100.0, 100.0, 0.20, 0.03, 1.0]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank, world, port, total, offset, out):
    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist
    from nablatensor_b200 import _lib
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    first, count = _lib.shard_range(total, offset, world, rank)
    r = O.replay(O.asian_tape(16), ATM, count, first, 42, threads=1, exact=True)
    t = torch.tensor(r.sums, dtype=torch.float64)
    dist.all_reduce(t)
    out[rank] = t.numpy().tolist()
    dist.destroy_process_group()


def _failing_worker(rank, world, port, out):
    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # dies between steps, before the all-reduce
    t = torch.ones(7, dtype=torch.float64)
    try:
        dist.all_reduce(t)
        out[rank] = "completed"
    except Exception as e:  # the survivor learns of the failure on the host
        out[rank] = "error: " + type(e).__name__


def test_sharded_sums_equal_the_whole_range(ntlib, oracle_mod):
    total, offset = 10_001, 0x1_0000_0003
    manager = mp.Manager()
    out = manager.dict()
    mp.start_processes(_shard_worker, args=(2, _free_port(), total, offset, out), nprocs=2, join=True,
                       start_method="spawn")
    whole = oracle_mod.replay(oracle_mod.asian_tape(16), ATM, total, offset, 42, threads=1, exact=True).sums
    for rank in (0, 1):
        np.testing.assert_allclose(np.array(out[rank]), whole, rtol=1e-14)


def test_a_dead_rank_ends_the_collective_with_an_error(ntlib):
    manager = mp.Manager()
    out = manager.dict()
    ctx = mp.start_processes(_failing_worker, args=(2, _free_port(), out), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung instead of failing"
    assert ctx.processes[1].exitcode == 3
    assert str(out.get(0, "")).startswith("error"), dict(out)
