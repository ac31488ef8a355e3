"""Scenario-range sharding across ranks, on CPU with gloo (world size 2).

The multi-GPU path splits [offset, offset + total) into contiguous shards
(nt_shard_range, the C ABI's own arithmetic) and all-reduces the sums vector
once.  Here each rank replays its shard with the CPU oracle and the sums are
all-reduced over gloo: the result must equal the single-process replay of
the whole range.  A second case makes one rank fail before the collective
(it raises and exits); the survivor's collective must end with an error
within the process-group timeout instead of hanging -- failure detection on
the host, no GPU involved.  A third case runs the multi-GPU reduction's
arithmetic on CPU ranks (tile-aligned shards, the kernel's butterfly tile
sums, exact words, one int64 all-reduce) and checks that world sizes 1, 2 and
3 give the same bits.
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


_XWORDS_SRC = r"""
#define NT_HOST 1
#include <stdint.h>
#include "nt_exact.cuh"
extern "C" void nt_x_add(long long* w, const double* x, long long n) {
  for (long long i = 0; i < n; ++i) nt_exact_add(w, x[i]);
}
extern "C" double nt_x_round(const long long* w) { return nt_exact_to_double(w); }
"""


def _exact_lib():
    import ctypes
    import subprocess
    import tempfile
    d = tempfile.mkdtemp(prefix="nt_xw_")
    src, so = os.path.join(d, "x.cpp"), os.path.join(d, "x.so")
    with open(src, "w") as f:
        f.write(_XWORDS_SRC)
    subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-I",
                    os.path.join(ROOT, "nablatensor_b200", "csrc"), "-o", so, src], check=True)
    lib = ctypes.CDLL(so)
    lib.nt_x_add.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong]
    lib.nt_x_round.argtypes = [ctypes.c_void_p]
    lib.nt_x_round.restype = ctypes.c_double
    return lib


def _tile_sums(values):
    """The replay kernel's per-tile sums: lane l of a 32-path tile holds path
    l's value (0 past the end), and five xor-butterfly steps add lane l and
    lane l ^ off in every lane, as nt_warp_allsum does with shuffles."""
    n = values.shape[0]
    tiles = -(-n // 32)
    lanes = np.zeros((tiles * 32,) + values.shape[1:])
    lanes[:n] = values
    lanes = lanes.reshape((tiles, 32) + values.shape[1:])
    idx = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        lanes = lanes + lanes[:, idx ^ off]
    return lanes[:, 0]


def _exact_worker(rank, world, port, per_path, total, out):
    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist
    from nablatensor_b200 import _lib

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    xl = _exact_lib()
    first, count = _lib.shard_range(total, 0, world, rank)
    mine = np.asarray(per_path)[first:first + count]
    channels = mine.shape[1]
    words = np.zeros((channels, 69), dtype=np.int64)
    if count:
        sums = _tile_sums(mine)
        for c in range(channels):
            col = np.ascontiguousarray(sums[:, c])
            xl.nt_x_add(words[c].ctypes.data, col.ctypes.data, col.size)
    t = torch.from_numpy(words)
    dist.all_reduce(t)  # int64 sum: exact, so associative
    w = t.numpy()
    out[rank] = [np.float64(xl.nt_x_round(np.ascontiguousarray(w[c]).ctypes.data)).hex() for c in range(channels)]
    dist.destroy_process_group()


def test_exact_words_all_reduce_to_the_same_bits_at_any_world_size(oracle_mod):
    """The multi-GPU reduction's arithmetic on CPU ranks: each rank takes its
    tile-aligned shard (nt_shard_range), sums its 32-path tiles by the
    kernel's butterfly, adds the tile sums into the exact words, and the ranks
    all-reduce the words as int64 over gloo.  The rounded sums must have the
    same bits at world sizes 1, 2 and 3 (and equal math.fsum of the tile sums),
    though 10,007 paths leave a ragged last tile."""
    import math
    total = 10_007
    _, pp = oracle_mod.replay(oracle_mod.asian_tape(16), ATM, total, 0x1_0000_0003, 42, threads=1, exact=True,
                              per_path=True)
    results = {}
    for world in (1, 2, 3):
        manager = mp.Manager()
        out = manager.dict()
        mp.start_processes(_exact_worker, args=(world, _free_port(), pp.tolist(), total, out), nprocs=world,
                           join=True, start_method="spawn")
        assert all(out[r] == out[0] for r in range(world))
        results[world] = out[0]
    assert results[1] == results[2] == results[3]
    tiles = _tile_sums(pp)
    want = [np.float64(math.fsum(tiles[:, c])).hex() for c in range(pp.shape[1])]
    assert results[1] == want
