"""Scenario-range sharding over several B200s with one NCCL all-reduce.

Runs tests/dist_worker.py under torchrun on every visible GPU (skipped with
fewer than two): the all-reduced sums of the shards must equal a single-GPU
replay of the whole range to reduction-order rounding (1e-13), including a
ragged total and a path offset above 2^32.
"""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_replay_matches_single_gpu(ntlib):
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "dist_worker.py")]
    p = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=700)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-4000:]
    line = [l for l in p.stdout.splitlines() if l.startswith("RESULT ")][-1]
    res = json.loads(line[len("RESULT "):])
    for total, r in res.items():
        assert r["value_rel"] <= 1e-13, (total, r)
        assert r["grad_rel"] <= 1e-13, (total, r)
