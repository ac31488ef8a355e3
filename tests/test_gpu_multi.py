"""Scenario-range sharding over several B200s with one NCCL all-reduce.

Runs tests/dist_worker.py under torchrun (skipped with fewer than two GPUs):
  - on every visible GPU, the all-reduced sums of the shards must have the
    same bits as a single-GPU replay of the whole range, and match the CPU
    oracle in all seven channels to 1e-12 relative, for 2,000,000 paths and
    for a ragged 2,000,003 at a path offset above 2^32;
  - on two GPUs, a rank that leaves between nt_dist_attach and
    nt_replay_sharded ends the survivor's call with NT_E_NCCL within its
    communicator timeout, not a hang.
NVLS is off (NCCL_NVLS_ENABLE=0): no rank's memory is bound to an NVLink
multicast object when a peer leaves.
"""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NT_E_NCCL = -6
LEAVE_TIMEOUT_S = 5.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _torchrun(n, case, limit):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", NT_DIST_CASE=case)
    cmd = ["timeout", "-k", "30", str(limit), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "dist_worker.py")]
    p = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=limit + 60)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-4000:]
    line = [l for l in p.stdout.splitlines() if l.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


def _gpus():
    import torch
    return torch.cuda.device_count()


def test_sharded_replay_has_the_bits_of_one_gpu_and_matches_the_oracle(ntlib):
    n = _gpus()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    res = _torchrun(n, "parity", 600)
    print(json.dumps(res, indent=1))
    for name, r in res.items():
        assert r["same_bits_as_one_gpu"], (name, r)
        assert len(r["rel_vs_oracle"]) == 7
        assert max(r["rel_vs_oracle"]) <= 1e-12, (name, r)


def test_a_rank_that_leaves_ends_the_survivors_call_with_an_error(ntlib):
    if _gpus() < 2:
        pytest.skip("needs at least two GPUs")
    res = _torchrun(2, "leave", 300)
    print(json.dumps(res))
    assert res["code"] == NT_E_NCCL, res
    assert res["elapsed_s"] < LEAVE_TIMEOUT_S + 30.0, res
    assert res["replay_after_abort_finite"], res
