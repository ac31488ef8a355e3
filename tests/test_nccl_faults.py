"""The engine's NCCL failure handling, on the host, against a stand-in NCCL.

A peer that fails or stalls around the all-reduce must end the call with an
error status (NT_E_NCCL), never a hang, and the communicator must be aborted
(ncclCommAbort) exactly once and not used or destroyed afterwards.  The
communicator code (nablatensor_b200/csrc/nt_dist.cpp) is compiled here from
the product source together with tests/nccl_fault_harness.cpp, and loads
tests/nccl_fake.c as its NCCL through NT_NCCL_LIBRARY -- the same dlopen seam
the library uses for the real NCCL.  No GPU is involved; the GPU-side
counterpart (a rank that leaves between attach and the sharded replay) is in
tests/test_gpu_multi.py.
"""
import json
import os
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "nablatensor_b200", "csrc")
NT_E_NCCL, NT_E_STATE, NT_E_CUDA = -6, -8, -4
TIMEOUT_MS = 300


@pytest.fixture(scope="module")
def outcomes():
    d = tempfile.mkdtemp(prefix="nt_nccl_fault_")
    fake, harness = os.path.join(d, "libnccl_fake.so"), os.path.join(d, "harness")
    subprocess.run(["gcc", "-O1", "-shared", "-fPIC", "-o", fake, os.path.join(ROOT, "tests", "nccl_fake.c")],
                   check=True)
    subprocess.run(["g++", "-O1", "-std=c++17", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
                    "-I", "/usr/local/cuda/include", "-o", harness,
                    os.path.join(ROOT, "tests", "nccl_fault_harness.cpp"), os.path.join(CSRC, "nt_dist.cpp"),
                    "-ldl", "-lpthread"], check=True)
    p = subprocess.run([harness], env=dict(os.environ, NT_NCCL_LIBRARY=fake), capture_output=True, text=True,
                       timeout=60)
    assert p.returncode == 0, p.stderr
    return {r["case"]: r for r in map(json.loads, p.stdout.splitlines())}


def test_a_healthy_communicator_joins_reduces_and_is_destroyed(outcomes):
    r = outcomes["healthy"]
    assert r["code"] == 0 and not r["aborted"], r
    assert (r["inits"], r["reduces"], r["aborts"], r["destroys"]) == (1, 1, 0, 1), r


def test_a_failed_unique_id_is_an_nccl_error(outcomes):
    r = outcomes["unique_id_fails"]
    assert r["code"] == NT_E_NCCL and r["inits"] == 0, r


@pytest.mark.parametrize("case", ["init_fails", "init_stalls"])
def test_a_failed_or_stalled_join_aborts_the_communicator(outcomes, case):
    r = outcomes[case]
    assert r["code"] == NT_E_NCCL, r
    assert (r["aborts"], r["destroys"]) == (1, 0), r
    if case == "init_stalls":  # bounded by the timeout, not a hang
        assert TIMEOUT_MS <= r["ms"] < TIMEOUT_MS + 2000, r
        assert "not complete" in r["message"]


@pytest.mark.parametrize("case", ["allreduce_fails", "remote_error_after_enqueue", "peer_never_joins"])
def test_an_all_reduce_failure_aborts_the_communicator(outcomes, case):
    r = outcomes[case]
    assert r["code"] == NT_E_NCCL and r["aborted"], r
    assert (r["aborts"], r["destroys"]) == (1, 0), r
    assert "communicator aborted" in r["message"], r
    if case == "peer_never_joins":
        assert TIMEOUT_MS <= r["ms"] < TIMEOUT_MS + 2000, r


def test_a_collective_that_never_completes_times_out_after_the_shard(outcomes):
    r = outcomes["collective_never_completes"]
    assert r["code"] == NT_E_NCCL and r["aborted"], r
    assert (r["aborts"], r["destroys"]) == (1, 0), r
    # The shard ran for 2 x timeout without a deadline; the deadline started
    # when only the collective was left.
    assert 3 * TIMEOUT_MS <= r["ms"] < 3 * TIMEOUT_MS + 2000, r
    assert "a peer left or stalled" in r["message"]


def test_a_cuda_error_while_waiting_aborts_and_propagates(outcomes):
    r = outcomes["cuda_error_while_waiting"]
    assert r["code"] == NT_E_CUDA and r["aborted"], r
    assert (r["aborts"], r["destroys"]) == (1, 0), r


def test_an_aborted_communicator_refuses_further_work(outcomes):
    r = outcomes["use_after_abort"]
    assert r["code"] == NT_E_STATE and r["aborted"], r
    assert (r["aborts"], r["reduces"], r["destroys"]) == (1, 0, 0), r
