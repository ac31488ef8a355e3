"""Shared fixtures.  `-m gpu` tests need a B200; everything else runs on CPU."""
from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (run with -m gpu)")


@pytest.fixture(scope="session")
def ntlib():
    """libnabla_b200.so, built in-tree if missing or stale."""
    from nablatensor_b200 import build, _lib
    build.build()
    return _lib.lib()


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O
    O.build()
    return O


_HOST_DIR = os.path.join(tempfile.gettempdir(), "nt_host_kernels")


def host_kernel(source: str, markets: bool = False):
    """Compiles an nt_emit_source(target=1) program with g++ (no FMA
    contraction, like the Java reference) and returns its nt_host_replay
    (markets=True: a target=3 program and its nt_host_replay_markets, taking
    an [n_markets][n_in] input matrix and returning [n_markets][channels])."""
    os.makedirs(_HOST_DIR, exist_ok=True)
    key = hashlib.sha1(source.encode()).hexdigest()[:16]
    src = os.path.join(_HOST_DIR, key + ".cpp")
    so = os.path.join(_HOST_DIR, key + ".so")
    if not os.path.exists(so):
        with open(src, "w") as f:
            f.write(source)
        subprocess.run(["g++", "-O1", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC",
                        "-I", os.path.join(ROOT, "nablatensor_b200", "csrc"), "-o", so + ".tmp", src],
                       check=True)
        os.replace(so + ".tmp", so)
    lib = ctypes.CDLL(so)
    if markets:
        fm = lib.nt_host_replay_markets
        fm.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64,
                       ctypes.c_uint64, ctypes.POINTER(ctypes.c_double)]
        fm.restype = None

        def run_markets(inputs, paths, offset, seed, channels):
            x = np.ascontiguousarray(inputs, dtype=np.float64)
            sums = np.zeros((x.shape[0], channels), dtype=np.float64)
            fm(x.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), x.shape[0], paths, offset & (2**64 - 1),
               seed & (2**64 - 1), sums.ctypes.data_as(ctypes.POINTER(ctypes.c_double)))
            return sums
        run_markets.lib = lib
        return run_markets
    fn = lib.nt_host_replay
    fn.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                   ctypes.POINTER(ctypes.c_double)]
    fn.restype = None

    def run(inputs, paths, offset, seed, channels):
        x = np.ascontiguousarray(inputs, dtype=np.float64)
        sums = np.zeros(channels, dtype=np.float64)
        fn(x.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), paths, offset & (2**64 - 1), seed & (2**64 - 1),
           sums.ctypes.data_as(ctypes.POINTER(ctypes.c_double)))
        return sums
    run.lib = lib
    return run
