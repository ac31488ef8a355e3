"""nt_replay_noalloc: the replay launch for callers that cannot allocate.

A host that hands the whole device to its own budgeted memory pool, or that
prices inside a latency-critical loop where cudaMalloc and cudaFree would
synchronise the device, cannot let the engine allocate.
nt_replay_noalloc runs an already-compiled kernel on the caller's device
buffers and stream, with its reduction scratch in a static device array.
Here it must give the same sums as nt_replay (the existing entry point) on
two calls in a row, reject an executable that needs global scratch, and
reject a launch whose reduction records exceed the static maximum.  This
file is collected last so a stopping run has already run every other test;
it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from nablatensor_b200 import _lib, quant
from nablatensor_b200.engine import AadOptions, B200AadExecutable, PrecisionEnum
from nablatensor_b200.tape import AadRecorder

pytestmark = pytest.mark.gpu

ATM = [100.0, 100.0, 0.20, 0.03, 1.0]
FP64 = AadOptions(precision=PrecisionEnum.FLOAT64)
NOALLOC_FLAGS = _lib.NT_FLAG_RECOMPUTE_ALL | _lib.NT_FLAG_SHARED_CKPT


def _noalloc(ex, paths, offset, seed, d_in, d_sums, stream):
    return _lib.lib().nt_replay_noalloc(ex._handle(), paths, offset & (2**64 - 1), seed & (2**64 - 1),
                                        ctypes.c_void_p(d_in.data_ptr()), ctypes.c_void_p(d_sums.data_ptr()),
                                        ctypes.c_void_p(stream.cuda_stream))


def test_noalloc_matches_replay_on_two_calls(ntlib):
    import torch
    tape = quant.asian_tape(252)
    ex = B200AadExecutable(tape, FP64, 0, flags=NOALLOC_FLAGS)
    try:
        want1, _ = ex.replay_sums(100_000, 0x1_0000_0003, 42)
        ex.setInputs([98.0, 100.0, 0.25, 0.01, 2.0])
        want2, _ = ex.replay_sums(33_333, 5, 0x12345678FEDCBA98)

        stream = torch.cuda.Stream(device=0)
        d_in1 = torch.tensor(ATM, dtype=torch.float64, device="cuda:0")
        d_in2 = torch.tensor([98.0, 100.0, 0.25, 0.01, 2.0], dtype=torch.float64, device="cuda:0")
        d_sums = torch.zeros(7, dtype=torch.float64, device="cuda:0")
        torch.cuda.synchronize()

        _lib.check(_noalloc(ex, 100_000, 0x1_0000_0003, 42, d_in1, d_sums, stream))
        stream.synchronize()
        got1 = d_sums.cpu().numpy()
        _lib.check(_noalloc(ex, 33_333, 5, 0x12345678FEDCBA98, d_in2, d_sums, stream))
        stream.synchronize()
        got2 = d_sums.cpu().numpy()
    finally:
        ex.close()
    np.testing.assert_allclose(got1, want1, rtol=1e-12, atol=0)
    np.testing.assert_allclose(got2, want2, rtol=1e-12, atol=0)


def test_noalloc_rejects_an_executable_with_global_scratch(ntlib):
    import torch
    ex = B200AadExecutable(quant.asian_tape(16), FP64, 0)  # value tape + L2 checkpoints
    try:
        d_in = torch.tensor(ATM, dtype=torch.float64, device="cuda:0")
        d_sums = torch.zeros(7, dtype=torch.float64, device="cuda:0")
        rc = _noalloc(ex, 1000, 0, 1, d_in, d_sums, torch.cuda.current_stream(0))
        assert rc == _lib.NT_E_UNSUPPORTED
        assert "NT_FLAG_RECOMPUTE_ALL" in _lib.lib().nt_last_error().decode()
    finally:
        ex.close()


def test_noalloc_rejects_scratch_beyond_the_maximum(ntlib):
    import torch
    n_in = 300  # 302 channels; with 32-thread blocks a full grid's reduction records exceed 1 MiB

    def body(rec):
        xs = [rec.input(f"x{j}", 1.0 + j) for j in range(n_in)]
        acc = rec.constant(0.0)
        for x in xs:
            acc = acc.add(x.mul(rec.randn()))
        rec.output(acc)

    tape = AadRecorder.record(body)
    ex = B200AadExecutable(tape, FP64.with_engine_option("cuda", "block", "32"), 0, flags=NOALLOC_FLAGS)
    try:
        assert ex.info()["grid"] * (2 + n_in) * 8 > (1 << 20)
        d_in = torch.ones(n_in, dtype=torch.float64, device="cuda:0")
        d_sums = torch.zeros(2 + n_in, dtype=torch.float64, device="cuda:0")
        rc = _noalloc(ex, 10_000_000, 0, 1, d_in, d_sums, torch.cuda.current_stream(0))
        assert rc == _lib.NT_E_INVALID_ARG
        assert "static maximum" in _lib.lib().nt_last_error().decode()
    finally:
        ex.close()
