"""nt_replay_noalloc: the replay launch for callers that cannot allocate.

A host that hands the whole device to its own budgeted memory pool, or that
prices inside a latency-critical loop where cudaMalloc and cudaFree would
synchronise the device, cannot let the engine allocate.
nt_replay_noalloc runs an already-compiled kernel on the caller's device
buffers and stream, with its reduction scratch in a static device array.
Here it must give the same sums as nt_replay (the existing entry point) on
two calls in a row -- the same kernel and the same exact reduction, so the
same bits -- also when two executables of different channel counts and grids
take turns on the shared scratch; it must reject an executable that needs
global scratch, one whose reduction words exceed the static maximum, and a
host pointer in place of device memory.  This file is collected last so a
stopping run has already run every other test; it also passes alone in a
fresh process.
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
                                        ctypes.c_void_p(d_in), ctypes.c_void_p(d_sums),
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

        _lib.check(_noalloc(ex, 100_000, 0x1_0000_0003, 42, d_in1.data_ptr(), d_sums.data_ptr(), stream))
        stream.synchronize()
        got1 = d_sums.cpu().numpy()
        _lib.check(_noalloc(ex, 33_333, 5, 0x12345678FEDCBA98, d_in2.data_ptr(), d_sums.data_ptr(), stream))
        stream.synchronize()
        got2 = d_sums.cpu().numpy()
    finally:
        ex.close()
    np.testing.assert_array_equal(got1, want1)
    np.testing.assert_array_equal(got2, want2)


def test_two_executables_take_turns_on_the_shared_scratch(ntlib):
    """A (the 252-step Asian: 7 channels, a full grid) then B (two named
    random streams: 4 channels, a 1-block launch) then A again, on one
    stream: each call clears what it uses, so each matches its own nt_replay
    bit for bit."""
    import torch
    from tapes import named_streams
    a = B200AadExecutable(quant.asian_tape(252), FP64, 0, flags=NOALLOC_FLAGS)
    b = B200AadExecutable(named_streams(16), FP64, 0, flags=NOALLOC_FLAGS)
    try:
        assert b.info()["channels"] < a.info()["channels"]
        xb = [100.0, 0.2]
        b.setInputs(xb)
        want_a, _ = a.replay_sums(500_000, 0, 7)
        want_b, _ = b.replay_sums(100, 3, 42)
        stream = torch.cuda.Stream(device=0)
        d_xa = torch.tensor(ATM, dtype=torch.float64, device="cuda:0")
        d_xb = torch.tensor(xb, dtype=torch.float64, device="cuda:0")
        d_sa = torch.zeros(a.info()["channels"], dtype=torch.float64, device="cuda:0")
        d_sb = torch.zeros(b.info()["channels"], dtype=torch.float64, device="cuda:0")
        torch.cuda.synchronize()
        got = []
        for ex, d_x, d_s, paths, off, seed in [(a, d_xa, d_sa, 500_000, 0, 7), (b, d_xb, d_sb, 100, 3, 42),
                                               (a, d_xa, d_sa, 500_000, 0, 7)]:
            _lib.check(_noalloc(ex, paths, off, seed, d_x.data_ptr(), d_s.data_ptr(), stream))
            stream.synchronize()
            got.append(d_s.cpu().numpy().copy())
    finally:
        a.close()
        b.close()
    np.testing.assert_array_equal(got[0], want_a)
    np.testing.assert_array_equal(got[1], want_b)
    np.testing.assert_array_equal(got[2], want_a)


def test_noalloc_rejects_a_host_pointer(ntlib):
    import torch
    ex = B200AadExecutable(quant.asian_tape(16), FP64, 0, flags=NOALLOC_FLAGS)
    try:
        host_in = np.array(ATM, dtype=np.float64)
        d_in = torch.tensor(ATM, dtype=torch.float64, device="cuda:0")
        d_sums = torch.zeros(7, dtype=torch.float64, device="cuda:0")
        host_sums = np.zeros(7, dtype=np.float64)
        stream = torch.cuda.current_stream(0)
        rc = _noalloc(ex, 1000, 0, 1, host_in.ctypes.data, d_sums.data_ptr(), stream)
        assert rc == _lib.NT_E_INVALID_ARG
        assert "d_inputs" in _lib.lib().nt_last_error().decode()
        rc = _noalloc(ex, 1000, 0, 1, d_in.data_ptr(), host_sums.ctypes.data, stream)
        assert rc == _lib.NT_E_INVALID_ARG
        assert "d_sums" in _lib.lib().nt_last_error().decode()
        torch.cuda.synchronize()  # nothing was launched; the context is fine
    finally:
        ex.close()


def test_noalloc_rejects_an_executable_with_global_scratch(ntlib):
    import torch
    ex = B200AadExecutable(quant.asian_tape(16), FP64, 0)  # value tape + L2 checkpoints
    try:
        d_in = torch.tensor(ATM, dtype=torch.float64, device="cuda:0")
        d_sums = torch.zeros(7, dtype=torch.float64, device="cuda:0")
        rc = _noalloc(ex, 1000, 0, 1, d_in.data_ptr(), d_sums.data_ptr(), torch.cuda.current_stream(0))
        assert rc == _lib.NT_E_UNSUPPORTED
        assert "NT_FLAG_RECOMPUTE_ALL" in _lib.lib().nt_last_error().decode()
    finally:
        ex.close()


def test_noalloc_rejects_scratch_beyond_the_maximum(ntlib):
    """118 inputs give 120 channels; their exact-sum words (69 int64 each)
    plus the ticket exceed the 64 KiB static array."""
    import torch
    n_in = 118

    def body(rec):
        xs = [rec.input(f"x{j}", 1.0 + j) for j in range(n_in)]
        acc = rec.constant(0.0)
        for x in xs:
            acc = acc.add(x)
        rec.output(acc.mul(rec.randn()))

    tape = AadRecorder.record(body)
    ex = B200AadExecutable(tape, FP64, 0, flags=NOALLOC_FLAGS)
    try:
        assert 256 + ex.info()["channels"] * 69 * 8 > (64 << 10)
        d_in = torch.ones(n_in, dtype=torch.float64, device="cuda:0")
        d_sums = torch.zeros(2 + n_in, dtype=torch.float64, device="cuda:0")
        rc = _noalloc(ex, 10_000, 0, 1, d_in.data_ptr(), d_sums.data_ptr(), torch.cuda.current_stream(0))
        assert rc == _lib.NT_E_INVALID_ARG
        assert "static maximum" in _lib.lib().nt_last_error().decode()
    finally:
        ex.close()
