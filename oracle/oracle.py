"""ctypes front-end of the CPU oracle (test infrastructure only).

The oracle restates NablaTensor's scalar ``cpu`` engine (ScalarReplay.java +
Philox.java + AadTotals.java, see nt_oracle.h for file:line citations).  Only
tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this
module; the B200 product path never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

OPS = ["CONST", "INPUT", "RANDN", "RANDU", "ADD", "SUB", "MUL", "DIV", "NEG",
       "EXP", "LOG", "SQRT", "MAX", "MIN", "ABS"]


class OrcTape(ctypes.Structure):
    _fields_ = [
        ("n", ctypes.c_int32),
        ("op", ctypes.POINTER(ctypes.c_int32)),
        ("arg_a", ctypes.POINTER(ctypes.c_int32)),
        ("arg_b", ctypes.POINTER(ctypes.c_int32)),
        ("constant", ctypes.POINTER(ctypes.c_double)),
        ("n_in", ctypes.c_int32),
        ("input_node", ctypes.POINTER(ctypes.c_int32)),
        ("n_out", ctypes.c_int32),
        ("output_node", ctypes.POINTER(ctypes.c_int32)),
        ("n_streams", ctypes.c_int32),
    ]


class OrcTapeBuf(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.POINTER(ctypes.c_int32)),
        ("arg_a", ctypes.POINTER(ctypes.c_int32)),
        ("arg_b", ctypes.POINTER(ctypes.c_int32)),
        ("constant", ctypes.POINTER(ctypes.c_double)),
        ("cap", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("input_node", ctypes.c_int32 * 8),
        ("n_in", ctypes.c_int32),
        ("output_node", ctypes.c_int32),
    ]


def build() -> str:
    """Compiles liboracle.so with the committed Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        u32p = ctypes.POINTER(ctypes.c_uint32)
        L.orc_philox2x32_10.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, u32p]
        L.orc_normal_words.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int32, ctypes.c_uint32, u32p]
        L.orc_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int32, ctypes.c_uint32]
        L.orc_normal.restype = ctypes.c_double
        L.orc_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int32, ctypes.c_uint32]
        L.orc_uniform.restype = ctypes.c_double
        L.orc_replay.argtypes = [ctypes.POINTER(OrcTape), ctypes.POINTER(ctypes.c_double), ctypes.c_int,
                                 ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int,
                                 ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        L.orc_replay.restype = ctypes.c_int
        L.orc_replay_ex.argtypes = [ctypes.POINTER(OrcTape), ctypes.POINTER(ctypes.c_double), ctypes.c_int,
                                    ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int,
                                    ctypes.c_int, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        L.orc_replay_ex.restype = ctypes.c_int
        L.orc_mark_active.argtypes = [ctypes.POINTER(OrcTape), ctypes.POINTER(ctypes.c_uint8)]
        for name in ("orc_build_european", "orc_build_asian"):
            getattr(L, name).argtypes = [ctypes.POINTER(OrcTapeBuf), ctypes.c_int, ctypes.c_int]
            getattr(L, name).restype = ctypes.c_int
        L.orc_build_barrier.argtypes = [ctypes.POINTER(OrcTapeBuf), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_double, ctypes.c_double]
        L.orc_build_barrier.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


@dataclass
class FlatTape:
    """Flat arrays in FlatTape.java order; a plain value object for the oracle."""
    op: np.ndarray
    arg_a: np.ndarray
    arg_b: np.ndarray
    constant: np.ndarray
    input_node: np.ndarray
    output_node: np.ndarray
    n_streams: int = 1

    @property
    def n(self):
        return int(self.op.shape[0])

    @classmethod
    def of(cls, tape) -> "FlatTape":
        """From any object with the same attribute names (e.g. the package's AadTape)."""
        return cls(np.ascontiguousarray(tape.op, dtype=np.int32), np.ascontiguousarray(tape.arg_a, dtype=np.int32),
                   np.ascontiguousarray(tape.arg_b, dtype=np.int32),
                   np.ascontiguousarray(tape.constant, dtype=np.float64),
                   np.ascontiguousarray(tape.input_node, dtype=np.int32),
                   np.ascontiguousarray(tape.output_node, dtype=np.int32), int(tape.n_streams))

    def _struct(self):
        self._keep = [np.ascontiguousarray(x) for x in
                      (self.op, self.arg_a, self.arg_b, self.constant, self.input_node, self.output_node)]
        op, a, b, c, inn, outn = self._keep
        return OrcTape(self.n, _ptr(op, ctypes.c_int32), _ptr(a, ctypes.c_int32), _ptr(b, ctypes.c_int32),
                       _ptr(c, ctypes.c_double), int(inn.shape[0]), _ptr(inn, ctypes.c_int32),
                       int(outn.shape[0]), _ptr(outn, ctypes.c_int32), int(self.n_streams))

    def active(self) -> np.ndarray:
        out = np.zeros(self.n, dtype=np.uint8)
        s = self._struct()
        lib().orc_mark_active(ctypes.byref(s), _ptr(out, ctypes.c_uint8))
        return out.astype(bool)


def _built(fn, *args, cap=1 << 16) -> FlatTape:
    op = np.zeros(cap, np.int32)
    a = np.zeros(cap, np.int32)
    b = np.zeros(cap, np.int32)
    c = np.zeros(cap, np.float64)
    buf = OrcTapeBuf(_ptr(op, ctypes.c_int32), _ptr(a, ctypes.c_int32), _ptr(b, ctypes.c_int32),
                     _ptr(c, ctypes.c_double), cap, 0)
    n = fn(ctypes.byref(buf), *args)
    if n < 0:
        raise ValueError("tape capacity exceeded")
    return FlatTape(op[:n].copy(), a[:n].copy(), b[:n].copy(), c[:n].copy(),
                    np.array(list(buf.input_node)[:buf.n_in], np.int32), np.array([buf.output_node], np.int32), 1)


def asian_tape(steps=252, call=True) -> FlatTape:
    return _built(lib().orc_build_asian, steps, int(call))


def european_tape(steps=1, call=True) -> FlatTape:
    return _built(lib().orc_build_european, steps, int(call))


BARRIER_KINDS = {"UP_OUT": 0, "UP_IN": 1, "DOWN_OUT": 2, "DOWN_IN": 3}


def barrier_tape(steps=252, call=True, kind="DOWN_IN", barrier=80.0, width=1.0) -> FlatTape:
    return _built(lib().orc_build_barrier, steps, int(call), BARRIER_KINDS[kind], float(barrier), float(width))


@dataclass
class OracleResult:
    value: np.ndarray       # per output
    stderr: np.ndarray      # per output
    gradients: np.ndarray   # [output, input]
    sums: np.ndarray        # raw n_out * (2 + n_in)
    paths: int


def finish(sums: np.ndarray, n_out: int, n_in: int, paths: int) -> OracleResult:
    """AadTotals.toResult (AadTotals.java:68-89) in numpy."""
    s = np.asarray(sums, dtype=np.float64).reshape(n_out, 2 + n_in)
    mean = s[:, 0] / paths
    if paths > 1:
        var = (s[:, 1] - paths * mean * mean) / (paths - 1)
        stderr = np.sqrt(np.maximum(0.0, var) / paths)
    else:
        stderr = np.full(n_out, np.nan)
    return OracleResult(mean, stderr, s[:, 2:] / paths, s.reshape(-1).copy(), paths)


def replay(tape: FlatTape, inputs, paths: int, path_offset: int = 0, seed: int = 42, f32: bool = False,
           adjoints: bool = True, threads: int = 0, per_path: bool = False, exact: bool = False):
    """ScalarReplay.replay on `threads` host threads.  Returns OracleResult
    (and the per-path [n_out*(1+n_in)] matrix when per_path=True).
    exact=True sums the per-path values with compensated arithmetic (the
    comparison basis for the device's reduction); exact=False is the
    reference's plain running sum."""
    n_in = int(tape.input_node.shape[0])
    n_out = int(tape.output_node.shape[0])
    x = np.ascontiguousarray(inputs, dtype=np.float64)
    sums = np.zeros(n_out * (2 + n_in), np.float64)
    pp = np.zeros((paths, n_out * (1 + n_in)), np.float64) if per_path else None
    s = tape._struct()
    rc = lib().orc_replay_ex(ctypes.byref(s), _ptr(x, ctypes.c_double), int(f32), int(adjoints), paths,
                             path_offset & (2**64 - 1), seed & (2**64 - 1), threads, int(exact),
                             _ptr(sums, ctypes.c_double), _ptr(pp, ctypes.c_double) if per_path else None)
    if rc != 0:
        raise ValueError(f"oracle rejected the tape (code {rc})")
    res = finish(sums, n_out, n_in, paths)
    return (res, pp) if per_path else res


def normal_words(path: int, seed: int, stream: int, pair: int):
    out = (ctypes.c_uint32 * 2)()
    lib().orc_normal_words(path & (2**64 - 1), seed & (2**64 - 1), stream, pair, out)
    return int(out[0]), int(out[1])


def philox(x0: int, x1: int, key: int):
    out = (ctypes.c_uint32 * 2)()
    lib().orc_philox2x32_10(x0, x1, key, out)
    return int(out[0]), int(out[1])


def normal(path: int, seed: int, stream: int, k: int) -> float:
    return lib().orc_normal(path & (2**64 - 1), seed & (2**64 - 1), stream, k)


def uniform(path: int, seed: int, stream: int, k: int) -> float:
    return lib().orc_uniform(path & (2**64 - 1), seed & (2**64 - 1), stream, k)
