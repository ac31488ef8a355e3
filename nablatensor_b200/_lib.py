"""ctypes binding of libnabla_b200.so (include/nabla_b200.h).

The library is built in-tree (``python -m nablatensor_b200.build``).  There is
no fallback: if the shared object is missing or fails to load, every engine
call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnabla_b200.so")

NT_OK = 0
NT_E_INVALID_ARG = -1
NT_E_TAPE = -2
NT_E_UNSUPPORTED = -3
NT_E_CUDA = -4
NT_E_NVRTC = -5
NT_E_NCCL = -6
NT_E_OOM = -7
NT_E_STATE = -8
NT_E_INTERNAL = -9

NT_FLOAT32 = 0
NT_FLOAT64 = 1
NT_FLAG_NO_LOOP = 0x1
NT_FLAG_SHARED_CKPT = 0x2
NT_FLAG_NO_DISK_CACHE = 0x4
NT_FLAG_F32_FAST = 0x8
NT_FLAG_NO_FMAD = 0x10
NT_FLAG_ACC_REGS = 0x20
NT_FLAG_RECOMPUTE_ALL = 0x40
NT_FLAG_TAPE_DRAWS = 0x80
NT_FLAG_TAPE_ALL = 0x100

_i32p = ctypes.POINTER(ctypes.c_int32)
_f64p = ctypes.POINTER(ctypes.c_double)


class NtTape(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int32), ("op", _i32p), ("arg_a", _i32p), ("arg_b", _i32p), ("constant", _f64p),
                ("n_in", ctypes.c_int32), ("input_node", _i32p), ("n_out", ctypes.c_int32),
                ("output_node", _i32p), ("n_streams", ctypes.c_int32), ("normal_count", _i32p),
                ("uniform_count", _i32p)]


class NtOptions(ctypes.Structure):
    _fields_ = [("precision", ctypes.c_int32), ("adjoints", ctypes.c_int32), ("device", ctypes.c_int32),
                ("block", ctypes.c_int32), ("seg_units", ctypes.c_int32), ("min_blocks", ctypes.c_int32),
                ("max_regs", ctypes.c_int32), ("flags", ctypes.c_int32), ("fwd_unroll", ctypes.c_int32),
                ("grid_blocks_per_sm", ctypes.c_int32), ("rev_unroll", ctypes.c_int32)]


class NtExecInfo(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in (
        "registers", "local_bytes", "static_smem", "dynamic_smem", "block", "blocks_per_sm", "grid", "sm_count",
        "channels", "loop_start", "loop_unit", "loop_units", "steps_per_unit", "seg_units", "segments",
        "ckpt_slots", "stored_per_unit", "ckpt_global", "tape_slots", "tape_mbytes", "markets_registers",
        "markets_local_bytes")] + [
        ("compile_seconds", ctypes.c_double), ("fwd_flops", ctypes.c_double), ("rev_flops", ctypes.c_double),
        ("wide_flops", ctypes.c_double), ("arith_flops", ctypes.c_double)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class NablaError(RuntimeError):
    """A failed C-ABI call: ``code`` is the NT_E_* status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


_lib = None
_lock = threading.Lock()

# The exported entry points and their C signatures; the tests check the
# header declares exactly these.
SIGNATURES = {
    "nt_version": ([], ctypes.c_int),
    "nt_last_error": ([], ctypes.c_char_p),
    "nt_init": ([_i32p], ctypes.c_int),
    "nt_compile": ([ctypes.POINTER(NtTape), ctypes.POINTER(NtOptions), ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "nt_set_inputs": ([ctypes.c_void_p, _f64p, ctypes.c_int32], ctypes.c_int),
    "nt_replay": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _f64p, _f64p], ctypes.c_int),
    "nt_replay_markets": ([ctypes.c_void_p, ctypes.c_int32, _f64p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                           _f64p, _f64p], ctypes.c_int),
    "nt_replay_accumulate": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "nt_accumulator_read": ([ctypes.c_void_p, _f64p, ctypes.c_int32], ctypes.c_int),
    "nt_exec_stream": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "nt_exec_info_get": ([ctypes.c_void_p, ctypes.POINTER(NtExecInfo)], ctypes.c_int),
    "nt_exec_source": ([ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)],
                       ctypes.c_int),
    "nt_emit_source": ([ctypes.POINTER(NtTape), ctypes.POINTER(NtOptions), ctypes.c_int32, ctypes.c_char_p,
                        ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "nt_nvrtc_check": ([ctypes.c_char_p, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "nt_nvrtc_version": ([ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32), ctypes.c_char_p,
                          ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "nt_destroy": ([ctypes.c_void_p], None),
    "nt_dist_unique_id": ([ctypes.POINTER(ctypes.c_uint8)], ctypes.c_int),
    "nt_dist_attach": ([ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint8),
                        ctypes.c_int32], ctypes.c_int),
    "nt_replay_sharded": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                           _f64p, _f64p], ctypes.c_int),
    "nt_replay_sharded_async": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                                 ctypes.c_uint64], ctypes.c_int),
    "nt_dist_detach": ([ctypes.c_void_p], ctypes.c_int),
    "nt_shard_range": ([ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int32, ctypes.c_int32,
                        ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "nt_philox_words": ([ctypes.c_int32, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int32,
                         ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32), _f64p], ctypes.c_int),
    "nt_fma_peak": ([ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _f64p], ctypes.c_int),
    "nt_fma_peak_sustained": ([ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _f64p], ctypes.c_int),
    "nt_dist_collective_ms": ([ctypes.c_void_p, _f64p], ctypes.c_int),
    "nt_math_eval": ([ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.POINTER(ctypes.c_uint32), _f64p, _f64p,
                      _f64p], ctypes.c_int),
    "nt_replay_noalloc": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p,
                           ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
}

def math_eval(device: int, which: int, words=None, x=None):
    """nt_math_eval: one of the replay's fp64 routines on the device over the
    given generator words (which 0, 1, 5, 6) or arguments (2, 3, 4, 7).
    Returns out0, or (out0, out1) for which 1, 5, 6 and 7."""
    import numpy as np
    w = None if words is None else np.ascontiguousarray(words, dtype=np.uint32)
    a = None if x is None else np.ascontiguousarray(x, dtype=np.float64)
    n = (len(w) // 2 if which in (5, 6) else len(w)) if w is not None else len(a)
    out0 = np.empty(n, dtype=np.float64)
    out1 = np.empty(n, dtype=np.float64) if which in (1, 5, 6, 7) else None
    check(lib().nt_math_eval(device, which, n,
                             None if w is None else w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                             None if a is None else a.ctypes.data_as(_f64p),
                             out0.ctypes.data_as(_f64p), None if out1 is None else out1.ctypes.data_as(_f64p)))
    return out0 if out1 is None else (out0, out1)


def fma_peak(device: int = 0, fp64: bool = True, iters: int = 4096) -> float:
    """Measured vector-FMA peak in TFLOP/s (nt_fma_peak)."""
    out = ctypes.c_double(0.0)
    check(lib().nt_fma_peak(device, int(fp64), iters, ctypes.byref(out)))
    return out.value


def fma_peak_sustained(device: int = 0, fp64: bool = True, millis: int = 3000) -> float:
    """Vector-FMA rate held over `millis` of back-to-back launches, in
    TFLOP/s (nt_fma_peak_sustained): the power-limited peak."""
    out = ctypes.c_double(0.0)
    check(lib().nt_fma_peak_sustained(device, int(fp64), millis, ctypes.byref(out)))
    return out.value


def lib():
    """Loads libnabla_b200.so once; raises if it is missing (no fallback)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m nablatensor_b200.build`")
            L = ctypes.CDLL(LIB_PATH)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = res
            _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != NT_OK:
        raise NablaError(rc, lib().nt_last_error().decode(errors="replace"))


def ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


def tape_struct(tape):
    """An NtTape view of an AadTape-like object; the returned keep-alive list
    must outlive the call."""
    keep = [np.ascontiguousarray(tape.op, dtype=np.int32), np.ascontiguousarray(tape.arg_a, dtype=np.int32),
            np.ascontiguousarray(tape.arg_b, dtype=np.int32), np.ascontiguousarray(tape.constant, dtype=np.float64),
            np.ascontiguousarray(tape.input_node, dtype=np.int32),
            np.ascontiguousarray(tape.output_node, dtype=np.int32),
            np.ascontiguousarray(tape.normal_count, dtype=np.int32),
            np.ascontiguousarray(tape.uniform_count, dtype=np.int32)]
    op, a, b, c, inn, outn, nc, uc = keep
    s = NtTape(int(op.shape[0]), ptr(op, ctypes.c_int32), ptr(a, ctypes.c_int32), ptr(b, ctypes.c_int32),
               ptr(c, ctypes.c_double), int(inn.shape[0]), ptr(inn, ctypes.c_int32), int(outn.shape[0]),
               ptr(outn, ctypes.c_int32), int(nc.shape[0]), ptr(nc, ctypes.c_int32), ptr(uc, ctypes.c_int32))
    return s, keep


def options_struct(precision=NT_FLOAT64, adjoints=True, device=0, block=0, seg_units=0, min_blocks=0, max_regs=0,
                   flags=0, fwd_unroll=0, grid_blocks_per_sm=0, rev_unroll=0) -> NtOptions:
    return NtOptions(int(precision), int(bool(adjoints)), int(device), int(block), int(seg_units), int(min_blocks),
                     int(max_regs), int(flags), int(fwd_unroll), int(grid_blocks_per_sm), int(rev_unroll))


def emit_source(tape, target: int = 0, **opts) -> str:
    s, keep = tape_struct(tape)
    o = options_struct(**opts)
    n = ctypes.c_size_t(0)
    check(lib().nt_emit_source(ctypes.byref(s), ctypes.byref(o), target, None, 0, ctypes.byref(n)))
    buf = ctypes.create_string_buffer(n.value + 1)
    check(lib().nt_emit_source(ctypes.byref(s), ctypes.byref(o), target, buf, n.value + 1, ctypes.byref(n)))
    return buf.value.decode()


def nvrtc_version():
    """(major, minor, library path) of the NVRTC the engine compiles with."""
    ma, mi, n = ctypes.c_int32(0), ctypes.c_int32(0), ctypes.c_size_t(0)
    check(lib().nt_nvrtc_version(ctypes.byref(ma), ctypes.byref(mi), None, 0, ctypes.byref(n)))
    buf = ctypes.create_string_buffer(n.value + 1)
    check(lib().nt_nvrtc_version(ctypes.byref(ma), ctypes.byref(mi), buf, n.value + 1, ctypes.byref(n)))
    return ma.value, mi.value, buf.value.decode()


def nvrtc_check(source: str) -> int:
    n = ctypes.c_size_t(0)
    check(lib().nt_nvrtc_check(source.encode(), ctypes.byref(n)))
    return n.value


def device_count() -> int:
    n = ctypes.c_int32(0)
    check(lib().nt_init(ctypes.byref(n)))
    return n.value


def shard_range(total: int, offset: int, nranks: int, rank: int):
    """(first path, count) of rank's contiguous shard (nt_shard_range)."""
    f, c = ctypes.c_uint64(0), ctypes.c_uint64(0)
    check(lib().nt_shard_range(total, offset, nranks, rank, ctypes.byref(f), ctypes.byref(c)))
    return f.value, c.value


def philox_words(device: int, path0: int, n_paths: int, seed: int, stream: int, pair0: int, n_pairs: int):
    out = np.zeros(n_paths * n_pairs * 2, dtype=np.uint32)
    normals = np.zeros(n_paths * n_pairs * 2, dtype=np.float64)
    check(lib().nt_philox_words(device, path0 & (2**64 - 1), n_paths, seed & (2**64 - 1), stream, pair0, n_pairs,
                                ptr(out, ctypes.c_uint32), ptr(normals, ctypes.c_double)))
    return out.reshape(n_paths, n_pairs, 2), normals.reshape(n_paths, n_pairs, 2)
