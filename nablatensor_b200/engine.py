"""The engine SPI: AadEngine / AadExecutable / AadResult / AadOptions.

Mirrors nablatensor-core/.../engine/{AadEngine,AadExecutable,AbstractAadExecutable,
AadResult,AadTotals,AadOptions,AadEngines}.java: same names, argument meaning
and error behaviour (ValueError for IllegalArgumentException, RuntimeError for
IllegalStateException, NotImplementedError for UnsupportedOperationException).
The engine registered here is "cuda" (priority 110, above the reference's
CudaAadEngine at 100, CudaAadEngine.java:26-34, so that a name lookup finds it
first, as the Java module java/nablatensor-engine-b200 does) and is backed by
libnabla_b200.so; there is no CPU fallback once it is selected.
"""
from __future__ import annotations

import ctypes
import math
import time
from dataclasses import dataclass, field, replace
from enum import IntEnum
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _lib
from .tape import AadTape


class PrecisionEnum(IntEnum):
    FLOAT32 = 0
    FLOAT64 = 1


@dataclass(frozen=True)
class AadOptions:
    """AadOptions.java:42-156 (FLOAT32 and adjoints on by default)."""
    precision: PrecisionEnum = PrecisionEnum.FLOAT32
    adjoints: bool = True
    threads: int = 0
    engine_options: Dict[str, Dict[str, str]] = field(default_factory=dict)

    @staticmethod
    def defaults() -> "AadOptions":
        return AadOptions()

    def with_precision(self, p: PrecisionEnum) -> "AadOptions":
        return replace(self, precision=p)

    def with_adjoints(self, a: bool) -> "AadOptions":
        return replace(self, adjoints=a)

    def with_engine_option(self, engine: str, key: str, value: str) -> "AadOptions":
        eo = {k: dict(v) for k, v in self.engine_options.items()}
        eo.setdefault(engine, {})[key] = str(value)
        return replace(self, engine_options=eo)

    def engine_options_for(self, engine: str) -> Dict[str, str]:
        return self.engine_options.get(engine, {})


class AadResult:
    """AadResult.java: per-output value, standard error and gradients."""

    def __init__(self, output_names, values, stderrs, gradients, input_names, paths, seconds):
        if not output_names:
            raise ValueError("a result needs at least one output")
        self._out = list(output_names)
        self._val = np.asarray(values, dtype=np.float64)
        self._se = np.asarray(stderrs, dtype=np.float64)
        self._grad = np.asarray(gradients, dtype=np.float64).reshape(len(self._out), -1)
        self._in = list(input_names)
        self._paths = int(paths)
        self._seconds = float(seconds)

    @staticmethod
    def from_sums(sums, tape: AadTape, paths: int, seconds: float) -> "AadResult":
        """AadTotals.toResult (AadTotals.java:68-89)."""
        n_out, n_in = tape.output_count(), tape.input_count()
        s = np.asarray(sums, dtype=np.float64).reshape(n_out, 2 + n_in)
        mean = s[:, 0] / paths
        if paths > 1:
            var = (s[:, 1] - paths * mean * mean) / (paths - 1)
            se = np.sqrt(np.maximum(0.0, var) / paths)
        else:
            se = np.full(n_out, np.nan)
        return AadResult(tape.output_names, mean, se, s[:, 2:] / paths, tape.input_names, paths, seconds)

    def value(self, output: Optional[str] = None) -> float:
        return float(self._val[self._oi(output)])

    def standardError(self, output: Optional[str] = None) -> float:
        return float(self._se[self._oi(output)])

    def gradients(self, output: Optional[str] = None) -> np.ndarray:
        return self._grad[self._oi(output)].copy()

    def gradient(self, *names) -> float:
        if len(names) == 1:
            return float(self._grad[0][self._ii(names[0])])
        return float(self._grad[self._oi(names[0])][self._ii(names[1])])

    def outputNames(self) -> List[str]:
        return list(self._out)

    def inputNames(self) -> List[str]:
        return list(self._in)

    def paths(self) -> int:
        return self._paths

    def seconds(self) -> float:
        return self._seconds

    def pathsPerSecond(self) -> float:
        return self._paths / self._seconds if self._seconds > 0 else math.inf

    def _oi(self, name):
        if name is None:
            return 0
        if name not in self._out:
            raise ValueError(f"unknown output: {name} (have {self._out})")
        return self._out.index(name)

    def _ii(self, name):
        if name not in self._in:
            raise ValueError(f"unknown input: {name}")
        return self._in.index(name)

    def __repr__(self):
        vals = ", ".join(f"{n}={v}" for n, v in zip(self._out, self._val))
        return f"AadResult({vals}, paths={self._paths})"


class AadEngine:
    """AadEngine.java:28-48."""

    def name(self) -> str:
        raise NotImplementedError

    def priority(self) -> int:
        raise NotImplementedError

    def isAvailable(self) -> bool:
        raise NotImplementedError

    def supports(self, options: AadOptions) -> bool:
        return True

    def describe(self) -> str:
        return self.name()

    def compile(self, tape: AadTape, options: AadOptions) -> "AadExecutable":
        raise NotImplementedError


class AadExecutable:
    """AadExecutable.java:37-78 with AbstractAadExecutable's chunking."""

    PROBE_PATHS = 65_536
    MIN_CHUNK_PATHS = 4_096

    def engineName(self) -> str:
        raise NotImplementedError

    def tape(self) -> AadTape:
        raise NotImplementedError


_ENGINE_KEYS = {"block": "block", "segUnits": "seg_units", "minBlocks": "min_blocks", "maxRegs": "max_regs",
                "fwdUnroll": "fwd_unroll", "gridBlocksPerSm": "grid_blocks_per_sm", "revUnroll": "rev_unroll"}
_ENGINE_FLAGS = {"noLoop": _lib.NT_FLAG_NO_LOOP, "sharedCheckpoints": _lib.NT_FLAG_SHARED_CKPT,
                 "fp32Fast": _lib.NT_FLAG_F32_FAST, "noFmad": _lib.NT_FLAG_NO_FMAD,
                 "accRegisters": _lib.NT_FLAG_ACC_REGS, "recomputeAll": _lib.NT_FLAG_RECOMPUTE_ALL,
                 "tapeDraws": _lib.NT_FLAG_TAPE_DRAWS, "tapeAll": _lib.NT_FLAG_TAPE_ALL}


class B200AadExecutable(AadExecutable):
    """One compiled tape on one B200 (AadExecutable for engine "cuda")."""

    def __init__(self, tape: AadTape, options: AadOptions, device: int = 0, flags: int = 0):
        self._tape = tape
        self._options = options
        self._closed = True
        knobs = {}
        for k, v in options.engine_options_for("cuda").items():
            if k == "device":
                device = int(v)
            elif k in _ENGINE_KEYS:
                knobs[_ENGINE_KEYS[k]] = int(v)
            elif k in _ENGINE_FLAGS and str(v).lower() in ("1", "true", "on"):
                flags |= _ENGINE_FLAGS[k]
            elif k not in _ENGINE_FLAGS:
                raise ValueError(f"unknown cuda engine option: {k}")
        s, keep = _lib.tape_struct(tape)
        o = _lib.options_struct(precision=int(options.precision), adjoints=options.adjoints, device=device,
                                flags=flags, **knobs)
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().nt_compile(ctypes.byref(s), ctypes.byref(o), ctypes.byref(h)))
        self._h = h
        self._closed = False
        self._device = device
        self._inputs = tape.recordedInputs()
        self._channels = tape.output_count() * (2 + tape.input_count())
        self._pps = 0.0
        # calibrate() grows its probes x8 until one takes a fifth of the budget;
        # at ~1e9 scenarios/s the reference's 2 s budget would spend about 2 s
        # on probes, while a chunk costs only one more launch here (the chunks
        # accumulate on the device), so the budget is 20 ms -- the Java
        # module's defaultMaxChunkSeconds() override.
        self._max_chunk_seconds = 0.02
        info = _lib.NtExecInfo()
        _lib.check(_lib.lib().nt_exec_info_get(self._h, ctypes.byref(info)))
        self._info = info.as_dict()

    # ---- AadExecutable ----
    def engineName(self) -> str:
        return "cuda"

    def tape(self) -> AadTape:
        return self._tape

    def compileSeconds(self) -> float:
        return self._info["compile_seconds"]

    def info(self) -> dict:
        info = _lib.NtExecInfo()
        _lib.check(_lib.lib().nt_exec_info_get(self._handle(), ctypes.byref(info)))
        return info.as_dict()

    def source(self) -> str:
        n = ctypes.c_size_t(0)
        _lib.check(_lib.lib().nt_exec_source(self._handle(), None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value + 1)
        _lib.check(_lib.lib().nt_exec_source(self._handle(), buf, n.value + 1, ctypes.byref(n)))
        return buf.value.decode()

    def _handle(self):
        if self._closed:
            raise RuntimeError("executable is closed")
        return self._h

    def setInput(self, name: str, value: float) -> None:
        """AbstractAadExecutable.setInput (AbstractAadExecutable.java:86-92)."""
        names = self._tape.input_names
        if name not in names:
            raise ValueError(f"unknown input: {name}")
        self._inputs[names.index(name)] = float(value)
        self._push_inputs()

    def setInputs(self, values: Sequence[float]) -> None:
        if len(values) != self._tape.input_count():
            raise ValueError(f"expected {self._tape.input_count()} inputs")
        self._inputs = np.asarray(values, dtype=np.float64).copy()
        self._push_inputs()

    def _push_inputs(self):
        x = np.ascontiguousarray(self._inputs, dtype=np.float64)
        _lib.check(_lib.lib().nt_set_inputs(self._handle(), _lib.ptr(x, ctypes.c_double), x.shape[0]))

    def replay_sums(self, paths: int, path_offset: int, seed: int):
        if paths <= 0:
            raise ValueError("paths must be positive")
        sums = np.zeros(self._channels, dtype=np.float64)
        secs = ctypes.c_double(0.0)
        _lib.check(_lib.lib().nt_replay(self._handle(), paths, path_offset & (2**64 - 1), seed & (2**64 - 1),
                                        _lib.ptr(sums, ctypes.c_double), ctypes.byref(secs)))
        return sums, secs.value

    def replay(self, paths: int, path_offset: int, seed: int) -> AadResult:
        """One dispatch over [path_offset, path_offset + paths) (AadExecutable.java:46-47)."""
        sums, secs = self.replay_sums(paths, path_offset, seed)
        return AadResult.from_sums(sums, self._tape, paths, secs)

    def _market_matrix(self, markets) -> np.ndarray:
        """Input vectors for nt_replay_markets: each market is a full input
        vector, or a dict of named inputs overriding the current inputs."""
        names = self._tape.input_names
        rows = []
        for m in markets:
            if isinstance(m, dict):
                row = np.asarray(self._inputs, dtype=np.float64).copy()
                for k, v in m.items():
                    if k not in names:
                        raise ValueError(f"unknown input: {k}")
                    row[names.index(k)] = float(v)
            else:
                row = np.asarray(m, dtype=np.float64)
                if row.shape != (len(names),):
                    raise ValueError(f"expected {len(names)} inputs per market")
            rows.append(row)
        if not rows:
            raise ValueError("at least one market is needed")
        return np.ascontiguousarray(np.stack(rows), dtype=np.float64)

    def replayMarkets_sums(self, markets, paths: int, path_offset: int, seed: int):
        if paths <= 0:
            raise ValueError("paths must be positive")
        x = self._market_matrix(markets)
        sums = np.zeros((x.shape[0], self._channels), dtype=np.float64)
        secs = ctypes.c_double(0.0)
        _lib.check(_lib.lib().nt_replay_markets(self._handle(), x.shape[0], _lib.ptr(x, ctypes.c_double), paths,
                                                path_offset & (2**64 - 1), seed & (2**64 - 1),
                                                _lib.ptr(sums, ctypes.c_double), ctypes.byref(secs)))
        return sums, secs.value

    def replayMarkets(self, markets, paths: int, path_offset: int, seed: int) -> List[AadResult]:
        """Re-prices under every market in one dispatch with common random
        numbers (nt_replay_markets): the per-market loop of
        ScenarioRunner.run (nablatensor-quant/.../scenario/ScenarioRunner.java:36-53)
        without a replay per market.  Each result equals replay() under that
        market's inputs with the same seed, up to the rounding of fused
        multiply-adds (1e-13 relative in fp64)."""
        sums, secs = self.replayMarkets_sums(markets, paths, path_offset, seed)
        return [AadResult.from_sums(s, self._tape, paths, secs) for s in sums]

    def ladder(self, name: str, values: Sequence[float], paths: int, path_offset: int, seed: int):
        """A 1-D ladder over one input, the others at their current values
        (ScenarioRunner.ladder, ScenarioRunner.java:58-71): returns
        (x, price, greek of `name`) arrays, all from one dispatch."""
        if name not in self._tape.input_names:
            raise ValueError(f"unknown input: {name}")
        x = [float(v) for v in values]
        res = self.replayMarkets([{name: v} for v in x], paths, path_offset, seed)
        price = np.array([r.value() for r in res])
        greek = np.array([r.gradient(name) for r in res])
        return np.array(x), price, greek

    def calibrate(self, seed: int) -> float:
        """AbstractAadExecutable.calibrate: probe dispatches growing x8."""
        paths = self.PROBE_PATHS
        for _ in range(12):
            _, secs = self.replay_sums(paths, 0, seed)
            self._observe(paths, secs)
            if secs >= self._max_chunk_seconds * 0.2:
                break
            nxt = self._budgeted_chunk()
            if nxt <= paths:
                break
            paths = min(nxt, paths * 8)
        return self._pps

    def replaySafe(self, total_paths: int, seed: int) -> AadResult:
        """Chunked replay (AbstractAadExecutable.java:101-121); the chunk sums
        accumulate on the device, exactly, and are read back once: the result
        has the same bits as replay(total_paths, 0, seed), whatever the chunk
        sizes the time budget picked."""
        if total_paths <= 0:
            raise ValueError("paths must be positive")
        if self._pps <= 0.0:
            self.calibrate(seed)
        t0 = time.perf_counter()
        h = self._handle()
        scratch = np.zeros(self._channels, dtype=np.float64)
        _lib.check(_lib.lib().nt_accumulator_read(h, _lib.ptr(scratch, ctypes.c_double), 1))
        done = 0
        while done < total_paths:
            chunk = min(self._budgeted_chunk(), total_paths - done)
            _lib.check(_lib.lib().nt_replay_accumulate(h, chunk, done, seed & (2**64 - 1)))
            done += chunk
        sums = np.zeros(self._channels, dtype=np.float64)
        _lib.check(_lib.lib().nt_accumulator_read(h, _lib.ptr(sums, ctypes.c_double), 1))
        secs = time.perf_counter() - t0
        self._observe(total_paths, secs)
        return AadResult.from_sums(sums, self._tape, total_paths, secs)

    def measuredPathsPerSecond(self) -> float:
        return self._pps

    def maxChunkSeconds(self) -> float:
        return self._max_chunk_seconds

    def setMaxChunkSeconds(self, seconds: float) -> None:
        if not seconds > 0.0:
            raise ValueError("maxChunkSeconds must be positive")
        self._max_chunk_seconds = float(seconds)

    def _observe(self, paths, secs):
        if secs <= 0.0:
            return
        sample = paths / secs
        self._pps = sample if self._pps <= 0.0 else 0.5 * (self._pps + sample)

    def _budgeted_chunk(self) -> int:
        """Paths per dispatch for the time budget: a whole number of 32-path
        warp tiles, so the chunked sums are the bits of one dispatch over the
        whole range."""
        if self._pps <= 0.0:
            return self.PROBE_PATHS
        return max(self.MIN_CHUNK_PATHS, int(self._pps * self._max_chunk_seconds) // 32 * 32)

    # ---- multi-GPU (scenario-range sharding + one NCCL all-reduce) ----
    def distAttach(self, nranks: int, rank: int, unique_id: bytes, timeout_ms: int = 60000) -> None:
        ident = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id.ljust(128, b"\0")[:128])
        _lib.check(_lib.lib().nt_dist_attach(self._handle(), nranks, rank, ident, timeout_ms))

    def distDetach(self) -> None:
        _lib.check(_lib.lib().nt_dist_detach(self._handle()))

    def replaySharded_sums(self, total_paths: int, path_offset: int, seed: int, chunk_paths: int = 0):
        if total_paths <= 0:
            raise ValueError("paths must be positive")
        sums = np.zeros(self._channels, dtype=np.float64)
        secs = ctypes.c_double(0.0)
        _lib.check(_lib.lib().nt_replay_sharded(self._handle(), total_paths, path_offset & (2**64 - 1),
                                                seed & (2**64 - 1), chunk_paths, _lib.ptr(sums, ctypes.c_double),
                                                ctypes.byref(secs)))
        return sums, secs.value

    def replaySharded(self, total_paths: int, path_offset: int, seed: int, chunk_paths: int = 0) -> AadResult:
        """This rank's shard of [path_offset, path_offset + total_paths) plus one
        all-reduce: every rank gets the global result, with the same bits as
        replay() of the whole range on one GPU."""
        sums, secs = self.replaySharded_sums(total_paths, path_offset, seed, chunk_paths)
        return AadResult.from_sums(sums, self._tape, total_paths, secs)

    def stream_handle(self) -> int:
        p = ctypes.c_void_p()
        _lib.check(_lib.lib().nt_exec_stream(self._handle(), ctypes.byref(p)))
        return int(p.value or 0)

    def close(self) -> None:
        if not self._closed:
            _lib.lib().nt_destroy(self._h)
            self._closed = True

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dist_unique_id() -> bytes:
    buf = (ctypes.c_uint8 * 128)()
    _lib.check(_lib.lib().nt_dist_unique_id(buf))
    return bytes(buf)


class CudaAadEngine(AadEngine):
    """Engine "cuda" on B200 (replaces nablatensor-engine-cuda's CudaAadEngine)."""

    def __init__(self, device: int = 0):
        self._device = device

    def name(self) -> str:
        return "cuda"

    def priority(self) -> int:
        return 110

    def isAvailable(self) -> bool:
        """Never raises (AadEngine.java:39-40)."""
        try:
            return _lib.device_count() > 0
        except Exception:
            return False

    def supports(self, options: AadOptions) -> bool:
        return options.precision in (PrecisionEnum.FLOAT32, PrecisionEnum.FLOAT64)

    def describe(self) -> str:
        return "B200 sm_100a · NVRTC tape kernels · fp32+fp64"

    def compile(self, tape: AadTape, options: AadOptions) -> B200AadExecutable:
        return B200AadExecutable(tape, options, self._device)


class AadEngines:
    """AadEngines.java:41-98: discovery and selection by name / priority."""

    _registry: List[AadEngine] = [CudaAadEngine()]

    @classmethod
    def discovered(cls) -> List[AadEngine]:
        return sorted(cls._registry, key=lambda e: -e.priority())

    @classmethod
    def find(cls, name: str) -> Optional[AadEngine]:
        for e in cls.discovered():
            if e.name() == name:
                return e
        return None

    @classmethod
    def require(cls, name: str, options: Optional[AadOptions] = None) -> AadEngine:
        e = cls.find(name)
        if e is None:
            raise ValueError(f"no AAD engine named '{name}'")
        if not e.isAvailable():
            raise RuntimeError(f"engine '{name}' is not available on this machine")
        if options is not None and not e.supports(options):
            raise NotImplementedError(f"engine '{name}' does not support {options}")
        return e
