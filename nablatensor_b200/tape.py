"""Recording: AadRecorder / ADouble / AadTape.

Mirrors the reference's recording API (nablatensor-core/src/main/java/com/
nablatensor/engine/AadRecorder.java:41-122, ADouble.java, AadTape.java):
every ADouble operation appends one node in evaluation order, so a product
recorded here yields the same node sequence as the Java recorder, and the
flat arrays are exactly what the C ABI (``nt_tape``) consumes.
"""
from __future__ import annotations

from enum import IntEnum
from typing import Callable, List, Optional

import numpy as np


class AadOpEnum(IntEnum):
    """Ordinal order of AadOpEnum.java:19-50."""
    CONST = 0
    INPUT = 1
    RANDN = 2
    RANDU = 3
    ADD = 4
    SUB = 5
    MUL = 6
    DIV = 7
    NEG = 8
    EXP = 9
    LOG = 10
    SQRT = 11
    MAX = 12
    MIN = 13
    ABS = 14


_UNARY = {AadOpEnum.NEG, AadOpEnum.EXP, AadOpEnum.LOG, AadOpEnum.SQRT, AadOpEnum.ABS}


class AadTape:
    """A recorded tape as flat arrays (FlatTape.java:37-79 + AadTape.java)."""

    def __init__(self, op, arg_a, arg_b, constant, input_node, input_names, recorded_inputs,
                 stream_names, normal_count, uniform_count, output_node, output_names):
        self.op = np.asarray(op, dtype=np.int32)
        self.arg_a = np.asarray(arg_a, dtype=np.int32)
        self.arg_b = np.asarray(arg_b, dtype=np.int32)
        self.constant = np.asarray(constant, dtype=np.float64)
        self.input_node = np.asarray(input_node, dtype=np.int32)
        self.input_names: List[str] = list(input_names)
        self.recorded_inputs = np.asarray(recorded_inputs, dtype=np.float64)
        self.stream_names: List[str] = list(stream_names)
        self.normal_count = np.asarray(normal_count, dtype=np.int32)
        self.uniform_count = np.asarray(uniform_count, dtype=np.int32)
        self.output_node = np.asarray(output_node, dtype=np.int32)
        self.output_names: List[str] = list(output_names)
        self.active = self._mark_active()

    def _mark_active(self) -> np.ndarray:
        """AadTape.markActive (AadTape.java:70-81)."""
        n = self.size()
        flags = np.zeros(n, dtype=bool)
        op, a, b = self.op, self.arg_a, self.arg_b
        for i in range(n):
            o = op[i]
            if o == AadOpEnum.INPUT:
                flags[i] = True
            elif o in (AadOpEnum.CONST, AadOpEnum.RANDN, AadOpEnum.RANDU):
                flags[i] = False
            elif o in _UNARY:
                flags[i] = flags[a[i]]
            else:
                flags[i] = flags[a[i]] or flags[b[i]]
        return flags

    # ---- AadTape accessors ----
    def size(self) -> int:
        return int(self.op.shape[0])

    @property
    def n(self) -> int:
        return self.size()

    @property
    def n_streams(self) -> int:
        return len(self.stream_names)

    def input_count(self) -> int:
        return len(self.input_names)

    def output_count(self) -> int:
        return len(self.output_names)

    def inputNames(self) -> List[str]:
        return list(self.input_names)

    def outputNames(self) -> List[str]:
        return list(self.output_names)

    def recordedInputs(self) -> np.ndarray:
        return self.recorded_inputs.copy()

    def randCount(self) -> int:
        return int(self.normal_count[0])

    def hasExtendedRandom(self) -> bool:
        """AadTape.hasExtendedRandom: more than one stream, or any uniform."""
        return self.n_streams > 1 or int(self.uniform_count[0]) > 0

    def active_count(self) -> int:
        return int(self.active.sum())

    def op_histogram(self) -> dict:
        vals, counts = np.unique(self.op, return_counts=True)
        return {AadOpEnum(int(v)).name: int(c) for v, c in zip(vals, counts)}

    def __repr__(self) -> str:
        return f"AadTape(nodes={self.size()}, inputs={self.input_names}, randoms={self.randCount()})"


class ADouble:
    """A recorded scalar (ADouble.java).  Operators record like the methods."""

    __slots__ = ("_rec", "node")

    def __init__(self, rec: "AadRecorder", node: int):
        self._rec = rec
        self.node = node

    def _bin(self, op: AadOpEnum, other) -> "ADouble":
        if not isinstance(other, ADouble):
            other = self._rec.constant(float(other))
        if other._rec is not self._rec:
            raise ValueError("operands come from different recordings")
        return self._rec._node(op, self.node, other.node)

    def _un(self, op: AadOpEnum) -> "ADouble":
        return self._rec._node(op, self.node, -1)

    def add(self, o): return self._bin(AadOpEnum.ADD, o)
    def sub(self, o): return self._bin(AadOpEnum.SUB, o)
    def mul(self, o): return self._bin(AadOpEnum.MUL, o)
    def div(self, o): return self._bin(AadOpEnum.DIV, o)
    def max(self, o): return self._bin(AadOpEnum.MAX, o)
    def min(self, o): return self._bin(AadOpEnum.MIN, o)
    def neg(self): return self._un(AadOpEnum.NEG)
    def exp(self): return self._un(AadOpEnum.EXP)
    def log(self): return self._un(AadOpEnum.LOG)
    def sqrt(self): return self._un(AadOpEnum.SQRT)
    def abs(self): return self._un(AadOpEnum.ABS)

    __add__ = add
    __sub__ = sub
    __mul__ = mul
    __truediv__ = div
    __neg__ = neg
    __abs__ = abs

    def __radd__(self, o): return self._rec.constant(float(o)).add(self)
    def __rsub__(self, o): return self._rec.constant(float(o)).sub(self)
    def __rmul__(self, o): return self._rec.constant(float(o)).mul(self)
    def __rtruediv__(self, o): return self._rec.constant(float(o)).div(self)


class RandomStream:
    """A named random stream (AadRecorder.RandomStream)."""

    def __init__(self, rec: "AadRecorder", name: str):
        self._rec = rec
        self.name = name

    def randn(self) -> ADouble:
        return self._rec._draw(AadOpEnum.RANDN, self.name)

    def randu(self) -> ADouble:
        return self._rec._draw(AadOpEnum.RANDU, self.name)


class AadRecorder:
    """AadRecorder.record(body) -> AadTape (AadRecorder.java:41-45)."""

    def __init__(self):
        self._op: List[int] = []
        self._a: List[int] = []
        self._b: List[int] = []
        self._c: List[float] = []
        self._inputs: List[int] = []
        self._input_names: List[str] = []
        self._input_values: List[float] = []
        self._streams: List[str] = ["default"]
        self._counts: List[List[int]] = [[0, 0]]
        self._outputs: List[int] = []
        self._output_names: List[str] = []

    @staticmethod
    def record(body: Callable[["AadRecorder"], None]) -> AadTape:
        rec = AadRecorder()
        body(rec)
        return rec.build()

    def _add(self, op: int, a: int, b: int, c: float) -> int:
        self._op.append(int(op))
        self._a.append(int(a))
        self._b.append(int(b))
        self._c.append(float(c))
        return len(self._op) - 1

    def _node(self, op: AadOpEnum, a: int, b: int) -> ADouble:
        return ADouble(self, self._add(op, a, b, 0.0))

    def _stream_index(self, name: str) -> int:
        if name in self._streams:
            return self._streams.index(name)
        self._streams.append(name)
        self._counts.append([0, 0])
        return len(self._streams) - 1

    def _draw(self, op: AadOpEnum, stream: str) -> ADouble:
        si = self._stream_index(stream)
        kind = 0 if op == AadOpEnum.RANDN else 1
        ordinal = self._counts[si][kind]
        self._counts[si][kind] += 1
        return ADouble(self, self._add(op, ordinal, si, 0.0))

    def input(self, name: str, value: float) -> ADouble:
        node = self._add(AadOpEnum.INPUT, len(self._inputs), -1, float(value))
        self._inputs.append(node)
        self._input_names.append(name)
        self._input_values.append(float(value))
        return ADouble(self, node)

    def constant(self, value: float) -> ADouble:
        return ADouble(self, self._add(AadOpEnum.CONST, -1, -1, float(value)))

    def randn(self) -> ADouble:
        return self._draw(AadOpEnum.RANDN, "default")

    def randu(self) -> ADouble:
        return self._draw(AadOpEnum.RANDU, "default")

    def stream(self, name: str) -> RandomStream:
        if not name or not name.strip():
            raise ValueError("stream name must be non-blank")
        return RandomStream(self, name)

    def output(self, name_or_value, value: Optional[ADouble] = None) -> None:
        if value is None:
            name, value = "value", name_or_value
        else:
            name = name_or_value
        if name in self._output_names:
            raise ValueError(f"output '{name}' recorded twice")
        self._output_names.append(name)
        self._outputs.append(value.node)

    def build(self) -> AadTape:
        if not self._outputs:
            raise RuntimeError("no output was recorded")
        return AadTape(self._op, self._a, self._b, self._c, self._inputs, self._input_names, self._input_values,
                       self._streams, [c[0] for c in self._counts], [c[1] for c in self._counts],
                       self._outputs, self._output_names)


__all__ = ["AadOpEnum", "AadTape", "ADouble", "AadRecorder", "RandomStream"]
