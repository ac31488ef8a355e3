"""The package's recorder reproduces the reference's node order.

The Python tape producers (nablatensor_b200.quant) and the oracle's C
builders (oracle/nt_oracle.c) restate the same Java recording independently;
they must agree node for node.
"""
import numpy as np
import pytest

from nablatensor_b200 import quant
from nablatensor_b200.tape import AadOpEnum, AadRecorder


def _same(py, orc):
    np.testing.assert_array_equal(py.op, orc.op)
    np.testing.assert_array_equal(py.arg_a, orc.arg_a)
    np.testing.assert_array_equal(py.arg_b, orc.arg_b)
    np.testing.assert_array_equal(py.constant.view(np.uint64), orc.constant.view(np.uint64))
    np.testing.assert_array_equal(py.input_node, orc.input_node)
    np.testing.assert_array_equal(py.output_node, orc.output_node)
    np.testing.assert_array_equal(py.active, orc.active())


@pytest.mark.parametrize("steps", [1, 2, 31, 64, 252])
def test_asian_matches_oracle_builder(oracle_mod, steps):
    _same(quant.asian_tape(steps), oracle_mod.asian_tape(steps))


@pytest.mark.parametrize("steps", [1, 7, 252])
def test_european_matches_oracle_builder(oracle_mod, steps):
    _same(quant.european_tape(steps), oracle_mod.european_tape(steps))


@pytest.mark.parametrize("kind", list(quant.Barrier))
def test_barrier_matches_oracle_builder(oracle_mod, kind):
    _same(quant.barrier_tape(40, 80.0, 1.0, kind), oracle_mod.barrier_tape(40, True, kind.name, 80.0, 1.0))


def test_barrier_config_tape_has_4057_nodes():
    t = quant.barrier_tape(252, 80.0, 1.0, quant.Barrier.DOWN_IN)
    assert t.size() == 4057
    assert t.input_names == ["spot", "strike", "vol", "rate", "maturity"]


def test_recorder_rules():
    def body(rec):
        x = rec.input("x", 2.0)
        rec.output("a", x.mul(3.0))
        with pytest.raises(ValueError):
            rec.output("a", x)
        s = rec.stream("s1")
        s.randn()
        s.randu()
        rec.randn()
        with pytest.raises(ValueError):
            rec.stream("  ")
    t = AadRecorder.record(body)
    assert t.output_names == ["a"]
    assert t.stream_names == ["default", "s1"]
    assert list(t.normal_count) == [1, 1] and list(t.uniform_count) == [0, 1]
    assert t.hasExtendedRandom()
    with pytest.raises(RuntimeError):
        AadRecorder.record(lambda rec: rec.input("x", 1.0))


def test_active_marking_follows_inputs():
    def body(rec):
        x = rec.input("x", 1.0)
        c = rec.constant(2.0).mul(rec.randn())
        rec.output(x.add(c))
    t = AadRecorder.record(body)
    assert list(t.active) == [True, False, False, False, True]
    assert t.op[2] == AadOpEnum.RANDN
