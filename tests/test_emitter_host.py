"""The emitter's scenario code, compiled for the host, against the oracle.

nt_emit_source(target=1) emits exactly the per-scenario code the CUDA kernel
runs (loop detection, step-wise checkpoints, segment recompute, reverse
sweep), wrapped in a sequential host loop.  Built with g++ without FMA
contraction and linked against the same libm as the oracle, it must
reproduce the oracle's sums BIT FOR BIT: any mistake in the loop plan, the
checkpoint slots, the recompute set or the adjoint order shows up as a
difference.  (Two carries fed by the same initial node accumulate that
node's adjoint in a different order than the interpreter; those tapes are
compared at 1e-14.)
"""
import numpy as np
import pytest

from nablatensor_b200 import _lib, quant
from oracle.oracle import FlatTape

from conftest import host_kernel
from tapes import (every_op_tape, fp32_asian_50, lookback, multi_output, named_streams, nonuniform_asian,
                   odd_steps_asian, pow2_divisions, random_branching, term_vol_asian)

ATM = [100.0, 100.0, 0.20, 0.03, 1.0]


def _run(oracle_mod, tape, inputs, paths, off, seed, rtol=0.0, f32=False, adjoints=True, **opts):
    src = _lib.emit_source(tape, target=1, precision=0 if f32 else 1, adjoints=adjoints, **opts)
    run = host_kernel(src)
    channels = tape.output_count() * (2 + tape.input_count())
    got = run(inputs, paths, off, seed, channels)
    want = oracle_mod.replay(FlatTape.of(tape), inputs, paths, off, seed, f32=f32, adjoints=adjoints,
                             threads=1).sums
    if not adjoints:
        stride = 2 + tape.input_count()
        keep = [o * stride + k for o in range(tape.output_count()) for k in (0, 1)]
        got, want = got[keep], want[keep]
    if rtol == 0.0:
        np.testing.assert_array_equal(got, want)
    else:
        np.testing.assert_allclose(got, want, rtol=rtol, atol=0)
    return src


@pytest.mark.parametrize("seg_units", [0, 1, 2, 3, 6, 7, 9, 14, 63])
def test_asian_loop_is_bit_exact(oracle_mod, seg_units):
    src = _run(oracle_mod, quant.asian_tape(252), ATM, 3_000, 0x1_0000_0003, 0x1234_5678_FEDC_BA98,
               seg_units=seg_units)
    assert "step loop: 126 units" in src


@pytest.mark.parametrize("flags,slots", [(0, 2), (_lib.NT_FLAG_TAPE_ALL, 4), (_lib.NT_FLAG_TAPE_DRAWS, 2),
                                         (_lib.NT_FLAG_RECOMPUTE_ALL, 0)])
def test_tape_plans_are_bit_exact(oracle_mod, flags, slots):
    """Every reverse-sweep storage plan reproduces the oracle: by default the
    normals are taped and the GBM exps (draws and invariants only) are
    recomputed; the barrier's smoothing exps, which read the spot carry, stay
    taped."""
    src = _run(oracle_mod, quant.asian_tape(252), ATM, 1_500, 3, 42, flags=flags)
    assert f"#define NT_NTAPE {max(1, slots)}" in src
    bsrc = _run(oracle_mod, quant.barrier_tape(60), ATM, 1_000, 3, 42, flags=flags)
    if flags == 0:
        assert "#define NT_NTAPE 6" in bsrc  # 2 normals + 2 x 2 smoothing exps per unit


def test_asian_straight_line_is_bit_exact(oracle_mod):
    src = _run(oracle_mod, quant.asian_tape(64), ATM, 2_000, 7, 42, flags=_lib.NT_FLAG_NO_LOOP)
    assert "step loop" not in src


@pytest.mark.parametrize("steps", [3, 4, 5, 31, 64])
def test_asian_odd_and_short_loops(oracle_mod, steps):
    _run(oracle_mod, odd_steps_asian(steps), ATM, 2_000, 11, 99)


def test_asian_bumped_inputs(oracle_mod):
    _run(oracle_mod, quant.asian_tape(252), [101.0, 97.0, 0.31, 0.01, 2.0], 1_000, 0, 42)


@pytest.mark.parametrize("steps", [1, 252])
def test_european(oracle_mod, steps):
    _run(oracle_mod, quant.european_tape(steps), ATM, 5_000, 0, 20260830)


@pytest.mark.parametrize("kind", list(quant.Barrier))
def test_barrier_kinds(oracle_mod, kind):
    _run(oracle_mod, quant.barrier_tape(60, 80.0 if "DOWN" in kind.name else 120.0, 1.0, kind), ATM, 2_000, 3, 42)


def test_barrier_config_tape(oracle_mod):
    _run(oracle_mod, quant.barrier_tape(252), ATM, 1_000, 0, 42)


def test_lookback_max_min_rules(oracle_mod):
    _run(oracle_mod, lookback(64, True), ATM, 2_000, 0, 5, rtol=1e-14)
    _run(oracle_mod, lookback(64, False), ATM, 2_000, 0, 5, rtol=1e-14)


def test_random_branching_tape(oracle_mod):
    _run(oracle_mod, random_branching(24), [1.2, 0.1], 4_000, 0x1_0000_0003, 42)
    _run(oracle_mod, random_branching(24), [1.5, 0.1], 4_000, 0x1_0000_0003, 0x1234_5678_FEDC_BA98)


def test_every_op_tape(oracle_mod):
    _run(oracle_mod, every_op_tape(), [1.3, 0.7], 20_000, 0, 0x5EED5)


def test_named_streams_and_uniforms(oracle_mod):
    _run(oracle_mod, named_streams(16), [100.0, 0.2], 5_000, 0, 0xC0FFEE)


def test_multi_output(oracle_mod):
    _run(oracle_mod, multi_output(40), [100.0, 0.25], 3_000, 0, 17)


def test_price_only(oracle_mod):
    _run(oracle_mod, quant.asian_tape(252), ATM, 1_000, 0, 42, adjoints=False)


@pytest.mark.parametrize("make,inputs", [
    (lambda: fp32_asian_50(50), [100.0, 0.2]),
    (every_op_tape, [1.3, 0.7]),
    (lambda: random_branching(24), [1.2, 0.1]),
    (lambda: lookback(64, True), ATM),
    (lambda: named_streams(16), [100.0, 0.2]),
])
def test_fp32_host_build_is_bit_exact(oracle_mod, make, inputs):
    """fp32 host builds against the oracle's fp32 mode, bit for bit: every
    node rounded to float on its own, transcendentals in double and narrowed,
    each adjoint partial formed as the interpreter forms it (a divisor's
    d z / b in double, rounded once)."""
    _run(oracle_mod, make(), inputs, 3_000, 0x1_0000_0003, 0xA51A17, f32=True)


def test_fp32_reciprocal_adjoint_within_an_ulp_of_the_oracle(oracle_mod):
    """The one fp32 partial formed differently: the adjoint of z = 1 / b is
    -d z z (two float products) where the interpreter forms -d z / b in
    double; the barrier's sums stay within 1e-7 of the fp32 oracle's."""
    _run(oracle_mod, quant.barrier_tape(252), ATM, 3_000, 0x1_0000_0003, 42, rtol=1e-7, f32=True)


@pytest.mark.parametrize("n,steps", [(3, 8), (4, 5)])
def test_correlated_basket(oracle_mod, n, steps):
    """Benchmark configuration 4's shape (Cholesky mix of n normals per step, n GBM
    assets, 2n + 1 inputs) at a size the host runs quickly."""
    tape = quant.basket_tape(n=n, steps=steps)
    _run(oracle_mod, tape, tape.recordedInputs(), 2_000, 5, 7)


@pytest.mark.parametrize("steps", [60, 61])
def test_loop_with_per_unit_constants(oracle_mod, steps):
    """A non-uniform time grid: the steps repeat with different dt constants,
    which the loop reads from its per-unit constant table."""
    tape = nonuniform_asian(steps)
    src = _run(oracle_mod, tape, [100.0, 100.0, 0.2, 0.03], 2_000, 9, 42)
    assert "step loop" in src and "#define NT_NVARY" in src
    dev = _lib.emit_source(tape, target=0, precision=1)
    # read-only loads on the device: an even row length loads aligned pairs
    assert "nt_ctab" in dev and ("__ldg(&nt_ctab" in dev or "__ldg(&reinterpret_cast<const double2*>(nt_ctab)" in dev)


@pytest.mark.parametrize("steps", [24, 25])
def test_loop_with_gathered_inputs(oracle_mod, steps):
    """A volatility per step: each unit reads its own input and its own drift
    node from before the loop, and their adjoints flow back to those nodes."""
    tape = term_vol_asian(steps)
    src = _run(oracle_mod, tape, tape.recordedInputs(), 2_000, 9, 42)
    assert "step loop" in src and "nt_gv0" in src and "nt_gd0" in src


def test_cva_book_is_bit_exact(oracle_mod):
    """Benchmark configuration 5's shape at a size the host runs quickly: 24 monthly
    dates over two years, 10 swaps; the per-date constants (live coupons,
    bond coefficients, curve weights) vary from unit to unit."""
    book = quant.SwapBook.config5(n=10)
    tape = quant.cva_tape(dates=24, horizon=2.0, book=book)
    src = _run(oracle_mod, tape, tape.recordedInputs(), 500, 3, 11)
    assert "step loop: 12 units" in src and "#define NT_NVARY" in src


@pytest.mark.parametrize("flags", [0, _lib.NT_FLAG_RECOMPUTE_ALL])
def test_cva_config5_carries_the_second_leg(oracle_mod, flags):
    """The full config-5 tape: one long unit per monthly date drawing one
    normal, so an even unit draws the Box-Muller pair and the next unit takes
    the kept second leg (recompute-all regenerates single draws instead)."""
    tape = quant.cva_tape()
    src = _run(oracle_mod, tape, tape.recordedInputs(), 40, 0x1_0000_0003, 11, flags=flags)
    assert "units of 224 nodes (1 steps each)" in src and "nt_hl" in src


def test_loop_plan_reported_for_config_tapes(ntlib):
    src = _lib.emit_source(quant.barrier_tape(252), target=0, precision=0)
    assert "step loop: 126 units of 32 nodes (2 steps each)" in src
    assert "nt_normal_pair32" in src


@pytest.mark.parametrize("f32", [False, True])
def test_power_of_two_divisions_become_exact_multiplications(oracle_mod, f32):
    """Division by a constant power of two is emitted as multiplication by
    the reciprocal, with bit-identical results (forward and adjoint); a
    shared constant and a non-power of two stay divisions.  Per step the tape
    has 7 divisions; 5 are by an unshared power of two (2, 0.5, 1, -4, tiny)."""
    steps = 24
    tape = pow2_divisions(steps, tiny=2.0 ** -100 if f32 else 2.0 ** -1000)
    assert sum(1 for op in tape.op if op == 7) == 7 * steps
    _run(oracle_mod, tape, [1.5, 0.3], 2_000, 7, 42, f32=f32)
    src = _run(oracle_mod, tape, [1.5, 0.3], 500, 7, 42, f32=f32, flags=_lib.NT_FLAG_NO_LOOP)
    # straight-line code: the 2 kept divisions per step, and their d/vb rules
    assert sum(line.count(" / ") for line in src.splitlines()) == 4 * steps


def test_power_of_two_constant_shared_by_divisions_and_kept_when_used_otherwise(oracle_mod):
    """A constant 4 that only divides (twice) is rewritten once for both
    divisions; a constant 8 that divides and is also an output stays a
    division; 2^1023 (reciprocal subnormal) stays a division."""
    from nablatensor_b200.tape import AadRecorder

    def body(rec):
        s = rec.input("s", 1.5)
        four = rec.constant(4.0)
        eight = rec.constant(8.0)
        big = rec.constant(2.0 ** 1023)
        z = rec.randn()
        y = s.div(four).add(z.div(four)).add(s.div(eight)).add(s.div(big).mul(2.0 ** 1000))
        rec.output("y", y)
        rec.output("eight", eight)
    tape = AadRecorder.record(body)
    src = _run(oracle_mod, tape, [1.5], 1_000, 3, 42, flags=_lib.NT_FLAG_NO_LOOP)
    fwd = [line for line in src.splitlines() if "const real v" in line and " / " in line]
    assert len(fwd) == 2  # s / 8 and s / 2^1023; both divisions by 4 became multiplications
