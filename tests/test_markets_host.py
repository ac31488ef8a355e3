"""Several markets in one dispatch (nt_replay_markets), host build.

The multi-market emission (nt_emit_source target 3) replays every scenario
under each market in turn: the first market draws the step loop's normals
into the value tape, the others read them back.  Built for the host like
test_emitter_host.py, each market's sums must equal the oracle's replay under
that market's inputs BIT FOR BIT -- so the reused draws are exactly the draws,
and nothing of one market leaks into the next (carries, checkpoints, tape
values, accumulators).  Covers tapes whose draws are taped (Asian, barrier,
basket), straight-line tapes (draws regenerated per market), recompute-all
(no tape) and named streams with uniforms.
"""
import numpy as np
import pytest

from nablatensor_b200 import _lib, quant
from oracle.oracle import FlatTape

from conftest import host_kernel
from tapes import every_op_tape, named_streams, nonuniform_asian, term_vol_asian

ATM = [100.0, 100.0, 0.20, 0.03, 1.0]


def _markets(base, shifts):
    out = []
    for k, (j, f) in enumerate(shifts):
        x = list(base)
        x[j] *= f
        out.append(x)
    return out


def _check(oracle_mod, tape, markets, paths, off, seed, **opts):
    src = _lib.emit_source(tape, target=3, precision=1, **opts)
    run = host_kernel(src, markets=True)
    channels = tape.output_count() * (2 + tape.input_count())
    got = run(markets, paths, off, seed, channels)
    flat = FlatTape.of(tape)
    for m, x in enumerate(markets):
        want = oracle_mod.replay(flat, x, paths, off, seed, threads=1).sums
        np.testing.assert_array_equal(got[m], want, err_msg=f"market {m}")
    return src


def test_asian_ladder_reuses_the_draws(oracle_mod):
    mk = _markets(ATM, [(0, 1.0), (0, 0.9), (0, 1.1), (2, 1.5), (3, 0.5), (4, 2.0)])
    src = _check(oracle_mod, quant.asian_tape(252), mk, 1_500, 0x1_0000_0003, 42)
    assert "if (nt_m == 0)" in src and "nt_normal_pair64" in src


@pytest.mark.parametrize("flags", [0, _lib.NT_FLAG_TAPE_DRAWS, _lib.NT_FLAG_TAPE_ALL, _lib.NT_FLAG_RECOMPUTE_ALL,
                                   _lib.NT_FLAG_NO_LOOP])
def test_plan_variants(oracle_mod, flags):
    mk = _markets(ATM, [(0, 1.0), (1, 1.05), (2, 0.8)])
    _check(oracle_mod, quant.asian_tape(64), mk, 1_000, 7, 99, flags=flags)


def test_barrier_markets(oracle_mod):
    mk = _markets(ATM, [(0, 1.0), (0, 0.85), (2, 1.25)])
    _check(oracle_mod, quant.barrier_tape(60), mk, 1_000, 3, 42)


def test_basket_markets(oracle_mod):
    tape = quant.basket_tape(n=3, steps=6)
    base = list(tape.recordedInputs())
    mk = _markets(base, [(0, 1.0), (1, 1.1), (4, 0.7)])
    _check(oracle_mod, tape, mk, 800, 5, 7)


def test_straight_line_and_streams(oracle_mod):
    _check(oracle_mod, every_op_tape(), [[1.3, 0.7], [1.1, 0.9], [2.0, 0.3]], 3_000, 0, 0x5EED5)
    _check(oracle_mod, named_streams(16), [[100.0, 0.2], [95.0, 0.3]], 2_000, 0, 0xC0FFEE)


def test_one_market_is_the_plain_replay(oracle_mod):
    _check(oracle_mod, quant.asian_tape(252), [ATM], 1_000, 0, 42)


def test_per_unit_constants_and_gathered_inputs(oracle_mod):
    """Loops whose units read a per-unit constant table or a node before the
    loop chosen by the unit: each market gathers its own values."""
    t = nonuniform_asian()
    _check(oracle_mod, t, _markets(list(t.recordedInputs()), [(0, 1.0), (2, 1.3)]), 800, 3, 42)
    t = term_vol_asian()
    base = list(t.recordedInputs())
    _check(oracle_mod, t, _markets(base, [(0, 1.0), (3, 1.5), (len(base) - 1, 0.7)]), 800, 5, 42)


def test_cva_book_markets(oracle_mod):
    """A small CVA book (24 monthly dates, 10 swaps) under a parallel and a
    single-pillar curve bump and a hazard bump."""
    t = quant.cva_tape(dates=24, horizon=2.0, book=quant.SwapBook.config5(n=10))
    base = list(t.recordedInputs())
    par = [x + 0.001 for x in base[:-1]] + [base[-1]]
    mk = [base, par] + _markets(base, [(5, 1.1), (len(base) - 1, 1.5)])
    _check(oracle_mod, t, mk, 300, 3, 11)
