"""Accuracy of the replay's dedicated fp64 routines as compiled for sm_100a.

nt_math_eval runs each routine on the device over given inputs; the results
are compared here with x87 long-double evaluations (64-bit significand) of
the same mathematics on the host.  The inputs are random generator words and
arguments plus the edge words of tests/test_device_math.py.  The bounds:
  -2 ln(u1)              2 ulp
  sin, cos of fl(2 pi u2) 2 ulp, with a floor of 2^-53 absolute (the
                         reference's own rounding of the angle dominates there)
  radius sqrt            1 ulp
  series exp, |x| <= 1/8 1 ulp
  full-range exp         1 ulp (and exact 0 / inf beyond the range)
  Box-Muller legs        3 ulp of the leg, floor 2^-52 absolute
"""
import numpy as np
import pytest

from nablatensor_b200 import _lib

pytestmark = pytest.mark.gpu

EDGES = np.array([0, 1, 2, 0x7fffffff, 0x80000000, 0xffffffff, 0xfffffffe, 0x3fffffff, 0x40000000, 0xbfffffff,
                  0xc0000000, 0x6a09e667, 0xb504f333, 0xb504f334, 0x20000000, 0x60000000, 0xa0000000, 0xe0000000,
                  0x00ffffff, 0x01000000, 0xfeffffff, 0xff000000, 0x7f7fffff, 0x80800000, 0x5fffffff, 0x9fffffff],
                 dtype=np.uint32)
LD = np.longdouble
TWO_PI = np.float64(6.283185307179586)


def _words(n, seed):
    rng = np.random.default_rng(seed)
    return np.concatenate([EDGES, rng.integers(0, 2 ** 32, size=n, dtype=np.uint64).astype(np.uint32)])


def _u(w):
    return (w.astype(np.float64) + 0.5) * 2.0 ** -32  # exact in double


def _ulps(got, want, floor=0.0):
    ref = np.asarray(want, dtype=np.float64)
    ulp = np.maximum(np.spacing(np.abs(ref)), floor)
    return np.abs(got.astype(LD) - want) / ulp


@pytest.fixture(scope="module")
def dev(ntlib):
    assert _lib.device_count() > 0, "these tests need a B200"
    return 0


def test_neg2log_u1(dev):
    w = _words(2_000_000, 1)
    got = _lib.math_eval(dev, 0, words=w)
    want = -2.0 * np.log(_u(w).astype(LD))
    assert np.max(_ulps(got, want)) <= 2.0


def test_sincos_of_the_reference_angle(dev):
    w = _words(2_000_000, 2)
    s, c = _lib.math_eval(dev, 1, words=w)
    th = (TWO_PI * _u(w)).astype(LD)  # the reference's angle, rounded to double
    assert np.max(_ulps(s, np.sin(th), 2.0 ** -53)) <= 2.0
    assert np.max(_ulps(c, np.cos(th), 2.0 ** -53)) <= 2.0


def test_radius_sqrt(dev):
    rng = np.random.default_rng(3)
    x = np.concatenate([[2.0 ** -33 * 2, 1e-9, 0.5, 1.0, 2.0, 46.0, 46.05],
                        -2.0 * np.log(_u(_words(1_000_000, 3))),
                        rng.uniform(1e-6, 50.0, 1_000_000)])
    x = x[x > 0]
    got = _lib.math_eval(dev, 2, x=x)
    assert np.max(_ulps(got, np.sqrt(x.astype(LD)))) <= 1.0


def test_series_exp(dev):
    rng = np.random.default_rng(4)
    x = np.concatenate([[0.0, -0.0, 0.125, -0.125, 2.0 ** -60, -2.0 ** -60],
                        rng.uniform(-0.125, 0.125, 2_000_000)])
    got = _lib.math_eval(dev, 3, x=x)
    assert np.max(_ulps(got, np.exp(x.astype(LD)))) <= 1.0


def test_full_range_exp(dev):
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.uniform(-745.0, 709.78, 1_000_000), rng.uniform(-1.0, 1.0, 500_000),
                        np.ldexp(1.0, rng.integers(-60, 10, 500_000)) * rng.choice([-1.0, 1.0], 500_000)])
    got = _lib.math_eval(dev, 4, x=x)
    want = np.exp(x.astype(LD))
    wd = want.astype(np.float64)
    nonzero = wd != 0.0
    assert np.max(_ulps(got[nonzero], want[nonzero], 2.0 ** -1074)) <= 1.0
    assert np.all(got[~nonzero] == 0.0)
    special = np.array([710.0, 1e300, -746.0, -1e300, np.inf, -np.inf, np.nan])
    s = _lib.math_eval(dev, 4, x=special)
    assert np.isinf(s[0]) and np.isinf(s[1]) and s[2] == 0.0 and s[3] == 0.0
    assert np.isinf(s[4]) and s[5] == 0.0 and np.isnan(s[6])


def test_first_pass_exp_of_taped_values(dev):
    """The forward loop's first-pass exp of a taped value (which 7) gives the
    full-range routine's bits wherever it does not flag the argument
    (|x| <= 700), and flags every other argument, NaN and infinities included,
    so that the warp's redo pass evaluates it with the full-range routine."""
    rng = np.random.default_rng(8)
    x = np.concatenate([rng.uniform(-700.0, 700.0, 1_000_000), rng.uniform(-1.0, 1.0, 500_000),
                        np.array([700.0, -700.0, 0.0, -0.0, 1e-300, -1e-300])])
    got, wide = _lib.math_eval(dev, 7, x=x)
    full = _lib.math_eval(dev, 4, x=x)
    assert np.all(wide == 0.0)
    assert np.array_equal(got.view(np.uint64), full.view(np.uint64))
    out = np.array([700.5, -700.5, 710.0, -746.0, 1e300, -1e300, np.inf, -np.inf, np.nan])
    _, wide = _lib.math_eval(dev, 7, x=out)
    assert np.all(wide == 1.0)


def test_box_muller_legs(dev):
    w = _words(2_000_000, 6)
    w = w[: len(w) // 2 * 2]
    c, s = _lib.math_eval(dev, 5, words=w)
    u1, u2 = _u(w[0::2]), _u(w[1::2])
    r = np.sqrt(-2.0 * np.log(u1.astype(LD)))
    th = (TWO_PI * u2).astype(LD)
    assert np.max(_ulps(c, r * np.cos(th), 2.0 ** -52)) <= 3.0
    assert np.max(_ulps(s, r * np.sin(th), 2.0 ** -52)) <= 3.0


def test_float_result_box_muller_legs(dev):
    """The fp32 tapes' Box-Muller (which 6) against the fp64 legs narrowed to
    float: the same float except where the double value lies within about
    2^-40 of a float rounding boundary, and never more than one float ulp
    away; both within one float ulp of the long-double legs."""
    w = _words(2_000_000, 7)
    w = w[: len(w) // 2 * 2]
    c64, s64 = _lib.math_eval(dev, 5, words=w)
    c32, s32 = _lib.math_eval(dev, 6, words=w)
    for got, want in ((c32, c64), (s32, s64)):
        narrowed = want.astype(np.float32)
        assert np.all(got == got.astype(np.float32))  # a float, widened
        diff = got.astype(np.float32) != narrowed
        print(f"float-result legs differing from the narrowed fp64 legs: {int(diff.sum())} of {len(got)}")
        assert diff.sum() <= len(got) * 2.0 ** -12
        gap = np.abs(got[diff] - narrowed[diff].astype(np.float64))
        assert np.all(gap <= np.spacing(np.abs(narrowed[diff])).astype(np.float64) * 1.0001)
    u1, u2 = _u(w[0::2]), _u(w[1::2])
    r = np.sqrt(-2.0 * np.log(u1.astype(LD)))
    th = (TWO_PI * u2).astype(LD)
    for got, want in ((c32, r * np.cos(th)), (s32, r * np.sin(th))):
        f = np.asarray(want, dtype=np.float64).astype(np.float32)
        ulp32 = np.maximum(np.spacing(np.abs(f)).astype(np.float64), 2.0 ** -149)
        assert np.max(np.abs(got.astype(LD) - want) / ulp32) <= 1.0
