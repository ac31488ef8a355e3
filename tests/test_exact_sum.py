"""The exact accumulator of the replay kernels (csrc/nt_exact.cuh), host build.

Every replay kernel reduces its per-path values into these fixed-point
words, so the sums a replay returns must be the correctly rounded exact sums
of what was added, whatever the grouping.  math.fsum is an independent
implementation of exactly that (Shewchuk's algorithm, correctly rounded), so
it is the oracle here: any set of doubles, added in any order or split into
any parts that are merged word by word, must round to math.fsum's result bit
for bit.
"""
import ctypes
import math
import os
import subprocess
import tempfile

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "nablatensor_b200", "csrc")

_SRC = r"""
#define NT_HOST 1
#include <stdint.h>
#include "nt_exact.cuh"
extern "C" int nt_x_words(void) { return NT_XWORDS; }
extern "C" void nt_x_add(long long* w, const double* x, long long n) {
  for (long long i = 0; i < n; ++i) nt_exact_add(w, x[i]);
}
extern "C" void nt_x_merge(long long* w, const long long* v) {
  for (int i = 0; i < NT_XWORDS; ++i) w[i] += v[i];
}
extern "C" void nt_x_normalize(long long* w) { nt_exact_normalize(w); }
extern "C" double nt_x_round(const long long* w) { return nt_exact_to_double(w); }
"""


@pytest.fixture(scope="module")
def xlib():
    d = tempfile.mkdtemp(prefix="nt_exact_")
    src, so = os.path.join(d, "x.cpp"), os.path.join(d, "x.so")
    with open(src, "w") as f:
        f.write(_SRC)
    subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-I", CSRC, "-o", so, src], check=True)
    lib = ctypes.CDLL(so)
    lib.nt_x_add.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong]
    lib.nt_x_merge.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.nt_x_normalize.argtypes = [ctypes.c_void_p]
    lib.nt_x_round.argtypes = [ctypes.c_void_p]
    lib.nt_x_round.restype = ctypes.c_double
    return lib


def _words(lib):
    return np.zeros(lib.nt_x_words(), dtype=np.int64)


def _add(lib, w, x):
    x = np.ascontiguousarray(x, dtype=np.float64)
    lib.nt_x_add(w.ctypes.data, x.ctypes.data, x.size)


def _round(lib, w):
    return lib.nt_x_round(w.ctypes.data)


def _same(a, b):
    return np.float64(a).tobytes() == np.float64(b).tobytes() or (math.isnan(a) and math.isnan(b))


def _cases():
    rng = np.random.default_rng(20261202)
    yield "normal", rng.normal(size=10_000)
    yield "payoffs", np.maximum(rng.normal(5, 10, size=50_000), 0.0)
    yield "wide exponents", rng.normal(size=4_000) * 2.0 ** rng.integers(-1000, 1000, size=4_000)
    yield "cancellation", np.concatenate([[1e300, -1e300, 1.0, 1e-300], rng.normal(size=100) * 1e-17])
    big = rng.normal(size=1000) * 1e16
    yield "cancelling pairs", np.concatenate([big, -big[::-1], [3.0, 2.0 ** -1074]])
    yield "subnormals", rng.integers(-2**52, 2**52, size=2000).astype(np.float64) * 2.0 ** -1074
    yield "subnormal to normal", np.array([2.0 ** -1022 - 2.0 ** -1074, 2.0 ** -1074, 2.0 ** -1074])
    yield "ties to even", np.array([1.0, 2.0 ** -53])
    yield "ties to even, odd", np.array([1.0 + 2.0 ** -52, 2.0 ** -53])
    yield "just above a tie", np.array([1.0, 2.0 ** -53, 2.0 ** -200])
    yield "just below a tie", np.array([1.0, 2.0 ** -53, -(2.0 ** -200)])
    yield "signed zeros", np.array([-0.0, 0.0, -0.0])
    yield "largest", np.array([np.finfo(np.float64).max, -np.finfo(np.float64).max / 2])
    yield "negative", -np.abs(rng.normal(size=1000)) * 1e5


@pytest.mark.parametrize("name,x", list(_cases()), ids=[c[0] for c in _cases()])
def test_rounds_the_exact_sum_like_fsum(xlib, name, x):
    w = _words(xlib)
    _add(xlib, w, x)
    got = _round(xlib, w)
    want = math.fsum(x)
    if want == 0.0:
        assert got == 0.0
    else:
        assert _same(got, want), (name, got, want)


def test_order_grouping_and_merging_do_not_change_the_bits(xlib):
    rng = np.random.default_rng(7)
    x = rng.normal(3.0, 40.0, size=30_000) * 2.0 ** rng.integers(-60, 60, size=30_000)
    want = math.fsum(x)
    for trial in range(6):
        perm = rng.permutation(x.size)
        cuts = np.sort(rng.choice(np.arange(1, x.size), size=trial * 7, replace=False))
        total = _words(xlib)
        for part in np.split(x[perm], cuts):
            w = _words(xlib)
            _add(xlib, w, part)
            if trial % 2:
                xlib.nt_x_normalize(w.ctypes.data)  # a normalised part merges the same
            xlib.nt_x_merge(total.ctypes.data, w.ctypes.data)
        assert _same(_round(xlib, total), want)


def test_non_finite_addends_follow_ieee_sums(xlib):
    inf, nan = float("inf"), float("nan")
    for x, want in [([1.0, inf], inf), ([-inf, 2.0], -inf), ([inf, -inf], nan), ([1.0, nan], nan),
                    ([inf, inf], inf)]:
        w = _words(xlib)
        _add(xlib, w, x)
        got = _round(xlib, w)
        assert _same(got, want), (x, got)
    # counts merge by addition, so a split across parts gives the same answer
    a, b = _words(xlib), _words(xlib)
    _add(xlib, a, [inf, 1.0])
    _add(xlib, b, [-inf])
    xlib.nt_x_merge(a.ctypes.data, b.ctypes.data)
    assert math.isnan(_round(xlib, a))


def test_overflow_rounds_to_infinity(xlib):
    m = np.finfo(np.float64).max
    w = _words(xlib)
    _add(xlib, w, [m, m])
    assert _round(xlib, w) == float("inf")
    w = _words(xlib)
    _add(xlib, w, [-m, -m, -m])
    assert _round(xlib, w) == -float("inf")
