"""Accuracy of the dedicated fp64 routines in nt_device_rt.cuh.

The device Box-Muller and the EXP fast path use routines written for the
replay (nt_neg2log_u1, nt_sincos_2pi_u2, nt_exp_small, the full-range
nt_exp_cw).  Here they are
compiled for the host from the same header and compared with x87 long-double
libm (64-bit significand) over random generator words and the edge words
(0, 1, 2^31, 2^32-1, the sqrt(2) fold, every quadrant boundary).  The bound
is 2 ulp of the result (or 2^-53 absolute for sin/cos results below 2^-52,
where the reference's own argument rounding dominates).  The same routines
run on the GPU in test_gpu_parity.py (normals vs the oracle).
"""
import os
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#define NT_HOST 1
#include <stdio.h>
#include <stdint.h>
#include <math.h>
#include "nt_device_rt.cuh"

static double ulp_of(double x) {
  x = fabs(x);
  if (x < 2.2250738585072014e-308) return 4.9406564584124654e-324;
  return nextafter(x, INFINITY) - x;
}

int main(void) {
  uint64_t st = 0x9E3779B97F4A7C15ull;
  double worst_log = 0, worst_sin = 0, worst_cos = 0, worst_exp = 0;
  double worst_log_t = 0, worst_sin_t = 0, worst_cos_t = 0;
  const uint32_t edges[] = {0u, 1u, 2u, 0x7fffffffu, 0x80000000u, 0xffffffffu, 0xfffffffeu, 0x3fffffffu,
                            0x40000000u, 0xbfffffffu, 0xc0000000u, 0x6a09e667u, 0xb504f333u, 0xb504f334u,
                            0x20000000u, 0x60000000u, 0xa0000000u, 0xe0000000u, 0x00ffffffu, 0x01000000u,
                            0xfeffffffu, 0xff000000u, 0x7f7fffffu, 0x80800000u, 0x5fffffffu, 0x9fffffffu};
  const int n_edges = sizeof(edges) / sizeof(edges[0]);
  for (long i = 0; i < 4000000 + n_edges; ++i) {
    uint32_t w;
    if (i < n_edges) w = edges[i];
    else { st ^= st << 13; st ^= st >> 7; st ^= st << 17; w = (uint32_t)(st >> 11); }
    /* -2 ln u1 */
    const double u1 = ((double)w + 0.5) * 2.3283064365386963e-10;
    const long double want_l = -2.0L * logl((long double)u1);
    const double got_l = nt_neg2log_u1(w);
    double e = fabsl((long double)got_l - want_l) / ulp_of((double)want_l);
    if (e > worst_log) worst_log = e;
    /* sin / cos of fl(2 pi u2) */
    const double th = 6.283185307179586 * u1;
    double s, c;
    nt_sincos_2pi_u2(w, &s, &c);
    const long double ws = sinl((long double)th), wc = cosl((long double)th);
    double es = fabsl((long double)s - ws) / fmax(ulp_of((double)ws), 1.1102230246251565e-16);
    double ec = fabsl((long double)c - wc) / fmax(ulp_of((double)wc), 1.1102230246251565e-16);
    if (es > worst_sin) worst_sin = es;
    if (ec > worst_cos) worst_cos = ec;
    /* the table-driven versions (what the device Box-Muller calls) */
    const double got_lt = nt_neg2log_u1_t(w);
    e = fabsl((long double)got_lt - want_l) / ulp_of((double)want_l);
    if (e > worst_log_t) worst_log_t = e;
    nt_sincos_2pi_u2_t(w, &s, &c);
    es = fabsl((long double)s - ws) / fmax(ulp_of((double)ws), 1.1102230246251565e-16);
    ec = fabsl((long double)c - wc) / fmax(ulp_of((double)wc), 1.1102230246251565e-16);
    if (es > worst_sin_t) worst_sin_t = es;
    if (ec > worst_cos_t) worst_cos_t = ec;
    /* exp on [-1/8, 1/8] */
    const double x = ((double)w / 4294967295.0 - 0.5) * 0.25;
    const long double we = expl((long double)x);
    double ee = fabsl((long double)nt_exp_small(x) - we) / ulp_of((double)we);
    if (ee > worst_exp) worst_exp = ee;
  }
  /* full-range exp: every binade of the argument from -745 to 709.78, the
     thresholds, gradual underflow, and the special values */
  double worst_cw = 0.0;
  int special_ok = 1;
  for (long i = 0; i < 3000000; ++i) {
    st ^= st << 13; st ^= st >> 7; st ^= st << 17;
    const double u = (double)(st >> 11) * 0x1p-53;
    double x;
    if (i % 3 == 0) x = -745.0 + u * (709.78 + 745.0);            /* whole range */
    else if (i % 3 == 1) x = (u - 0.5) * 2.0;                     /* near 0 */
    else x = (u < 0.5 ? -1.0 : 1.0) * ldexp(1.0, -60 + (int)(u * 70.0)) * (1.0 + u);  /* tiny to ~1 */
    const long double want = expl((long double)x);
    const double got = nt_exp_cw(x);
    const double w = (double)want;
    double e;
    if (w == 0.0) e = got == 0.0 ? 0.0 : 99.0;
    else e = fabsl((long double)got - want) / ulp_of(w);
    if (e > worst_cw) worst_cw = e;
  }
  const double specials[] = {0.0, -0.0, 709.78, 709.79, 710.0, 1e300, -744.4, -745.13, -745.2, -746.0, -1e300};
  for (int i = 0; i < 11; ++i) {
    const double x = specials[i], got = nt_exp_cw(x), want = exp(x);
    if (!(got == want || fabs(got - want) <= ulp_of(want))) special_ok = 0;
  }
  if (!isinf(nt_exp_cw(INFINITY)) || nt_exp_cw(-INFINITY) != 0.0 || !isnan(nt_exp_cw(NAN))) special_ok = 0;
  printf("%.6f %.6f %.6f %.6f %.6f %.6f %.6f %.6f %d\n", worst_log, worst_sin, worst_cos, worst_exp, worst_log_t,
         worst_sin_t, worst_cos_t, worst_cw, special_ok);
  return 0;
}
"""


@pytest.fixture(scope="module")
def worst():
    d = tempfile.mkdtemp()
    src = os.path.join(d, "math_check.cpp")
    exe = os.path.join(d, "math_check")
    with open(src, "w") as f:
        f.write(PROGRAM)
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-I",
                    os.path.join(ROOT, "nablatensor_b200", "csrc"), "-o", exe, src, "-lm"], check=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()
    return dict(zip(["log", "sin", "cos", "exp", "log_t", "sin_t", "cos_t", "exp_cw", "special"], map(float, out)))


def test_neg2log_u1_within_2_ulp(worst):
    assert worst["log"] <= 2.0, worst


def test_table_driven_box_muller_within_2_ulp(worst):
    assert worst["log_t"] <= 2.0 and worst["sin_t"] <= 2.0 and worst["cos_t"] <= 2.0, worst


def test_sincos_within_2_ulp(worst):
    assert worst["sin"] <= 2.0 and worst["cos"] <= 2.0, worst


def test_exp_small_within_1_ulp(worst):
    assert worst["exp"] <= 1.0, worst


def test_full_range_exp_within_1_ulp(worst):
    """nt_exp_cw (the device's exp for arguments of any size) against
    long-double exp over the whole range, with overflow, gradual underflow,
    infinities and NaN."""
    assert worst["exp_cw"] <= 1.0, worst
    assert worst["special"] == 1.0, worst
