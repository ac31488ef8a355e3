"""The float-result exps of fp32 tapes (nt_exp_f32, nt_exp_f32s in
nt_device_rt.cuh), host build.

Under the reference's fp32 semantics an EXP node is (float)exp((double)x)
(ScalarReplay.java:37-51).  The device evaluates it to about 2^-43 relative
in double instead of to full double accuracy; the float it rounds to must be
(float)exp((double)x) except where e^x lies that close to a float rounding
boundary.  Over 16M random floats of each routine's domain plus the edges
(overflow and float-subnormal boundaries, signed zeros, infinities, NaN):
at most 1 in 10^4 results differ, and none by more than one float ulp.
The reference value is x87 long-double expl rounded to float.
"""
import os
import subprocess
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#define NT_HOST 1
#include <stdio.h>
#include <stdint.h>
#include <math.h>
#include "nt_device_rt.cuh"

static long ulps_apart(float a, float b) {
  if (a == b) return 0;
  if (a != a || b != b) return (a != a && b != b) ? 0 : 1000000;
  int32_t ia, ib;
  memcpy(&ia, &a, 4);
  memcpy(&ib, &b, 4);
  if (ia < 0) ia = INT32_MIN - ia;
  if (ib < 0) ib = INT32_MIN - ib;
  return labs((long)ia - (long)ib);
}

static void run(const char* name, float (*fn)(float), float lo, float hi, const float* edges, int n_edges) {
  uint64_t st = 0x2545F4914F6CDD1Dull;
  long differ = 0, worst = 0, n = 16000000 + n_edges;
  for (long i = 0; i < n; ++i) {
    float x;
    if (i < n_edges) x = edges[i];
    else { st ^= st << 13; st ^= st >> 7; st ^= st << 17; x = lo + (hi - lo) * (float)((st >> 40) * 0x1p-24); }
    const float want = (float)expl((long double)x);
    const float got = fn(x);
    const long u = ulps_apart(got, want);
    if (u) ++differ;
    if (u > worst) worst = u;
  }
  printf("%s %ld %ld %ld\n", name, n, differ, worst);
}

int main(void) {
  const float e1[] = {-105.0f, -104.0f, -103.97f, -103.278929f, -87.3365f, -87.3f, -20.0f, -1.0f, -0.0f, 0.0f,
                      1e-30f, -1e-30f, 0.5f, 1.0f, 20.0f, 88.0f, 88.7228f, 88.72284f, 88.7229f, 89.0f, 1e30f,
                      -1e30f, INFINITY, -INFINITY, NAN};
  const float e2[] = {-0.125f, -0.0625f, -1e-7f, -0.0f, 0.0f, 1e-7f, 0.0625f, 0.125f};
  run("full", nt_exp_f32, -105.0f, 90.0f, e1, sizeof(e1) / sizeof(e1[0]));
  run("series", nt_exp_f32s, -0.125f, 0.125f, e2, sizeof(e2) / sizeof(e2[0]));
  return 0;
}
"""


def test_float_result_exps_round_as_the_double_exp_does():
    d = tempfile.mkdtemp(prefix="nt_fexp_")
    src, exe = os.path.join(d, "f.cpp"), os.path.join(d, "f")
    with open(src, "w") as f:
        f.write(PROGRAM)
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-I",
                    os.path.join(ROOT, "nablatensor_b200", "csrc"), "-o", exe, src], check=True)
    out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    for line in out.splitlines():
        name, n, differ, worst = line.split()
        n, differ, worst = int(n), int(differ), int(worst)
        print(f"{name}: {differ} of {n} differ, worst {worst} ulp")
        assert worst <= 1, line
        assert differ <= n * 1e-4, line
