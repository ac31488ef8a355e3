/*
 * nt_device_rt.cuh -- device runtime shared by every replay kernel.
 *
 * One source, three consumers:
 *   - NVRTC: the emitter hands this file to nvrtcCreateProgram as a named
 *     header, so every generated sm_100a replay kernel includes it;
 *   - nvcc: nt_kat.cu includes it for the known-answer kernels that expose
 *     the raw generator words to the tests;
 *   - g++ (NT_HOST defined): the emitter's host target, used by the CPU tests
 *     to check the emitted scenario code against the oracle bit for bit.
 *
 * Contents:
 *   - Philox2x32-10 keyed per (path, seed, stream) exactly as the reference's
 *     `cpu` engine keys it (nablatensor-engine-cpu/.../cpu/Philox.java:41-95):
 *       lo = (u32)path ^ (u32)seed, hi = (u32)(path>>32) ^ (u32)(seed>>32),
 *       stream s != 0: hi ^= s * 0x9E3779B1;
 *       normal pair c: counter (lo, hi ^ c), key 0x1BD11BDA, 10 rounds of
 *       (H, L) = 0xD256D193 * x0; x0 = H ^ key ^ x1; x1 = L; key += 0x9E3779B9;
 *       uniform k: counter (lo, hi ^ (k | 0x40000000)).
 *   - Box-Muller computing BOTH legs of a pair once (the reference device
 *     generator recomputes the whole pair per draw,
 *     nablatensor-core/.../CudaAadCodegen.java:485-510).
 *   - java.lang.Math.max/min semantics (NaN-propagating, -0 < +0), which the
 *     oracle uses (ScalarReplay.java:115-116).
 *   - the exact per-path accumulation: warp tiles of 32 paths summed into
 *     fixed-point words (nt_exact.cuh), block words folded into the launch's
 *     by atomics, the last block (atomic ticket, no spin-wait) rounding them.
 */
#ifndef NT_DEVICE_RT_CUH
#define NT_DEVICE_RT_CUH

#ifdef NT_HOST
#include <math.h>
#include <string.h>
#define NT_FN static inline
#else
#define NT_FN static __device__ __forceinline__
#endif

#include "nt_exact.cuh"

typedef unsigned int nt_u32;
typedef unsigned long long nt_u64;

#define NT_PHILOX_M 0xD256D193u
#define NT_PHILOX_W 0x9E3779B9u
#define NT_PHILOX_K0 0x1BD11BDAu
#define NT_STREAM_MIX 0x9E3779B1u
#define NT_UNIFORM_TAG 0x40000000u
#define NT_UINT_SCALE 2.3283064365386963e-10
#define NT_TWO_PI 6.283185307179586

/* The reference's Box-Muller angle theta = fl(2 pi u2): the product is
 * rounded on its own, never fused into the subtraction that reduces it (a
 * contracted fma would take sin of the unrounded product, up to 4 ulp away
 * from the reference's normals). */
#ifdef NT_HOST
#define NT_THETA(u2) (NT_TWO_PI * (u2))
#else
#define NT_THETA(u2) __dmul_rn(NT_TWO_PI, (u2))
#endif

/* Per-(path, seed, stream) key words. */
struct nt_key {
  nt_u32 lo;
  nt_u32 hi;
};

NT_FN nt_key nt_make_key(nt_u64 path, nt_u64 seed, int stream) {
  nt_key k;
  k.lo = (nt_u32)path ^ (nt_u32)seed;
  k.hi = (nt_u32)(path >> 32) ^ (nt_u32)(seed >> 32);
  if (stream != 0) k.hi ^= (nt_u32)stream * NT_STREAM_MIX;
  return k;
}

NT_FN nt_u32 nt_mulhi(nt_u32 a, nt_u32 b) {
#ifdef NT_HOST
  return (nt_u32)(((nt_u64)a * (nt_u64)b) >> 32);
#else
  return __umulhi(a, b);
#endif
}

/* Ten Philox2x32 rounds on counter (x0, x1).  The per-round keys are
 * compile-time constants once the loop is unrolled. */
NT_FN void nt_philox(nt_u32 x0, nt_u32 x1, nt_u32* o0, nt_u32* o1) {
  nt_u32 key = NT_PHILOX_K0;
#ifndef NT_HOST
#pragma unroll
#endif
  for (int i = 0; i < 10; ++i) {
    nt_u32 hi = nt_mulhi(NT_PHILOX_M, x0);
    nt_u32 lo = NT_PHILOX_M * x0;
    x0 = hi ^ key ^ x1;
    x1 = lo;
    key += NT_PHILOX_W;
  }
  *o0 = x0;
  *o1 = x1;
}

/* Words of normal pair `pair` (draw ordinals 2*pair and 2*pair+1). */
NT_FN void nt_normal_words(nt_key k, nt_u32 pair, nt_u32* w0, nt_u32* w1) {
  nt_philox(k.lo, k.hi ^ pair, w0, w1);
}

/* ---- fp64 elementary functions for the replay kernels ---------------------
 *
 * Written from the textbook methods (Cody and Waite, "Software Manual for the
 * Elementary Functions", 1980: argument reduction with a constant split in
 * two parts; Taylor / atanh series on the reduced range).  They exploit what
 * the replay knows about its arguments -- the Box-Muller inputs are 32-bit
 * generator words, GBM log-returns are small -- so they carry none of the
 * special-case handling a general-purpose routine needs.  Accuracy (checked
 * by the tests against libm and the device library): within 2 ulp.
 */

NT_FN int nt_hiword(double x) {
#ifdef NT_HOST
  long long b;
  memcpy(&b, &x, sizeof b);
  return (int)(b >> 32);
#else
  return __double2hiint(x);
#endif
}

NT_FN unsigned nt_loword(double x) {
#ifdef NT_HOST
  long long b;
  memcpy(&b, &x, sizeof b);
  return (unsigned)b;
#else
  return (unsigned)__double2loint(x);
#endif
}

NT_FN double nt_from_words(int hi, unsigned lo) {
#ifdef NT_HOST
  long long b = ((long long)hi << 32) | (long long)lo;
  double x;
  memcpy(&x, &b, sizeof x);
  return x;
#else
  return __hiloint2double(hi, (int)lo);
#endif
}

/* -2 ln(u1), u1 = (w0 + 0.5) 2^-32 (exact, in (2^-33, 1)).
 * u1 = m 2^k with m in [sqrt(1/2), sqrt(2)); ln m = 2 atanh(s), s = (m-1)/(m+1),
 * |s| < 0.1716, summed to s^23 (truncation < 2^-60 relative); ln2 is split so
 * that k ln2_hi is exact.  1/(m+1) is a single-precision seed refined by two
 * Newton steps, and s by one residual correction. */
NT_FN double nt_neg2log_u1(nt_u32 w0) {
  const double u = ((double)w0 + 0.5) * NT_UINT_SCALE;
  const int hi = nt_hiword(u);
  int k = ((hi >> 20) & 0x7ff) - 1023;
  int mhi = (hi & 0x000fffff) | 0x3ff00000; /* m in [1, 2) */
  if (mhi >= 0x3ff6a09f) {                   /* m >= sqrt(2): use m / 2 */
    mhi -= 0x00100000;
    k += 1;
  }
  const double m = nt_from_words(mhi, nt_loword(u));
  const double f = m - 1.0; /* exact */
  const double d = m + 1.0;
#ifdef NT_HOST
  double y = (double)(1.0f / (float)d);
#else
  float yf;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(yf) : "f"((float)d));
  double y = (double)yf;
#endif
  double e = fma(-d, y, 1.0);
  y = fma(y, e, y);
  e = fma(-d, y, 1.0);
  y = fma(y, e, y);
  double s = f * y;
  s = fma(fma(-s, d, f), y, s);
  const double z = s * s;
  double p = 1.0 / 23.0;
  p = fma(p, z, 1.0 / 21.0);
  p = fma(p, z, 1.0 / 19.0);
  p = fma(p, z, 1.0 / 17.0);
  p = fma(p, z, 1.0 / 15.0);
  p = fma(p, z, 1.0 / 13.0);
  p = fma(p, z, 1.0 / 11.0);
  p = fma(p, z, 1.0 / 9.0);
  p = fma(p, z, 1.0 / 7.0);
  p = fma(p, z, 1.0 / 5.0);
  p = fma(p, z, 1.0 / 3.0);
  const double lnm = 2.0 * fma(s * z, p, s);
  const double kd = (double)k;
  const double ln_u = fma(kd, 0x1.62e42p-1 /* ln2 hi */, fma(kd, 0x1.fdf473de6af28p-22 /* ln2 lo */, lnm));
  return -2.0 * ln_u;
}

/* sin and cos of the reference's angle fl(2 pi u2), u2 = (w1 + 0.5) 2^-32.
 * theta = k pi/2 + x with pi/2 in two parts (the first product exact), then
 * Taylor series on |x| <= pi/4 to x^17 (sin) and x^16 (cos). */
NT_FN void nt_sincos_2pi_u2(nt_u32 w1, double* sn, double* cs) {
  const double u2 = ((double)w1 + 0.5) * NT_UINT_SCALE;
  const double th = NT_THETA(u2);
#ifdef NT_HOST
  const int k = (int)nearbyint(th * 0.6366197723675814);
#else
  const int k = __double2int_rn(th * 0.6366197723675814);
#endif
  const double kd = (double)k;
  double x = fma(-kd, 0x1.921fb54442d18p+0 /* pi/2 hi */, th);
  x = fma(-kd, 0x1.1a62633145c07p-54 /* pi/2 lo */, x);
  const double z = x * x;
  double ps = 1.0 / 355687428096000.0;     /* 1/17! */
  ps = fma(ps, z, -1.0 / 1307674368000.0); /* 1/15! */
  ps = fma(ps, z, 1.0 / 6227020800.0);     /* 1/13! */
  ps = fma(ps, z, -1.0 / 39916800.0);      /* 1/11! */
  ps = fma(ps, z, 1.0 / 362880.0);         /* 1/9!  */
  ps = fma(ps, z, -1.0 / 5040.0);          /* 1/7!  */
  ps = fma(ps, z, 1.0 / 120.0);            /* 1/5!  */
  ps = fma(ps, z, -1.0 / 6.0);             /* 1/3!  */
  const double s = fma(x * z, ps, x);
  double pc = 1.0 / 20922789888000.0;      /* 1/16! */
  pc = fma(pc, z, -1.0 / 87178291200.0);   /* 1/14! */
  pc = fma(pc, z, 1.0 / 479001600.0);      /* 1/12! */
  pc = fma(pc, z, -1.0 / 3628800.0);       /* 1/10! */
  pc = fma(pc, z, 1.0 / 40320.0);          /* 1/8!  */
  pc = fma(pc, z, -1.0 / 720.0);           /* 1/6!  */
  pc = fma(pc, z, 1.0 / 24.0);             /* 1/4!  */
  pc = fma(pc, z, -0.5);                   /* 1/2!  */
  const double c = fma(z, pc, 1.0);
  const int q = k & 3;
  double so = (q & 1) ? c : s;
  double co = (q & 1) ? s : c;
  if (q & 2) so = -so;
  if ((q + 1) & 2) co = -co;
  *sn = so;
  *cs = co;
}

/* The generated tables and constants (nt_math_tables.cuh, 60-digit decimal
 * arithmetic): the Box-Muller tables below and the exp series coefficients. */
#ifdef NT_HOST
#define NT_TABLE_QUAL const
#else
#define NT_TABLE_QUAL __device__ const
#endif
#include "nt_math_tables.cuh"

/* exp(x) for |x| <= 1/8 (every GBM log-return): 1 + x (1 + x q(x)) with q
 * the degree-7 polynomial interpolating (e^x - 1 - x) / x^2 at the 8
 * Chebyshev nodes of [-1/8, 1/8] (coefficients in nt_math_tables.cuh; 2.2e-18
 * relative error with the rounded coefficients), in Horner form: 9 FMAs, one
 * fewer than the Taylor series to x^10 of the same accuracy.  (Estrin's
 * scheme measured slower in the replay: the kernel is bound by the fp64 pipe
 * and by instructions issued, not by the dependent chain.) */
NT_FN double nt_exp_small(double x) {
  double q = NT_EXPS_C7;
  q = fma(q, x, NT_EXPS_C6);
  q = fma(q, x, NT_EXPS_C5);
  q = fma(q, x, NT_EXPS_C4);
  q = fma(q, x, NT_EXPS_C3);
  q = fma(q, x, NT_EXPS_C2);
  q = fma(q, x, NT_EXPS_C1);
  q = fma(q, x, NT_EXPS_C0);
  return fma(fma(q, x, 1.0), x, 1.0);
}

/* exp(x) over the whole double range, without a branch (Cody and Waite 1980):
 * k = rint(x / ln2) by the rounding constant 1.5 * 2^52, r = x - k ln2 with
 * ln2 in two parts (the high part has 42 significant bits, so k * hi is exact
 * for |k| < 2^11), |r| <= ln2 / 2; exp(r) = 1 + r (1 + r q(r)) with q the
 * degree-9 Chebyshev interpolant of (e^r - 1 - r) / r^2 on the reduced range
 * (nt_math_tables.cuh; 1.6e-17 relative, 11 FMAs where the Taylor series to
 * r^13 took 13); then scaled by 2^(k/2) * 2^(k - k/2), each factor a normal
 * power of two, so the overflow threshold and gradual underflow round once.
 * x is clamped to [-746, 710] first (exp is 0 or infinite beyond); NaN
 * passes through. */
NT_FN double nt_exp_cw(double x) {
  const double xc = fmin(fmax(x, -746.0), 710.0);
  const double kt = fma(xc, 0x1.71547652b82fep+0 /* 1/ln2 */, 0x1.8p52);
  const double kd = kt - 0x1.8p52;
  const int k = (int)nt_loword(kt);
  double r = fma(kd, -0x1.62e42fefa3800p-1 /* ln2 hi */, xc);
  r = fma(kd, -0x1.ef35793c76730p-45 /* ln2 lo */, r);
  double q = NT_EXPW_C9;
  q = fma(q, r, NT_EXPW_C8);
  q = fma(q, r, NT_EXPW_C7);
  q = fma(q, r, NT_EXPW_C6);
  q = fma(q, r, NT_EXPW_C5);
  q = fma(q, r, NT_EXPW_C4);
  q = fma(q, r, NT_EXPW_C3);
  q = fma(q, r, NT_EXPW_C2);
  q = fma(q, r, NT_EXPW_C1);
  q = fma(q, r, NT_EXPW_C0);
  const double p = fma(fma(q, r, 1.0), r, 1.0);
  const int k1 = k >> 1, k2 = k - k1;
  const double y = (p * nt_from_words((k1 + 1023) << 20, 0u)) * nt_from_words((k2 + 1023) << 20, 0u);
  return x != x ? x : y;
}

/* sqrt of a positive normal argument (the Box-Muller radius, in
 * (4.6e-10, 46.1)): the hardware reciprocal square-root approximation y as
 * the seed; the root g = a y and the half reciprocal h = y / 2 refined
 * together by one coupled Newton step (Goldschmidt's iteration), then one
 * residual correction of the root (Markstein's method), which squares the
 * remaining relative error: 7 fp64 operations.  Measured on the device
 * against long-double sqrt (tests/test_gpu_math.py): 0.5 ulp worst over 5M
 * arguments, i.e. correctly rounded; a second Newton step changed no result
 * and cost 3 % of the replay's speed. */
NT_FN double nt_sqrt_pos(double a) {
#ifdef NT_HOST
  return sqrt(a);
#else
  double y;
  asm("rsqrt.approx.ftz.f64 %0, %1;" : "=d"(y) : "d"(a));
  double g = a * y;    /* sqrt(a) */
  double h = 0.5 * y;  /* 1 / (2 sqrt(a)) */
  const double r = fma(-g, h, 0.5);
  g = fma(g, r, g);
  h = fma(h, r, h);
  return fma(fma(-g, g, a), h, g);
#endif
}

/*
 * exp for fp32 tapes, whose nodes the reference rounds to float after
 * evaluating exp in double ((float)Math.exp(x), ScalarReplay.java:37-51).  A
 * float result needs far less than a double's accuracy: evaluated in double
 * to about 2^-43 relative (q of degree 7 on the Cody-Waite range, the
 * construction of nt_exp_cw), the rounding to float is the reference's
 * except when e^x lies within 2^-43 of a float rounding boundary, about one
 * argument in 2^19.  x is clamped in single precision to [-105, 89], beyond
 * which the float result is 0 or +inf anyway, so 2^k is applied by adding k
 * to p's exponent (p * 2^k stays a normal double) and the one rounding to
 * float handles overflow and float subnormals.  NaN passes through.
 */
NT_FN float nt_exp_f32(float x) {
  const double d = (double)fminf(fmaxf(x, -105.0f), 89.0f);
  const double kt = fma(d, 0x1.71547652b82fep+0 /* 1/ln2 */, 0x1.8p52);
  const double kd = kt - 0x1.8p52;
  const int k = (int)nt_loword(kt);
  double r = fma(kd, -0x1.62e42fefa3800p-1 /* ln2 hi */, d);
  r = fma(kd, -0x1.ef35793c76730p-45 /* ln2 lo */, r);
  double q = NT_EXPF_C7;
  q = fma(q, r, NT_EXPF_C6);
  q = fma(q, r, NT_EXPF_C5);
  q = fma(q, r, NT_EXPF_C4);
  q = fma(q, r, NT_EXPF_C3);
  q = fma(q, r, NT_EXPF_C2);
  q = fma(q, r, NT_EXPF_C1);
  q = fma(q, r, NT_EXPF_C0);
  const double p = fma(fma(q, r, 1.0), r, 1.0);
  const double y = nt_from_words(nt_hiword(p) + (int)((unsigned)k << 20), nt_loword(p));
  return x != x ? x : (float)y;
}

/* The float-result exp for |x| <= 1/8 (a GBM log-return): the series form of
 * nt_exp_small with q of degree 5, about 2^-43 relative. */
NT_FN float nt_exp_f32s(float x) {
  const double d = (double)x;
  double q = NT_EXPFS_C5;
  q = fma(q, d, NT_EXPFS_C4);
  q = fma(q, d, NT_EXPFS_C3);
  q = fma(q, d, NT_EXPFS_C2);
  q = fma(q, d, NT_EXPFS_C1);
  q = fma(q, d, NT_EXPFS_C0);
  return (float)fma(fma(q, d, 1.0), d, 1.0);
}

#ifndef NT_HOST
/* nt_exp_cw that also records in `wide` whether this lane's argument left the
 * series range: the redo pass of the forward loop (see NT_EXP64F), after
 * which the reverse sweep takes its full-range copy. */
NT_FN double nt_exp_cw_flag(double x, bool& wide) {
  wide |= !(fabs(x) <= 0.125);
  return nt_exp_cw(x);
}

/* The float-result forms' flagging twins (see nt_exp_series_flag). */
NT_FN float nt_exp_f32s_flag(float x, bool& wide) {
  wide |= !(fabsf(x) <= 0.125f);
  return nt_exp_f32s(x);
}

NT_FN float nt_exp_f32_flag(float x, bool& wide) {
  wide |= !(fabsf(x) <= 0.125f);
  return nt_exp_f32(x);
}
#endif

#ifndef NT_HOST
/* The forward loop's form of an exp the reverse sweep recomputes: the bare
 * series, with a wide argument recorded in `wide`.  A warp in which any lane
 * recorded one runs the loop again with nt_exp_cw_flag (the emitted kernel's
 * redo pass), so the series is only ever kept where it is accurate. */
NT_FN double nt_exp_series_flag(double x, bool& wide) {
  wide |= !(fabs(x) <= 0.125);
  return nt_exp_small(x);
}

/* The forward loop's first-pass form of an exp whose value is taped: the
 * reduction and polynomial of nt_exp_cw, without its clamp, NaN select and
 * two-step scaling.  For |x| <= 700 the result p 2^k is a normal double, so
 * adding k to p's exponent gives nt_exp_cw's bits; any other argument (NaN
 * included) is recorded in `wide`, and the warp's redo pass evaluates the
 * whole loop again with nt_exp_cw. */
NT_FN double nt_exp_cw_fast_flag(double x, bool& wide) {
  wide |= !(fabs(x) <= 700.0);
  const double kt = fma(x, 0x1.71547652b82fep+0 /* 1/ln2 */, 0x1.8p52);
  const double kd = kt - 0x1.8p52;
  const int k = (int)nt_loword(kt);
  double r = fma(kd, -0x1.62e42fefa3800p-1 /* ln2 hi */, x);
  r = fma(kd, -0x1.ef35793c76730p-45 /* ln2 lo */, r);
  double q = NT_EXPW_C9;
  q = fma(q, r, NT_EXPW_C8);
  q = fma(q, r, NT_EXPW_C7);
  q = fma(q, r, NT_EXPW_C6);
  q = fma(q, r, NT_EXPW_C5);
  q = fma(q, r, NT_EXPW_C4);
  q = fma(q, r, NT_EXPW_C3);
  q = fma(q, r, NT_EXPW_C2);
  q = fma(q, r, NT_EXPW_C1);
  q = fma(q, r, NT_EXPW_C0);
  const double p = fma(fma(q, r, 1.0), r, 1.0);
  return nt_from_words(nt_hiword(p) + (int)((unsigned)k << 20), nt_loword(p));
}
#endif

/* EXP nodes of fp64 tapes: the dedicated routine on the device (the emitted
 * kernel declares nt_lanes = __activemask() and nt_wide at the top of each
 * scenario), libm in the host build (bit-for-bit with the oracle).
 * NT_EXP64 is the full-range routine (no branch); NT_EXP64F is the forward
 * loop's form for an exp the reverse sweep recomputes (the bare series, wide
 * arguments recorded in nt_wide), NT_EXP64W the redo pass's (full range,
 * recording too); NT_EXP64_SERIES is the recompute once the forward sweep has
 * shown every argument of the warp in the series range; NT_EXP64T is the
 * forward loop's first-pass form for a taped exp (full range up to |x| = 700,
 * larger arguments recorded for the redo pass).  NT_EXPF32... are the four
 * forms for fp32 tapes under the reference's fp32 semantics, with float
 * arguments and results (nt_exp_f32, nt_exp_f32s). */
#ifdef NT_HOST
#define NT_EXP64(x) exp(x)
#define NT_EXP64T(x) exp(x)
#define NT_EXP64W(x) exp(x)
#define NT_EXP64F(x) exp(x)
#define NT_EXP64_SERIES(x) exp(x)
#define NT_EXPF32(x) ((float)exp((double)(x)))
#define NT_EXPF32W(x) ((float)exp((double)(x)))
#define NT_EXPF32F(x) ((float)exp((double)(x)))
#define NT_EXPF32_SERIES(x) ((float)exp((double)(x)))
#else
#define NT_EXP64(x) nt_exp_cw(x)
#define NT_EXP64T(x) nt_exp_cw_fast_flag((x), nt_wide)
#define NT_EXP64W(x) nt_exp_cw_flag((x), nt_wide)
#define NT_EXP64F(x) nt_exp_series_flag((x), nt_wide)
#define NT_EXP64_SERIES(x) nt_exp_small(x)
#define NT_EXPF32(x) nt_exp_f32(x)
#define NT_EXPF32W(x) nt_exp_f32_flag((x), nt_wide)
#define NT_EXPF32F(x) nt_exp_f32s_flag((x), nt_wide)
#define NT_EXPF32_SERIES(x) nt_exp_f32s(x)
#endif

/* ---- table-driven Box-Muller ---------------------------------------------
 * Short polynomials on a small reduced range plus tabulated values
 * (nt_math_tables.cuh, generated in 60-digit decimal arithmetic): fewer and
 * shorter dependent chains than the series above.  On the device every block
 * stages the tables in shared memory (nt_math_tables_load) before its first
 * draw; the host build reads the constant arrays. */

#ifdef NT_HOST
#define NT_LN_TAB nt_ln_tab_g
#define NT_LN_LO nt_ln_lo_g
#define NT_SC_TAB nt_sc_tab_g
#define NT_SC_ARG nt_sc_arg_g
NT_FN void nt_math_tables_load(void) {}
#else
__shared__ __align__(16) double nt_ln_tab_s[NT_LN_TAB_N * 2];
__shared__ double nt_ln_lo_s[NT_LN_TAB_N];
__shared__ __align__(16) double nt_sc_tab_s[NT_SC_TAB_N * 2];
__shared__ double nt_sc_arg_s[NT_SC_TAB_N];
#define NT_LN_TAB nt_ln_tab_s
#define NT_LN_LO nt_ln_lo_s
#define NT_SC_TAB nt_sc_tab_s
#define NT_SC_ARG nt_sc_arg_s
/* Every thread of the block must call this before any Box-Muller draw. */
NT_FN void nt_math_tables_load(void) {
  for (int i = threadIdx.x; i < NT_LN_TAB_N * 2; i += blockDim.x) nt_ln_tab_s[i] = nt_ln_tab_g[i];
  for (int i = threadIdx.x; i < NT_LN_TAB_N; i += blockDim.x) nt_ln_lo_s[i] = nt_ln_lo_g[i];
  for (int i = threadIdx.x; i < NT_SC_TAB_N * 2; i += blockDim.x) nt_sc_tab_s[i] = nt_sc_tab_g[i];
  for (int i = threadIdx.x; i < NT_SC_TAB_N; i += blockDim.x) nt_sc_arg_s[i] = nt_sc_arg_g[i];
  __syncthreads();
}
#endif

/* Entry j of a two-wide table: one 16-byte load on the device. */
NT_FN void nt_tab2(const double* tab, int j, double* a, double* b) {
#ifdef NT_HOST
  *a = tab[2 * j];
  *b = tab[2 * j + 1];
#else
  const double2 p = reinterpret_cast<const double2*>(tab)[j];
  *a = p.x;
  *b = p.y;
#endif
}

/* -2 ln(u1) by Tang's table method (ACM TOMS 15(2), 1989): u1 = m 2^k with m
 * folded into [0.75, 1.5); c_j = 0.75 + j/128 the nearest centre (c_32 = 1
 * exactly, so u1 near 1 keeps full relative precision).  j and c_j come from
 * the top 20 fraction bits of m in integer arithmetic: c_j is m rounded to 7
 * fraction bits (6 when folded, where the binade is [0.5, 1)), a carry into
 * the exponent giving c = 1 or 1.5 exactly; f = m - c_j is exact.  The table
 * carries -2/c_j and -2 ln c_j (a double-double), so the factor -2 costs
 * nothing: with v = -2 f / c_j, |v| <= 1/96,
 * -2 ln(1 + f/c_j) = v + v^2/4 + v^3/12 + v^4/32 + v^5/80 + v^6/192 + v^7/448
 * (the series of ln(1 + t) at t = -v/2; truncation below 2^-55 of the
 * result), in Horner form. */
NT_FN double nt_neg2log_u1_t(nt_u32 w0) {
  const double u = fma((double)w0, 0x1p-32, 0x1p-33); /* (w0 + 0.5) 2^-32, exact */
  const int hi = nt_hiword(u);
  const int f20 = hi & 0x000fffff;
  const bool fold = f20 >= 0x00080000; /* m >= 1.5: use m / 2 in [0.75, 1) */
  const int k = (hi >> 20) - (fold ? 1022 : 1023);
  const int mhi = f20 | (fold ? 0x3fe00000 : 0x3ff00000);
  /* (m - 0.75) * 128 rounded: (f20 / 2^20 - 0.5) * 64 when folded, else 32 + f20 / 2^13 */
  const int j = fold ? (f20 - 0x00080000 + 0x2000) >> 14 : 32 + ((f20 + 0x1000) >> 13);
  const int chi = fold ? (mhi + 0x2000) & ~0x3fff : (mhi + 0x1000) & ~0x1fff;
  const double m = nt_from_words(mhi, nt_loword(u));
  double rc, lh;
  nt_tab2(NT_LN_TAB, j, &rc, &lh);
  const double v = (m - nt_from_words(chi, 0u)) * rc; /* m - c_j exact */
  double p = 1.0 / 448.0;
  p = fma(p, v, 1.0 / 192.0);
  p = fma(p, v, 1.0 / 80.0);
  p = fma(p, v, 1.0 / 32.0);
  p = fma(p, v, 1.0 / 12.0);
  p = fma(p, v, 0.25);
  const double g = fma(v * v, p, v);
  const double kd = (double)k;
  const double s1 = fma(kd, -0x1.62e42p+0 /* -2 ln2 hi */, lh);
  const double s2 = fma(kd, -0x1.fdf473de6af28p-21 /* -2 ln2 lo */, NT_LN_LO[j] + g);
  return s1 + s2;
}

/* sin and cos of the reference's angle theta = fl(2 pi u2): theta = a_j + b
 * with j = w1 >> 24, the top 8 bits of the generator word, and a_j = j times
 * pi/128 rounded to 33 significant bits, an exact double within 2.5e-10 of
 * j pi/128; sin a_j and cos a_j are tabulated at that double, so b = theta -
 * a_j (exact, Sterbenz) is the whole reduction.  Since u2 lies at least 2^-33
 * inside [j/256, (j+1)/256), b is in (0, pi/128 + 2.5e-10) whatever theta's
 * rounding; sin b to b^7 and cos b - 1 to b^6 (truncation < 2^-61). */
NT_FN void nt_sincos_2pi_u2_t(nt_u32 w1, double* sn, double* cs) {
  const double u2 = fma((double)w1, 0x1p-32, 0x1p-33); /* (w1 + 0.5) 2^-32, exact */
  const double th = NT_THETA(u2);
  const int j = (int)(w1 >> 24);
  double S, C;
  nt_tab2(NT_SC_TAB, j, &S, &C);
  const double b = th - NT_SC_ARG[j];
  const double z = b * b;
  double ps = -1.0 / 5040.0;
  ps = fma(ps, z, 1.0 / 120.0);
  ps = fma(ps, z, -1.0 / 6.0);
  const double sb = fma(b * z, ps, b);
  double pc = -1.0 / 720.0;
  pc = fma(pc, z, 1.0 / 24.0);
  pc = fma(pc, z, -0.5);
  const double cm1 = z * pc;
  *sn = S + fma(C, sb, S * cm1);
  *cs = C + fma(C, cm1, -S * sb);
}

/* Box-Muller legs from the table-driven routines. */
NT_FN void nt_bm64_words(nt_u32 w0, nt_u32 w1, double* cos_leg, double* sin_leg) {
  const double r = nt_sqrt_pos(nt_neg2log_u1_t(w0));
  double s, c;
  nt_sincos_2pi_u2_t(w1, &s, &c);
  *cos_leg = r * c;
  *sin_leg = r * s;
}

/* fp64 Box-Muller of one block: cosine leg (even ordinal) and sine leg (odd).
 * The device uses the dedicated routines; the host build (the emitter's
 * test target) uses libm exactly as the oracle does. */
NT_FN void nt_bm64(nt_u32 w0, nt_u32 w1, double* cos_leg, double* sin_leg) {
#ifdef NT_HOST
  double u1 = ((double)w0 + 0.5) * NT_UINT_SCALE;
  double u2 = ((double)w1 + 0.5) * NT_UINT_SCALE;
  double r = sqrt(-2.0 * log(u1));
  double a = NT_TWO_PI * u2;
  *cos_leg = r * cos(a);
  *sin_leg = r * sin(a);
#else
  nt_bm64_words(w0, w1, cos_leg, sin_leg);
#endif
}

#ifndef NT_HOST
/* ---- float-result Box-Muller ---------------------------------------------
 * For fp32 tapes under the reference's fp32 semantics, where each normal is
 * the double Box-Muller value rounded to float.  A value that is only ever
 * narrowed needs about 2^-40 relative, not a double's 2^-53, so the radius
 * stops earlier than the fp64 routines above (same tables, same reduction):
 *   -2 ln u1: the series to v^5 (truncation below 2^-40.5 of the result) and
 *     one rounding of k (-2 ln 2) + (-2 ln c_j), the table's low part unused;
 *   the radius: one coupled Newton step from the hardware rsqrt (relative
 *     error 1.5 e^2 for a seed error e).
 * The angle keeps the fp64 sin and cos: near a zero of cos or sin the leg is
 * a difference of two products, and a shorter series would leave its
 * truncation as an absolute error, far above 2^-40 of a small leg.  The
 * narrowed legs are the narrowed fp64 legs except where the double value lies
 * within about 2^-40 of a float rounding boundary, there one float ulp away
 * (measured on the device against the fp64 legs: tests/test_gpu_math.py). */
NT_FN double nt_neg2log_u1_f(nt_u32 w0) {
  const double u = fma((double)w0, 0x1p-32, 0x1p-33); /* (w0 + 0.5) 2^-32, exact */
  const int hi = nt_hiword(u);
  const int f20 = hi & 0x000fffff;
  const bool fold = f20 >= 0x00080000;
  const int k = (hi >> 20) - (fold ? 1022 : 1023);
  const int mhi = f20 | (fold ? 0x3fe00000 : 0x3ff00000);
  const int j = fold ? (f20 - 0x00080000 + 0x2000) >> 14 : 32 + ((f20 + 0x1000) >> 13);
  const int chi = fold ? (mhi + 0x2000) & ~0x3fff : (mhi + 0x1000) & ~0x1fff;
  const double m = nt_from_words(mhi, nt_loword(u));
  double rc, lh;
  nt_tab2(NT_LN_TAB, j, &rc, &lh);
  const double v = (m - nt_from_words(chi, 0u)) * rc; /* m - c_j exact */
  double p = 1.0 / 80.0;
  p = fma(p, v, 1.0 / 32.0);
  p = fma(p, v, 1.0 / 12.0);
  p = fma(p, v, 0.25);
  const double g = fma(v * v, p, v);
  return fma((double)k, -0x1.62e42fefa39efp+0 /* -2 ln 2 */, lh) + g;
}

NT_FN double nt_sqrt_pos_f(double a) {
  double y;
  asm("rsqrt.approx.ftz.f64 %0, %1;" : "=d"(y) : "d"(a));
  const double g = a * y;
  const double r = fma(-g, 0.5 * y, 0.5);
  return fma(g, r, g);
}

NT_FN void nt_bm64f_words(nt_u32 w0, nt_u32 w1, float* cos_leg, float* sin_leg) {
  const double r = nt_sqrt_pos_f(nt_neg2log_u1_f(w0));
  double s, c;
  nt_sincos_2pi_u2_t(w1, &s, &c);
  *cos_leg = (float)(r * c);
  *sin_leg = (float)(r * s);
}
#endif

/* fp32 Box-Muller: the uint32 words are the fp64 generator's; u1 is rounded
 * to the nearest float and clamped below 1 so the radius never collapses. */
NT_FN void nt_bm32(nt_u32 w0, nt_u32 w1, float* cos_leg, float* sin_leg) {
  const float scale = 2.3283064365386963e-10f; /* 2^-32, exact */
  const float half_scale = 1.1641532182693481e-10f; /* 2^-33, exact */
  const float below_one = 0.99999994039535522f; /* 1 - 2^-24 */
  float u1 = fminf(fmaf((float)w0, scale, half_scale), below_one);
  float u2 = fmaf((float)w1, scale, half_scale);
  float r = sqrtf(-2.0f * logf(u1));
  float a = 6.28318530717958648f * u2;
  float s, c;
#ifdef NT_HOST
  s = sinf(a);
  c = cosf(a);
#else
  sincosf(a, &s, &c);
#endif
  *cos_leg = r * c;
  *sin_leg = r * s;
}

NT_FN void nt_normal_pair64(nt_key k, nt_u32 pair, double* c, double* s) {
  nt_u32 w0, w1;
  nt_normal_words(k, pair, &w0, &w1);
  nt_bm64(w0, w1, c, s);
}

NT_FN void nt_normal_pair32(nt_key k, nt_u32 pair, float* c, float* s) {
  nt_u32 w0, w1;
  nt_normal_words(k, pair, &w0, &w1);
  nt_bm32(w0, w1, c, s);
}

/* fp32 pair evaluated in fp64 and narrowed: the reference's fp32 semantics
 * (each stored value is the double result rounded to float); on the device
 * by the float-result routines. */
NT_FN void nt_normal_pair32w(nt_key k, nt_u32 pair, float* c, float* s) {
#ifdef NT_HOST
  double cd, sd;
  nt_normal_pair64(k, pair, &cd, &sd);
  *c = (float)cd;
  *s = (float)sd;
#else
  nt_u32 w0, w1;
  nt_normal_words(k, pair, &w0, &w1);
  nt_bm64f_words(w0, w1, c, s);
#endif
}

NT_FN float nt_normal32w(nt_key k, nt_u32 ordinal) {
  float c, s;
  nt_normal_pair32w(k, ordinal >> 1, &c, &s);
  return (ordinal & 1u) ? s : c;
}

/* A single draw when its partner leg is not used in the same region. */
NT_FN double nt_normal64(nt_key k, nt_u32 ordinal) {
  double c, s;
  nt_normal_pair64(k, ordinal >> 1, &c, &s);
  return (ordinal & 1u) ? s : c;
}

NT_FN float nt_normal32(nt_key k, nt_u32 ordinal) {
  float c, s;
  nt_normal_pair32(k, ordinal >> 1, &c, &s);
  return (ordinal & 1u) ? s : c;
}

NT_FN double nt_uniform64(nt_key k, nt_u32 ordinal) {
  nt_u32 w0, w1;
  nt_philox(k.lo, k.hi ^ (ordinal | NT_UNIFORM_TAG), &w0, &w1);
  return ((double)w0 + 0.5) * NT_UINT_SCALE;
}

NT_FN float nt_uniform32(nt_key k, nt_u32 ordinal) {
  return (float)nt_uniform64(k, ordinal);
}

/* A double from its IEEE-754 bits (non-finite tape constants). */
NT_FN double nt_from_bits64(nt_u64 bits) {
#ifdef NT_HOST
  double x;
  memcpy(&x, &bits, sizeof x);
  return x;
#else
  return __longlong_as_double((long long)bits);
#endif
}

/* Hint the line holding *p into L2 ahead of its load (no register, no wait). */
NT_FN void nt_prefetch_l2(const void* p) {
#ifdef NT_HOST
  (void)p;
#else
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
#endif
}

/* Hint `bytes` bytes from p into L2 as one bulk request (p 16-byte aligned,
 * bytes a multiple of 16): one thread covers a whole contiguous tile. */
NT_FN void nt_prefetch_l2_bulk(const void* p, unsigned bytes) {
#ifdef NT_HOST
  (void)p;
  (void)bytes;
#else
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
#endif
}

/* A value tape whose whole grid's share is at most this many bytes stays in
 * the B200's 126 MB L2 between its forward write and its reverse read (about
 * three quarters of it, leaving room for everything else the kernel touches). */
#define NT_L2_TAPE_BYTES (96ull << 20)

#ifndef NT_HOST
/* Drops this warp's part of ROWS tape rows from L2 without writing them back
 * (discard.global.L2: the lines' contents become undefined).  The reverse
 * sweep of the last output calls it once a segment's taped values are
 * consumed: nothing reads them again before the next path's forward sweep
 * writes them anew, so their write-back to DRAM is wasted traffic.  A warp's
 * part of a row is 32 consecutive values at src + r * BLOCK (the warp's first
 * value at src): 256 bytes in fp64, two 128-byte lines; 128 bytes in fp32.
 * Every line starts on a 128-byte boundary, as the instruction needs: the
 * tile's rows and the warps' parts are multiples of 32 * sizeof(T) bytes from
 * a 256-byte aligned allocation. */
template <typename T, int ROWS, int BLOCK>
NT_FN void nt_discard_rows_l2(const T* src, unsigned lane) {
  constexpr int kLines = 32 * (int)sizeof(T) / 128;
  constexpr int kTotal = ROWS * kLines;
#pragma unroll
  for (int i = 0; i < (kTotal + 31) / 32; ++i) {
    const int c = i * 32 + (int)lane;
    if (c < kTotal) {
      const int r = c / kLines, k = c % kLines;
      const char* line = reinterpret_cast<const char*>(src + (size_t)r * BLOCK) + 128 * k;
      asm volatile("discard.global.L2 [%0], 128;" ::"l"(line) : "memory");
    }
  }
}
#endif

#ifndef NT_HOST
/* Component B of a vector pair (the per-unit constant table's paired loads). */
template <int B> NT_FN double nt_pick(double2 v) { return B ? v.y : v.x; }
template <int B> NT_FN float nt_pick(float2 v) { return B ? v.y : v.x; }
#endif

/* ---- java.lang.Math semantics ------------------------------------------- */

NT_FN bool nt_signbit64(double x) {
#ifdef NT_HOST
  long long bits;
  memcpy(&bits, &x, sizeof bits);
  return bits < 0;
#else
  return __double_as_longlong(x) < 0;
#endif
}

NT_FN bool nt_signbit32(float x) {
#ifdef NT_HOST
  int bits;
  memcpy(&bits, &x, sizeof bits);
  return bits < 0;
#else
  return __float_as_int(x) < 0;
#endif
}

NT_FN double nt_max64(double a, double b) {
  if (a != a) return a;
  if (a == 0.0 && b == 0.0 && nt_signbit64(a)) return b;
  return a >= b ? a : b;
}

NT_FN double nt_min64(double a, double b) {
  if (a != a) return a;
  if (a == 0.0 && b == 0.0 && nt_signbit64(b)) return b;
  return a <= b ? a : b;
}

/* 1 / x correctly rounded: the bits of the IEEE division 1.0f / x. */
NT_FN float nt_rcp32(float x) {
#ifdef NT_HOST
  return 1.0f / x;
#else
  return __frcp_rn(x);
#endif
}

/* a * b rounded once, never contracted into a neighbouring add. */
NT_FN float nt_fmul_rn(float a, float b) {
#ifdef NT_HOST
  return a * b;
#else
  return __fmul_rn(a, b);
#endif
}

NT_FN float nt_max32(float a, float b) {
  if (a != a) return a;
  if (a == 0.0f && b == 0.0f && nt_signbit32(a)) return b;
  return a >= b ? a : b;
}

NT_FN float nt_min32(float a, float b) {
  if (a != a) return a;
  if (a == 0.0f && b == 0.0f && nt_signbit32(b)) return b;
  return a <= b ? a : b;
}

/* Knuth's TwoSum: after the call s + c holds the exact value of the old
 * s + c + x to within the rounding of c.  Per-thread accumulators use it so a
 * thread's running sum over thousands of scenarios keeps full precision. */
NT_FN void nt_two_sum(double* s, double* c, double x) {
  const double t = *s + x;
  const double bp = t - *s;
  *c += (*s - (t - bp)) + (x - bp);
  *s = t;
}

/* ---- deterministic reduction (device only) ------------------------------ */
#ifndef NT_HOST

NT_FN double nt_warp_sum(double x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_down_sync(0xffffffffu, x, off);
  return x;
}

/*
 * Per-path accumulation of the replay kernels, exact and independent of how
 * the path range is split.  A warp replays one tile of 32 consecutive paths
 * of the launch (lanes past the end contribute 0).  For each channel the
 * lanes' values are summed by a fixed xor butterfly (nt_warp_allsum), which
 * leaves the same bits in every lane (each step adds the same two values in
 * either order); lane k % 32 keeps channel k's tile sum in a register until
 * the tile is done, then adds it to the block's exact words (nt_exact.cuh)
 * in shared memory, or straight to the launch's words in global memory when
 * the channels' words do not fit in shared memory (nt_tile_xadd).  A tile's
 * sum depends on its 32 paths alone and the words add exactly, so the
 * launch total is the same whatever grid, chunking or number of GPUs
 * produced it, as long as tiles start at the same paths.  Every lane of the
 * warp must call nt_warp_allsum at the same point.
 */
NT_FN double nt_warp_allsum(double x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

/* Adds this lane's tile sums (channel lane + 32 r in ws[r]) to the words. */
NT_FN void nt_tile_xadd(nt_i64* words, const double* ws, int nws, int channels) {
  const int lane = (int)(threadIdx.x & 31);
#pragma unroll
  for (int r = 0; r < nws; ++r) {
    const int k = lane + 32 * r;
    if (k < channels) nt_exact_add_atomic(words + (nt_u64)k * NT_XWORDS, ws[r]);
  }
}

/*
 * Block -> launch: when `fold` is set, adds the block's exact words (shared,
 * `channels` records of NT_XWORDS) to the launch's words `glim` (global, zero
 * on entry); a kernel whose channels' words do not fit in shared memory adds
 * its tile sums to glim directly and passes fold = 0.  Then the last block to
 * finish (atomic ticket, no waiting) either writes the correctly rounded sums
 * to out[0..channels) (accumulate == 0) or adds the launch's words to the
 * accumulator words `acc` and carries them (accumulate != 0).  It leaves glim
 * and the ticket zero for the next launch.
 */
NT_FN void nt_xgrid_finish(const nt_i64* blk, int fold, int channels, nt_i64* glim, unsigned int* ticket,
                           double* out, nt_i64* acc, int accumulate) {
  __syncthreads();
  const int words = channels * NT_XWORDS;
  if (fold)
    for (int i = threadIdx.x; i < words; i += blockDim.x) {
      const nt_i64 v = blk[i];
      if (v) atomicAdd((nt_x64*)&glim[i], (nt_x64)v);
    }
  __shared__ unsigned int last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(ticket, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int c = threadIdx.x; c < channels; c += blockDim.x) {
    nt_i64* g = glim + (nt_u64)c * NT_XWORDS;
    if (accumulate) {
      nt_i64* a = acc + (nt_u64)c * NT_XWORDS;
      NT_XLOOP
      for (int i = 0; i < NT_XWORDS; ++i) {
        a[i] += __ldcg(&g[i]);
        g[i] = 0;
      }
      nt_exact_normalize(a);
    } else {
      out[c] = nt_exact_round_inplace(g);
      NT_XLOOP
      for (int i = 0; i < NT_XWORDS; ++i) g[i] = 0;
    }
  }
  if (threadIdx.x == 0) *ticket = 0u;
}

/* The multi-market kernel's reduction, whose channel count is a launch
 * argument: per-thread compensated sums kept in a block tile, channel k of
 * this thread being col[2k * stride] + col[(2k + 1) * stride].  Channels pass
 * through the block `chunk` at a time (scratch holds chunk * warps doubles):
 * warp shuffle, then one record per block; the last block to finish (atomic
 * ticket, no waiting) sums the block records in block order and writes (or,
 * when accumulate != 0, adds to) out. */
NT_FN void nt_grid_reduce_cols(const double* col, int stride, int channels, int chunk, double* scratch,
                               double* partials, unsigned int* ticket, double* out, int accumulate) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  for (int c0 = 0; c0 < channels; c0 += chunk) {
    const int n = channels - c0 < chunk ? channels - c0 : chunk;
    for (int c = 0; c < n; ++c) {
      const int k = c0 + c;
      double v = nt_warp_sum(col[(nt_u64)(2 * k) * stride] + col[(nt_u64)(2 * k + 1) * stride]);
      if (lane == 0) scratch[c * warps + warp] = v;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
      double s = 0.0;
      for (int w = 0; w < warps; ++w) s += scratch[c * warps + w];
      partials[(nt_u64)blockIdx.x * channels + c0 + c] = s;
    }
    __syncthreads();
  }
  __shared__ unsigned int last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(ticket, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (last) {
    __threadfence();
    for (int c = threadIdx.x; c < channels; c += blockDim.x) {
      double s = 0.0;
      for (unsigned int b = 0; b < gridDim.x; ++b) s += __ldcg(&partials[(nt_u64)b * channels + c]);
      out[c] = accumulate ? out[c] + s : s;
    }
    if (threadIdx.x == 0) *ticket = 0u;
  }
}

#endif /* !NT_HOST */

#endif /* NT_DEVICE_RT_CUH */
