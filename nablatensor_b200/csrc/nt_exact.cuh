/*
 * nt_exact.cuh -- exact, order-independent summation of doubles.
 *
 * A sum is kept as a fixed-point integer over the whole double range: 66
 * signed 64-bit words ("digits"), digit k weighing 2^(32k - 1074), so bit 0
 * is the smallest subnormal and the top digit reaches past the largest
 * double.  Adding a double is exact: its 53-bit significand, shifted to its
 * exponent, lands in three consecutive digits as three integers below 2^32.
 * Integer addition is associative, so the sum of a set of doubles does not
 * depend on the order, the grouping or the number of threads, blocks, chunks
 * or GPUs that added them; two sums are merged by adding word by word
 * (atomically on the GPU, or with one int64 all-reduce across ranks).
 * Digits hold up to 2^31 additions before nt_exact_normalize must carry them
 * into the range [0, 2^32) (the top digit keeps the sign).  Words 66-68
 * count the NaN, +inf and -inf addends, so that merging two sums stays a
 * word-by-word addition: the result is NaN after a NaN or after both
 * infinities, else the infinity seen, as an IEEE sum would give.
 * nt_exact_to_double rounds the exact sum to the nearest double (ties to
 * even), so the result is the correctly rounded sum of every addend.
 *
 * Used by the replay kernels (nt_device_rt.cuh) and by the host code that
 * reads device accumulators back (nt_exec.cpp).  Host builds define NT_HOST.
 */
#ifndef NT_EXACT_CUH
#define NT_EXACT_CUH

#ifndef NT_FN
#ifdef NT_HOST
#define NT_FN static inline
#else
#define NT_FN static __device__ __forceinline__
#endif
#endif

#ifdef NT_HOST
#include <string.h>
#endif

/* Loops over the words stay rolled on the device: they run once per channel
 * at the end of a launch, and unrolled they would set the register budget of
 * the whole replay kernel. */
#if defined(__CUDA_ARCH__)
#define NT_XLOOP _Pragma("unroll 1")
#else
#define NT_XLOOP
#endif

#define NT_XDIGITS 66
#define NT_XWORDS 69 /* digits, then the counts of NaN, +inf and -inf addends */
#define NT_XNAN 66
#define NT_XPINF 67
#define NT_XNINF 68

typedef long long nt_i64;
typedef unsigned long long nt_x64;

NT_FN nt_x64 nt_x_bits(double x) {
#ifdef NT_HOST
  nt_x64 b;
  memcpy(&b, &x, sizeof b);
  return b;
#else
  return (nt_x64)__double_as_longlong(x);
#endif
}

NT_FN double nt_x_from_bits(nt_x64 b) {
#ifdef NT_HOST
  double x;
  memcpy(&x, &b, sizeof x);
  return x;
#else
  return __longlong_as_double((long long)b);
#endif
}

NT_FN int nt_x_clz(nt_x64 v) {
#ifdef NT_HOST
  return v ? __builtin_clzll(v) : 64;
#else
  return __clzll((long long)v);
#endif
}

/*
 * Splits x into digit contributions: returns 0 for a zero (nothing to add),
 * 1 with *k and d[0..2] set for a finite x (add d[j] to digit k + j), or 2
 * with *k set to the count word of an infinity or NaN (add 1 to it).
 */
NT_FN int nt_exact_split(double x, int* k, nt_i64 d[3]) {
  const nt_x64 b = nt_x_bits(x);
  const int e = (int)((b >> 52) & 0x7ff);
  const nt_x64 f = b & 0xfffffffffffffull;
  if (e == 0x7ff) {
    *k = f ? NT_XNAN : ((b >> 63) ? NT_XNINF : NT_XPINF);
    return 2;
  }
  const nt_x64 m = e ? (f | 0x10000000000000ull) : f;
  if (m == 0) return 0;
  const int p = e ? e - 1 : 0; /* position of the significand's bit 0 above 2^-1074 */
  const int sh = p & 31;
  const nt_x64 lo = m << sh;
  const nt_x64 hi = sh ? (m >> (64 - sh)) : 0ull;
  nt_i64 d0 = (nt_i64)(lo & 0xffffffffull), d1 = (nt_i64)(lo >> 32), d2 = (nt_i64)hi;
  if (b >> 63) {
    d0 = -d0;
    d1 = -d1;
    d2 = -d2;
  }
  *k = p >> 5;
  d[0] = d0;
  d[1] = d1;
  d[2] = d2;
  return 1;
}

/* Adds x to the words a[0..NT_XWORDS) without atomics (one thread owns a). */
NT_FN void nt_exact_add(nt_i64* a, double x) {
  int k = 0;
  nt_i64 d[3];
  const int r = nt_exact_split(x, &k, d);
  if (r == 1) {
    a[k] += d[0];
    a[k + 1] += d[1];
    a[k + 2] += d[2];
  } else if (r == 2) {
    a[k] += 1;
  }
}

/* Carries every digit but the top one into [0, 2^32); the value is unchanged. */
NT_FN void nt_exact_normalize(nt_i64* a) {
  NT_XLOOP
  for (int i = 0; i < NT_XDIGITS - 1; ++i) {
    const nt_i64 carry = a[i] >> 32; /* floor division by 2^32 */
    a[i] -= (nt_i64)((nt_x64)carry << 32);
    a[i + 1] += carry;
  }
}

/*
 * The exact sum held in w[0..NT_XWORDS), rounded to the nearest double (ties
 * to even); +0 for an exact zero.  The digits are carried in place, and a
 * negative sum is negated in place, so `w` no longer holds the sum afterwards
 * (the device rounds a launch's words this way, in global memory, instead of
 * copying them to local memory).
 */
NT_FN double nt_exact_round_inplace(nt_i64* w) {
  if (w[NT_XNAN] || (w[NT_XPINF] && w[NT_XNINF])) return nt_x_from_bits(0x7ff8000000000000ull);
  if (w[NT_XPINF]) return nt_x_from_bits(0x7ff0000000000000ull);
  if (w[NT_XNINF]) return nt_x_from_bits(0xfff0000000000000ull);
  nt_exact_normalize(w);
  nt_x64 sign = 0;
  if (w[NT_XDIGITS - 1] < 0) {
    sign = 1ull << 63;
    NT_XLOOP
    for (int i = 0; i < NT_XDIGITS; ++i) w[i] = -w[i];
    nt_exact_normalize(w);
  }
  int h = NT_XDIGITS - 1;
  while (h >= 0 && w[h] == 0) --h;
  if (h < 0) return 0.0;
  if ((nt_x64)w[NT_XDIGITS - 1] >> 32) return nt_x_from_bits(sign | 0x7ff0000000000000ull);
  /* The top 96 bits: digits h, h-1 (a 64-bit word) and h-2; below them only
   * whether anything is non-zero matters. */
  const nt_x64 top = ((nt_x64)w[h] << 32) | (nt_x64)(h >= 1 ? w[h - 1] : 0);
  const nt_x64 low = (nt_x64)(h >= 2 ? w[h - 2] : 0);
  int sticky = 0;
  NT_XLOOP
  for (int i = 0; i < h - 2; ++i) sticky |= w[i] != 0;
  const int lz = nt_x_clz(top);           /* in [0, 31]: w[h] is non-zero and below 2^32 */
  const int msb = 32 * (h - 1) + 63 - lz; /* bit position of the leading one above 2^-1074 */
  if (msb < 52) {
    /* Below 2^-1022: a subnormal, exact (bit 0 is 2^-1074).  Only digits 0
     * and 1 can be non-zero here. */
    return nt_x_from_bits(sign | ((nt_x64)(h >= 1 ? w[1] : 0) << 32) | (nt_x64)w[0]);
  }
  const nt_x64 head = lz ? ((top << lz) | (low >> (32 - lz))) : top; /* bits msb-63 .. msb */
  const nt_x64 rest = (low << (32 + lz)) & 0xffffffff00000000ull;  /* the bits of `low` below head */
  nt_x64 mant = head >> 11;                                         /* 53 bits */
  const nt_x64 round = head & 0x7ffull;
  const int guard = (int)(round >> 10);
  const int below = (round & 0x3ffull) != 0 || rest != 0 || sticky;
  int ex = msb - 51; /* biased exponent of 2^(msb - 1074) */
  if (guard && (below || (mant & 1ull))) {
    ++mant;
    if (mant >> 53) {
      mant >>= 1;
      ++ex;
    }
  }
  if (ex >= 0x7ff) return nt_x_from_bits(sign | 0x7ff0000000000000ull);
  return nt_x_from_bits(sign | ((nt_x64)ex << 52) | (mant & 0xfffffffffffffull));
}

/* The exact sum held in a[0..NT_XWORDS), rounded to the nearest double (ties
 * to even); `a` is not modified. */
NT_FN double nt_exact_to_double(const nt_i64* a) {
  nt_i64 w[NT_XWORDS];
  for (int i = 0; i < NT_XWORDS; ++i) w[i] = a[i];
  return nt_exact_round_inplace(w);
}

#ifndef NT_HOST
/* Adds x to the words a[0..NT_XWORDS) in shared or global memory with
 * atomics; any number of threads may add to the same words at once. */
NT_FN void nt_exact_add_atomic(nt_i64* a, double x) {
  int k = 0;
  nt_i64 d[3];
  const int r = nt_exact_split(x, &k, d);
  if (r == 1) {
    if (d[0]) atomicAdd((nt_x64*)&a[k], (nt_x64)d[0]);
    if (d[1]) atomicAdd((nt_x64*)&a[k + 1], (nt_x64)d[1]);
    if (d[2]) atomicAdd((nt_x64*)&a[k + 2], (nt_x64)d[2]);
  } else if (r == 2) {
    atomicAdd((nt_x64*)&a[k], 1ull);
  }
}
#endif

#endif /* NT_EXACT_CUH */
