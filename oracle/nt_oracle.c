/*
 * nt_oracle.c -- CPU restatement of NablaTensor's scalar `cpu` engine.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker, never the product).  See
 * nt_oracle.h for the reference files each function restates.
 */
#define _GNU_SOURCE
#include "nt_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* Philox.java:30 -- 2^-32 as a double literal. */
static const double UINT_SCALE = 2.3283064365386963e-10;
/* Philox.java:31 -- high tag that separates uniform counters from normal ones. */
static const uint32_t UNIFORM_TAG = 0x40000000u;

/* Philox.java:62-70: ten rounds of (hi, lo) = M * x0; x0 = hi ^ key ^ x1; x1 = lo; key += W. */
void orc_philox2x32_10(uint32_t x0, uint32_t x1, uint32_t key, uint32_t out[2]) {
  for (int i = 0; i < 10; i++) {
    uint64_t product = (uint64_t)0xD256D193u * (uint64_t)x0;
    uint32_t high = (uint32_t)(product >> 32);
    uint32_t low = (uint32_t)product;
    x0 = high ^ key ^ x1;
    x1 = low;
    key += 0x9E3779B9u;
  }
  out[0] = x0;
  out[1] = x1;
}

/* Philox.java:45-54. */
void orc_stream_words(uint64_t path, uint64_t seed, int32_t stream, uint32_t* lo, uint32_t* hi) {
  uint32_t l = (uint32_t)path ^ (uint32_t)seed;
  uint32_t h = (uint32_t)(path >> 32) ^ (uint32_t)(seed >> 32);
  if (stream != 0) {
    h ^= (uint32_t)stream * 0x9E3779B1u; /* Java int multiply wraps mod 2^32 */
  }
  *lo = l;
  *hi = h;
}

void orc_normal_words(uint64_t path, uint64_t seed, int32_t stream, uint32_t pair, uint32_t out[2]) {
  uint32_t lo, hi;
  orc_stream_words(path, seed, stream, &lo, &hi);
  orc_philox2x32_10(lo, hi ^ pair, 0x1BD11BDAu, out);
}

/* Box-Muller of one Philox block: Philox.java:71-77. */
static void box_muller(const uint32_t w[2], double* cos_leg, double* sin_leg) {
  double u1 = ((double)w[0] + 0.5) * UINT_SCALE;
  double u2 = ((double)w[1] + 0.5) * UINT_SCALE;
  double radius = sqrt(-2.0 * log(u1));
  double angle = 6.283185307179586 * u2;
  *sin_leg = radius * sin(angle);
  *cos_leg = radius * cos(angle);
}

double orc_normal(uint64_t path, uint64_t seed, int32_t stream, uint32_t k) {
  uint32_t w[2];
  double c, s;
  orc_normal_words(path, seed, stream, k >> 1, w);
  box_muller(w, &c, &s);
  return (k & 1u) ? s : c;
}

double orc_uniform(uint64_t path, uint64_t seed, int32_t stream, uint32_t k) {
  uint32_t lo, hi, w[2];
  orc_stream_words(path, seed, stream, &lo, &hi);
  orc_philox2x32_10(lo, hi ^ (k | UNIFORM_TAG), 0x1BD11BDAu, w);
  return ((double)w[0] + 0.5) * UINT_SCALE;
}

/* A stateful stream, Philox.java:33-78: a normal pair per counter, the sine
 * leg kept as a spare for the next call. */
typedef struct orc_stream {
  uint32_t lo, hi;
  uint32_t counter;
  uint32_t uniform_counter;
  double spare;
  int has;
} orc_stream;

static void stream_init(orc_stream* s, uint64_t path, uint64_t seed, int32_t stream) {
  orc_stream_words(path, seed, stream, &s->lo, &s->hi);
  s->counter = 0;
  s->uniform_counter = 0;
  s->has = 0;
  s->spare = 0.0;
}

static double stream_normal(orc_stream* s) {
  if (s->has) {
    s->has = 0;
    return s->spare;
  }
  uint32_t w[2];
  orc_philox2x32_10(s->lo, s->hi ^ s->counter++, 0x1BD11BDAu, w);
  double c, sn;
  box_muller(w, &c, &sn);
  s->spare = sn;
  s->has = 1;
  return c;
}

static double stream_uniform(orc_stream* s) {
  uint32_t w[2];
  orc_philox2x32_10(s->lo, s->hi ^ (s->uniform_counter++ | UNIFORM_TAG), 0x1BD11BDAu, w);
  return ((double)w[0] + 0.5) * UINT_SCALE;
}

/* java.lang.Math.max / min: NaN-propagating, -0.0 < +0.0. */
static double java_max(double a, double b) {
  if (a != a) return a;
  if (a == 0.0 && b == 0.0 && signbit(a)) return b;
  return a >= b ? a : b;
}

static double java_min(double a, double b) {
  if (a != a) return a;
  if (a == 0.0 && b == 0.0 && signbit(b)) return b;
  return a <= b ? a : b;
}

void orc_mark_active(const orc_tape* t, uint8_t* active) {
  for (int32_t i = 0; i < t->n; i++) {
    switch (t->op[i]) {
      case ORC_INPUT: active[i] = 1; break;
      case ORC_CONST: case ORC_RANDN: case ORC_RANDU: active[i] = 0; break;
      case ORC_NEG: case ORC_EXP: case ORC_LOG: case ORC_SQRT: case ORC_ABS:
        active[i] = active[t->arg_a[i]];
        break;
      default:
        active[i] = active[t->arg_a[i]] || active[t->arg_b[i]];
    }
  }
}

static int validate(const orc_tape* t) {
  if (t->n <= 0 || t->n_out <= 0 || t->n_in < 0 || t->n_streams <= 0) return -1;
  for (int32_t i = 0; i < t->n; i++) {
    int32_t op = t->op[i];
    if (op < ORC_CONST || op > ORC_ABS) return -2;
    int unary = op == ORC_NEG || op == ORC_EXP || op == ORC_LOG || op == ORC_SQRT || op == ORC_ABS;
    int binary = op >= ORC_ADD && op <= ORC_MIN && !unary;
    if ((unary || binary) && (t->arg_a[i] < 0 || t->arg_a[i] >= i)) return -3;
    if (binary && (t->arg_b[i] < 0 || t->arg_b[i] >= i)) return -3;
    if (op == ORC_INPUT && (t->arg_a[i] < 0 || t->arg_a[i] >= t->n_in)) return -4;
    if ((op == ORC_RANDN || op == ORC_RANDU) && (t->arg_b[i] < 0 || t->arg_b[i] >= t->n_streams)) return -5;
  }
  for (int32_t o = 0; o < t->n_out; o++)
    if (t->output_node[o] < 0 || t->output_node[o] >= t->n) return -6;
  for (int32_t j = 0; j < t->n_in; j++)
    if (t->input_node[j] < 0 || t->input_node[j] >= t->n) return -7;
  return 0;
}

typedef struct range_job {
  const orc_tape* t;
  const uint8_t* active;
  const double* inputs;
  int f32, adjoints, exact;
  uint64_t from, count, seed, path_offset;
  double* sums;     /* n_out * (2 + n_in), private to the job */
  double* comp;     /* compensation terms (exact mode) */
  double* per_path; /* global array or NULL */
} range_job;

/* Knuth's TwoSum: s + c carries the exact sum of s and x. */
static inline void two_sum_add(double* s, double* c, double x) {
  double t = *s + x;
  double bp = t - *s;
  *c += (*s - (t - bp)) + (x - bp);
  *s = t;
}

/* Accumulate into channel k: naive (the reference's AadTotals) or compensated. */
static inline void acc_add(range_job* job, int k, double x) {
  if (job->exact) two_sum_add(&job->sums[k], &job->comp[k], x);
  else job->sums[k] += x;
}

/* ScalarReplay.add (ScalarReplay.java:177-183). */
static inline void add_adj(double* d, int32_t node, double c, int f32) {
  if (f32) d[node] = (double)(float)(d[node] + (double)(float)c);
  else d[node] += c;
}

/* ScalarReplay.run (ScalarReplay.java:78-174) over one contiguous range. */
static void* run_range(void* arg) {
  range_job* job = (range_job*)arg;
  const orc_tape* t = job->t;
  const int32_t n = t->n, n_in = t->n_in, n_out = t->n_out;
  const int f32 = job->f32;
  double* v = (double*)calloc((size_t)n, sizeof(double));
  double* d = (double*)calloc((size_t)n, sizeof(double));
  orc_stream* rng = (orc_stream*)calloc((size_t)t->n_streams, sizeof(orc_stream));
  const int stride = 2 + n_in;
  for (uint64_t path = job->from; path < job->from + job->count; path++) {
    for (int32_t s = 0; s < t->n_streams; s++) stream_init(&rng[s], path, job->seed, s);
    for (int32_t i = 0; i < n; i++) {
      int32_t a = t->arg_a[i], b = t->arg_b[i];
      double value;
      switch (t->op[i]) {
        case ORC_CONST: value = t->constant[i]; break;
        case ORC_INPUT: value = job->inputs[a]; break;
        case ORC_RANDN: value = stream_normal(&rng[b]); break;
        case ORC_RANDU: value = stream_uniform(&rng[b]); break;
        case ORC_ADD: value = v[a] + v[b]; break;
        case ORC_SUB: value = v[a] - v[b]; break;
        case ORC_MUL: value = v[a] * v[b]; break;
        case ORC_DIV: value = v[a] / v[b]; break;
        case ORC_NEG: value = -v[a]; break;
        case ORC_EXP: value = exp(v[a]); break;
        case ORC_LOG: value = log(v[a]); break;
        case ORC_SQRT: value = sqrt(v[a]); break;
        case ORC_ABS: value = fabs(v[a]); break;
        case ORC_MAX: value = java_max(v[a], v[b]); break;
        case ORC_MIN: value = java_min(v[a], v[b]); break;
        default: value = NAN;
      }
      v[i] = f32 ? (double)(float)value : value;
    }
    double* pp = job->per_path ? job->per_path + (path - job->path_offset) * (uint64_t)(n_out * (1 + n_in)) : NULL;
    for (int32_t o = 0; o < n_out; o++) {
      double y = v[t->output_node[o]];
      acc_add(job, o * stride + 0, y);
      acc_add(job, o * stride + 1, y * y);
      if (pp) pp[o * (1 + n_in)] = y;
    }
    if (!job->adjoints) continue;
    for (int32_t o = 0; o < n_out; o++) {
      memset(d, 0, (size_t)n * sizeof(double));
      d[t->output_node[o]] = 1.0;
      for (int32_t i = n - 1; i >= 0; i--) {
        double adj = d[i];
        if (adj == 0.0 || !job->active[i]) continue;
        int32_t a = t->arg_a[i], b = t->arg_b[i];
        switch (t->op[i]) {
          case ORC_ADD: add_adj(d, a, adj, f32); add_adj(d, b, adj, f32); break;
          case ORC_SUB: add_adj(d, a, adj, f32); add_adj(d, b, -adj, f32); break;
          case ORC_MUL: add_adj(d, a, adj * v[b], f32); add_adj(d, b, adj * v[a], f32); break;
          case ORC_DIV: add_adj(d, a, adj / v[b], f32); add_adj(d, b, -adj * v[i] / v[b], f32); break;
          case ORC_NEG: add_adj(d, a, -adj, f32); break;
          case ORC_EXP: add_adj(d, a, adj * v[i], f32); break;
          case ORC_LOG: add_adj(d, a, adj / v[a], f32); break;
          case ORC_SQRT: add_adj(d, a, adj * 0.5 / v[i], f32); break;
          case ORC_ABS: add_adj(d, a, v[a] < 0.0 ? -adj : adj, f32); break;
          case ORC_MAX: add_adj(d, v[a] >= v[b] ? a : b, adj, f32); break;
          case ORC_MIN: add_adj(d, v[a] <= v[b] ? a : b, adj, f32); break;
          default: break;
        }
      }
      for (int32_t j = 0; j < n_in; j++) {
        double g = d[t->input_node[j]];
        acc_add(job, o * stride + 2 + j, g);
        if (pp) pp[o * (1 + n_in) + 1 + j] = g;
      }
    }
  }
  free(v);
  free(d);
  free(rng);
  return NULL;
}

int orc_replay(const orc_tape* t, const double* inputs, int f32, int adjoints,
               uint64_t paths, uint64_t path_offset, uint64_t seed, int threads,
               double* sums, double* per_path) {
  return orc_replay_ex(t, inputs, f32, adjoints, paths, path_offset, seed, threads, 0, sums, per_path);
}

int orc_replay_ex(const orc_tape* t, const double* inputs, int f32, int adjoints,
                  uint64_t paths, uint64_t path_offset, uint64_t seed, int threads, int exact,
                  double* sums, double* per_path) {
  int rc = validate(t);
  if (rc) return rc;
  if (paths == 0) return -8;
  uint8_t* active = (uint8_t*)malloc((size_t)t->n);
  orc_mark_active(t, active);
  if (threads <= 0) threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (threads < 1) threads = 1;
  const size_t width = (size_t)t->n_out * (size_t)(2 + t->n_in);
  memset(sums, 0, width * sizeof(double));

  /* HostAadExecutable.runRanges: units split as evenly as possible, the
   * first `extra` threads taking one more; totals combined in thread order. */
  uint64_t each = paths / (uint64_t)threads, extra = paths % (uint64_t)threads;
  range_job* jobs = (range_job*)calloc((size_t)threads, sizeof(range_job));
  pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  uint64_t cursor = path_offset, remaining = paths;
  int launched = 0;
  for (int k = 0; k < threads && remaining > 0; k++) {
    uint64_t count = each + ((uint64_t)k < extra ? 1 : 0);
    if (count > remaining) count = remaining;
    if (count == 0) continue;
    range_job* j = &jobs[launched];
    j->t = t; j->active = active; j->inputs = inputs; j->f32 = f32; j->adjoints = adjoints; j->exact = exact;
    j->from = cursor; j->count = count; j->seed = seed; j->path_offset = path_offset;
    j->sums = (double*)calloc(width, sizeof(double));
    j->comp = (double*)calloc(width, sizeof(double));
    j->per_path = per_path;
    cursor += count;
    remaining -= count;
    launched++;
  }
  if (launched == 1) {
    run_range(&jobs[0]);
  } else {
    for (int k = 0; k < launched; k++) pthread_create(&tids[k], NULL, run_range, &jobs[k]);
    for (int k = 0; k < launched; k++) pthread_join(tids[k], NULL);
  }
  if (exact) {
    /* Double-double combine of every job's (sum, compensation) pair. */
    double* hi = (double*)calloc(width, sizeof(double));
    double* lo = (double*)calloc(width, sizeof(double));
    for (int k = 0; k < launched; k++)
      for (size_t c = 0; c < width; c++) {
        two_sum_add(&hi[c], &lo[c], jobs[k].sums[c]);
        two_sum_add(&hi[c], &lo[c], jobs[k].comp[c]);
      }
    for (size_t c = 0; c < width; c++) sums[c] = hi[c] + lo[c];
    free(hi);
    free(lo);
  } else {
    for (int k = 0; k < launched; k++)
      for (size_t c = 0; c < width; c++) sums[c] += jobs[k].sums[c];
  }
  for (int k = 0; k < launched; k++) {
    free(jobs[k].sums);
    free(jobs[k].comp);
  }
  free(jobs);
  free(tids);
  free(active);
  return 0;
}

/* AadTotals.toResult (AadTotals.java:68-89). */
void orc_finish(int32_t n_out, int32_t n_in, const double* sums, uint64_t paths,
                double* mean, double* stderr_out, double* gradients) {
  const int stride = 2 + n_in;
  for (int32_t o = 0; o < n_out; o++) {
    double m = sums[o * stride] / (double)paths;
    mean[o] = m;
    if (paths > 1) {
      double variance = (sums[o * stride + 1] - (double)paths * m * m) / (double)(paths - 1);
      stderr_out[o] = sqrt(fmax(0.0, variance) / (double)paths);
    } else {
      stderr_out[o] = NAN;
    }
    for (int32_t j = 0; j < n_in; j++) gradients[o * n_in + j] = sums[o * stride + 2 + j] / (double)paths;
  }
}

/* ---- tape producers ------------------------------------------------------ */

static int32_t put(orc_tape_buf* t, int32_t op, int32_t a, int32_t b, double c) {
  if (t->n >= t->cap) return -1;
  t->op[t->n] = op;
  t->arg_a[t->n] = a;
  t->arg_b[t->n] = b;
  t->constant[t->n] = c;
  return t->n++;
}

#define PUT(op, a, b, c)                                   \
  ({ int32_t _r = put(t, (op), (a), (b), (c)); if (_r < 0) return -1; _r; })

typedef struct sim {
  int32_t spot, strike, vol, rate, maturity;
  int32_t drift, diffusion;
  int32_t draws;
} sim;

/* Nabla.Inputs (Nabla.java:201-207) with EquityMarket's field order, then
 * GbmPath's uniform-grid set-up (GbmPath.java:48-58). */
static int sim_setup(orc_tape_buf* t, sim* s, int steps) {
  t->n = 0;
  t->n_in = 5;
  s->draws = 0;
  s->spot = PUT(ORC_INPUT, 0, -1, 100.0);
  s->strike = PUT(ORC_INPUT, 1, -1, 100.0);
  s->vol = PUT(ORC_INPUT, 2, -1, 0.20);
  s->rate = PUT(ORC_INPUT, 3, -1, 0.03);
  s->maturity = PUT(ORC_INPUT, 4, -1, 1.0);
  for (int j = 0; j < 5; j++) t->input_node[j] = j;
  int32_t vv = PUT(ORC_MUL, s->vol, s->vol, 0.0);
  int32_t half = PUT(ORC_CONST, -1, -1, 0.5);
  int32_t hv = PUT(ORC_MUL, vv, half, 0.0);
  int32_t half_var = PUT(ORC_SUB, s->rate, hv, 0.0);
  int32_t frac = PUT(ORC_CONST, -1, -1, 1.0 / steps);
  int32_t dt = PUT(ORC_MUL, s->maturity, frac, 0.0);
  s->drift = PUT(ORC_MUL, half_var, dt, 0.0);
  int32_t sq = PUT(ORC_SQRT, dt, -1, 0.0);
  s->diffusion = PUT(ORC_MUL, s->vol, sq, 0.0);
  return 0;
}

/* GbmPath.step (GbmPath.java:89-91): spot * exp(drift + diffusion * z). */
static int32_t gbm_step(orc_tape_buf* t, sim* s, int32_t spot) {
  int32_t z = PUT(ORC_RANDN, s->draws++, 0, 0.0);
  int32_t m = PUT(ORC_MUL, s->diffusion, z, 0.0);
  int32_t a = PUT(ORC_ADD, s->drift, m, 0.0);
  int32_t e = PUT(ORC_EXP, a, -1, 0.0);
  return PUT(ORC_MUL, spot, e, 0.0);
}

/* Products.intrinsic: max(sign * (x - K), 0). */
static int32_t intrinsic(orc_tape_buf* t, int call, int32_t x, int32_t strike) {
  int32_t diff = call ? PUT(ORC_SUB, x, strike, 0.0) : PUT(ORC_SUB, strike, x, 0.0);
  int32_t zero = PUT(ORC_CONST, -1, -1, 0.0);
  return PUT(ORC_MAX, diff, zero, 0.0);
}

/* Sim.discount: payoff * exp(-rate * maturity). */
static int32_t discount(orc_tape_buf* t, sim* s, int32_t payoff) {
  int32_t nr = PUT(ORC_NEG, s->rate, -1, 0.0);
  int32_t rt = PUT(ORC_MUL, nr, s->maturity, 0.0);
  int32_t df = PUT(ORC_EXP, rt, -1, 0.0);
  return PUT(ORC_MUL, payoff, df, 0.0);
}

/* Products.european (Products.java:70-80). */
int orc_build_european(orc_tape_buf* t, int steps, int call) {
  sim s;
  if (sim_setup(t, &s, steps)) return -1;
  int32_t path = s.spot;
  for (int k = 0; k < steps; k++) {
    path = gbm_step(t, &s, path);
    if (path < 0) return -1;
  }
  int32_t pay = intrinsic(t, call, path, s.strike);
  if (pay < 0) return -1;
  int32_t out = discount(t, &s, pay);
  if (out < 0) return -1;
  t->output_node = out;
  return t->n;
}

/* Products.asian (Products.java:82-94). */
int orc_build_asian(orc_tape_buf* t, int steps, int call) {
  sim s;
  if (sim_setup(t, &s, steps)) return -1;
  int32_t path = s.spot;
  int32_t sum = PUT(ORC_CONST, -1, -1, 0.0);
  for (int k = 0; k < steps; k++) {
    path = gbm_step(t, &s, path);
    if (path < 0) return -1;
    sum = PUT(ORC_ADD, sum, path, 0.0);
  }
  int32_t n = PUT(ORC_CONST, -1, -1, (double)steps);
  int32_t avg = PUT(ORC_DIV, sum, n, 0.0);
  int32_t pay = intrinsic(t, call, avg, s.strike);
  if (pay < 0) return -1;
  int32_t out = discount(t, &s, pay);
  if (out < 0) return -1;
  t->output_node = out;
  return t->n;
}

/* Smooth.step (Smooth.java:44-48): 1 / (1 + exp(-x / width)). */
static int32_t smooth_step(orc_tape_buf* t, int32_t x, double width) {
  int32_t w = PUT(ORC_CONST, -1, -1, width);
  int32_t q = PUT(ORC_DIV, x, w, 0.0);
  int32_t nq = PUT(ORC_NEG, q, -1, 0.0);
  int32_t e = PUT(ORC_EXP, nq, -1, 0.0);
  int32_t one = PUT(ORC_CONST, -1, -1, 1.0);
  int32_t one2 = PUT(ORC_CONST, -1, -1, 1.0);
  int32_t den = PUT(ORC_ADD, e, one2, 0.0);
  return PUT(ORC_DIV, one, den, 0.0);
}

/* ExoticProducts.createBarrier (ExoticProducts.java:55-75) with Smooth.gt/lt
 * against a constant level (Smooth.java:56-63). */
int orc_build_barrier(orc_tape_buf* t, int steps, int call, int kind, double barrier, double width) {
  sim s;
  if (sim_setup(t, &s, steps)) return -1;
  int32_t path = s.spot;
  int32_t survival = PUT(ORC_CONST, -1, -1, 1.0);
  int up = kind == 0 || kind == 1;
  for (int k = 0; k < steps; k++) {
    path = gbm_step(t, &s, path);
    if (path < 0) return -1;
    int32_t x;
    if (up) {
      int32_t neg = PUT(ORC_NEG, path, -1, 0.0);
      int32_t lvl = PUT(ORC_CONST, -1, -1, barrier);
      x = PUT(ORC_ADD, neg, lvl, 0.0);
    } else {
      int32_t lvl = PUT(ORC_CONST, -1, -1, barrier);
      x = PUT(ORC_SUB, path, lvl, 0.0);
    }
    int32_t not_breached = smooth_step(t, x, width);
    if (not_breached < 0) return -1;
    survival = PUT(ORC_MUL, survival, not_breached, 0.0);
  }
  int32_t vanilla = intrinsic(t, call, path, s.strike);
  if (vanilla < 0) return -1;
  int knock_out = kind == 0 || kind == 2;
  int32_t alive;
  if (knock_out) {
    alive = survival;
  } else {
    int32_t one = PUT(ORC_CONST, -1, -1, 1.0);
    alive = PUT(ORC_SUB, one, survival, 0.0);
  }
  int32_t pay = PUT(ORC_MUL, vanilla, alive, 0.0);
  int32_t out = discount(t, &s, pay);
  if (out < 0) return -1;
  t->output_node = out;
  return t->n;
}
