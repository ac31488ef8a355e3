/*
 * nt_oracle.h -- CPU restatement of NablaTensor's scalar `cpu` engine.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 engine in nablatensor_b200/.  Only tests/, __graft_entry__.smoke() and
 * the cpu_baseline / --impl reference legs of bench.py may load it; the
 * product path never links, calls or falls back to it.
 *
 * What it restates (paths relative to the reference project root):
 *   - Philox2x32-10 + Box-Muller normal / tagged uniform draws:
 *       nablatensor-engine-cpu/src/main/java/com/nablatensor/engine/cpu/Philox.java:29-95
 *   - the scalar forward / adjoint interpreter, fp32 rounding rules, the
 *     d==0 / inactive skip and the MAX/MIN tie rules:
 *       nablatensor-engine-cpu/src/main/java/com/nablatensor/engine/cpu/ScalarReplay.java:78-183
 *   - per-thread contiguous path ranges combined in thread order:
 *       nablatensor-core/src/main/java/com/nablatensor/engine/HostAadExecutable.java:85-117
 *   - mean / standard error / gradient normalisation:
 *       nablatensor-core/src/main/java/com/nablatensor/engine/AadTotals.java:68-89
 *   - active-node marking:
 *       nablatensor-core/src/main/java/com/nablatensor/engine/AadTape.java:70-81
 *   - tape producers (node order) for the equity products:
 *       nablatensor-quant/.../quant/Products.java:70-161, GbmPath.java:48-91,
 *       ExoticProducts.java:55-75, nablatensor-ops/.../ops/Smooth.java:44-68,
 *       nablatensor-core/.../engine/Nabla.java:201-207 (inputs first, in
 *       EquityMarket field order spot, strike, vol, rate, maturity).
 *
 * Transcendentals come from the C library (glibc libm) where the reference
 * calls java.lang.Math; both are within 1 ulp of the exact result, so the
 * uint32 Philox words are bit-exact and the doubles agree to a few ulps per
 * call.  Parity is pinned to the reference's published golden results
 * (docs/validation.md:56-63, docs/examples/asian-greeks.md:43-46).
 */
#ifndef NT_ORACLE_H
#define NT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Op codes: the ordinal order of AadOpEnum (nablatensor-core/.../AadOpEnum.java:19-50). */
enum {
  ORC_CONST = 0, ORC_INPUT = 1, ORC_RANDN = 2, ORC_RANDU = 3, ORC_ADD = 4, ORC_SUB = 5,
  ORC_MUL = 6, ORC_DIV = 7, ORC_NEG = 8, ORC_EXP = 9, ORC_LOG = 10, ORC_SQRT = 11,
  ORC_MAX = 12, ORC_MIN = 13, ORC_ABS = 14
};

/* A flat tape, the FlatTape.java:37-79 layout.  For RANDN/RANDU argA is the
 * draw ordinal within (stream, kind) and argB the stream; for INPUT argA is the
 * input index. */
typedef struct orc_tape {
  int32_t n;
  const int32_t* op;
  const int32_t* arg_a;
  const int32_t* arg_b;
  const double* constant;
  int32_t n_in;
  const int32_t* input_node;
  int32_t n_out;
  const int32_t* output_node;
  int32_t n_streams;
} orc_tape;

/* One Philox2x32-10 block: counter (x0, x1), initial key, 10 rounds. */
void orc_philox2x32_10(uint32_t x0, uint32_t x1, uint32_t key, uint32_t out[2]);

/* Stream key words for (path, seed, stream): Philox.java:41-54. */
void orc_stream_words(uint64_t path, uint64_t seed, int32_t stream, uint32_t* lo, uint32_t* hi);

/* The uint32 words of normal pair `pair` (draw ordinals 2*pair, 2*pair+1). */
void orc_normal_words(uint64_t path, uint64_t seed, int32_t stream, uint32_t pair, uint32_t out[2]);

/* Draw `k` of the normal sequence of (path, seed, stream), as Philox.normal()
 * returns it on its k-th call. */
double orc_normal(uint64_t path, uint64_t seed, int32_t stream, uint32_t k);

/* Draw `k` of the uniform sequence (Philox.uniform()). */
double orc_uniform(uint64_t path, uint64_t seed, int32_t stream, uint32_t k);

/* Active flags (AadTape.markActive). `active` has tape->n entries. */
void orc_mark_active(const orc_tape* tape, uint8_t* active);

/*
 * Replay `paths` scenarios starting at `path_offset`, exactly as
 * ScalarReplay.replay does on `threads` host threads (0 = all cores).
 * `sums` receives n_out * (2 + n_in) doubles laid out per output o as
 *   [sum v, sum v^2, sum dv/din_0 ... sum dv/din_{n_in-1}].
 * `per_path` (may be NULL) receives, per path, n_out * (1 + n_in) doubles:
 *   the output values and adjoints of that scenario.
 * Returns 0 on success, a negative code on a malformed tape.
 */
int orc_replay(const orc_tape* tape, const double* inputs, int f32, int adjoints,
               uint64_t paths, uint64_t path_offset, uint64_t seed, int threads,
               double* sums, double* per_path);

/* orc_replay with exact = 1: every channel is summed with compensated
 * (TwoSum) arithmetic and the per-thread totals combined in double-double, so
 * the sums are the per-path values' exact sum to ~1e-30 relative and differ
 * from a device reduction only by the device's own rounding.  exact = 0 is
 * the reference's plain running sum (AadTotals.add). */
int orc_replay_ex(const orc_tape* tape, const double* inputs, int f32, int adjoints,
                  uint64_t paths, uint64_t path_offset, uint64_t seed, int threads, int exact,
                  double* sums, double* per_path);

/* AadTotals.toResult: mean, standard error and gradients from the sums. */
void orc_finish(int32_t n_out, int32_t n_in, const double* sums, uint64_t paths,
                double* mean, double* stderr_out, double* gradients);

/*
 * Reference tape producers.  Each writes into caller-provided arrays of
 * capacity `cap` nodes and returns the node count (or -1 if cap is too small).
 * Inputs are recorded first in the order spot, strike, vol, rate, maturity.
 * `kind` for the barrier: 0 up-out, 1 up-in, 2 down-out, 3 down-in
 * (BarrierEnum order); `call` selects call (1) or put (0).
 */
typedef struct orc_tape_buf {
  int32_t* op;
  int32_t* arg_a;
  int32_t* arg_b;
  double* constant;
  int32_t cap;
  int32_t n;
  int32_t input_node[8];
  int32_t n_in;
  int32_t output_node;
} orc_tape_buf;

int orc_build_european(orc_tape_buf* t, int steps, int call);
int orc_build_asian(orc_tape_buf* t, int steps, int call);
int orc_build_barrier(orc_tape_buf* t, int steps, int call, int kind, double barrier, double width);

#ifdef __cplusplus
}
#endif

#endif
