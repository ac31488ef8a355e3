// nt_internal.hpp -- internal types of libnabla_b200 (tape, loop plan, emitter).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/nabla_b200.h"

namespace nt {

// Words of one channel's exact sum (NT_XWORDS of nt_exact.cuh; checked
// against it where both are visible).
constexpr int kXWords = 69;
// Paths of one warp tile: launches and shards start on multiples of it
// (relative to the start of the whole range), so every tile holds the same
// paths however the range is split.
constexpr uint64_t kTile = 32;

// An error that crosses no ABI: the C entry points turn it into a status code
// and a thread-local message.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& msg) : std::runtime_error(msg), code(c) {}
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error(code, msg); }

inline bool is_unary(int op) {
  return op == NT_NEG || op == NT_EXP || op == NT_LOG || op == NT_SQRT || op == NT_ABS;
}
inline bool is_binary(int op) {
  return op == NT_ADD || op == NT_SUB || op == NT_MUL || op == NT_DIV || op == NT_MAX || op == NT_MIN;
}
inline bool is_draw(int op) { return op == NT_RANDN || op == NT_RANDU; }
const char* op_name(int op);

// A validated tape (FlatTape.java:37-79 plus AadTape's stream counts).
struct Tape {
  int32_t n = 0;
  std::vector<int32_t> op, a, b;
  std::vector<double> c;
  std::vector<int32_t> input_node, output_node;
  int32_t n_streams = 1;
  std::vector<int32_t> normal_count, uniform_count;
  std::vector<uint8_t> active;  // AadTape.markActive (AadTape.java:70-81)
  int32_t n_in() const { return (int32_t)input_node.size(); }
  int32_t n_out() const { return (int32_t)output_node.size(); }
};

// Copies and validates a caller's tape; throws Error(NT_E_TAPE, ...) on any
// malformed index, op code or count.
Tape ingest(const nt_tape* t);

// Division by a constant power of two becomes multiplication by its exact
// reciprocal (x / 2^k and x * 2^-k are the same correctly rounded number, and
// so are the adjoint contributions d / 2^k and d * 2^-k), when the constant
// node feeds nothing else and both 2^k and 2^-k are normal in the working
// precision.  Returns the number of divisions rewritten.
int32_t reduce_pow2_divisions(Tape& t, bool f32);

// How a loop-body argument is reached.
// An argument of a loop unit: the same unit, the previous unit (a carry), one
// fixed node before the loop (an invariant), or a node before the loop that
// changes from unit to unit (gathered through Loop::gather[idx]).
enum RefKind : int8_t { REF_NONE = 0, REF_SAME = 1, REF_CARRY = 2, REF_OUT = 3, REF_GATHER = 4 };
struct Ref {
  RefKind kind = REF_NONE;
  int32_t idx = -1;  // SAME/CARRY: offset in the unit; OUT: node index outside the loop
};

struct BodyNode {
  int32_t op = 0;
  Ref ra, rb;
  double c = 0.0;
  int32_t stream = 0;       // draws
  int32_t draw_base = 0;    // ordinal in unit 0
  int32_t draw_stride = 0;  // ordinal increase per unit
  int32_t cslot = -1;       // CONST whose value differs between units: column of Loop::ctab
  bool active = false;      // OR over all units
};

// The step loop of a tape: units [B + u*L, B + (u+1)*L) for u in [0, N).
struct Loop {
  bool present = false;
  int32_t B = -1, L = 0, N = 0;
  int32_t steps_per_unit = 1;  // tape iterations folded into one unit (RNG pairing)
  // A long unit with one normal per stream and stride 1 is not folded: an even
  // unit draws the Box-Muller pair and keeps the second leg for the next unit.
  bool half_pairs = false;
  std::vector<BodyNode> body;
  std::vector<int32_t> carries;     // unit offsets read by the next unit
  std::vector<int32_t> carry_init;  // per carry: the node feeding unit 0
  std::vector<int32_t> exits;       // unit offsets read outside the loop (last unit)
  std::vector<uint8_t> is_carry;    // per offset
  std::vector<int32_t> carry_slot;  // per offset: index into carries or -1
  std::vector<uint8_t> is_exit;     // per offset
  std::vector<int32_t> ckpt;        // carries saved at each segment boundary
  std::vector<uint8_t> stored;      // per offset: value kept for the reverse sweep
  std::vector<uint8_t> recompute;   // per offset: recomputed from the segment checkpoint
  std::vector<int32_t> tape_slot;   // per offset: slot in the per-thread value tape, or -1
  int32_t n_tape = 0;               // taped values per unit
  std::vector<std::vector<int32_t>> gather;  // per REF_GATHER slot: the node each unit reads
  int32_t n_vary = 0;               // CONST offsets whose value differs between units
  std::vector<double> ctab;         // their values, [unit][cslot] (a non-uniform time grid, date tables)
  int32_t G = 0;                    // units per segment
  int32_t K = 0;                    // segments (N = K * G)
  int32_t end() const { return B + N * L; }
  bool in(int32_t i) const { return present && i >= B && i < end(); }
  int32_t off(int32_t i) const { return (i - B) % L; }
  int32_t unit(int32_t i) const { return (i - B) / L; }
};

struct Plan {
  Loop loop;
  double fwd_flops = 0.0;  // algorithmic, per scenario
  double rev_flops = 0.0;
  double wide_flops = 0.0;  // of fwd_flops: what an fp32 tape evaluates in fp64 (reference fp32 semantics)
  double arith_flops = 0.0;  // fwd + rev without the transcendentals' weighted flops
  int32_t stored_per_unit = 0;
  int32_t per_unit_regs = 0;  // registers one loop unit's reverse values take (estimate)
};

struct EmitConfig {
  bool f32 = false;
  bool adjoints = true;
  bool no_loop = false;
  bool global_ckpt = false;
  bool wide32 = false;     // fp32: transcendentals + Box-Muller in fp64, narrowed
  bool fmad = true;        // allow multiply-add contraction
  bool tape = true;        // expensive loop values go to a per-thread tape instead of being recomputed
  bool tape_all = true;    // tape draws and transcendentals (else draws only)
  bool tape_every_exp = false;  // tape_all: also the exps of draws and invariants alone
  int32_t grid_blocks_per_sm = 0;  // 0: as many as fit
  int32_t fwd_unroll = 0;  // unroll of the forward unit loop, 0: the whole segment
  int32_t rev_unroll = 1;  // unroll of the reverse segment loop
  int32_t block = 128;
  int32_t min_blocks = 0;
  int32_t max_regs = 0;    // register cap (__maxnreg__; launch bounds would override --maxrregcount)
  int32_t seg_units = 0;   // 0 = automatic
  int32_t target = 0;      // 0 CUDA, 1 host C++
  // Multi-market variant: one launch replays every scenario under n_states
  // input vectors; the first state draws, later states read the draws back
  // from the value tape (common random numbers).
  bool markets = false;
};

// Emitter configuration from the C ABI options (validates them).
EmitConfig config_from(const nt_options* opt, int32_t target);

// Finds the step loop and the checkpoint / recompute sets.
Plan plan_tape(const Tape& t, const EmitConfig& cfg);

// Emits CUDA C (target 0) or host C++ (target 1) for the plan.
std::string emit(const Tape& t, const Plan& p, const EmitConfig& cfg);
// Threads per block when nt_options.block is 0: 256 for a loop whose units are
// light (their reverse values take <= 32 registers: larger blocks give the
// bulk prefetches longer tiles at the same occupancy), 64 for heavier units
// (a register-bound kernel keeps more, smaller blocks resident), 128 without a
// loop.
int32_t auto_block(const Plan& p);

// Number of checkpointed values per thread for this plan (shared/global sizing).
int32_t ckpt_values(const Plan& p);

extern const char* kDeviceRuntimeSource;  // nt_device_rt.cuh, embedded at build time
extern const char* kMathTablesSource;     // nt_math_tables.cuh, embedded at build time
extern const char* kExactSource;          // nt_exact.cuh, embedded at build time

// Frozen flop weights of the fp64 transcendentals {exp, log, sqrt, sincos}
// (nt_flops.cpp), used for the algorithmic flop count of a tape.
extern const double kFlopWeights[4];

void math_eval(int32_t device, int32_t which, int64_t n, const uint32_t* words, const double* x, double* out0,
               double* out1);

// Vector-FMA peak (TFLOP/s) measured with independent FMA chains: a burst
// (best of a few short launches) and a sustained rate (launches back to back
// for `millis`, rate over the second half, under the board's power limit).
double fma_peak_tflops(int32_t device, int32_t fp64, int32_t iters);
double fma_peak_sustained_tflops(int32_t device, int32_t fp64, int32_t millis);

// Runs the device Philox/Box-Muller for the known-answer interface.
void philox_words(int32_t device, uint64_t path0, uint32_t n_paths, uint64_t seed, int32_t stream,
                  uint32_t pair0, uint32_t n_pairs, uint32_t* out, double* normals);

// NVRTC: compile to an sm_100a cubin (cached in memory and on disk);
// max_regs > 0 caps the registers per thread (--maxrregcount).
// The NVRTC the engine compiles with (loaded by path; see nt_nvrtc.cpp).
void nvrtc_version(int* major, int* minor);
std::string nvrtc_path();
std::vector<char> nvrtc_compile(const std::string& source, const std::string& arch, bool use_disk_cache,
                                double* seconds, bool fmad = true, int max_regs = 0);

}  // namespace nt
