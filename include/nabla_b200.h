/*
 * nabla_b200.h -- C ABI of the B200 tape-replay engine (libnabla_b200.so).
 *
 * This is the boundary a NablaTensor host binds through the Panama FFM API
 * (java.lang.foreign) to serve engine name "cuda": plain C types, borrowed
 * host pointers, no exceptions across the ABI, every call returns 0 or a
 * negative NT_E_* status with a thread-local message from nt_last_error().
 *
 * Paths in the "replaces" notes are relative to the reference project root.
 *
 * Ownership: host arrays passed in are borrowed for the duration of the call
 * and copied; every device allocation is owned by an nt_exec and released by
 * nt_destroy.  An nt_exec is internally serialised (one mutex), so any host
 * thread may call it; it binds its device on every call.
 */
#ifndef NABLA_B200_H
#define NABLA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NT_ABI_VERSION 1

/* Status codes. */
#define NT_OK 0
#define NT_E_INVALID_ARG (-1)  /* bad pointer/size/argument (IllegalArgumentException) */
#define NT_E_TAPE (-2)         /* malformed tape */
#define NT_E_UNSUPPORTED (-3)  /* tape/options this engine declines (UnsupportedOperationException) */
#define NT_E_CUDA (-4)         /* CUDA runtime/driver failure */
#define NT_E_NVRTC (-5)        /* run-time compilation failure */
#define NT_E_NCCL (-6)         /* collective failure or timeout */
#define NT_E_OOM (-7)          /* device allocation failed */
#define NT_E_STATE (-8)        /* call not valid in the current state (IllegalStateException) */
#define NT_E_INTERNAL (-9)

/* Op codes: the ordinal order of AadOpEnum
 * (nablatensor-core/src/main/java/com/nablatensor/engine/AadOpEnum.java:19-50). */
enum nt_op {
  NT_CONST = 0, NT_INPUT = 1, NT_RANDN = 2, NT_RANDU = 3, NT_ADD = 4, NT_SUB = 5, NT_MUL = 6,
  NT_DIV = 7, NT_NEG = 8, NT_EXP = 9, NT_LOG = 10, NT_SQRT = 11, NT_MAX = 12, NT_MIN = 13,
  NT_ABS = 14
};

/* Precision: the ordinal order of AadOptions.PrecisionEnum
 * (nablatensor-core/.../engine/AadOptions.java, FLOAT32 then FLOAT64). */
enum nt_precision { NT_FLOAT32 = 0, NT_FLOAT64 = 1 };

/*
 * A recorded tape as flat arrays: the FlatTape layout
 * (nablatensor-core/.../engine/FlatTape.java:37-79) plus the random-stream
 * counts of AadTape (AadTape.java:128-196).
 *   op[i], arg_a[i], arg_b[i], constant[i] for node i in recording order;
 *   INPUT: arg_a = input index; RANDN/RANDU: arg_a = ordinal within
 *   (stream, kind), arg_b = stream; unused arguments are -1.
 * normal_count/uniform_count may be NULL (derived from the nodes).
 */
typedef struct nt_tape {
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
  const int32_t* normal_count;
  const int32_t* uniform_count;
} nt_tape;

/* Option flags. */
#define NT_FLAG_NO_LOOP 0x1      /* emit straight-line code even when the tape has a step loop */
#define NT_FLAG_SHARED_CKPT 0x2  /* keep step checkpoints in shared memory instead of (L2-resident)
                                    global memory */
#define NT_FLAG_NO_DISK_CACHE 0x4
#define NT_FLAG_F32_FAST 0x8     /* fp32: exp/log and Box-Muller in single precision, with
                                    multiply-add contraction.  By default they are evaluated in fp64
                                    and narrowed on store, and no product is fused into an add: every
                                    node is rounded on its own, the reference's fp32 semantics
                                    (ScalarReplay.java:37-51) */
#define NT_FLAG_NO_FMAD 0x10     /* no multiply-add contraction (every product rounded); already the
                                    default of fp32 tapes without NT_FLAG_F32_FAST */
#define NT_FLAG_ACC_REGS 0x20    /* no effect: the per-thread accumulators it placed were replaced by
                                    the exact per-warp accumulation; kept so old callers still compile */
#define NT_FLAG_RECOMPUTE_ALL 0x40 /* reverse sweep recomputes every loop value from the step
                                      checkpoints (no per-thread value tape in global memory) */
#define NT_FLAG_TAPE_DRAWS 0x80    /* tape only the draws and recompute exp/log/sqrt/div in the
                                      reverse sweep.  By default the draws, log, sqrt, division
                                      and every exp whose argument depends on a loop carry are
                                      taped; an exp of the unit's draws and invariants alone (a
                                      GBM log-return) is recomputed by the branch-free series,
                                      unless the unit's reverse values alone need more than 32
                                      registers */
#define NT_FLAG_TAPE_ALL 0x100     /* tape every draw, exp, log, sqrt and division */

/*
 * Compile options: AadOptions (AadOptions.java:42-156) plus the engine knobs a
 * caller may pass through AadOptions.engineOptions("cuda").  Zero means
 * "choose automatically" for every tuning field.
 */
typedef struct nt_options {
  int32_t precision;   /* NT_FLOAT32 or NT_FLOAT64 */
  int32_t adjoints;    /* 1: value + adjoints of every input; 0: value only */
  int32_t device;      /* CUDA device ordinal */
  int32_t block;       /* threads per block */
  int32_t seg_units;   /* loop units per checkpoint segment */
  int32_t min_blocks;  /* __launch_bounds__ minimum blocks per SM */
  int32_t max_regs;    /* register cap per thread */
  int32_t flags;       /* NT_FLAG_* */
  int32_t fwd_unroll;  /* unroll of the forward step-unit loop; 0: the whole checkpoint segment, so
                          one unit's draws and transcendentals overlap the previous unit's chain */
  int32_t grid_blocks_per_sm; /* cap on resident blocks per SM of the persistent grid */
  int32_t rev_unroll;  /* unroll of the reverse sweep's segment loop (0 or 1: rolled) */
} nt_options;

typedef struct nt_exec nt_exec;

/* Kernel statistics (the -Dnablatensor.cuda.kernelStats idea,
 * nablatensor-engine-cuda/.../backend/cuda/CudaRuntime.java:584-593). */
typedef struct nt_exec_info {
  int32_t registers;        /* per thread */
  int32_t local_bytes;      /* per thread; 0 means no spill */
  int32_t static_smem;      /* bytes per block */
  int32_t dynamic_smem;     /* bytes per block (step checkpoints) */
  int32_t block;            /* threads per block */
  int32_t blocks_per_sm;    /* resident blocks per SM at this configuration */
  int32_t grid;             /* persistent grid size */
  int32_t sm_count;
  int32_t channels;         /* accumulators: n_out * (2 + n_in) */
  int32_t loop_start;       /* first node of the step loop, -1 when none */
  int32_t loop_unit;        /* nodes per loop unit */
  int32_t loop_units;       /* number of loop units */
  int32_t steps_per_unit;   /* tape iterations folded into one unit */
  int32_t seg_units;        /* units per checkpoint segment */
  int32_t segments;
  int32_t ckpt_slots;       /* checkpointed values per segment boundary */
  int32_t stored_per_unit;  /* values kept per unit for the reverse sweep */
  int32_t ckpt_global;      /* 1 when checkpoints live in global memory */
  int32_t tape_slots;       /* values per loop unit written to the per-thread tape (0: recompute all) */
  int32_t tape_mbytes;      /* device memory held by the value tape, MiB */
  int32_t markets_registers;   /* the multi-market kernel's, 0 until nt_replay_markets compiled it */
  int32_t markets_local_bytes;
  double compile_seconds;   /* NVRTC + module load, 0 on a cache hit */
  double fwd_flops;         /* algorithmic flops per scenario, forward: arithmetic 1, exp 29,
                               log 44, sqrt 13, sincos 36 (nt_flops.cpp) */
  double rev_flops;         /* algorithmic flops per scenario, reverse */
  double wide_flops;        /* fp32 tapes: the part of fwd_flops evaluated in fp64 (exp, log and
                               Box-Muller under the reference's fp32 semantics); 0 for fp64 tapes */
  double arith_flops;       /* fwd_flops + rev_flops less the transcendentals (exp, log, sqrt and
                               Box-Muller's log, sqrt, sincos): arithmetic-only flops per scenario */
} nt_exec_info;

/* ABI version (NT_ABI_VERSION of the built library). */
int nt_version(void);

/* Last error message of the calling thread ("" when none). */
const char* nt_last_error(void);

/* Device discovery; never faults.  Replaces CudaAadEngine.isAvailable()
 * (nablatensor-engine-cuda/.../engine/CudaAadEngine.java) and the context set-up
 * in CudaRuntime.initContext (CudaRuntime.java:206-212). */
int nt_init(int32_t* n_devices);

/* Validates the tape, emits the sm_100a replay kernel, compiles it with NVRTC
 * (cached by source hash) and allocates the executable's device state.
 * Replaces AadEngine.compile (nablatensor-core/.../engine/AadEngine.java:28-48)
 * as implemented by CudaAadEngine.compile (CudaAadEngine.java:60-73) and
 * DeviceAadExecutable.compile (DeviceAadExecutable.java:107-119). */
int nt_compile(const nt_tape* tape, const nt_options* options, nt_exec** out);

/* Binds all n input values (input order); re-pricing never recompiles.
 * Replaces AadExecutable.setInput (AbstractAadExecutable.java:86-92,
 * DeviceAadExecutable.java:134-137). */
int nt_set_inputs(nt_exec* exec, const double* inputs, int32_t n);

/*
 * One dispatch over `paths` scenarios starting at `path_offset`.
 * sums receives n_out * (2 + n_in) doubles, per output o:
 *   [sum v, sum v^2, sum dv/din_0, ..., sum dv/din_{n_in-1}]
 * (the caller divides by `paths` and forms the standard error as
 * AadTotals.toResult does, AadTotals.java:68-89).  seconds (may be NULL)
 * receives the wall time of launch + synchronise + read-back.
 * Each sum is the correctly rounded exact sum of per-tile sums, a tile being
 * 32 consecutive scenarios from path_offset on; any split of the range into
 * pieces that start on tile boundaries (nt_replay_accumulate chunks,
 * nt_replay_sharded ranks) gives the same bits.
 * Replaces AadExecutable.replay (AadExecutable.java:46-47) as implemented by
 * DeviceAadExecutable.replay (DeviceAadExecutable.java:140-168).
 */
int nt_replay(nt_exec* exec, uint64_t paths, uint64_t path_offset, uint64_t seed, double* sums,
              double* seconds);

/*
 * Re-pricing under several markets in one dispatch, with common random
 * numbers: inputs holds n_states input vectors ([n_states][n_in], input
 * order), sums receives n_states blocks in nt_replay's layout
 * ([n_states][n_out * (2 + n_in)]).  Every scenario is replayed under each
 * market in turn; the first market draws the step loop's normals and tapes
 * them, the others read them back, so the generator and the Box-Muller
 * transform run once per scenario instead of once per market.  Each
 * market's sums equal nt_replay with those inputs up to the
 * rounding of a multiply-add the compiler fuses differently in the two
 * kernels (bit for bit in the host build, which fuses none).  The executable's own
 * inputs (nt_set_inputs) are not used or changed.  The kernel is compiled on
 * the first call.  Replaces the per-market loop of
 * ScenarioRunner.run/ladder (nablatensor-quant/.../scenario/ScenarioRunner.java:36-71),
 * and the draw cache of the cpu-jit engine, CategoryEnum.DRAW_CACHE
 * (nablatensor-engine-cpu/.../jit/JitReplay.java:69-89).
 */
int nt_replay_markets(nt_exec* exec, int32_t n_states, const double* inputs, uint64_t paths, uint64_t path_offset,
                      uint64_t seed, double* sums, double* seconds);

/*
 * Device-resident accumulation for long runs (the many-chunk replaySafe of
 * AbstractAadExecutable.java:101-121 without a read-back per chunk):
 * nt_replay_accumulate enqueues one dispatch that ADDS its sums, exactly,
 * into the executable's device accumulator and returns without waiting;
 * nt_accumulator_read waits, rounds the accumulator into `sums` and, when
 * reset != 0, zeroes it.  Chunks that start on 32-scenario tile boundaries
 * of one range sum to the bits of one nt_replay over the whole range.
 */
int nt_replay_accumulate(nt_exec* exec, uint64_t paths, uint64_t path_offset, uint64_t seed);
int nt_accumulator_read(nt_exec* exec, double* sums, int32_t reset);

/* The CUDA stream (cudaStream_t) every launch of this executable goes to. */
int nt_exec_stream(nt_exec* exec, void** stream);

/* Kernel statistics and plan of the compiled executable. */
int nt_exec_info_get(nt_exec* exec, nt_exec_info* info);

/* The generated CUDA C source (NUL-terminated, truncated to cap).  *len gets
 * the full length. */
int nt_exec_source(nt_exec* exec, char* buf, size_t cap, size_t* len);

/*
 * Emits the replay source without compiling or touching a GPU.
 * target 0: the CUDA C that nt_compile hands to NVRTC;
 * target 1: the same scenario code as host C++ with an
 *   extern "C" void nt_host_replay(const double* inputs, uint64_t paths,
 *                                  uint64_t path_offset, uint64_t seed,
 *                                  double* sums)
 *   entry point (paths in order, sums in nt_replay's layout); it includes
 *   nt_device_rt.cuh and must be compiled with -DNT_HOST;
 * target 2: the CUDA C of the multi-market kernel nt_replay_markets runs;
 * target 3: its host C++, entry point
 *   extern "C" void nt_host_replay_markets(const double* inputs, int n_states,
 *                                          uint64_t paths, uint64_t path_offset,
 *                                          uint64_t seed, double* sums)
 *   (inputs [n_states][n_in], sums [n_states][channels]).
 */
int nt_emit_source(const nt_tape* tape, const nt_options* options, int32_t target, char* buf,
                   size_t cap, size_t* len);

/* Compiles a source emitted for target 0 with NVRTC to an sm_100a cubin
 * (no GPU needed); *cubin_bytes gets the image size. */
int nt_nvrtc_check(const char* source, size_t* cubin_bytes);

/* The NVRTC the engine compiles with: its version, and (when path is not
 * null) the library file it was loaded from, copied like nt_emit_source's
 * text.  The engine loads the CUDA toolkit's NVRTC by path, privately, so a
 * host that has loaded another libnvrtc.so.12 (PyTorch bundles one) does not
 * change the kernels; NT_NVRTC_LIBRARY in the environment names another file.
 * No GPU needed.  No counterpart in the reference (its CudaRuntime binds
 * whatever NVRTC the JVM finds). */
int nt_nvrtc_version(int32_t* major, int32_t* minor, char* path, size_t cap, size_t* len);

/* Releases the executable (AadExecutable.close). NULL is a no-op. */
void nt_destroy(nt_exec* exec);

/* ---- multi-GPU: scenario-range sharding + one NCCL all-reduce ------------- */

/* 128-byte NCCL unique id for rank 0 to broadcast. */
int nt_dist_unique_id(uint8_t id[128]);

/* Joins this executable to an nranks-wide NCCL communicator (one rank per
 * GPU, one process per rank; NCCL is loaded with dlopen, from
 * $NT_NCCL_LIBRARY when set, else libnccl.so.2).  timeout_ms bounds the join
 * and, later, each all-reduce once this rank's shard is done; on expiry or on
 * an NCCL error the communicator is aborted (ncclCommAbort) and NT_E_NCCL
 * returned, after which the executable is detached. */
int nt_dist_attach(nt_exec* exec, int32_t nranks, int32_t rank, const uint8_t id[128],
                   int32_t timeout_ms);

/*
 * Replays the global scenario range [path_offset, path_offset + total_paths)
 * with this rank's contiguous shard (nt_shard_range), then all-reduces the
 * exact accumulator words (one int64 ncclAllReduce of n_out * (2 + n_in) x 69
 * words).  Every rank receives the global sums, with the same bits as a
 * single-GPU nt_replay of the whole range, whatever the number of ranks.
 * chunk_paths > 0 splits this rank's shard into dispatches of at most that
 * many scenarios (rounded down to a multiple of 32), accumulated on the
 * device.  A peer that leaves or stalls ends the call with NT_E_NCCL within
 * the attach timeout after this rank's shard is done.  seconds (may be NULL)
 * gets this rank's wall time of the call.
 */
int nt_replay_sharded(nt_exec* exec, uint64_t total_paths, uint64_t path_offset, uint64_t seed,
                      uint64_t chunk_paths, double* sums, double* seconds);

/*
 * nt_replay without any allocation, for callers that cannot let the engine
 * allocate device memory: a host that hands the whole device to its own
 * memory pool under a fixed budget, or one pricing inside a latency-critical
 * loop, where cudaMalloc/cudaFree would synchronise the device.  No
 * counterpart in the reference.
 *
 * Launches `exec`'s kernel on the caller's stream (a cudaStream_t, NULL for
 * the legacy default stream) over [path_offset, path_offset + paths), reading
 * the n_in input doubles from device memory `d_inputs` and writing the
 * n_out * (2 + n_in) sums (nt_replay's layout and bits) to device memory
 * `d_sums`; both must be device (or managed) memory of exec's GPU, else
 * NT_E_INVALID_ARG.  Returns once the work is enqueued; synchronise the
 * stream before reading.  Calls no cudaMalloc, cudaFree or other allocating
 * routine.
 *
 * The kernel's reduction scratch lives in a static device array of 64 KiB
 * that every GPU loading the library holds until exit; an executable needing
 * more (256 + channels x 69 x 8 bytes, i.e. more than 118 channels, for
 * example more than 116 inputs of a one-output tape) is rejected with
 * NT_E_INVALID_ARG.  `exec` must have no value tape and no global
 * checkpoints -- compile it with NT_FLAG_RECOMPUTE_ALL | NT_FLAG_SHARED_CKPT
 * -- else NT_E_UNSUPPORTED.  All calls on a device share the scratch and
 * keep the last call's contents (each call clears it on its stream first):
 * calls that overlap on the GPU race.  The first call on each device looks up
 * the scratch address (cudaGetSymbolAddress), so make it before any stream
 * capture, and do not use the entry point across a cudaDeviceReset.
 */
int nt_replay_noalloc(nt_exec* exec, uint64_t paths, uint64_t path_offset, uint64_t seed, const double* d_inputs,
                      double* d_sums, void* stream);

/* Enqueue-only variant for device timing: the shard dispatches plus the
 * all-reduce go to the executable's stream; results land in the device
 * accumulator (read with nt_accumulator_read). */
int nt_replay_sharded_async(nt_exec* exec, uint64_t total_paths, uint64_t path_offset,
                            uint64_t seed, uint64_t chunk_paths);

/* Device time in milliseconds (CUDA events on the executable's stream) of
 * the last all-reduce nt_replay_sharded(_async) enqueued; waits for it.
 * NT_E_STATE before the first one.  The kernelStats-style figure that tells
 * the collective's share of a sharded step.  No counterpart in the reference
 * (it has no multi-GPU path). */
int nt_dist_collective_ms(nt_exec* exec, double* ms);

/* Leaves the communicator (ncclCommDestroy). */
int nt_dist_detach(nt_exec* exec);

/* The contiguous shard of [path_offset, path_offset + total_paths) that rank
 * `rank` of `nranks` replays: the range's ceil(total_paths / 32) tiles of 32
 * scenarios are split into nranks contiguous runs, the first
 * (tiles % nranks) runs one tile longer; a rank may get no scenario.  Host
 * arithmetic only (no device needed); nt_replay_sharded uses it. */
int nt_shard_range(uint64_t total_paths, uint64_t path_offset, int32_t nranks, int32_t rank, uint64_t* from,
                   uint64_t* count);

/* ---- generator known-answer access (tests) -------------------------------- */

/*
 * Runs the device generator and copies its raw uint32 words to the host:
 * for p in [0, n_paths), q in [0, n_pairs):
 *   out[(p * n_pairs + q) * 2 + {0,1}] = Philox words of normal pair
 *   (pair0 + q) of (path0 + p, seed, stream).
 * normals (may be NULL) receives the fp64 Box-Muller legs in the same layout.
 * This is Philox.normal() of nablatensor-engine-cpu/.../cpu/Philox.java:56-78
 * evaluated on the GPU.
 */
int nt_philox_words(int32_t device, uint64_t path0, uint32_t n_paths, uint64_t seed, int32_t stream,
                    uint32_t pair0, uint32_t n_pairs, uint32_t* out, double* normals);

/* Measured vector-FMA peak of the device in TFLOP/s (FMA = 2 flops): the
 * roofline denominator of the replay kernels, which run on the fp64 (or fp32)
 * pipe, not the tensor cores.  fp64 != 0 measures DFMA, else FFMA.  No
 * counterpart in the reference (it reports no roofline). */
int nt_fma_peak(int32_t device, int32_t fp64, int32_t iters, double* tflops);

/* The same FMA chains launched back to back for `millis` milliseconds; the
 * rate over the second half, once the clocks have settled under the board's
 * power limit.  The denominator for a replay timed over seconds (a burst
 * figure would credit clocks the long run cannot hold).  No counterpart in
 * the reference. */
int nt_fma_peak_sustained(int32_t device, int32_t fp64, int32_t millis, double* tflops);

/* Evaluates one of the replay's dedicated fp64 routines on the device over n
 * host inputs (copied in and out), so the tests can measure their accuracy as
 * compiled for sm_100a:
 *   which 0: out0[i] = -2 ln(u1), u1 = (words[i] + 0.5) 2^-32 (table-driven)
 *   which 1: out0[i], out1[i] = sin, cos of fl(2 pi u2), u2 from words[i]
 *   which 2: out0[i] = the Box-Muller radius sqrt of x[i] (x[i] > 0, normal)
 *   which 3: out0[i] = the series exp of x[i] (|x[i]| <= 1/8)
 *   which 4: out0[i] = the full-range exp of x[i]
 *   which 5: out0[i], out1[i] = the cosine and sine Box-Muller legs of the
 *            word pair (words[2i], words[2i+1])
 *   which 6: the same legs from the float-result routines of fp32 tapes,
 *            as floats widened to double
 *   which 7: out0[i] = the first-pass exp of a taped loop value at x[i],
 *            out1[i] = 1 where it records the argument for the redo pass
 * words is read for which 0, 1 (n words), 5 and 6 (2n words), x for 2, 3, 4
 * and 7; out1 is written for 1, 5, 6 and 7.  n is in [1, 2^24].  Test
 * support; no counterpart in the reference. */
int nt_math_eval(int32_t device, int32_t which, int64_t n, const uint32_t* words, const double* x, double* out0,
                 double* out1);

#ifdef __cplusplus
}
#endif

#endif /* NABLA_B200_H */
