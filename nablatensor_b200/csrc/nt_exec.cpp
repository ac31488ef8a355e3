// nt_exec.cpp -- executables: device state, launch, reduction read-back,
// scenario-range sharding with one NCCL all-reduce.
//
// The reference's device executable (nablatensor-core/.../DeviceAadExecutable.java:140-221)
// launched 256-thread blocks over min(ceil(paths/256), 4096) blocks, copied
// one partial record per block to the host and summed there.  Here:
//   - one persistent grid of (SMs x resident blocks) walks the path range in
//     warp tiles of 32 paths;
//   - every tile's sums are added exactly into fixed-point words
//     (nt_exact.cuh), so the result is the correctly rounded sum of the tile
//     sums, the same bits for any grid, chunking or number of GPUs;
//   - the last block rounds the words on the device (atomic ticket, no spin)
//     and the host reads n_out*(2+n_in) doubles;
//   - long runs accumulate exact words on the device across dispatches;
//   - several GPUs split the range into contiguous runs of tiles and
//     all-reduce the words once (one int64 NCCL all-reduce over
//     NVLink/NVSwitch).
#include "nt_exec.hpp"

#define NT_HOST 1
#include "nt_exact.cuh"

#include <algorithm>
#include <chrono>
#include <cstring>
#include <thread>

namespace nt {

static_assert(kXWords == NT_XWORDS, "exact-sum word count");

// ---- driver API through the runtime's entry-point query (no libcuda link) ----

namespace {

struct Driver {
  CUresult (*moduleLoadData)(CUmodule*, const void*) = nullptr;
  CUresult (*moduleUnload)(CUmodule) = nullptr;
  CUresult (*moduleGetFunction)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*launchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                           CUstream, void**, void**) = nullptr;
  CUresult (*funcGetAttribute)(int*, CUfunction_attribute, CUfunction) = nullptr;
  CUresult (*funcSetAttribute)(CUfunction, CUfunction_attribute, int) = nullptr;
  CUresult (*occupancy)(int*, CUfunction, int, size_t) = nullptr;
  CUresult (*getErrorName)(CUresult, const char**) = nullptr;
  bool ok = false;
};

template <class F>
void entry(const char* name, F& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
    fail(NT_E_CUDA, std::string("driver entry point unavailable: ") + name);
  fn = reinterpret_cast<F>(p);
}

Driver& driver() {
  static Driver d;
  static std::once_flag once;
  static std::string err;
  std::call_once(once, [] {
    try {
      entry("cuModuleLoadData", d.moduleLoadData);
      entry("cuModuleUnload", d.moduleUnload);
      entry("cuModuleGetFunction", d.moduleGetFunction);
      entry("cuLaunchKernel", d.launchKernel);
      entry("cuFuncGetAttribute", d.funcGetAttribute);
      entry("cuFuncSetAttribute", d.funcSetAttribute);
      entry("cuOccupancyMaxActiveBlocksPerMultiprocessor", d.occupancy);
      entry("cuGetErrorName", d.getErrorName);
      d.ok = true;
    } catch (const Error& e) {
      err = e.what();
    }
  });
  if (!d.ok) fail(NT_E_CUDA, err.empty() ? "CUDA driver unavailable" : err);
  return d;
}

void cu_check(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return;
  const char* name = "?";
  if (driver().getErrorName) driver().getErrorName(r, &name);
  fail(NT_E_CUDA, std::string(what) + ": " + name);
}

}  // namespace

void cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return;
  const int code = e == cudaErrorMemoryAllocation ? NT_E_OOM : NT_E_CUDA;
  fail(code, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

// ---- compile / set-up ---------------------------------------------------------

Exec* Exec::create(const nt_tape* tape, const nt_options* opt) {
  std::unique_ptr<Exec> x(new Exec());
  x->cfg = config_from(opt, 0);
  x->tape = ingest(tape);
  reduce_pow2_divisions(x->tape, x->cfg.f32);
  x->device = opt->device;
  x->use_disk_cache = (opt->flags & NT_FLAG_NO_DISK_CACHE) == 0;
  x->plan = plan_tape(x->tape, x->cfg);
  if (opt->block == 0) x->cfg.block = auto_block(x->plan);
  x->channels = x->tape.n_out() * (2 + x->tape.n_in());
  const size_t real_bytes = x->cfg.f32 ? 4 : 8;
  // Checkpoints in shared memory unless they would starve occupancy.
  const size_t ck_bytes = (size_t)ckpt_values(x->plan) * x->cfg.block * real_bytes;
  if (!x->cfg.global_ckpt && ck_bytes > 96 * 1024) x->cfg.global_ckpt = true;
  x->dyn_smem = x->cfg.global_ckpt ? 0 : (int)ck_bytes;
  x->source = emit(x->tape, x->plan, x->cfg);
  x->inputs.assign(x->tape.n_in(), 0.0);
  for (int32_t j = 0; j < x->tape.n_in(); ++j) x->inputs[j] = tape->constant[x->tape.input_node[j]];
  x->auto_regs = opt->max_regs == 0 && opt->min_blocks == 0;
  x->auto_seg = x->auto_regs && opt->seg_units == 0 && opt->block == 0;
  x->load(opt->max_regs);
  return x.release();
}

void Exec::bind() const { cuda_check(cudaSetDevice(device), "cudaSetDevice"); }

void Exec::load(int max_regs) {
  int ndev = 0;
  cuda_check(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
  if (device < 0 || device >= ndev) fail(NT_E_INVALID_ARG, "device ordinal out of range");
  bind();
  cudaDeviceProp prop;
  cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10) fail(NT_E_UNSUPPORTED, std::string("this engine targets sm_100 (B200); device is ") + prop.name);
  sm_count = prop.multiProcessorCount;
  double secs = 0.0;
  max_regs_opt = max_regs;
  std::vector<char> cubin = nvrtc_compile(source, "sm_100a", use_disk_cache, &secs, cfg.fmad, max_regs);
  const auto t0 = std::chrono::steady_clock::now();
  Driver& d = driver();
  cu_check(d.moduleLoadData(&module, cubin.data()), "cuModuleLoadData");
  cu_check(d.moduleGetFunction(&function, module, "nt_replay_kernel"), "cuModuleGetFunction");
  // Static + dynamic shared memory above 48 KB needs the opt-in attribute.
  if (dyn_smem > 0)
    cu_check(d.funcSetAttribute(function, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, dyn_smem),
             "cuFuncSetAttribute");
  int regs = 0, local = 0, ssm = 0;
  cu_check(d.funcGetAttribute(&regs, CU_FUNC_ATTRIBUTE_NUM_REGS, function), "cuFuncGetAttribute");
  if (auto_regs && regs >= 248) {
    // The register file ran out (or came within a granule of it): one block
    // of 64 threads per quarter SM, and a latency-bound sweep gains more from
    // twice the resident warps than it loses to spills (a 118-unit CVA book:
    // +56 %).  Recompile with a cap of 128 registers.
    double secs2 = 0.0;
    cfg.max_regs = 128;
    source = emit(tape, plan, cfg);
    std::vector<char> capped = nvrtc_compile(source, "sm_100a", use_disk_cache, &secs2, cfg.fmad, max_regs);
    secs += secs2;
    cu_check(d.moduleUnload(module), "cuModuleUnload");
    module = nullptr;
    cu_check(d.moduleLoadData(&module, capped.data()), "cuModuleLoadData");
    cu_check(d.moduleGetFunction(&function, module, "nt_replay_kernel"), "cuModuleGetFunction");
    if (dyn_smem > 0)
      cu_check(d.funcSetAttribute(function, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, dyn_smem),
               "cuFuncSetAttribute");
    cu_check(d.funcGetAttribute(&regs, CU_FUNC_ATTRIBUTE_NUM_REGS, function), "cuFuncGetAttribute");
  }
  cu_check(d.funcGetAttribute(&local, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, function), "cuFuncGetAttribute");
  if (auto_seg && cfg.global_ckpt && plan.loop.present && plan.loop.G == 1 && plan.loop.K >= 4 && regs <= 192 &&
      local <= 64) {
    // A heavy unit (one unit per segment) whose kernel left registers
    // unused (a few spilled words aside): two units per segment give the
    // reverse sweep two units of independent work to overlap (the 10-asset
    // basket: +17 %).  Kept when the wider kernel still fits in 255 registers
    // and spills no more; the choice depends only on the compiler's register
    // and local-memory counts, never on timing.
    EmitConfig c2 = cfg;
    c2.seg_units = 2;
    Plan p2 = plan_tape(tape, c2);
    if (p2.loop.present && p2.loop.G == 2) {
      c2.seg_units = cfg.seg_units;
      std::string s2 = emit(tape, p2, c2);
      // The wider kernel is optional: if it fails to compile or load, the
      // first one stays.
      CUmodule m2 = nullptr;
      CUfunction f2 = nullptr;
      int regs2 = 255, local2 = 1;
      try {
        double secs2 = 0.0;
        std::vector<char> bin2 = nvrtc_compile(s2, "sm_100a", use_disk_cache, &secs2, cfg.fmad, max_regs);
        secs += secs2;
        cu_check(d.moduleLoadData(&m2, bin2.data()), "cuModuleLoadData");
        cu_check(d.moduleGetFunction(&f2, m2, "nt_replay_kernel"), "cuModuleGetFunction");
        cu_check(d.funcGetAttribute(&regs2, CU_FUNC_ATTRIBUTE_NUM_REGS, f2), "cuFuncGetAttribute");
        cu_check(d.funcGetAttribute(&local2, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, f2), "cuFuncGetAttribute");
      } catch (const Error&) {
        regs2 = 255;
      }
      if (m2 && regs2 < 255 && local2 <= local) {
        cu_check(d.moduleUnload(module), "cuModuleUnload");
        module = m2;
        function = f2;
        plan = std::move(p2);
        source = std::move(s2);
        regs = regs2;
        local = local2;
      } else if (m2) {
        cu_check(d.moduleUnload(m2), "cuModuleUnload");
      }
    }
  }
  int per_sm = 0;
  cu_check(d.occupancy(&per_sm, function, cfg.block, (size_t)dyn_smem), "cuOccupancyMaxActiveBlocksPerMultiprocessor");
  if (per_sm < 1) fail(NT_E_CUDA, "kernel does not fit on an SM");
  const int fit = (65536 / ((per_sm + 1) * cfg.block)) & ~7;  // registers that admit one more block
  if (auto_regs && cfg.max_regs == 0 && local <= 64 && per_sm < 8 && regs > fit && regs - fit <= 16) {
    // The compiler sized the kernel a few registers above an occupancy step
    // (the fp32 barrier: 91 registers, 2 blocks of 256 threads; at 80, 3).
    // Ask for one more resident block; keep the result when it gets there
    // with a spill of a few words at most (the barrier: +11 %).  The choice
    // depends only on the compiler's register and local-memory counts.
    EmitConfig c3 = cfg;
    c3.min_blocks = per_sm + 1;
    CUmodule m3 = nullptr;
    CUfunction f3 = nullptr;
    int regs3 = 255, local3 = 1 << 20, per_sm3 = 0;
    std::string s3 = emit(tape, plan, c3);
    try {
      double secs3 = 0.0;
      std::vector<char> bin3 = nvrtc_compile(s3, "sm_100a", use_disk_cache, &secs3, cfg.fmad, max_regs);
      secs += secs3;
      cu_check(d.moduleLoadData(&m3, bin3.data()), "cuModuleLoadData");
      cu_check(d.moduleGetFunction(&f3, m3, "nt_replay_kernel"), "cuModuleGetFunction");
      if (dyn_smem > 0)
        cu_check(d.funcSetAttribute(f3, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, dyn_smem),
                 "cuFuncSetAttribute");
      cu_check(d.funcGetAttribute(&regs3, CU_FUNC_ATTRIBUTE_NUM_REGS, f3), "cuFuncGetAttribute");
      cu_check(d.funcGetAttribute(&local3, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, f3), "cuFuncGetAttribute");
      cu_check(d.occupancy(&per_sm3, f3, cfg.block, (size_t)dyn_smem), "cuOccupancyMaxActiveBlocksPerMultiprocessor");
    } catch (const Error&) {
      per_sm3 = 0;
    }
    if (m3 && per_sm3 > per_sm && local3 <= 64) {
      cu_check(d.moduleUnload(module), "cuModuleUnload");
      module = m3;
      function = f3;
      cfg = c3;
      source = std::move(s3);
      regs = regs3;
      local = local3;
      per_sm = per_sm3;
    } else if (m3) {
      cu_check(d.moduleUnload(m3), "cuModuleUnload");
    }
  }
  cu_check(d.funcGetAttribute(&ssm, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, function), "cuFuncGetAttribute");
  if (cfg.grid_blocks_per_sm > 0) per_sm = std::min(per_sm, cfg.grid_blocks_per_sm);
  blocks_per_sm = per_sm;
  grid = sm_count * per_sm;
  cuda_check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda_check(cudaMalloc(&d_inputs, sizeof(double) * std::max<int32_t>(1, tape.n_in())), "cudaMalloc inputs");
  const size_t words = sizeof(long long) * (size_t)channels * kXWords;
  cuda_check(cudaMalloc(&d_glim, words), "cudaMalloc exact words");
  cuda_check(cudaMalloc(&d_ticket, sizeof(unsigned int)), "cudaMalloc ticket");
  cuda_check(cudaMalloc(&d_out, sizeof(double) * channels), "cudaMalloc out");
  cuda_check(cudaMalloc(&d_acc, words), "cudaMalloc accumulator");
  cuda_check(cudaMemset(d_glim, 0, words), "cudaMemset exact words");
  cuda_check(cudaMemset(d_ticket, 0, sizeof(unsigned int)), "cudaMemset ticket");
  cuda_check(cudaMemset(d_acc, 0, words), "cudaMemset accumulator");
  cuda_check(cudaEventCreate(&ev_shard), "cudaEventCreate");
  cuda_check(cudaEventCreate(&ev_reduced), "cudaEventCreate");
  if (cfg.global_ckpt && ckpt_values(plan) > 0) {
    const size_t bytes = (size_t)ckpt_values(plan) * grid * cfg.block * (cfg.f32 ? 4 : 8);
    cuda_check(cudaMalloc(&d_gck, bytes), "cudaMalloc checkpoints");
  }
  // The value tape: one slab per resident thread (indexed by the launched
  // grid, never larger than the persistent grid sized here).
  size_t tape_bytes = 0;
  if (plan.loop.present && plan.loop.n_tape > 0) {
    tape_bytes = (size_t)plan.loop.N * plan.loop.n_tape * grid * cfg.block * (cfg.f32 ? 4 : 8);
    cuda_check(cudaMalloc(&d_tape, tape_bytes), "cudaMalloc value tape");
  }
  cuda_check(cudaMallocHost(&h_stage, sizeof(double) * (tape.n_in() + 2 * channels + 2)), "cudaMallocHost");
  cuda_check(cudaMallocHost(&h_words, words), "cudaMallocHost");
  compile_seconds = secs + std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  std::memset(&info, 0, sizeof info);
  info.registers = regs;
  info.local_bytes = local;
  info.static_smem = ssm;
  info.dynamic_smem = dyn_smem;
  info.block = cfg.block;
  info.blocks_per_sm = per_sm;
  info.grid = grid;
  info.sm_count = sm_count;
  info.channels = channels;
  const Loop& lp = plan.loop;
  info.loop_start = lp.present ? lp.B : -1;
  info.loop_unit = lp.present ? lp.L : 0;
  info.loop_units = lp.present ? lp.N : 0;
  info.steps_per_unit = lp.present ? lp.steps_per_unit : 0;
  info.seg_units = lp.present ? lp.G : 0;
  info.segments = lp.present ? lp.K : 0;
  info.ckpt_slots = lp.present ? (int32_t)lp.ckpt.size() : 0;
  info.stored_per_unit = plan.stored_per_unit;
  info.ckpt_global = cfg.global_ckpt ? 1 : 0;
  info.tape_slots = lp.present ? lp.n_tape : 0;
  info.tape_mbytes = (int32_t)(tape_bytes >> 20);
  info.compile_seconds = compile_seconds;
  info.fwd_flops = plan.fwd_flops;
  info.rev_flops = plan.rev_flops;
  info.wide_flops = plan.wide_flops;
  info.arith_flops = plan.arith_flops;
}

Exec::~Exec() {
  comm.reset();
  if (device >= 0) cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  cudaFree(d_inputs);
  cudaFree(d_glim);
  cudaFree(d_ticket);
  cudaFree(d_out);
  cudaFree(d_acc);
  cudaFree(d_gck);
  cudaFree(d_tape);
  cudaFree(d_mk_inputs);
  cudaFree(d_mk_acc);
  cudaFree(d_mk_partials);
  cudaFree(d_mk_out);
  cudaFree(d_mk_gck);
  cudaFree(d_mk_tape);
  if (h_stage) cudaFreeHost(h_stage);
  if (h_words) cudaFreeHost(h_words);
  if (ev_shard) cudaEventDestroy(ev_shard);
  if (ev_reduced) cudaEventDestroy(ev_reduced);
  if (stream) cudaStreamDestroy(stream);
  if (module) driver().moduleUnload(module);
  if (mk_module) driver().moduleUnload(mk_module);
}

// ---- launch ---------------------------------------------------------------------

void Exec::upload_inputs_if_dirty() {
  if (!dirty) return;
  std::memcpy(h_stage, inputs.data(), sizeof(double) * inputs.size());
  if (!inputs.empty())
    cuda_check(cudaMemcpyAsync(d_inputs, h_stage, sizeof(double) * inputs.size(), cudaMemcpyHostToDevice, stream),
               "upload inputs");
  dirty = false;
}

void Exec::launch(uint64_t paths, uint64_t offset, uint64_t seed, int accumulate) {
  if (paths == 0) fail(NT_E_INVALID_ARG, "paths must be positive");
  const uint64_t need = (paths + cfg.block - 1) / cfg.block;
  const unsigned g = (unsigned)std::min<uint64_t>(need, (uint64_t)grid);
  void* gck = d_gck;
  void* tp = d_tape;
  unsigned long long n = paths, off = offset, sd = seed;
  void* args[] = {&d_inputs, &n, &off, &sd, &d_glim, &d_ticket, &d_out, &d_acc, &accumulate, &gck, &tp};
  cu_check(driver().launchKernel(function, g, 1, 1, (unsigned)cfg.block, 1, 1, (unsigned)dyn_smem,
                                 (CUstream)stream, args, nullptr),
           "cuLaunchKernel");
  ++launches;
}

unsigned Exec::grid_for(uint64_t paths) const {
  const uint64_t need = (paths + cfg.block - 1) / cfg.block;
  return (unsigned)std::max<uint64_t>(1, std::min<uint64_t>(need, (uint64_t)grid));
}

void Exec::launch_external(uint64_t paths, uint64_t offset, uint64_t seed, const double* d_in, double* d_sums,
                           unsigned int* ticket, long long* glim, cudaStream_t s, unsigned grid_blocks) {
  void* gck = nullptr;
  void* tp = nullptr;
  const double* in = d_in;
  long long* no_acc = nullptr;
  int accumulate = 0;
  unsigned long long n = paths, off = offset, sd = seed;
  void* args[] = {&in, &n, &off, &sd, &glim, &ticket, &d_sums, &no_acc, &accumulate, &gck, &tp};
  cu_check(driver().launchKernel(function, grid_blocks, 1, 1, (unsigned)cfg.block, 1, 1, (unsigned)dyn_smem,
                                 (CUstream)s, args, nullptr),
           "cuLaunchKernel");
}

void Exec::replay(uint64_t paths, uint64_t offset, uint64_t seed, double* sums, double* seconds) {
  const auto t0 = std::chrono::steady_clock::now();
  bind();
  upload_inputs_if_dirty();
  launch(paths, offset, seed, 0);
  double* h_out = h_stage + tape.n_in();
  cuda_check(cudaMemcpyAsync(h_out, d_out, sizeof(double) * channels, cudaMemcpyDeviceToHost, stream), "read sums");
  cuda_check(cudaStreamSynchronize(stream), "replay");
  std::memcpy(sums, h_out, sizeof(double) * channels);
  if (seconds) *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// ---- several markets in one launch (common random numbers) ----------------------
//
// The reference re-prices a shocked market by a full replay per market
// (nablatensor-quant/.../scenario/ScenarioRunner.java:36-71), and its cpu-jit
// engine can cache the draw block between such replays
// (nablatensor-engine-cpu/.../jit/JitReplay.java:69-89).  Here one launch runs
// every scenario under all markets in turn: the first market draws and tapes
// the loop's normals, the others read them back, so Philox and Box-Muller are
// paid once per scenario.  Sums per market equal separate replays with the same
// seed (the same per-thread order, the same block-order reduction), up to the
// rounding of multiply-adds the compiler fuses differently in the two kernels.

void Exec::markets(int32_t n_states, const double* h_inputs, uint64_t paths, uint64_t offset, uint64_t seed,
                   double* sums, double* seconds) {
  if (n_states < 1 || n_states > 4096) fail(NT_E_INVALID_ARG, "n_states must be in [1, 4096]");
  if (paths == 0) fail(NT_E_INVALID_ARG, "paths must be positive");
  if (!h_inputs || !sums) fail(NT_E_INVALID_ARG, "inputs and sums must not be null");
  const auto t0 = std::chrono::steady_clock::now();
  bind();
  Driver& d = driver();
  if (!mk_function) {
    // The multi-market kernel keeps the executable's plan, so its reverse
    // sweep is the plain kernel's.  (Taping the draws only and recomputing
    // each market's transcendentals in the reverse sweep moves half the bytes
    // but needs more registers; it measured slower.)
    EmitConfig mk = cfg;
    mk.markets = true;
    mk_plan = plan_tape(tape, mk);
    const size_t real_bytes = cfg.f32 ? 4 : 8;
    if (mk.global_ckpt && ckpt_values(mk_plan) > 0)
      cuda_check(cudaMalloc(&d_mk_gck, (size_t)ckpt_values(mk_plan) * grid * cfg.block * real_bytes),
                 "cudaMalloc market checkpoints");
    if (mk_plan.loop.present && mk_plan.loop.n_tape > 0)
      cuda_check(cudaMalloc(&d_mk_tape, (size_t)mk_plan.loop.N * mk_plan.loop.n_tape * grid * cfg.block * real_bytes),
                 "cudaMalloc market value tape");
    const int mk_smem = mk.global_ckpt ? 0 : (int)((size_t)ckpt_values(mk_plan) * cfg.block * real_bytes);
    if (mk_smem != dyn_smem) fail(NT_E_INTERNAL, "multi-market plan changed the shared checkpoint size");
    double secs = 0.0;
    std::vector<char> cubin =
        nvrtc_compile(emit(tape, mk_plan, mk), "sm_100a", use_disk_cache, &secs, cfg.fmad, max_regs_opt);
    cu_check(d.moduleLoadData(&mk_module, cubin.data()), "cuModuleLoadData (markets)");
    cu_check(d.moduleGetFunction(&mk_function, mk_module, "nt_markets_kernel"), "cuModuleGetFunction (markets)");
    if (dyn_smem > 0)
      cu_check(d.funcSetAttribute(mk_function, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, dyn_smem),
               "cuFuncSetAttribute (markets)");
    cu_check(d.funcGetAttribute(&info.markets_registers, CU_FUNC_ATTRIBUTE_NUM_REGS, mk_function),
             "cuFuncGetAttribute (markets)");
    cu_check(d.funcGetAttribute(&info.markets_local_bytes, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, mk_function),
             "cuFuncGetAttribute (markets)");
  }
  const size_t nin = (size_t)std::max<int32_t>(1, tape.n_in());
  const size_t total = (size_t)n_states * (size_t)channels;
  if ((size_t)n_states > mk_capacity) {
    cudaFree(d_mk_inputs);
    cudaFree(d_mk_acc);
    cudaFree(d_mk_partials);
    cudaFree(d_mk_out);
    d_mk_inputs = d_mk_acc = d_mk_partials = d_mk_out = nullptr;
    mk_capacity = 0;
    cuda_check(cudaMalloc(&d_mk_inputs, sizeof(double) * nin * n_states), "cudaMalloc market inputs");
    cuda_check(cudaMalloc(&d_mk_acc, sizeof(double) * 2 * total * (size_t)grid * cfg.block), "cudaMalloc market sums");
    cuda_check(cudaMalloc(&d_mk_partials, sizeof(double) * total * (size_t)grid), "cudaMalloc market partials");
    cuda_check(cudaMalloc(&d_mk_out, sizeof(double) * total), "cudaMalloc market out");
    mk_capacity = (size_t)n_states;
  }
  if (tape.n_in() > 0)
    cuda_check(cudaMemcpyAsync(d_mk_inputs, h_inputs, sizeof(double) * tape.n_in() * n_states,
                               cudaMemcpyHostToDevice, stream),
               "upload market inputs");
  const unsigned g = grid_for(paths);
  cuda_check(cudaMemsetAsync(d_mk_acc, 0, sizeof(double) * 2 * total * (size_t)g * cfg.block, stream),
             "clear market sums");
  void* gck = d_mk_gck;
  void* tp = d_mk_tape;
  int ns = n_states, accumulate = 0;
  unsigned long long n = paths, off = offset, sd = seed;
  void* args[] = {&d_mk_inputs, &ns, &n, &off, &sd, &d_mk_partials, &d_ticket, &d_mk_out, &accumulate, &gck, &tp,
                  &d_mk_acc};
  cu_check(d.launchKernel(mk_function, g, 1, 1, (unsigned)cfg.block, 1, 1, (unsigned)dyn_smem, (CUstream)stream, args,
                          nullptr),
           "cuLaunchKernel (markets)");
  ++launches;
  cuda_check(cudaMemcpyAsync(sums, d_mk_out, sizeof(double) * total, cudaMemcpyDeviceToHost, stream), "read sums");
  cuda_check(cudaStreamSynchronize(stream), "markets replay");
  if (seconds) *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

void Exec::accumulate(uint64_t paths, uint64_t offset, uint64_t seed) {
  bind();
  upload_inputs_if_dirty();
  launch(paths, offset, seed, 1);
}

// The accumulator holds exact words; the host rounds each channel's sum.
void Exec::read_accumulator(double* sums, bool reset) {
  bind();
  const size_t words = sizeof(long long) * (size_t)channels * kXWords;
  cuda_check(cudaMemcpyAsync(h_words, d_acc, words, cudaMemcpyDeviceToHost, stream), "read sums");
  if (reset) cuda_check(cudaMemsetAsync(d_acc, 0, words, stream), "reset accumulator");
  cuda_check(cudaStreamSynchronize(stream), "read accumulator");
  for (int32_t c = 0; c < channels; ++c) sums[c] = nt_exact_to_double(h_words + (size_t)c * kXWords);
}

// ---- sharding + all-reduce ------------------------------------------------------

// Shards are whole warp tiles: rank r takes a contiguous run of the
// ceil(total / 32) tiles of the range (the first ones one tile more when they
// do not divide evenly), so a tile never straddles two ranks and every rank's
// tiles hold the same paths as in a single-GPU replay.
void shard_range(uint64_t total, uint64_t offset, int32_t nranks, int32_t rank, uint64_t* from, uint64_t* count) {
  if (nranks < 1 || rank < 0 || rank >= nranks) fail(NT_E_INVALID_ARG, "bad rank / world size");
  const uint64_t r = (uint64_t)rank, n = (uint64_t)nranks;
  const uint64_t tiles = total / kTile + (total % kTile ? 1 : 0);
  const uint64_t base = tiles / n, extra = tiles % n;
  const uint64_t t0 = r * base + std::min(r, extra), nt = base + (r < extra ? 1 : 0);
  const uint64_t lo = std::min(total, t0 * kTile), hi = std::min(total, (t0 + nt) * kTile);
  *from = offset + lo;
  *count = hi - lo;
}

void Exec::shard(uint64_t total, uint64_t offset, uint64_t* from, uint64_t* count) const {
  shard_range(total, offset, nranks, rank, from, count);
}

void Exec::sharded_enqueue(uint64_t total, uint64_t offset, uint64_t seed, uint64_t chunk) {
  if (total == 0) fail(NT_E_INVALID_ARG, "paths must be positive");
  if (nranks > 1 && !comm) fail(NT_E_STATE, "executable is not attached to a communicator");
  bind();
  upload_inputs_if_dirty();
  uint64_t from = 0, count = 0;
  shard(total, offset, &from, &count);
  cuda_check(cudaMemsetAsync(d_acc, 0, sizeof(long long) * (size_t)channels * kXWords, stream), "reset accumulator");
  // Chunks are whole tiles too, so the chunking changes no tile.
  const uint64_t step = chunk > 0 ? std::max<uint64_t>(kTile, chunk - chunk % kTile) : count;
  for (uint64_t done = 0; done < count; done += step) {
    const uint64_t k = std::min(step, count - done);
    launch(k, from + done, seed, 1);
  }
  if (nranks > 1) {
    // The exact words of every rank add up to the words of the whole range:
    // one int64 all-reduce, and the sums are the same bits on any number of
    // GPUs.
    cuda_check(cudaEventRecord(ev_shard, stream), "cudaEventRecord");
    comm->allreduce_i64(d_acc, (size_t)channels * kXWords, (void*)stream);
    cuda_check(cudaEventRecord(ev_reduced, stream), "cudaEventRecord");
    reduced_once = true;
  }
}

double Exec::collective_ms() {
  if (!reduced_once) fail(NT_E_STATE, "no all-reduce has run on this executable");
  bind();
  cuda_check(cudaEventSynchronize(ev_reduced), "cudaEventSynchronize");
  float ms = 0.0f;
  cuda_check(cudaEventElapsedTime(&ms, ev_shard, ev_reduced), "cudaEventElapsedTime");
  return ms;
}

void Exec::sharded(uint64_t total, uint64_t offset, uint64_t seed, uint64_t chunk, double* sums, double* seconds) {
  const auto t0 = std::chrono::steady_clock::now();
  try {
    sharded_enqueue(total, offset, seed, chunk);
    if (nranks > 1) {
      // Bounded wait: once this rank's shard has finished, a peer that never
      // joins the all-reduce ends the call with NT_E_NCCL within the
      // communicator's timeout instead of a hang.
      comm->wait([&] {
        const cudaError_t q = cudaStreamQuery(stream);
        if (q == cudaSuccess) return Comm::Progress::Done;
        if (q != cudaErrorNotReady) cuda_check(q, "sharded replay");
        const cudaError_t e = cudaEventQuery(ev_shard);
        if (e == cudaSuccess) return Comm::Progress::Collective;
        if (e != cudaErrorNotReady) cuda_check(e, "sharded replay");
        return Comm::Progress::Computing;
      });
    }
  } catch (...) {
    if (comm && comm->aborted()) comm.reset();
    throw;
  }
  read_accumulator(sums, true);
  if (seconds) *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

void Exec::attach(int32_t n, int32_t r, const uint8_t id[128], int32_t timeout_ms) {
  if (n < 1 || r < 0 || r >= n) fail(NT_E_INVALID_ARG, "bad rank / world size");
  if (comm) fail(NT_E_STATE, "already attached");
  if (n > 1) {
    bind();
    comm = std::make_unique<Comm>(n, r, id, timeout_ms);
  }
  nranks = n;
  rank = r;
}

void Exec::detach() {
  if (comm) {
    bind();
    cudaStreamSynchronize(stream);
    comm.reset();
  }
  nranks = 1;
  rank = 0;
}

}  // namespace nt
