// nt_api.cpp -- the extern "C" boundary (include/nabla_b200.h).
//
// Every entry point catches everything: no C++ exception crosses the ABI, no
// abort/exit.  Failures become a negative NT_E_* status plus a thread-local
// message, the way the reference mapped driver errors to exceptions with the
// driver's error name (nablatensor-engine-cuda/.../CudaRuntime.java:124-137).
#include <cstring>
#include <new>

#include "nt_exec.hpp"

namespace {

thread_local std::string g_error;

int set_error(int code, const std::string& msg) {
  g_error = msg;
  return code;
}

template <class F>
int guarded(F&& f) {
  try {
    g_error.clear();
    f();
    return NT_OK;
  } catch (const nt::Error& e) {
    return set_error(e.code, e.what());
  } catch (const std::bad_alloc&) {
    return set_error(NT_E_OOM, "host allocation failed");
  } catch (const std::exception& e) {
    return set_error(NT_E_INTERNAL, e.what());
  } catch (...) {
    return set_error(NT_E_INTERNAL, "unknown failure");
  }
}

nt::Exec& impl(nt_exec* x) {
  if (!x || !x->impl) nt::fail(NT_E_STATE, "executable is closed");
  return *x->impl;
}

void copy_out(const std::string& s, char* buf, size_t cap, size_t* len) {
  if (len) *len = s.size();
  if (buf && cap) {
    const size_t k = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), k);
    buf[k] = '\0';
  }
}

}  // namespace

extern "C" {

int nt_version(void) { return NT_ABI_VERSION; }

const char* nt_last_error(void) { return g_error.c_str(); }

int nt_init(int32_t* n_devices) {
  return guarded([&] {
    if (!n_devices) nt::fail(NT_E_INVALID_ARG, "n_devices is null");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
      cudaGetLastError();
      *n_devices = 0;
      return;
    }
    nt::cuda_check(e, "cudaGetDeviceCount");
    *n_devices = n;
  });
}

int nt_compile(const nt_tape* tape, const nt_options* options, nt_exec** out) {
  return guarded([&] {
    if (!out) nt::fail(NT_E_INVALID_ARG, "out is null");
    *out = nullptr;
    nt::Exec* e = nt::Exec::create(tape, options);
    *out = new nt_exec{e};
  });
}

int nt_set_inputs(nt_exec* exec, const double* inputs, int32_t n) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    if (n != x.tape.n_in()) nt::fail(NT_E_INVALID_ARG, "expected " + std::to_string(x.tape.n_in()) + " inputs");
    if (n > 0 && !inputs) nt::fail(NT_E_INVALID_ARG, "inputs is null");
    for (int32_t j = 0; j < n; ++j) x.inputs[j] = inputs[j];
    x.dirty = true;
  });
}

int nt_replay(nt_exec* exec, uint64_t paths, uint64_t path_offset, uint64_t seed, double* sums, double* seconds) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    if (!sums) nt::fail(NT_E_INVALID_ARG, "sums is null");
    if (paths == 0) nt::fail(NT_E_INVALID_ARG, "paths must be positive");
    x.replay(paths, path_offset, seed, sums, seconds);
  });
}

int nt_replay_markets(nt_exec* exec, int32_t n_states, const double* inputs, uint64_t paths, uint64_t path_offset,
                      uint64_t seed, double* sums, double* seconds) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    x.markets(n_states, inputs, paths, path_offset, seed, sums, seconds);
  });
}

int nt_replay_accumulate(nt_exec* exec, uint64_t paths, uint64_t path_offset, uint64_t seed) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    if (paths == 0) nt::fail(NT_E_INVALID_ARG, "paths must be positive");
    x.accumulate(paths, path_offset, seed);
  });
}

int nt_accumulator_read(nt_exec* exec, double* sums, int32_t reset) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    if (!sums) nt::fail(NT_E_INVALID_ARG, "sums is null");
    x.read_accumulator(sums, reset != 0);
  });
}

int nt_exec_stream(nt_exec* exec, void** stream) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    if (!stream) nt::fail(NT_E_INVALID_ARG, "stream is null");
    *stream = (void*)x.stream;
  });
}

int nt_exec_info_get(nt_exec* exec, nt_exec_info* info) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    if (!info) nt::fail(NT_E_INVALID_ARG, "info is null");
    *info = x.info;
  });
}

int nt_exec_source(nt_exec* exec, char* buf, size_t cap, size_t* len) {
  return guarded([&] { copy_out(impl(exec).source, buf, cap, len); });
}

int nt_emit_source(const nt_tape* tape, const nt_options* options, int32_t target, char* buf, size_t cap,
                   size_t* len) {
  return guarded([&] {
    nt::EmitConfig cfg = nt::config_from(options, target);
    nt::Tape t = nt::ingest(tape);
    nt::reduce_pow2_divisions(t, cfg.f32);
    nt::Plan p = nt::plan_tape(t, cfg);
    if (options->block == 0) cfg.block = nt::auto_block(p);
    copy_out(nt::emit(t, p, cfg), buf, cap, len);
  });
}

int nt_nvrtc_check(const char* source, size_t* cubin_bytes) {
  return guarded([&] {
    if (!source) nt::fail(NT_E_INVALID_ARG, "source is null");
    double secs = 0;
    std::vector<char> bin = nt::nvrtc_compile(source, "sm_100a", false, &secs);
    if (cubin_bytes) *cubin_bytes = bin.size();
  });
}

int nt_nvrtc_version(int32_t* major, int32_t* minor, char* path, size_t cap, size_t* len) {
  return guarded([&] {
    if (!major || !minor) nt::fail(NT_E_INVALID_ARG, "major / minor is null");
    int ma = 0, mi = 0;
    nt::nvrtc_version(&ma, &mi);
    *major = ma;
    *minor = mi;
    copy_out(nt::nvrtc_path(), path, cap, len);
  });
}

void nt_destroy(nt_exec* exec) {
  if (!exec) return;
  try {
    delete exec->impl;
  } catch (...) {
  }
  exec->impl = nullptr;
  delete exec;
}

int nt_dist_unique_id(uint8_t id[128]) {
  return guarded([&] {
    if (!id) nt::fail(NT_E_INVALID_ARG, "id is null");
    nt::dist_unique_id(id);
  });
}

int nt_dist_attach(nt_exec* exec, int32_t nranks, int32_t rank, const uint8_t id[128], int32_t timeout_ms) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    if (nranks > 1 && !id) nt::fail(NT_E_INVALID_ARG, "id is null");
    x.attach(nranks, rank, id, timeout_ms);
  });
}

int nt_replay_sharded(nt_exec* exec, uint64_t total_paths, uint64_t path_offset, uint64_t seed, uint64_t chunk_paths,
                      double* sums, double* seconds) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    if (!sums) nt::fail(NT_E_INVALID_ARG, "sums is null");
    x.sharded(total_paths, path_offset, seed, chunk_paths, sums, seconds);
  });
}

int nt_replay_sharded_async(nt_exec* exec, uint64_t total_paths, uint64_t path_offset, uint64_t seed,
                            uint64_t chunk_paths) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    x.sharded_enqueue(total_paths, path_offset, seed, chunk_paths);
  });
}

int nt_shard_range(uint64_t total_paths, uint64_t path_offset, int32_t nranks, int32_t rank, uint64_t* from,
                   uint64_t* count) {
  return guarded([&] {
    if (!from || !count) nt::fail(NT_E_INVALID_ARG, "from/count is null");
    nt::shard_range(total_paths, path_offset, nranks, rank, from, count);
  });
}

int nt_dist_collective_ms(nt_exec* exec, double* ms) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    if (!ms) nt::fail(NT_E_INVALID_ARG, "ms is null");
    *ms = x.collective_ms();
  });
}

int nt_dist_detach(nt_exec* exec) {
  return guarded([&] {
    nt::Exec& x = impl(exec);
    std::lock_guard<std::mutex> lk(x.mu);
    x.detach();
  });
}

}  // extern "C"

extern "C" int nt_philox_words(int32_t device, uint64_t path0, uint32_t n_paths, uint64_t seed, int32_t stream,
                               uint32_t pair0, uint32_t n_pairs, uint32_t* out, double* normals) {
  return guarded([&] { nt::philox_words(device, path0, n_paths, seed, stream, pair0, n_pairs, out, normals); });
}

extern "C" int nt_replay_noalloc(nt_exec* exec, uint64_t paths, uint64_t path_offset, uint64_t seed,
                                 const double* d_inputs, double* d_sums, void* stream) {
  return guarded([&] { nt::replay_noalloc(exec, paths, path_offset, seed, d_inputs, d_sums, stream); });
}

extern "C" int nt_math_eval(int32_t device, int32_t which, int64_t n, const uint32_t* words, const double* x,
                            double* out0, double* out1) {
  return guarded([&] { nt::math_eval(device, which, n, words, x, out0, out1); });
}

extern "C" int nt_fma_peak(int32_t device, int32_t fp64, int32_t iters, double* tflops) {
  return guarded([&] {
    if (!tflops) nt::fail(NT_E_INVALID_ARG, "tflops is null");
    if (iters <= 0) nt::fail(NT_E_INVALID_ARG, "iters must be positive");
    *tflops = nt::fma_peak_tflops(device, fp64, iters);
  });
}

extern "C" int nt_fma_peak_sustained(int32_t device, int32_t fp64, int32_t millis, double* tflops) {
  return guarded([&] {
    if (!tflops) nt::fail(NT_E_INVALID_ARG, "tflops is null");
    if (millis <= 0 || millis > 60000) nt::fail(NT_E_INVALID_ARG, "millis must be in [1, 60000]");
    *tflops = nt::fma_peak_sustained_tflops(device, fp64, millis);
  });
}
