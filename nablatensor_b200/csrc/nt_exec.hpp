// nt_exec.hpp -- the compiled executable behind an nt_exec handle.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <memory>
#include <mutex>

#include "nt_dist.hpp"
#include "nt_internal.hpp"

namespace nt {

void cuda_check(cudaError_t e, const char* what);
void shard_range(uint64_t total, uint64_t offset, int32_t nranks, int32_t rank, uint64_t* from, uint64_t* count);
size_t noalloc_scratch_bytes();

struct Exec {
  std::mutex mu;
  Tape tape;
  Plan plan;
  EmitConfig cfg;
  std::string source;
  int device = -1;
  bool use_disk_cache = true;
  int max_regs_opt = 0;  // nt_options.max_regs, kept for the kernels compiled later
  bool auto_seg = true;   // no segment length or block size given: load() may widen a one-unit segment
  bool auto_regs = true;  // no register cap or block minimum given: load() may cap a kernel that ran out
  CUmodule module = nullptr;
  CUfunction function = nullptr;
  cudaStream_t stream = nullptr;
  int sm_count = 0, blocks_per_sm = 0, grid = 0, dyn_smem = 0;
  int32_t channels = 0;
  double* d_inputs = nullptr;
  long long* d_glim = nullptr;  // a launch's exact words, channels x kXWords (left zero by every launch)
  unsigned int* d_ticket = nullptr;
  double* d_out = nullptr;      // a launch's rounded sums
  long long* d_acc = nullptr;   // the device accumulator: exact words, channels x kXWords
  void* d_gck = nullptr;
  void* d_tape = nullptr;
  double* h_stage = nullptr;    // pinned: inputs, then sums
  long long* h_words = nullptr; // pinned: the accumulator's words on their way to the host
  cudaEvent_t ev_shard = nullptr;  // recorded once this rank's shard is enqueued, before the all-reduce
  cudaEvent_t ev_reduced = nullptr;  // recorded after the all-reduce (timing: ev_shard -> ev_reduced)
  bool reduced_once = false;
  std::vector<double> inputs;
  bool dirty = true;
  double compile_seconds = 0.0;
  uint64_t launches = 0;
  nt_exec_info info{};
  // Multi-market kernel (compiled on first use) and its buffers, grown to
  // the largest market count seen.
  CUmodule mk_module = nullptr;
  CUfunction mk_function = nullptr;
  double* d_mk_inputs = nullptr;
  double* d_mk_acc = nullptr;
  double* d_mk_partials = nullptr;
  double* d_mk_out = nullptr;
  size_t mk_capacity = 0;  // markets the buffers hold
  Plan mk_plan;            // draws-only value tape (see markets())
  void* d_mk_gck = nullptr;
  void* d_mk_tape = nullptr;
  // multi-GPU
  std::unique_ptr<Comm> comm;
  int32_t nranks = 1, rank = 0;

  static Exec* create(const nt_tape* tape, const nt_options* opt);
  ~Exec();

  void bind() const;
  void load(int max_regs);
  void upload_inputs_if_dirty();
  // accumulate == 0: the rounded sums go to d_out; else the exact words are
  // added to d_acc.
  void launch(uint64_t paths, uint64_t offset, uint64_t seed, int accumulate);
  // Launch with caller-provided device pointers on a caller stream (no
  // executable-owned buffers); `grid` blocks, the launch's exact words in
  // `glim` (zero on entry, left zero).
  void launch_external(uint64_t paths, uint64_t offset, uint64_t seed, const double* d_inputs, double* d_out,
                       unsigned int* ticket, long long* glim, cudaStream_t s, unsigned grid_blocks);
  unsigned grid_for(uint64_t paths) const;
  void replay(uint64_t paths, uint64_t offset, uint64_t seed, double* sums, double* seconds);
  void accumulate(uint64_t paths, uint64_t offset, uint64_t seed);
  void read_accumulator(double* sums, bool reset);
  void shard(uint64_t total, uint64_t offset, uint64_t* from, uint64_t* count) const;
  void sharded_enqueue(uint64_t total, uint64_t offset, uint64_t seed, uint64_t chunk);
  void sharded(uint64_t total, uint64_t offset, uint64_t seed, uint64_t chunk, double* sums, double* seconds);
  void attach(int32_t n, int32_t r, const uint8_t id[128], int32_t timeout_ms);
  // One launch over `n_states` input vectors sharing each scenario's draws.
  void markets(int32_t n_states, const double* inputs, uint64_t paths, uint64_t offset, uint64_t seed,
               double* sums, double* seconds);
  void detach();
  // Device time of the last all-reduce (waits for it), in milliseconds.
  double collective_ms();
};

}  // namespace nt

// The opaque handle behind the C ABI's nt_exec*.
struct nt_exec {
  nt::Exec* impl;
};

namespace nt {
// nt_replay_noalloc (nt_noalloc.cu).
void replay_noalloc(nt_exec* handle, uint64_t paths, uint64_t path_offset, uint64_t seed, const double* d_inputs,
                    double* d_sums, void* stream);
}  // namespace nt
