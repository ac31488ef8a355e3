// nt_noalloc.cu -- a replay launch that allocates nothing.
//
// Some callers cannot let the engine allocate device memory on their behalf:
// a host that hands the whole device to its own memory pool under a fixed
// budget (NablaTensor's Java runtime pools and budgets every device
// allocation, so memory taken behind its back breaks its accounting), and a
// host pricing inside a latency-critical loop, where cudaMalloc and cudaFree
// would synchronise the device.  For them nt_replay_noalloc launches an
// already-compiled replay kernel on the caller's own device buffers and
// stream.  The kernel's only scratch --
// one partial record per block and the reduction ticket -- lives in the
// file-scope array below, of a fixed maximum size that every GPU loading this
// library holds until the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents, so calls that overlap on the same GPU race on it; the caller
// serialises them (one stream, or events).  The ticket is cleared at the
// start of every call; the partial records are fully rewritten by each
// launch before they are read.
#include <mutex>

#include "nt_exec.hpp"

namespace {

// Bytes of scratch: 256 for the ticket, the rest partial records.
constexpr size_t kScratchBytes = 1u << 20;
constexpr size_t kTicketBytes = 256;

static __device__ __align__(256) unsigned char nt_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};

// Per-device set-up, on the device that is current: the host-side name of a
// __device__ array is not a device address, so the address comes from
// cudaGetSymbolAddress.  The ticket is zeroed synchronously here, so the
// first call on a device must come before any stream capture.
void* scratch_for(int device) {
  if (device < 0 || device >= kMaxDevices) nt::fail(NT_E_INVALID_ARG, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch[device]) {
    void* p = nullptr;
    nt::cuda_check(cudaGetSymbolAddress(&p, nt_noalloc_scratch), "cudaGetSymbolAddress(nt_noalloc_scratch)");
    nt::cuda_check(cudaMemset(p, 0, kTicketBytes), "clear the reduction ticket");
    g_scratch[device] = p;
  }
  return g_scratch[device];
}

}  // namespace

namespace nt {

size_t noalloc_scratch_bytes() { return kScratchBytes; }

void replay_noalloc(nt_exec* handle, uint64_t paths, uint64_t path_offset, uint64_t seed, const double* d_inputs,
                    double* d_sums, void* stream) {
  if (!handle || !handle->impl) fail(NT_E_STATE, "executable is closed");
  Exec& x = *handle->impl;
  std::lock_guard<std::mutex> lk(x.mu);
  if (paths == 0) fail(NT_E_INVALID_ARG, "paths must be positive");
  if (!d_sums || (x.tape.n_in() > 0 && !d_inputs)) fail(NT_E_INVALID_ARG, "device inputs / sums pointer is null");
  if (x.d_tape != nullptr || x.d_gck != nullptr) {
    fail(NT_E_UNSUPPORTED,
         "nt_replay_noalloc needs an executable compiled with NT_FLAG_RECOMPUTE_ALL | NT_FLAG_SHARED_CKPT "
         "(its kernel then uses no global scratch beyond the reduction records)");
  }
  const unsigned grid = x.grid_for(paths);
  const size_t need = kTicketBytes + (size_t)grid * (size_t)x.channels * sizeof(double);
  if (need > kScratchBytes) {
    fail(NT_E_INVALID_ARG, "nt_replay_noalloc: " + std::to_string(grid) + " blocks x " + std::to_string(x.channels) +
                               " channels need " + std::to_string(need) + " bytes of reduction scratch; the static "
                               "maximum is " + std::to_string(kScratchBytes) + " bytes");
  }
  x.bind();
  unsigned char* base = (unsigned char*)scratch_for(x.device);
  unsigned int* ticket = (unsigned int*)base;
  double* partials = (double*)(base + kTicketBytes);
  cudaStream_t s = (cudaStream_t)stream;
  cuda_check(cudaMemsetAsync(ticket, 0, sizeof(unsigned int), s), "clear the reduction ticket");
  x.launch_external(paths, path_offset, seed, d_inputs, d_sums, ticket, partials, s, grid);
}

}  // namespace nt
