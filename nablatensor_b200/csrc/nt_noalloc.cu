// nt_noalloc.cu -- a replay launch that allocates nothing.
//
// Some callers cannot let the engine allocate device memory on their behalf:
// a host that hands the whole device to its own memory pool under a fixed
// budget (NablaTensor's Java runtime pools and budgets every device
// allocation, so memory taken behind its back breaks its accounting), and a
// host pricing inside a latency-critical loop, where cudaMalloc and cudaFree
// would synchronise the device.  For them nt_replay_noalloc launches an
// already-compiled replay kernel on the caller's own device buffers and
// stream.  The kernel's only scratch -- the reduction ticket and the launch's
// exact-sum words (one record of 69 int64 per channel) -- lives in the
// file-scope array below, of a fixed maximum size that every GPU loading
// this library holds until the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents, so calls that overlap on the same GPU race on it; the caller
// serialises them (one stream, or events).  Each call clears the ticket and
// its words on the caller's stream before the launch.
#include <mutex>

#include "nt_exec.hpp"

namespace {

// Bytes of scratch: 256 for the ticket, the rest the exact-sum words.
constexpr size_t kScratchBytes = 64u << 10;  // 118 channels at most
constexpr size_t kTicketBytes = 256;

static __device__ __align__(256) unsigned char nt_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};

// Per-device set-up, once per device, with that device current: the
// host-side name of a __device__ array is not a device address, so the
// address comes from cudaGetSymbolAddress (which can load the module on
// first use; make the first call on a device before any stream capture).
// The address stays valid until the process ends or the device is reset:
// nt_replay_noalloc must not be used across a cudaDeviceReset.
void* scratch_for(int device) {
  if (device < 0 || device >= kMaxDevices) nt::fail(NT_E_INVALID_ARG, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch[device]) {
    void* p = nullptr;
    nt::cuda_check(cudaGetSymbolAddress(&p, nt_noalloc_scratch), "cudaGetSymbolAddress(nt_noalloc_scratch)");
    g_scratch[device] = p;
  }
  return g_scratch[device];
}

// A caller's buffer must be device (or managed) memory of the executable's
// GPU: a host pointer or another GPU's memory handed to the kernel would
// fault the device instead of failing the call.
void require_device_memory(const void* p, int device, const char* what) {
  cudaPointerAttributes a{};
  const cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    nt::fail(NT_E_INVALID_ARG, std::string(what) + " is not a CUDA pointer");
  }
  if ((a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) || a.device != device)
    nt::fail(NT_E_INVALID_ARG, std::string(what) + " must be device memory of GPU " + std::to_string(device));
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
         "nt_replay_noalloc needs an executable with no value tape and no global checkpoints "
         "(compile it with NT_FLAG_RECOMPUTE_ALL | NT_FLAG_SHARED_CKPT)");
  }
  const size_t words = (size_t)x.channels * kXWords * sizeof(long long);
  const size_t need = kTicketBytes + words;
  if (need > kScratchBytes) {
    fail(NT_E_INVALID_ARG, "nt_replay_noalloc: " + std::to_string(x.channels) + " channels need " +
                               std::to_string(need) + " bytes of reduction scratch; the static maximum is " +
                               std::to_string(kScratchBytes) + " bytes");
  }
  x.bind();
  require_device_memory(d_sums, x.device, "d_sums");
  if (x.tape.n_in() > 0) require_device_memory(d_inputs, x.device, "d_inputs");
  unsigned char* base = (unsigned char*)scratch_for(x.device);
  unsigned int* ticket = (unsigned int*)base;
  long long* glim = (long long*)(base + kTicketBytes);
  cudaStream_t s = (cudaStream_t)stream;
  cuda_check(cudaMemsetAsync(base, 0, need, s), "clear the reduction scratch");
  x.launch_external(paths, path_offset, seed, d_inputs, d_sums, ticket, glim, s, x.grid_for(paths));
}

}  // namespace nt
