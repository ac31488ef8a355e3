// nt_dist.hpp -- the NCCL communicator of a sharded executable.
//
// NCCL is reached through dlopen, never linked: the process may already hold
// torch's copy, and a host without NCCL still loads the engine.  The library
// is $NT_NCCL_LIBRARY when that is set (the way the reference lets
// CUDA_DRIVER_PATH / NVRTC_PATH name its native libraries,
// nablatensor-engine-cuda/.../backend/cuda/CudaRuntime.java:80,102), else
// libnccl.so.2.
//
// Every wait is bounded.  The communicator is non-blocking
// (ncclConfig_t.blocking = 0); each wait polls ncclCommGetAsyncError against a
// host deadline.  On an error or at the deadline the communicator is aborted
// (ncclCommAbort, which also ends NCCL kernels still waiting on the device)
// and the call fails with NT_E_NCCL.  An aborted communicator is never used
// or destroyed again.
#pragma once

#include <nccl.h>

#include <cstddef>
#include <cstdint>
#include <functional>

#include "nt_internal.hpp"

namespace nt {

// 128-byte NCCL unique id (rank 0 creates it and broadcasts it by any means).
void dist_unique_id(uint8_t out[128]);

class Comm {
 public:
  // Progress of the work a wait covers, as the caller's poll reports it:
  // still computing (no deadline runs), the collective is the only work left
  // (the deadline runs from the first such report), or done.
  enum class Progress { Computing, Collective, Done };

  // Joins an nranks-wide communicator as `rank` on the current CUDA device.
  // Fails with NT_E_NCCL (communicator aborted) on an NCCL error or when the
  // join has not completed within timeout_ms.
  Comm(int32_t nranks, int32_t rank, const uint8_t id[128], int32_t timeout_ms);
  ~Comm();
  Comm(const Comm&) = delete;
  Comm& operator=(const Comm&) = delete;

  // Enqueues an in-place sum of `count` int64 words on `stream` and waits
  // (bounded) until NCCL has enqueued it.
  void allreduce_i64(long long* buf, size_t count, void* stream);

  // Waits until poll() returns Done.  While polling, an asynchronous NCCL
  // error aborts the communicator; so does a Collective phase that lasts
  // longer than the timeout.  poll may throw (a CUDA error); the
  // communicator is then aborted too, and the exception propagates.
  void wait(const std::function<Progress()>& poll);

  bool aborted() const { return comm_ == nullptr; }
  int32_t timeout_ms() const { return timeout_ms_; }

 private:
  [[noreturn]] void abort_and_fail(const std::string& msg);
  void wait_enqueued(const char* what);

  ncclComm_t comm_ = nullptr;
  int32_t timeout_ms_;
};

}  // namespace nt
