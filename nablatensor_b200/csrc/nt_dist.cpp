// nt_dist.cpp -- the NCCL communicator of a sharded executable (nt_dist.hpp).
//
// The reference has no distributed code; this is the one collective of the
// multi-GPU replay: every rank replays a contiguous shard of the scenario
// range and the ranks sum their accumulators with one ncclAllReduce over
// NVLink / NVSwitch.  Nothing here calls the CUDA runtime, so the failure
// handling can be exercised on a host without a GPU against a stand-in NCCL
// library named by NT_NCCL_LIBRARY.
#include "nt_dist.hpp"

#include <dlfcn.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>

namespace nt {

namespace {

struct NcclApi {
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*getErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
  std::string err;
};

NcclApi& nccl() {
  static NcclApi n;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* named = std::getenv("NT_NCCL_LIBRARY");
    void* h = nullptr;
    if (named && *named) {
      h = dlopen(named, RTLD_NOW | RTLD_GLOBAL);
    } else {
      h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
      if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    }
    if (!h) {
      const char* e = dlerror();
      n.err = std::string("cannot load ") + (named && *named ? named : "libnccl.so.2") + ": " + (e ? e : "?");
      return;
    }
    auto sym = [&](const char* s) { return dlsym(h, s); };
    n.getUniqueId = (decltype(n.getUniqueId))sym("ncclGetUniqueId");
    n.commInitRankConfig = (decltype(n.commInitRankConfig))sym("ncclCommInitRankConfig");
    n.commGetAsyncError = (decltype(n.commGetAsyncError))sym("ncclCommGetAsyncError");
    n.commAbort = (decltype(n.commAbort))sym("ncclCommAbort");
    n.commDestroy = (decltype(n.commDestroy))sym("ncclCommDestroy");
    n.allReduce = (decltype(n.allReduce))sym("ncclAllReduce");
    n.getErrorString = (decltype(n.getErrorString))sym("ncclGetErrorString");
    n.ok = n.getUniqueId && n.commInitRankConfig && n.commGetAsyncError && n.commAbort && n.commDestroy &&
           n.allReduce && n.getErrorString;
    if (!n.ok) n.err = "the NCCL library lacks a required symbol";
  });
  if (!n.ok) fail(NT_E_NCCL, n.err);
  return n;
}

std::string nccl_error(ncclResult_t r) {
  const char* s = nccl().getErrorString(r);
  return std::string(s ? s : "unknown NCCL error") + " (" + std::to_string((int)r) + ")";
}

using Clock = std::chrono::steady_clock;

}  // namespace

void dist_unique_id(uint8_t out[128]) {
  ncclUniqueId uid;
  static_assert(sizeof(uid.internal) == 128, "NCCL unique id is 128 bytes");
  const ncclResult_t r = nccl().getUniqueId(&uid);
  if (r != ncclSuccess) fail(NT_E_NCCL, "ncclGetUniqueId: " + nccl_error(r));
  std::memcpy(out, uid.internal, 128);
}

Comm::Comm(int32_t nranks, int32_t rank, const uint8_t id[128], int32_t timeout_ms)
    : timeout_ms_(timeout_ms > 0 ? timeout_ms : 60000) {
  if (nranks < 2 || rank < 0 || rank >= nranks) fail(NT_E_INVALID_ARG, "bad rank / world size");
  ncclUniqueId uid;
  std::memcpy(uid.internal, id, 128);
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  ncclComm_t c = nullptr;
  const ncclResult_t r = nccl().commInitRankConfig(&c, nranks, uid, rank, &config);
  comm_ = c;
  if (r != ncclSuccess && r != ncclInProgress) {
    if (comm_) abort_and_fail("ncclCommInitRankConfig: " + nccl_error(r));
    fail(NT_E_NCCL, "ncclCommInitRankConfig: " + nccl_error(r));
  }
  if (!comm_) fail(NT_E_NCCL, "ncclCommInitRankConfig returned no communicator");
  wait_enqueued("ncclCommInitRank");
}

Comm::~Comm() {
  if (comm_) nccl().commDestroy(comm_);
}

void Comm::abort_and_fail(const std::string& msg) {
  ncclComm_t c = comm_;
  comm_ = nullptr;
  if (c) nccl().commAbort(c);
  fail(NT_E_NCCL, msg + "; communicator aborted");
}

// A non-blocking call returns before NCCL has finished it; the communicator
// reports ncclInProgress until then.
void Comm::wait_enqueued(const char* what) {
  if (!comm_) fail(NT_E_STATE, "the communicator was aborted by an earlier failure");
  const auto t0 = Clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t q = nccl().commGetAsyncError(comm_, &st);
    if (q != ncclSuccess) abort_and_fail(std::string(what) + ": ncclCommGetAsyncError: " + nccl_error(q));
    if (st == ncclSuccess) return;
    if (st != ncclInProgress) abort_and_fail(std::string(what) + ": " + nccl_error(st));
    if (Clock::now() - t0 > std::chrono::milliseconds(timeout_ms_))
      abort_and_fail(std::string(what) + ": not complete after " + std::to_string(timeout_ms_) + " ms");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void Comm::allreduce_i64(long long* buf, size_t count, void* stream) {
  if (!comm_) fail(NT_E_STATE, "the communicator was aborted by an earlier failure");
  const ncclResult_t r = nccl().allReduce(buf, buf, count, ncclInt64, ncclSum, comm_, (cudaStream_t)stream);
  if (r != ncclSuccess && r != ncclInProgress) abort_and_fail("ncclAllReduce: " + nccl_error(r));
  wait_enqueued("ncclAllReduce");
}

void Comm::wait(const std::function<Progress()>& poll) {
  if (!comm_) fail(NT_E_STATE, "the communicator was aborted by an earlier failure");
  bool timing = false;
  Clock::time_point t0;
  for (;;) {
    Progress p;
    try {
      p = poll();
    } catch (...) {
      ncclComm_t c = comm_;
      comm_ = nullptr;
      if (c) nccl().commAbort(c);
      throw;
    }
    if (p == Progress::Done) return;
    ncclResult_t st = ncclSuccess;
    const ncclResult_t q = nccl().commGetAsyncError(comm_, &st);
    if (q != ncclSuccess) abort_and_fail("all-reduce: ncclCommGetAsyncError: " + nccl_error(q));
    if (st != ncclSuccess && st != ncclInProgress) abort_and_fail("all-reduce failed: " + nccl_error(st));
    if (p == Progress::Collective) {
      if (!timing) {
        timing = true;
        t0 = Clock::now();
      } else if (Clock::now() - t0 > std::chrono::milliseconds(timeout_ms_)) {
        abort_and_fail("all-reduce not complete " + std::to_string(timeout_ms_) +
                       " ms after this rank's shard finished (a peer left or stalled)");
      }
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

}  // namespace nt
