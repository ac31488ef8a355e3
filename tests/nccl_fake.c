/*
 * nccl_fake.c -- a stand-in NCCL library for tests/test_nccl_faults.py.
 *
 * The engine loads NCCL with dlopen from $NT_NCCL_LIBRARY when that is set.
 * This library exports the seven NCCL entry points the engine binds, with
 * NCCL's signatures, and fails on command: the host side of a peer that
 * stalls, a remote error, a failed call.  Nothing here touches a GPU.  It
 * counts the calls the engine makes, so a test can check that a failure
 * aborted the communicator exactly once and never destroyed it afterwards.
 */
#include <string.h>

typedef enum {
  ncclSuccess = 0, ncclUnhandledCudaError = 1, ncclSystemError = 2, ncclInternalError = 3,
  ncclInvalidArgument = 4, ncclInvalidUsage = 5, ncclRemoteError = 6, ncclInProgress = 7
} ncclResult_t;
typedef struct { char internal[128]; } ncclUniqueId;
typedef struct fake_comm* ncclComm_t;
struct fake_comm {
  int polls;
  int reduces;
};

enum {
  FAKE_HEALTHY = 0,          /* joins after a few polls, all-reduces complete */
  FAKE_INIT_FAILS = 1,       /* ncclCommInitRankConfig returns ncclSystemError (with a communicator) */
  FAKE_INIT_STALLS = 2,      /* the join never completes: a peer that never arrives */
  FAKE_REDUCE_FAILS = 3,     /* ncclAllReduce returns ncclInvalidUsage */
  FAKE_REMOTE_ERROR = 4,     /* after the first all-reduce, the communicator reports ncclRemoteError */
  FAKE_UNIQUE_ID_FAILS = 5,  /* ncclGetUniqueId returns ncclSystemError */
  FAKE_REDUCE_STALLS = 6     /* all-reduces are accepted but the communicator stays in progress */
};

static int g_mode = FAKE_HEALTHY;
static int g_inits, g_aborts, g_destroys, g_reduces, g_polls;
static struct fake_comm g_comm;

void fake_nccl_set_mode(int mode) {
  g_mode = mode;
  g_inits = g_aborts = g_destroys = g_reduces = g_polls = 0;
  memset(&g_comm, 0, sizeof g_comm);
}

void fake_nccl_counts(int out[5]) {
  out[0] = g_inits;
  out[1] = g_aborts;
  out[2] = g_destroys;
  out[3] = g_reduces;
  out[4] = g_polls;
}

ncclResult_t ncclGetUniqueId(ncclUniqueId* id) {
  if (g_mode == FAKE_UNIQUE_ID_FAILS) return ncclSystemError;
  memset(id->internal, 7, sizeof id->internal);
  return ncclSuccess;
}

ncclResult_t ncclCommInitRankConfig(ncclComm_t* comm, int nranks, ncclUniqueId id, int rank, void* config) {
  (void)nranks;
  (void)id;
  (void)rank;
  (void)config;
  ++g_inits;
  *comm = &g_comm;
  if (g_mode == FAKE_INIT_FAILS) return ncclSystemError;
  return ncclInProgress;
}

ncclResult_t ncclCommGetAsyncError(ncclComm_t comm, ncclResult_t* err) {
  ++g_polls;
  ++comm->polls;
  if (g_mode == FAKE_INIT_STALLS) {
    *err = ncclInProgress;
  } else if (g_mode == FAKE_REMOTE_ERROR && comm->reduces > 0) {
    *err = ncclRemoteError;
  } else if (g_mode == FAKE_REDUCE_STALLS && comm->reduces > 0) {
    *err = ncclInProgress;
  } else {
    *err = comm->polls < 3 ? ncclInProgress : ncclSuccess;
  }
  return ncclSuccess;
}

ncclResult_t ncclCommAbort(ncclComm_t comm) {
  (void)comm;
  ++g_aborts;
  return ncclSuccess;
}

ncclResult_t ncclCommDestroy(ncclComm_t comm) {
  (void)comm;
  ++g_destroys;
  return ncclSuccess;
}

ncclResult_t ncclAllReduce(const void* send, void* recv, unsigned long count, int type, int op, ncclComm_t comm,
                           void* stream) {
  (void)send;
  (void)recv;
  (void)count;
  (void)type;
  (void)op;
  (void)stream;
  ++g_reduces;
  ++comm->reduces;
  if (g_mode == FAKE_REDUCE_FAILS) return ncclInvalidUsage;
  return ncclSuccess;
}

const char* ncclGetErrorString(ncclResult_t r) {
  switch (r) {
    case ncclSuccess: return "no error";
    case ncclSystemError: return "unhandled system error (fake)";
    case ncclInvalidUsage: return "invalid usage (fake)";
    case ncclRemoteError: return "remote process exited or there was a network error (fake)";
    case ncclInProgress: return "NCCL operation in progress";
    default: return "fake NCCL error";
  }
}
