// nccl_fault_harness.cpp -- drives the engine's communicator (csrc/nt_dist.cpp,
// compiled from the product source by tests/test_nccl_faults.py) against the
// stand-in NCCL of tests/nccl_fake.c, on the host, without a GPU.
//
// For each case it prints one JSON line: the status code the engine raised
// (0 when none), whether the communicator ended aborted, the fake's call
// counts and the elapsed milliseconds.
#include <dlfcn.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <stdexcept>
#include <string>

#include "nt_dist.hpp"

namespace {

void (*set_mode)(int) = nullptr;
void (*counts)(int*) = nullptr;

struct Outcome {
  int code = 0;
  bool aborted = false;
  std::string message;
};

void report(const char* name, const Outcome& o, double ms) {
  int c[5];
  counts(c);
  std::string msg;
  for (char ch : o.message) msg += (ch == '"' || ch == '\\') ? ' ' : ch;
  std::printf(
      "{\"case\": \"%s\", \"code\": %d, \"aborted\": %s, \"inits\": %d, \"aborts\": %d, \"destroys\": %d, "
      "\"reduces\": %d, \"ms\": %.1f, \"message\": \"%s\"}\n",
      name, o.code, o.aborted ? "true" : "false", c[0], c[1], c[2], c[3], ms, msg.c_str());
  std::fflush(stdout);
}

template <class F>
void run(const char* name, int mode, F&& body) {
  set_mode(mode);
  Outcome o;
  const auto t0 = std::chrono::steady_clock::now();
  try {
    body(o);
  } catch (const nt::Error& e) {
    o.code = e.code;
    o.message = e.what();
  } catch (const std::exception& e) {
    o.code = 1000;
    o.message = e.what();
  }
  report(name, o, std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
}

const uint8_t kId[128] = {};
long long g_words[4];

}  // namespace

int main() {
  const char* path = std::getenv("NT_NCCL_LIBRARY");
  void* h = path ? dlopen(path, RTLD_NOW | RTLD_GLOBAL) : nullptr;
  if (!h) {
    std::fprintf(stderr, "NT_NCCL_LIBRARY must name the fake NCCL library\n");
    return 2;
  }
  set_mode = (void (*)(int))dlsym(h, "fake_nccl_set_mode");
  counts = (void (*)(int*))dlsym(h, "fake_nccl_counts");
  const int timeout = 300;
  using P = nt::Comm::Progress;

  run("healthy", 0, [&](Outcome& o) {
    std::unique_ptr<nt::Comm> c(new nt::Comm(2, 0, kId, timeout));
    c->allreduce_i64(g_words, 4, nullptr);
    int polls = 0;
    c->wait([&] { return ++polls < 5 ? P::Collective : P::Done; });
    o.aborted = c->aborted();
  });
  run("unique_id_fails", 5, [&](Outcome&) {
    uint8_t id[128];
    nt::dist_unique_id(id);
  });
  run("init_fails", 1, [&](Outcome&) { nt::Comm c(2, 1, kId, timeout); });
  run("init_stalls", 2, [&](Outcome&) { nt::Comm c(2, 1, kId, timeout); });
  run("allreduce_fails", 3, [&](Outcome& o) {
    std::unique_ptr<nt::Comm> c(new nt::Comm(2, 0, kId, timeout));
    try {
      c->allreduce_i64(g_words, 4, nullptr);
    } catch (...) {
      o.aborted = c->aborted();
      throw;
    }
  });
  run("remote_error_after_enqueue", 4, [&](Outcome& o) {
    std::unique_ptr<nt::Comm> c(new nt::Comm(2, 0, kId, timeout));
    try {
      c->allreduce_i64(g_words, 4, nullptr);
    } catch (...) {
      o.aborted = c->aborted();
      throw;
    }
  });
  run("peer_never_joins", 6, [&](Outcome& o) {
    std::unique_ptr<nt::Comm> c(new nt::Comm(2, 0, kId, timeout));
    try {
      c->allreduce_i64(g_words, 4, nullptr);
    } catch (...) {
      o.aborted = c->aborted();
      throw;
    }
  });
  // The collective is enqueued (the healthy fake), but the stream never
  // finishes it: the peer left.  The deadline runs only once the shard is
  // done, so a long Computing phase is not cut short.
  run("collective_never_completes", 0, [&](Outcome& o) {
    std::unique_ptr<nt::Comm> c(new nt::Comm(2, 0, kId, timeout));
    c->allreduce_i64(g_words, 4, nullptr);
    const auto t0 = std::chrono::steady_clock::now();
    try {
      c->wait([&] {
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        return ms < 2.0 * timeout ? P::Computing : P::Collective;
      });
    } catch (...) {
      o.aborted = c->aborted();
      throw;
    }
  });
  run("cuda_error_while_waiting", 0, [&](Outcome& o) {
    std::unique_ptr<nt::Comm> c(new nt::Comm(2, 0, kId, timeout));
    c->allreduce_i64(g_words, 4, nullptr);
    try {
      c->wait([]() -> P { throw nt::Error(NT_E_CUDA, "simulated CUDA failure of the stream"); });
    } catch (...) {
      o.aborted = c->aborted();
      throw;
    }
  });
  run("use_after_abort", 0, [&](Outcome& o) {
    std::unique_ptr<nt::Comm> c(new nt::Comm(2, 0, kId, timeout));
    try {
      c->wait([]() -> P { throw nt::Error(NT_E_CUDA, "first failure"); });
    } catch (const nt::Error&) {
    }
    o.aborted = c->aborted();
    c->allreduce_i64(g_words, 4, nullptr);  // must refuse, not touch the aborted communicator
  });
  return 0;
}
