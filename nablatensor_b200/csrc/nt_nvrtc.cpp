// nt_nvrtc.cpp -- run-time compilation of emitted replay kernels to sm_100a.
//
// The reference compiled its generated CUDA C with NVRTC to arch-generic PTX
// (nablatensor-engine-cuda/.../backend/cuda/CudaRuntime.java:516-542) and
// cached kernels by source text (DeviceAadExecutable.java:66,114).  Here NVRTC
// produces an sm_100a cubin directly (no PTX JIT at load), the device runtime
// header is supplied as an in-memory include, and cubins are cached in memory
// and on disk keyed by a hash of (source, options, NVRTC version).
#include <nvrtc.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <mutex>
#include <sstream>
#include <sys/stat.h>
#include <unistd.h>
#include <unordered_map>

#include "nt_internal.hpp"

namespace nt {

namespace {

uint64_t fnv1a(const std::string& s, uint64_t h = 1469598103934665603ull) {
  for (unsigned char ch : s) {
    h ^= ch;
    h *= 1099511628211ull;
  }
  return h;
}

std::string cache_dir() {
  if (const char* d = std::getenv("NT_CACHE_DIR")) return d;
  if (const char* h = std::getenv("HOME")) return std::string(h) + "/.cache/nablatensor_b200";
  return "/tmp/nablatensor_b200";
}

void mkdirs(const std::string& path) {
  std::string cur;
  std::stringstream ss(path);
  std::string part;
  if (!path.empty() && path[0] == '/') cur = "/";
  while (std::getline(ss, part, '/')) {
    if (part.empty()) continue;
    cur += part + "/";
    ::mkdir(cur.c_str(), 0755);
  }
}

std::mutex g_mu;
std::unordered_map<uint64_t, std::vector<char>> g_mem;

void check(nvrtcResult r, const char* what) {
  if (r != NVRTC_SUCCESS) fail(NT_E_NVRTC, std::string(what) + ": " + nvrtcGetErrorString(r));
}

}  // namespace

std::vector<char> nvrtc_compile(const std::string& source, const std::string& arch, bool use_disk_cache,
                                double* seconds, bool fmad, int max_regs) {
  int major = 0, minor = 0;
  nvrtcVersion(&major, &minor);
  std::vector<std::string> opts = {
      "--gpu-architecture=" + arch,
      "--std=c++17",
      fmad ? "--fmad=true" : "--fmad=false",
      "-default-device",
      "--extra-device-vectorization",
      "-lineinfo",
  };
  if (max_regs > 0) opts.push_back("--maxrregcount=" + std::to_string(max_regs));
  std::string key_text = source + "\x01" + kDeviceRuntimeSource + "\x01" + kMathTablesSource + "\x01" +
                         kExactSource + "\x01" +
                         std::to_string(major) + "." + std::to_string(minor);
  for (auto& o : opts) key_text += "\x02" + o;
  const uint64_t key = fnv1a(key_text);
  if (seconds) *seconds = 0.0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_mem.find(key);
    if (it != g_mem.end()) return it->second;
  }
  char name[32];
  std::snprintf(name, sizeof name, "%016llx.cubin", (unsigned long long)key);
  const std::string path = cache_dir() + "/" + name;
  if (use_disk_cache) {
    std::ifstream f(path, std::ios::binary);
    if (f) {
      std::vector<char> bin((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
      if (bin.size() > 16) {
        std::lock_guard<std::mutex> lk(g_mu);
        g_mem[key] = bin;
        return bin;
      }
    }
  }
  const auto t0 = std::chrono::steady_clock::now();
  nvrtcProgram prog;
  const char* hdr_src[] = {kDeviceRuntimeSource, kMathTablesSource, kExactSource};
  const char* hdr_name[] = {"nt_device_rt.cuh", "nt_math_tables.cuh", "nt_exact.cuh"};
  check(nvrtcCreateProgram(&prog, source.c_str(), "nt_replay.cu", 3, hdr_src, hdr_name), "nvrtcCreateProgram");
  std::vector<const char*> copts;
  for (auto& o : opts) copts.push_back(o.c_str());
  nvrtcResult rc = nvrtcCompileProgram(prog, (int)copts.size(), copts.data());
  if (rc != NVRTC_SUCCESS) {
    size_t log_size = 0;
    nvrtcGetProgramLogSize(prog, &log_size);
    std::string log(log_size, '\0');
    if (log_size) nvrtcGetProgramLog(prog, &log[0]);
    nvrtcDestroyProgram(&prog);
    if (log.size() > 4000) log = log.substr(0, 4000) + "...";
    fail(NT_E_NVRTC, "NVRTC compile failed: " + log);
  }
  size_t n = 0;
  check(nvrtcGetCUBINSize(prog, &n), "nvrtcGetCUBINSize");
  std::vector<char> bin(n);
  check(nvrtcGetCUBIN(prog, bin.data()), "nvrtcGetCUBIN");
  nvrtcDestroyProgram(&prog);
  if (seconds) *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  if (use_disk_cache) {
    mkdirs(cache_dir());
    const std::string tmp = path + ".tmp" + std::to_string((unsigned long long)key ^ (uint64_t)::getpid());
    std::ofstream f(tmp, std::ios::binary);
    if (f) {
      f.write(bin.data(), (std::streamsize)bin.size());
      f.close();
      std::rename(tmp.c_str(), path.c_str());
    }
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_mem[key] = bin;
  return bin;
}

}  // namespace nt
