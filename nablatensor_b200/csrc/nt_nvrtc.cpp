// nt_nvrtc.cpp -- run-time compilation of emitted replay kernels to sm_100a.
//
// The reference compiled its generated CUDA C with NVRTC to arch-generic PTX
// (nablatensor-engine-cuda/.../backend/cuda/CudaRuntime.java:516-542) and
// cached kernels by source text (DeviceAadExecutable.java:66,114).  Here NVRTC
// produces an sm_100a cubin directly (no PTX JIT at load), the device runtime
// header is supplied as an in-memory include, and cubins are cached in memory
// and on disk keyed by a hash of (source, options, NVRTC version).
//
// NVRTC is loaded by path, privately (RTLD_LOCAL), from the CUDA toolkit the
// library was built with -- not as whichever libnvrtc.so.12 the process
// happens to hold.  A host that imports another copy first (PyTorch ships
// its own) would otherwise swap the compiler under the engine, and two NVRTC
// versions may fuse a multiply-add differently: an fp32 kernel's sums then
// depend on import order.  NT_NVRTC_LIBRARY names another copy explicitly.
#include <dlfcn.h>
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

#ifndef NT_NVRTC_DEFAULT
#define NT_NVRTC_DEFAULT "libnvrtc.so.12"
#endif

namespace nt {

namespace {

struct NvrtcApi {
  nvrtcResult (*version)(int*, int*) = nullptr;
  nvrtcResult (*create)(nvrtcProgram*, const char*, const char*, int, const char* const*,
                        const char* const*) = nullptr;
  nvrtcResult (*compile)(nvrtcProgram, int, const char* const*) = nullptr;
  nvrtcResult (*log_size)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*log)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*cubin_size)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*cubin)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*destroy)(nvrtcProgram*) = nullptr;
  const char* (*error_string)(nvrtcResult) = nullptr;
  std::string path, err;
  bool ok = false;
};

const NvrtcApi& api() {
  static NvrtcApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* named = std::getenv("NT_NVRTC_LIBRARY");
    a.path = named && *named ? named : NT_NVRTC_DEFAULT;
    void* h = dlopen(a.path.c_str(), RTLD_NOW | RTLD_LOCAL);
    if (!h && !(named && *named)) {  // the toolkit moved: any libnvrtc.so.12
      a.path = "libnvrtc.so.12";
      h = dlopen(a.path.c_str(), RTLD_NOW | RTLD_LOCAL);
    }
    if (!h) {
      const char* e = dlerror();
      a.err = "cannot load NVRTC (" + a.path + "): " + (e ? e : "?");
      return;
    }
    auto sym = [&](const char* n) { return dlsym(h, n); };
    a.version = (decltype(a.version))sym("nvrtcVersion");
    a.create = (decltype(a.create))sym("nvrtcCreateProgram");
    a.compile = (decltype(a.compile))sym("nvrtcCompileProgram");
    a.log_size = (decltype(a.log_size))sym("nvrtcGetProgramLogSize");
    a.log = (decltype(a.log))sym("nvrtcGetProgramLog");
    a.cubin_size = (decltype(a.cubin_size))sym("nvrtcGetCUBINSize");
    a.cubin = (decltype(a.cubin))sym("nvrtcGetCUBIN");
    a.destroy = (decltype(a.destroy))sym("nvrtcDestroyProgram");
    a.error_string = (decltype(a.error_string))sym("nvrtcGetErrorString");
    a.ok = a.version && a.create && a.compile && a.log_size && a.log && a.cubin_size && a.cubin && a.destroy &&
           a.error_string;
    if (!a.ok) a.err = "NVRTC at " + a.path + " lacks an entry point";
  });
  if (!a.ok) fail(NT_E_NVRTC, a.err);
  return a;
}

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
  if (r != NVRTC_SUCCESS) fail(NT_E_NVRTC, std::string(what) + ": " + api().error_string(r));
}

}  // namespace

void nvrtc_version(int* major, int* minor) {
  check(api().version(major, minor), "nvrtcVersion");
}

std::string nvrtc_path() { return api().path; }

std::vector<char> nvrtc_compile(const std::string& source, const std::string& arch, bool use_disk_cache,
                                double* seconds, bool fmad, int max_regs) {
  const NvrtcApi& nv = api();
  int major = 0, minor = 0;
  check(nv.version(&major, &minor), "nvrtcVersion");
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
  check(nv.create(&prog, source.c_str(), "nt_replay.cu", 3, hdr_src, hdr_name), "nvrtcCreateProgram");
  std::vector<const char*> copts;
  for (auto& o : opts) copts.push_back(o.c_str());
  nvrtcResult rc = nv.compile(prog, (int)copts.size(), copts.data());
  if (rc != NVRTC_SUCCESS) {
    size_t log_size = 0;
    nv.log_size(prog, &log_size);
    std::string log(log_size, '\0');
    if (log_size) nv.log(prog, &log[0]);
    nv.destroy(&prog);
    if (log.size() > 4000) log = log.substr(0, 4000) + "...";
    fail(NT_E_NVRTC, "NVRTC compile failed: " + log);
  }
  size_t n = 0;
  check(nv.cubin_size(prog, &n), "nvrtcGetCUBINSize");
  std::vector<char> bin(n);
  check(nv.cubin(prog, bin.data()), "nvrtcGetCUBIN");
  nv.destroy(&prog);
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
