// nt_kat.cu -- known-answer access to the device generator (tests only).
//
// Exposes the raw Philox2x32-10 words and fp64 Box-Muller legs that every
// replay kernel draws, so the tests can compare them with the oracle's
// restatement of Philox.java bit for bit.
#include "nt_device_rt.cuh"
#include "nt_exec.hpp"

namespace {

__global__ void kat_kernel(nt_u64 path0, unsigned n_paths, nt_u64 seed, int stream, unsigned pair0,
                           unsigned n_pairs, unsigned* out, double* normals) {
  const nt_u64 idx = (nt_u64)blockIdx.x * blockDim.x + threadIdx.x;
  const nt_u64 total = (nt_u64)n_paths * n_pairs;
  if (idx >= total) return;
  const nt_u64 p = idx / n_pairs;
  const unsigned q = (unsigned)(idx % n_pairs);
  const nt_key key = nt_make_key(path0 + p, seed, stream);
  nt_u32 w0, w1;
  nt_normal_words(key, pair0 + q, &w0, &w1);
  out[2 * idx] = w0;
  out[2 * idx + 1] = w1;
  if (normals) {
    double c, s;
    nt_bm64(w0, w1, &c, &s);
    normals[2 * idx] = c;
    normals[2 * idx + 1] = s;
  }
}

}  // namespace

namespace nt {

void philox_words(int32_t device, uint64_t path0, uint32_t n_paths, uint64_t seed, int32_t stream, uint32_t pair0,
                  uint32_t n_pairs, uint32_t* out, double* normals) {
  if (!out) fail(NT_E_INVALID_ARG, "out is null");
  const uint64_t total = (uint64_t)n_paths * n_pairs;
  if (total == 0 || total > (1ull << 26)) fail(NT_E_INVALID_ARG, "n_paths * n_pairs must be in [1, 2^26]");
  cuda_check(cudaSetDevice(device), "cudaSetDevice");
  unsigned* d_out = nullptr;
  double* d_norm = nullptr;
  cudaStream_t s = nullptr;
  cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
  try {
    cuda_check(cudaMalloc(&d_out, total * 2 * sizeof(unsigned)), "cudaMalloc");
    if (normals) cuda_check(cudaMalloc(&d_norm, total * 2 * sizeof(double)), "cudaMalloc");
    const unsigned threads = 256;
    const unsigned blocks = (unsigned)((total + threads - 1) / threads);
    kat_kernel<<<blocks, threads, 0, s>>>(path0, n_paths, seed, stream, pair0, n_pairs, d_out, d_norm);
    cuda_check(cudaGetLastError(), "kat_kernel launch");
    cuda_check(cudaMemcpyAsync(out, d_out, total * 2 * sizeof(unsigned), cudaMemcpyDeviceToHost, s), "copy words");
    if (normals)
      cuda_check(cudaMemcpyAsync(normals, d_norm, total * 2 * sizeof(double), cudaMemcpyDeviceToHost, s), "copy normals");
    cuda_check(cudaStreamSynchronize(s), "kat_kernel");
  } catch (...) {
    cudaFree(d_out);
    cudaFree(d_norm);
    cudaStreamDestroy(s);
    throw;
  }
  cudaFree(d_out);
  cudaFree(d_norm);
  cudaStreamDestroy(s);
}

}  // namespace nt
