// nt_kat.cu -- known-answer access to the device generator (tests only).
//
// Exposes the raw Philox2x32-10 words and fp64 Box-Muller legs that every
// replay kernel draws, so the tests can compare them with the oracle's
// restatement of Philox.java bit for bit.
#include <vector>
#include "nt_device_rt.cuh"
#include "nt_exec.hpp"

namespace {

__global__ void kat_kernel(nt_u64 path0, unsigned n_paths, nt_u64 seed, int stream, unsigned pair0,
                           unsigned n_pairs, unsigned* out, double* normals) {
  nt_math_tables_load();  // every thread, before the bounds check
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

// ---- the dedicated routines over given inputs (accuracy tests) -----------------

namespace {

__global__ void math_eval_kernel(int which, long long n, const unsigned* words, const double* x, double* out0,
                                 double* out1) {
  nt_math_tables_load();  // every thread, before the bounds check
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  switch (which) {
    case 0: out0[i] = nt_neg2log_u1_t(words[i]); break;
    case 1: nt_sincos_2pi_u2_t(words[i], &out0[i], &out1[i]); break;
    case 2: out0[i] = nt_sqrt_pos(x[i]); break;
    case 3: out0[i] = nt_exp_small(x[i]); break;
    case 4: out0[i] = nt_exp_cw(x[i]); break;
    case 5: nt_bm64_words(words[2 * i], words[2 * i + 1], &out0[i], &out1[i]); break;
    case 7: {
      bool wide = false;
      out0[i] = nt_exp_cw_fast_flag(x[i], wide);
      out1[i] = wide ? 1.0 : 0.0;
      break;
    }
    case 6: {
      float c, sn;
      nt_bm64f_words(words[2 * i], words[2 * i + 1], &c, &sn);
      out0[i] = c;
      out1[i] = sn;
      break;
    }
    default: break;
  }
}

}  // namespace

namespace nt {

void math_eval(int32_t device, int32_t which, int64_t n, const uint32_t* words, const double* x, double* out0,
               double* out1) {
  if (which < 0 || which > 7) fail(NT_E_INVALID_ARG, "which must be in [0, 7]");
  if (n < 1 || n > (1ll << 24)) fail(NT_E_INVALID_ARG, "n must be in [1, 2^24]");
  const bool use_words = which == 0 || which == 1 || which == 5 || which == 6;
  const bool two_out = which == 1 || which >= 5;
  const int64_t n_words = which == 5 || which == 6 ? 2 * n : n;
  if (!out0 || (two_out && !out1) || (use_words && !words) || (!use_words && !x))
    fail(NT_E_INVALID_ARG, "a required array is null");
  cuda_check(cudaSetDevice(device), "cudaSetDevice");
  unsigned* d_w = nullptr;
  double *d_x = nullptr, *d_o0 = nullptr, *d_o1 = nullptr;
  cudaStream_t s = nullptr;
  cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
  try {
    if (use_words) {
      cuda_check(cudaMalloc(&d_w, n_words * sizeof(unsigned)), "cudaMalloc");
      cuda_check(cudaMemcpyAsync(d_w, words, n_words * sizeof(unsigned), cudaMemcpyHostToDevice, s), "copy in");
    } else {
      cuda_check(cudaMalloc(&d_x, n * sizeof(double)), "cudaMalloc");
      cuda_check(cudaMemcpyAsync(d_x, x, n * sizeof(double), cudaMemcpyHostToDevice, s), "copy in");
    }
    cuda_check(cudaMalloc(&d_o0, n * sizeof(double)), "cudaMalloc");
    if (two_out) cuda_check(cudaMalloc(&d_o1, n * sizeof(double)), "cudaMalloc");
    const unsigned threads = 256;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads);
    math_eval_kernel<<<blocks, threads, 0, s>>>(which, n, d_w, d_x, d_o0, d_o1);
    cuda_check(cudaGetLastError(), "math_eval_kernel launch");
    cuda_check(cudaMemcpyAsync(out0, d_o0, n * sizeof(double), cudaMemcpyDeviceToHost, s), "copy out");
    if (two_out) cuda_check(cudaMemcpyAsync(out1, d_o1, n * sizeof(double), cudaMemcpyDeviceToHost, s), "copy out");
    cuda_check(cudaStreamSynchronize(s), "math_eval_kernel");
  } catch (...) {
    cudaFree(d_w);
    cudaFree(d_x);
    cudaFree(d_o0);
    cudaFree(d_o1);
    cudaStreamDestroy(s);
    throw;
  }
  cudaFree(d_w);
  cudaFree(d_x);
  cudaFree(d_o0);
  cudaFree(d_o1);
  cudaStreamDestroy(s);
}

}  // namespace nt

// ---- fp64 / fp32 vector-FMA peak ------------------------------------------------
//
// The roofline denominator for the replay kernels: MEASURED_PEAKS.json holds
// HBM and bf16 tensor figures only.  Each thread runs `chains` independent
// FMA chains (enough to cover the pipe latency) for `iters` iterations; the
// result is stored so nothing is optimised away.

namespace {

template <typename T>
__global__ void __launch_bounds__(256) fma_peak_kernel(T* out, int iters, T a, T b) {
  T x0 = (T)threadIdx.x, x1 = x0 + (T)1, x2 = x0 + (T)2, x3 = x0 + (T)3;
  T x4 = x0 + (T)4, x5 = x0 + (T)5, x6 = x0 + (T)6, x7 = x0 + (T)7;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      x0 = fma(x0, a, b); x1 = fma(x1, a, b); x2 = fma(x2, a, b); x3 = fma(x3, a, b);
      x4 = fma(x4, a, b); x5 = fma(x5, a, b); x6 = fma(x6, a, b); x7 = fma(x7, a, b);
    }
  }
  out[(size_t)blockIdx.x * blockDim.x + threadIdx.x] = x0 + x1 + x2 + x3 + x4 + x5 + x6 + x7;
}

}  // namespace

namespace nt {

double fma_peak_tflops(int32_t device, int32_t fp64, int32_t iters) {
  cuda_check(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  int per_sm = 0;
  if (fp64)
    cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fma_peak_kernel<double>, 256, 0), "occupancy");
  else
    cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fma_peak_kernel<float>, 256, 0), "occupancy");
  const int blocks = prop.multiProcessorCount * per_sm;
  void* out = nullptr;
  cudaStream_t s = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda_check(cudaMalloc(&out, (size_t)blocks * 256 * 8), "cudaMalloc");
  cuda_check(cudaEventCreate(&e0), "cudaEventCreate");
  cuda_check(cudaEventCreate(&e1), "cudaEventCreate");
  float best_ms = 1e30f;
  for (int rep = 0; rep < 4; ++rep) {
    cuda_check(cudaEventRecord(e0, s), "cudaEventRecord");
    if (fp64) fma_peak_kernel<double><<<blocks, 256, 0, s>>>((double*)out, iters, 0.999999, 1e-7);
    else fma_peak_kernel<float><<<blocks, 256, 0, s>>>((float*)out, iters, 0.999999f, 1e-7f);
    cuda_check(cudaGetLastError(), "fma_peak_kernel");
    cuda_check(cudaEventRecord(e1, s), "cudaEventRecord");
    cuda_check(cudaEventSynchronize(e1), "fma_peak_kernel");
    float ms = 0;
    cuda_check(cudaEventElapsedTime(&ms, e0, e1), "cudaEventElapsedTime");
    if (rep > 0 && ms < best_ms) best_ms = ms;  // first launch is warm-up
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(out);
  cudaStreamDestroy(s);
  const double flops = 2.0 * 8 * 16 * (double)iters * blocks * 256;
  return flops / (best_ms * 1e-3) / 1e12;
}

double fma_peak_sustained_tflops(int32_t device, int32_t fp64, int32_t millis) {
  cuda_check(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  int per_sm = 0;
  if (fp64)
    cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fma_peak_kernel<double>, 256, 0), "occupancy");
  else
    cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fma_peak_kernel<float>, 256, 0), "occupancy");
  const int blocks = prop.multiProcessorCount * per_sm;
  const int iters = 4096;  // about 10 ms per launch
  void* out = nullptr;
  cudaStream_t s = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda_check(cudaMalloc(&out, (size_t)blocks * 256 * 8), "cudaMalloc");
  cuda_check(cudaEventCreate(&e0), "cudaEventCreate");
  cuda_check(cudaEventCreate(&e1), "cudaEventCreate");
  // Launch back to back for `millis`; the rate is taken over the second half,
  // once the clocks have settled under the board's power limit.
  std::vector<float> ms_list;
  double elapsed = 0.0;
  while (elapsed < millis) {
    cuda_check(cudaEventRecord(e0, s), "cudaEventRecord");
    for (int k = 0; k < 8; ++k) {
      if (fp64) fma_peak_kernel<double><<<blocks, 256, 0, s>>>((double*)out, iters, 0.999999, 1e-7);
      else fma_peak_kernel<float><<<blocks, 256, 0, s>>>((float*)out, iters, 0.999999f, 1e-7f);
    }
    cuda_check(cudaGetLastError(), "fma_peak_kernel");
    cuda_check(cudaEventRecord(e1, s), "cudaEventRecord");
    cuda_check(cudaEventSynchronize(e1), "fma_peak_kernel");
    float ms = 0;
    cuda_check(cudaEventElapsedTime(&ms, e0, e1), "cudaEventElapsedTime");
    ms_list.push_back(ms);
    elapsed += ms;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(out);
  cudaStreamDestroy(s);
  double tail_ms = 0.0;
  size_t n = 0;
  for (size_t i = ms_list.size() / 2; i < ms_list.size(); ++i, ++n) tail_ms += ms_list[i];
  const double flops = 2.0 * 8 * 16 * (double)iters * blocks * 256 * 8 * (double)n;
  return flops / (tail_ms * 1e-3) / 1e12;
}

}  // namespace nt
