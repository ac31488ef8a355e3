// math_probes.cu -- per-call instruction and flop counts of the replay's
// fp64 routines, for ncu.  Test support, not part of libnabla_b200.
//
// One launch per routine (148 SMs x 4 blocks x 256 threads, each thread
// evaluating it `iters` times on inputs derived from a cheap counter hash,
// results folded into a checksum so nothing is removed).  ncu's
// smsp__inst_executed and dfma/dadd/dmul counters on these launches, minus the
// `which = 0` empty loop, give the per-call counts behind the frozen flop
// weights of nablatensor_b200/csrc/nt_flops.cpp.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3 \
//        -I nablatensor_b200/csrc -o math_probes tests/probes/math_probes.cu
//   ./math_probes [iters]
#include <cstdio>
#include <cstdlib>

#include "nt_device_rt.cuh"

namespace {

__device__ __forceinline__ unsigned probe_word(unsigned x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  return x;
}

__global__ void __launch_bounds__(256) math_probe_kernel(int which, int iters, double* out) {
  nt_math_tables_load();
  const unsigned tid = blockIdx.x * blockDim.x + threadIdx.x;
  double acc = 0.0, acc2 = 0.0;
  unsigned bits = 0;
  for (int i = 0; i < iters; ++i) {
    const unsigned w = probe_word(tid * 2654435761u + (unsigned)i);
    const double u = ((double)w + 0.5) * NT_UINT_SCALE;
    double s = 0.0, c = 0.0;
    switch (which) {
      case 0: acc += u; break;                                        // loop + input only
      case 1: acc += exp((u - 0.5) * 0.25); break;                    // library exp, GBM range
      case 2: acc += log(u); break;                                   // library log
      case 3: sincos(NT_TWO_PI * u, &s, &c); acc += s; acc2 += c; break;  // library sincos
      case 4: acc += sqrt(u * 46.0); break;                           // library sqrt
      case 5: acc += nt_exp_cw((u - 0.5) * 0.25); break;              // full-range exp
      case 6: acc += nt_neg2log_u1(w); break;                         // dedicated -2 ln u1
      case 7: nt_sincos_2pi_u2(w, &s, &c); acc += s; acc2 += c; break;  // dedicated sincos
      case 8: acc += exp((u - 0.5) * 8.0); break;                     // library exp, wide range
      case 9: acc += nt_neg2log_u1_t(w); break;                       // table-driven -2 ln u1
      case 10: nt_sincos_2pi_u2_t(w, &s, &c); acc += s; acc2 += c; break;  // table-driven sincos
      case 11: acc += nt_sqrt_pos(u * 46.0); break;                   // the replay's radius sqrt
      case 12: acc += nt_exp_small((u - 0.5) * 0.25); break;          // series exp, |x| <= 1/8
      case 13: {                                                       // one Philox block
        nt_u32 a, b;
        nt_philox(w, (unsigned)i, &a, &b);
        bits ^= a ^ b;
        break;
      }
      default: break;
    }
  }
  out[tid] = acc + acc2 + (double)bits;
}

}  // namespace

int main(int argc, char** argv) {
  const int iters = argc > 1 ? std::atoi(argv[1]) : 64;
  const char* names[] = {"loop", "exp(lib, |x|<=1/8)", "log(lib)", "sincos(lib)", "sqrt(lib)", "exp(full range)",
                         "-2ln(u1)(series)", "sincos(2pi u2)(series)", "exp(lib, |x|<=4)", "-2ln(u1)(table)",
                         "sincos(2pi u2)(table)", "sqrt(replay radius)", "exp(series, |x|<=1/8)",
                         "philox2x32-10 block"};
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, 0) != cudaSuccess) {
    std::fprintf(stderr, "no CUDA device\n");
    return 1;
  }
  const int blocks = prop.multiProcessorCount * 4;
  double* out = nullptr;
  if (cudaMalloc(&out, (size_t)blocks * 256 * sizeof(double)) != cudaSuccess) return 1;
  for (int which = 0; which < 14; ++which) {
    math_probe_kernel<<<blocks, 256>>>(which, iters, out);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    double first = 0.0;
    if (e == cudaSuccess) e = cudaMemcpy(&first, out, sizeof(double), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
      std::fprintf(stderr, "probe %d: %s\n", which, cudaGetErrorString(e));
      return 1;
    }
    std::printf("probe %d: %s (checksum %.17g)\n", which, names[which], first);
  }
  cudaFree(out);
  return 0;
}
