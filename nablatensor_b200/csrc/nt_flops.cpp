// nt_flops.cpp -- the frozen flop convention for roofline accounting.
//
// Algorithmic flops per scenario are counted from the tape: +, -, *, /, neg,
// max/min/abs = 1; each adjoint contribution d += dy*v = 2 (nt_plan.cpp).
// A transcendental counts the fp64 flops (DFMA = 2, DADD = DMUL = 1) that the
// CUDA library routine executes per call, measured once with ncu's
// smsp__sass_thread_inst_executed_op_d{fma,add,mul}_pred_on counters on the
// isolated probe kernels of the standalone program tests/probes/math_probes.cu
// (summary in profiles/fp64_math_probes_ncu.md), less the probe's own input
// arithmetic.
// The replay kernels call dedicated routines for the Box-Muller and small-
// argument exp, which execute fewer instructions; the weights stay those of
// the library routines, so a faster routine raises the reported fraction of
// peak only through time.
#include "nt_internal.hpp"

namespace nt {

// {exp, log, sqrt, sincos}
const double kFlopWeights[4] = {29.0, 44.0, 13.0, 36.0};

}  // namespace nt
