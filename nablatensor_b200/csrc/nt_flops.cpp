// nt_flops.cpp -- the frozen flop convention for roofline accounting.
//
// Algorithmic flops per scenario are counted from the tape: +, -, *, /, neg,
// max/min/abs = 1; each adjoint contribution d += dy*v = 2 (see nt_plan.cpp).
// A transcendental counts the fp64 flops its device routine executes
// (DFMA = 2, DADD/DMUL = 1), measured once with ncu's
// smsp__sass_thread_inst_executed_op_d{fma,add,mul}_pred_on counters on an
// isolated loop of that routine alone (profiles/fp64_transcendental_flops.md).
#include "nt_internal.hpp"

namespace nt {

// {exp, log, sqrt, sincos}
const double kFlopWeights[4] = {28.0, 28.0, 10.0, 40.0};

}  // namespace nt
