// nt_plan.cpp -- step-loop detection and the step-wise checkpoint plan.
//
// A Monte-Carlo tape is a prologue (inputs, set-up), a body recorded once per
// time step, and an epilogue (payoff, discount).  Emitting the body once as a
// rolled loop keeps the kernel small (instruction-cache resident) and lets the
// reverse sweep work step-wise: the forward loop saves the loop-carried values
// every G units, and the reverse sweep, segment by segment from the last,
// restores them, recomputes the segment's units into registers and walks them
// backwards.  The reference reached long tapes with node-count segments
// (nablatensor-core/.../AadCheckpointPlan.java:95-172) and the cpu-jit engine
// with a rolled loop (nablatensor-engine-cpu/.../jit/KernelGenerator.java:536-708);
// this plan is loop-aware from the start.
//
// Detection: a unit of L nodes starting at B repeats N times when, for every
// offset j, node B+uL+j has the same op (and constant, stream) in every unit
// and each argument is either the same offset in the same unit, an offset in
// the previous unit (a carry; unit 0 reads a prologue node instead, the carry's
// initial value), or one fixed node before B (an invariant).  Nodes after the
// loop may read only the last unit.
#include <algorithm>
#include <cstring>
#include <map>

#include "nt_internal.hpp"

namespace nt {

namespace {

bool same_double(double x, double y) { return std::memcmp(&x, &y, sizeof x) == 0; }

int nargs(int op) { return is_binary(op) ? 2 : (is_unary(op) ? 1 : 0); }

int32_t arg(const Tape& t, int32_t i, int w) { return w == 0 ? t.a[i] : t.b[i]; }

// Strict shift compatibility of node i with node i+L.
bool compat(const Tape& t, int32_t i, int32_t L) {
  const int32_t j = i + L;
  const int op = t.op[i];
  if (t.op[j] != op) return false;
  if (op == NT_INPUT) return false;
  if (op == NT_CONST) return true;  // a constant may change from unit to unit (per-unit table)
  if (is_draw(op)) return t.b[i] == t.b[j] && t.a[j] > t.a[i];
  for (int w = 0; w < nargs(op); ++w) {
    const int32_t x = arg(t, i, w), y = arg(t, j, w);
    // shifted with the unit, the same node, or two nodes before the unit
    // (a per-unit gathered value; validate() checks they precede the loop)
    if (y != x + L && y != x && !(x < i - L && y < i)) return false;
  }
  return true;
}

struct Candidate {
  int32_t B = -1, L = 0, N = 0, carries = 0;
};

// Full check of (B, L): returns the number of units N >= 2 that repeat, with
// outside readers restricted to the last unit, or 0.
int32_t validate(const Tape& t, int32_t B, int32_t L, int32_t* ncarries) {
  if (B < 0 || L <= 0 || (int64_t)B + 2 * (int64_t)L > t.n) return 0;
  std::vector<Ref> ra(L), rb(L);
  std::vector<int32_t> init(L, -1), stride(L, 0);
  // Classify from unit 1 (the template).
  for (int32_t j = 0; j < L; ++j) {
    const int32_t i1 = B + L + j, i0 = B + j;
    const int op = t.op[i1];
    if (t.op[i0] != op || op == NT_INPUT) return 0;
    if (is_draw(op)) {
      if (t.b[i0] != t.b[i1]) return 0;
      stride[j] = t.a[i1] - t.a[i0];
      if (stride[j] <= 0) return 0;
    }
    for (int w = 0; w < nargs(op); ++w) {
      const int32_t x1 = arg(t, i1, w), x0 = arg(t, i0, w);
      Ref r;
      if (x1 >= B + L) {
        r = {REF_SAME, x1 - (B + L)};
        if (x0 != B + r.idx) return 0;
      } else if (x1 >= B) {
        r = {REF_CARRY, x1 - B};
        if (x0 >= B) return 0;
        if (init[r.idx] < 0) init[r.idx] = x0;
        else if (init[r.idx] != x0) return 0;
      } else {
        // before the loop: one invariant node, or a different node per unit
        r = {x0 == x1 ? REF_OUT : REF_GATHER, x1};
      }
      (w == 0 ? ra : rb)[j] = r;
    }
  }
  // Extend over units 2, 3, ...
  int32_t N = 2;
  for (;; ++N) {
    const int64_t base = (int64_t)B + (int64_t)N * L;
    if (base + L > t.n) break;
    bool ok = true;
    for (int32_t j = 0; j < L && ok; ++j) {
      const int32_t i = (int32_t)base + j, i0 = B + j;
      const int op = t.op[i];
      if (op != t.op[i0]) { ok = false; break; }
      if (op == NT_CONST) continue;
      if (is_draw(op)) {
        ok = t.b[i] == t.b[i0] && (int64_t)t.a[i] == (int64_t)t.a[i0] + (int64_t)N * stride[j];
        continue;
      }
      for (int w = 0; w < nargs(op) && ok; ++w) {
        const Ref& r = w == 0 ? ra[j] : rb[j];
        const int32_t x = arg(t, i, w);
        if (r.kind == REF_SAME) ok = x == (int32_t)base + r.idx;
        else if (r.kind == REF_CARRY) ok = x == (int32_t)(base - L) + r.idx;
        else if (r.kind == REF_GATHER) ok = x < B;
        else ok = x == r.idx;
      }
    }
    if (!ok) break;
  }
  // Readers after the loop (and outputs) may only see the last unit.
  for (bool changed = true; changed && N >= 2;) {
    changed = false;
    const int32_t end = B + N * L;
    auto check = [&](int32_t x) {
      if (x >= B && x < end) {
        const int32_t u = (x - B) / L;
        if (u < N - 1) { N = u + 1; changed = true; }
      }
    };
    for (int32_t i = end; i < t.n && !changed; ++i) {
      const int op = t.op[i];
      for (int w = 0; w < nargs(op); ++w) check(arg(t, i, w));
    }
    for (int32_t o = 0; o < t.n_out() && !changed; ++o) check(t.output_node[o]);
  }
  if (N < 2) return 0;
  if (ncarries) {
    int32_t c = 0;
    for (int32_t j = 0; j < L; ++j) c += init[j] >= 0;
    *ncarries = c;
  }
  return N;
}

std::vector<int32_t> candidate_periods(const Tape& t) {
  std::vector<int32_t> draws;
  for (int32_t i = 0; i < t.n; ++i)
    if (is_draw(t.op[i])) draws.push_back(i);
  std::vector<int32_t> out;
  const int32_t nd = (int32_t)draws.size();
  for (int32_t r = 1; r <= 32 && 4 * r <= nd; ++r) {
    std::map<int32_t, int32_t> hist;
    const int32_t lo = nd / 4, hi = std::min(nd - r, lo + 512);
    for (int32_t k = lo; k < hi; ++k) hist[draws[k + r] - draws[k]]++;
    int32_t best = 0, bestc = 0;
    for (auto& kv : hist)
      if (kv.second > bestc) { best = kv.first; bestc = kv.second; }
    if (best > 0 && 2 * bestc >= (hi - lo)) out.push_back(best);
  }
  for (int32_t L = 1; L <= 64 && 4 * L <= t.n; ++L) out.push_back(L);
  std::sort(out.begin(), out.end());
  out.erase(std::unique(out.begin(), out.end()), out.end());
  return out;
}

Candidate find_loop(const Tape& t) {
  Candidate best;
  std::vector<int32_t> found;  // periods that gave a loop
  for (int32_t L : candidate_periods(t)) {
    if (3 * (int64_t)L > t.n) continue;
    // A multiple of a period that already gave a loop only folds its units.
    bool multiple = false;
    for (int32_t f : found) multiple |= L % f == 0;
    if (multiple) continue;
    // Longest strict run of compat(i, L).
    int32_t run_s = -1, run_len = 0, cur_s = -1, cur_len = 0;
    for (int32_t i = 0; i + L < t.n; ++i) {
      if (compat(t, i, L)) {
        if (cur_len == 0) cur_s = i;
        ++cur_len;
        if (cur_len > run_len) { run_len = cur_len; run_s = cur_s; }
      } else {
        cur_len = 0;
      }
    }
    if (run_len < 2 * L) continue;
    // Every rotation of a periodic body validates, each at a cost of the whole
    // loop: a long unit is tried only at the starts that are draws (and the
    // run's own start), a short one at every start.
    const bool long_unit = L > 64;
    bool any = false;
    for (int32_t B = std::max(0, run_s - 2 * L); B <= run_s; ++B) {
      if (long_unit && B != run_s && !is_draw(t.op[B])) continue;
      int32_t carries = 0;
      const int32_t N = validate(t, B, L, &carries);
      if (N < 3) continue;
      any = true;
      const int64_t cover = (int64_t)N * L, bcover = (int64_t)best.N * best.L;
      if (cover > bcover || (cover == bcover && carries < best.carries)) best = {B, L, N, carries};
    }
    if (any) found.push_back(L);
  }
  return best;
}

// Fills the unit description for a validated (B, L, N).
void describe(const Tape& t, Loop& lp) {
  const int32_t B = lp.B, L = lp.L, N = lp.N;
  lp.body.assign(L, BodyNode{});
  lp.gather.clear();
  lp.is_carry.assign(L, 0);
  lp.carry_slot.assign(L, -1);
  lp.is_exit.assign(L, 0);
  std::vector<int32_t> init(L, -1);
  for (int32_t j = 0; j < L; ++j) {
    const int32_t i1 = B + L + j, i0 = B + j;
    BodyNode& bn = lp.body[j];
    bn.op = t.op[i1];
    bn.c = t.c[i1];
    if (is_draw(bn.op)) {
      bn.stream = t.b[i1];
      bn.draw_base = t.a[i0];
      bn.draw_stride = t.a[i1] - t.a[i0];
    }
    for (int w = 0; w < nargs(bn.op); ++w) {
      const int32_t x1 = arg(t, i1, w), x0 = arg(t, i0, w);
      Ref r;
      if (x1 >= B + L) r = {REF_SAME, x1 - (B + L)};
      else if (x1 >= B) { r = {REF_CARRY, x1 - B}; init[r.idx] = x0; lp.is_carry[r.idx] = 1; }
      else if (x0 == x1) r = {REF_OUT, x1};
      else {
        // A different node before the loop in each unit.  Arguments that read
        // the same node in every unit share one slot, so that node's adjoint
        // collects its unit's contributions in one place, in the reverse
        // sweep's order.
        std::vector<int32_t> nodes(N);
        for (int32_t u = 0; u < N; ++u) nodes[u] = arg(t, B + u * L + j, w);
        int32_t slot = -1;
        for (size_t k = 0; k < lp.gather.size() && slot < 0; ++k)
          if (lp.gather[k] == nodes) slot = (int32_t)k;
        if (slot < 0) {
          slot = (int32_t)lp.gather.size();
          lp.gather.push_back(std::move(nodes));
        }
        r = {REF_GATHER, slot};
      }
      (w == 0 ? bn.ra : bn.rb) = r;
    }
    uint8_t act = 0;
    for (int32_t u = 0; u < N && !act; ++u) act |= t.active[B + u * L + j];
    bn.active = act != 0;
  }
  lp.carries.clear();
  lp.carry_init.clear();
  for (int32_t k = 0; k < L; ++k)
    if (lp.is_carry[k]) {
      lp.carry_slot[k] = (int32_t)lp.carries.size();
      lp.carries.push_back(k);
      lp.carry_init.push_back(init[k]);
    }
  // Constants that differ between units go to the per-unit table.
  lp.n_vary = 0;
  for (int32_t j = 0; j < L; ++j) {
    BodyNode& bn = lp.body[j];
    if (bn.op != NT_CONST) continue;
    bool same = true;
    for (int32_t u = 1; u < N && same; ++u) same = same_double(t.c[B + u * L + j], t.c[B + j]);
    bn.c = t.c[B + j];
    if (!same) bn.cslot = lp.n_vary++;
  }
  lp.ctab.assign((size_t)N * lp.n_vary, 0.0);
  for (int32_t j = 0; j < L; ++j)
    if (lp.body[j].cslot >= 0)
      for (int32_t u = 0; u < N; ++u) lp.ctab[(size_t)u * lp.n_vary + lp.body[j].cslot] = t.c[B + u * L + j];
  const int32_t end = B + N * L;
  auto mark = [&](int32_t x) {
    if (x >= B && x < end) lp.is_exit[(x - B) % L] = 1;
  };
  for (int32_t i = end; i < t.n; ++i)
    for (int w = 0; w < nargs(t.op[i]); ++w) mark(arg(t, i, w));
  for (int32_t o = 0; o < t.n_out(); ++o) mark(t.output_node[o]);
  lp.exits.clear();
  for (int32_t k = 0; k < L; ++k)
    if (lp.is_exit[k]) lp.exits.push_back(k);
}

// Values the reverse sweep of a unit reads (ScalarReplay.java:129-171 rules,
// restricted to contributions into active arguments as the device sweep does).
void reverse_reads(const Loop& lp, int32_t j, std::vector<Ref>& out) {
  const BodyNode& bn = lp.body[j];
  out.clear();
  if (!bn.active) return;
  auto act = [&](const Ref& r) {
    if (r.kind == REF_SAME || r.kind == REF_CARRY) return lp.body[r.idx].active;
    return true;  // outside node: activity decided by the tape; reading its value is harmless
  };
  const Ref self{REF_SAME, j};
  switch (bn.op) {
    case NT_MUL:
      if (act(bn.ra)) out.push_back(bn.rb);
      if (act(bn.rb)) out.push_back(bn.ra);
      break;
    case NT_DIV:
      out.push_back(bn.rb);
      if (act(bn.rb)) out.push_back(self);
      break;
    case NT_EXP: case NT_SQRT: out.push_back(self); break;
    case NT_LOG: case NT_ABS: out.push_back(bn.ra); break;
    case NT_MAX: case NT_MIN: out.push_back(bn.ra); out.push_back(bn.rb); break;
    default: break;
  }
}

// Algorithmic flop weights per op, frozen: an arithmetic op is 1 flop, an
// adjoint contribution d += dy*v is 2.  Transcendentals count the fp64 flops
// of the library routine measured once on the device (FMA = 2, nt_flops.cpp).
struct Weights {
  double add = 1, mul = 1, div = 1, neg = 1, minmax = 1, abs = 1;
  double exp = 0, log = 0, sqrt = 0, sincos = 0;  // filled from kFlopWeights
};

}  // namespace

EmitConfig config_from(const nt_options* opt, int32_t target) {
  if (!opt) fail(NT_E_INVALID_ARG, "options are null");
  if (opt->precision != NT_FLOAT32 && opt->precision != NT_FLOAT64) fail(NT_E_INVALID_ARG, "bad precision");
  if (target < 0 || target > 3)
    fail(NT_E_INVALID_ARG, "target must be 0 (CUDA), 1 (host), 2 (CUDA multi-market) or 3 (host multi-market)");
  EmitConfig cfg;
  cfg.markets = target >= 2;
  target &= 1;
  cfg.f32 = opt->precision == NT_FLOAT32;
  cfg.adjoints = opt->adjoints != 0;
  cfg.no_loop = (opt->flags & NT_FLAG_NO_LOOP) != 0;
  cfg.global_ckpt = (opt->flags & NT_FLAG_SHARED_CKPT) == 0;
  cfg.wide32 = cfg.f32 && (opt->flags & NT_FLAG_F32_FAST) == 0;
  // Under the reference's fp32 semantics every node is rounded to float on its
  // own, so a multiply-add is not contracted there (it costs the barrier tape
  // 1.6 % and brings its sums to the fp32 oracle's within 2e-9, where a fused
  // kernel sits up to 8e-6 away, by however the compiler chose to fuse).
  cfg.fmad = (opt->flags & NT_FLAG_NO_FMAD) == 0 && !cfg.wide32;
  cfg.block = opt->block > 0 ? opt->block : 128;
  if (cfg.block % 32 != 0 || cfg.block > 1024) fail(NT_E_INVALID_ARG, "block must be a multiple of 32, <= 1024");
  if (opt->min_blocks < 0 || opt->min_blocks > 32) fail(NT_E_INVALID_ARG, "min_blocks must be in [0, 32]");
  if (opt->seg_units < 0) fail(NT_E_INVALID_ARG, "seg_units must be >= 0");
  if (opt->max_regs != 0 && (opt->max_regs < 32 || opt->max_regs > 255))
    fail(NT_E_INVALID_ARG, "max_regs must be 0 or in [32, 255]");
  cfg.min_blocks = opt->min_blocks;
  cfg.max_regs = opt->max_regs;
  if (cfg.max_regs > 0 && cfg.min_blocks > 0) fail(NT_E_INVALID_ARG, "max_regs and min_blocks are exclusive");
  cfg.seg_units = opt->seg_units;
  cfg.target = target;
  if (opt->fwd_unroll < 0 || opt->fwd_unroll > 16) fail(NT_E_INVALID_ARG, "fwd_unroll must be in [0, 16]");
  cfg.fwd_unroll = opt->fwd_unroll;
  if (opt->rev_unroll < 0 || opt->rev_unroll > 8) fail(NT_E_INVALID_ARG, "rev_unroll must be in [0, 8]");
  cfg.rev_unroll = std::max(1, opt->rev_unroll);
  cfg.tape = (opt->flags & NT_FLAG_RECOMPUTE_ALL) == 0;
  cfg.tape_all = (opt->flags & NT_FLAG_TAPE_DRAWS) == 0;
  cfg.tape_every_exp = (opt->flags & NT_FLAG_TAPE_ALL) != 0;
  if (!cfg.tape_all && cfg.tape_every_exp) fail(NT_E_INVALID_ARG, "NT_FLAG_TAPE_DRAWS and NT_FLAG_TAPE_ALL conflict");
  if (opt->grid_blocks_per_sm < 0) fail(NT_E_INVALID_ARG, "grid_blocks_per_sm must be >= 0");
  cfg.grid_blocks_per_sm = opt->grid_blocks_per_sm;
  return cfg;
}

int32_t auto_block(const Plan& p) {
  if (!p.loop.present) return 128;
  return p.per_unit_regs <= 32 ? 256 : 64;
}

int32_t ckpt_values(const Plan& p) {
  return p.loop.present ? p.loop.K * (int32_t)p.loop.ckpt.size() : 0;
}

Plan plan_tape(const Tape& t, const EmitConfig& cfg) {
  Plan p;
  Loop& lp = p.loop;
  int32_t per_unit = 0;  // values one unit's reverse sweep reads (register estimate)
  if (!cfg.no_loop) {
    Candidate c = find_loop(t);
    if (c.N >= 3) {
      lp.present = true;
      lp.B = c.B;
      lp.L = c.L;
      lp.N = c.N;
    }
  }
  if (lp.present) {
    // Fold iterations so each unit draws whole Box-Muller pairs: a pair's two
    // legs must land in the same unit and start at an even ordinal.
    describe(t, lp);
    bool odd_stride = false, odd_base = false, single_draws = true;
    std::map<int32_t, int32_t> per_stream;
    for (const BodyNode& bn : lp.body)
      if (bn.op == NT_RANDN) {
        odd_stride |= (bn.draw_stride & 1) != 0;
        single_draws &= bn.draw_stride == 1 && ++per_stream[bn.stream] == 1;
      }
    // A long unit keeps its recorded length and carries the second Box-Muller
    // leg from an even unit to the next (fewer values live in a unit's
    // reverse sweep); a short one is folded in pairs.
    const bool half = odd_stride && single_draws && lp.L > 128;
    int32_t U = (odd_stride && !half) ? 2 : 1;
    // Smallest normal ordinal per stream in unit 0.
    std::map<int32_t, int32_t> first;
    for (const BodyNode& bn : lp.body)
      if (bn.op == NT_RANDN) {
        auto it = first.find(bn.stream);
        if (it == first.end() || bn.draw_base < it->second) first[bn.stream] = bn.draw_base;
      }
    for (auto& kv : first) odd_base |= (kv.second & 1) != 0;
    int32_t B = lp.B, L = lp.L, N = lp.N;
    if (odd_base && odd_stride) { B += L; N -= 1; }  // peel one iteration into the prologue
    int32_t units = N / U;
    // Units per checkpoint segment: a divisor of the unit count close to the
    // target; otherwise the remainder units are peeled into the epilogue.  The
    // automatic target keeps one segment's reverse-sweep values within about
    // 64 registers (the values a unit's reverse reads, 2 registers each in fp64).
    if (units >= 2 && validate(t, B, L * U, nullptr) >= 2) {
      Loop probe;
      probe.present = true;
      probe.B = B;
      probe.L = L * U;
      probe.N = units;
      describe(t, probe);
      std::vector<uint8_t> kept(probe.L, 0);
      std::vector<Ref> rd;
      for (int32_t j = 0; j < probe.L; ++j) {
        reverse_reads(probe, j, rd);
        for (const Ref& r : rd)
          if (r.kind == REF_SAME || r.kind == REF_CARRY) kept[r.idx] = 1;
      }
      for (uint8_t k : kept) per_unit += k;
    }
    const int32_t words = cfg.f32 ? 1 : 2;
    // fp64 with a value tape: about 112 registers.  A light unit then runs
    // longer segments (the 252-step Asian: 9 units where 64 registers gave 6;
    // 156 registers, one 256-thread block per SM): the reverse sweep has more
    // independent work per segment, and the tape in flight, half as many
    // threads', stays in L2 -- +2.7 % in a 2^27-scenario launch, +6.6 % over
    // 1e9 scenarios per step under the power limit (7 units, still two
    // blocks per SM, gained 1 %).  fp32 tapes keep 64: the barrier with 6
    // units instead of 3 fell from 5 to 2 resident blocks and ran 5 % slower.
    const int32_t budget = (!cfg.f32 && cfg.tape) ? 112 : 64;
    const int32_t auto_target =
        per_unit > 0 ? std::max(1, std::min(16, budget / (per_unit * words))) : std::max(1, 8 / U);
    const int32_t target = cfg.seg_units > 0 ? cfg.seg_units : auto_target;
    int32_t G = target;
    if (units >= 2) {
      int32_t bestG = -1;
      for (int32_t g = std::max(1, target - target / 3); g <= target + target / 3 + 1; ++g)
        if (units % g == 0 && (bestG < 0 || std::abs(g - target) < std::abs(bestG - target))) bestG = g;
      if (cfg.seg_units > 0) bestG = (units % cfg.seg_units == 0) ? cfg.seg_units : -1;
      if (bestG > 0) G = bestG;
    }
    G = std::max(1, std::min(G, units));
    const int32_t K = units / G;
    if (K < 1 || units < 2) {
      lp = Loop{};
    } else {
      lp.B = B;
      lp.L = L * U;
      lp.N = K * G;
      lp.steps_per_unit = U;
      int32_t nc = 0;
      const int32_t N2 = validate(t, lp.B, lp.L, &nc);
      if (N2 < lp.N) {
        lp = Loop{};
      } else {
        describe(t, lp);
        lp.G = G;
        lp.K = K;
        lp.half_pairs = half;
      }
    }
  }
  if (lp.present) {
    const int32_t L = lp.L;
    // Stored values: everything the reverse of a unit reads from its own unit
    // or (for unit 0 of a segment) from the previous unit's carries.
    lp.stored.assign(L, 0);
    std::vector<uint8_t> carry_read(L, 0);
    std::vector<Ref> reads;
    for (int32_t j = 0; j < L; ++j) {
      reverse_reads(lp, j, reads);
      for (const Ref& r : reads) {
        if (r.kind == REF_SAME) lp.stored[r.idx] = 1;
        else if (r.kind == REF_CARRY) { lp.stored[r.idx] = 1; carry_read[r.idx] = 1; }
      }
    }
    // Recompute closure: nodes needed to regenerate the stored values.  In
    // tape mode an expensive node is a leaf: the forward sweep writes its value
    // to the thread's tape and the reverse sweep reads it back instead of
    // recomputing its inputs.  Expensive are the draws, and (unless only draws
    // are taped) log, sqrt, division, and an exp whose argument depends on a
    // loop carry.  An exp of the unit's draws and loop invariants alone -- a
    // GBM log-return -- is recomputed: its argument is small, the reverse sweep
    // evaluates it by the branch-free series, and that is cheaper than moving
    // 16 bytes per value through HBM.  Not in a unit whose reverse values
    // already fill the register budget on their own (more than 32 registers,
    // one unit per segment, e.g. a 10-asset basket step): there the recompute
    // lengthens a latency-bound sweep, and the tape wins.
    p.per_unit_regs = per_unit * (cfg.f32 ? 1 : 2);
    const bool light_unit = p.per_unit_regs <= 32;
    std::vector<uint8_t> carry_dep(L, 0);
    for (int32_t j = 0; j < L; ++j) {
      const BodyNode& bn = lp.body[j];
      for (int w = 0; w < nargs(bn.op); ++w) {
        const Ref& r = w == 0 ? bn.ra : bn.rb;
        if (r.kind == REF_CARRY || (r.kind == REF_SAME && carry_dep[r.idx])) carry_dep[j] = 1;
      }
    }
    auto expensive = [&](int32_t j) {
      const int op = lp.body[j].op;
      if (op == NT_RANDN || op == NT_RANDU) return true;
      if (!cfg.tape_all) return false;
      if (op == NT_LOG || op == NT_SQRT || op == NT_DIV) return true;
      return op == NT_EXP && (carry_dep[j] != 0 || cfg.tape_every_exp || !light_unit);
    };
    std::vector<uint8_t> need(lp.stored);
    lp.tape_slot.assign(L, -1);
    for (bool changed = true; changed;) {
      changed = false;
      for (int32_t j = L - 1; j >= 0; --j) {
        if (!need[j]) continue;
        const BodyNode& bn = lp.body[j];
        if (cfg.tape && expensive(j)) continue;  // a tape leaf
        for (int w = 0; w < nargs(bn.op); ++w) {
          const Ref& r = w == 0 ? bn.ra : bn.rb;
          if ((r.kind == REF_SAME || r.kind == REF_CARRY) && !need[r.idx]) { need[r.idx] = 1; changed = true; }
          if (r.kind == REF_CARRY) carry_read[r.idx] = 1;
        }
      }
    }
    lp.recompute = need;
    lp.n_tape = 0;
    if (cfg.tape)
      for (int32_t j = 0; j < L; ++j)
        if (need[j] && expensive(j)) lp.tape_slot[j] = lp.n_tape++;
    lp.ckpt.clear();
    for (int32_t k : lp.carries)
      if (carry_read[k]) lp.ckpt.push_back(k);
    p.stored_per_unit = 0;
    for (int32_t j = 0; j < L; ++j) p.stored_per_unit += lp.stored[j];
  }

  // Algorithmic flops per scenario (tape ops only; Box-Muller per pair).
  Weights w;
  w.exp = kFlopWeights[0];
  w.log = kFlopWeights[1];
  w.sqrt = kFlopWeights[2];
  w.sincos = kFlopWeights[3];
  double fwd = 0, rev = 0, wide = 0, transc = 0;
  for (int32_t i = 0; i < t.n; ++i) {
    const int op = t.op[i];
    // fp32 under the reference's semantics: exp, log and Box-Muller run in fp64.
    if (cfg.f32 && cfg.wide32) {
      if (op == NT_EXP) wide += w.exp;
      else if (op == NT_LOG) wide += w.log;
      else if (op == NT_RANDN) wide += 0.5 * (w.log + w.sqrt + w.sincos + 8.0);
    }
    switch (op) {
      case NT_ADD: case NT_SUB: fwd += w.add; break;
      case NT_MUL: fwd += w.mul; break;
      case NT_DIV: fwd += w.div; break;
      case NT_NEG: fwd += w.neg; break;
      case NT_MAX: case NT_MIN: fwd += w.minmax; break;
      case NT_ABS: fwd += w.abs; break;
      case NT_EXP: fwd += w.exp; transc += w.exp; break;
      case NT_LOG: fwd += w.log; transc += w.log; break;
      case NT_SQRT: fwd += w.sqrt; transc += w.sqrt; break;
      case NT_RANDN:
        // one Box-Muller pair per two normals: log + sqrt + sincos, plus
        // u1, u2 (2 adds, 2 multiplies), -2 ln u1, the angle, r*cos, r*sin = 8
        fwd += 0.5 * (w.log + w.sqrt + w.sincos + 8.0);
        transc += 0.5 * (w.log + w.sqrt + w.sincos);
        break;
      case NT_RANDU: fwd += 2.0; break;
      default: break;
    }
    if (!cfg.adjoints || !t.active[i]) continue;
    const bool aa = (is_unary(op) || is_binary(op)) && t.active[t.a[i]];
    const bool ab = is_binary(op) && t.active[t.b[i]];
    switch (op) {
      case NT_ADD: case NT_SUB: rev += aa + ab; break;             // d += dy
      case NT_MUL: rev += 2.0 * (aa + ab); break;                  // d += dy*v
      case NT_DIV: rev += 2.0 * aa + 3.0 * ab; break;              // d += dy/vb ; d -= dy*vi/vb
      case NT_NEG: rev += aa; break;
      case NT_EXP: rev += 2.0 * aa; break;
      case NT_LOG: rev += 2.0 * aa; break;
      case NT_SQRT: rev += 3.0 * aa; break;
      case NT_ABS: case NT_MAX: case NT_MIN: rev += aa + ab; break;
      default: break;
    }
  }
  p.fwd_flops = fwd;
  p.wide_flops = wide;
  p.rev_flops = cfg.adjoints ? rev * t.n_out() : 0.0;
  p.arith_flops = fwd - transc + p.rev_flops;
  return p;
}

}  // namespace nt
