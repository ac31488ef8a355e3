// nt_emit.cpp -- tape -> sm_100a CUDA C (or host C++) for one scenario per thread.
//
// Layout of the emitted scenario (one thread, one path at a time):
//   prologue forward   straight-line, values in registers (v<i>)
//   loop forward       rolled over units; every G units the checkpointed
//                      carries go to shared memory (or global scratch)
//   epilogue forward   straight-line; reads the last unit through cv/xv
//   value accumulators
//   per output:
//     epilogue reverse straight-line adjoints d<i>; loop exits cd<k>/xd<j>
//     loop reverse     per segment, last first: restore carries, recompute the
//                      segment's G units into registers (r<g>_<j>), walk the
//                      units backwards; invariant adjoints stay in registers
//     prologue reverse
//     adjoint accumulators
// The adjoint rules and their order follow ScalarReplay.run's reverse switch
// (nablatensor-engine-cpu/.../cpu/ScalarReplay.java:129-171), emitted only for
// contributions into active arguments as the reference device sweep does
// (nablatensor-core/.../CudaAadCodegen.java:386-448).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <set>
#include <sstream>

#include "nt_internal.hpp"

namespace nt {

namespace {

int nargs(int op) { return is_binary(op) ? 2 : (is_unary(op) ? 1 : 0); }

struct Out {
  std::string s;
  int ind = 0;
  void line(const std::string& x) {
    s.append((size_t)ind * 2, ' ');
    s += x;
    s += '\n';
  }
  void open(const std::string& x) { line(x); ++ind; }
  void close(const std::string& x = "}") { --ind; line(x); }
};

std::string lit(double x, bool f32) {
  char buf[64];
  if (std::isfinite(x)) {
    std::snprintf(buf, sizeof buf, "%a", x);
    std::string s(buf);
    if (x < 0) s = "(" + s + ")";
    return f32 ? "((float)" + s + ")" : s;
  }
  uint64_t bits;
  std::memcpy(&bits, &x, sizeof bits);
  std::snprintf(buf, sizeof buf, "nt_from_bits64(0x%016llxULL)", (unsigned long long)bits);
  return f32 ? "((float)" + std::string(buf) + ")" : std::string(buf);
}

class Emitter {
 public:
  Emitter(const Tape& t, const Plan& p, const EmitConfig& cfg)
      : t_(t), p_(p), lp_(p.loop), cfg_(cfg) {}

  std::string run();

 private:
  // The block's exact words live in shared memory while they take at most
  // 8 KB (14 channels of 69 words: the Asian's 7 take 3.9 KB); beyond that
  // the kernel adds its tile sums to the launch's words in global memory, so
  // that many-input tapes with small, register-heavy blocks (the CVA book's
  // 43 channels, 64 threads) keep their resident blocks.
  bool xshared() const { return (int64_t)channels() * kXWords * 8 <= 8 * 1024; }
  const Tape& t_;
  const Plan& p_;
  const Loop& lp_;
  const EmitConfig& cfg_;
  Out o_;
  // Adjoint registers that still hold their initial zero at this point of the
  // emitted straight-line code.  In fp64 the first contribution to one is
  // emitted as an assignment: `0 + x` and `x` differ only in the sign of an
  // exact zero, which no later adjoint rule can observe (adjoints are only
  // scaled and summed, and every accumulator starts at +0).  fp32 keeps the
  // explicit `0 + x`: the product then stays rounded on its own instead of
  // being fused into the next addition, which is what the reference's
  // node-by-node fp32 rounding needs.
  std::set<std::string> zero_;
  // Multi-market kernel, states after the first: loop draws come back from
  // the value tape instead of the generator.
  bool reuse_draws_ = false;
  // Reverse-sweep copy for warps whose forward exps all stayed in the series
  // range: recomputed EXP nodes use the bare series (no per-node branch).
  bool series_exp_ = false;
  // The fp64 exp form fwd_expr emits (NT_EXP64, NT_EXP64W, NT_EXP64F or
  // NT_EXP64_SERIES).
  std::string exp_fn_ = "NT_EXP64(";
  // Forward loop pass that evaluates the recomputed exps by the bare series.
  bool fwd_fast_ = false;
  // Gathered arguments that depend on no draw are the same for every path of
  // a launch: the CUDA kernel evaluates them once per block into shared
  // memory (nt_gvs[k * N + unit]) instead of a per-thread array per scenario.
  bool gv_shared_ = false;
  // A light unit's value tape (the Asian's 2 KB per thread) can stay in L2
  // while in flight, at the occupancy such kernels run: the last reverse sweep
  // then drops each consumed segment's rows from L2 (nt_discard_rows_l2),
  // when the kernel finds at run time that the grid's whole tape fits
  // (nt_tape_in_l2).  Measured on the 252-step Asian over 1e9 scenarios per
  // step: +1.1 to +1.4 %, the same bits.  Heavy units (basket, CVA) move
  // tapes far beyond L2 and do not emit it: on the CVA book the extra code
  // alone cost 5 %.
  bool discard_ = false;
  std::string gv_ref(int32_t k, const std::string& unit) const {
    if (gv_shared_) return "nt_gvs[" + std::to_string(k * lp_.N) + " + " + unit + "]";
    return "nt_gv" + std::to_string(k) + "[" + unit + "]";
  }
  std::string contrib(const std::string& x, char sign, const std::string& e) {
    if (zero_.erase(x) && !cfg_.f32) return x + " = " + (sign == '-' ? "-(" + e + ")" : e) + ";";
    return x + (sign == '-' ? " -= " : " += ") + e + ";";
  }

  std::string R(const char* f64, const char* f32) const { return cfg_.f32 ? f32 : f64; }
  std::string rng_pair() const {
    return cfg_.f32 ? (cfg_.wide32 ? "nt_normal_pair32w(" : "nt_normal_pair32(") : "nt_normal_pair64(";
  }
  std::string rng_single() const {
    return cfg_.f32 ? (cfg_.wide32 ? "nt_normal32w(" : "nt_normal32(") : "nt_normal64(";
  }
  int32_t channels() const { return t_.n_out() * (2 + t_.n_in()); }
  bool in_loop(int32_t x) const { return lp_.in(x); }

  // ---- names of outside nodes and loop exits ----
  std::string val_outside(int32_t x) const {
    if (in_loop(x)) {
      const int32_t j = lp_.off(x);
      return lp_.is_carry[j] ? "cv" + std::to_string(j) : "xv" + std::to_string(j);
    }
    return "v" + std::to_string(x);
  }
  std::string adj_outside(int32_t x) const {
    if (in_loop(x)) {
      const int32_t j = lp_.off(x);
      return lp_.is_carry[j] ? "cd" + std::to_string(j) : "xd" + std::to_string(j);
    }
    return "d" + std::to_string(x);
  }
  bool active_outside(int32_t x) const { return in_loop(x) ? lp_.body[lp_.off(x)].active : t_.active[x] != 0; }
  // A gathered argument is active when any unit's node is.
  bool gather_active(int32_t k) const {
    for (int32_t x : lp_.gather[k])
      if (t_.active[x]) return true;
    return false;
  }

  std::string fwd_expr(int op, const std::string& A, const std::string& B, double c, int32_t a,
                       bool a_one = false) const;
  // The node is the constant 1 (in every unit, for a loop node): a division
  // by it is a reciprocal.
  bool node_is_one(int32_t x) const { return t_.op[x] == NT_CONST && t_.c[x] == 1.0; }
  bool ref_is_one(const Ref& r) const {
    if (r.kind == REF_SAME) {
      const BodyNode& n = lp_.body[r.idx];
      return n.op == NT_CONST && n.cslot < 0 && n.c == 1.0;
    }
    return r.kind == REF_OUT && node_is_one(r.idx);
  }
  void emit_straight_forward(int32_t lo, int32_t hi);
  void emit_straight_reverse(int32_t lo, int32_t hi);
  void emit_rule(int op, const std::string& D, const std::string& Va, const std::string& Vb,
                 const std::string& Vi, const std::string* da, const std::string* db, bool a_one = false);
  void emit_body_forward(const std::string& pre, const std::string& unit, bool recompute, int g);
  void emit_body_reverse(int g);
  void emit_scenario();
  bool gather_is_launch_invariant() const;
  void emit_shared_gather();
  void emit_reverse_for_output(int o);
  void acc_line(int32_t k, const std::string& x);
};

std::string Emitter::fwd_expr(int op, const std::string& A, const std::string& B, double c, int32_t a,
                              bool a_one) const {
  switch (op) {
    case NT_CONST: return lit(c, cfg_.f32);
    case NT_INPUT: return "in" + std::to_string(a);
    case NT_ADD: return A + " + " + B;
    case NT_SUB: return A + " - " + B;
    case NT_MUL: return A + " * " + B;
    case NT_DIV:
      // 1 / x in single precision: the correctly rounded reciprocal, the bits
      // of the IEEE division without its general-quotient path.
      if (cfg_.f32 && a_one) return "nt_rcp32(" + B + ")";
      return A + " / " + B;
    case NT_NEG: return "-" + A;
    case NT_EXP: {
      // fp32 tapes under the reference's fp32 semantics take the float-result
      // forms (NT_EXPF32...): evaluated in double, rounded once to float.
      const std::string e64 = exp_fn_;
      if (!cfg_.wide32) return R(e64.c_str(), "expf(") + A + ")";
      return "NT_EXPF32" + e64.substr(std::string("NT_EXP64").size()) + A + ")";
    }
    case NT_LOG: return cfg_.wide32 ? "((float)log((double)" + A + "))" : R("log(", "logf(") + A + ")";
    case NT_SQRT: return R("sqrt(", "sqrtf(") + A + ")";
    case NT_ABS: return R("fabs(", "fabsf(") + A + ")";
    case NT_MAX: return R("nt_max64(", "nt_max32(") + A + ", " + B + ")";
    case NT_MIN: return R("nt_min64(", "nt_min32(") + A + ", " + B + ")";
  }
  fail(NT_E_INTERNAL, "fwd_expr: unexpected op");
}

// Adjoint contribution of one node (ScalarReplay.java:139-165).  da/db are
// null when that argument is inactive (no contribution emitted).
void Emitter::emit_rule(int op, const std::string& D, const std::string& Va, const std::string& Vb,
                        const std::string& Vi, const std::string* da, const std::string* db, bool a_one) {
  const std::string half = cfg_.f32 ? "0.5f" : "0.5";
  const std::string zero = cfg_.f32 ? "0.0f" : "0.0";
  switch (op) {
    case NT_ADD:
      if (da) o_.line(contrib(*da, '+', D));
      if (db) o_.line(contrib(*db, '+', D));
      break;
    case NT_SUB:
      if (da) o_.line(contrib(*da, '+', D));
      if (db) o_.line(contrib(*db, '-', D));
      break;
    case NT_MUL:
      if (da) o_.line(contrib(*da, '+', D + " * " + Vb));
      if (db) o_.line(contrib(*db, '+', D + " * " + Va));
      break;
    case NT_DIV:
      if (!cfg_.f32) {  // the interpreter's order, so the host build keeps its bits
        if (da) o_.line(contrib(*da, '+', D + " / " + Vb));
        if (db) o_.line(contrib(*db, '-', D + " * " + Vi + " / " + Vb));
      } else if (a_one && db && !da) {
        // z = 1 / b, dz/db = -z / b = -z^2 to within the reciprocal's
        // rounding (2^-24 relative): no division in the reverse sweep, whose
        // tiny adjoint quotients sent the IEEE division down its slow path.
        // The products are rounded as written (never fused into the update),
        // so every kernel built from the tape gives the same bits.
        o_.line(contrib(*db, '-', "nt_fmul_rn(nt_fmul_rn(" + D + ", " + Vi + "), " + Vi + ")"));
      } else {
        // The interpreter's partials exactly: d / b is the correctly rounded
        // float quotient either way, and d z / b is formed in double (the
        // product of two floats is exact there) and rounded once to float.
        if (da) o_.line(contrib(*da, '+', D + " / " + Vb));
        if (db) o_.line(contrib(*db, '-', "(real)((double)" + D + " * (double)" + Vi + " / (double)" + Vb + ")"));
      }
      break;
    case NT_NEG:
      if (da) o_.line(contrib(*da, '-', D));
      break;
    case NT_EXP:
      if (da) o_.line(contrib(*da, '+', D + " * " + Vi));
      break;
    case NT_LOG:
      if (da) o_.line(contrib(*da, '+', D + " / " + Va));
      break;
    case NT_SQRT:
      if (da) o_.line(contrib(*da, '+', D + " * " + half + " / " + Vi));
      break;
    case NT_ABS:
      if (da) o_.line(contrib(*da, '+', "(" + Va + " < " + zero + " ? -" + D + " : " + D + ")"));
      break;
    case NT_MAX:
    case NT_MIN: {
      // A branch that is not taken leaves its register as it was, so an
      // assignment in the branch is still exact.
      const std::string cmp = "(" + Va + (op == NT_MAX ? " >= " : " <= ") + Vb + ")";
      if (da && db) {
        const std::string sa = contrib(*da, '+', D), sb = contrib(*db, '+', D);
        o_.line("if " + cmp + " " + sa + " else " + sb);
      } else if (da) {
        o_.line("if " + cmp + " " + contrib(*da, '+', D));
      } else if (db) {
        o_.line("if (!" + cmp + ") " + contrib(*db, '+', D));
      }
      break;
    }
    default: break;
  }
}

// Straight-line forward over [lo, hi) (prologue or epilogue).  Normal draws
// whose pair partner is in the same range share one Philox block.
void Emitter::emit_straight_forward(int32_t lo, int32_t hi) {
  std::map<std::pair<int32_t, int32_t>, std::vector<int32_t>> pairs;  // (stream, pair) -> nodes
  for (int32_t i = lo; i < hi; ++i)
    if (t_.op[i] == NT_RANDN) pairs[{t_.b[i], t_.a[i] >> 1}].push_back(i);
  std::map<int32_t, bool> done;
  const std::string real_t = "real";
  for (int32_t i = lo; i < hi; ++i) {
    const int op = t_.op[i];
    const std::string vi = "v" + std::to_string(i);
    if (op == NT_RANDN) {
      if (done.count(i)) continue;
      const auto& grp = pairs[{t_.b[i], t_.a[i] >> 1}];
      int32_t even = -1, odd = -1;
      for (int32_t x : grp) ((t_.a[x] & 1) ? odd : even) = x;
      const std::string key = "key" + std::to_string(t_.b[i]);
      if (even >= 0 && odd >= 0) {
        o_.line("real v" + std::to_string(even) + ", v" + std::to_string(odd) + ";");
        o_.line(rng_pair() + key + ", " + std::to_string(t_.a[i] >> 1) +
                "u, &v" + std::to_string(even) + ", &v" + std::to_string(odd) + ");");
        done[even] = done[odd] = true;
      } else {
        o_.line("const real " + vi + " = " + rng_single() + key + ", " +
                std::to_string(t_.a[i]) + "u);");
      }
      continue;
    }
    if (op == NT_RANDU) {
      o_.line("const real " + vi + " = " + R("nt_uniform64(", "nt_uniform32(") + "key" +
              std::to_string(t_.b[i]) + ", " + std::to_string(t_.a[i]) + "u);");
      continue;
    }
    const std::string A = nargs(op) >= 1 ? val_outside(t_.a[i]) : "";
    const std::string B = nargs(op) >= 2 ? val_outside(t_.b[i]) : "";
    o_.line("const " + real_t + " " + vi + " = " +
            fwd_expr(op, A, B, t_.c[i], t_.a[i], nargs(op) >= 1 && node_is_one(t_.a[i])) + ";");
  }
}

void Emitter::emit_straight_reverse(int32_t lo, int32_t hi) {
  for (int32_t i = hi - 1; i >= lo; --i) {
    if (!t_.active[i]) continue;
    const int op = t_.op[i];
    if (nargs(op) == 0) continue;
    const std::string D = "d" + std::to_string(i);
    const int32_t a = t_.a[i], b = nargs(op) == 2 ? t_.b[i] : -1;
    const std::string Va = val_outside(a), Vb = b >= 0 ? val_outside(b) : "", Vi = "v" + std::to_string(i);
    std::string da = adj_outside(a), db = b >= 0 ? adj_outside(b) : "";
    const bool aa = active_outside(a), ab = b >= 0 && active_outside(b);
    emit_rule(op, D, Va, Vb, Vi, aa ? &da : nullptr, ab ? &db : nullptr, node_is_one(a));
  }
}

// One unit of the loop body.  Forward loop: pre = "f", unit = "u".
// Recompute: pre = "r<g>_", unit = "(s * G + g)", carry refs of unit 0 read the
// restored segment-start carries cs<k>, later units read unit g-1.
void Emitter::emit_body_forward(const std::string& pre, const std::string& unit, bool recompute, int g) {
  const int32_t L = lp_.L;
  auto name = [&](int32_t j) { return pre + std::to_string(j); };
  auto ref = [&](const Ref& r) -> std::string {
    if (r.kind == REF_SAME) return name(r.idx);
    if (r.kind == REF_CARRY) {
      if (!recompute) return "cv" + std::to_string(r.idx);
      if (g == 0) return "cs" + std::to_string(r.idx);
      return "r" + std::to_string(g - 1) + "_" + std::to_string(r.idx);
    }
    if (r.kind == REF_GATHER) return gv_ref(r.idx, unit);
    return val_outside(r.idx);
  };
  // Pairing of normal draws inside the unit.
  std::map<int32_t, int32_t> partner;  // j -> partner j'
  for (int32_t j = 0; j < L; ++j) {
    const BodyNode& x = lp_.body[j];
    if (x.op != NT_RANDN || (x.draw_stride & 1)) continue;
    for (int32_t k = 0; k < L; ++k) {
      const BodyNode& y = lp_.body[k];
      if (k != j && y.op == NT_RANDN && y.stream == x.stream && y.draw_stride == x.draw_stride &&
          (y.draw_base ^ 1) == x.draw_base) {
        partner[j] = k;
      }
    }
  }
  std::vector<uint8_t> emitted(L, 0);
  for (int32_t j = 0; j < L; ++j) {
    if (recompute && !lp_.recompute[j]) continue;
    if (emitted[j]) continue;
    const BodyNode& bn = lp_.body[j];
    if (lp_.tape_slot[j] >= 0 && (recompute || (reuse_draws_ && is_draw(bn.op)))) {
      o_.line(name(j) + " = NT_TAPE(" + unit + ", " + std::to_string(lp_.tape_slot[j]) + ");");
      emitted[j] = 1;
      continue;
    }
    const std::string key = "key" + std::to_string(bn.stream);
    if (bn.op == NT_RANDN && !recompute && lp_.half_pairs && (bn.draw_stride & 1)) {
      // Units alternate: an even ordinal draws the pair, the next unit takes
      // the kept second leg (the loop starts at an even ordinal).
      const std::string ord = "(nt_u32)(" + std::to_string(bn.draw_base) + " + " + unit + " * " +
                              std::to_string(bn.draw_stride) + ")";
      o_.line("if ((" + ord + " & 1u) == 0u) " + rng_pair() + key + ", " + ord + " >> 1, &" + name(j) +
              ", &nt_hl" + std::to_string(j) + "); else " + name(j) + " = nt_hl" + std::to_string(j) + ";");
      emitted[j] = 1;
      continue;
    }
    if (bn.op == NT_RANDN) {
      auto it = partner.find(j);
      if (it != partner.end()) {
        const int32_t k = it->second;
        const int32_t ev = (bn.draw_base & 1) ? k : j, od = (bn.draw_base & 1) ? j : k;
        const int32_t pb = lp_.body[ev].draw_base >> 1, ps = bn.draw_stride >> 1;
        o_.line(rng_pair() + key + ", (nt_u32)(" + std::to_string(pb) + " + " +
                unit + " * " + std::to_string(ps) + "), &" + name(ev) + ", &" + name(od) + ");");
        emitted[ev] = emitted[od] = 1;
      } else {
        o_.line(name(j) + " = " + rng_single() + key + ", (nt_u32)(" +
                std::to_string(bn.draw_base) + " + " + unit + " * " + std::to_string(bn.draw_stride) + "));");
        emitted[j] = 1;
      }
      continue;
    }
    if (bn.op == NT_RANDU) {
      o_.line(name(j) + " = " + R("nt_uniform64(", "nt_uniform32(") + key + ", (nt_u32)(" +
              std::to_string(bn.draw_base) + " + " + unit + " * " + std::to_string(bn.draw_stride) + "));");
      emitted[j] = 1;
      continue;
    }
    const std::string A = nargs(bn.op) >= 1 ? ref(bn.ra) : "";
    const std::string B = nargs(bn.op) >= 2 ? ref(bn.rb) : "";
    // Loop exps the reverse sweep recomputes record wide arguments in the
    // forward sweep; the recompute itself takes the series when none was.
    if (recompute) exp_fn_ = series_exp_ ? "NT_EXP64_SERIES(" : "NT_EXP64(";
    else if (lp_.recompute[j] && lp_.tape_slot[j] < 0) exp_fn_ = fwd_fast_ ? "NT_EXP64F(" : "NT_EXP64W(";
    else if (fwd_fast_ && !cfg_.f32) exp_fn_ = "NT_EXP64T(";
    if (bn.op == NT_CONST && bn.cslot >= 0)
      o_.line(name(j) + " = NT_CTAB(" + unit + ", " + std::to_string(bn.cslot) + ");");
    else
      o_.line(name(j) + " = " + fwd_expr(bn.op, A, B, bn.c, -1, nargs(bn.op) >= 1 && ref_is_one(bn.ra)) + ";");
    exp_fn_ = "NT_EXP64(";
    emitted[j] = 1;
  }
}

// Reverse of unit g of the current segment (values from the recompute).
void Emitter::emit_body_reverse(int g) {
  const int32_t L = lp_.L;
  const std::string G = std::to_string(g);
  const std::string unit = "(s * " + std::to_string(lp_.G) + " + " + G + ")";
  auto val = [&](const Ref& r) -> std::string {
    if (r.kind == REF_SAME) return "r" + G + "_" + std::to_string(r.idx);
    if (r.kind == REF_CARRY) {
      if (g == 0) return "cs" + std::to_string(r.idx);
      return "r" + std::to_string(g - 1) + "_" + std::to_string(r.idx);
    }
    if (r.kind == REF_GATHER) return gv_ref(r.idx, unit);
    return val_outside(r.idx);
  };
  auto adj = [&](const Ref& r, bool* active) -> std::string {
    if (r.kind == REF_SAME) { *active = lp_.body[r.idx].active; return "b" + std::to_string(r.idx); }
    if (r.kind == REF_CARRY) { *active = lp_.body[r.idx].active; return "n" + std::to_string(r.idx); }
    if (r.kind == REF_GATHER) { *active = gather_active(r.idx); return "gd" + std::to_string(r.idx); }
    *active = t_.active[r.idx] != 0;
    return "d" + std::to_string(r.idx);
  };
  o_.open("{");
  zero_.clear();  // the unit's own registers start at zero; outer ones never do here
  // A gathered argument's adjoint collects the unit's contributions in a
  // register (in the interpreter's order) and is stored to the unit's slot
  // once, at the end of the unit: one local store per unit instead of a
  // load and a store per contribution.
  std::vector<int32_t> gathered;
  for (int32_t j = 0; j < L; ++j) {
    const BodyNode& bn = lp_.body[j];
    for (const Ref* r : {&bn.ra, &bn.rb})
      if (r->kind == REF_GATHER && gather_active(r->idx) &&
          std::find(gathered.begin(), gathered.end(), r->idx) == gathered.end())
        gathered.push_back(r->idx);
  }
  for (int32_t k : gathered) {
    o_.line("real gd" + std::to_string(k) + " = " + (cfg_.f32 ? "0.0f;" : "0.0;"));
    zero_.insert("gd" + std::to_string(k));
  }
  for (int32_t j = 0; j < L; ++j) {
    const BodyNode& bn = lp_.body[j];
    if (!bn.active) continue;
    std::string init = cfg_.f32 ? "0.0f" : "0.0";
    if (lp_.is_carry[j]) init = "cd" + std::to_string(j);
    else if (lp_.is_exit[j]) init = "xd" + std::to_string(j);
    else zero_.insert("b" + std::to_string(j));
    o_.line("real b" + std::to_string(j) + " = " + init + ";");
  }
  for (int32_t k : lp_.carries)
    if (lp_.body[k].active) {
      o_.line("real n" + std::to_string(k) + " = " + (cfg_.f32 ? "0.0f;" : "0.0;"));
      zero_.insert("n" + std::to_string(k));
    }
  for (int32_t j = L - 1; j >= 0; --j) {
    const BodyNode& bn = lp_.body[j];
    if (!bn.active || nargs(bn.op) == 0) continue;
    bool aa = false, ab = false;
    std::string da = adj(bn.ra, &aa);
    std::string db = nargs(bn.op) == 2 ? adj(bn.rb, &ab) : "";
    const std::string Va = val(bn.ra), Vb = nargs(bn.op) == 2 ? val(bn.rb) : "";
    const std::string Vi = "r" + G + "_" + std::to_string(j);
    emit_rule(bn.op, "b" + std::to_string(j), Va, Vb, Vi, aa ? &da : nullptr, ab ? &db : nullptr,
              ref_is_one(bn.ra));
  }
  for (int32_t k : lp_.carries)
    if (lp_.body[k].active) o_.line("cd" + std::to_string(k) + " = n" + std::to_string(k) + ";");
  for (int32_t j : lp_.exits)
    if (!lp_.is_carry[j] && lp_.body[j].active) o_.line("xd" + std::to_string(j) + " = " + (cfg_.f32 ? "0.0f;" : "0.0;"));
  for (int32_t k : gathered) o_.line("nt_gd" + std::to_string(k) + "[" + unit + "] = gd" + std::to_string(k) + ";");
  zero_.clear();
  o_.close();
}

void Emitter::emit_reverse_for_output(int o) {
  const std::string zero = cfg_.f32 ? "0.0f" : "0.0";
  const std::string one = cfg_.f32 ? "1.0f" : "1.0";
  const int32_t out = t_.output_node[o];
  const int32_t stride = 2 + t_.n_in();
  o_.open("{  // reverse sweep, output " + std::to_string(o));
  // Adjoint registers of every active node outside the loop.
  zero_.clear();
  for (int32_t i = 0; i < t_.n; ++i) {
    if (in_loop(i) || !t_.active[i]) continue;
    o_.line("real d" + std::to_string(i) + " = " + zero + ";");
    zero_.insert("d" + std::to_string(i));
  }
  if (lp_.present) {
    for (int32_t k : lp_.carries)
      if (lp_.body[k].active) {
        o_.line("real cd" + std::to_string(k) + " = " + zero + ";");
        zero_.insert("cd" + std::to_string(k));
      }
    for (int32_t j : lp_.exits)
      if (!lp_.is_carry[j] && lp_.body[j].active) {
        o_.line("real xd" + std::to_string(j) + " = " + zero + ";");
        zero_.insert("xd" + std::to_string(j));
      }
  }
  if (active_outside(out)) {
    o_.line(adj_outside(out) + " = " + one + ";");
    zero_.erase(adj_outside(out));
  }

  if (!lp_.present) {
    emit_straight_reverse(0, t_.n);
  } else {
    emit_straight_reverse(lp_.end(), t_.n);
    zero_.clear();  // the segment loop runs its code more than once
    const int32_t L = lp_.L, G = lp_.G, K = lp_.K;
    const int32_t nck = (int32_t)lp_.ckpt.size();
    // Every unit stores its slot of each active gathered adjoint (see
    // emit_body_reverse), so the arrays need no initial zeroing.
    for (size_t k = 0; k < lp_.gather.size(); ++k)
      if (gather_active((int32_t)k))
        o_.line("real nt_gd" + std::to_string(k) + "[" + std::to_string(lp_.N) + "];");
    if (cfg_.target != 1 && cfg_.rev_unroll > 1) o_.line("#pragma unroll " + std::to_string(cfg_.rev_unroll));
    o_.open("for (int s = " + std::to_string(K - 1) + "; s >= 0; --s) {");
    for (int32_t c = 0; c < nck; ++c)
      o_.line("const real cs" + std::to_string(lp_.ckpt[c]) + " = NT_CK(s * " + std::to_string(nck) + " + " +
              std::to_string(c) + ");");
    if (lp_.n_tape > 0 && cfg_.target == 0) {
      // The previous segment's tape (and checkpoint) rows of the whole block
      // are one contiguous range of the block's tile: one thread sends them
      // to L2 as a bulk prefetch while this segment is reversed.
      const std::string seg = std::to_string(G) + " * NT_NTAPE * NT_BLOCK";
      o_.open("if (s > 0 && threadIdx.x == 0) {");
      o_.line("nt_prefetch_l2_bulk(nt_tape_blk + (nt_u64)(s - 1) * (" + seg + "), (unsigned)(" + seg +
              " * sizeof(real)));");
      if (cfg_.global_ckpt && nck > 0)
        o_.line("nt_prefetch_l2_bulk(nt_gck_blk + (nt_u64)(s - 1) * (" + std::to_string(nck) +
                " * NT_BLOCK), (unsigned)(" + std::to_string(nck) + " * NT_BLOCK * sizeof(real)));");
      o_.close();
    }
    for (int g = 0; g < G; ++g) {
      std::string decl;
      for (int32_t j = 0; j < L; ++j)
        decl += (decl.empty() ? "real " : ", ") + ("r" + std::to_string(g) + "_" + std::to_string(j));
      o_.line(decl + ";");
    }
    for (int g = 0; g < G; ++g) {
      o_.line("// recompute unit " + std::to_string(g));
      emit_body_forward("r" + std::to_string(g) + "_", "(s * " + std::to_string(G) + " + " + std::to_string(g) + ")",
                        true, g);
    }
    for (int g = G - 1; g >= 0; --g) emit_body_reverse(g);
    if (discard_ && o == t_.n_out() - 1) {
      // The last output's sweep has consumed this segment's tape rows; no
      // read follows before the next path rewrites them, so when the tape in
      // flight fits in L2 the warp drops its part of them there instead of
      // leaving dirty lines to be written back.  Every lane's loads of the
      // rows are done (their values are used above, and the __syncwarp orders
      // them before any lane's discard).
      o_.open("if (nt_tape_in_l2) {");
      o_.line("__syncwarp();");
      o_.line("nt_discard_rows_l2<real, " + std::to_string(G) + " * NT_NTAPE, NT_BLOCK>(nt_tape_blk + (nt_u64)s * (" +
              std::to_string(G) + " * NT_NTAPE * NT_BLOCK) + (threadIdx.x & ~31u), nt_lane);");
      o_.close();
    }
    o_.close();
    // Unit 0's carry adjoints belong to the carries' initial values.
    for (size_t c = 0; c < lp_.carries.size(); ++c) {
      const int32_t k = lp_.carries[c], x = lp_.carry_init[c];
      if (lp_.body[k].active && t_.active[x]) o_.line("d" + std::to_string(x) + " += cd" + std::to_string(k) + ";");
    }
    // Each unit's gathered adjoint belongs to the node that unit read (last
    // unit first, the order in which the interpreter would have added them).
    for (size_t k = 0; k < lp_.gather.size(); ++k)
      if (gather_active((int32_t)k))
        for (int32_t u = lp_.N - 1; u >= 0; --u)
          if (t_.active[lp_.gather[k][u]])
            o_.line("d" + std::to_string(lp_.gather[k][u]) + " += nt_gd" + std::to_string(k) + "[" + std::to_string(u) +
                    "];");
    emit_straight_reverse(0, lp_.B);
  }
  for (int32_t j = 0; j < t_.n_in(); ++j) {
    const int32_t node = t_.input_node[j];
    acc_line(o * stride + 2 + j, "(double)" + adj_outside(node));
  }
  o_.close();
}

// Per-path accumulation.  The replay kernel sums each warp tile of 32 paths
// with a fixed butterfly (lane k % 32 keeps channel k's tile sum) and adds the
// tile sums exactly at the end of the tile (nt_tile_xadd), so its totals do
// not depend on the grid, the chunking or the GPU count; the multi-market
// kernel keeps compensated (TwoSum) per-thread sums; the host target keeps a
// plain running sum, which reproduces AadTotals.add exactly.
void Emitter::acc_line(int32_t k, const std::string& x) {
  const std::string K = std::to_string(k);
  if (cfg_.target == 1 && cfg_.markets) o_.line("nt_acc[nt_m * NT_CH + " + K + "] += " + x + ";");
  else if (cfg_.target == 1) o_.line("nt_acc[" + K + "] += " + x + ";");
  else if (cfg_.markets) o_.line("nt_two_sum(&NT_ACC(" + K + "), &NT_CMP(" + K + "), " + x + ");");
  else
    o_.line("{ const double nt_s = nt_warp_allsum(nt_live ? " + x + " : 0.0); if (nt_lane == " + std::to_string(k % 32) +
            "u) nt_ws[" + std::to_string(k / 32) + "] = nt_s; }");
}

// True when no gathered node depends on a draw: then every path of a launch
// reads the same gathered values.
bool Emitter::gather_is_launch_invariant() const {
  if (!lp_.present || lp_.gather.empty()) return false;
  std::vector<uint8_t> drawn(lp_.B, 0);
  for (int32_t i = 0; i < lp_.B; ++i) {
    const int op = t_.op[i];
    if (is_draw(op)) drawn[i] = 1;
    else if (is_unary(op) || is_binary(op))
      drawn[i] = drawn[t_.a[i]] | (is_binary(op) ? drawn[t_.b[i]] : 0);
  }
  for (const auto& g : lp_.gather)
    for (int32_t x : g)
      if (drawn[x]) return false;
  return true;
}

// The gathered values' cone of prologue nodes, evaluated by every thread
// before the path loop (no draw among them), written to shared memory by
// thread 0.
void Emitter::emit_shared_gather() {
  std::vector<uint8_t> need(lp_.B, 0);
  for (const auto& g : lp_.gather)
    for (int32_t x : g) need[x] = 1;
  for (int32_t i = lp_.B - 1; i >= 0; --i) {
    if (!need[i]) continue;
    const int op = t_.op[i];
    if (is_unary(op) || is_binary(op)) need[t_.a[i]] = 1;
    if (is_binary(op)) need[t_.b[i]] = 1;
  }
  const int32_t NG = (int32_t)lp_.gather.size();
  o_.line("__shared__ real nt_gvs[" + std::to_string(NG * lp_.N) + "];");
  o_.open("{  // gathered arguments: the same for every path of the launch");
  const std::string saved = exp_fn_;
  exp_fn_ = "NT_EXP64(";
  for (int32_t i = 0; i < lp_.B; ++i) {
    if (!need[i]) continue;
    const int op = t_.op[i];
    const std::string A = nargs(op) >= 1 ? val_outside(t_.a[i]) : "";
    const std::string B = nargs(op) >= 2 ? val_outside(t_.b[i]) : "";
    o_.line("const real v" + std::to_string(i) + " = " +
            fwd_expr(op, A, B, t_.c[i], t_.a[i], nargs(op) >= 1 && node_is_one(t_.a[i])) + ";");
  }
  exp_fn_ = saved;
  o_.open("if (threadIdx.x == 0) {");
  for (int32_t k = 0; k < NG; ++k)
    for (int32_t u = 0; u < lp_.N; ++u)
      o_.line("nt_gvs[" + std::to_string(k * lp_.N + u) + "] = " + val_outside(lp_.gather[k][u]) + ";");
  o_.close();
  o_.close();
  o_.line("__syncthreads();");
}

void Emitter::emit_scenario() {
  if (cfg_.target == 0) o_.line("bool nt_wide = false;  // some EXP argument left the series range");
  // Stream keys.
  std::vector<uint8_t> used(t_.n_streams, 0);
  for (int32_t i = 0; i < t_.n; ++i)
    if (is_draw(t_.op[i])) used[t_.b[i]] = 1;
  for (int32_t s = 0; s < t_.n_streams; ++s)
    if (used[s]) o_.line("const nt_key key" + std::to_string(s) + " = nt_make_key(path, seed, " + std::to_string(s) + ");");

  if (!lp_.present) {
    emit_straight_forward(0, t_.n);
  } else {
    const int32_t L = lp_.L, G = lp_.G, K = lp_.K;
    emit_straight_forward(0, lp_.B);
    // Gathered arguments: the prologue node each unit reads, as one array
    // indexed by the unit (in shared memory, filled before the path loop,
    // when they depend on no draw).
    for (size_t k = 0; k < lp_.gather.size() && !gv_shared_; ++k) {
      std::string init;
      for (int32_t x : lp_.gather[k]) init += (init.empty() ? "" : ", ") + val_outside(x);
      o_.line("const real nt_gv" + std::to_string(k) + "[" + std::to_string(lp_.N) + "] = {" + init + "};");
    }
    o_.line("// step loop: " + std::to_string(lp_.N) + " units of " + std::to_string(L) + " nodes (" +
            std::to_string(lp_.steps_per_unit) + " steps each), " + std::to_string(K) + " segments of " +
            std::to_string(G) + " units");
    for (size_t c = 0; c < lp_.carries.size(); ++c)
      o_.line("real cv" + std::to_string(lp_.carries[c]) + " = " + val_outside(lp_.carry_init[c]) + ";");
    if (lp_.half_pairs)
      for (int32_t j = 0; j < L; ++j)
        if (lp_.body[j].op == NT_RANDN && (lp_.body[j].draw_stride & 1))
          o_.line("real nt_hl" + std::to_string(j) + " = " + (cfg_.f32 ? "0.0f;" : "0.0;") +
                  "  // second Box-Muller leg, kept for the next unit");
    for (int32_t j : lp_.exits)
      if (!lp_.is_carry[j]) o_.line("real xv" + std::to_string(j) + " = " + (cfg_.f32 ? "0.0f;" : "0.0;"));
    const int32_t nck = (int32_t)lp_.ckpt.size();
    auto forward_loop = [&]() {
      o_.open("for (int s = 0; s < " + std::to_string(K) + "; ++s) {");
      for (int32_t c = 0; c < nck; ++c)
        o_.line("NT_CK(s * " + std::to_string(nck) + " + " + std::to_string(c) + ") = cv" +
                std::to_string(lp_.ckpt[c]) + ";");
      if (reuse_draws_ && cfg_.target == 0) {
        // The forward now reads the tape: the next segment's rows head for L2
        // while this one runs, as in the reverse sweep.
        const std::string seg = std::to_string(G) + " * NT_NTAPE * NT_BLOCK";
        o_.line("if (s + 1 < " + std::to_string(K) + " && threadIdx.x == 0) nt_prefetch_l2_bulk(nt_tape_blk + "
                "(nt_u64)(s + 1) * (" + seg + "), (unsigned)(" + seg + " * sizeof(real)));");
      }
      // The segment's units are unrolled by default: a unit's draws and
      // transcendentals depend only on its counter, so the compiler overlaps
      // them with the previous unit's carry chain (+13 % on the 252-step
      // Asian).  A market that reads its draws back unrolls the segment too,
      // so the segment's tape loads are all in flight before the first unit
      // needs one.
      if (cfg_.target == 0)
        o_.line(reuse_draws_ || cfg_.fwd_unroll <= 0 ? std::string("#pragma unroll")
                                                      : "#pragma unroll " + std::to_string(cfg_.fwd_unroll));
      o_.open("for (int g = 0; g < " + std::to_string(G) + "; ++g) {");
      o_.line("const int u = s * " + std::to_string(G) + " + g;");
      std::string decl;
      for (int32_t j = 0; j < L; ++j) decl += (j ? ", f" : "real f") + std::to_string(j);
      o_.line(decl + ";");
      emit_body_forward("f", "u", false, 0);
      for (int32_t j = 0; j < L; ++j)
        if (lp_.tape_slot[j] >= 0 && !(reuse_draws_ && is_draw(lp_.body[j].op)))
          o_.line("NT_TAPE(u, " + std::to_string(lp_.tape_slot[j]) + ") = f" + std::to_string(j) + ";");
      for (int32_t k : lp_.carries) o_.line("cv" + std::to_string(k) + " = f" + std::to_string(k) + ";");
      for (int32_t j : lp_.exits)
        if (!lp_.is_carry[j]) o_.line("xv" + std::to_string(j) + " = f" + std::to_string(j) + ";");
      o_.close();
      o_.close();
    };
    // Exps the reverse sweep recomputes run in the forward loop as the bare
    // series, recording wide arguments, and fp64 exps whose values are taped
    // skip the full-range routine's clamp and two-step scaling up to |x| =
    // 700; a warp that recorded a wide argument runs the loop again from its
    // initial carries with the full-range routine (which rewrites the tape
    // and the checkpoints).  GBM steps and bond prices never take the redo.
    bool fast_exp = false;
    if (cfg_.target == 0 && (!cfg_.f32 || cfg_.wide32))
      for (int32_t j = 0; j < L; ++j)
        fast_exp |= lp_.body[j].op == NT_EXP &&
                    ((lp_.recompute[j] && lp_.tape_slot[j] < 0) || (!cfg_.f32 && lp_.tape_slot[j] >= 0));
    auto guarded_loop = [&]() {
      if (!fast_exp) {
        forward_loop();
        return;
      }
      fwd_fast_ = true;
      forward_loop();
      fwd_fast_ = false;
      o_.open("if (__any_sync(nt_lanes, nt_wide)) {  // an exp argument left the series range: redo, full range");
      for (size_t c = 0; c < lp_.carries.size(); ++c)
        o_.line("cv" + std::to_string(lp_.carries[c]) + " = " + val_outside(lp_.carry_init[c]) + ";");
      forward_loop();
      o_.close();
    };
    bool taped_draws = false;
    for (int32_t j = 0; j < L; ++j) taped_draws |= is_draw(lp_.body[j].op) && lp_.tape_slot[j] >= 0;
    if (cfg_.markets && taped_draws) {
      // The first market draws and tapes them; the others read them back.
      o_.open("if (nt_m == 0) {");
      guarded_loop();
      o_.close("} else {");
      ++o_.ind;
      reuse_draws_ = true;
      guarded_loop();
      reuse_draws_ = false;
      o_.close();
    } else {
      guarded_loop();
    }
    emit_straight_forward(lp_.end(), t_.n);
  }
  const int32_t stride = 2 + t_.n_in();
  for (int32_t o = 0; o < t_.n_out(); ++o) {
    const std::string y = "(double)" + val_outside(t_.output_node[o]);
    acc_line(o * stride, y);
    acc_line(o * stride + 1, y + " * " + y);
  }
  if (cfg_.adjoints) {
    // The reverse sweep recomputes EXP nodes when they are not taped
    // (draws-only tape, recompute-all).  On the device it is emitted twice:
    // the copy for warps whose forward exps all stayed in the series range
    // uses the bare series, the other the full-range routine.
    bool rev_exp = false;
    if (lp_.present && cfg_.target == 0 && (!cfg_.f32 || cfg_.wide32))
      for (int32_t j = 0; j < lp_.L; ++j)
        rev_exp |= lp_.recompute[j] && lp_.tape_slot[j] < 0 && lp_.body[j].op == NT_EXP;
    if (rev_exp) {
      o_.open("if (!__any_sync(nt_lanes, nt_wide)) {");
      series_exp_ = true;
      for (int32_t o = 0; o < t_.n_out(); ++o) emit_reverse_for_output(o);
      series_exp_ = false;
      o_.close("} else {");
      ++o_.ind;
      for (int32_t o = 0; o < t_.n_out(); ++o) emit_reverse_for_output(o);
      o_.close();
    } else {
      for (int32_t o = 0; o < t_.n_out(); ++o) emit_reverse_for_output(o);
    }
  }
}

std::string Emitter::run() {
  const bool host = cfg_.target == 1;
  const bool mk = cfg_.markets;
  gv_shared_ = cfg_.target == 0 && !mk && gather_is_launch_invariant();
  // Emitted only where the tape can fit at all: one block on each of the
  // B200's 148 SMs must stay within the run-time budget (96 MB, the device
  // runtime's NT_L2_TAPE_BYTES; the fp32 barrier's 256 x 3 KB x 148 = 114 MB
  // never does, and the code alone cost it 16 registers).
  discard_ = cfg_.target == 0 && !mk && cfg_.adjoints && lp_.present && lp_.n_tape > 0 && p_.per_unit_regs <= 32 &&
             (uint64_t)148 * cfg_.block * lp_.N * lp_.n_tape * (cfg_.f32 ? 4 : 8) <= (96ull << 20);
  const int32_t nck_total = ckpt_values(p_);
  o_.line("// Generated by libnabla_b200 from a " + std::to_string(t_.n) + "-node tape.");
  if (host) {
    o_.line("#define NT_HOST 1");
    o_.line("#include <stdint.h>");
  }
  o_.line("#include \"nt_device_rt.cuh\"");
  o_.line(std::string("typedef ") + (cfg_.f32 ? "float" : "double") + " real;");
  o_.line("#define NT_CH " + std::to_string(channels()));
  o_.line("#define NT_WS " + std::to_string((channels() + 31) / 32));
  o_.line("#define NT_NIN " + std::to_string(std::max(1, t_.n_in())));
  const int32_t ntape = lp_.present ? lp_.n_tape : 0;
  o_.line("#define NT_NTAPE " + std::to_string(std::max(1, ntape)));
  if (lp_.present && lp_.n_vary > 0) {
    // Loop constants that change from unit to unit (a non-uniform time grid,
    // per-date weights): one row per unit.  Every thread reads the same row at
    // the same time, so the loads are broadcasts from L1.
    o_.line("#define NT_NVARY " + std::to_string(lp_.n_vary));
    o_.line(std::string(host ? "static const real" : "__device__ __align__(16) const real") + " nt_ctab[" +
            std::to_string(lp_.ctab.size()) + "] = {");
    std::string row;
    for (size_t k = 0; k < lp_.ctab.size(); ++k) {
      row += "(real)" + lit(lp_.ctab[k], false) + ",";
      if (row.size() > 100 || k + 1 == lp_.ctab.size()) {
        o_.line("  " + row);
        row.clear();
      }
    }
    o_.line("};");
    if (!host && lp_.n_vary % 2 == 0) {
      // Rows of an even length start on 16-byte boundaries (8 in fp32): a
      // constant comes from its aligned pair by one vector load, which the
      // compiler shares with the pair's other constant -- half the load
      // instructions of the CVA book's 62 constants per date (+2 to +4 %).
      o_.line(std::string("#define NT_CTAB(u, k) nt_pick<(k) & 1>(__ldg(&reinterpret_cast<const ") +
              (cfg_.f32 ? "float2" : "double2") + "*>(nt_ctab)[((u) * NT_NVARY + (k)) >> 1]))");
    } else {
      o_.line(std::string("#define NT_CTAB(u, k) ") + (host ? "nt_ctab" : "__ldg(&nt_ctab") +
              "[(u) * NT_NVARY + (k)]" + (host ? "" : ")"));
    }
  }
  // Input registers: once per launch, or once per market in the multi-market
  // variant (inputs[m * NT_NIN + j]).
  auto load_inputs = [&](const std::string& base) {
    for (int32_t j = 0; j < t_.n_in(); ++j)
      o_.line("const real in" + std::to_string(j) + " = (real)inputs[" + base + std::to_string(j) + "];");
  };
  if (host) {
    o_.line("#define NT_CK(slot) nt_ckbuf[(slot)]");
    o_.line("#define NT_TAPE(u, slot) nt_tapebuf[(nt_u64)(u) * NT_NTAPE + (slot)]");
    if (mk)
      o_.open("extern \"C\" void nt_host_replay_markets(const double* inputs, int n_states, uint64_t n_paths, "
              "uint64_t path_offset, uint64_t seed, double* sums) {");
    else
      o_.open("extern \"C\" void nt_host_replay(const double* inputs, uint64_t n_paths, uint64_t path_offset, "
              "uint64_t seed, double* sums) {");
    if (!mk) load_inputs("");
    const std::string nacc = mk ? "n_states * NT_CH" : "NT_CH";
    o_.line("double* nt_acc = new double[" + nacc + "];");
    o_.line("for (int c = 0; c < " + nacc + "; ++c) nt_acc[c] = 0.0;");
    o_.line("real nt_ckbuf[" + std::to_string(std::max(1, nck_total)) + "];");
    o_.line("(void)nt_ckbuf;");
    o_.line("real* nt_tapebuf = new real[" + std::to_string(std::max(1, (lp_.present ? lp_.N : 1) * std::max(1, ntape))) + "];");
    o_.line("(void)nt_tapebuf;");
    o_.open("for (nt_u64 p = 0; p < n_paths; ++p) {");
    o_.line("const nt_u64 path = p + path_offset;");
    if (mk) {
      o_.open("for (int nt_m = 0; nt_m < n_states; ++nt_m) {");
      load_inputs("nt_m * NT_NIN + ");
      emit_scenario();
      o_.close();
    } else {
      emit_scenario();
    }
    o_.close();
    o_.line("for (int c = 0; c < " + nacc + "; ++c) sums[c] = nt_acc[c];");
    o_.line("delete[] nt_acc;");
    o_.line("delete[] nt_tapebuf;");
    o_.close();
    return o_.s;
  }
  o_.line("#define NT_BLOCK " + std::to_string(cfg_.block));
  // Global checkpoints and the value tape are laid out in one tile per block,
  // value-major inside the tile: a warp's store or load of one value is 32
  // consecutive words (one coalesced 256-byte transaction in fp64), and the
  // distance between two values is the compile-time constant NT_BLOCK, so the
  // unrolled segment code addresses them with immediate offsets.
  const bool gck = cfg_.global_ckpt && lp_.present && !lp_.ckpt.empty();
  const bool tape = lp_.present && lp_.n_tape > 0;
  if (cfg_.global_ckpt) {
    o_.line("#define NT_CKV " + std::to_string(lp_.present ? lp_.K * (int32_t)lp_.ckpt.size() : 0));
    o_.line("#define NT_CK(slot) nt_gck_b[(slot) * NT_BLOCK]");
  } else {
    o_.line("#define NT_CK(slot) nt_ck[(slot) * NT_BLOCK + threadIdx.x]");
  }
  o_.line("#define NT_NLOOP " + std::to_string(lp_.present ? lp_.N : 0));
  o_.line("#define NT_TAPE(u, slot) nt_tape_b[((u) * NT_NTAPE + (slot)) * NT_BLOCK]");
  // Launch bounds size the register budget for NT_BLOCK threads (and
  // min_blocks resident blocks); an explicit cap replaces them (NVRTC ignores
  // --maxrregcount on a kernel that has launch bounds).
  std::string bounds = cfg_.max_regs > 0
                           ? "__maxnreg__(" + std::to_string(cfg_.max_regs) + ")"
                           : "__launch_bounds__(NT_BLOCK" +
                                 (cfg_.min_blocks > 0 ? ", " + std::to_string(cfg_.min_blocks) : std::string()) + ")";
  if (mk) {
    o_.line("extern \"C\" __global__ void " + bounds + " nt_markets_kernel(");
    o_.line("    const double* __restrict__ inputs, int n_states, nt_u64 n_paths, nt_u64 path_offset, nt_u64 seed,");
    o_.line("    double* __restrict__ partials, unsigned int* __restrict__ ticket, double* __restrict__ out,");
    o_.line("    int accumulate, real* __restrict__ nt_gck, real* __restrict__ nt_tape, double* __restrict__ nt_gacc) {");
  } else {
    o_.line("extern \"C\" __global__ void " + bounds + " nt_replay_kernel(");
    o_.line("    const double* __restrict__ inputs, nt_u64 n_paths, nt_u64 path_offset, nt_u64 seed,");
    o_.line("    nt_i64* __restrict__ glim, unsigned int* __restrict__ ticket, double* __restrict__ out,");
    o_.line("    nt_i64* __restrict__ acc, int accumulate, real* __restrict__ nt_gck, real* __restrict__ nt_tape) {");
  }
  ++o_.ind;
  if (!cfg_.global_ckpt) o_.line("extern __shared__ real nt_ck[];");
  if (mk) o_.line("__shared__ double nt_red[NT_CH * (NT_BLOCK / 32)];");
  o_.line("const nt_u64 nt_gtid = (nt_u64)blockIdx.x * NT_BLOCK + threadIdx.x;");
  o_.line("const nt_u64 nt_gthreads = (nt_u64)gridDim.x * NT_BLOCK;");
  o_.line("(void)nt_gck; (void)nt_gthreads; (void)nt_tape;");
  if (gck) {
    o_.line("real* __restrict__ const nt_gck_blk = nt_gck + (nt_u64)blockIdx.x * (NT_CKV * NT_BLOCK);");
    o_.line("real* __restrict__ const nt_gck_b = nt_gck_blk + threadIdx.x;");
  }
  if (tape) {
    o_.line("real* __restrict__ const nt_tape_blk = nt_tape + (nt_u64)blockIdx.x * ((nt_u64)NT_NLOOP * NT_NTAPE * "
            "NT_BLOCK);");
    o_.line("real* __restrict__ const nt_tape_b = nt_tape_blk + threadIdx.x;");
  }
  if (discard_)
    o_.line("const bool nt_tape_in_l2 = (nt_u64)gridDim.x * NT_BLOCK * NT_NLOOP * NT_NTAPE * sizeof(real) <= "
            "NT_L2_TAPE_BYTES;");
  if (mk) {
    // Compensated per-market accumulators in a global block tile
    // [block][2 * market * NT_CH + 2k (+1)][thread of block], zeroed by the
    // host before the launch: touched once per scenario and market.
    o_.line("double* __restrict__ const nt_gacc_b = nt_gacc + (nt_u64)blockIdx.x * ((nt_u64)2 * n_states * NT_CH * "
            "NT_BLOCK) + threadIdx.x;");
    o_.line("#define NT_ACC(k) nt_gacc_b[(nt_u64)(2 * (nt_m * NT_CH + (k))) * NT_BLOCK]");
    o_.line("#define NT_CMP(k) nt_gacc_b[(nt_u64)(2 * (nt_m * NT_CH + (k)) + 1) * NT_BLOCK]");
  } else {
    load_inputs("");
    if (xshared()) {
      // The block's exact words (nt_exact.cuh), one record per channel.
      o_.line("__shared__ nt_i64 nt_xblk[NT_CH * NT_XWORDS];");
      o_.line("for (int i = threadIdx.x; i < NT_CH * NT_XWORDS; i += NT_BLOCK) nt_xblk[i] = 0;");
    } else {
      // Too many channels for shared memory: tile sums go straight to the
      // launch's words.
      o_.line("nt_i64* const nt_xblk = glim;");
    }
  }
  o_.line("nt_math_tables_load();");  // ends with __syncthreads()
  if (gv_shared_) emit_shared_gather();
  if (mk) {
    o_.open("for (nt_u64 p = nt_gtid; p < n_paths; p += nt_gthreads) {");
    o_.line("const nt_u64 path = p + path_offset;");
    o_.line("const unsigned nt_lanes = __activemask();");
  } else {
    // Warp tiles: the warp's lanes replay 32 consecutive paths of the launch,
    // the tile starting at a multiple of 32.  Lanes past the end replay the
    // tile's first path again (so they vote as it does) and contribute 0.
    o_.line("const unsigned nt_lane = threadIdx.x & 31u;");
    o_.open("for (nt_u64 nt_pw = nt_gtid - nt_lane; nt_pw < n_paths; nt_pw += nt_gthreads) {");
    o_.line("const bool nt_live = nt_pw + nt_lane < n_paths;");
    o_.line("const nt_u64 path = (nt_live ? nt_pw + nt_lane : nt_pw) + path_offset;");
    o_.line("const unsigned nt_lanes = 0xffffffffu;");
    o_.line("double nt_ws[NT_WS];  // this lane's tile sums: channel nt_lane + 32 r in nt_ws[r]");
  }
  o_.line("(void)nt_lanes;");
  if (mk) {
    o_.open("for (int nt_m = 0; nt_m < n_states; ++nt_m) {");
    load_inputs("nt_m * NT_NIN + ");
    emit_scenario();
    o_.close();
  } else {
    emit_scenario();
    o_.line("nt_tile_xadd(nt_xblk, nt_ws, NT_WS, NT_CH);");
  }
  o_.close();
  if (mk) {
    o_.line("nt_grid_reduce_cols(nt_gacc_b, NT_BLOCK, n_states * NT_CH, NT_CH, nt_red, partials, ticket, out, "
            "accumulate);");
  } else {
    o_.line(std::string("nt_xgrid_finish(nt_xblk, ") + (xshared() ? "1" : "0") +
            ", NT_CH, glim, ticket, out, acc, accumulate);");
  }
  o_.close();
  return o_.s;
}

}  // namespace

std::string emit(const Tape& t, const Plan& p, const EmitConfig& cfg) {
  Emitter e(t, p, cfg);
  return e.run();
}

}  // namespace nt
