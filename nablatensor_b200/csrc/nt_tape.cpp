// nt_tape.cpp -- tape ingest and validation.
//
// The C ABI borrows the caller's flat arrays; ingest() copies them and checks
// every index before anything is emitted, so a malformed tape becomes an
// NT_E_TAPE status instead of an out-of-bounds access in generated code.
#include <cmath>
#include <sstream>

#include "nt_internal.hpp"

namespace nt {

const char* op_name(int op) {
  static const char* names[] = {"CONST", "INPUT", "RANDN", "RANDU", "ADD", "SUB", "MUL", "DIV",
                                "NEG",   "EXP",   "LOG",   "SQRT",  "MAX", "MIN", "ABS"};
  return (op >= 0 && op <= NT_ABS) ? names[op] : "?";
}

static std::string where(int32_t i, int op) {
  std::ostringstream s;
  s << "node " << i << " (" << op_name(op) << ")";
  return s.str();
}

Tape ingest(const nt_tape* src) {
  if (!src) fail(NT_E_INVALID_ARG, "tape is null");
  const int32_t kMaxNodes = 1 << 26;
  if (src->n <= 0 || src->n > kMaxNodes) fail(NT_E_TAPE, "tape size out of range");
  if (!src->op || !src->arg_a || !src->arg_b || !src->constant)
    fail(NT_E_INVALID_ARG, "tape arrays must not be null");
  if (src->n_in < 0 || (src->n_in > 0 && !src->input_node)) fail(NT_E_TAPE, "bad input list");
  if (src->n_out <= 0 || !src->output_node) fail(NT_E_TAPE, "no output was recorded");
  if (src->n_streams <= 0 || src->n_streams > 1 << 20) fail(NT_E_TAPE, "bad stream count");

  Tape t;
  t.n = src->n;
  t.op.assign(src->op, src->op + t.n);
  t.a.assign(src->arg_a, src->arg_a + t.n);
  t.b.assign(src->arg_b, src->arg_b + t.n);
  t.c.assign(src->constant, src->constant + t.n);
  t.input_node.assign(src->input_node, src->input_node + src->n_in);
  t.output_node.assign(src->output_node, src->output_node + src->n_out);
  t.n_streams = src->n_streams;

  std::vector<int32_t> normals(t.n_streams, 0), uniforms(t.n_streams, 0);
  std::vector<int32_t> input_seen(t.n_in(), -1);
  for (int32_t i = 0; i < t.n; ++i) {
    const int op = t.op[i];
    if (op < NT_CONST || op > NT_ABS) fail(NT_E_TAPE, where(i, op) + ": unknown op code");
    if (is_unary(op) || is_binary(op)) {
      if (t.a[i] < 0 || t.a[i] >= i) fail(NT_E_TAPE, where(i, op) + ": first argument out of order");
    }
    if (is_binary(op)) {
      if (t.b[i] < 0 || t.b[i] >= i) fail(NT_E_TAPE, where(i, op) + ": second argument out of order");
    }
    if (op == NT_INPUT) {
      if (t.a[i] < 0 || t.a[i] >= t.n_in()) fail(NT_E_TAPE, where(i, op) + ": input index out of range");
      if (input_seen[t.a[i]] >= 0) fail(NT_E_TAPE, where(i, op) + ": input recorded twice");
      input_seen[t.a[i]] = i;
    }
    if (is_draw(op)) {
      if (t.b[i] < 0 || t.b[i] >= t.n_streams) fail(NT_E_TAPE, where(i, op) + ": stream out of range");
      if (t.a[i] < 0) fail(NT_E_TAPE, where(i, op) + ": negative draw ordinal");
      auto& cnt = op == NT_RANDN ? normals[t.b[i]] : uniforms[t.b[i]];
      // Ordinals are handed out in recording order (AadTape.Builder.addRandn).
      if (t.a[i] != cnt) fail(NT_E_TAPE, where(i, op) + ": draw ordinals must follow recording order");
      ++cnt;
    }
  }
  for (int32_t j = 0; j < t.n_in(); ++j) {
    const int32_t node = t.input_node[j];
    if (node < 0 || node >= t.n || t.op[node] != NT_INPUT || t.a[node] != j)
      fail(NT_E_TAPE, "input_node[" + std::to_string(j) + "] is not INPUT " + std::to_string(j));
  }
  for (int32_t o = 0; o < t.n_out(); ++o)
    if (t.output_node[o] < 0 || t.output_node[o] >= t.n)
      fail(NT_E_TAPE, "output_node[" + std::to_string(o) + "] out of range");
  if (src->normal_count) {
    for (int32_t s = 0; s < t.n_streams; ++s)
      if (src->normal_count[s] != normals[s]) fail(NT_E_TAPE, "normal_count disagrees with the nodes");
  }
  if (src->uniform_count) {
    for (int32_t s = 0; s < t.n_streams; ++s)
      if (src->uniform_count[s] != uniforms[s]) fail(NT_E_TAPE, "uniform_count disagrees with the nodes");
  }
  t.normal_count = normals;
  t.uniform_count = uniforms;

  t.active.assign(t.n, 0);
  for (int32_t i = 0; i < t.n; ++i) {
    const int op = t.op[i];
    if (op == NT_INPUT) t.active[i] = 1;
    else if (op == NT_CONST || is_draw(op)) t.active[i] = 0;
    else if (is_unary(op)) t.active[i] = t.active[t.a[i]];
    else t.active[i] = t.active[t.a[i]] || t.active[t.b[i]];
  }
  return t;
}

int32_t reduce_pow2_divisions(Tape& t, bool f32) {
  std::vector<int32_t> uses(t.n, 0), div_uses(t.n, 0);
  for (int32_t i = 0; i < t.n; ++i) {
    const int op = t.op[i];
    if (is_unary(op) || is_binary(op)) ++uses[t.a[i]];
    if (is_binary(op)) ++uses[t.b[i]];
    if (op == NT_DIV && t.a[i] != t.b[i]) ++div_uses[t.b[i]];
  }
  for (int32_t o : t.output_node) ++uses[o];  // an output constant keeps its value
  const int max_exp = f32 ? 126 : 1022;
  auto pow2 = [&](double c) {
    if (!std::isfinite(c) || c == 0.0) return false;
    int e = 0;
    const double m = std::frexp(std::fabs(c), &e);  // |c| = m 2^e, m in [0.5, 1)
    return m == 0.5 && std::abs(e - 1) <= max_exp;
  };
  int32_t n = 0;
  for (int32_t i = 0; i < t.n; ++i) {
    if (t.op[i] != NT_DIV) continue;
    const int32_t b = t.b[i];
    if (t.op[b] != NT_CONST || uses[b] != div_uses[b] || !pow2(t.c[b])) continue;
    // every use of b is a division by it: the node can hold the reciprocal
    for (int32_t k = i; k < t.n; ++k)
      if (t.op[k] == NT_DIV && t.b[k] == b) {
        t.op[k] = NT_MUL;
        ++n;
      }
    t.c[b] = 1.0 / t.c[b];
  }
  return n;
}

}  // namespace nt
