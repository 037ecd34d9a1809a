// The xt dialect's canonicalization: x + 0 -> x, 0 + x -> x, x - 0 -> x.
//
// Restates the reference's rewrite patterns (lib/xt/XTOps.cpp:395-449,
// pinned by test/xt/canonicalize.mlir): an operand is zero when an
// arith.constant defines it as a splat dense tensor of 0 (integer or float,
// either sign).  After the folds, ops the reference marks Pure
// (include/xt/XTOps.td: get_tile_block_id, the elementwise, cast, matmul,
// mma, reduce and shape ops) and arith.constant are erased when nothing uses
// their results, as MLIR's canonicalizer erases trivially dead ops; loads,
// stores and conv loads are kept.  Constants are not hoisted or merged.
#include <algorithm>
#include <set>
#include <string>

#include "ir.h"

namespace xt {
namespace {

bool is_zero_splat(const Module& m, const Func& f, int id) {
  const Value& v = m.value(id);
  if (v.def_op < 0 || v.def_op >= static_cast<int>(f.ops.size())) return false;
  const Op& d = f.ops[v.def_op];
  return d.name == "arith.constant" && d.is_dense && v.type.kind == Type::Tensor && d.fvalue == 0.0;
}

bool is_pure(const std::string& n) {
  static const std::set<std::string> kPure = {
      "arith.constant", "xt.get_tile_block_id", "xt.add", "xt.sub", "xt.mul", "xt.exp", "xt.cos", "xt.sin",
      "xt.reciprocal", "xt.rsqrt", "xt.sigmoid", "xt.tanh", "xt.silu", "xt.itof", "xt.ftoi", "xt.matmul",
      "xt.mma", "xt.reduce_sum", "xt.reduce_max", "xt.reshape", "xt.transpose", "xt.permute"};
  return kPure.count(n) > 0;
}

void canonicalize_func(Module& m, Func& f) {
  // 1. folds: map each folded result to the value that replaces it
  std::vector<int> repl(m.values.size(), -1);
  auto resolve = [&](int id) {
    while (id >= 0 && id < static_cast<int>(repl.size()) && repl[id] >= 0) id = repl[id];
    return id;
  };
  for (Op& op : f.ops) {
    for (int& v : op.operands) v = resolve(v);
    if ((op.name != "xt.add" && op.name != "xt.sub") || op.operands.size() != 2 || op.results.size() != 1)
      continue;
    const int res = op.results[0];
    const Type& rt = m.value(res).type;
    int keep = -1;
    if (is_zero_splat(m, f, op.operands[1]))
      keep = op.operands[0];
    else if (op.name == "xt.add" && is_zero_splat(m, f, op.operands[0]))
      keep = op.operands[1];
    // the replacement must be usable in place of the result: same type
    if (keep >= 0 && m.value(keep).type == rt) repl[res] = keep;
  }
  for (int& v : f.returned) v = resolve(v);
  for (Op& op : f.ops)
    if (op.name == "func.return" || op.name == "return") op.operands = f.returned;

  // 2. erase ops whose results are all unused, when they have no side effects
  //    (folded ops are unused now); repeat until nothing changes
  bool changed = true;
  while (changed) {
    changed = false;
    std::vector<int> uses(m.values.size(), 0);
    for (const Op& op : f.ops)
      for (int v : op.operands) ++uses[v];
    std::vector<Op> kept;
    kept.reserve(f.ops.size());
    for (Op& op : f.ops) {
      bool dead = is_pure(op.name) && !op.results.empty() &&
                  std::all_of(op.results.begin(), op.results.end(), [&](int r) { return uses[r] == 0; });
      if (dead) {
        changed = true;
        for (int r : op.results) m.values[r].def_op = -1;  // no longer defined (and unused)
      } else
        kept.push_back(std::move(op));
    }
    f.ops = std::move(kept);
  }
  for (size_t i = 0; i < f.ops.size(); ++i)
    for (int r : f.ops[i].results) m.values[r].def_op = static_cast<int>(i);
}

}  // namespace

void canonicalize_module(Module& m) {
  for (Func& f : m.funcs) canonicalize_func(m, f);
}

}  // namespace xt
