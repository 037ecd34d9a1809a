// Printing of the xt IR, and the grid-unrolling stage dump.
#include <sstream>
#include <tuple>

#include "ir.h"

namespace xt {
namespace {

std::string vname(const Module& m, int id) { return "%" + m.value(id).name; }

std::string attr_dict(const AttrList& attrs) {
  std::string s = "{";
  for (size_t k = 0; k < attrs.size(); ++k) {
    if (k) s += ", ";
    s += attrs[k].first;
    if (!(attrs[k].second.kind == Attr::Text && attrs[k].second.text == "unit"))
      s += " = " + attrs[k].second.str();
  }
  return s + "}";
}

void print_op(std::ostringstream& os, const Module& m, const Op& op, const std::string& indent) {
  const std::string& n = op.name;
  if (n == "func.return" || n == "return") {
    os << indent << "func.return";
    if (!op.operands.empty()) {
      os << " ";
      for (size_t k = 0; k < op.operands.size(); ++k) os << (k ? ", " : "") << vname(m, op.operands[k]);
      os << " : ";
      for (size_t k = 0; k < op.operands.size(); ++k)
        os << (k ? ", " : "") << m.value(op.operands[k]).type.str();
    }
    os << "\n";
    return;
  }
  if (n == "cf.br" || n == "cf.cond_br") {
    os << indent << n << "\n";
    return;
  }
  os << indent;
  if (!op.results.empty()) {
    if (!op.group_name.empty()) {
      os << "%" << op.group_name << ":" << op.results.size();
    } else {
      for (size_t k = 0; k < op.results.size(); ++k) os << (k ? ", " : "") << vname(m, op.results[k]);
    }
    os << " = ";
  }
  if (n == "xt.get_tile_block_id") {
    os << n << " : ";
    for (size_t k = 0; k < op.result_types.size(); ++k) os << (k ? ", " : "") << op.result_types[k].str();
    os << "\n";
    return;
  }
  if (n == "arith.constant") {
    const Type& t = op.result_types[0];
    if (op.is_dense) {
      char buf[64];
      snprintf(buf, sizeof buf, "%.6e", op.fvalue);
      os << "arith.constant dense<" << buf << "> : " << t.str() << "\n";
    } else if (t.kind == Type::Scalar && elem_is_float(t.elem)) {
      char buf[64];
      snprintf(buf, sizeof buf, "%.6e", op.fvalue);
      os << "arith.constant " << buf << " : " << t.str() << "\n";
    } else {
      os << "arith.constant " << op.ivalue << " : " << t.str() << "\n";
    }
    return;
  }
  os << n << "(";
  for (size_t k = 0; k < op.operands.size(); ++k) os << (k ? ", " : "") << vname(m, op.operands[k]);
  os << ")";
  if (!op.attrs.empty()) os << " " << attr_dict(op.attrs);
  os << " : ";
  bool functional = n == "xt.load" || n == "xt.store" || n == "xt.load_conv2d";
  if (functional) os << "(";
  for (size_t k = 0; k < op.operand_types.size(); ++k) os << (k ? ", " : "") << op.operand_types[k].str();
  if (functional) os << ")";
  os << " -> ";
  if (op.result_types.empty()) os << "()";
  else os << op.result_types[0].str();
  os << "\n";
}

}  // namespace

std::string print_module(const Module& m) {
  std::ostringstream os;
  os << "module";
  if (!m.attrs.empty()) os << " attributes " << attr_dict(m.attrs);
  os << " {\n";
  for (const Func& f : m.funcs) {
    os << "  func.func @" << f.name << "(";
    for (size_t k = 0; k < f.args.size(); ++k)
      os << (k ? ", " : "") << vname(m, f.args[k]) << ": " << m.value(f.args[k]).type.str();
    os << ")";
    if (!f.result_types.empty()) {
      os << " -> ";
      if (f.result_types.size() > 1) os << "(";
      for (size_t k = 0; k < f.result_types.size(); ++k) os << (k ? ", " : "") << f.result_types[k].str();
      if (f.result_types.size() > 1) os << ")";
    }
    if (!f.attrs.empty()) os << " attributes " << attr_dict(f.attrs);
    os << " {\n";
    for (const Op& op : f.ops) print_op(os, m, op, "    ");
    os << "  }\n";
  }
  os << "}\n";
  return os.str();
}

// Grid unrolling with the reference's rules (lib/xt/XTSerialize.cpp):
// requires xt.grid (:29-33), a void (:34-38, :53-58) single-block (:45-49)
// function; walks z, y, x (:68-70); a load with shared = k > 0 is emitted
// once per key (op, k == 2 ? 0 : y, z) and reused (:86-102).
std::unique_ptr<Module> serialize_module(const Module& src) {
  auto out = std::make_unique<Module>();
  out->attrs = src.attrs;
  out->module_line = src.module_line;
  for (const Func& f : src.funcs) {
    bool has_grid = false;
    std::vector<int64_t> grid = func_grid(f, &has_grid);
    std::string where = "line " + std::to_string(f.line) + ": 'func.func' op ";
    if (!has_grid) throw Error(kPassError, where + "xt-serialize requires func.func xt.grid attribute");
    if (!f.result_types.empty()) throw Error(kPassError, where + "xt-serialize only supports void functions");
    if (f.num_blocks != 1) throw Error(kPassError, where + "xt-serialize only supports single-block functions");

    Func nf;
    nf.name = f.name;
    nf.attrs = f.attrs;
    nf.line = f.line;
    std::map<int, int> argmap;
    for (int a : f.args) {
      int id = out->add_value(src.value(a).name, src.value(a).type, -1, src.value(a).arg_index);
      argmap[a] = id;
      nf.args.push_back(id);
    }
    std::map<std::tuple<int, int64_t, int64_t>, int> shared_loads;
    Type i32;
    i32.kind = Type::Scalar;
    i32.elem = Elem::I32;
    int counter = 0;
    auto fresh = [&](const std::string& base) { return base + "_" + std::to_string(counter++); };
    for (int64_t z = 0; z < grid[2]; ++z)
      for (int64_t y = 0; y < grid[1]; ++y)
        for (int64_t x = 0; x < grid[0]; ++x) {
          std::map<int, int> vmap(argmap);
          int64_t coord[3] = {x, y, z};
          int bconst[3];
          for (int d = 0; d < 3; ++d) {
            Op c;
            c.name = "arith.constant";
            c.ivalue = coord[d];
            c.result_types = {i32};
            bconst[d] = out->add_value(fresh("c" + std::to_string(coord[d]) + "_i32"), i32,
                                       static_cast<int>(nf.ops.size()));
            c.results = {bconst[d]};
            nf.ops.push_back(c);
          }
          for (size_t oi = 0; oi < f.ops.size(); ++oi) {
            const Op& op = f.ops[oi];
            if (op.name == "xt.get_tile_block_id") {
              for (int d = 0; d < 3; ++d) vmap[op.results[d]] = bconst[d];
              continue;
            }
            if (op.name == "func.return" || op.name == "return") continue;
            if (op.name == "xt.load") {
              const Attr* sh = find_attr(op.attrs, "shared");
              if (sh && sh->kind == Attr::Int && sh->i > 0) {
                auto key = std::make_tuple(static_cast<int>(oi), sh->i == 2 ? 0 : y, z);
                auto it = shared_loads.find(key);
                if (it != shared_loads.end()) {
                  vmap[op.results[0]] = it->second;
                  continue;
                }
              }
            }
            Op c = op;
            c.operands.clear();
            for (int v : op.operands) c.operands.push_back(vmap.at(v));
            c.results.clear();
            c.group_name.clear();
            for (size_t r = 0; r < op.results.size(); ++r) {
              int id = out->add_value(fresh(src.value(op.results[r]).name), src.value(op.results[r]).type,
                                      static_cast<int>(nf.ops.size()));
              vmap[op.results[r]] = id;
              c.results.push_back(id);
            }
            if (op.name == "xt.load") {
              const Attr* sh = find_attr(op.attrs, "shared");
              if (sh && sh->kind == Attr::Int && sh->i > 0)
                shared_loads[std::make_tuple(static_cast<int>(oi), sh->i == 2 ? 0 : y, z)] = c.results[0];
            }
            nf.ops.push_back(c);
          }
        }
    Op ret;
    ret.name = "func.return";
    nf.ops.push_back(ret);
    out->funcs.push_back(std::move(nf));
  }
  return out;
}

}  // namespace xt
