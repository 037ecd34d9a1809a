// In-memory form of an xt-dialect module, and the front-end passes over it.
//
// The reference keeps xt programs in MLIR (include/xt/XTOps.td:15-170).  This
// runtime has no MLIR: the text the DSL prints (and the lit-test syntax of
// the reference's test/xt/*.mlir) is parsed into the small SSA form below.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace xt {

enum class Elem { F32, BF16, F16, I8, I32, I64, I1, Index, Unknown };

const char* elem_name(Elem e);
int elem_bytes(Elem e);
bool elem_is_float(Elem e);
bool elem_is_int(Elem e);

struct Type {
  enum Kind { Tensor, MemRef, Scalar, None } kind = None;
  std::vector<int64_t> shape;
  Elem elem = Elem::Unknown;

  bool operator==(const Type& o) const {
    return kind == o.kind && shape == o.shape && elem == o.elem;
  }
  bool operator!=(const Type& o) const { return !(*this == o); }
  int rank() const { return static_cast<int>(shape.size()); }
  int64_t numel() const;
  std::string str() const;
};

// Attribute values that occur in xt programs.
struct Attr {
  enum Kind { Int, IntArray, Float, Text } kind = Int;
  int64_t i = 0;
  std::string int_type = "i64";          // printed suffix of Int ("i64", "i32")
  std::vector<int64_t> arr;
  std::string arr_type = "i64";          // "i64"/"i32" for array<iN: ...>, "" for [a, b]
  double f = 0.0;
  std::string text;
  std::string str() const;
};

using AttrList = std::vector<std::pair<std::string, Attr>>;
const Attr* find_attr(const AttrList& attrs, const std::string& name);

struct Value {
  std::string name;       // printed name without '%', e.g. "x2" or "bid#0"
  Type type;
  int def_op = -1;        // index into Func::ops, -1 for function arguments
  int arg_index = -1;     // position in the argument list, or -1
};

struct Op {
  std::string name;               // "xt.load", "arith.constant", ...
  std::vector<int> results;       // value ids
  std::vector<int> operands;      // value ids
  AttrList attrs;
  std::vector<Type> operand_types;  // as written in the op's signature
  std::vector<Type> result_types;
  // arith.constant payload
  bool is_dense = false;
  double fvalue = 0.0;
  int64_t ivalue = 0;
  std::string group_name;         // for "%bid:3 = ..." result groups
  int line = 0;
};

struct Func {
  std::string name;
  std::vector<int> args;          // value ids
  std::vector<Type> result_types;
  AttrList attrs;
  std::vector<Op> ops;
  std::vector<int> returned;      // operands of func.return
  int num_blocks = 1;
  int line = 0;
};

struct Module {
  std::vector<Value> values;
  std::vector<Func> funcs;
  AttrList attrs;                 // attributes written on the module op
  int module_line = 0;

  int add_value(const std::string& name, const Type& t, int def_op, int arg_index = -1);
  const Value& value(int id) const { return values.at(id); }
};

// A failure carrying the diagnostic text; ``category`` selects the error
// class the C ABI reports (parse, verify, pass, unsupported, argument).
struct Error : std::runtime_error {
  int category;
  Error(int cat, const std::string& msg) : std::runtime_error(msg), category(cat) {}
};

enum ErrorCategory { kParseError = 1, kVerifyError = 2, kPassError = 3, kUnsupported = 4,
                     kArgumentError = 5, kCudaError = 6, kTypeError = 7 };

// Front-end entry points.
std::unique_ptr<Module> parse_module(const std::string& text);
void verify_module(const Module& m);            // throws Error(kVerifyError)
std::string print_module(const Module& m);
// Unrolls every function's grid the way the reference's xt-serialize pass
// does (lib/xt/XTSerialize.cpp:29-105); used for the stage dump only.
std::unique_ptr<Module> serialize_module(const Module& m);
// The xt dialect's canonicalization in place: x + 0, 0 + x and x - 0 fold to
// x (lib/xt/XTOps.cpp:395-449), then side-effect-free ops left unused are
// erased.
void canonicalize_module(Module& m);

// Grid of a function (attribute xt.grid), or {1,1,1} when absent.
std::vector<int64_t> func_grid(const Func& f, bool* present = nullptr);

}  // namespace xt
