// Parser for xt-dialect text: the function the DSL prints
// (reference xtile/dsl.py:490-620) and the generic MLIR spelling used by the
// reference's lit tests (test/xt/*.mlir): optional ``module {}`` wrapper,
// numbered values, ``%a:3`` result groups, ``dense<...>`` constants.
#include <cctype>
#include <cstdlib>
#include <sstream>

#include "ir.h"

namespace xt {

// ---------------------------------------------------------------------------
// types and helpers
// ---------------------------------------------------------------------------
const char* elem_name(Elem e) {
  switch (e) {
    case Elem::F32: return "f32";
    case Elem::BF16: return "bf16";
    case Elem::F16: return "f16";
    case Elem::I8: return "i8";
    case Elem::I32: return "i32";
    case Elem::I64: return "i64";
    case Elem::I1: return "i1";
    case Elem::Index: return "index";
    default: return "?";
  }
}

int elem_bytes(Elem e) {
  switch (e) {
    case Elem::F32: case Elem::I32: return 4;
    case Elem::BF16: case Elem::F16: return 2;
    case Elem::I8: case Elem::I1: return 1;
    case Elem::I64: case Elem::Index: return 8;
    default: return 0;
  }
}

bool elem_is_float(Elem e) { return e == Elem::F32 || e == Elem::BF16 || e == Elem::F16; }
bool elem_is_int(Elem e) {
  return e == Elem::I8 || e == Elem::I32 || e == Elem::I64 || e == Elem::I1;
}

int64_t Type::numel() const {
  int64_t n = 1;
  for (int64_t d : shape) n *= d;
  return n;
}

std::string Type::str() const {
  if (kind == Scalar) return elem_name(elem);
  if (kind == None) return "()";
  std::string s = kind == Tensor ? "tensor<" : "memref<";
  for (int64_t d : shape) s += std::to_string(d) + "x";
  return s + elem_name(elem) + ">";
}

std::string Attr::str() const {
  switch (kind) {
    case Int: return std::to_string(i) + " : " + int_type;
    case IntArray: {
      std::string s = arr_type.empty() ? "[" : "array<" + arr_type + ": ";
      for (size_t k = 0; k < arr.size(); ++k) s += (k ? ", " : "") + std::to_string(arr[k]);
      return s + (arr_type.empty() ? "]" : ">");
    }
    case Float: {
      char buf[64];
      snprintf(buf, sizeof buf, "%.6e", f);
      return buf;
    }
    default: return text;
  }
}

const Attr* find_attr(const AttrList& attrs, const std::string& name) {
  for (auto& kv : attrs)
    if (kv.first == name) return &kv.second;
  return nullptr;
}

int Module::add_value(const std::string& name, const Type& t, int def_op, int arg_index) {
  values.push_back(Value{name, t, def_op, arg_index});
  return static_cast<int>(values.size()) - 1;
}

std::vector<int64_t> func_grid(const Func& f, bool* present) {
  const Attr* a = find_attr(f.attrs, "xt.grid");
  if (present) *present = a != nullptr;
  if (!a || a->kind != Attr::IntArray) return {1, 1, 1};
  return a->arr;
}

// ---------------------------------------------------------------------------
// tokenizer
// ---------------------------------------------------------------------------
namespace {

struct Tok {
  enum Kind { Ident, ValueRef, Symbol, Label, Number, Angle, Punct, Arrow, End } kind;
  std::string text;
  int line;
};

bool ident_char(char c) { return std::isalnum(static_cast<unsigned char>(c)) || c == '_' || c == '.' || c == '$'; }

std::vector<Tok> tokenize(const std::string& src) {
  std::vector<Tok> out;
  int line = 1;
  size_t i = 0, n = src.size();
  auto fail = [&](const std::string& msg) { throw Error(kParseError, "line " + std::to_string(line) + ": " + msg); };
  while (i < n) {
    char c = src[i];
    if (c == '\n') { ++line; ++i; continue; }
    if (std::isspace(static_cast<unsigned char>(c))) { ++i; continue; }
    if (c == '/' && i + 1 < n && src[i + 1] == '/') {
      while (i < n && src[i] != '\n') ++i;
      continue;
    }
    if (c == '%') {
      size_t j = i + 1;
      while (j < n && ident_char(src[j])) ++j;
      if (j == i + 1) fail("expected a value name after '%'");
      // result groups ("%bid:3") and group members ("%bid#0")
      if (j < n && (src[j] == '#' || src[j] == ':') && j + 1 < n &&
          std::isdigit(static_cast<unsigned char>(src[j + 1]))) {
        size_t k = j + 1;
        while (k < n && std::isdigit(static_cast<unsigned char>(src[k]))) ++k;
        j = k;
      }
      out.push_back({Tok::ValueRef, src.substr(i + 1, j - i - 1), line});
      i = j;
      continue;
    }
    if (c == '@' || c == '^') {
      size_t j = i + 1;
      while (j < n && ident_char(src[j])) ++j;
      out.push_back({c == '@' ? Tok::Symbol : Tok::Label, src.substr(i + 1, j - i - 1), line});
      i = j;
      continue;
    }
    if (std::isalpha(static_cast<unsigned char>(c)) || c == '_') {
      size_t j = i;
      while (j < n && ident_char(src[j])) ++j;
      std::string word = src.substr(i, j - i);
      if (j < n && src[j] == '<') {
        // tensor<...>, memref<...>, array<...>, dense<...>: keep as one token
        int depth = 0;
        size_t k = j;
        for (; k < n; ++k) {
          if (src[k] == '<') ++depth;
          if (src[k] == '>' && --depth == 0) break;
          if (src[k] == '\n') ++line;
        }
        if (k >= n) fail("unterminated '<'");
        out.push_back({Tok::Angle, src.substr(i, k + 1 - i), line});
        i = k + 1;
        continue;
      }
      out.push_back({Tok::Ident, word, line});
      i = j;
      continue;
    }
    if (std::isdigit(static_cast<unsigned char>(c)) ||
        ((c == '-' || c == '+') && i + 1 < n && std::isdigit(static_cast<unsigned char>(src[i + 1])))) {
      size_t j = i + 1;
      while (j < n && (std::isalnum(static_cast<unsigned char>(src[j])) || src[j] == '.' ||
                       ((src[j] == '-' || src[j] == '+') && (src[j - 1] == 'e' || src[j - 1] == 'E'))))
        ++j;
      out.push_back({Tok::Number, src.substr(i, j - i), line});
      i = j;
      continue;
    }
    if (c == '-' && i + 1 < n && src[i + 1] == '>') {
      out.push_back({Tok::Arrow, "->", line});
      i += 2;
      continue;
    }
    if (std::string("(){}[],:=").find(c) != std::string::npos) {
      out.push_back({Tok::Punct, std::string(1, c), line});
      ++i;
      continue;
    }
    if (c == '"') {
      size_t j = src.find('"', i + 1);
      if (j == std::string::npos) fail("unterminated string");
      out.push_back({Tok::Ident, src.substr(i, j + 1 - i), line});
      i = j + 1;
      continue;
    }
    fail(std::string("unexpected character '") + c + "'");
  }
  out.push_back({Tok::End, "", line});
  return out;
}

Elem parse_elem(const std::string& s) {
  if (s == "f32") return Elem::F32;
  if (s == "bf16") return Elem::BF16;
  if (s == "f16") return Elem::F16;
  if (s == "i8") return Elem::I8;
  if (s == "i32") return Elem::I32;
  if (s == "i64") return Elem::I64;
  if (s == "i1") return Elem::I1;
  if (s == "index") return Elem::Index;
  return Elem::Unknown;
}

class Parser {
 public:
  explicit Parser(const std::string& text) : toks_(tokenize(text)) {}

  std::unique_ptr<Module> run() {
    mod_ = std::make_unique<Module>();
    if (peek_ident("module")) {
      mod_->module_line = cur().line;
      next();
      if (peek_ident("attributes")) {
        next();
        mod_->attrs = parse_attr_dict();
      }
      expect_punct("{");
      while (!peek_punct("}")) {
        if (cur().kind == Tok::End) fail("expected '}' to close the module");
        parse_func();
      }
      next();
    } else {
      while (cur().kind != Tok::End) parse_func();
    }
    if (cur().kind != Tok::End) fail("unexpected text after the module");
    return std::move(mod_);
  }

 private:
  std::vector<Tok> toks_;
  size_t pos_ = 0;
  std::unique_ptr<Module> mod_;
  std::map<std::string, int> scope_;

  const Tok& cur() const { return toks_[pos_]; }
  const Tok& next() { return toks_[pos_++]; }
  [[noreturn]] void fail(const std::string& msg) const {
    throw Error(kParseError, "line " + std::to_string(cur().line) + ": " + msg +
                                 (cur().kind == Tok::End ? "" : " (at '" + cur().text + "')"));
  }
  bool peek_punct(const char* p) const { return cur().kind == Tok::Punct && cur().text == p; }
  bool peek_ident(const char* w) const { return cur().kind == Tok::Ident && cur().text == w; }
  void expect_punct(const char* p) {
    if (!peek_punct(p)) fail(std::string("expected '") + p + "'");
    next();
  }
  bool accept_punct(const char* p) {
    if (!peek_punct(p)) return false;
    next();
    return true;
  }

  Type parse_type() {
    const Tok& t = cur();
    if (t.kind == Tok::Angle) {
      std::string s = t.text;
      Type ty;
      if (s.rfind("tensor<", 0) == 0) ty.kind = Type::Tensor;
      else if (s.rfind("memref<", 0) == 0) ty.kind = Type::MemRef;
      else fail("expected a tensor or memref type");
      std::string body = s.substr(7, s.size() - 8);
      size_t start = 0;
      while (true) {
        size_t x = body.find('x', start);
        std::string part = body.substr(start, x == std::string::npos ? std::string::npos : x - start);
        bool digits = !part.empty() && part.find_first_not_of("0123456789") == std::string::npos;
        if (digits && x != std::string::npos) {
          ty.shape.push_back(std::stoll(part));
          start = x + 1;
          continue;
        }
        if (part == "?" ) fail("dynamic shapes are not supported");
        ty.elem = parse_elem(body.substr(start));
        break;
      }
      if (ty.elem == Elem::Unknown) fail("unsupported element type in " + s);
      next();
      return ty;
    }
    if (t.kind == Tok::Ident) {
      Elem e = parse_elem(t.text);
      if (e == Elem::Unknown) fail("unknown type '" + t.text + "'");
      next();
      Type ty;
      ty.kind = Type::Scalar;
      ty.elem = e;
      return ty;
    }
    fail("expected a type");
  }

  std::vector<Type> parse_type_list_parens() {
    std::vector<Type> out;
    expect_punct("(");
    if (accept_punct(")")) return out;
    do out.push_back(parse_type()); while (accept_punct(","));
    expect_punct(")");
    return out;
  }

  Attr parse_attr_value() {
    Attr a;
    const Tok& t = cur();
    if (t.kind == Tok::Angle && t.text.rfind("array<", 0) == 0) {
      a.kind = Attr::IntArray;
      std::string body = t.text.substr(6, t.text.size() - 7);
      size_t colon = body.find(':');
      a.arr_type = body.substr(0, colon);
      std::stringstream ss(colon == std::string::npos ? "" : body.substr(colon + 1));
      std::string item;
      while (std::getline(ss, item, ','))
        if (item.find_first_not_of(" ") != std::string::npos) a.arr.push_back(std::stoll(item));
      next();
      return a;
    }
    if (accept_punct("[")) {
      a.kind = Attr::IntArray;
      a.arr_type = "";
      if (!accept_punct("]")) {
        do {
          if (cur().kind != Tok::Number) fail("expected an integer");
          a.arr.push_back(std::stoll(next().text));
        } while (accept_punct(","));
        expect_punct("]");
      }
      return a;
    }
    if (t.kind == Tok::Number) {
      std::string num = next().text;
      if (num.find_first_of(".eE") != std::string::npos) {
        a.kind = Attr::Float;
        a.f = std::strtod(num.c_str(), nullptr);
        if (accept_punct(":")) next();
        return a;
      }
      a.kind = Attr::Int;
      a.i = std::stoll(num);
      if (accept_punct(":")) {
        if (cur().kind != Tok::Ident) fail("expected an integer type");
        a.int_type = next().text;
      }
      return a;
    }
    if (t.kind == Tok::Ident || t.kind == Tok::Angle) {
      a.kind = Attr::Text;
      a.text = next().text;
      return a;
    }
    fail("expected an attribute value");
  }

  AttrList parse_attr_dict() {
    AttrList out;
    expect_punct("{");
    if (accept_punct("}")) return out;
    do {
      if (cur().kind != Tok::Ident) fail("expected an attribute name");
      std::string key = next().text;
      if (accept_punct("=")) out.emplace_back(key, parse_attr_value());
      else out.emplace_back(key, Attr{Attr::Text, 0, "", {}, "", 0.0, "unit"});
    } while (accept_punct(","));
    expect_punct("}");
    return out;
  }

  int lookup(const std::string& name) {
    auto it = scope_.find(name);
    if (it == scope_.end()) fail("use of undefined value '%" + name + "'");
    return it->second;
  }

  void define(const std::string& name, int id) {
    if (scope_.count(name)) fail("redefinition of SSA value '%" + name + "'");
    scope_[name] = id;
  }

  void parse_func() {
    if (!peek_ident("func.func")) fail("expected 'func.func'");
    Func f;
    f.line = cur().line;
    next();
    if (peek_ident("private") || peek_ident("public")) next();
    if (cur().kind != Tok::Symbol) fail("expected a function name");
    f.name = next().text;
    scope_.clear();
    expect_punct("(");
    if (!accept_punct(")")) {
      do {
        if (cur().kind != Tok::ValueRef) fail("expected an argument name");
        std::string name = next().text;
        expect_punct(":");
        Type t = parse_type();
        int id = mod_->add_value(name, t, -1, static_cast<int>(f.args.size()));
        define(name, id);
        f.args.push_back(id);
      } while (accept_punct(","));
      expect_punct(")");
    }
    if (cur().kind == Tok::Arrow) {
      next();
      if (peek_punct("(")) f.result_types = parse_type_list_parens();
      else f.result_types.push_back(parse_type());
    }
    if (peek_ident("attributes")) {
      next();
      f.attrs = parse_attr_dict();
    }
    expect_punct("{");
    mod_->funcs.push_back(std::move(f));
    Func& fn = mod_->funcs.back();
    while (!peek_punct("}")) {
      if (cur().kind == Tok::End) fail("expected '}' to close the function");
      parse_statement(fn);
    }
    next();
  }

  // Operands between parentheses: "(%a, %b#0, ...)".
  std::vector<int> parse_operand_list() {
    std::vector<int> ops;
    expect_punct("(");
    if (accept_punct(")")) return ops;
    do {
      if (cur().kind != Tok::ValueRef) fail("expected an SSA operand");
      ops.push_back(lookup(next().text));
    } while (accept_punct(","));
    expect_punct(")");
    return ops;
  }

  void skip_line(int line) {
    while (cur().kind != Tok::End && cur().line == line) next();
  }

  void parse_statement(Func& f) {
    int line = cur().line;
    if (cur().kind == Tok::Label) {
      // a second block: the serialize pass rejects these (XTSerialize.cpp:45-49)
      f.num_blocks++;
      next();
      if (peek_punct("(")) {
        while (!peek_punct(")")) next();
        next();
      }
      expect_punct(":");
      return;
    }
    std::vector<std::string> result_names;
    std::string group;
    int group_count = 0;
    if (cur().kind == Tok::ValueRef) {
      do {
        if (cur().kind != Tok::ValueRef) fail("expected a result name");
        std::string r = next().text;
        size_t c = r.find(':');
        if (c != std::string::npos) {
          group = r.substr(0, c);
          group_count = std::stoi(r.substr(c + 1));
        } else {
          result_names.push_back(r);
        }
      } while (accept_punct(","));
      expect_punct("=");
    }
    if (cur().kind != Tok::Ident) fail("expected an operation name");
    std::string name = next().text;
    Op op;
    op.name = name;
    op.line = line;

    if (name == "func.return" || name == "return") {
      while (cur().kind == Tok::ValueRef) {
        f.returned.push_back(lookup(next().text));
        if (!accept_punct(",")) break;
      }
      if (accept_punct(":")) {
        do parse_type(); while (accept_punct(","));
      }
      op.operands = f.returned;
      f.ops.push_back(op);
      return;
    }
    if (name == "cf.br" || name == "cf.cond_br") {
      skip_line(line);
      f.ops.push_back(op);
      return;
    }
    if (name == "xt.get_tile_block_id") {
      expect_punct(":");
      std::vector<Type> ts;
      do ts.push_back(parse_type()); while (accept_punct(","));
      op.result_types = ts;
      int idx = static_cast<int>(f.ops.size());
      if (!group.empty()) {
        if (group_count != 3) fail("xt.get_tile_block_id produces 3 results");
        op.group_name = group;
        for (int k = 0; k < 3; ++k) {
          std::string nm = group + "#" + std::to_string(k);
          int id = mod_->add_value(nm, ts.at(std::min<size_t>(k, ts.size() - 1)), idx);
          define(nm, id);
          op.results.push_back(id);
        }
      } else {
        if (result_names.size() != 3) fail("xt.get_tile_block_id produces 3 results");
        for (int k = 0; k < 3; ++k) {
          int id = mod_->add_value(result_names[k], ts.at(std::min<size_t>(k, ts.size() - 1)), idx);
          define(result_names[k], id);
          op.results.push_back(id);
        }
      }
      f.ops.push_back(op);
      return;
    }
    if (name == "arith.constant") {
      if (cur().kind == Tok::Angle && cur().text.rfind("dense<", 0) == 0) {
        std::string body = cur().text.substr(6, cur().text.size() - 7);
        op.is_dense = true;
        if (body == "true") op.fvalue = 1;
        else if (body == "false") op.fvalue = 0;
        else op.fvalue = std::strtod(body.c_str(), nullptr);
        next();
      } else if (cur().kind == Tok::Number) {
        std::string num = next().text;
        op.fvalue = std::strtod(num.c_str(), nullptr);
        op.ivalue = std::strtoll(num.c_str(), nullptr, 10);
      } else {
        fail("expected a constant value");
      }
      expect_punct(":");
      Type t = parse_type();
      op.result_types = {t};
      finish_results(f, op, result_names, 1);
      return;
    }
    if (name.rfind("xt.", 0) != 0) fail("custom op '" + name + "' is unknown");

    static const char* kFunctional[] = {"xt.load", "xt.store", "xt.load_conv2d"};
    bool functional = false;
    for (const char* k : kFunctional) functional |= name == k;
    static const char* kKnown[] = {
        "xt.load", "xt.store", "xt.load_conv2d", "xt.add", "xt.sub", "xt.mul", "xt.exp",
        "xt.cos", "xt.sin", "xt.reciprocal", "xt.rsqrt", "xt.sigmoid", "xt.tanh", "xt.silu",
        "xt.itof", "xt.ftoi", "xt.matmul", "xt.mma", "xt.reduce_sum", "xt.reduce_max",
        "xt.reshape", "xt.transpose", "xt.permute"};
    bool known = false;
    for (const char* k : kKnown) known |= name == k;
    if (!known) fail("custom op '" + name + "' is unknown");

    op.operands = parse_operand_list();
    if (peek_punct("{")) op.attrs = parse_attr_dict();
    expect_punct(":");
    if (functional) {
      op.operand_types = parse_type_list_parens();
      if (cur().kind != Tok::Arrow) fail("expected '->'");
      next();
      if (peek_punct("(")) op.result_types = parse_type_list_parens();
      else op.result_types.push_back(parse_type());
    } else {
      do op.operand_types.push_back(parse_type()); while (accept_punct(","));
      if (cur().kind != Tok::Arrow) fail("expected '->'");
      next();
      op.result_types.push_back(parse_type());
    }
    if (op.operand_types.size() != op.operands.size())
      fail("'" + name + "' op has " + std::to_string(op.operands.size()) +
           " operands but its signature lists " + std::to_string(op.operand_types.size()) + " types");
    for (size_t k = 0; k < op.operands.size(); ++k) {
      if (mod_->values[op.operands[k]].type != op.operand_types[k])
        fail("use of value '%" + mod_->values[op.operands[k]].name + "' expects type " +
             op.operand_types[k].str() + " but it has type " + mod_->values[op.operands[k]].type.str());
    }
    finish_results(f, op, result_names, name == "xt.store" ? 0 : 1);
  }

  void finish_results(Func& f, Op& op, const std::vector<std::string>& names, size_t expected) {
    if (names.size() != expected)
      fail("'" + op.name + "' produces " + std::to_string(expected) + " result(s)");
    int idx = static_cast<int>(f.ops.size());
    for (size_t k = 0; k < names.size(); ++k) {
      int id = mod_->add_value(names[k], op.result_types.at(k), idx);
      define(names[k], id);
      op.results.push_back(id);
    }
    f.ops.push_back(op);
  }
};

}  // namespace

std::unique_ptr<Module> parse_module(const std::string& text) {
  Parser p(text);
  return p.run();
}

}  // namespace xt
