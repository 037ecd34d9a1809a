// Op verifiers for the xt dialect.  The rules and the diagnostic wording
// follow the reference's lib/xt/XTOps.cpp (cited per rule) and the xt.grid
// attribute check of lib/xt/XTDialect.cpp:18-36, so that programs the
// reference rejects are rejected here with the same message.  The two
// bfloat16 extensions (matmul and load_conv2d on bf16 operands) are marked.
#include <algorithm>
#include <set>

#include "ir.h"

namespace xt {
namespace {

struct Checker {
  const Module& m;
  const Func& f;
  const Op& op;

  [[noreturn]] void fail(const std::string& msg) const {
    throw Error(kVerifyError, "line " + std::to_string(op.line) + ": '" + op.name + "' op " + msg);
  }
  const Type& in(size_t k) const { return op.operand_types.at(k); }
  const Type& out(size_t k = 0) const { return op.result_types.at(k); }
  bool is_tensor(const Type& t) const { return t.kind == Type::Tensor; }
};

bool is_coord(const Type& t) {
  return t.kind == Type::Scalar && (t.elem == Elem::I32 || t.elem == Elem::Index);
}

// verifyMemRefAndTensor (XTOps.cpp:14-25)
void memref_and_tensor(const Checker& c, const Type& mem, const Type& ten) {
  if (mem.kind != Type::MemRef) c.fail("requires a ranked memref operand");
  if (ten.kind != Type::Tensor) c.fail("requires a statically shaped tensor");
  if (mem.rank() != ten.rank()) c.fail("memref rank must match tensor rank");
  if (mem.elem != ten.elem) c.fail("requires matching memref/tensor element types");
}

void verify_load(const Checker& c) {  // LoadOp::verify (XTOps.cpp:27-41)
  const Type& res = c.out();
  if (!c.is_tensor(res)) c.fail("requires a ranked tensor result");
  size_t ncoords = c.op.operands.size() - 1;
  if (ncoords == 0) c.fail("requires at least one coordinate");
  if (const Attr* s = find_attr(c.op.attrs, "shared"))
    if (s->kind != Attr::Int || (s->i != 0 && s->i != 1 && s->i != 2))
      c.fail("shared attribute must be 0, 1, or 2");
  if (static_cast<int>(ncoords) != res.rank()) c.fail("coordinate count must match tensor rank");
  for (size_t k = 1; k < c.op.operands.size(); ++k)
    if (!is_coord(c.in(k))) c.fail("coordinates must be i32 or index values");
  memref_and_tensor(c, c.in(0), res);
}

void verify_store(const Checker& c) {  // StoreOp::verify (XTOps.cpp:92-102)
  const Type& val = c.in(0);
  if (!c.is_tensor(val)) c.fail("requires a ranked tensor operand");
  size_t ncoords = c.op.operands.size() - 2;
  if (c.op.operands.size() < 2 || ncoords == 0) c.fail("requires at least one coordinate");
  if (static_cast<int>(ncoords) != val.rank()) c.fail("coordinate count must match tensor rank");
  for (size_t k = 2; k < c.op.operands.size(); ++k)
    if (!is_coord(c.in(k))) c.fail("coordinates must be i32 or index values");
  memref_and_tensor(c, c.in(1), val);
}

void verify_load_conv2d(const Checker& c) {  // LoadConv2DOp::verify (XTOps.cpp:43-90)
  if (c.op.operands.size() != 6) c.fail("expects a source, a filter and 4 coordinates");
  const Type& mem = c.in(0);
  const Type& filt = c.in(1);
  const Type& res = c.out();
  if (mem.kind != Type::MemRef) c.fail("requires a ranked memref source operand");
  if (!c.is_tensor(filt) || !c.is_tensor(res)) c.fail("requires ranked tensor filter operand and result");
  if (mem.rank() != 4 || filt.rank() != 4 || res.rank() != 4)
    c.fail("requires rank-4 source, filter, and result types");
  const Attr* pad = find_attr(c.op.attrs, "pad");
  const Attr* stride = find_attr(c.op.attrs, "stride");
  const Attr* dil = find_attr(c.op.attrs, "dilation");
  if (!pad || pad->kind != Attr::IntArray || pad->arr.size() != 4)
    c.fail("pad attribute must have exactly 4 entries");
  if (!stride || stride->kind != Attr::IntArray || stride->arr.size() != 2)
    c.fail("stride attribute must have exactly 2 entries");
  if (!dil || dil->kind != Attr::IntArray || dil->arr.size() != 2)
    c.fail("dilation attribute must have exactly 2 entries");
  if (const Attr* g = find_attr(c.op.attrs, "group"))
    if (g->kind != Attr::Int || g->i <= 0) c.fail("group attribute must be positive");
  for (int64_t p : pad->arr)
    if (p < 0) c.fail("pad attribute entries must be non-negative");
  for (int64_t s : stride->arr)
    if (s <= 0) c.fail("stride attribute entries must be positive");
  for (int64_t d : dil->arr)
    if (d <= 0) c.fail("dilation attribute entries must be positive");
  // i8 per the reference; bf16 source+filter is this backend's extension
  bool i8 = mem.elem == Elem::I8 && filt.elem == Elem::I8;
  bool bf16 = mem.elem == Elem::BF16 && filt.elem == Elem::BF16;
  if (!i8 && !bf16) c.fail("load_conv2d requires i8 source and filter element types");
  if (res.elem != Elem::F32 && res.elem != Elem::BF16)
    c.fail("load_conv2d requires f32 or bf16 result element type");
  if (mem.shape[3] != filt.shape[2])
    c.fail("load_conv2d requires source and filter channel dimensions to match");
  if (res.shape[3] > filt.shape[3])
    c.fail("load_conv2d result channel dimension must not exceed filter output channels");
  for (size_t k = 2; k < 6; ++k)
    if (!is_coord(c.in(k))) c.fail("coordinates must be i32 or index values");
}

// computeBroadcastShape + verifyBroadcastableTensorTypes (XTOps.cpp:104-144)
void verify_broadcast(const Checker& c) {
  const Type& l = c.in(0);
  const Type& r = c.in(1);
  const Type& res = c.out();
  if (!c.is_tensor(l) || !c.is_tensor(r) || !c.is_tensor(res))
    c.fail("requires ranked tensor operands and result");
  if (l.elem != r.elem || l.elem != res.elem)
    c.fail("requires operand and result element types to match");
  int rank = std::max(l.rank(), r.rank());
  std::vector<int64_t> shape(rank, 1);
  for (int i = 0; i < rank; ++i) {
    int li = l.rank() - 1 - i, ri = r.rank() - 1 - i;
    int64_t ld = li >= 0 ? l.shape[li] : 1;
    int64_t rd = ri >= 0 ? r.shape[ri] : 1;
    if (ld != rd && ld != 1 && rd != 1)
      c.fail("operands are not broadcast-compatible with result tensor type");
    shape[rank - 1 - i] = std::max(ld, rd);
  }
  if (shape != res.shape) c.fail("operands are not broadcast-compatible with result tensor type");
}

void verify_same_unary(const Checker& c) {  // verifySameUnaryTensorTypes (XTOps.cpp:146-157)
  if (!c.is_tensor(c.in(0)) || !c.is_tensor(c.out()))
    c.fail("requires ranked tensor operand and result");
  if (c.in(0) != c.out()) c.fail("requires operand and result tensor types to match");
}

void verify_cast(const Checker& c, bool int_to_float) {  // verifyTensorCastTypes (XTOps.cpp:159-183)
  if (!c.is_tensor(c.in(0)) || !c.is_tensor(c.out()))
    c.fail("requires ranked tensor operand and result");
  if (c.in(0).shape != c.out().shape) c.fail("requires operand and result tensor shapes to match");
  if (int_to_float) {
    if (!elem_is_int(c.in(0).elem) || !elem_is_float(c.out().elem))
      c.fail("requires integer input and floating-point result element types");
  } else {
    if (!elem_is_float(c.in(0).elem) || !elem_is_int(c.out().elem))
      c.fail("requires floating-point input and integer result element types");
  }
}

// verifyMatmulLikeShape (XTOps.cpp:222-235)
void matmul_shape(const Checker& c, const Type& l, const Type& r, const Type& res) {
  if (!c.is_tensor(l) || !c.is_tensor(r) || !c.is_tensor(res))
    c.fail("requires ranked tensor operands and result");
  if (l.rank() != 2 || r.rank() != 2 || res.rank() != 2) c.fail("requires rank-2 tensors");
  if (l.shape[1] != r.shape[0])
    c.fail("matmul requires lhs inner dimension to match rhs outer dimension");
  if (res.shape[0] != l.shape[0] || res.shape[1] != r.shape[1])
    c.fail("result shape must match matmul output shape");
}

void verify_matmul(const Checker& c) {  // MatmulOp::verify (XTOps.cpp:237-253)
  const Type &l = c.in(0), &r = c.in(1), &res = c.out();
  matmul_shape(c, l, r, res);
  if (l.elem == r.elem && l.elem == res.elem) return;
  if (l.elem == Elem::I8 && r.elem == Elem::I8 && (res.elem == Elem::F32 || res.elem == Elem::BF16))
    return;
  // extension: bf16 x bf16 accumulates into f32
  if (l.elem == Elem::BF16 && r.elem == Elem::BF16 && res.elem == Elem::F32) return;
  c.fail("requires matching element types or i8 inputs with f32/bf16 result");
}

void verify_mma(const Checker& c) {  // MMAOp::verify (XTOps.cpp:255-272)
  const Type &l = c.in(0), &r = c.in(1), &acc = c.in(2), &res = c.out();
  matmul_shape(c, l, r, res);
  if (!c.is_tensor(acc) || acc.rank() != 2) c.fail("requires a rank-2 statically shaped accumulator");
  if (acc != res) c.fail("accumulator and result tensor types must match");
  if (l.elem != Elem::I8 || r.elem != Elem::I8) c.fail("mma requires i8 input tensors");
  if (acc.elem != Elem::F32 && acc.elem != Elem::BF16)
    c.fail("mma requires f32 or bf16 accumulator and result tensors");
}

void verify_reduce(const Checker& c) {  // verifyLastDimReductionShape (XTOps.cpp:274-299)
  const Type &in = c.in(0), &res = c.out();
  if (!c.is_tensor(in) || !c.is_tensor(res)) c.fail("requires ranked tensor operand and result");
  if (in.elem != res.elem) c.fail("requires operand and result element types to match");
  if (in.rank() != res.rank()) c.fail("requires operand and result ranks to match");
  if (in.rank() != 2) c.fail("reduce currently supports rank-2 tensors only");
  const Attr* a = find_attr(c.op.attrs, "axis");
  if (!a || a->kind != Attr::Int) c.fail("requires an integer axis attribute");
  int64_t rank = in.rank();
  if (a->i < -rank || a->i >= rank) c.fail("axis must be in range [-rank, rank)");
  int64_t axis = a->i >= 0 ? a->i : a->i + rank;
  for (int64_t i = 0; i < rank; ++i) {
    int64_t expect = i == axis ? 1 : in.shape[i];
    if (res.shape[i] != expect)
      c.fail("reduce result shape must match input shape except for the reduced dimension, "
             "which must be 1");
  }
}

void verify_reshape(const Checker& c) {  // ReshapeOp::verify (XTOps.cpp:360-372)
  const Type &in = c.in(0), &res = c.out();
  if (!c.is_tensor(in) || !c.is_tensor(res)) c.fail("requires ranked tensor operand and result");
  if (in.elem != res.elem) c.fail("requires operand and result element types to match");
  if (in.numel() != res.numel())
    c.fail("reshape requires operand and result to have the same number of elements");
}

void verify_transpose(const Checker& c) {  // verifyTransposeShape (XTOps.cpp:301-319)
  const Type &in = c.in(0), &res = c.out();
  if (!c.is_tensor(in) || !c.is_tensor(res)) c.fail("requires ranked tensor operand and result");
  if (in.elem != res.elem) c.fail("requires operand and result element types to match");
  if (in.rank() != 3 || res.rank() != 3) c.fail("transpose requires rank-3 operand and result tensors");
  if (in.shape[0] != res.shape[0] || in.shape[1] != res.shape[2] || in.shape[2] != res.shape[1])
    c.fail("transpose result shape must preserve dim 0 and swap dims 1 and 2");
}

void verify_permute(const Checker& c) {  // verifyPermuteShape (XTOps.cpp:321-351)
  const Type &in = c.in(0), &res = c.out();
  if (!c.is_tensor(in) || !c.is_tensor(res)) c.fail("requires ranked tensor operand and result");
  if (in.elem != res.elem) c.fail("requires operand and result element types to match");
  if (in.rank() != res.rank()) c.fail("requires operand and result ranks to match");
  const Attr* p = find_attr(c.op.attrs, "permutation");
  if (!p || p->kind != Attr::IntArray) c.fail("requires a permutation attribute");
  if (static_cast<int>(p->arr.size()) != in.rank())
    c.fail("permutation attribute length must match tensor rank");
  std::vector<bool> seen(in.rank(), false);
  for (int64_t d : p->arr) {
    if (d < 0 || d >= in.rank()) c.fail("permutation entries must be in range [0, rank)");
    if (seen[d]) c.fail("permutation attribute must contain each dimension exactly once");
    seen[d] = true;
  }
  for (int i = 0; i < in.rank(); ++i)
    if (res.shape[i] != in.shape[p->arr[i]])
      c.fail("permute result shape must match the input shape reordered by permutation");
}

void verify_grid_attr(const Func& f) {  // XTDialect::verifyOperationAttribute (XTDialect.cpp:18-36)
  const Attr* g = find_attr(f.attrs, "xt.grid");
  if (!g) return;
  std::string where = "line " + std::to_string(f.line) + ": 'func.func' op ";
  if (g->kind != Attr::IntArray || g->arr_type != "i32")
    throw Error(kVerifyError, where + "xt.grid must be a dense i32 array attribute");
  if (g->arr.size() != 3) throw Error(kVerifyError, where + "xt.grid must have exactly 3 entries");
  for (int64_t d : g->arr)
    if (d <= 0) throw Error(kVerifyError, where + "xt.grid entries must be positive");
}

}  // namespace

void verify_module(const Module& m) {
  if (find_attr(m.attrs, "xt.grid"))
    throw Error(kVerifyError, "line " + std::to_string(m.module_line) +
                                  ": 'builtin.module' op xt.grid is only valid on func.func operations");
  for (const Func& f : m.funcs) {
    verify_grid_attr(f);
    for (const Op& op : f.ops) {
      Checker c{m, f, op};
      const std::string& n = op.name;
      if (n == "xt.load") verify_load(c);
      else if (n == "xt.store") verify_store(c);
      else if (n == "xt.load_conv2d") verify_load_conv2d(c);
      else if (n == "xt.add" || n == "xt.sub" || n == "xt.mul") verify_broadcast(c);
      else if (n == "xt.itof") verify_cast(c, true);
      else if (n == "xt.ftoi") verify_cast(c, false);
      else if (n == "xt.matmul") verify_matmul(c);
      else if (n == "xt.mma") verify_mma(c);
      else if (n == "xt.reduce_sum" || n == "xt.reduce_max") verify_reduce(c);
      else if (n == "xt.reshape") verify_reshape(c);
      else if (n == "xt.transpose") verify_transpose(c);
      else if (n == "xt.permute") verify_permute(c);
      else if (n.rfind("xt.", 0) == 0 && n != "xt.get_tile_block_id") verify_same_unary(c);
    }
  }
}

}  // namespace xt
