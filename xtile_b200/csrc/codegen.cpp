// Source generation for the per-program ew, rows and tile kernels
// (codegen.h).
//
// For ew and rows programs the generated text is the register program of
// plan.h written out: every program register becomes a local variable (an
// array of float4 groups in the vector kernels), every instruction one
// statement applying the op_math.cuh function, whose text is embedded at the
// top of each source.  The semantics are those of the register program, op
// for op; nothing is decoded or dispatched per element and the values stay
// in registers.  Tile programs are written out op by op over shared-memory
// slots (below).
#include "codegen.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <set>
#include <sstream>
#include <vector>

#include "ir.h"

namespace xt {
namespace jit {
namespace {

// op_math.cuh's text (written into the build directory by the build)
const char kOpMath[] =
#include "op_math_src.inc"
    ;

const char kHelpers[] = R"XTSRC(
typedef long long xt_i64;
#define XT_MAP1(f, a) make_float4(f((a).x), f((a).y), f((a).z), f((a).w))
#define XT_MAP2(f, a, b) make_float4(f((a).x, (b).x), f((a).y, (b).y), f((a).z, (b).z), f((a).w, (b).w))
#define XT_MAP2S(f, a, s) make_float4(f((a).x, s), f((a).y, s), f((a).z, s), f((a).w, s))
// programmatic dependent launch: let the next launch start its set-up, then
// wait for the previous one before touching global memory
__device__ __forceinline__ void xt_pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void xt_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// four consecutive elements as f32 values, at an element index that is a
// multiple of 4 of an aligned array (one 16-, 8- or 4-byte access)
__device__ __forceinline__ float4 xt_ld4_f32(const void* p, xt_i64 i) {
  return __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i));
}
__device__ __forceinline__ float4 xt_ld4_f32_kept(const void* p, xt_i64 i) {  // a broadcast row: read again
  return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i));
}
__device__ __forceinline__ float4 xt_ld4_bf16(const void* p, xt_i64 i) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const unsigned short*>(p) + i));
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xffff0000u));
}
__device__ __forceinline__ float4 xt_ld4_i8(const void* p, xt_i64 i) {
  const unsigned int w = __ldg(reinterpret_cast<const unsigned int*>(static_cast<const signed char*>(p) + i));
  return make_float4(static_cast<float>(static_cast<signed char>(w)), static_cast<float>(static_cast<signed char>(w >> 8)),
                     static_cast<float>(static_cast<signed char>(w >> 16)),
                     static_cast<float>(static_cast<signed char>(w >> 24)));
}
__device__ __forceinline__ void xt_st4_f32(void* p, xt_i64 i, float4 v) {
  __stcs(reinterpret_cast<float4*>(static_cast<float*>(p) + i), v);
}
__device__ __forceinline__ void xt_st4_bf16(void* p, xt_i64 i, float4 v) {
  *reinterpret_cast<uint2*>(static_cast<unsigned short*>(p) + i) =
      make_uint2(xt_f32_to_bf16_bits(v.x) | (xt_f32_to_bf16_bits(v.y) << 16),
                 xt_f32_to_bf16_bits(v.z) | (xt_f32_to_bf16_bits(v.w) << 16));
}
__device__ __forceinline__ void xt_st4_i8(void* p, xt_i64 i, float4 v) {
  *reinterpret_cast<unsigned int*>(static_cast<signed char*>(p) + i) =
      xt_f32_to_i8_bits(v.x) | (xt_f32_to_i8_bits(v.y) << 8) | (xt_f32_to_i8_bits(v.z) << 16) |
      (xt_f32_to_i8_bits(v.w) << 24);
}
// one element
__device__ __forceinline__ float xt_ld1_f32(const void* p, xt_i64 i) { return __ldg(static_cast<const float*>(p) + i); }
__device__ __forceinline__ float xt_ld1_f32_kept(const void* p, xt_i64 i) { return __ldg(static_cast<const float*>(p) + i); }
__device__ __forceinline__ float xt_ld1_bf16(const void* p, xt_i64 i) {
  return xt_bf16_bits_to_f32(__ldg(static_cast<const unsigned short*>(p) + i));
}
__device__ __forceinline__ float xt_ld1_i8(const void* p, xt_i64 i) {
  return static_cast<float>(__ldg(static_cast<const signed char*>(p) + i));
}
__device__ __forceinline__ void xt_st1_f32(void* p, xt_i64 i, float v) { static_cast<float*>(p)[i] = v; }
__device__ __forceinline__ void xt_st1_bf16(void* p, xt_i64 i, float v) {
  static_cast<unsigned short*>(p)[i] = static_cast<unsigned short>(xt_f32_to_bf16_bits(v));
}
__device__ __forceinline__ void xt_st1_i8(void* p, xt_i64 i, float v) {
  static_cast<unsigned char*>(p)[i] = static_cast<unsigned char>(xt_f32_to_i8_bits(v));
}
__device__ __forceinline__ float xt_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float xt_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
)XTSRC";

const char* unary_fn(uint8_t op) {
  switch (op & 0x7f) {
    case kExp: return "xt_exp";
    case kCos: return "xt_cos";
    case kSin: return "xt_sin";
    case kRecip: return "xt_recip";
    case kRsqrt: return "xt_rsqrt";
    case kSigmoid: return "xt_sigmoid";
    case kTanh: return "xt_tanh";
    case kSilu: return "xt_silu";
    case kItof: return "xt_itof";
    case kFtoi: return "xt_ftoi";
    default: return nullptr;
  }
}

const char* binary_fn(uint8_t op) {
  switch (op & 0x7f) {
    case kAdd: case kBcastAdd: return "xt_add";
    case kSub: case kBcastSub: return "xt_sub";
    case kMul: case kBcastMul: return "xt_mul";
    default: return nullptr;
  }
}

const char* elem_suffix(uint8_t e) { return e == dev::kF32 ? "f32" : e == dev::kBF16 ? "bf16" : "i8"; }

bool is_binary(uint8_t op) {
  const uint8_t o = op & 0x7f;
  return o == kAdd || o == kSub || o == kMul;
}

void fail(const std::string& msg) { throw Error(kUnsupported, "code generation: " + msg); }

// the ew program on one element i (scalar registers)
void ew_scalar_body(std::ostringstream& s, const dev::EwArgs& a, const std::set<int>& regs, const char* ind) {
  s << ind << "float";
  bool first = true;
  for (int r : regs) s << (first ? " r" : ", r") << r, first = false;
  s << ";\n";
  for (int pc = 0; pc < a.n_code; ++pc) {
    const Instr& in = a.code[pc];
    if (in.op == kLoad) {
      const bool b = a.in_bcast[in.a];
      s << ind << "r" << int(in.dst) << " = xt_ld1_" << elem_suffix(a.in_elem[in.a]) << (b && a.in_elem[in.a] == dev::kF32 ? "_kept" : "")
        << "(p.in[" << int(in.a) << "], " << (b ? "i % p.period" : "i") << ");\n";
    } else if (in.op == kStore) {
      s << ind << "xt_st1_" << elem_suffix(a.out_elem[in.dst]) << "(p.out[" << int(in.dst) << "], i, r" << int(in.a)
        << ");\n";
    } else if (is_binary(in.op)) {
      s << ind << "r" << int(in.dst) << " = " << binary_fn(in.op) << "(r" << int(in.a) << ", r" << int(in.b) << ");\n";
    } else if (unary_fn(in.op)) {
      s << ind << "r" << int(in.dst) << " = " << unary_fn(in.op) << "(r" << int(in.a) << ");\n";
    } else {
      fail("opcode " + std::to_string(in.op) + " in an elementwise program");
    }
  }
}

}  // namespace

std::string ew_source(const dev::EwArgs& a) {
  if (a.n_code <= 0 || a.n_code > kMaxInstr) fail("elementwise program length");
  std::set<int> regs;
  bool bcast = false;
  for (int pc = 0; pc < a.n_code; ++pc) {
    const Instr& in = a.code[pc];
    if (in.op != kStore) regs.insert(in.dst);
    if (in.op == kLoad) bcast = bcast || a.in_bcast[in.a];
  }
  std::ostringstream s;
  s << kOpMath << kHelpers;
  s << "#define XT_NV " << kEwVec << "\n";
  s << "struct XtEwArgs { const void* in[" << kMaxSlots << "]; void* out[" << kMaxSlots
    << "]; xt_i64 begin, end, period; };\n";
  // one element: the any-alignment kernel and the vector kernel's tail
  s << "__device__ __forceinline__ void xt_ew_elem(const XtEwArgs& p, xt_i64 i) {\n";
  ew_scalar_body(s, a, regs, "  ");
  s << "}\n";
  s << "extern \"C\" __global__ void __launch_bounds__(" << kEwThreads << ") xt_ew_s(const XtEwArgs p) {\n"
       "  xt_pdl_launch();\n  xt_pdl_wait();\n"
       "  const xt_i64 stride = static_cast<xt_i64>(gridDim.x) * blockDim.x;\n"
       "  for (xt_i64 i = p.begin + static_cast<xt_i64>(blockIdx.x) * blockDim.x + threadIdx.x; i < p.end; i += stride)\n"
       "    xt_ew_elem(p, i);\n}\n";
  // 4 * XT_NV consecutive elements per thread and pass; every input group of
  // the pass is loaded before any result is stored
  s << "extern \"C\" __global__ void __launch_bounds__(" << kEwThreads << ") xt_ew_v(const XtEwArgs p) {\n"
       "  xt_pdl_launch();\n  xt_pdl_wait();\n"
       "  const xt_i64 n = p.end - p.begin, groups = n / (4 * XT_NV);\n"
       "  const xt_i64 stride = static_cast<xt_i64>(gridDim.x) * blockDim.x;\n"
       "  for (xt_i64 v = static_cast<xt_i64>(blockIdx.x) * blockDim.x + threadIdx.x; v < groups; v += stride) {\n"
       "    const xt_i64 i0 = p.begin + 4 * XT_NV * v;\n";
  if (bcast) {
    // a broadcast row's column of each group: the period is a multiple of 4,
    // so a group never wraps inside itself
    s << "    xt_i64 ib[XT_NV];\n"
         "    {\n      xt_i64 c = i0 % p.period;\n"
         "#pragma unroll\n"
         "      for (int j = 0; j < XT_NV; ++j) {\n        ib[j] = c;\n        c += 4;\n"
         "        if (c >= p.period) c -= p.period;\n      }\n    }\n";
  }
  s << "    float4";
  bool first = true;
  for (int r : regs) s << (first ? " r" : ", r") << r << "[XT_NV]", first = false;
  s << ";\n";
  for (int pc = 0; pc < a.n_code; ++pc) {
    const Instr& in = a.code[pc];
    s << "#pragma unroll\n    for (int j = 0; j < XT_NV; ++j) ";
    if (in.op == kLoad) {
      const bool b = a.in_bcast[in.a];
      s << "r" << int(in.dst) << "[j] = xt_ld4_" << elem_suffix(a.in_elem[in.a])
        << (b && a.in_elem[in.a] == dev::kF32 ? "_kept" : "") << "(p.in[" << int(in.a) << "], "
        << (b ? "ib[j]" : "i0 + 4 * j") << ");\n";
    } else if (in.op == kStore) {
      s << "xt_st4_" << elem_suffix(a.out_elem[in.dst]) << "(p.out[" << int(in.dst) << "], i0 + 4 * j, r" << int(in.a)
        << "[j]);\n";
    } else if (is_binary(in.op)) {
      s << "r" << int(in.dst) << "[j] = XT_MAP2(" << binary_fn(in.op) << ", r" << int(in.a) << "[j], r" << int(in.b)
        << "[j]);\n";
    } else {
      s << "r" << int(in.dst) << "[j] = XT_MAP1(" << unary_fn(in.op) << ", r" << int(in.a) << "[j]);\n";
    }
  }
  s << "  }\n"
       "  for (xt_i64 e = groups * 4 * XT_NV + static_cast<xt_i64>(blockIdx.x) * blockDim.x + threadIdx.x; e < n;"
       " e += stride)\n"
       "    xt_ew_elem(p, p.begin + e);\n}\n";
  return s.str();
}

namespace {

int64_t rows_pl4(int64_t cols) { return ((cols + 3) / 4 + 31) / 32; }
int64_t rows_pls(int64_t cols) { return (cols + 31) / 32; }

// the rows program; ``vec``: float4 chunks (cols % 4 == 0), else elements;
// ``cta``: the row spread over the CTA's XT_TPR threads (block reductions),
// else over a warp
void rows_body(std::ostringstream& s, const dev::RowArgs& a, bool vec, bool cta) {
  const int n_v = std::max(a.n_vregs, 1);
  const char* T = vec ? "float4" : "float";
  const char* N = vec ? "XT_PL4" : "XT_PLS";
  s << "  " << T;
  for (int k = 0; k < n_v; ++k) s << (k ? ", v" : " v") << k << "[" << N << "]";
  s << ";\n";
  std::set<int> sregs;  // scalar registers the program writes
  for (int pc = 0; pc < a.n_code; ++pc) {
    const uint8_t o = a.code[pc].op & 0x7f;
    if (o == kRowMax || o == kRowSum || o == kLoadScalar || (a.code[pc].op & 0x80)) sregs.insert(a.code[pc].dst);
  }
  if (!sregs.empty()) {
    s << "  float";
    bool first = true;
    for (int k : sregs) s << (first ? " s" : ", s") << k, first = false;
    s << ";\n";
  }
  // index of chunk / element j of this lane, and whether it lies in the row
  const std::string width = cta ? "XT_TPR" : "32";
  const std::string idx = vec ? "const int c = j * " + width + " + lane; const bool in = c < XT_C4;"
                              : "const int c = j * " + width + " + lane; const bool in = c < XT_COLS;";
  for (int pc = 0; pc < a.n_code; ++pc) {
    const Instr& in = a.code[pc];
    const uint8_t op = in.op & 0x7f;
    const bool scalar = (in.op & 0x80) != 0;
    const std::string d = std::to_string(in.dst), x = std::to_string(in.a), y = std::to_string(in.b);
    auto loop = [&](const std::string& body, bool guarded = false) {
      s << "#pragma unroll\n  for (int j = 0; j < " << N << "; ++j) { " << (guarded ? idx + " " : std::string())
        << body << " }\n";
    };
    if (op == kLoad) {
      if (vec)
        loop("v" + d + "[j] = in ? __ldcs(reinterpret_cast<const float4*>(p.in[" + x +
             "] + row * XT_COLS) + c) : make_float4(0.f, 0.f, 0.f, 0.f);",
             true);
      else
        loop("v" + d + "[j] = in ? __ldcs(p.in[" + x + "] + row * XT_COLS + c) : 0.0f;", true);
    } else if (op == kLoadScalar) {
      s << "  s" << d << " = __ldg(p.in[" << x << "] + row);\n";
    } else if (op == kStore) {
      if (vec)
        loop("if (in) __stcs(reinterpret_cast<float4*>(p.out[" + d + "] + row * XT_COLS) + c, v" + x + "[j]);",
             true);
      else
        loop("if (in) p.out[" + d + "][row * XT_COLS + c] = v" + x + "[j];", true);
    } else if (op == kStoreScalar) {
      s << "  if (lane == 0) p.out[" << d << "][row] = s" << x << ";\n";
    } else if (op == kRowMax || op == kRowSum) {
      const bool mx = op == kRowMax;
      s << "  {\n    float acc = " << (mx ? "__int_as_float(0xff800000)" : "0.0f") << ";\n";
      if (vec)
        s << "#pragma unroll\n    for (int j = 0; j < XT_PL4; ++j) { " << idx << " if (in) { const float4 t = v" << x
          << "[j]; acc = "
          << (mx ? "fmaxf(fmaxf(fmaxf(acc, t.x), fmaxf(t.y, t.z)), t.w)"
                 : "__fadd_rn(acc, __fadd_rn(__fadd_rn(t.x, t.y), __fadd_rn(t.z, t.w)))")
          << "; } }\n";
      else
        s << "#pragma unroll\n    for (int j = 0; j < XT_PLS; ++j) { " << idx << " if (in) acc = "
          << (mx ? "fmaxf(acc, v" + x + "[j])" : "__fadd_rn(acc, v" + x + "[j])") << "; }\n";
      s << "    s" << d << " = " << (mx ? (cta ? "xt_cta_max" : "xt_warp_max") : (cta ? "xt_cta_sum" : "xt_warp_sum"))
        << "(acc);\n  }\n";
    } else if (scalar) {
      if (binary_fn(op) && is_binary(op))
        s << "  s" << d << " = " << binary_fn(op) << "(s" << x << ", s" << y << ");\n";
      else if (unary_fn(op))
        s << "  s" << d << " = " << unary_fn(op) << "(s" << x << ");\n";
      else
        fail("opcode " + std::to_string(in.op) + " on row scalars");
    } else if (op == kBcastAdd || op == kBcastSub || op == kBcastMul) {
      loop(vec ? "v" + d + "[j] = XT_MAP2S(" + binary_fn(op) + ", v" + x + "[j], s" + y + ");"
               : "v" + d + "[j] = " + binary_fn(op) + "(v" + x + "[j], s" + y + ");");
    } else if (is_binary(op)) {
      loop(vec ? "v" + d + "[j] = XT_MAP2(" + binary_fn(op) + ", v" + x + "[j], v" + y + "[j]);"
               : "v" + d + "[j] = " + binary_fn(op) + "(v" + x + "[j], v" + y + "[j]);");
    } else if (unary_fn(op)) {
      loop(vec ? "v" + d + "[j] = XT_MAP1(" + std::string(unary_fn(op)) + ", v" + x + "[j]);"
               : "v" + d + "[j] = " + unary_fn(op) + "(v" + x + "[j]);");
    } else {
      fail("opcode " + std::to_string(in.op) + " in a row program");
    }
  }
}

}  // namespace

bool rows_fit(const dev::RowArgs& a) { return row_warp_fits(a.cols, std::max(a.n_vregs, 1)); }

std::string rows_cta_source(const dev::RowArgs& a, int tpr) {
  if (a.n_code <= 0 || a.n_code > kMaxInstr) fail("row program length");
  if (a.cols <= 0) fail("row length");
  if (tpr < 128 || tpr > 1024 || (tpr & (tpr - 1))) fail("threads per row");
  std::ostringstream s;
  s << kOpMath << kHelpers;
  s << "#define XT_COLS " << a.cols << "\n#define XT_C4 " << (a.cols + 3) / 4 << "\n#define XT_TPR " << tpr
    << "\n#define XT_PL4 " << ((a.cols + 3) / 4 + tpr - 1) / tpr << "\n#define XT_PLS " << (a.cols + tpr - 1) / tpr
    << "\n";
  s << "struct XtRowArgs { const float* in[" << kMaxSlots << "]; float* out[" << kMaxSlots
    << "]; xt_i64 row_begin, row_end; };\n";
  // block reductions: warp trees, then the warps' results in a fixed order;
  // the first barrier keeps the previous reduction's readers ahead of the
  // writes, the second publishes them
  s << "__device__ __forceinline__ float xt_cta_reduce(float v, bool mx) {\n"
       "  __shared__ float red[XT_TPR / 32];\n"
       "  v = mx ? xt_warp_max(v) : xt_warp_sum(v);\n"
       "  __syncthreads();\n"
       "  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;\n"
       "  __syncthreads();\n"
       "  float r = red[0];\n"
       "#pragma unroll\n"
       "  for (int w = 1; w < XT_TPR / 32; ++w) r = mx ? fmaxf(r, red[w]) : __fadd_rn(r, red[w]);\n"
       "  return r;\n}\n"
       "__device__ __forceinline__ float xt_cta_max(float v) { return xt_cta_reduce(v, true); }\n"
       "__device__ __forceinline__ float xt_cta_sum(float v) { return xt_cta_reduce(v, false); }\n";
  for (int vec = 1; vec >= 0; --vec) {
    s << "extern \"C\" __global__ void __launch_bounds__(" << tpr << ") " << (vec ? "xt_rows_cv" : "xt_rows_cs")
      << "(const XtRowArgs p) {\n"
         "  const int lane = threadIdx.x;\n"
         "  const xt_i64 row = p.row_begin + static_cast<xt_i64>(blockIdx.x);\n"
         "  xt_pdl_launch();\n  if (row >= p.row_end) return;\n  xt_pdl_wait();\n";
    rows_body(s, a, vec == 1, true);
    s << "}\n";
  }
  return s.str();
}

std::string rows_kernel_source(const dev::RowArgs& a) {
  if (rows_fit(a)) return rows_source(a);
  const int tpr = row_cta_threads(a.cols, std::max(a.n_vregs, 1));
  if (!tpr) fail("the row program's live rows exceed a CTA's registers");
  return rows_cta_source(a, tpr);
}

std::string rows_source(const dev::RowArgs& a) {
  if (a.n_code <= 0 || a.n_code > kMaxInstr) fail("row program length");
  if (a.cols <= 0) fail("row length");
  std::ostringstream s;
  s << kOpMath << kHelpers;
  s << "#define XT_COLS " << a.cols << "\n#define XT_C4 " << (a.cols + 3) / 4 << "\n#define XT_PL4 "
    << rows_pl4(a.cols) << "\n#define XT_PLS " << rows_pls(a.cols) << "\n#define XT_ROWS_PER_CTA " << kRowsPerCta
    << "\n";
  s << "struct XtRowArgs { const float* in[" << kMaxSlots << "]; float* out[" << kMaxSlots
    << "]; xt_i64 row_begin, row_end; };\n";
  for (int vec = 1; vec >= 0; --vec) {
    s << "extern \"C\" __global__ void __launch_bounds__(" << 32 * kRowsPerCta << ") " << (vec ? "xt_rows_v" : "xt_rows_s")
      << "(const XtRowArgs p) {\n"
         "  const int lane = threadIdx.x & 31;\n"
         "  const xt_i64 row = p.row_begin + static_cast<xt_i64>(blockIdx.x) * XT_ROWS_PER_CTA + (threadIdx.x >> 5);\n"
         "  xt_pdl_launch();\n  if (row >= p.row_end) return;\n  xt_pdl_wait();\n";
    rows_body(s, a, vec == 1, false);
    s << "}\n";
  }
  return s.str();
}


// ---------------------------------------------------------------------------
// Tile programs.  One CTA per Block, every tile value in its planned shared-memory slot (f32,
// row-major, rows padded to an odd pitch), the ops in program order with a
// CTA barrier between them -- but every shape, pitch, slot offset, array
// stride, tile coordinate and edge limit is a constant of the source.  A
// value of shape (s0, s1, s2, s3) is s0*s1*s2 rows of s3 elements at one
// pitch, so each op is a loop of the CTA's threads over (row q, column c)
// with constant bounds; when the CTA width is a multiple of the row length a
// thread keeps one column and steps whole rows.  Loads keep up to 8 accesses
// in flight per thread; accesses whose rows are whole 4-element groups at
// 4-element array offsets move 4 elements per access in the aligned kernel.
// Reductions with fewer outputs than threads split each output's elements
// over several threads and combine the partial results in a fixed order.
namespace {

struct TileGeom {
  int64_t s[kTileRank];   // shape
  int64_t st[kTileRank];  // shared-memory strides (st[3] = 1)
  int64_t off;
  int64_t rows() const { return s[0] * s[1] * s[2]; }
};

// ``compact``: rows at a pitch of exactly one row (the slot's planned pitch
// is one float longer for even rows)
TileGeom tile_geom(const TileVal& v, bool compact) {
  TileGeom g;
  for (int d = 0; d < kTileRank; ++d) g.s[d] = v.shape[d];
  if (compact) {
    g.st[3] = 1;
    g.st[2] = g.s[3];
    g.st[1] = g.s[2] * g.st[2];
    g.st[0] = g.s[1] * g.st[1];
  } else {
    for (int d = 0; d < kTileRank; ++d) g.st[d] = d == kTileRank - 1 ? 1 : v.stride[d];
  }
  g.off = v.offset;
  return g;
}

// Which values keep their rows at a pitch of one row.  The planner pads
// even rows to an odd pitch so that a warp walking down a column hits 32
// banks; values that no op walks down a column (the operands of permutes,
// of stores that read through a permutation and of reductions along the
// last dim) drop the pad: a warp's row-major accesses then touch
// consecutive words, and 4-element groups are 16-byte aligned.  A value
// computed in place of its operand keeps the operand's pitch.
std::vector<bool> compact_values(const dev::TileArgs& a) {
  std::vector<bool> c(kTileMaxVals, true);
  for (int o = 0; o < a.n_ops; ++o) {
    const TileOp& op = a.ops[o];
    if (op.kind == kTPermute || (op.kind == kTReduce && op.axis == kTileRank - 1)) c[op.a] = false;
    if (op.kind == kTStore && op.code == 1) c[op.b] = false;
  }
  for (bool changed = true; changed;) {
    changed = false;
    for (int o = 0; o < a.n_ops; ++o) {
      const TileOp& op = a.ops[o];
      if (op.kind != kTUnary && op.kind != kTBinary) continue;
      for (int x : {static_cast<int>(op.a), op.kind == kTBinary ? static_cast<int>(op.b) : -1}) {
        if (x < 0 || a.vals[x].offset != a.vals[op.dst].offset || c[x] == c[op.dst]) continue;
        c[x] = c[op.dst] = false;
        changed = true;
      }
    }
  }
  return c;
}

std::string float_lit(float v) {
  uint32_t u;
  std::memcpy(&u, &v, sizeof u);
  char buf[40];
  std::snprintf(buf, sizeof buf, "__int_as_float(0x%08x)", u);
  return buf;
}

// the multi-index (i0, i1, i2) of row ``q`` (< s0 * s1 * s2) of a value of
// shape ``s``; dims of size 1 have index 0
std::string row_index(const int64_t (&s)[kTileRank], const char* q) {
  std::ostringstream o;
  const std::string Q(q);
  const std::string i2 = s[0] == 1 && s[1] == 1 ? Q : s[2] == 1 ? "0" : Q + " % " + std::to_string(s[2]);
  const std::string above = s[2] == 1 ? Q : "(" + Q + " / " + std::to_string(s[2]) + ")";
  const std::string i1 = s[1] == 1 ? "0" : s[0] == 1 ? above : above + " % " + std::to_string(s[1]);
  const std::string i0 = s[0] == 1 ? "0" : Q + " / " + std::to_string(s[2] * s[1]);
  o << "const int i2 = " << i2 << ", i1 = " << i1 << ", i0 = " << i0 << "; (void)i0; (void)i1; (void)i2;";
  return o.str();
}

// i0 * k0 + i1 * k1 + i2 * k2 (+ c * k3), leaving out zero strides and the
// dims of size 1 in ``s`` (index 0)
std::string dot(const int64_t (&k)[kTileRank], const int64_t (&s)[kTileRank], const char* c = "c", bool wide = false) {
  std::ostringstream o;
  const char* idx[kTileRank] = {"i0", "i1", "i2", c};
  bool any = false;
  for (int d = 0; d < kTileRank; ++d) {
    if (k[d] == 0 || s[d] == 1) continue;
    o << (any ? " + " : "") << (wide ? "static_cast<xt_i64>(" : "") << idx[d] << (wide ? ")" : "");
    if (k[d] != 1) o << " * " << k[d];
    any = true;
  }
  if (!any) o << "0";
  return o.str();
}

// A load's or store's place in its array: the Block's first element (an
// expression of the block ids), the array strides, and per dim the number of
// the tile's elements inside the array when that can be less than the tile
// (``lim``, empty when the tile always lies inside along that dim).
struct Access {
  std::string decl;   // declarations of run-time limits
  std::string base;   // xt_i64 expression
  int64_t A[kTileRank];
  std::string lim[kTileRank];
  bool vec;           // rows are whole 4-element groups at 4-element offsets
  std::string inb(const char* c) const {
    std::string s;
    const char* idx[kTileRank] = {"i0", "i1", "i2", c};
    for (int d = 0; d < kTileRank; ++d)
      if (!lim[d].empty()) s += (s.empty() ? "" : " && ") + std::string(idx[d]) + " < " + lim[d];
    return s.empty() ? "true" : s;
  }
};

Access access_of(const dev::TileArgs& a, const TileOp& op, const TileGeom& v, int n) {
  const int32_t* ext = a.shape[op.arg];
  Access g;
  int64_t run = 1;
  for (int d = kTileRank - 1; d >= 0; --d) {
    g.A[d] = run;
    run *= ext[d];
  }
  int64_t cst = 0, mult[3] = {0, 0, 0};
  std::ostringstream decl;
  for (int d = 0; d < kTileRank; ++d) {
    const int cb = op.coord_bid[d];
    if (cb >= 0) {
      mult[cb] += v.s[d] * g.A[d];
      if (a.grid[cb] * v.s[d] > ext[d]) {
        // a Block past the edge along this dim: its own limit at run time
        decl << "    const int l" << n << "_" << d << " = static_cast<int>(max(static_cast<xt_i64>(0), min(static_cast<xt_i64>("
             << v.s[d] << "), static_cast<xt_i64>(" << ext[d] << ") - b" << cb << " * " << v.s[d] << ")));\n";
        g.lim[d] = "l" + std::to_string(n) + "_" + std::to_string(d);
      }
    } else {
      const int64_t start = static_cast<int64_t>(op.coord[d]) * v.s[d];
      cst += start * g.A[d];
      const int64_t left = ext[d] - start;
      const int64_t lim = left <= 0 ? 0 : std::min(left, v.s[d]);
      if (lim < v.s[d]) g.lim[d] = std::to_string(lim);
    }
  }
  std::ostringstream base;
  base << "static_cast<xt_i64>(" << cst << ")";
  for (int k = 0; k < 3; ++k)
    if (mult[k]) base << " + b" << k << " * " << mult[k];
  g.decl = decl.str();
  g.base = base.str();
  g.vec = v.s[3] % 4 == 0 && ext[3] % 4 == 0;
  return g;
}

const char* ld1(uint8_t e) { return e == dev::kF32 ? "xt_ld1_f32" : e == dev::kBF16 ? "xt_ld1_bf16" : "xt_ld1_i8"; }
const char* ld4(uint8_t e) { return e == dev::kF32 ? "xt_ld4_f32_kept" : e == dev::kBF16 ? "xt_ld4_bf16" : "xt_ld4_i8"; }
const char* st1(uint8_t e) { return e == dev::kF32 ? "xt_st1_f32" : e == dev::kBF16 ? "xt_st1_bf16" : "xt_st1_i8"; }
const char* st4(uint8_t e) { return e == dev::kF32 ? "xt_st4_f32" : e == dev::kBF16 ? "xt_st4_bf16" : "xt_st4_i8"; }

// A loop of the CTA's ``th`` threads over the rows x width index space,
// defining ``q`` and ``cv`` (the column, or 4-column group) for ``body``.
void loop_rows(std::ostringstream& s, int th, int64_t rows, int64_t width, const std::string& body) {
  if (th % width == 0) {
    s << "    {\n      const int cv = t % " << width << ";\n#pragma unroll 4\n      for (int q = t / " << width << "; q < "
      << rows << "; q += " << th / width << ") {\n" << body << "      }\n    }\n";
  } else {
    s << "#pragma unroll 4\n    for (int e = t; e < " << rows * width << "; e += " << th << ") {\n      const int q = e / "
      << width << ", cv = e % " << width << ";\n" << body << "    }\n";
  }
}

// A load: up to 8 accesses in flight per thread before their shared-memory
// stores.  ``vec``: 4 elements per access.
void emit_load(std::ostringstream& s, const dev::TileArgs& a, const TileOp& op, const TileGeom& v, const Access& g,
               int th, bool vec) {
  const int64_t width = vec ? v.s[3] / 4 : v.s[3], rows = v.rows();
  const uint8_t e = a.elem[op.arg];
  const char* T = vec ? "float4" : "float";
  const char* zero = vec ? "make_float4(0.f, 0.f, 0.f, 0.f)" : "0.0f";
  const std::string col = vec ? "const int c = 4 * cv;" : "const int c = cv;";
  const std::string addr = "gb + " + dot(g.A, v.s, "c", true);
  const std::string ld = std::string(vec ? ld4(e) : ld1(e)) + "(p.arr[" + std::to_string(op.arg) + "], " + addr + ")";
  std::ostringstream st;  // the shared-memory store of v[u] at row q, column c
  const std::string sm = "xt_sm + " + std::to_string(v.off) + " + q * " + std::to_string(v.st[2]) + " + c";
  if (vec && v.st[2] % 4 == 0 && v.off % 4 == 0)
    st << "*reinterpret_cast<float4*>(" << sm << ") = v[u];";
  else if (vec)
    st << "{ float* d = " << sm << "; d[0] = v[u].x; d[1] = v[u].y; d[2] = v[u].z; d[3] = v[u].w; }";
  else
    st << "xt_sm[" << v.off << " + q * " << v.st[2] << " + c] = v[u];";
  if (th % width == 0) {
    const int64_t rs = th / width;
    const int64_t kb = std::min<int64_t>(8, (rows + rs - 1) / rs);
    s << "    {\n      const int cv = t % " << width << "; " << col << "\n"
      << "      for (int q0 = t / " << width << "; q0 < " << rows << "; q0 += " << kb * rs << ") {\n"
      << "        " << T << " v[" << kb << "];\n#pragma unroll\n"
      << "        for (int u = 0; u < " << kb << "; ++u) {\n          const int q = q0 + u * " << rs << "; "
      << row_index(v.s, "q") << "\n          v[u] = (q < " << rows << " && " << g.inb("c") << ") ? " << ld << " : "
      << zero << ";\n        }\n#pragma unroll\n"
      << "        for (int u = 0; u < " << kb << "; ++u) {\n          const int q = q0 + u * " << rs << ";\n"
      << "          if (q < " << rows << ") " << st.str() << "\n        }\n      }\n    }\n";
  } else {
    const int64_t n = rows * width;
    const int64_t kb = std::min<int64_t>(8, (n + th - 1) / th);
    s << "    for (int e0 = t; e0 < " << n << "; e0 += " << kb * th << ") {\n"
      << "      " << T << " v[" << kb << "];\n#pragma unroll\n"
      << "      for (int u = 0; u < " << kb << "; ++u) {\n        const int e = e0 + u * " << th << ", q = e / " << width
      << ", cv = e % " << width << "; " << col << " " << row_index(v.s, "q") << "\n"
      << "        v[u] = (e < " << n << " && " << g.inb("c") << ") ? " << ld << " : " << zero << ";\n      }\n#pragma unroll\n"
      << "      for (int u = 0; u < " << kb << "; ++u) {\n        const int e = e0 + u * " << th << ", q = e / " << width
      << ", cv = e % " << width << "; " << col << "\n        if (e < " << n << ") " << st.str() << "\n      }\n    }\n";
  }
}

// A store of tile ``v`` reading shared memory at ``rd_off`` through the
// strides ``rd`` (its own slot, or a folded permute's operand).
void emit_store(std::ostringstream& s, const dev::TileArgs& a, const TileOp& op, const TileGeom& v, int64_t rd_off,
                const int64_t (&rd)[kTileRank], const Access& g, int th, bool vec) {
  const uint8_t e = a.elem[op.arg];
  const std::string arr = "p.arr[" + std::to_string(op.arg) + "]";
  std::ostringstream b;
  b << "        const int c = " << (vec ? "4 * cv" : "cv") << "; " << row_index(v.s, "q") << "\n";
  b << "        if (" << g.inb("c") << ") {\n          const int r = " << rd_off << " + " << dot(rd, v.s) << ";\n";
  bool aligned4 = rd[3] == 1 && rd_off % 4 == 0;
  for (int d = 0; d < kTileRank - 1; ++d) aligned4 = aligned4 && (v.s[d] == 1 || rd[d] % 4 == 0);
  if (vec && aligned4)
    b << "          " << st4(e) << "(" << arr << ", gb + " << dot(g.A, v.s, "c", true)
      << ", *reinterpret_cast<const float4*>(xt_sm + r));\n";
  else if (vec)
    b << "          " << st4(e) << "(" << arr << ", gb + " << dot(g.A, v.s, "c", true) << ", make_float4(xt_sm[r], xt_sm[r + "
      << rd[3] << "], xt_sm[r + " << 2 * rd[3] << "], xt_sm[r + " << 3 * rd[3] << "]));\n";
  else
    b << "          " << st1(e) << "(" << arr << ", gb + " << dot(g.A, v.s, "c", true) << ", xt_sm[r]);\n";
  b << "        }\n";
  loop_rows(s, th, v.rows(), vec ? v.s[3] / 4 : v.s[3], b.str());
}

// Threads sharing one output of a reduction with ``outs`` outputs over ``n``
// elements: a power of two that fits the CTA and leaves each thread at
// least 4 elements, or 1.
int64_t reduce_parts(int64_t outs, int64_t n, int th) {
  int64_t k = 1;
  while (outs * k * 2 <= th && k * 2 * 4 <= n) k *= 2;
  return k;
}

// Accumulates src[j * step] for j = first, first + stride, ... < n into
// ``acc`` (double sum, or float max with NaN propagating) with four
// independent accumulators combined in a fixed order.
void emit_accumulate(std::ostringstream& s, bool sum, int64_t n, int64_t step, int64_t stride, const char* first) {
  const int64_t count = (n + stride - 1) / stride, groups = (count + 3) / 4;
  const char* T = sum ? "double" : "float";
  const char* init = sum ? "0.0" : "__int_as_float(0xff800000)";
  s << "        " << T << " a0 = " << init << ", a1 = " << init << ", a2 = " << init << ", a3 = " << init << ";\n"
    << "#pragma unroll 4\n        for (int k = 0; k < " << groups << "; ++k) {\n"
    << "          const int j = " << first << " + k * " << 4 * stride << ";\n";
  for (int u = 0; u < 4; ++u) {
    const std::string j = u ? "j + " + std::to_string(u * stride) : std::string("j");
    s << "          if (" << j << " < " << n << ") a" << u << " = "
      << (sum ? "a" + std::to_string(u) + " + static_cast<double>(src[(" + j + ") * " + std::to_string(step) + "])"
              : "xt_max_nan(a" + std::to_string(u) + ", src[(" + j + ") * " + std::to_string(step) + "])")
      << ";\n";
  }
  s << "        }\n        const " << T << " acc = "
    << (sum ? "(a0 + a1) + (a2 + a3)" : "xt_max_nan(xt_max_nan(a0, a1), xt_max_nan(a2, a3))") << ";\n";
}

// The end of the run of elementwise ops (const, unary, binary) from ``o``
// that can share one pass over their common result shape with no barrier
// between them: a thread then handles the same elements in every op, so an
// op reading the result of an earlier op of the run reads what that thread
// itself computed.  The run stops before an op whose result has another
// shape, that reads a result of the run along a broadcast dim (another
// thread's element), or whose result slot overlaps shared memory that the
// run has read or written other than at the same element of a same-shaped,
// same-pitch value (a slot the planner recycled while other threads may
// still be reading its previous value).
template <class Ew, class Same, class Reads>
int elementwise_run(const dev::TileArgs& a, int o, const std::vector<bool>& compact, Ew elementwise, Same same_shape,
                    Reads reads) {
  struct Touch {
    int64_t lo, hi, pitch;
    int val;
    bool own;  // accessed only at the thread's own elements
  };
  auto geom = [&](int v) { return tile_geom(a.vals[v], compact[v]); };
  auto touch = [&](int v, bool own) {
    const TileGeom g = geom(v);
    return Touch{g.off, g.off + g.rows() * g.st[2], g.st[2], v, own};
  };
  const int shape_of = a.ops[o].dst;
  std::vector<Touch> touched;
  std::set<int> made;
  int e = o;
  for (; e < a.n_ops; ++e) {
    const TileOp& op = a.ops[e];
    if (!elementwise(op) || !same_shape(op.dst, shape_of)) break;
    bool ok = true;
    for (int x : reads(op))
      if (made.count(x) && !same_shape(x, shape_of)) ok = false;
    const Touch w = touch(op.dst, true);
    for (const Touch& t : touched) {
      const bool overlap = w.lo < t.hi && t.lo < w.hi;
      const bool same_element = t.own && t.lo == w.lo && t.pitch == w.pitch;
      if (overlap && !same_element) ok = false;
    }
    if (!ok && e > o) break;
    for (int x : reads(op))
      if (!made.count(x)) touched.push_back(touch(x, same_shape(x, shape_of)));
    touched.push_back(w);
    made.insert(op.dst);
  }
  return e;
}

// Ops [o, e) (a run from elementwise_run) as one loop over their result
// shape: each result a register; a result goes to its shared-memory slot
// only when an op after the run reads it.
void emit_elementwise(std::ostringstream& s, const dev::TileArgs& a, int o, int e, int th,
                      const std::vector<bool>& compact, const std::vector<std::vector<int>>& readers) {
  auto geom = [&](int v) { return tile_geom(a.vals[v], compact[v]); };
  const TileGeom S = geom(a.ops[o].dst);
  // whether a result is read after the run (and so goes to its slot)
  auto later = [&](int v) {
    for (int r : readers[v])
      if (r >= e) return true;
    return false;
  };
  // broadcast dims (size 1) contribute no stride
  auto strides = [&](int x, int64_t (&sx)[kTileRank]) {
    const TileGeom g = geom(x);
    for (int k = 0; k < kTileRank; ++k) sx[k] = g.s[k] == 1 ? 0 : g.st[k];
    return g;
  };
  // Four consecutive columns per step when the rows hold whole 4-element
  // groups and every shared-memory access of the run is 16-byte aligned or
  // a broadcast along the columns.
  bool vec = S.s[3] % 4 == 0;
  {
    std::set<int> made;
    for (int j = o; j < e && vec; ++j) {
      const TileOp& op = a.ops[j];
      std::vector<int> xs;
      if (op.kind != kTConst) xs.push_back(op.a);
      if (op.kind == kTBinary) xs.push_back(op.b);
      for (int x : xs) {
        if (made.count(x)) continue;
        int64_t sx[kTileRank];
        const TileGeom g = strides(x, sx);
        if (sx[3] == 0) continue;  // one value per row: read once, used four times
        vec = vec && g.off % 4 == 0;
        for (int k = 0; k < kTileRank - 1; ++k) vec = vec && sx[k] % 4 == 0;
      }
      made.insert(op.dst);
      if (later(op.dst)) {
        const TileGeom d = geom(op.dst);
        vec = vec && d.off % 4 == 0 && d.st[2] % 4 == 0;
      }
    }
  }
  std::set<int> made;
  std::ostringstream b;
  b << "        const int c = " << (vec ? "4 * cv" : "cv") << "; " << row_index(S.s, "q") << "\n";
  auto operand = [&](int x) {
    if (made.count(x)) return "r" + std::to_string(x);
    int64_t sx[kTileRank];
    const TileGeom g = strides(x, sx);
    const std::string at = std::to_string(g.off) + " + " + dot(sx, S.s);
    if (!vec) return "xt_sm[" + at + "]";
    if (sx[3] == 0) {
      const std::string one = "xt_sm[" + at + "]";
      return "make_float4(" + one + ", " + one + ", " + one + ", " + one + ")";
    }
    return "*reinterpret_cast<const float4*>(xt_sm + " + at + ")";
  };
  const char* T = vec ? "float4" : "float";
  // an operand as a named value (the macros of the vector form use it four times)
  auto bind = [&](int x, int j, int k) {
    if (made.count(x)) return "r" + std::to_string(x);
    const std::string name = "x" + std::to_string(j) + "_" + std::to_string(k);
    b << "        const " << T << " " << name << " = " << operand(x) << ";\n";
    return name;
  };
  for (int j = o; j < e; ++j) {
    const TileOp& op = a.ops[j];
    std::string expr;
    if (op.kind == kTConst) {
      const std::string v = float_lit(op.value);
      expr = vec ? "make_float4(" + v + ", " + v + ", " + v + ", " + v + ")" : v;
    } else if (op.kind == kTUnary) {
      const char* fn = unary_fn(op.code);
      if (!fn) fail("unary opcode " + std::to_string(op.code) + " in a tile program");
      const std::string x = bind(op.a, j, 0);
      expr = vec ? "XT_MAP1(" + std::string(fn) + ", " + x + ")" : std::string(fn) + "(" + x + ")";
    } else {
      const char* fn = binary_fn(op.code);
      if (!fn || !is_binary(op.code)) fail("binary opcode " + std::to_string(op.code) + " in a tile program");
      const std::string x = bind(op.a, j, 0), y = bind(op.b, j, 1);
      expr = vec ? "XT_MAP2(" + std::string(fn) + ", " + x + ", " + y + ")" : std::string(fn) + "(" + x + ", " + y + ")";
      if (a.vals[op.dst].i8) expr = vec ? "XT_MAP1(xt_wrap_i8, " + expr + ")" : "xt_wrap_i8(" + expr + ")";
    }
    b << "        const " << T << " r" << int(op.dst) << " = " << expr << ";  // op " << j << "\n";
    made.insert(op.dst);
    if (later(op.dst)) {
      const TileGeom d = geom(op.dst);
      if (vec)
        b << "        *reinterpret_cast<float4*>(xt_sm + " << d.off << " + q * " << d.st[2] << " + c) = r" << int(op.dst)
          << ";\n";
      else
        b << "        xt_sm[" << d.off << " + q * " << d.st[2] << " + c] = r" << int(op.dst) << ";\n";
    }
  }
  s << "  {  // ops " << o << "-" << e - 1 << ": one pass" << (vec ? ", 4 columns per step" : "") << "\n";
  loop_rows(s, th, S.rows(), vec ? S.s[3] / 4 : S.s[3], b.str());
  s << "  }\n";
}

// first float of the split reductions' partial results (8-byte aligned)
int64_t red_offset(const dev::TileArgs& a) { return (a.smem_floats + 1) & ~1; }

}  // namespace

int tile_smem_floats(const dev::TileArgs& a, int th) {
  bool reduces = false;
  for (int o = 0; o < a.n_ops; ++o) reduces = reduces || a.ops[o].kind == kTReduce;
  return static_cast<int>(red_offset(a)) + (reduces ? 2 * th : 0);
}

int tile_threads(const dev::TileArgs& a) {
  int64_t most = 0;
  for (int v = 0; v < kTileMaxVals; ++v) most = std::max<int64_t>(most, a.vals[v].numel);
  return most <= 4096 ? 128 : most <= 8192 ? 256 : most <= 16384 ? 512 : 1024;
}

std::string tile_source(const dev::TileArgs& a, int th) {
  if (a.n_ops <= 0 || a.n_ops > kTileMaxOps) fail("tile program length");
  if (th != 64 && th != 128 && th != 256 && th != 512 && th != 1024) fail("tile CTA width");
  std::ostringstream s;
  s << kOpMath << kHelpers;
  s << "struct XtTileArgs { void* arr[" << kTileMaxArgs << "]; xt_i64 bid0_begin; };\n"
       "extern __shared__ __align__(16) float xt_sm[];\n"
       "__device__ __forceinline__ float xt_wrap_i8(float x) {\n"
       "  return static_cast<float>(static_cast<signed char>(static_cast<int>(x)));\n}\n"
       "// the larger of two values; a NaN operand gives NaN, as np.max\n"
       "__device__ __forceinline__ float xt_max_nan(float r, float v) { return (v != v || v > r) ? v : r; }\n";
  // partial results of split reductions, after the planned slots
  s << "#define xt_red_f64 reinterpret_cast<double*>(xt_sm + " << red_offset(a) << ")\n"
    << "#define xt_red_f32 (xt_sm + " << red_offset(a) << ")\n";
  const std::vector<bool> compact = compact_values(a);
  // a value's layout (its planned slot, rows unpadded when compact)
  auto value_geom = [&](int v) { return tile_geom(a.vals[v], compact[v]); };
  s << "template <bool V>\n__device__ __forceinline__ void xt_tile_body(const XtTileArgs& p) {\n"
       "  const int t = threadIdx.x;\n"
       "  const xt_i64 b0 = p.bid0_begin + blockIdx.x, b1 = blockIdx.y, b2 = blockIdx.z;\n"
       "  (void)b0; (void)b1; (void)b2;\n";
  // the ops reading each value, and whether each op is elementwise
  std::vector<std::vector<int>> readers(kTileMaxVals);
  auto reads = [&](const TileOp& op) {
    std::vector<int> r;
    if (op.kind == kTStore) r.push_back(op.code == 1 ? op.b : op.a);
    if (op.kind == kTUnary || op.kind == kTBinary || op.kind == kTReduce || op.kind == kTReshape || op.kind == kTPermute)
      r.push_back(op.a);
    if (op.kind == kTBinary) r.push_back(op.b);
    return r;
  };
  for (int o = 0; o < a.n_ops; ++o)
    for (int x : reads(a.ops[o])) readers[x].push_back(o);
  auto elementwise = [&](const TileOp& op) { return op.kind == kTConst || op.kind == kTUnary || op.kind == kTBinary; };
  auto same_shape = [&](int u, int v) {
    for (int d = 0; d < kTileRank; ++d)
      if (a.vals[u].shape[d] != a.vals[v].shape[d]) return false;
    return true;
  };
  // Shared memory read and written since the last barrier.  A unit (one op,
  // or a run of elementwise ops in one pass) needs a barrier before it only
  // when it writes what was read or written since, or reads what was
  // written since: its threads may touch other elements than the threads
  // that did.
  struct Span {
    int64_t lo, hi;
  };
  std::vector<Span> rd, wr;
  auto span = [&](int v) {
    const TileGeom g = value_geom(v);
    return Span{g.off, g.off + g.rows() * g.st[2]};
  };
  const Span scratch{red_offset(a), red_offset(a) + 2 * th};
  auto hits = [](const std::vector<Span>& xs, const std::vector<Span>& ys) {
    for (const Span& x : xs)
      for (const Span& y : ys)
        if (x.lo < y.hi && y.lo < x.hi) return true;
    return false;
  };
  for (int o = 0; o < a.n_ops;) {
    const TileOp& op = a.ops[o];
    const int end = elementwise(op) ? elementwise_run(a, o, compact, elementwise, same_shape, reads) : o + 1;
    std::vector<Span> r_u, w_u;
    if (elementwise(op)) {
      std::set<int> made;
      for (int j = o; j < end; ++j) {
        for (int x : reads(a.ops[j]))
          if (!made.count(x)) r_u.push_back(span(x));
        made.insert(a.ops[j].dst);
        bool later = false;
        for (int r : readers[a.ops[j].dst]) later = later || r >= end;
        if (later) w_u.push_back(span(a.ops[j].dst));
      }
    } else {
      for (int x : reads(op)) r_u.push_back(span(x));
      if (op.kind != kTStore) w_u.push_back(span(op.dst));
      // global arrays as spans below shared memory: a store orders against
      // an earlier load or store of the same array by the Block's threads
      const Span array{-2 - 2 * static_cast<int64_t>(op.arg), -1 - 2 * static_cast<int64_t>(op.arg)};
      if (op.kind == kTLoad) r_u.push_back(array);
      if (op.kind == kTStore) w_u.push_back(array);
      if (op.kind == kTReduce) {
        const TileVal &dv = a.vals[op.dst], &xv = a.vals[op.a];
        const int64_t outs = static_cast<int64_t>(dv.numel);
        if (reduce_parts(outs, xv.shape[op.axis], th) > 1) {
          r_u.push_back(scratch);
          w_u.push_back(scratch);
        }
      }
    }
    if (o > 0 && (hits(w_u, rd) || hits(w_u, wr) || hits(r_u, wr))) {
      s << "  __syncthreads();\n";
      rd.clear();
      wr.clear();
    }
    rd.insert(rd.end(), r_u.begin(), r_u.end());
    wr.insert(wr.end(), w_u.begin(), w_u.end());
    if (elementwise(op)) {
      emit_elementwise(s, a, o, end, th, compact, readers);
      o = end;
      continue;
    }
    s << "  {  // op " << o << "\n";
    switch (op.kind) {
      case kTLoad: {
        const TileGeom v = value_geom(op.dst);
        const Access g = access_of(a, op, v, o);
        s << g.decl << "    const xt_i64 gb = " << g.base << ";\n";
        if (g.vec) {
          s << "    if (V) {\n";
          emit_load(s, a, op, v, g, th, true);
          s << "    } else {\n";
        }
        emit_load(s, a, op, v, g, th, false);
        if (g.vec) s << "    }\n";
        break;
      }
      case kTStore: {
        const TileGeom v = value_geom(op.a);
        const Access g = access_of(a, op, v, o);
        int64_t rd[kTileRank], rd_off;
        if (op.code == 1) {
          const TileGeom src = value_geom(op.b);
          rd_off = src.off;
          for (int d = 0; d < kTileRank; ++d) rd[d] = src.st[op.perm[d]];
        } else {
          rd_off = v.off;
          for (int d = 0; d < kTileRank; ++d) rd[d] = v.st[d];
        }
        s << g.decl << "    const xt_i64 gb = " << g.base << ";\n";
        if (g.vec) {
          s << "    if (V) {\n";
          emit_store(s, a, op, v, rd_off, rd, g, th, true);
          s << "    } else {\n";
        }
        emit_store(s, a, op, v, rd_off, rd, g, th, false);
        if (g.vec) s << "    }\n";
        break;
      }
      case kTReduce: {
        const TileGeom d = value_geom(op.dst), x = value_geom(op.a);
        if (op.axis >= kTileRank) fail("reduction axis");
        const int64_t n = x.s[op.axis], step = x.st[op.axis], outs = d.rows() * d.s[3];
        const bool sum = op.code != 0;
        const int64_t parts = reduce_parts(outs, n, th);
        // output o: row q, column c; the reduced dim's index is 0 in its multi-index
        const std::string at = "        const int q = o / " + std::to_string(d.s[3]) + ", c = o % " +
                               std::to_string(d.s[3]) + "; " + row_index(d.s, "q") + "\n" +
                               "        const float* src = xt_sm + " + std::to_string(x.off) + " + " + dot(x.st, d.s) + ";\n";
        const std::string put = "        xt_sm[" + std::to_string(d.off) + " + q * " + std::to_string(d.st[2]) + " + c] = ";
        if (parts == 1) {
          s << "#pragma unroll 2\n    for (int o = t; o < " << outs << "; o += " << th << ") {\n" << at;
          emit_accumulate(s, sum, n, step, 1, "0");
          s << put << (sum ? "static_cast<float>(acc);\n" : "acc;\n") << "    }\n";
          break;
        }
        if (parts >= 32 && op.axis == kTileRank - 1) {
          // Few outputs along rows (a softmax's row max and sum): an output's
          // parts in whole warps, each warp reading consecutive words of one
          // row, combined by a fixed shuffle tree and then across warps
          // through shared memory.  (With fewer parts, several rows would
          // share a warp and their words, a row pitch apart, would collide
          // in the same banks.)
          const int64_t lanes = 32, warps = parts / lanes;
          const char* T = sum ? "double" : "float";
          const char* ident = sum ? "0.0" : "__int_as_float(0xff800000)";
          auto comb = [&](const std::string& x, const std::string& y) {
            return sum ? x + " + " + y : "xt_max_nan(" + x + ", " + y + ")";
          };
          s << "    {\n      const int o = t / " << parts << ", part = t % " << parts << ";\n"
            << "      " << T << " part_acc = " << ident << ";\n"
            << "      if (o < " << outs << ") {\n" << at;
          emit_accumulate(s, sum, n, step, parts, "part");
          s << "        part_acc = acc;\n      }\n"
            << "#pragma unroll\n      for (int off = 1; off < " << lanes << "; off <<= 1)\n"
            << "        part_acc = " << comb("part_acc", "__shfl_xor_sync(0xffffffffu, part_acc, off)") << ";\n";
          if (warps == 1) {
            s << "      if (o < " << outs << " && part == 0) {\n        const int q = o / " << d.s[3] << ", c = o % "
              << d.s[3] << ";\n        const " << T << " acc = part_acc;\n"
              << put << (sum ? "static_cast<float>(acc);\n" : "acc;\n") << "      }\n    }\n";
          } else {
            const char* red = sum ? "xt_red_f64" : "xt_red_f32";
            s << "      if (o < " << outs << " && (part & 31) == 0) " << red << "[o * " << warps << " + part / 32] = part_acc;\n"
              << "      __syncthreads();\n"
              << "      if (t < " << outs << ") {\n        const int o = t, q = o / " << d.s[3] << ", c = o % " << d.s[3]
              << ";\n        " << T << " acc = " << red << "[o * " << warps << "];\n"
              << "#pragma unroll\n        for (int k = 1; k < " << warps << "; ++k) acc = "
              << comb("acc", std::string(red) + "[o * " + std::to_string(warps) + " + k]") << ";\n"
              << put << (sum ? "static_cast<float>(acc);\n" : "acc;\n") << "      }\n    }\n";
          }
          break;
        }
        // ``parts`` threads per output, each over every parts-th element from
        // its own; their partial results combine in a fixed order
        s << "    {\n      const int o = t % " << outs << ", part = t / " << outs << ";\n"
          << "      if (part < " << parts << ") {\n" << at;
        emit_accumulate(s, sum, n, step, parts, "part");
        s << "        " << (sum ? "xt_red_f64" : "xt_red_f32") << "[part * " << outs << " + o] = acc;\n      }\n"
          << "      __syncthreads();\n"
          << "      if (t < " << outs << ") {\n        const int o = t, q = o / " << d.s[3] << ", c = o % " << d.s[3]
          << ";\n        " << (sum ? "double" : "float") << " acc = " << (sum ? "xt_red_f64" : "xt_red_f32") << "[o];\n"
          << "#pragma unroll\n        for (int k = 1; k < " << parts << "; ++k) "
          << (sum ? "acc += xt_red_f64[k * " + std::to_string(outs) + " + o];\n"
                  : "acc = xt_max_nan(acc, xt_red_f32[k * " + std::to_string(outs) + " + o]);\n")
          << put << (sum ? "static_cast<float>(acc);\n" : "acc;\n") << "      }\n    }\n";
        break;
      }
      case kTReshape: {
        const TileGeom d = value_geom(op.dst), x = value_geom(op.a);
        std::ostringstream b;
        b << "        const int e = q * " << d.s[3] << " + cv;\n"
          << "        xt_sm[" << d.off << " + q * " << d.st[2] << " + cv] = xt_sm[" << x.off << " + e / " << x.s[3]
          << " * " << x.st[2] << " + e % " << x.s[3] << "];\n";
        loop_rows(s, th, d.rows(), d.s[3], b.str());
        break;
      }
      case kTPermute: {
        const TileGeom d = value_geom(op.dst), x = value_geom(op.a);
        // dst dim k is src dim perm[k]
        int64_t ss[kTileRank];
        for (int k = 0; k < kTileRank; ++k) ss[k] = x.st[op.perm[k]];
        std::ostringstream b;
        b << "        const int c = cv; " << row_index(d.s, "q") << "\n"
          << "        xt_sm[" << d.off << " + q * " << d.st[2] << " + c] = xt_sm[" << x.off << " + " << dot(ss, d.s) << "];\n";
        loop_rows(s, th, d.rows(), d.s[3], b.str());
        break;
      }
      default:
        fail("tile op kind " + std::to_string(op.kind));
    }
    s << "  }\n";
    ++o;
  }
  s << "}\n";
  for (int v = 1; v >= 0; --v)
    s << "extern \"C\" __global__ void __launch_bounds__(" << th << ") " << (v ? "xt_tile_v" : "xt_tile_s")
      << "(const XtTileArgs p) {\n  xt_pdl_launch();\n  xt_pdl_wait();\n  xt_tile_body<" << (v ? "true" : "false")
      << ">(p);\n}\n";
  return s.str();
}
}  // namespace jit
}  // namespace xt
