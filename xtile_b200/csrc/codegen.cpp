// Source generation for the per-program ew and rows kernels (codegen.h).
//
// The generated text is the register program of plan.h written out: every
// program register becomes a local variable (an array of float4 groups in
// the vector kernels), every instruction one statement applying the
// op_math.cuh function, whose text is embedded at the top of each source.
// The semantics are therefore those of the compiled interpreters, op for op;
// what changes is that nothing is decoded or dispatched per element and the
// values stay in registers.
#include "codegen.h"

#include <algorithm>
#include <set>
#include <sstream>

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

// the rows program; ``vec``: float4 chunks (cols % 4 == 0), else elements
void rows_body(std::ostringstream& s, const dev::RowArgs& a, bool vec) {
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
  const std::string idx = vec ? "const int c = j * 32 + lane; const bool in = c < XT_C4;"
                              : "const int c = j * 32 + lane; const bool in = c < XT_COLS;";
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
      s << "    s" << d << " = " << (mx ? "xt_warp_max" : "xt_warp_sum") << "(acc);\n  }\n";
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

bool rows_fit(const dev::RowArgs& a) {
  // values a lane holds for the program's row registers
  const int64_t n_v = std::max(a.n_vregs, 1);
  return n_v * 4 * rows_pl4(a.cols) <= 160 && n_v * rows_pls(a.cols) <= 160;
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
    rows_body(s, a, vec == 1);
    s << "}\n";
  }
  return s.str();
}

}  // namespace jit
}  // namespace xt
