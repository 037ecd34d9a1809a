// Elementwise and row-program kernels (HBM-bound families).
//
// ew:   a flat map over arrays of identical shape.  A single binary
//       add/sub/mul of two f32 arrays (the kernels/add.py pattern) runs in a
//       dedicated 128-bit vector kernel; any other register program runs in
//       a kernel generated for it at run time (codegen.h).
// rows: programs over whole rows (one warp per row, the row held in
//       registers, warp-shuffle reductions).  The softmax chain
//       max -> sub -> exp -> sum -> reciprocal -> mul (kernels/softmax.py,
//       xtile/dsl.py:354-357) has a dedicated kernel; other row programs run
//       in a generated kernel, or, when their live rows exceed the register
//       file, in the shared-memory interpreter below.
//
// f32 arithmetic is IEEE round-to-nearest with no contraction (the __f*_rn
// intrinsics), so add/sub/mul/reciprocal/rsqrt match the CPU oracle bit for bit.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../kernels.h"
#include "elem_ops.cuh"
#include "pdl.cuh"
#include "../codegen.h"

namespace xt {
namespace dev {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------------------
// ew: dedicated f32 binary kernel
// ---------------------------------------------------------------------------
template <int OP>
__global__ void __launch_bounds__(kThreads) ew_binary_f32(const float* __restrict__ a,
                                                           const float* __restrict__ b,
                                                           float* __restrict__ c, int64_t n4,
                                                           int64_t n) {
  // One 16-byte vector per operand per thread over a grid that covers the
  // array (the loop only runs again past the grid-size limit): every load is
  // issued at kernel start, which measured faster on this HBM-bound op than
  // a persistent grid-stride loop with two vectors in flight per thread.
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kThreads;
  if (threadIdx.x == 0 && first < n4) {
    // this CTA's first vectors of both operands into L2 while the previous launch drains
    const uint32_t bytes = static_cast<uint32_t>((n4 - first < kThreads ? n4 - first : kThreads) * 16);
    prefetch_l2(a4 + first, bytes);
    prefetch_l2(b4 + first, bytes);
  }
  griddep_launch_dependents();
  griddep_wait();
  float4* c4 = reinterpret_cast<float4*>(c);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += stride) {
    const float4 x = __ldcs(a4 + i), y = __ldcs(b4 + i);
    float4 r;
    r.x = binary_op(OP, x.x, y.x); r.y = binary_op(OP, x.y, y.y);
    r.z = binary_op(OP, x.z, y.z); r.w = binary_op(OP, x.w, y.w);
    __stcs(c4 + i, r);
  }
  // scalar tail (n not a multiple of 4)
  if (blockIdx.x == 0 && threadIdx.x < n - n4 * 4) {
    const int64_t t = n4 * 4 + threadIdx.x;
    c[t] = binary_op(OP, a[t], b[t]);
  }
}

// ---------------------------------------------------------------------------
// register selection and float4 op dispatch of the rows interpreter
// ---------------------------------------------------------------------------
template <int N>
__device__ __forceinline__ float pick(const float (&r)[N], int idx) {
  float v = 0.0f;
#pragma unroll
  for (int k = 0; k < N; ++k) v = (k == idx) ? r[k] : v;
  return v;
}

template <int N>
__device__ __forceinline__ void put(float (&r)[N], int idx, float v) {
#pragma unroll
  for (int k = 0; k < N; ++k) r[k] = (k == idx) ? v : r[k];
}

template <uint8_t OP>
__device__ __forceinline__ float4 unary4_of(float4 x) {
  return make_float4(unary_op(OP, x.x), unary_op(OP, x.y), unary_op(OP, x.z), unary_op(OP, x.w));
}

// unary_op on four values with one dispatch on the (warp-uniform) opcode
__device__ __forceinline__ float4 unary4(uint8_t op, float4 x) {
  switch (op & 0x7f) {
    case kExp: return unary4_of<kExp>(x);
    case kCos: return unary4_of<kCos>(x);
    case kSin: return unary4_of<kSin>(x);
    case kRecip: return unary4_of<kRecip>(x);
    case kRsqrt: return unary4_of<kRsqrt>(x);
    case kSigmoid: return unary4_of<kSigmoid>(x);
    case kTanh: return unary4_of<kTanh>(x);
    case kSilu: return unary4_of<kSilu>(x);
    case kFtoi: return unary4_of<kFtoi>(x);
    default: return x;
  }
}

template <uint8_t OP>
__device__ __forceinline__ float4 binary4_of(float4 x, float4 y) {
  return make_float4(binary_op(OP, x.x, y.x), binary_op(OP, x.y, y.y), binary_op(OP, x.z, y.z),
                     binary_op(OP, x.w, y.w));
}

__device__ __forceinline__ float4 binary4(uint8_t op, float4 x, float4 y) {
  switch (op & 0x7f) {
    case kAdd: case kBcastAdd: return binary4_of<kAdd>(x, y);
    case kSub: case kBcastSub: return binary4_of<kSub>(x, y);
    default: return binary4_of<kMul>(x, y);
  }
}

// ---------------------------------------------------------------------------
// rows: dedicated softmax kernel.  One warp per row; lane l holds float4
// chunks l, l+32, l+64, ... of the row (coalesced 512-byte warp accesses).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// CHUNKS float4 chunks per lane: row length <= 128 * CHUNKS.  FULL: the row
// is exactly 128 * CHUNKS long, so the exp and store loops need no column
// guard.  The loads keep theirs: in that form (80 registers, 3 CTAs per SM)
// the 8-chunk kernel measured 11.0 us on the 8192 x 1024 softmax, against
// 11.7 us with every guard (61 registers, 4 CTAs per SM) and 12.5 us with
// registers capped at 40 for 6 CTAs per SM (one B200, CUDA-graph replay over
// rotating buffers).
//
// Up to 8 chunks the launch bound names one CTA per SM as the minimum, which
// leaves ptxas free to keep every chunk's exp in flight (without a minimum it
// held the 8-chunk kernel to 48 registers).  The 16-chunk kernel would then
// take 168 registers, one CTA per SM, so it asks for three.
template <int CHUNKS, bool FULL>
__global__ void __launch_bounds__(kThreads, CHUNKS <= 8 ? 1 : 3) softmax_rows_vec4(const float* __restrict__ x,
                                                               float* __restrict__ y, int64_t row_begin,
                                                               int64_t row_end, int64_t cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = row_begin + static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  if (lane == 0 && row < row_end && (cols & 3) == 0)
    prefetch_l2(x + row * cols, static_cast<uint32_t>(cols * 4));  // this warp's row into L2 (see pdl.cuh)
  griddep_launch_dependents();
  if (row >= row_end) return;
  griddep_wait();
  const int64_t c4 = cols >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + row * cols);
  float4* yr = reinterpret_cast<float4*>(y + row * cols);
  float4 v[CHUNKS];
#pragma unroll
  for (int j = 0; j < CHUNKS; ++j) {
    const int64_t idx = j * 32 + lane;
    v[j] = idx < c4 ? __ldcs(xr + idx) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  }
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < CHUNKS; ++j) m = fmaxf(fmaxf(fmaxf(m, v[j].x), fmaxf(v[j].y, v[j].z)), v[j].w);
  m = warp_max(m);
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < CHUNKS; ++j) {
    const int64_t idx = j * 32 + lane;
    if (FULL || idx < c4) {
      v[j].x = expf(__fsub_rn(v[j].x, m));
      v[j].y = expf(__fsub_rn(v[j].y, m));
      v[j].z = expf(__fsub_rn(v[j].z, m));
      v[j].w = expf(__fsub_rn(v[j].w, m));
      s = __fadd_rn(s, __fadd_rn(__fadd_rn(v[j].x, v[j].y), __fadd_rn(v[j].z, v[j].w)));
    }
  }
  s = warp_sum(s);
  const float inv = __frcp_rn(s);
#pragma unroll
  for (int j = 0; j < CHUNKS; ++j) {
    const int64_t idx = j * 32 + lane;
    if (FULL || idx < c4) {
      float4 o;
      o.x = __fmul_rn(v[j].x, inv);
      o.y = __fmul_rn(v[j].y, inv);
      o.z = __fmul_rn(v[j].z, inv);
      o.w = __fmul_rn(v[j].w, inv);
      __stcs(yr + idx, o);
    }
  }
}

// ---------------------------------------------------------------------------
// rows: register-program interpreter
// ---------------------------------------------------------------------------
constexpr int kRowS = 8;

// One warp per row; lane l holds the float4 chunks l, l + 32, ... (elements
// 4c .. 4c + 3 of chunk c) of each row register.  The row registers live in
// shared memory, one float4 slot per register, chunk and lane, so an operand
// is read at a computed address rather than selected out of every register;
// scalar registers (one value per row) stay in registers.  VEC: rows of a
// multiple of 4 columns at 16-byte aligned addresses, accessed as float4;
// otherwise element by element with a guard on each element.  A first form
// held the row registers in registers (3 x 32 values per lane at 1024
// columns, 224 registers, one CTA per SM) and measured 684 GB/s on a
// max-centre-square program over 128 MiB; this one 4297 GB/s.  The launch
// bound asks for four CTAs per SM (without a minimum ptxas held the 8-chunk
// kernel to 32 registers and spilled).
constexpr int kRowMaxThreads = 128;

template <int PL4, bool VEC>  // float4 chunks per lane: row length <= 128 * PL4
__global__ void __launch_bounds__(kRowMaxThreads, 4) rows_program(const __grid_constant__ RowArgs p) {
  extern __shared__ float4 row_rf[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = p.row_begin + static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + warp;
  griddep_launch_dependents();
  if (row >= p.row_end) return;
  griddep_wait();
  float4* rf = row_rf + warp * (p.n_vregs * PL4 * 32) + lane;  // register k, chunk j: rf[(k * PL4 + j) * 32]
  const int64_t cols = p.cols, c4n = (cols + 3) >> 2;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float s[kRowS];
#pragma unroll
  for (int k = 0; k < kRowS; ++k) s[k] = 0.0f;
  for (int pc = 0; pc < p.n_code; ++pc) {
    const Instr ins = p.code[pc];
    const uint8_t op = ins.op & 0x7f;
    const bool scalar = ins.op & 0x80;
    if (op == kLoad) {
      const float* src = p.in[ins.a] + row * cols;
      float4 t[PL4];
#pragma unroll
      for (int j = 0; j < PL4; ++j) {
        const int64_t c = j * 32 + lane;
        if (VEC) {
          t[j] = c < c4n ? __ldg(reinterpret_cast<const float4*>(src) + c) : zero;
        } else {
          const int64_t e = 4 * c;
          t[j] = make_float4(e < cols ? __ldg(src + e) : 0.f, e + 1 < cols ? __ldg(src + e + 1) : 0.f,
                             e + 2 < cols ? __ldg(src + e + 2) : 0.f, e + 3 < cols ? __ldg(src + e + 3) : 0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < PL4; ++j) rf[(ins.dst * PL4 + j) * 32] = t[j];
    } else if (op == kLoadScalar) {
      put(s, ins.dst, __ldg(p.in[ins.a] + row));
    } else if (op == kStore) {
      float* dst = p.out[ins.dst] + row * cols;
#pragma unroll
      for (int j = 0; j < PL4; ++j) {
        const int64_t c = j * 32 + lane;
        if (c >= c4n) continue;
        const float4 v = rf[(ins.a * PL4 + j) * 32];
        if (VEC) {
          reinterpret_cast<float4*>(dst)[c] = v;
        } else {
          const int64_t e = 4 * c;
          dst[e] = v.x;
          if (e + 1 < cols) dst[e + 1] = v.y;
          if (e + 2 < cols) dst[e + 2] = v.z;
          if (e + 3 < cols) dst[e + 3] = v.w;
        }
      }
    } else if (op == kStoreScalar) {
      if (lane == 0) p.out[ins.dst][row] = pick(s, ins.a);
    } else if (op == kRowMax || op == kRowSum) {
      const bool mx = op == kRowMax;
      const float pad = mx ? -INFINITY : 0.0f;  // elements past the row end
      float acc = pad;
#pragma unroll
      for (int j = 0; j < PL4; ++j) {
        const int64_t c = j * 32 + lane;
        if (c < c4n) {
          float4 x = rf[(ins.a * PL4 + j) * 32];
          if (!VEC) {
            const int64_t e = 4 * c;
            if (e + 1 >= cols) x.y = pad;
            if (e + 2 >= cols) x.z = pad;
            if (e + 3 >= cols) x.w = pad;
          }
          acc = mx ? fmaxf(fmaxf(fmaxf(acc, x.x), fmaxf(x.y, x.z)), x.w)
                   : __fadd_rn(acc, __fadd_rn(__fadd_rn(x.x, x.y), __fadd_rn(x.z, x.w)));
        }
      }
      put(s, ins.dst, mx ? warp_max(acc) : warp_sum(acc));
    } else if (scalar) {
      const float a = pick(s, ins.a);
      put(s, ins.dst, (op == kAdd || op == kSub || op == kMul) ? binary_op(op, a, pick(s, ins.b))
                                                               : unary_op(op, a));
    } else if (op == kBcastAdd || op == kBcastSub || op == kBcastMul) {
      const float b = pick(s, ins.b);
      const float4 b4 = make_float4(b, b, b, b);
#pragma unroll
      for (int j = 0; j < PL4; ++j) rf[(ins.dst * PL4 + j) * 32] = binary4(op, rf[(ins.a * PL4 + j) * 32], b4);
    } else if (op == kAdd || op == kSub || op == kMul) {
#pragma unroll
      for (int j = 0; j < PL4; ++j)
        rf[(ins.dst * PL4 + j) * 32] = binary4(op, rf[(ins.a * PL4 + j) * 32], rf[(ins.b * PL4 + j) * 32]);
    } else {
#pragma unroll
      for (int j = 0; j < PL4; ++j) rf[(ins.dst * PL4 + j) * 32] = unary4(op, rf[(ins.a * PL4 + j) * 32]);
    }
  }
}

int grid_for(int64_t work_items, int per_block, int max_blocks) {
  int64_t b = (work_items + per_block - 1) / per_block;
  if (b < 1) b = 1;
  return static_cast<int>(b < max_blocks ? b : max_blocks);
}

int sm_count() {
  static int n = [] {
    int dev = 0, v = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

}  // namespace

cudaError_t launch_ew(const EwArgs& a, cudaStream_t stream) {
  const int64_t n = a.end - a.begin;
  if (n <= 0) return cudaSuccess;
  const int max_blocks = sm_count() * 8;
  // dedicated path: out = in0 (op) in1, all f32, 16-byte aligned
  if (a.n_code == 4 && a.n_in == 2 && a.n_out == 1 && !a.in_bcast[0] && !a.in_bcast[1] &&
      a.code[0].op == kLoad && a.code[1].op == kLoad &&
      a.code[3].op == kStore && a.code[3].a == a.code[2].dst && a.in_elem[0] == kF32 &&
      a.in_elem[1] == kF32 && a.out_elem[0] == kF32 &&
      (a.code[2].op == kAdd || a.code[2].op == kSub || a.code[2].op == kMul) && a.begin % 4 == 0) {
    const bool swap = a.code[2].a == a.code[1].dst;  // operand order of the op
    const float* x = static_cast<const float*>(a.in[swap ? 1 : 0]) + a.begin;
    const float* y = static_cast<const float*>(a.in[swap ? 0 : 1]) + a.begin;
    float* z = static_cast<float*>(a.out[0]) + a.begin;
    if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(z)) &
         15) == 0) {
      const int64_t n4 = n / 4;
      const int blocks = grid_for(n4 > 0 ? n4 : 1, kThreads, 0x7fffffff);
      PdlLaunch launch(blocks, kThreads, 0, stream);
      switch (a.code[2].op) {
        case kAdd: return launch(ew_binary_f32<kAdd>, x, y, z, n4, n);
        case kSub: return launch(ew_binary_f32<kSub>, x, y, z, n4, n);
        default: return launch(ew_binary_f32<kMul>, x, y, z, n4, n);
      }
    }
  }
  // every other program: its own kernel, generated and compiled at run time
  (void)max_blocks;
  return jit::launch_ew(a, stream);
}

cudaError_t launch_rows(const RowArgs& a, cudaStream_t stream) {
  const int64_t rows = a.row_end - a.row_begin;
  if (rows <= 0) return cudaSuccess;
  const int rows_per_block = kThreads / 32;
  const int blocks = static_cast<int>((rows + rows_per_block - 1) / rows_per_block);
  bool aligned = a.cols % 4 == 0 && ((reinterpret_cast<uintptr_t>(a.in[0]) |
                                      reinterpret_cast<uintptr_t>(a.out[0])) & 15) == 0;
  if (a.softmax && aligned) {
    const int64_t chunks = (a.cols / 4 + 31) / 32;
    const float* x = a.in[0];
    float* y = a.out[0];
    PdlLaunch launch(blocks, kThreads, 0, stream);
    auto go = [&](auto full_kernel, auto ragged_kernel, int64_t ch) {
      return a.cols == 128 * ch ? launch(full_kernel, x, y, a.row_begin, a.row_end, a.cols)
                                : launch(ragged_kernel, x, y, a.row_begin, a.row_end, a.cols);
    };
    if (chunks <= 1) return go(softmax_rows_vec4<1, true>, softmax_rows_vec4<1, false>, 1);
    if (chunks <= 2) return go(softmax_rows_vec4<2, true>, softmax_rows_vec4<2, false>, 2);
    if (chunks <= 4) return go(softmax_rows_vec4<4, true>, softmax_rows_vec4<4, false>, 4);
    if (chunks <= 8) return go(softmax_rows_vec4<8, true>, softmax_rows_vec4<8, false>, 8);
    return go(softmax_rows_vec4<16, true>, softmax_rows_vec4<16, false>, 16);
  }
  // other row programs: their own kernel, generated and compiled at run time,
  // when the program's row registers fit the register file; wider ones (three
  // live rows of more than 1024 columns) run the shared-memory interpreter
  if (jit::rows_fit(a)) return jit::launch_rows(a, stream);
  bool vec = a.cols % 4 == 0;
  for (int k = 0; k < kMaxSlots && vec; ++k) {
    if (a.in[k] && !a.in_scalar[k]) vec = (reinterpret_cast<uintptr_t>(a.in[k]) & 15) == 0;
    if (vec && a.out[k] && !a.out_scalar[k]) vec = (reinterpret_cast<uintptr_t>(a.out[k]) & 15) == 0;
  }
  const int64_t pl4 = ((a.cols + 3) / 4 + 31) / 32;
  const int nv = a.n_vregs > 0 ? a.n_vregs : 1;
  auto go = [&](auto vec_kernel, auto any_kernel, int pl4c) {
    // rows per CTA: four, two for 2048-column rows (48 KiB of row registers at most)
    const int rpb = pl4c <= 8 ? 4 : 2;
    const int vblocks = static_cast<int>((rows + rpb - 1) / rpb);
    const size_t smem = static_cast<size_t>(rpb) * nv * pl4c * 32 * sizeof(float4);
    PdlLaunch launch(vblocks, rpb * 32, smem, stream);
    return vec ? launch(vec_kernel, a) : launch(any_kernel, a);
  };
  if (pl4 <= 1) return go(rows_program<1, true>, rows_program<1, false>, 1);
  if (pl4 <= 2) return go(rows_program<2, true>, rows_program<2, false>, 2);
  if (pl4 <= 4) return go(rows_program<4, true>, rows_program<4, false>, 4);
  if (pl4 <= 8) return go(rows_program<8, true>, rows_program<8, false>, 8);
  if (pl4 <= 16) return go(rows_program<16, true>, rows_program<16, false>, 16);
  return cudaErrorInvalidValue;  // the planner admits rows up to 2048
}

}  // namespace dev
}  // namespace xt
