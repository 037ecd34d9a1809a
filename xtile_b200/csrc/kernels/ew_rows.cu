// Elementwise and row-program kernels (HBM-bound families).
//
// ew:   a flat map over arrays of identical shape.  A single binary
//       add/sub/mul of two f32 arrays (the kernels/add.py pattern) runs in a
//       dedicated 128-bit vector kernel; any other register program runs in
//       a kernel generated for it at run time (codegen.h).
// rows: programs over whole rows (the row held in registers).  The softmax
//       chain max -> sub -> exp -> sum -> reciprocal -> mul
//       (kernels/softmax.py, xtile/dsl.py:354-357) on rows of at most 2048
//       columns has a dedicated kernel (one warp per row, warp-shuffle
//       reductions); other row programs run in a kernel generated for them
//       (one warp per row, or one CTA per row for wide rows).
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
// the dedicated f32 add/sub/mul kernel (2048^2 add over 200 graph-replayed
// launches: 6200-6209 GB/s with 256 threads, 5584 with 128)
constexpr int kAddThreads = 256;

// ---------------------------------------------------------------------------
// ew: dedicated f32 binary kernel
// ---------------------------------------------------------------------------
template <int OP>
__global__ void __launch_bounds__(kAddThreads) ew_binary_f32(const float* __restrict__ a,
                                                           const float* __restrict__ b,
                                                           float* __restrict__ c, int64_t n4,
                                                           int64_t n) {
  // One 16-byte vector per operand per thread over a grid that covers the
  // array (the loop only runs again past the grid-size limit): every load is
  // issued at kernel start, which measured faster on this HBM-bound op than
  // a persistent grid-stride loop with two vectors in flight per thread.
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kAddThreads;
  if (threadIdx.x == 0 && first < n4) {
    // this CTA's first vectors of both operands into L2 while the previous launch drains
    const uint32_t bytes = static_cast<uint32_t>((n4 - first < kAddThreads ? n4 - first : kAddThreads) * 16);
    prefetch_l2(a4 + first, bytes);
    prefetch_l2(b4 + first, bytes);
  }
  griddep_launch_dependents();
  griddep_wait();
  float4* c4 = reinterpret_cast<float4*>(c);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kAddThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kAddThreads + threadIdx.x; i < n4; i += stride) {
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

int grid_for(int64_t work_items, int per_block, int max_blocks) {
  int64_t b = (work_items + per_block - 1) / per_block;
  if (b < 1) b = 1;
  return static_cast<int>(b < max_blocks ? b : max_blocks);
}

}  // namespace

cudaError_t launch_ew(const EwArgs& a, cudaStream_t stream) {
  const int64_t n = a.end - a.begin;
  if (n <= 0) return cudaSuccess;
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
      const int blocks = grid_for(n4 > 0 ? n4 : 1, kAddThreads, 0x7fffffff);
      PdlLaunch launch(blocks, kAddThreads, 0, stream);
      switch (a.code[2].op) {
        case kAdd: return launch(ew_binary_f32<kAdd>, x, y, z, n4, n);
        case kSub: return launch(ew_binary_f32<kSub>, x, y, z, n4, n);
        default: return launch(ew_binary_f32<kMul>, x, y, z, n4, n);
      }
    }
  }
  // every other program: its own kernel, generated and compiled at run time
  return jit::launch_ew(a, stream);
}

cudaError_t launch_rows(const RowArgs& a, cudaStream_t stream) {
  const int64_t rows = a.row_end - a.row_begin;
  if (rows <= 0) return cudaSuccess;
  const int rows_per_block = kThreads / 32;
  const int blocks = static_cast<int>((rows + rows_per_block - 1) / rows_per_block);
  bool aligned = a.cols % 4 == 0 && ((reinterpret_cast<uintptr_t>(a.in[0]) |
                                      reinterpret_cast<uintptr_t>(a.out[0])) & 15) == 0;
  if (a.softmax && aligned && a.cols <= 2048) {
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
  // other row programs: their own kernel, generated and compiled at run time
  // (one warp per row, or one CTA per row for wide rows)
  return jit::launch_rows(a, stream);
}

}  // namespace dev
}  // namespace xt
