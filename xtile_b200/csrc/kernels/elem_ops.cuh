// Scalar element operations of the compiled interpreter kernels (tile, and
// the ew / rows forms compiled ahead of time): the xt unary and binary ops on
// f32 values, dispatched on an opcode, and element loads/stores of f32, bf16
// and int8 arrays.  The arithmetic itself is op_math.cuh's, shared with the
// kernels generated per program at run time.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../kernels.h"
#include "op_math.cuh"

namespace xt {
namespace dev {

__device__ __forceinline__ float unary_op(uint8_t op, float x) {
  switch (op & 0x7f) {
    case kExp: return xt_exp(x);
    case kCos: return xt_cos(x);
    case kSin: return xt_sin(x);
    case kRecip: return xt_recip(x);
    case kRsqrt: return xt_rsqrt(x);
    case kSigmoid: return xt_sigmoid(x);
    case kTanh: return xt_tanh(x);
    case kSilu: return xt_silu(x);
    case kItof: return xt_itof(x);
    case kFtoi: return xt_ftoi(x);
    default: return x;
  }
}

__device__ __forceinline__ float binary_op(uint8_t op, float a, float b) {
  switch (op & 0x7f) {
    case kAdd: case kBcastAdd: return xt_add(a, b);
    case kSub: case kBcastSub: return xt_sub(a, b);
    case kMul: case kBcastMul: return xt_mul(a, b);
    default: return a;
  }
}

__device__ __forceinline__ float load_elem(const void* p, uint8_t e, int64_t i) {
  if (e == kF32) return __ldg(static_cast<const float*>(p) + i);
  if (e == kBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return static_cast<float>(static_cast<const int8_t*>(p)[i]);
}

__device__ __forceinline__ void store_elem(void* p, uint8_t e, int64_t i, float v) {
  if (e == kF32) static_cast<float*>(p)[i] = v;
  else if (e == kBF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<int8_t*>(p)[i] = static_cast<int8_t>(static_cast<int>(v));
}

}  // namespace dev
}  // namespace xt
