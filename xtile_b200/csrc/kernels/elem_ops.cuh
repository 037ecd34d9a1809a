// Scalar element operations of the compiled kernels (the dedicated f32
// add/sub/mul kernel): the xt unary and binary ops on f32 values, dispatched
// on an opcode.  The arithmetic itself is op_math.cuh's, shared with the
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

}  // namespace dev
}  // namespace xt
