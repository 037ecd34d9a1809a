// Scalar element operations shared by the interpreter kernels (ew, rows,
// tile): the xt unary and binary ops on f32 values and element loads/stores
// of f32, bf16 and int8 arrays.
//
// f32 arithmetic is IEEE round-to-nearest with no contraction (the __f*_rn
// intrinsics), so add/sub/mul/reciprocal/rsqrt match the CPU oracle bit for
// bit; ftoi rounds half to even and saturates to [-128, 127], NaN -> 0.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../kernels.h"

namespace xt {
namespace dev {

__device__ __forceinline__ float unary_op(uint8_t op, float x) {
  switch (op & 0x7f) {
    case kExp: return expf(x);
    case kCos: return cosf(x);
    case kSin: return sinf(x);
    case kRecip: return __frcp_rn(x);
    case kRsqrt: return __frcp_rn(__fsqrt_rn(x));
    case kSigmoid: return __frcp_rn(__fadd_rn(1.0f, expf(-x)));
    case kTanh: return tanhf(x);
    case kSilu: return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
    case kItof: return x;
    case kFtoi: return x != x ? 0.0f : fminf(fmaxf(rintf(x), -128.0f), 127.0f);
    default: return x;
  }
}

__device__ __forceinline__ float binary_op(uint8_t op, float a, float b) {
  switch (op & 0x7f) {
    case kAdd: case kBcastAdd: return __fadd_rn(a, b);
    case kSub: case kBcastSub: return __fsub_rn(a, b);
    case kMul: case kBcastMul: return __fmul_rn(a, b);
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
