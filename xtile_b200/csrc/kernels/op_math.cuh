// The xt element operations on f32 values, and the element conversions of
// f32, bf16 and int8 arrays: the one definition shared by the compiled
// kernels (elem_ops.cuh) and the kernels generated per program at run time
// (codegen.cpp embeds this file's text in every generated source and
// compiles it with NVRTC).  Self-contained: no includes, CUDA built-ins only.
//
// f32 arithmetic is IEEE round-to-nearest with no contraction (the __f*_rn
// intrinsics), so add/sub/mul/reciprocal/rsqrt match the CPU oracle bit for
// bit; ftoi rounds half to even and saturates to [-128, 127], NaN -> 0.
// Unary ops the reference never lowers (cos, sin, sigmoid, tanh, silu) use
// their mathematical definitions through CUDA's f32 math functions.
#pragma once

__device__ __forceinline__ float xt_exp(float x) { return expf(x); }
__device__ __forceinline__ float xt_cos(float x) { return cosf(x); }
__device__ __forceinline__ float xt_sin(float x) { return sinf(x); }
__device__ __forceinline__ float xt_recip(float x) { return __frcp_rn(x); }
__device__ __forceinline__ float xt_rsqrt(float x) { return __frcp_rn(__fsqrt_rn(x)); }
__device__ __forceinline__ float xt_sigmoid(float x) { return __frcp_rn(__fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float xt_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ float xt_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float xt_itof(float x) { return x; }
__device__ __forceinline__ float xt_ftoi(float x) { return x != x ? 0.0f : fminf(fmaxf(rintf(x), -128.0f), 127.0f); }
__device__ __forceinline__ float xt_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float xt_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float xt_mul(float a, float b) { return __fmul_rn(a, b); }

// bf16 <-> f32: a bf16 value is the high half of an f32; f32 -> bf16 rounds
// to nearest even (the hardware conversion; NaN stays NaN).
__device__ __forceinline__ float xt_bf16_bits_to_f32(unsigned int bits16) { return __uint_as_float(bits16 << 16); }
__device__ __forceinline__ unsigned int xt_f32_to_bf16_bits(float x) {
  unsigned short r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(x));
  return r;
}
// int8 storage of a value the program holds as f32: truncation to an
// integer, then the low 8 bits (int8 add / sub / mul wrap modulo 256)
__device__ __forceinline__ unsigned int xt_f32_to_i8_bits(float x) {
  return static_cast<unsigned int>(static_cast<unsigned char>(static_cast<signed char>(static_cast<int>(x))));
}
