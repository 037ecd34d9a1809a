// Device-side entry points of the B200 kernels and their launch arguments.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "plan.h"

namespace xt {
namespace dev {

// Element storage codes used inside kernels.
enum ElemCode : uint8_t { kF32 = 0, kBF16 = 1, kI8 = 2 };

// ------------------------------------------------------------------ ew
struct EwArgs {
  const void* in[kMaxSlots];
  void* out[kMaxSlots];
  uint8_t in_elem[kMaxSlots];
  uint8_t out_elem[kMaxSlots];
  Instr code[kMaxInstr];
  int n_code;
  int n_in, n_out;
  int64_t begin, end;        // element range [begin, end)
  uint8_t in_bcast[kMaxSlots];  // input read at element i mod bcast_period (a broadcast row)
  int64_t bcast_period;
};
cudaError_t launch_ew(const EwArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- rows
struct RowArgs {
  const float* in[kMaxSlots];
  float* out[kMaxSlots];
  uint8_t in_scalar[kMaxSlots];
  uint8_t out_scalar[kMaxSlots];
  Instr code[kMaxInstr];
  int n_code;
  int n_vregs, n_sregs;
  int64_t row_begin, row_end;  // rows [row_begin, row_end)
  int64_t cols;
  uint8_t softmax;             // run the dedicated softmax kernel
};
cudaError_t launch_rows(const RowArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- tile
struct TileArgs {
  void* arr[kTileMaxArgs];
  uint8_t elem[kTileMaxArgs];
  int32_t shape[kTileMaxArgs][kTileRank];
  TileVal vals[kTileMaxVals];
  TileOp ops[kTileMaxOps];
  int n_ops;
  int32_t smem_floats;
  int64_t grid[3];
  int64_t bid0_begin, bid0_end;  // Blocks [bid0_begin, bid0_end) along xt.bid(0)
};
cudaError_t launch_tile(const TileArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- gemm
struct GemmArgs {
  const void* A;           // [M, lda] row-major (bf16 or i8)
  const void* B;           // [K, ldb] row-major (bf16 or i8)
  void* C;                 // [M, ldc] row-major (f32 or i8)
  const float* acc;        // optional [M, ldc] f32 tile added first (xt.mma)
  int64_t M, N, K, lda, ldb, ldc;
  int64_t m_begin;         // first row of A/C this launch computes (bid0 sharding)
  uint8_t ab_elem;         // kBF16 or kI8
  uint8_t c_elem;          // kF32 or kI8
  int n_epi;
  uint8_t epi_kind[4];
  const float* epi_ptr[4];
  uint32_t* error_word;
  int max_sms;             // SMs the persistent grid may occupy (0: all)
  uint64_t wait_limit_cycles;  // SM cycles a pipeline wait may take before the kernel gives up (0: 2 s)
};
cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- conv
struct ConvArgs {
  const void* in;          // NHWC
  const void* filt;        // HWIO
  float* out;              // [N, out_h, out_w, out_c]
  int64_t N, H, W, C, KH, KW, KO;
  int64_t ON, OH, OW;      // covered output extents
  int64_t n_begin;         // first batch image (bid0 sharding)
  int64_t out_h, out_w, out_c;
  int64_t pad_t, pad_l, dil_h, dil_w;
  uint8_t elem;
  uint32_t* error_word;
  int max_sms;             // SMs the persistent grid may occupy (0: all)
  uint64_t wait_limit_cycles;  // SM cycles a pipeline wait may take before the kernel gives up (0: 2 s)
};
cudaError_t launch_conv(const ConvArgs& a, cudaStream_t stream);

// Driver entry point for tensor-map encoding (resolved once).
void* tensor_map_encoder();

}  // namespace dev

// Launch arguments of the GEMM of plan ``p`` for the Blocks with bid0 in
// [b0, b1), the one place they are built for every GEMM entry point
// (capi.cpp).  Returns XT_OK or an XT_E* code with the calling thread's last
// error set.
int gemm_launch_args(const Plan& p, void* const* args, int64_t b0, int64_t b1, uint32_t* error_word,
                     const char* who, dev::GemmArgs* out);

}  // namespace xt
