// Tensor-core implicit-GEMM convolution for xt.load_conv2d programs.
//
// out[n, h, w, k] = sum_{r, s, c} in[n, h - pad_t + r*dil_h, w - pad_l + s*dil_w, c] * f[r, s, c, k],
// zero outside the input image: the zero-padded convolution the reference's
// halo-slice lowering computes (lib/xt/XTToNova.cpp:103-142,353-437), stride 1.
// Input NHWC and filter HWIO are bf16 (f32 accumulation) or int8 (s32
// accumulation); the output is f32.
//
// GEMM view: M = output pixels, N = output channels (KO), K = taps x channels.
// One A tile is 128 GEMM rows = 2 output rows x 64 output columns of one image,
// 128 bytes of channels each: a single 4D TMA box {channels, 64 w, 2 h, 1 n}
// per (tap, channel chunk), placed at the tap's shifted (h, w) coordinates.
// TMA fills coordinates outside the image with zeros, which is exactly the
// padding (negative starts are allowed; the channel coordinate stays 16-byte
// aligned).  Filter taps stream through the same smem ring from a 3D view
// [taps][C][KO] (N-major B operand; its swizzle span, 128/64/32 bytes, is the
// widest that the KO row divides into, so each MMA's N covers whole atoms).
//
// Roles as in gemm_tc.cu: warp 0 TMA producer, warp 1 one thread issuing
// tcgen05.mma (M=128, N=KO), warp 2 TMEM allocation (double-buffered
// accumulator), warps 4-7 epilogue straight from TMEM to NHWC rows.  All
// waits are bounded; a timeout sets the error word and every role stops.
#include <cuda.h>
#include <cuda_runtime.h>

#include "../kernels.h"
#include "sm100.cuh"

namespace xt {
namespace dev {
namespace {

using namespace sm100;

constexpr int kThreads = 256;
constexpr int kBM = 128;
constexpr int kAStage = kBM * 128;  // 16 KiB
constexpr int kMaxStages = 8;

enum : uint32_t { kErrProducer = 0x201, kErrMma = 0x202, kErrEpilogue = 0x203 };

struct Params {
  float* out;
  int64_t out_h, out_w, out_c;
  int ON, OH, OW, n_begin;
  int tiles_h, tiles_w, num_tiles;
  int kc;              // channel chunks per tap
  int KH, KW, pad_t, pad_l, dil_h, dil_w;
  int N;               // output channels = MMA N
  int b_chunks;        // column chunks of the filter tile, b_span bytes wide each
  int b_span;          // swizzle span of the filter operand: 128, 64 or 32 bytes
  uint32_t b_layout;   // UMMA layout code of that span
  int stages, stage_bytes, b_chunk_bytes;
  int tmem_cols;
  uint32_t idesc;
  uint32_t* error_word;
};

template <int AB>
struct ConvTraits;
template <>
struct ConvTraits<kBF16> {
  static constexpr int kCh = 64;       // channels per 128-byte chunk
  static constexpr int kMmaK = 16;
  static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    umma_bf16(d, a, b, idesc, acc);
  }
};
template <>
struct ConvTraits<kI8> {
  static constexpr int kCh = 128;
  static constexpr int kMmaK = 32;
  static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    umma_i8(d, a, b, idesc, acc);
  }
};

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& n, int& h0, int& w0) {
  const int per_img = p.tiles_h * p.tiles_w;
  n = t / per_img;
  const int r = t - n * per_img;
  h0 = (r / p.tiles_w) * 2;
  w0 = (r % p.tiles_w) * 64;
}

template <int AB>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tc(const __grid_constant__ CUtensorMap tma_in, const __grid_constant__ CUtensorMap tma_f,
            const __grid_constant__ Params p) {
  using T = ConvTraits<AB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * p.stage_bytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tma_in);
    tma_prefetch(&tma_f);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const Abort ab{abort_flag, p.error_word};
  const int num_kb = p.KH * p.KW * p.kc;

  if (warp == 0) {
    if (lane == 0) {
      // -------------------------------------------------------------- producer
      int stage = 0;
      uint32_t phase = 0;
      int pending[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) pending[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int n, h0, w0;
        tile_coords(p, t, n, h0, w0);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, ab, kErrProducer)) {
            ok = false;
            break;
          }
          const int tap = kb / p.kc, chunk = kb - tap * p.kc;
          const int r = tap / p.KW, s = tap - r * p.KW;
          uint8_t* st = smem + stage * p.stage_bytes;
          mbar_arrive_expect_tx(&full[stage], p.stage_bytes);
          tma_load_4d(st, &tma_in, &full[stage], chunk * T::kCh, w0 + s * p.dil_w - p.pad_l,
                      h0 + r * p.dil_h - p.pad_t, p.n_begin + n);
          const int chunk_elems = p.b_span / (AB == kBF16 ? 2 : 1);
          for (int j = 0; j < p.b_chunks; ++j)
            tma_load_3d(st + kAStage + j * p.b_chunk_bytes, &tma_f, &full[stage], j * chunk_elems,
                        chunk * T::kCh, tap);
          pending[stage] = static_cast<int>(phase);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag)
        for (int s = 0; s < p.stages; ++s)
          if (pending[s] >= 0) mbar_wait_drain(&full[s], static_cast<uint32_t>(pending[s]), 500000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // -------------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++iter) {
        const int acc = iter & 1;
        const uint32_t acc_phase = (iter >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, ab, kErrMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * (p.tmem_cols / 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, ab, kErrMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_addr(smem + stage * p.stage_bytes);
          const uint32_t b_base = a_base + kAStage;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = smem_desc_sw128(a_base + k * 32, 16, 1024);
            // N-major filter tile: chunks of b_span bytes are b_chunk_bytes apart
            // (LBO), 8-row K groups are 8 * b_span bytes apart (SBO)
            const uint64_t bd = smem_desc(b_base + k * T::kMmaK * p.b_span, p.b_chunk_bytes, 8 * p.b_span,
                                          p.b_layout);
            T::mma(d_tmem, ad, bd, p.idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
      if (*abort_flag) {
        umma_commit(drain);
        mbar_wait_drain(drain, 0, 500000000ull);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp - 4;
    const int row = q * 32 + lane;  // GEMM row of the tile = (hh, ww)
    const int hh = row >> 6, ww = row & 63;
    int iter = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++iter) {
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      const bool ok = mbar_wait(&tfull[acc], acc_phase, ab, kErrEpilogue);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      int n, h0, w0;
      tile_coords(p, t, n, h0, w0);
      const int h = h0 + hh, w = w0 + ww;
      const bool valid = h < p.OH && w < p.OW;
      float* dst = p.out + ((static_cast<int64_t>(p.n_begin + n) * p.out_h + h) * p.out_w + w) * p.out_c;
      for (int c = 0; c < p.N / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * (p.tmem_cols / 2) + c * 32,
                           r);
        tmem_wait_ld();
        if (!valid) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
          v[j] = AB == kI8 ? __int2float_rn(static_cast<int>(r[j])) : __uint_as_float(r[j]);
        if ((p.out_c & 3) == 0) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            __stcs(reinterpret_cast<float4*>(dst + c * 32 + j), make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) dst[c * 32 + j] = v[j];
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

template <int AB>
cudaError_t launch_typed(const ConvArgs& a, cudaStream_t stream) {
  using T = ConvTraits<AB>;
  auto encode = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!encode) return cudaErrorInvalidValue;
  const int eb = AB == kBF16 ? 2 : 1;
  const CUtensorMapDataType dt = AB == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  cuuint32_t estr[4] = {1, 1, 1, 1};
  // input NHWC: dims {C, W, H, N}, box {128 B of channels, 64 w, 2 h, 1 n}
  CUtensorMap m_in, m_f;
  {
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.C), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                          static_cast<cuuint64_t>(a.N)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(a.C) * eb, static_cast<cuuint64_t>(a.W * a.C) * eb,
                             static_cast<cuuint64_t>(a.H * a.W * a.C) * eb};
    cuuint32_t box[4] = {static_cast<cuuint32_t>(T::kCh), 64, 2, 1};
    if (encode(&m_in, dt, 4, const_cast<void*>(a.in), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  // The filter is the N-major B operand.  Its swizzle span is the widest of
  // 128 / 64 / 32 bytes that the KO row divides into, so every MMA's N is a
  // whole number of swizzle atoms.
  const int row_bytes = static_cast<int>(a.KO) * eb;
  const int span = row_bytes % 128 == 0 ? 128 : row_bytes % 64 == 0 ? 64 : 32;
  const CUtensorMapSwizzle f_swizzle = span == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                       : span == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
  // filter HWIO viewed as [taps][C][KO]: dims {KO, C, taps}, box {span bytes of KO, chunk of C, 1}
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(a.KO), static_cast<cuuint64_t>(a.C),
                          static_cast<cuuint64_t>(a.KH * a.KW)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(a.KO) * eb, static_cast<cuuint64_t>(a.C * a.KO) * eb};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(span / eb), static_cast<cuuint32_t>(T::kCh), 1};
    if (encode(&m_f, dt, 3, const_cast<void*>(a.filt), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               f_swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  Params p{};
  p.out = a.out;
  p.out_h = a.out_h;
  p.out_w = a.out_w;
  p.out_c = a.out_c;
  p.ON = static_cast<int>(a.ON);
  p.OH = static_cast<int>(a.OH);
  p.OW = static_cast<int>(a.OW);
  p.n_begin = static_cast<int>(a.n_begin);
  p.tiles_h = static_cast<int>((a.OH + 1) / 2);
  p.tiles_w = static_cast<int>((a.OW + 63) / 64);
  p.num_tiles = p.ON * p.tiles_h * p.tiles_w;
  p.kc = static_cast<int>((a.C + T::kCh - 1) / T::kCh);
  p.KH = static_cast<int>(a.KH);
  p.KW = static_cast<int>(a.KW);
  p.pad_t = static_cast<int>(a.pad_t);
  p.pad_l = static_cast<int>(a.pad_l);
  p.dil_h = static_cast<int>(a.dil_h);
  p.dil_w = static_cast<int>(a.dil_w);
  p.N = static_cast<int>(a.KO);
  p.b_span = span;
  p.b_layout = swizzle_layout_code(span);
  p.b_chunks = row_bytes / span;
  p.b_chunk_bytes = T::kCh * span;  // kCh rows of C x span bytes of KO
  p.stage_bytes = kAStage + p.b_chunks * p.b_chunk_bytes;
  p.stages = (190 * 1024) / p.stage_bytes;
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  int cols = 32;
  while (cols < 2 * p.N) cols *= 2;
  p.tmem_cols = cols;
  p.idesc = instr_desc(AB == kBF16 ? 1 : 2, 1, 1, 0, 1, kBM, static_cast<uint32_t>(p.N));
  p.error_word = a.error_word;
  if (p.num_tiles == 0) return cudaSuccess;
  const int smem = p.stages * p.stage_bytes + 1024 + 256;
  cudaError_t e = cudaFuncSetAttribute(conv_tc<AB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  conv_tc<AB><<<p.num_tiles < sms ? p.num_tiles : sms, kThreads, smem, stream>>>(m_in, m_f, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_conv(const ConvArgs& a, cudaStream_t stream) {
  if (a.KO % 32 != 0 || a.KO > 256) return cudaErrorInvalidValue;
  if (a.elem == kBF16) return launch_typed<kBF16>(a, stream);
  return launch_typed<kI8>(a, stream);
}

}  // namespace dev
}  // namespace xt
