// Tensor-core GEMM for xt matmul programs: C = epilogue(A . B).
//
// A [M, K] row-major (K-major), B [K, N] row-major (N-major), both bf16 or
// both int8; f32 (or s32 for int8) accumulation in TMEM; C f32 or int8.
// The epilogue applies, in program order, an optional f32 accumulator tile
// (xt.mma), row/scalar scales and biases (the t * s + b of kernels/matmul.py,
// folded like lib/nova/NovaOptimize.cpp:126-296 folds them into nova.matmul)
// and the int8 cast (round half to even, saturate).
//
// Structure (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0      TMA producer: A 128x(128 B) and B (128 B)x256 per stage,
//               4-stage ring; per stage an "empty" mbarrier (the MMAs that
//               read it completed), per pair of stages a "full" mbarrier
//               (arrival count 2: both stages' bytes landed).  The MMA thread
//               waits once per pair: a wait issued behind queued MMAs costs
//               a few hundred cycles, as much as two 128x256x16 MMAs.
//   warp 1      one thread issues tcgen05.mma (M=128, N=256, K=16|32) into a
//               double-buffered TMEM accumulator (2 x 256 columns)
//   warp 2      allocates / frees the 512 TMEM columns
//   warps 4-7   epilogue: tcgen05.ld 32 columns at a time, apply the
//               epilogue, store to global; overlaps the next tile's MMAs
// Every mbarrier wait is bounded (2 s); a timeout records an error code in
// the workspace error word and all roles stop, drain in-flight copies and
// MMAs, free TMEM and return.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../kernels.h"
#include "sm100.cuh"

namespace xt {
namespace dev {
namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kStages = 4;
constexpr int kGroup = 2;                      // stages per "full" barrier (one MMA-side wait each)
constexpr int kThreads = 256;
constexpr int kAStage = kBM * 128;             // 16 KiB: 128 rows x 128 B of K
constexpr int kBStage = kBN * 128;             // 32 KiB: 128 B of K rows... x 256 columns
constexpr int kStageBytes = kAStage + kBStage;
constexpr int kTmemCols = 2 * kBN;
constexpr int kGroupM = 16;                    // tile rasterization group (L2 reuse)
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;

enum : uint32_t { kErrProducer = 0x101, kErrMma = 0x102, kErrEpilogue = 0x103 };

struct Params {
  void* C;
  const float* acc;
  int64_t M, N, ldc, m_begin;
  int tiles_m, tiles_n, num_kb;
  uint8_t c_elem;
  int n_epi;
  uint8_t epi_kind[4];
  const float* epi_ptr[4];
  uint32_t* error_word;
};

template <int AB>
struct Traits;
template <>
struct Traits<kBF16> {
  static constexpr int kBK = 64;               // K elements per stage (128 B)
  static constexpr int kChunkN = 64;           // N elements per 128-byte B chunk
  static constexpr int kChunks = kBN / kChunkN;
  static constexpr int kChunkBytes = kBK * 128;
  static constexpr int kMmaK = 16;
  static constexpr uint32_t kIdesc = instr_desc(1 /*f32*/, 1 /*bf16*/, 1 /*bf16*/, 0, 1, kBM, kBN);
  static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
    umma_bf16(d, a, b, kIdesc, acc);
  }
};
template <>
struct Traits<kI8> {
  static constexpr int kBK = 128;
  static constexpr int kChunkN = 128;
  static constexpr int kChunks = kBN / kChunkN;
  static constexpr int kChunkBytes = kBK * 128;
  static constexpr int kMmaK = 32;
  static constexpr uint32_t kIdesc = instr_desc(2 /*s32*/, 1 /*s8*/, 1 /*s8*/, 0, 1, kBM, kBN);
  static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
    umma_i8(d, a, b, kIdesc, acc);
  }
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mt, int& nt) {
  const int per_group = kGroupM * tiles_n;
  const int group = t / per_group;
  const int first_m = group * kGroupM;
  const int gm = min(tiles_m - first_m, kGroupM);
  const int r = t - group * per_group;
  mt = first_m + r % gm;
  nt = r / gm;
}

__device__ __forceinline__ float epilogue_value(const Params& p, float v, int64_t row, int64_t col) {
  if (p.acc) v = __fadd_rn(__ldg(p.acc + row * p.ldc + col), v);
  for (int s = 0; s < p.n_epi; ++s) {
    const uint8_t k = p.epi_kind[s];
    const float e = __ldg(p.epi_ptr[s] + ((k == kEpiMulRow || k == kEpiAddRow) ? col : 0));
    v = (k == kEpiMulRow || k == kEpiMulScalar) ? __fmul_rn(v, e) : __fadd_rn(v, e);
  }
  return v;
}

__device__ __forceinline__ int8_t to_i8(float v) {
  return v != v ? 0 : static_cast<int8_t>(static_cast<int>(fminf(fmaxf(rintf(v), -128.0f), 127.0f)));
}

template <int AB>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
            const __grid_constant__ Params p) {
  using T = Traits<AB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kStages * kAStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + kStages * kBStage);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int g = 0; g < kStages / kGroup; ++g) mbar_init(&full[g], kGroup);
    for (int s = 0; s < kStages; ++s) mbar_init(&empty[s], 1);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tma_a);
    tma_prefetch(&tma_b);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const Abort ab{abort_flag, p.error_word};
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      int stage = 0, grp = 0, gi = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_phase = 0;  // per group: armed at least once / parity of its last arming
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, p.tiles_m, p.tiles_n, mt, nt);
        const int32_t row0 = static_cast<int32_t>(p.m_begin + static_cast<int64_t>(mt) * kBM);
        const int32_t col0 = nt * kBN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, ab, kErrProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[grp], kStageBytes);
          armed |= 1u << grp;
          armed_phase = (armed_phase & ~(1u << grp)) | (phase << grp);
          tma_load_2d(sa + stage * kAStage, &tma_a, &full[grp], kb * T::kBK, row0);
#pragma unroll
          for (int c = 0; c < T::kChunks; ++c)
            tma_load_2d(sb + stage * kBStage + c * T::kChunkBytes, &tma_b, &full[grp], col0 + c * T::kChunkN,
                        kb * T::kBK);
          ++stage;
          if (++gi == kGroup) {
            gi = 0;
            ++grp;
          }
          if (stage == kStages) {
            stage = 0;
            grp = 0;
            phase ^= 1;
          }
        }
      }
      // A CTA whose k-block count is not whole groups ends inside a group:
      // complete it with plain arrivals so its last wait (and a drain) ends.
      for (int i = gi; i > 0 && i < kGroup; ++i) mbar_arrive(&full[grp]);
      if (*abort_flag) {
        // let every issued copy land before the CTA's shared memory is released
        for (int g = 0; g < kStages / kGroup; ++g)
          if ((armed >> g) & 1u) mbar_wait_drain(&full[g], (armed_phase >> g) & 1u, 500000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      int stage = 0, grp = 0, gi = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = true;
      const uint32_t sa_base = smem_addr(sa), sb_base = smem_addr(sb);
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++iter) {
        const int acc = iter & 1;
        const uint32_t acc_phase = (iter >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, ab, kErrMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (gi == 0) {
            // one wait covers the kGroup stages of a group
            if (!mbar_wait(&full[grp], phase, ab, kErrMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          // A: K-major, 128-byte swizzle, 32 bytes of K per MMA.  B: N-major,
          // 128-byte swizzle; chunks of 128 B of N are kChunkBytes apart (LBO),
          // 8-row K groups 1024 B apart (SBO), kMmaK rows of K per MMA.
          // Descriptor start addresses are in 16-byte units in the low bits.
          const uint64_t ad = smem_desc_sw128(sa_base + stage * kAStage, 16, 1024);
          const uint64_t bd = smem_desc_sw128(sb_base + stage * kBStage, T::kChunkBytes, 1024);
#pragma unroll
          for (int k = 0; k < 128 / 32; ++k)
            T::mma(d_tmem, ad + static_cast<uint64_t>(k * 2), bd + static_cast<uint64_t>(k * T::kMmaK * 8),
                   (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          ++stage;
          if (++gi == kGroup) {
            gi = 0;
            ++grp;
          }
          if (stage == kStages) {
            stage = 0;
            grp = 0;
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
    // -------------------------------------------------------------------- epilogue
    const int q = warp - 4;  // TMEM lane quarter
    int iter = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++iter) {
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, ab, kErrEpilogue)) break;
      tc_fence_after();
      int mt, nt;
      tile_coords(t, p.tiles_m, p.tiles_n, mt, nt);
      const int64_t r_local = static_cast<int64_t>(mt) * kBM + q * 32 + lane;
      const int64_t row = p.m_begin + r_local;
      const bool row_ok = r_local < p.M;
      const bool plain = p.acc == nullptr && p.n_epi == 0;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kBN + c * 32, r);
        tmem_wait_ld();
        const int64_t col0 = static_cast<int64_t>(nt) * kBN + c * 32;
        if (!row_ok || col0 >= p.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
          v[j] = AB == kI8 ? __int2float_rn(static_cast<int>(r[j])) : __uint_as_float(r[j]);
        const bool full_chunk = col0 + 32 <= p.N;
        if (!plain) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.N) v[j] = epilogue_value(p, v[j], row, col0 + j);
        }
        if (p.c_elem == kF32) {
          float* dst = static_cast<float*>(p.C) + row * p.ldc + col0;
          if (full_chunk && (p.ldc & 3) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          } else {
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) dst[j] = v[j];
          }
        } else {
          int8_t* dst = static_cast<int8_t*>(p.C) + row * p.ldc + col0;
          if (full_chunk && (p.ldc & 15) == 0) {
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              w[j] = (static_cast<uint32_t>(static_cast<uint8_t>(to_i8(v[4 * j]))) |
                      (static_cast<uint32_t>(static_cast<uint8_t>(to_i8(v[4 * j + 1]))) << 8) |
                      (static_cast<uint32_t>(static_cast<uint8_t>(to_i8(v[4 * j + 2]))) << 16) |
                      (static_cast<uint32_t>(static_cast<uint8_t>(to_i8(v[4 * j + 3]))) << 24));
            *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(dst + 16) = make_uint4(w[4], w[5], w[6], w[7]);
          } else {
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) dst[j] = to_i8(v[j]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  auto encode = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!encode) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * static_cast<cuuint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int AB>
cudaError_t launch_typed(const GemmArgs& a, cudaStream_t stream) {
  using T = Traits<AB>;
  const CUtensorMapDataType dt = AB == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const int eb = AB == kBF16 ? 2 : 1;
  CUtensorMap ma, mb;
  // A: [rows up to m_begin + M] x [K], box 128 rows x 128 bytes of K
  if (!make_map_2d(&ma, a.A, dt, eb, a.K, a.m_begin + a.M, a.lda, 128 / eb, kBM)) return cudaErrorInvalidValue;
  // B: [K] x [N], box kBK rows x 128 bytes of N
  if (!make_map_2d(&mb, a.B, dt, eb, a.N, a.K, a.ldb, 128 / eb, T::kBK)) return cudaErrorInvalidValue;
  Params p{};
  p.C = a.C;
  p.acc = a.acc;
  p.M = a.M;
  p.N = a.N;
  p.ldc = a.ldc;
  p.m_begin = a.m_begin;
  p.tiles_m = static_cast<int>((a.M + kBM - 1) / kBM);
  p.tiles_n = static_cast<int>((a.N + kBN - 1) / kBN);
  p.num_kb = static_cast<int>((a.K + T::kBK - 1) / T::kBK);
  p.c_elem = a.c_elem;
  p.n_epi = a.n_epi;
  for (int i = 0; i < 4; ++i) {
    p.epi_kind[i] = a.epi_kind[i];
    p.epi_ptr[i] = a.epi_ptr[i];
  }
  p.error_word = a.error_word;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc<AB>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = p.tiles_m * p.tiles_n;
  if (tiles == 0 || p.num_kb == 0) return cudaSuccess;
  gemm_tc<AB><<<tiles < sms ? tiles : sms, kThreads, kSmemBytes, stream>>>(ma, mb, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (a.ab_elem == kBF16) return launch_typed<kBF16>(a, stream);
  return launch_typed<kI8>(a, stream);
}

void* tensor_map_encoder() {
  static void* fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<void*>(nullptr);
    return f;
  }();
  return fn;
}

}  // namespace dev
}  // namespace xt
