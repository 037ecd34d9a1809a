// Tensor-core GEMM for xt matmul programs: C = epilogue(A . B).
//
// A [M, K] row-major (K-major), B [K, N] row-major (N-major), both bf16 or
// both int8; f32 (or s32 for int8) accumulation in TMEM; C f32 or int8.
// The epilogue applies, in program order, an optional f32 accumulator tile
// (xt.mma), row/scalar scales and biases (the t * s + b of kernels/matmul.py,
// folded like lib/nova/NovaOptimize.cpp:126-296 folds them into nova.matmul)
// and the int8 cast (round half to even, saturate).
//
// Structure: clusters of two CTAs on neighbouring SMs (cta_group::2), one
// CTA per SM, persistent over 256 x 256 output tiles; each CTA of a pair
// owns 128 rows of the tile:
//   warp 0      TMA producer (both CTAs): this CTA's A 128x(128 B) and B
//               (128 B)x128 per stage, 6-stage ring
//   warp 1      leader CTA only: one elected thread issues
//               tcgen05.mma.cta_group::2 (M=256, N=256, K=16|32) into a
//               double-buffered TMEM accumulator (2 x 256 columns per CTA)
//   warp 2      allocates / frees the 512 TMEM columns (pair allocation)
//   warps 4-7   epilogue (both CTAs): tcgen05.ld 32 columns at a time, apply
//               the epilogue, store to global; overlaps the next tile's MMAs
// Every mbarrier wait is bounded (2 s); a timeout records an error code in
// the workspace error word and all roles stop, drain in-flight copies and
// MMAs, free TMEM and return.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "../kernels.h"
#include "pdl.cuh"
#include "sm100.cuh"

namespace xt {
namespace dev {
namespace {

using namespace sm100;

constexpr int kBN = 256;                       // accumulator columns per tile
constexpr int kThreads = 256;
constexpr int kTmemCols = 2 * kBN;
constexpr int kGroupM = 16;                    // tile rasterization group (L2 reuse)

enum : uint32_t { kErrProducer = 0x101, kErrMma = 0x102, kErrEpilogue = 0x103 };

struct Params {
  void* C;
  const float* acc;
  int64_t M, N, ldc, m_begin;
  int tiles_m, tiles_n, num_kb;
  int tail_begin, num_items;  // work items: whole tiles, then the last partial wave split in column halves
  uint8_t c_elem;
  int n_epi;
  uint8_t epi_kind[4];
  const float* epi_ptr[4];
  int tma_store;  // plain f32 output: epilogue stores through shared memory with TMA
  uint32_t* error_word;
  uint64_t wait_limit;  // SM cycles per pipeline wait
};

// After an abort, the time a CTA waits before it passes the final cluster
// barrier: every TMA load a producer issued lands within it.  A pair's
// producers issue into their own shared memory but complete on the leader's
// barriers, and the follower cannot observe those; the leader drains the
// stages it armed, and this wait covers loads the follower issued for a
// stage the leader gave up on before arming it.  Only the abort path pays it.
constexpr uint64_t kAbortSettleNs = 1000000ull;

// Work item -> tile and its column range.  Items below tail_begin are whole
// 256 x 256 tiles; the tiles of the last, partial wave are split into two
// 256 x 128 items each, so that wave finishes in half the time.
struct Item {
  int mt, col0, ncols;  // pair-tile row, first output column, 256 or 128 columns
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mt, int& nt);

template <class P>
__device__ __forceinline__ Item item_coords(const P& p, int item) {
  Item it;
  int nt;
  if (item < p.tail_begin) {
    tile_coords(item, p.tiles_m, p.tiles_n, it.mt, nt);
    it.col0 = nt * 256;
    it.ncols = 256;
  } else {
    const int j = item - p.tail_begin;
    tile_coords(p.tail_begin + (j >> 1), p.tiles_m, p.tiles_n, it.mt, nt);
    it.col0 = nt * 256 + (j & 1) * 128;
    it.ncols = 128;
  }
  return it;
}

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mt, int& nt) {
  const int per_group = kGroupM * tiles_n;
  const int group = t / per_group;
  const int first_m = group * kGroupM;
  const int gm = min(tiles_m - first_m, kGroupM);
  const int r = t - group * per_group;
  mt = first_m + r % gm;
  nt = r / gm;
}

__device__ __forceinline__ int8_t to_i8(float v) {
  return v != v ? 0 : static_cast<int8_t>(static_cast<int>(fminf(fmaxf(rintf(v), -128.0f), 127.0f)));
}

// ---------------------------------------------------------------------------
// CTA-pair kernel (cta_group::2): a cluster of two CTAs on neighbouring SMs
// computes a 256 x 256 tile.  Each CTA loads its 128 rows of A and its 128
// columns of B; one thread of the leader CTA (cluster rank 0) issues
// tcgen05.mma.cta_group::2 with M = 256, N = 256, and the tensor cores of the
// pair exchange the B halves.  Per SM and k-block that is 32 KiB of TMA
// writes and 32 KiB of operand reads for 128 x 256 x 64 multiply-adds, where
// the single-CTA 128 x 256 tile needs 48 + 48 KiB: shared-memory bandwidth
// (about 128 B per cycle per SM) bounds the single-CTA tile at roughly 70% of
// the tensor pipe, the pair tile runs at its full rate.
//
// Barriers: both CTAs' loads complete on the leader's "full" barrier (the
// leader's producer arms it with both CTAs' bytes); the leader's MMA commits
// arrive on "empty" and "tfull" in both CTAs (commit multicast); each CTA's
// epilogue, once it has read an accumulator, arrives once on the leader's
// "tempty" (arrival count 2).  The CTAs pass a cluster barrier after set-up
// and before freeing TMEM, so no CTA exits while its peer still uses its
// shared memory or TMEM.
constexpr int kPStages = 6;
constexpr int kPAStage = 128 * 128;             // this CTA's 128 rows x 128 B of K
constexpr int kPBStage = 128 * 128;             // this CTA's 128 columns: 128 B of K-rows x 128 columns
constexpr int kPStageBytes = kPAStage + kPBStage;
constexpr int kPStaging = 4 * 2 * 32 * 128;     // per epilogue warp: two 32-row x 32-column f32 buffers
constexpr int kPSmemBytes = kPStages * kPStageBytes + kPStaging + 1024 + 256;

template <int AB>
struct PairTraits;
template <>
struct PairTraits<kBF16> {
  static constexpr int kBK = 64;        // K elements per stage
  static constexpr int kChunkN = 64;    // N elements per 128-byte B chunk
  static constexpr int kChunks = 2;     // chunks for this CTA's 128 columns
  static constexpr int kChunkBytes = kBK * 128;
  static constexpr int kMmaK = 16;
  static constexpr uint32_t kIdesc = instr_desc(1, 1, 1, 0, 1, 256, 256);
  static constexpr uint32_t kIdescHalf = instr_desc(1, 1, 1, 0, 1, 256, 128);
  static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    umma_bf16_pair(d, a, b, idesc, acc);
  }
};
template <>
struct PairTraits<kI8> {
  static constexpr int kBK = 128;
  static constexpr int kChunkN = 128;
  static constexpr int kChunks = 1;
  static constexpr int kChunkBytes = kBK * 128;
  static constexpr int kMmaK = 32;
  static constexpr uint32_t kIdesc = instr_desc(2, 1, 1, 0, 1, 256, 256);
  static constexpr uint32_t kIdescHalf = instr_desc(2, 1, 1, 0, 1, 256, 128);  // unused: int8 tiles are never split
  static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    umma_i8_pair(d, a, b, idesc, acc);
  }
};

template <int AB>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
              const __grid_constant__ CUtensorMap tma_c, const __grid_constant__ Params p) {
  using T = PairTraits<AB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kPStages * kPAStage;
  uint8_t* staging = sb + kPStages * kPBStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + kPStaging);
  uint64_t* empty = full + kPStages;
  uint64_t* tfull = empty + kPStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tma_a);
    tma_prefetch(&tma_b);
    if (p.tma_store) tma_prefetch(&tma_c);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any cross-CTA arrive or load
  tc_fence_after();
  // set-up done: the next launch may be scheduled; global memory only after
  // the previous one has completed
  griddep_launch_dependents();
  griddep_wait();
  const uint32_t tmem_base = *tmem_slot;
  const Abort ab{abort_flag, p.error_word, p.wait_limit};
  const int num_items = p.num_items;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer (both CTAs)
      const uint32_t full0 = mapa_shared(smem_addr(full), 0);  // the leader's barriers
      int stage = 0;
      uint32_t phase = 0, armed = 0, armed_phase = 0;
      bool ok = true;
      // A's rows are reused by every N-tile of a rasterization group (kGroupM
      // M-tiles, one wave after another): keep them in L2 ahead of B, which is
      // shared within a wave, so A is not re-read from DRAM for each wave
      const uint64_t pol_a = l2_policy_evict_last();
      for (int t = pair; t < num_items && ok; t += npairs) {
        const Item it = item_coords(p, t);
        const int32_t row0 = static_cast<int32_t>(p.m_begin + static_cast<int64_t>(it.mt) * 256 + rank * 128);
        // this CTA's half of the item's columns: 128 (two 64-column chunks, or one int8 chunk) or 64
        const int32_t col0 = it.col0 + static_cast<int32_t>(rank) * (it.ncols / 2);
        const int chunks = it.ncols == 256 ? T::kChunks : 1;
        const uint32_t bytes = static_cast<uint32_t>(2 * (kPAStage + chunks * T::kChunkBytes));
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, ab, kErrProducer)) {
            ok = false;
            break;
          }
          if (leader) {
            mbar_arrive_expect_tx(&full[stage], bytes);
            armed |= 1u << stage;
            armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          }
          const uint32_t bar = full0 + static_cast<uint32_t>(stage) * 8u;
          tma_load_2d_pair_hint(sa + stage * kPAStage, &tma_a, bar, kb * T::kBK, row0, pol_a);
          for (int c = 0; c < chunks; ++c)
            tma_load_2d_pair(sb + stage * kPBStage + c * T::kChunkBytes, &tma_b, bar, col0 + c * T::kChunkN,
                             kb * T::kBK);
          if (++stage == kPStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag && leader)
        for (int s = 0; s < kPStages; ++s)
          if ((armed >> s) & 1u) mbar_wait_drain(&full[s], (armed_phase >> s) & 1u, 500000000ull);
    }
  } else if (warp == 1) {
    if (leader) {
      // ---------------------------------------------------------------- MMA issuer (leader CTA)
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = true;
      const uint32_t sa_base = smem_addr(sa), sb_base = smem_addr(sb);
      for (int t = pair; t < num_items && ok; t += npairs, ++iter) {
        const int acc = iter & 1;
        const uint32_t acc_phase = (iter >> 1) & 1;
        const uint32_t idesc = t < p.tail_begin ? T::kIdesc : T::kIdescHalf;
        if (!__all_sync(0xffffffffu, mbar_wait(&tempty[acc], acc_phase ^ 1, ab, kErrMma))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, ab, kErrMma))) {
            ok = false;
            break;
          }
          tc_fence_after();
          // A: K-major, 128-byte swizzle, 32 bytes of K per MMA.  B: N-major,
          // 128-byte swizzle; chunks of 128 B of N kChunkBytes apart (LBO),
          // 8-row K groups 1024 B apart (SBO), kMmaK rows of K per MMA.
          const uint64_t ad = smem_desc_sw128(sa_base + stage * kPAStage, 16, 1024);
          const uint64_t bd = smem_desc_sw128(sb_base + stage * kPBStage, T::kChunkBytes, 1024);
          if (elect_sync()) {
#pragma unroll
            for (int k = 0; k < 128 / 32; ++k)
              T::mma(d_tmem, ad + static_cast<uint64_t>(k * 2), bd + static_cast<uint64_t>(k * T::kMmaK * 8), idesc,
                     (kb | k) != 0 ? 1u : 0u);
            umma_commit_pair(&empty[stage], 0x3);
          }
          __syncwarp();
          if (++stage == kPStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) {
          if (elect_sync()) umma_commit_pair(&tfull[acc], 0x3);
          __syncwarp();
        }
      }
      if (*abort_flag) {
        if (elect_sync()) umma_commit_pair(drain, 0x1);
        __syncwarp();
        mbar_wait_drain(drain, 0, 500000000ull);
      }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------------- epilogue (both CTAs)
    const int q = warp - 4;  // TMEM lane quarter
    const uint32_t tempty0 = mapa_shared(smem_addr(tempty), 0);
    int iter = 0;
    for (int t = pair; t < num_items; t += npairs, ++iter) {
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      const bool ok = mbar_wait_warp(&tfull[acc], acc_phase, ab, kErrEpilogue);
      if (named_barrier_or(2, 128, !ok)) break;  // all four warps stop together (named barriers below)
      tc_fence_after();
      const Item it = item_coords(p, t);
      const int mt = it.mt;
      const int nchunks = it.ncols / 32;
      const int64_t r_local = static_cast<int64_t>(mt) * 256 + rank * 128 + q * 32 + lane;
      const int64_t row = p.m_begin + r_local;
      const bool row_ok = r_local < p.M;
      const bool plain = p.acc == nullptr && p.n_epi == 0;
#pragma unroll 1
      for (int c = 0; c < nchunks; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kBN + c * 32, r);
        tmem_wait_ld();
        if (c == nchunks - 1) {
          // every thread of this CTA has read the accumulator: one arrival for the CTA
          tc_fence_before();
          named_barrier_sync(1, 128);
          if (threadIdx.x == 128) mbar_arrive_cluster(tempty0 + static_cast<uint32_t>(acc) * 8u);
        }
        if (p.tma_store) {
          // Stage this warp's 32 rows x 32 columns in a 128-byte swizzled
          // buffer and write them with one TMA store: whole 128-byte row
          // segments, clipped at the array's edges by TMA.  That matters most
          // when C is another GPU's memory (row gathers over NVLink).
          uint8_t* buf = staging + (q * 2 + (c & 1)) * 4096;
          if (lane == 0) bulk_wait_group_read<1>();  // the store that last used buf has read it
          __syncwarp();
          const uint32_t sw = static_cast<uint32_t>(lane & 7);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 v4;
            if (AB == kI8)
              v4 = make_float4(__int2float_rn(static_cast<int>(r[4 * j])), __int2float_rn(static_cast<int>(r[4 * j + 1])),
                               __int2float_rn(static_cast<int>(r[4 * j + 2])),
                               __int2float_rn(static_cast<int>(r[4 * j + 3])));
            else
              v4 = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                               __uint_as_float(r[4 * j + 3]));
            *reinterpret_cast<float4*>(buf + lane * 128 + ((static_cast<uint32_t>(j) ^ sw) << 4)) = v4;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            // C is not read again by this kernel: its lines leave L2 first
            tma_store_2d_hint(&tma_c, buf, it.col0 + c * 32,
                              static_cast<int32_t>(p.m_begin + static_cast<int64_t>(mt) * 256 + rank * 128 + q * 32),
                              l2_policy_evict_first());
            bulk_commit_group();
          }
          continue;
        }
        const int64_t col0 = static_cast<int64_t>(it.col0) + c * 32;
        if (!row_ok || col0 >= p.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
          v[j] = AB == kI8 ? __int2float_rn(static_cast<int>(r[j])) : __uint_as_float(r[j]);
        const bool full_chunk = col0 + 32 <= p.N;
        if (!plain) {
          // the epilogue in program order (accumulator tile + t, then each
          // scale / bias step), each step applied to the chunk's 32 columns
          // at once: the accumulator tile's and each row vector's 32 values
          // are read once per chunk (8 x 16-byte loads when aligned).  Read
          // per element inside the step loop they made the int8 GEMM with
          // kernels/matmul.py's epilogue epilogue-bound (tensor pipe 15% busy)
          auto load32 = [&](const float* src, float (&e)[32]) {
            if (full_chunk && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 q4 = __ldg(reinterpret_cast<const float4*>(src + j));
                e[j] = q4.x;
                e[j + 1] = q4.y;
                e[j + 2] = q4.z;
                e[j + 3] = q4.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) e[j] = col0 + j < p.N ? __ldg(src + j) : 0.0f;
            }
          };
          float e[32];
          if (p.acc) {
            load32(p.acc + row * p.ldc + col0, e);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(e[j], v[j]);
          }
          for (int s = 0; s < p.n_epi; ++s) {
            const uint8_t k = p.epi_kind[s];
            const bool mul = k == kEpiMulRow || k == kEpiMulScalar;
            if (k == kEpiMulRow || k == kEpiAddRow) {
              load32(p.epi_ptr[s] + col0, e);
            } else {
              const float x = __ldg(p.epi_ptr[s]);
#pragma unroll
              for (int j = 0; j < 32; ++j) e[j] = x;
            }
            if (mul) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(v[j], e[j]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], e[j]);
            }
          }
        }
        if (p.c_elem == kF32) {
          float* dst = static_cast<float*>(p.C) + row * p.ldc + col0;
          if (full_chunk && (p.ldc & 7) == 0 && (reinterpret_cast<uintptr_t>(p.C) & 31) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 8)
              st_global_cs_v8(dst + j, v[j], v[j + 1], v[j + 2], v[j + 3], v[j + 4], v[j + 5], v[j + 6], v[j + 7]);
          } else if (full_chunk && (p.ldc & 3) == 0) {
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
    }
    if (p.tma_store && lane == 0) bulk_wait_group<0>();  // this warp's stores are complete
  }
  __syncthreads();
  // every role of this CTA has stopped; if any gave up, let issued loads land
  if (*abort_flag && threadIdx.x == 0) spin_ns(kAbortSettleNs);
  cluster_sync();  // the peer is done with this CTA's shared memory and TMEM, and vice versa
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
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
cudaError_t launch_pair(const GemmArgs& a, cudaStream_t stream) {
  using T = PairTraits<AB>;
  const CUtensorMapDataType dt = AB == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const int eb = AB == kBF16 ? 2 : 1;
  CUtensorMap ma, mb;
  // A: [rows up to m_begin + M] x [K], box 128 rows x 128 bytes of K (one CTA's half of a pair tile)
  if (!make_map_2d(&ma, a.A, dt, eb, a.K, a.m_begin + a.M, a.lda, 128 / eb, 128)) return cudaErrorInvalidValue;
  // B: [K] x [N], box kBK rows x 128 bytes of N
  if (!make_map_2d(&mb, a.B, dt, eb, a.N, a.K, a.ldb, 128 / eb, T::kBK)) return cudaErrorInvalidValue;
  // C through TMA stores for plain f32 output: [rows up to m_begin + M] x [N], box 32 rows x 32 columns
  CUtensorMap mc = ma;
  const bool tma_store = a.c_elem == kF32 && a.acc == nullptr && a.n_epi == 0 && (a.ldc * 4) % 16 == 0 &&
                         (reinterpret_cast<uintptr_t>(a.C) & 15) == 0 &&
                         make_map_2d(&mc, a.C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.N, a.m_begin + a.M, a.ldc, 32, 32);
  Params p{};
  p.C = a.C;
  p.acc = a.acc;
  p.M = a.M;
  p.N = a.N;
  p.ldc = a.ldc;
  p.m_begin = a.m_begin;
  p.tiles_m = static_cast<int>((a.M + 255) / 256);
  p.tiles_n = static_cast<int>((a.N + 255) / 256);
  p.num_kb = static_cast<int>((a.K + T::kBK - 1) / T::kBK);
  p.c_elem = a.c_elem;
  p.tail_begin = p.num_items = p.tiles_m * p.tiles_n;
  p.n_epi = a.n_epi;
  for (int i = 0; i < 4; ++i) {
    p.epi_kind[i] = a.epi_kind[i];
    p.epi_ptr[i] = a.epi_ptr[i];
  }
  p.error_word = a.error_word;
  p.wait_limit = wait_limit_or_default(a.wait_limit_cycles);
  p.tma_store = tma_store ? 1 : 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  // the shared-memory opt-in is per device: remember which devices have it
  static std::atomic<uint64_t> attr_devices{0};
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
  if (!(attr_devices.load(std::memory_order_relaxed) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_pair<AB>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytes);
    if (e != cudaSuccess) return e;
    attr_devices.fetch_or(bit, std::memory_order_relaxed);
  }
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = p.tiles_m * p.tiles_n;
  if (tiles == 0 || p.num_kb == 0) return cudaSuccess;
  if (a.max_sms > 0 && a.max_sms < sms) sms = a.max_sms;
  int pairs = tiles < sms / 2 ? tiles : sms / 2;
  if (pairs < 1) pairs = 1;
  // Split the last partial wave's tiles into column halves (bf16 only: an
  // int8 half is 64 bytes wide, narrower than the 128-byte swizzle atom).
  const int tail = tiles % pairs;
  if (AB == kBF16 && tiles > pairs && tail > 0 && 2 * tail <= pairs) {
    p.tail_begin = tiles - tail;
    p.num_items = tiles + tail;
  }
  return PdlLaunch(dim3(2 * pairs), dim3(kThreads), kPSmemBytes, stream, 2)(gemm_pair<AB>, ma, mb, mc, p);
}

}  // namespace

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (a.ab_elem == kBF16) return launch_pair<kBF16>(a, stream);
  return launch_pair<kI8>(a, stream);
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
