// Tensor-core implicit-GEMM convolution for xt.load_conv2d programs.
//
// out[n, h, w, k] = sum_{r, s, c} in[n, h - pad_t + r*dil_h, w - pad_l + s*dil_w, c] * f[r, s, c, k],
// zero outside the input image: the zero-padded convolution the reference's
// halo-slice lowering computes (lib/xt/XTToNova.cpp:103-142,353-437), stride 1.
// Input NHWC and filter HWIO are bf16 (f32 accumulation) or int8 (s32
// accumulation); the output is f32.
//
// GEMM view: M = output pixels, N = output channels (KO), K = taps x channels.
// One A tile is 128 GEMM rows = 2 output rows x 64 output columns of one
// image, 128 bytes of channels each: one 4D TMA box {channels, 64 w, 2 h, 1 n}
// per k-block (a filter tap and a channel chunk), placed at the tap's shifted
// (h, w) coordinates.  TMA fills coordinates outside the image with zeros,
// which is exactly the padding (negative starts are allowed; the channel
// coordinate stays 128-byte aligned).
//
// The filter is the N-major B operand, read from a 3D view [taps][C][KO]; its
// swizzle span (128/64/32 bytes) is the widest the KO row divides into, so
// each MMA's N covers whole swizzle atoms.  When the whole filter fits in
// shared memory (72 KiB for 3x3x64x64 bf16) it is loaded once per CTA and a
// k-block costs one TMA; otherwise each k-block also streams its filter slice.
//
// Pipeline: a ring of per-k-block stages, each with an "empty" barrier the
// MMAs' commit releases; "full" barriers guard groups of G consecutive stages
// (arrival count G, one arrive.expect_tx per k-block), so the MMA thread
// waits once per G k-blocks.  A wait issued behind queued MMAs costs a few
// hundred cycles on sm_100a, which at N = 64 would otherwise cost more than
// the MMAs themselves.
//
// Roles: warp 0 TMA producer, warp 1 one thread issuing tcgen05.mma (M=128,
// N=KO) into a double-buffered TMEM accumulator, warp 2 TMEM allocation,
// warps 4-7 the epilogue.  The epilogue reads 32 accumulator columns at a time
// from TMEM, writes them to a 128-byte-swizzled staging tile in shared memory
// and stores the tile with one TMA store; the store's tensor map spans only
// the covered output, so ragged tiles are clipped by TMA.  All waits are
// bounded; a timeout sets the error word and every role stops.
#include <cuda.h>
#include <cuda_runtime.h>

#include "../kernels.h"
#include "pdl.cuh"
#include "sm100.cuh"

namespace xt {
namespace dev {
namespace {

using namespace sm100;

constexpr int kThreads = 256;
constexpr int kBM = 128;
constexpr int kAStage = kBM * 128;    // 16 KiB
constexpr int kStaging = kBM * 128;   // one 128 x 32-column f32 staging tile
constexpr int kMaxStages = 12;
constexpr int kMaxGroups = kMaxStages;

enum : uint32_t { kErrProducer = 0x201, kErrMma = 0x202, kErrEpilogue = 0x203 };

struct Params {
  int ON, OH, OW, n_begin;
  int tiles_h, tiles_w, num_tiles;
  int kc;              // channel chunks per tap
  int KH, KW, pad_t, pad_l, dil_h, dil_w;
  int N;               // output channels = MMA N
  int b_chunks;        // column chunks of a k-block's filter slice, b_span bytes wide each
  int b_span;          // swizzle span of the filter operand: 128, 64 or 32 bytes
  uint32_t b_layout;   // UMMA layout code of that span
  int b_chunk_bytes;   // kCh rows of C x b_span bytes
  int b_kblock_bytes;  // b_chunks * b_chunk_bytes
  int resident;        // 1: whole filter loaded once; 0: streamed per k-block
  int stages, group, stage_bytes;  // ring of ``stages``; full barriers per ``group`` stages
  int filter_offset, staging_offset, barrier_offset;  // shared-memory layout
  int tmem_cols;
  uint32_t idesc;
  uint32_t* error_word;
  uint64_t wait_limit;  // SM cycles per pipeline wait
};

template <int AB>
struct ConvTraits;
template <>
struct ConvTraits<kBF16> {
  static constexpr int kCh = 64;   // channels per 128-byte chunk
  static constexpr int kMmaK = 16;
  static constexpr int kEb = 2;
  static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    umma_bf16(d, a, b, idesc, acc);
  }
};
template <>
struct ConvTraits<kI8> {
  static constexpr int kCh = 128;
  static constexpr int kMmaK = 32;
  static constexpr int kEb = 1;
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
            const __grid_constant__ CUtensorMap tma_out, const __grid_constant__ Params p) {
  using T = ConvTraits<AB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* filt = smem + p.filter_offset;
  uint8_t* staging = smem + p.staging_offset;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.barrier_offset);  // one per group of stages
  uint64_t* empty = full + kMaxGroups;                                    // one per stage
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* fbar = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fbar + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const int n_groups = p.stages / p.group;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int g = 0; g < n_groups; ++g) mbar_init(&full[g], p.group);
    for (int s = 0; s < p.stages; ++s) mbar_init(&empty[s], 1);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    mbar_init(fbar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tma_in);
    tma_prefetch(&tma_f);
    tma_prefetch(&tma_out);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // set-up done: the next launch may be scheduled; global memory only after
  // the previous one has completed
  griddep_launch_dependents();
  griddep_wait();
  const uint32_t tmem_base = *tmem_slot;
  const Abort ab{abort_flag, p.error_word, p.wait_limit};
  const int num_kb = p.KH * p.KW * p.kc;
  const int chunk_elems = p.b_span / T::kEb;

  if (warp == 0) {
    if (lane == 0) {
      // -------------------------------------------------------------- producer
      if (p.resident) {
        // The whole filter, k-block by k-block, once per CTA.
        mbar_arrive_expect_tx(fbar, static_cast<uint32_t>(num_kb * p.b_kblock_bytes));
        int tap = 0, ci = 0;
        for (int kb = 0; kb < num_kb; ++kb) {
          for (int j = 0; j < p.b_chunks; ++j)
            tma_load_3d(filt + kb * p.b_kblock_bytes + j * p.b_chunk_bytes, &tma_f, fbar, j * chunk_elems,
                        ci * T::kCh, tap);
          if (++ci == p.kc) {
            ci = 0;
            ++tap;
          }
        }
      }
      const uint32_t kb_bytes = static_cast<uint32_t>(p.stage_bytes);
      int stage = 0, grp = 0, gi = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_phase = 0;  // per group: armed at least once / parity of its last arming
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int n, h0, w0;
        tile_coords(p, t, n, h0, w0);
        const int img = p.n_begin + n;
        int ci = 0, s = 0, tap = 0;
        int wc = w0 - p.pad_l, hc = h0 - p.pad_t;  // input coordinates of tap (r, s)
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, ab, kErrProducer)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + stage * p.stage_bytes;
          mbar_arrive_expect_tx(&full[grp], kb_bytes);
          armed |= 1u << grp;
          armed_phase = (armed_phase & ~(1u << grp)) | (phase << grp);
          tma_load_4d(st, &tma_in, &full[grp], ci * T::kCh, wc, hc, img);
          if (!p.resident)
            for (int j = 0; j < p.b_chunks; ++j)
              tma_load_3d(st + kAStage + j * p.b_chunk_bytes, &tma_f, &full[grp], j * chunk_elems, ci * T::kCh,
                          tap);
          if (++ci == p.kc) {
            ci = 0;
            ++tap;
            wc += p.dil_w;
            if (++s == p.KW) {
              s = 0;
              wc = w0 - p.pad_l;
              hc += p.dil_h;
            }
          }
          ++stage;
          if (++gi == p.group) {
            gi = 0;
            ++grp;
          }
          if (stage == p.stages) {
            stage = 0;
            grp = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag) {
        // Complete the partly armed group with plain arrivals, then wait for
        // every load still in flight before the CTA's shared memory goes away.
        for (int i = gi; i > 0 && i < p.group; ++i) mbar_arrive(&full[grp]);
        for (int g = 0; g < n_groups; ++g)
          if ((armed >> g) & 1u) mbar_wait_drain(&full[g], (armed_phase >> g) & 1u, 500000000ull);
        if (p.resident) mbar_wait_drain(fbar, 0, 500000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // -------------------------------------------------------------- MMA issuer
      int stage = 0, grp = 0, gi = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = !p.resident || mbar_wait(fbar, 0, ab, kErrMma);
      const uint32_t smem_base = smem_addr(smem);
      const uint32_t filt_base = smem_addr(filt);
      const uint32_t b_lbo = static_cast<uint32_t>(p.b_chunk_bytes), b_sbo = 8u * p.b_span;
      const uint32_t b_step = static_cast<uint32_t>(T::kMmaK * p.b_span);
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++iter) {
        const int acc = iter & 1;
        const uint32_t acc_phase = (iter >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, ab, kErrMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * (p.tmem_cols / 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (gi == 0) {
            if (!mbar_wait(&full[grp], phase, ab, kErrMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const uint32_t a_base = smem_base + stage * p.stage_bytes;
          const uint32_t b_base = p.resident ? filt_base + kb * p.b_kblock_bytes : a_base + kAStage;
          const uint64_t ad = smem_desc_sw128(a_base, 16, 1024);
          const uint64_t bd = smem_desc(b_base, b_lbo, b_sbo, p.b_layout);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            // A: K-major, 32 bytes of K per MMA; B: N-major, kMmaK rows of K
            // (b_span bytes each) per MMA.  Descriptor addresses are in
            // 16-byte units in the low bits.
            T::mma(d_tmem, ad + static_cast<uint64_t>(k * 2), bd + static_cast<uint64_t>((k * b_step) >> 4), p.idesc,
                   (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          ++stage;
          if (++gi == p.group) {
            gi = 0;
            ++grp;
          }
          if (stage == p.stages) {
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
    // ------------------------------------------------------------------ epilogue
    const int q = warp - 4;
    const int row = q * 32 + lane;  // GEMM row of the tile = (hh, ww) = (row / 64, row % 64)
    const uint32_t sw = static_cast<uint32_t>(row & 7);
    const bool leader = threadIdx.x == 128;
    const int nchunks = p.N / 32;
    int iter = 0, cc = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++iter) {
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      const bool ok = mbar_wait_warp(&tfull[acc], acc_phase, ab, kErrEpilogue);
      if (named_barrier_or(2, 128, !ok)) break;
      tc_fence_after();
      int n, h0, w0;
      tile_coords(p, t, n, h0, w0);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * (p.tmem_cols / 2);
      for (int c = 0; c < nchunks; ++c, ++cc) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_wait_ld();
        if (c == nchunks - 1) {
          tc_fence_before();
          mbar_arrive(&tempty[acc]);  // accumulator free for the MMAs of tile + 2
        }
        // 128-byte swizzled staging row: 16-byte unit j of row goes to unit j ^ (row % 8),
        // the layout the output tensor map's 128-byte swizzle expects.
        uint8_t* rowp = staging + (cc & 1) * kStaging + row * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 v;
          if (AB == kI8) {
            v = make_float4(__int2float_rn(static_cast<int>(r[4 * j])), __int2float_rn(static_cast<int>(r[4 * j + 1])),
                            __int2float_rn(static_cast<int>(r[4 * j + 2])),
                            __int2float_rn(static_cast<int>(r[4 * j + 3])));
          } else {
            v = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                            __uint_as_float(r[4 * j + 3]));
          }
          *reinterpret_cast<float4*>(rowp + ((static_cast<uint32_t>(j) ^ sw) << 4)) = v;
        }
        fence_proxy_async_smem();
        // Before the barrier the leader waits until the previous store has read
        // its buffer: that buffer is the one the next chunk writes.
        if (leader) bulk_wait_group_read<0>();
        named_barrier_sync(1, 128);
        if (leader) {
          tma_store_4d(&tma_out, staging + (cc & 1) * kStaging, c * 32, w0, h0, p.n_begin + n);
          bulk_commit_group();
        }
      }
    }
    if (leader) bulk_wait_group<0>();
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Window variant: one TMA box per (tile, channel chunk) holds every input
// pixel that the tile's KH x KW taps read, and each tap's A operand is that
// same shared-memory window starting at a different row.
//
// The GEMM rows of a tile are 128 * sub consecutive positions f of a
// padded-width raster of one strip (image n, output columns [w0, w0 + Wt)):
// f = h * Wp + w with Wp = Wt + (KW - 1) * dil_w.  Output (h, w0 + w) is valid
// when w < Wt (and w0 + w < OW, h < OH); the other rows compute values nobody
// stores.  The window is the input box {channels, Wp columns from w0 - pad_l,
// Hwin rows from h_first - pad_t, image}, written by TMA as 128-byte rows, so
// tap (r, s) of GEMM row i reads window row (f0 - h_first * Wp) + i
// + r * dil_h * Wp + s * dil_w: its A descriptor starts at that row.  The
// 128-byte swizzle is a function of the shared-memory address bits (the
// window is 1024-byte aligned), so a start at any row needs no descriptor
// base offset.  A tile of sub = 2 M=128 sub-tiles shares one window and one
// pair of barrier waits; for the 3x3, 56-wide case a tile moves 2x its own
// input bytes from L2 (one box per tap would move 9x).
//
// The MMA warp issues a whole (tile, chunk) burst - sub x taps x 4 MMAs -
// from one elected lane with every descriptor offset precomputed: with N = 64
// the tensor pipe is bound by the issue rate, and a burst issues about 1.8x
// faster than a loop that elects a lane per MMA.
//
// With N = 64 each 128x64x16 MMA reads 6 KiB of operands from shared memory,
// so the MMAs are bound by shared-memory bandwidth (about 128 B per cycle),
// not by the tensor pipe; nothing else in the kernel goes through shared
// memory except the TMA window writes.  The epilogue reads two 32-column
// accumulator slices per TMEM wait and each thread stores its own output
// pixel's 128-byte slices from registers.
constexpr int kWinMaxStages = 4;
constexpr int kWinThreads = 384;      // warps 0-3 roles, 4-11 epilogue
constexpr int kWinEpiThreads = 256;
constexpr int kMaxFBars = 8;

struct WinParams {
  int ON, OH, OW, n_begin;
  int Wt, Wp, Hwin, tiles_w, tiles_per_strip, num_tiles;
  int sub;  // M=128 sub-tiles per tile (1 or 2)
  int kc, KH, KW, pad_t, pad_l, dil_h, dil_w;
  int N;
  int b_span, b_chunks, b_chunk_bytes, b_kblock_bytes;
  uint32_t b_layout;
  int stages, stage_bytes, box_bytes;
  int filter_offset, barrier_offset;
  int tmem_cols;
  uint32_t idesc;
  float* out;
  int64_t out_h, out_w, out_c;
  int v8;  // output rows 32-byte aligned: 32-byte stores
  uint32_t* error_word;
  uint64_t wait_limit;  // SM cycles per pipeline wait
};

__device__ __forceinline__ void win_tile(const WinParams& p, int t, int& n, int& w0, int& f0) {
  const int strip = t / p.tiles_per_strip;
  f0 = (t - strip * p.tiles_per_strip) * (kBM * p.sub);
  n = strip / p.tiles_w;
  w0 = (strip - n * p.tiles_w) * p.Wt;
}

// Stores 32 accumulator columns (f32, or s32 converted to f32) to 128
// contiguous bytes of global memory with streaming stores: 32-byte stores
// when ``dst`` is 32-byte aligned (half the store requests of 16-byte ones,
// which matters because every thread writes a different output row), else
// 16-byte stores.
template <int AB>
__device__ __forceinline__ float acc_value(uint32_t r) {
  return AB == kI8 ? __int2float_rn(static_cast<int>(r)) : __uint_as_float(r);
}

template <int AB>
__device__ __forceinline__ void store_row(float* dst, const uint32_t (&r)[32], bool v8) {
  if (v8) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      st_global_cs_v8(dst + 8 * j, acc_value<AB>(r[8 * j]), acc_value<AB>(r[8 * j + 1]), acc_value<AB>(r[8 * j + 2]),
                      acc_value<AB>(r[8 * j + 3]), acc_value<AB>(r[8 * j + 4]), acc_value<AB>(r[8 * j + 5]),
                      acc_value<AB>(r[8 * j + 6]), acc_value<AB>(r[8 * j + 7]));
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      __stcs(reinterpret_cast<float4*>(dst) + j, make_float4(acc_value<AB>(r[4 * j]), acc_value<AB>(r[4 * j + 1]),
                                                             acc_value<AB>(r[4 * j + 2]), acc_value<AB>(r[4 * j + 3])));
  }
}

// KH_ x KW_ > 0: taps known at compile time (unrolled bursts); 0: any shape.
template <int AB, int KH_, int KW_>
__global__ void __launch_bounds__(kWinThreads, 1)
    conv_window(const __grid_constant__ CUtensorMap tma_in, const __grid_constant__ CUtensorMap tma_f,
                const __grid_constant__ WinParams p) {
  using T = ConvTraits<AB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* filt = smem + p.filter_offset;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.barrier_offset);
  uint64_t* empty = full + kWinMaxStages;
  uint64_t* tfull = empty + kWinMaxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;  // one per MMA warp
  uint64_t* fbar = drain + 2;  // one per filter row (rows past the last barrier share it)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fbar + kMaxFBars);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 32 && blockIdx.x < p.num_tiles) {
    // Start this CTA's first window on its way from HBM into L2 while the
    // previous launch on the stream drains (programmatic dependent launch):
    // the window's TMA loads, issued after griddepcontrol.wait, then hit L2.
    int n, w0, f0;
    win_tile(p, blockIdx.x, n, w0, f0);
    for (int c = 0; c < p.kc; ++c)
      tma_prefetch_l2_4d(&tma_in, c * T::kCh, w0 - p.pad_l, f0 / p.Wp - p.pad_t, p.n_begin + n);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kWinEpiThreads);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    for (int g = 0; g < kMaxFBars; ++g) mbar_init(&fbar[g], 1);
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
  // set-up done: the next launch may be scheduled; global memory only after
  // the previous one has completed
  griddep_launch_dependents();
  griddep_wait();
  const uint32_t tmem_base = *tmem_slot;
  const Abort ab{abort_flag, p.error_word, p.wait_limit};
  const int n_fbars = p.KH < kMaxFBars ? p.KH : kMaxFBars;

  if (warp == 0) {
    if (lane == 0) {
      // -------------------------------------------------------------- producer
      // The first window goes out before the filter so the two loads overlap.
      const int chunk_elems = p.b_span / T::kEb;
      bool filter_pending = true;
      auto load_filter = [&]() {
        // The whole filter, (tap, chunk) k-block by k-block, once per CTA, one
        // barrier per filter row: the first tile's MMAs start on row 0 while
        // the other rows are still in flight.
        int tap = 0, ci = 0, kb = 0;
        for (int g = 0; g < n_fbars; ++g) {
          const int rows = g + 1 < n_fbars ? 1 : p.KH - g;
          const int kbs = rows * p.KW * p.kc;
          mbar_arrive_expect_tx(&fbar[g], static_cast<uint32_t>(kbs * p.b_kblock_bytes));
          for (int i = 0; i < kbs; ++i, ++kb) {
            for (int j = 0; j < p.b_chunks; ++j)
              tma_load_3d(filt + kb * p.b_kblock_bytes + j * p.b_chunk_bytes, &tma_f, &fbar[g], j * chunk_elems,
                          ci * T::kCh, tap);
            if (++ci == p.kc) {
              ci = 0;
              ++tap;
            }
          }
        }
        filter_pending = false;
      };
      int stage = 0;
      uint32_t phase = 0, issued = 0, issued_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int n, w0, f0;
        win_tile(p, t, n, w0, f0);
        const int h_first = f0 / p.Wp;
        for (int c = 0; c < p.kc; ++c) {
          if (!mbar_wait(&empty[stage], phase ^ 1, ab, kErrProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(p.box_bytes));
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          tma_load_4d(smem + stage * p.stage_bytes, &tma_in, &full[stage], c * T::kCh, w0 - p.pad_l,
                      h_first - p.pad_t, p.n_begin + n);
          if (filter_pending) load_filter();
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (filter_pending) load_filter();
      if (*abort_flag) {
        for (int s = 0; s < p.stages; ++s)
          if ((issued >> s) & 1u) mbar_wait_drain(&full[s], (issued_phase >> s) & 1u, 500000000ull);
        for (int g = 0; g < n_fbars; ++g) mbar_wait_drain(&fbar[g], 0, 500000000ull);
      }
    }
  } else if (warp == 1 || warp == 3) {
    // --------------------------------------------------------------- MMA issuers
    // Warp 1 issues the CTA's even tiles into accumulator 0, warp 3 the odd
    // ones into accumulator 1.  A warp's barrier checks between bursts cost a
    // few hundred cycles while the MMAs saturate shared memory; the other
    // warp's burst keeps the tensor pipe fed meanwhile.  Each warp runs its
    // loop converged; one elected lane issues each burst.
    const int mw = warp == 1 ? 0 : 1;
    constexpr bool kFixed = KH_ > 0 && KW_ > 0;
    constexpr int kTaps = kFixed ? KH_ * KW_ : 1;
    constexpr int kKW = kFixed ? KW_ : 1;
    int iter = mw;
    bool ok = true;
    bool first = true;  // this warp's first chunk waits for the filter, row by row
    const uint32_t smem_base = smem_addr(smem);
    const uint64_t b_desc0 = smem_desc(smem_addr(filt), p.b_chunk_bytes, 8 * p.b_span, p.b_layout);
    const uint32_t b_kb16 = static_cast<uint32_t>(p.b_kblock_bytes) >> 4;
    const uint32_t b_step16 = static_cast<uint32_t>(T::kMmaK * p.b_span) >> 4;
    // Descriptor offsets in 16-byte units: window rows are 128 bytes (8 units),
    // 32 bytes of K per MMA step along a row.
    uint32_t a_tap[kTaps], b_tap[kTaps];
#pragma unroll
    for (int t = 0; t < kTaps; ++t) {
      a_tap[t] = kFixed ? static_cast<uint32_t>(((t / kKW) * p.dil_h * p.Wp + (t % kKW) * p.dil_w) * 8) : 0u;
      b_tap[t] = static_cast<uint32_t>(t * p.kc) * b_kb16;
    }
    const uint32_t r_step16 = static_cast<uint32_t>(p.dil_h * p.Wp) * 8u;
    const uint32_t s_step16 = static_cast<uint32_t>(p.dil_w) * 8u;
    const uint32_t half_cols = static_cast<uint32_t>(p.tmem_cols / 2);
    for (int t = blockIdx.x + mw * gridDim.x; t < p.num_tiles && ok; t += 2 * gridDim.x, iter += 2) {
      const int acc = mw;
      const uint32_t acc_phase = (iter >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&tempty[acc], acc_phase ^ 1, ab, kErrMma))) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * half_cols;
      int n, w0, f0;
      win_tile(p, t, n, w0, f0);
      const uint32_t base_row = static_cast<uint32_t>(f0 - (f0 / p.Wp) * p.Wp);
      for (int c = 0; c < p.kc; ++c) {
        // position of this chunk in the producer's sequence of (tile, chunk) windows
        const int g = iter * p.kc + c;
        const int stage = g % p.stages;
        const uint32_t phase = static_cast<uint32_t>(g / p.stages) & 1u;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, ab, kErrMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t a0 = smem_desc_sw128(smem_base + stage * p.stage_bytes + base_row * 128u, 16, 1024);
        const uint64_t b0 = b_desc0 + static_cast<uint64_t>(c * b_kb16);
        if (kFixed) {
          // one burst per filter row
#pragma unroll
          for (int r = 0; r < KH_; ++r) {
            if (first && r < n_fbars) {
              ok = __all_sync(0xffffffffu, mbar_wait(&fbar[r], 0, ab, kErrMma));
              if (!ok) break;
              tc_fence_after();
            }
            if (elect_sync()) {
              for (int s = 0; s < p.sub; ++s) {
                const uint64_t as = a0 + static_cast<uint64_t>(s * kBM * 8);  // sub-tile s: window rows + 128 s
                const uint32_t ds = d_tmem + static_cast<uint32_t>(s * p.N);
#pragma unroll
                for (int q = 0; q < kKW; ++q)
#pragma unroll
                  for (int k = 0; k < 4; ++k)
                    T::mma(ds, as + a_tap[r * kKW + q] + 2 * k, b0 + b_tap[r * kKW + q] + k * b_step16, p.idesc,
                           (c | r | q | k) != 0 ? 1u : 0u);
              }
              if (r == KH_ - 1) umma_commit(&empty[stage]);
            }
            __syncwarp();
          }
          if (!ok) break;
        } else {
          for (int s = 0; s < p.sub; ++s) {
            const uint32_t ds = d_tmem + static_cast<uint32_t>(s * p.N);
            uint64_t a_r = a0 + static_cast<uint64_t>(s * kBM * 8);
            int tap = 0;
            for (int r = 0; r < p.KH && ok; ++r, a_r += r_step16) {
              if (first && s == 0 && r < n_fbars) {
                ok = __all_sync(0xffffffffu, mbar_wait(&fbar[r], 0, ab, kErrMma));
                if (!ok) break;
                tc_fence_after();
              }
              uint64_t a_s = a_r;
              for (int q = 0; q < p.KW; ++q, ++tap, a_s += s_step16) {
                const uint64_t bd = b0 + static_cast<uint64_t>(tap * p.kc) * b_kb16;
                if (elect_sync()) {
#pragma unroll
                  for (int k = 0; k < 4; ++k)
                    T::mma(ds, a_s + 2 * k, bd + k * b_step16, p.idesc, (c | tap | k) != 0 ? 1u : 0u);
                }
                __syncwarp();
              }
            }
          }
          if (!ok) break;
          if (elect_sync()) umma_commit(&empty[stage]);
          __syncwarp();
        }
        first = false;
      }
      if (ok) {
        if (elect_sync()) umma_commit(&tfull[acc]);
        __syncwarp();
      }
    }
    if (*abort_flag) {
      if (elect_sync()) umma_commit(&drain[mw]);
      __syncwarp();
      mbar_wait_drain(&drain[mw], 0, 500000000ull);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    // Each thread owns one GEMM row (one output pixel) of a sub-tile and
    // stores its accumulator slices straight from registers: 128 contiguous
    // bytes per 32 columns.  Staging through shared memory would add 64 KiB
    // of shared-memory traffic per sub-tile, and with N = 64 the MMAs' operand
    // reads already use most of the shared-memory bandwidth.  Two groups of
    // four warps: with two sub-tiles each group takes one, otherwise they
    // alternate over pairs of 32-column slices.  A warp reads the TMEM lane
    // quarter warp % 4.
    const int q = warp & 3;
    const int eg = (warp - 4) >> 2;
    const int row = q * 32 + lane;  // TMEM lane = GEMM row within a sub-tile
    const int nchunks = p.N / 32;
    const uint32_t half_cols = static_cast<uint32_t>(p.tmem_cols / 2);
    int iter = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++iter) {
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, ab, kErrEpilogue)) break;
      tc_fence_after();
      int n, w0, f0;
      win_tile(p, t, n, w0, f0);
      bool arrived = false;
      for (int s = (p.sub == 2 ? eg : 0); s < p.sub; s += (p.sub == 2 ? 2 : 1)) {
        const int f = f0 + s * kBM + row;
        const int h = f / p.Wp, w = f - h * p.Wp;
        const bool valid = h < p.OH && w < p.Wt && w0 + w < p.OW;
        float* dst = p.out + ((static_cast<int64_t>(p.n_begin + n) * p.out_h + h) * p.out_w + w0 + w) * p.out_c;
        const uint32_t taddr =
            tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * half_cols + static_cast<uint32_t>(s * p.N);
        for (int c = (p.sub == 2 ? 0 : 2 * eg); c < nchunks; c += (p.sub == 2 ? 2 : 4)) {
          const bool two = c + 1 < nchunks;
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(taddr + c * 32, r0);
          if (two) tmem_ld_32x32b_x32(taddr + (c + 1) * 32, r1);
          tmem_wait_ld();
          if (c + (p.sub == 2 ? 2 : 4) >= nchunks) {
            tc_fence_before();
            mbar_arrive(&tempty[acc]);  // this thread's last read: accumulators free for tile + 2
            arrived = true;
          }
          if (valid) {
            store_row<AB>(dst + c * 32, r0, p.v8);
            if (two) store_row<AB>(dst + (c + 1) * 32, r1, p.v8);
          }
        }
      }
      if (!arrived) {  // a group with no slice of this tile
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      }
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

constexpr int kSmemLimit = 227 * 1024;                              // per-CTA dynamic shared memory
constexpr int kDataBudget = kSmemLimit - 1024 - 256 - 2 * kStaging;  // stages + resident filter
constexpr int kResidentLimit = 100 * 1024;
constexpr int kWinDataBudget = kSmemLimit - 1024 - 256;              // window stages + filter

// Plans and launches the window kernel when its shapes fit: the filter stays
// resident, the padded window row is at most 256 pixels (a TMA box limit),
// at least two window stages fit beside the filter, and at least half of the
// padded raster is output columns.  Tiles of two M=128 sub-tiles are used
// when their window and accumulators fit.  Returns false (nothing launched)
// otherwise.
template <int AB, class EncodeInput>
bool launch_window(const ConvArgs& a, const CUtensorMap& m_f, int span, EncodeInput& encode_input, CUtensorMap& m_in,
                   int sms, cudaStream_t stream, cudaError_t* err) {
  using T = ConvTraits<AB>;
  const int eb = T::kEb;
  WinParams p{};
  p.KH = static_cast<int>(a.KH);
  p.KW = static_cast<int>(a.KW);
  p.dil_h = static_cast<int>(a.dil_h);
  p.dil_w = static_cast<int>(a.dil_w);
  p.pad_t = static_cast<int>(a.pad_t);
  p.pad_l = static_cast<int>(a.pad_l);
  p.kc = static_cast<int>((a.C + T::kCh - 1) / T::kCh);
  p.N = static_cast<int>(a.KO);
  p.b_span = span;
  p.b_layout = swizzle_layout_code(span);
  p.b_chunks = p.N * eb / span;
  p.b_chunk_bytes = T::kCh * span;
  p.b_kblock_bytes = p.b_chunks * p.b_chunk_bytes;
  const int filter_bytes = p.KH * p.KW * p.kc * p.b_kblock_bytes;
  if (filter_bytes > kWinDataBudget) return false;
  const int OW = static_cast<int>(a.OW), halo_w = (p.KW - 1) * p.dil_w;
  bool fits = false;
  for (int sub = 4 * p.N <= 512 ? 2 : 1; sub >= 1 && !fits; --sub) {
    for (int tw = 1; tw <= OW && !fits; ++tw) {
      p.Wt = (OW + tw - 1) / tw;
      p.Wp = p.Wt + halo_w;
      if (2 * p.Wt < p.Wp) break;  // mostly halo: the per-tap kernel does better
      if (p.Wp > 256) continue;
      p.Hwin = (p.Wp - 1 + (p.KH - 1) * p.dil_h * p.Wp + halo_w + kBM * sub + p.Wp - 1) / p.Wp;
      if (p.Hwin > 256) continue;
      p.box_bytes = p.Hwin * p.Wp * 128;
      p.stage_bytes = (p.box_bytes + 1023) & ~1023;
      p.stages = (kWinDataBudget - filter_bytes) / p.stage_bytes;
      if (p.stages > kWinMaxStages) p.stages = kWinMaxStages;
      fits = p.stages >= 2;
      p.tiles_w = tw;
      p.sub = sub;
    }
  }
  if (!fits) return false;
  if (!encode_input(p.Wp, p.Hwin)) {
    *err = cudaErrorInvalidValue;
    return true;
  }
  p.ON = static_cast<int>(a.ON);
  p.OH = static_cast<int>(a.OH);
  p.OW = OW;
  p.n_begin = static_cast<int>(a.n_begin);
  p.tiles_per_strip = (p.OH * p.Wp + kBM * p.sub - 1) / (kBM * p.sub);
  p.num_tiles = p.ON * p.tiles_w * p.tiles_per_strip;
  p.filter_offset = p.stages * p.stage_bytes;
  p.barrier_offset = p.filter_offset + filter_bytes;
  int cols = 32;
  while (cols < 2 * p.sub * p.N) cols *= 2;
  p.tmem_cols = cols;
  p.idesc = instr_desc(AB == kBF16 ? 1 : 2, 1, 1, 0, 1, kBM, static_cast<uint32_t>(p.N));
  p.out = a.out;
  p.out_h = a.out_h;
  p.out_w = a.out_w;
  p.out_c = a.out_c;
  p.v8 = a.out_c % 8 == 0 && reinterpret_cast<uintptr_t>(a.out) % 32 == 0;
  p.error_word = a.error_word;
  p.wait_limit = wait_limit_or_default(a.wait_limit_cycles);
  *err = cudaSuccess;
  if (p.num_tiles == 0) return true;
  const int smem = p.barrier_offset + 256 + 1024;
  const int grid = p.num_tiles < sms ? p.num_tiles : sms;
  auto go = [&](auto kernel) {
    *err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (*err != cudaSuccess) return;
    *err = PdlLaunch(grid, kWinThreads, smem, stream)(kernel, m_in, m_f, p);
  };
  if (p.KH == 3 && p.KW == 3)
    go(conv_window<AB, 3, 3>);
  else if (p.KH == 1 && p.KW == 1)
    go(conv_window<AB, 1, 1>);
  else
    go(conv_window<AB, 0, 0>);
  return true;
}

template <int AB>
cudaError_t launch_typed(const ConvArgs& a, cudaStream_t stream) {
  using T = ConvTraits<AB>;
  auto encode = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!encode) return cudaErrorInvalidValue;
  const int eb = T::kEb;
  const CUtensorMapDataType dt = AB == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap m_in, m_f, m_out;
  // input NHWC: dims {C, W, H, N}, box {128 B of channels, box_w, box_h, 1 image}
  auto encode_input = [&](int box_w, int box_h) {
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.C), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                          static_cast<cuuint64_t>(a.N)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(a.C) * eb, static_cast<cuuint64_t>(a.W * a.C) * eb,
                             static_cast<cuuint64_t>(a.H * a.W * a.C) * eb};
    cuuint32_t box[4] = {static_cast<cuuint32_t>(T::kCh), static_cast<cuuint32_t>(box_w),
                         static_cast<cuuint32_t>(box_h), 1};
    return encode(&m_in, dt, 4, const_cast<void*>(a.in), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
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
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (a.max_sms > 0 && a.max_sms < sms) sms = a.max_sms;
  {
    cudaError_t e;
    if (launch_window<AB>(a, m_f, span, encode_input, m_in, sms, stream, &e)) return e;
  }
  if (!encode_input(64, 2)) return cudaErrorInvalidValue;
  // output f32 [N][out_h][out_w][out_c], viewed over the covered extents only
  // ({KO, OW, OH, n_begin + ON}) so TMA clips ragged tiles; box {32 channels, 64 w, 2 h, 1 n}
  {
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.KO), static_cast<cuuint64_t>(a.OW),
                          static_cast<cuuint64_t>(a.OH), static_cast<cuuint64_t>(a.n_begin + a.ON)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(a.out_c) * 4, static_cast<cuuint64_t>(a.out_w * a.out_c) * 4,
                             static_cast<cuuint64_t>(a.out_h * a.out_w * a.out_c) * 4};
    cuuint32_t box[4] = {32, 64, 2, 1};
    if (encode(&m_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.out, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  Params p{};
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
  p.b_kblock_bytes = p.b_chunks * p.b_chunk_bytes;
  const int num_kb = p.KH * p.KW * p.kc;
  const int filter_bytes = num_kb * p.b_kblock_bytes;
  p.resident = filter_bytes <= kResidentLimit && kDataBudget - filter_bytes >= 4 * kAStage;
  p.stage_bytes = kAStage + (p.resident ? 0 : p.b_kblock_bytes);
  const int ring_bytes = kDataBudget - (p.resident ? filter_bytes : 0);
  p.stages = ring_bytes / p.stage_bytes;
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  if (p.stages < 2) return cudaErrorInvalidValue;
  // Largest group of k-blocks per full barrier that divides a tile's k-blocks
  // (so every CTA's k-block count is whole groups) and leaves two groups in
  // the ring, so loading one group overlaps the MMAs of the other.
  p.group = 1;
  for (int g = 4; g > 1; --g)
    if (num_kb % g == 0 && 2 * g <= p.stages) {
      p.group = g;
      break;
    }
  p.stages -= p.stages % p.group;
  p.filter_offset = p.stages * p.stage_bytes;
  p.staging_offset = p.filter_offset + (p.resident ? filter_bytes : 0);
  p.barrier_offset = p.staging_offset + 2 * kStaging;
  int cols = 32;
  while (cols < 2 * p.N) cols *= 2;
  p.tmem_cols = cols;
  p.idesc = instr_desc(AB == kBF16 ? 1 : 2, 1, 1, 0, 1, kBM, static_cast<uint32_t>(p.N));
  p.error_word = a.error_word;
  p.wait_limit = wait_limit_or_default(a.wait_limit_cycles);
  if (p.num_tiles == 0) return cudaSuccess;
  const int smem = p.barrier_offset + 256 + 1024;
  cudaError_t e = cudaFuncSetAttribute(conv_tc<AB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return PdlLaunch(p.num_tiles < sms ? p.num_tiles : sms, kThreads, smem, stream)(conv_tc<AB>, m_in, m_f, m_out, p);
}

}  // namespace

cudaError_t launch_conv(const ConvArgs& a, cudaStream_t stream) {
  if (a.KO % 32 != 0 || a.KO > 256 || a.out_c % 4 != 0) return cudaErrorInvalidValue;
  if (a.elem == kBF16) return launch_typed<kBF16>(a, stream);
  return launch_typed<kI8>(a, stream);
}

}  // namespace dev
}  // namespace xt
