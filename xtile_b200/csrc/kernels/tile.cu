// Tile-program kernel: any Block program the dedicated families do not take.
//
// One CTA runs one Block.  Every tile value of the program has a slot in
// shared memory (f32 elements, row-major, rows padded to an odd length so
// that column walks hit distinct banks).  The program's ops run in order,
// each as a loop of the CTA's threads over the result tile's elements, with a
// CTA barrier between ops:
//   load / store  tile (coordinates x tile dims) of a global array, row-major,
//                 consecutive threads on consecutive elements of the innermost
//                 dim; elements past the array edge load 0 and are not stored
//                 (the reference's tile semantics, XTToNova.cpp:98);
//   const         a splat tensor constant;
//   unary/binary  the xt elementwise ops (binary operands broadcast along
//                 their size-1 dims); int8 results of add/sub/mul wrap
//                 modulo 256 like the reference's int8 arithmetic;
//   reduce        max or sum along one dim (kept as size 1); sums accumulate
//                 in f64 and round once to f32;
//   reshape       the same row-major element order in a new shape;
//   permute       dims reordered (xt.transpose is the rank-3 swap of the last
//                 two dims, XTOps.cpp:318-327).  A permute whose result only
//                 feeds one store is folded into it by the planner: the
//                 store reads the operand through the permuted strides.
#include <cuda_runtime.h>

#include <atomic>

#include "../kernels.h"
#include "elem_ops.cuh"
#include "pdl.cuh"

namespace xt {
namespace dev {
namespace {

constexpr int kTileThreads = 256;

__device__ __forceinline__ void unravel(int e, const int32_t (&s)[kTileRank], int (&i)[kTileRank]) {
  i[3] = e % s[3];
  e /= s[3];
  i[2] = e % s[2];
  e /= s[2];
  i[1] = e % s[1];
  i[0] = e / s[1];
}

// Walks the multi-indices of elements e = t, t + TH, ... of a rank-4 shape
// (TH threads per CTA): one unravel per thread, then a mixed-radix add of the
// stride's digits with one carry per dim (no division per element).
template <int TH>
struct Walker {
  int i[kTileRank];
  int step[kTileRank];
  int s[kTileRank];
  __device__ __forceinline__ Walker(int t, const int (&shape)[kTileRank]) {
    int32_t sh[kTileRank];
#pragma unroll
    for (int k = 0; k < kTileRank; ++k) s[k] = sh[k] = shape[k];
    unravel(t, sh, i);
    unravel(TH, sh, step);
  }
  __device__ __forceinline__ void next() {
    int c = 0;
#pragma unroll
    for (int k = kTileRank - 1; k >= 0; --k) {
      i[k] += step[k] + c;
      c = i[k] >= s[k];
      i[k] -= c ? s[k] : 0;
    }
  }
};

// A tile value's layout, copied once from the kernel parameters into registers.
struct TV {
  int shape[kTileRank], stride[kTileRank];
  int offset, numel;
  bool i8;
  __device__ __forceinline__ explicit TV(const TileVal& v) {
#pragma unroll
    for (int k = 0; k < kTileRank; ++k) {
      shape[k] = v.shape[k];
      stride[k] = v.stride[k];
    }
    offset = v.offset;
    numel = v.numel;
    i8 = v.i8 != 0;
  }
  __device__ __forceinline__ int at(const int (&i)[kTileRank]) const {
    return offset + i[0] * stride[0] + i[1] * stride[1] + i[2] * stride[2] + i[3];
  }
};

// A tile whose two leading dims are 1 is R x C (R = shape[2], C = shape[3]).
// When C divides the CTA width TH, each thread keeps one column and steps
// whole rows: every offset then advances by a constant, with no index
// arithmetic.
template <int TH>
__device__ __forceinline__ bool rows_of(const TV& v) {
  return v.shape[0] == 1 && v.shape[1] == 1 && TH % v.shape[3] == 0;
}

__device__ __forceinline__ float wrap_i8(float x) {
  return static_cast<float>(static_cast<int8_t>(static_cast<int>(x)));
}

// Where a store reads its tile in shared memory: the stored value's own
// slot, or, for a store with a folded permute (TileOp code 1), the permute's
// operand through the permuted strides.
struct SmemView {
  int offset;
  int stride[kTileRank];
};

__device__ __forceinline__ SmemView store_view(const TileArgs& p, const TileOp& op, const TV& v) {
  SmemView rd;
  if (op.code == 1) {
    rd.offset = p.vals[op.b].offset;
#pragma unroll
    for (int k = 0; k < kTileRank; ++k) rd.stride[k] = p.vals[op.b].stride[op.perm[k]];
  } else {
    rd.offset = v.offset;
#pragma unroll
    for (int k = 0; k < kTileRank; ++k) rd.stride[k] = v.stride[k];
  }
  return rd;
}

// Load or store of one tile: elements past the array edge load 0 / are skipped.
// A load writes the slot of ``v``; a store writes the tile ``v`` (its shape)
// reading each element through ``rd``.
template <bool LOAD, bool ROWS, int TH>
__device__ __forceinline__ void move_tile(float* sm, const TileArgs& p, const TileOp& op, const TV& v,
                                          const int64_t (&bid)[3], const SmemView& rd) {
  int64_t astride[kTileRank];
  int lim[kTileRank];
  int64_t base = 0;
  int64_t run = 1;
#pragma unroll
  for (int d = kTileRank - 1; d >= 0; --d) {
    const int64_t ext = p.shape[op.arg][d];
    const int cb = op.coord_bid[d];
    const int64_t c = cb == 0 ? bid[0] : cb == 1 ? bid[1] : cb == 2 ? bid[2] : op.coord[d];
    const int64_t start = c * static_cast<int64_t>(v.shape[d]);
    astride[d] = run;
    base += start * run;
    run *= ext;
    const int64_t left = ext - start;  // elements of this dim inside the array
    lim[d] = left <= 0 ? 0 : (left > v.shape[d] ? v.shape[d] : static_cast<int>(left));
  }
  void* arr = p.arr[op.arg];
  const uint8_t elem = p.elem[op.arg];
  constexpr int kBatch = 8;
  if ((ROWS || rows_of<TH>(v)) && elem == kF32 && v.shape[3] % 4 == 0 && lim[3] % 4 == 0 && base % 4 == 0 &&
      astride[2] % 4 == 0 && (reinterpret_cast<uintptr_t>(arr) & 15) == 0) {
    constexpr int kVecBatch = 4;  // float4s in flight per thread
    // f32 rows of a multiple of 4 elements at 16-byte aligned global offsets:
    // one float4 per thread per access (shared memory stays scalar: its rows
    // are padded to an odd length)
    const int C4 = v.shape[3] / 4, R = v.shape[2];
    const int c = (threadIdx.x % C4) * 4, rs = TH / C4;
    const bool col_in = c < lim[3] && lim[0] > 0 && lim[1] > 0;
    const int r_lim = lim[2];
    float4* g = reinterpret_cast<float4*>(arr);
    for (int r = threadIdx.x / C4; r < R; r += kVecBatch * rs) {
      if (LOAD) {
        float4 val[kVecBatch];
#pragma unroll
        for (int u = 0; u < kVecBatch; ++u) {
          const int ru = r + u * rs;
          val[u] = (col_in && ru < r_lim) ? __ldg(g + (base + ru * astride[2] + c) / 4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kVecBatch; ++u) {
          const int ru = r + u * rs;
          if (ru < R) {
            float* d = sm + v.offset + ru * v.stride[2] + c;
            d[0] = val[u].x;
            d[1] = val[u].y;
            d[2] = val[u].z;
            d[3] = val[u].w;
          }
        }
      } else if (col_in) {
        const int cs = rd.stride[3];
#pragma unroll
        for (int u = 0; u < kVecBatch; ++u) {
          const int ru = r + u * rs;
          if (ru < r_lim) {
            const float* s4 = sm + rd.offset + ru * rd.stride[2] + c * cs;
            g[(base + ru * astride[2] + c) / 4] = make_float4(s4[0], s4[cs], s4[2 * cs], s4[3 * cs]);
          }
        }
      }
    }
    return;
  }
  if (ROWS || rows_of<TH>(v)) {
    const int C = v.shape[3], R = v.shape[2];
    const int c = threadIdx.x % C, rs = TH / C;
    const bool col_in = c < lim[3] && lim[0] > 0 && lim[1] > 0;
    const int r_lim = lim[2];
    const int64_t gstep = rs * astride[2];
    const int sstep = rs * v.stride[2];
    int r = threadIdx.x / C;
    int64_t goff = base + r * astride[2] + c;
    int soff = v.offset + r * v.stride[2] + c;
    if (LOAD) {
      for (; r < R; r += kBatch * rs) {
        float val[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int ru = r + u * rs;
          val[u] = (col_in && ru < r_lim) ? load_elem(arr, elem, goff + u * gstep) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
          if (r + u * rs < R) sm[soff + u * sstep] = val[u];
        goff += kBatch * gstep;
        soff += kBatch * sstep;
      }
    } else if (col_in) {
      int roff = rd.offset + r * rd.stride[2] + c * rd.stride[3];
      const int rstep = rs * rd.stride[2];
      for (; r < r_lim; r += rs, goff += gstep, roff += rstep) store_elem(arr, elem, goff, sm[roff]);
    }
    return;
  }
  if constexpr (ROWS) return;
  Walker<TH> w(threadIdx.x, v.shape);
  if (LOAD) {
    // kBatch independent loads in flight per thread before their shared-memory
    // stores: one HBM round trip per kBatch elements, not per element
    for (int e0 = threadIdx.x; e0 < v.numel; e0 += kBatch * TH) {
      float val[kBatch];
      int dst[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const bool live = e0 + u * TH < v.numel;
        const bool in = live && w.i[0] < lim[0] && w.i[1] < lim[1] && w.i[2] < lim[2] && w.i[3] < lim[3];
        const int64_t off = base + w.i[0] * astride[0] + w.i[1] * astride[1] + w.i[2] * astride[2] + w.i[3];
        val[u] = in ? load_elem(arr, elem, off) : 0.0f;
        dst[u] = live ? v.at(w.i) : -1;
        w.next();
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (dst[u] >= 0) sm[dst[u]] = val[u];
    }
  } else {
    for (int e = threadIdx.x; e < v.numel; e += TH, w.next()) {
      const bool in = w.i[0] < lim[0] && w.i[1] < lim[1] && w.i[2] < lim[2] && w.i[3] < lim[3];
      const int64_t off = base + w.i[0] * astride[0] + w.i[1] * astride[1] + w.i[2] * astride[2] + w.i[3];
      if (in)
        store_elem(arr, elem, off,
                   sm[rd.offset + w.i[0] * rd.stride[0] + w.i[1] * rd.stride[1] + w.i[2] * rd.stride[2] +
                      w.i[3] * rd.stride[3]]);
    }
  }
}

// ROWS: every tile of the program is R x C with C dividing the CTA width (the
// planner checks), so only the row paths are compiled: fewer registers, more
// CTAs per SM.
//
// TH threads per CTA: 256, or 128 for programs of small tiles (the launcher
// decides), which halves what the per-op set-up costs a Block while twice as
// many CTAs share an SM.
template <bool ROWS, int TH>
__global__ void __launch_bounds__(TH, ROWS ? (TH == 256 ? 5 : TH == 128 ? 10 : 20) : (256 / TH))
    tile_program(const __grid_constant__ TileArgs p) {
  extern __shared__ float sm[];
  griddep_launch_dependents();
  griddep_wait();
  const int64_t bid[3] = {p.bid0_begin + blockIdx.x, blockIdx.y, blockIdx.z};
  const int n_ops = p.n_ops;
  for (int o = 0; o < n_ops; ++o) {
    const TileOp& op = p.ops[o];
    const uint8_t kind = op.kind, code = op.code;
    switch (kind) {
      case kTLoad: {
        const TV v(p.vals[op.dst]);
        move_tile<true, ROWS, TH>(sm, p, op, v, bid, SmemView{});
        break;
      }
      case kTStore: {
        const TV v(p.vals[op.a]);
        move_tile<false, ROWS, TH>(sm, p, op, v, bid, store_view(p, op, v));
        break;
      }
      case kTConst: {
        const TV d(p.vals[op.dst]);
        const float value = op.value;
        if (ROWS || rows_of<TH>(d)) {
          const int C = d.shape[3], c = threadIdx.x % C, rs = TH / C;
          for (int r = threadIdx.x / C; r < d.shape[2]; r += rs) sm[d.offset + r * d.stride[2] + c] = value;
          break;
        }
        if constexpr (!ROWS) {
          Walker<TH> w(threadIdx.x, d.shape);
          for (int e = threadIdx.x; e < d.numel; e += TH, w.next()) sm[d.at(w.i)] = value;
        }
        break;
      }
      case kTUnary: {
        const TV d(p.vals[op.dst]), a(p.vals[op.a]);
        if (ROWS || rows_of<TH>(d)) {
          const int C = d.shape[3], c = threadIdx.x % C, rs = TH / C;
          for (int r = threadIdx.x / C; r < d.shape[2]; r += rs)
            sm[d.offset + r * d.stride[2] + c] = unary_op(code, sm[a.offset + r * a.stride[2] + c]);
          break;
        }
        if constexpr (!ROWS) {
          Walker<TH> w(threadIdx.x, d.shape);
          for (int e = threadIdx.x; e < d.numel; e += TH, w.next())
            sm[d.at(w.i)] = unary_op(code, sm[a.at(w.i)]);
        }
        break;
      }
      case kTBinary: {
        const TV d(p.vals[op.dst]), a(p.vals[op.a]), b(p.vals[op.b]);
        // broadcast dims (size 1) contribute no stride
        int sa[kTileRank], sb[kTileRank];
#pragma unroll
        for (int k = 0; k < kTileRank; ++k) {
          sa[k] = a.shape[k] == 1 ? 0 : a.stride[k];
          sb[k] = b.shape[k] == 1 ? 0 : b.stride[k];
        }
        if (ROWS || rows_of<TH>(d)) {
          const int C = d.shape[3], c = threadIdx.x % C, rs = TH / C;
          for (int r = threadIdx.x / C; r < d.shape[2]; r += rs) {
            const float x = sm[a.offset + r * sa[2] + c * sa[3]];
            const float y = sm[b.offset + r * sb[2] + c * sb[3]];
            const float v = binary_op(code, x, y);
            sm[d.offset + r * d.stride[2] + c] = d.i8 ? wrap_i8(v) : v;
          }
          break;
        }
        if constexpr (!ROWS) {
          Walker<TH> w(threadIdx.x, d.shape);
          for (int e = threadIdx.x; e < d.numel; e += TH, w.next()) {
            const int(&i)[kTileRank] = w.i;
            const float x = sm[a.offset + i[0] * sa[0] + i[1] * sa[1] + i[2] * sa[2] + i[3] * sa[3]];
            const float y = sm[b.offset + i[0] * sb[0] + i[1] * sb[1] + i[2] * sb[2] + i[3] * sb[3]];
            const float r = binary_op(code, x, y);
            sm[d.at(i)] = d.i8 ? wrap_i8(r) : r;
          }
        }
        break;
      }
      case kTReduce: {
        const TV d(p.vals[op.dst]), a(p.vals[op.a]);
        const int n = p.vals[op.a].shape[op.axis];  // parameter reads: no runtime index into registers
        const int step = p.vals[op.a].stride[op.axis];
        if constexpr (ROWS) {
          // rows mode: d is R x C with the reduced dim (2 or 3) of size 1
          const int C = d.shape[3];
          for (int e = threadIdx.x; e < d.numel; e += TH) {
            const int r = e / C, c = e - (e / C) * C;
            const float* src = sm + a.offset + r * a.stride[2] + c;
            float v;
            if (code == 0) {
              v = src[0];
              for (int j = 1; j < n; ++j) {
                const float x = src[j * step];
                if (x != x || x > v) v = x;
              }
            } else {
              double acc = 0.0;
              for (int j = 0; j < n; ++j) acc += static_cast<double>(src[j * step]);
              v = static_cast<float>(acc);
            }
            sm[d.offset + r * d.stride[2] + c] = v;
          }
          break;
        }
        Walker<TH> w(threadIdx.x, d.shape);
        for (int e = threadIdx.x; e < d.numel; e += TH, w.next()) {
          const float* src = sm + a.at(w.i);  // the reduced dim's index is 0 in w.i
          float r;
          if (code == 0) {
            r = src[0];
            for (int j = 1; j < n; ++j) {
              const float x = src[j * step];
              if (x != x || x > r) r = x;  // NaN propagates, as np.max
            }
          } else {
            double s = 0.0;
            for (int j = 0; j < n; ++j) s += static_cast<double>(src[j * step]);
            r = static_cast<float>(s);
          }
          sm[d.at(w.i)] = r;
        }
        break;
      }
      case kTReshape: {
        const TV d(p.vals[op.dst]), a(p.vals[op.a]);
        if constexpr (ROWS) {
          const int dc = d.shape[3], ac = a.shape[3];
          for (int e = threadIdx.x; e < d.numel; e += TH)
            sm[d.offset + (e / dc) * d.stride[2] + e % dc] = sm[a.offset + (e / ac) * a.stride[2] + e % ac];
        } else {
          Walker<TH> wd(threadIdx.x, d.shape), wa(threadIdx.x, a.shape);
          for (int e = threadIdx.x; e < d.numel; e += TH, wd.next(), wa.next())
            sm[d.at(wd.i)] = sm[a.at(wa.i)];
        }
        break;
      }
      case kTPermute: {
        const TV d(p.vals[op.dst]), a(p.vals[op.a]);
        // dst dim k is src dim perm[k]: the source offset walks the source strides in dst order
        int ss[kTileRank];
#pragma unroll
        for (int k = 0; k < kTileRank; ++k) ss[k] = p.vals[op.a].stride[op.perm[k]];
        if (ROWS || rows_of<TH>(d)) {
          const int C = d.shape[3], c = threadIdx.x % C, rs = TH / C;
          for (int r = threadIdx.x / C; r < d.shape[2]; r += rs)
            sm[d.offset + r * d.stride[2] + c] = sm[a.offset + r * ss[2] + c * ss[3]];
          break;
        }
        if constexpr (!ROWS) {
          Walker<TH> w(threadIdx.x, d.shape);
          for (int e = threadIdx.x; e < d.numel; e += TH, w.next()) {
            const int(&i)[kTileRank] = w.i;
            sm[d.at(i)] = sm[a.offset + i[0] * ss[0] + i[1] * ss[1] + i[2] * ss[2] + i[3] * ss[3]];
          }
        }
        break;
      }
      default:
        break;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Pure data movement: the program is one row-tile load and one store of that
// tile, unchanged or transposed (a permute folded into the store), with both
// arrays of one element type.  The interpreter above spends most of its issue
// slots on per-op set-up (64-bit geometry, runtime divisions, op decoding)
// for 8 elements per thread; this kernel takes the tile geometry
// precomputed on the host as per-axis multipliers and moves 16 bytes per
// thread access (4 f32, 8 bf16 or 16 int8 elements) with power-of-two thread
// layouts.  Shared memory holds the tile as f32 values, which every f32,
// bf16 and int8 value converts to and from exactly.
struct MoveGeom {
  int64_t cst;          // first element of the tile for bid = (0, 0, 0)
  int64_t mult[3];      // elements per unit of bid(k)
  int64_t row;          // array row stride (elements)
  int64_t r_cst, c_cst;      // first tile row / column (array indices) for bid = (0, 0, 0)
  int32_t r_mult[3], c_mult[3];  // rows / columns per unit of bid(k)
  int32_t ext_r, ext_c;      // array rows / columns
};

struct MoveArgs {
  const void* in;
  void* out;
  MoveGeom g_in, g_out;
  int32_t R, C;         // loaded tile rows x columns
  int32_t lc, lo;       // log2 of 16-byte vectors per loaded / stored tile row
  int32_t sp;           // shared-memory row stride of the loaded tile (odd)
  int64_t bid0_begin;
};

// 16 bytes of elements of EB bytes each <-> f32 values.
template <int EB>
struct Vec16 {
  static constexpr int n = 16 / EB;
  static __device__ __forceinline__ void unpack(const uint4& u, float (&f)[n]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (EB == 4) {
        f[i] = __uint_as_float(w[i]);
      } else if constexpr (EB == 2) {  // bf16: the high half of an f32
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      } else {  // int8
#pragma unroll
        for (int k = 0; k < 4; ++k) f[4 * i + k] = static_cast<float>(static_cast<int8_t>(w[i] >> (8 * k)));
      }
    }
  }
  // exact for values that came from this element type
  static __device__ __forceinline__ uint4 pack(const float (&f)[n]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (EB == 4) {
        w[i] = __float_as_uint(f[i]);
      } else if constexpr (EB == 2) {
        w[i] = (__float_as_uint(f[2 * i]) >> 16) | (__float_as_uint(f[2 * i + 1]) & 0xffff0000u);
      } else {
        w[i] = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          w[i] |= static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(f[4 * i + k]))) << (8 * k);
      }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

__device__ __forceinline__ void move_geom(const MoveGeom& g, const int64_t (&bid)[3], int rows, int cols,
                                          int64_t& base, int& nr, int& nc) {
  base = g.cst + bid[0] * g.mult[0] + bid[1] * g.mult[1] + bid[2] * g.mult[2];
  const int64_t r0 = g.r_cst + bid[0] * g.r_mult[0] + bid[1] * g.r_mult[1] + bid[2] * g.r_mult[2];
  const int64_t c0 = g.c_cst + bid[0] * g.c_mult[0] + bid[1] * g.c_mult[1] + bid[2] * g.c_mult[2];
  const int64_t lr = g.ext_r - r0, lc = g.ext_c - c0;
  nr = lr <= 0 ? 0 : (lr < rows ? static_cast<int>(lr) : rows);
  nc = lc <= 0 ? 0 : (lc < cols ? static_cast<int>(lc) : cols);
}

template <int EB, bool TRANSPOSE>
__global__ void __launch_bounds__(kTileThreads) tile_move(const __grid_constant__ MoveArgs p) {
  using V = Vec16<EB>;
  constexpr int kN = V::n;
  extern __shared__ float sm[];
  griddep_launch_dependents();
  griddep_wait();
  const int64_t bid[3] = {p.bid0_begin + blockIdx.x, blockIdx.y, blockIdx.z};
  const int R = p.R, C = p.C, sp = p.sp;
  int64_t base;
  int nr, nc;
  move_geom(p.g_in, bid, R, C, base, nr, nc);
  {
    // loaded tile: vector column cv of rows r, r + rs, ...; up to 4 in flight
    const int cv = threadIdx.x & ((1 << p.lc) - 1);
    const int rs = kTileThreads >> p.lc;
    const bool col_in = kN * cv < nc;
    const uint4* g = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.in) + base * EB) + cv;
    const int64_t rowv = p.g_in.row / kN;
    for (int r = threadIdx.x >> p.lc; r < R; r += 4 * rs) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int ru = r + u * rs;
        v[u] = (col_in && ru < nr) ? __ldg(g + ru * rowv) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int ru = r + u * rs;
        if (ru < R) {
          float f[kN];
          V::unpack(v[u], f);
          float* d = sm + ru * sp + kN * cv;
#pragma unroll
          for (int k = 0; k < kN; ++k) d[k] = f[k];
        }
      }
    }
  }
  __syncthreads();
  const int OR = TRANSPOSE ? C : R, OC = TRANSPOSE ? R : C;
  move_geom(p.g_out, bid, OR, OC, base, nr, nc);
  const int cv = threadIdx.x & ((1 << p.lo) - 1);
  if (kN * cv >= nc) return;
  const int rs = kTileThreads >> p.lo;
  uint4* g = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + base * EB) + cv;
  const int64_t rowv = p.g_out.row / kN;
  for (int r = threadIdx.x >> p.lo; r < nr; r += rs) {
    float f[kN];
    if (TRANSPOSE) {
      const float* s = sm + kN * cv * sp + r;  // output (r, kN cv + k) = loaded (kN cv + k, r)
#pragma unroll
      for (int k = 0; k < kN; ++k) f[k] = s[k * sp];
    } else {
      const float* s = sm + r * sp + kN * cv;
#pragma unroll
      for (int k = 0; k < kN; ++k) f[k] = s[k];
    }
    g[r * rowv] = V::pack(f);
  }
}

// The move kernel's arguments when the program is a plain row-tile load and
// store (optionally transposed) that it can run; false otherwise.
bool plan_move(const TileArgs& a, MoveArgs& m, bool& transpose, int& eb) {
  if (a.n_ops != 2 || a.ops[0].kind != kTLoad || a.ops[1].kind != kTStore) return false;
  const TileOp &ld = a.ops[0], &st = a.ops[1];
  const TileVal& v = a.vals[ld.dst];
  const TileVal& o = a.vals[st.a];
  const bool copy = st.code == 0 && st.a == ld.dst;
  transpose = st.code == 1 && st.b == ld.dst && st.perm[0] == 0 && st.perm[1] == 1 && st.perm[2] == 3 &&
              st.perm[3] == 2;
  if (!copy && !transpose) return false;
  if (a.elem[ld.arg] != a.elem[st.arg]) return false;
  eb = a.elem[ld.arg] == kF32 ? 4 : a.elem[ld.arg] == kBF16 ? 2 : 1;
  const int vn = 16 / eb;  // elements per 16-byte vector
  if (v.shape[0] != 1 || v.shape[1] != 1 || o.shape[0] != 1 || o.shape[1] != 1) return false;
  const int R = v.shape[2], C = v.shape[3];
  const int OC = transpose ? R : C;
  auto log2_of = [](int x) {
    int l = 0;
    while ((1 << l) < x) ++l;
    return (1 << l) == x ? l : -1;
  };
  if (C % vn || OC % vn) return false;
  const int lc = log2_of(C / vn), lo = log2_of(OC / vn);
  if (lc < 0 || lo < 0 || C / vn > kTileThreads || OC / vn > kTileThreads) return false;
  const int sp = C % 2 == 0 ? C + 1 : C;
  if (static_cast<int64_t>(R) * sp > 12 * 1024) return false;  // 48 KiB of shared memory
  if ((reinterpret_cast<uintptr_t>(a.arr[ld.arg]) | reinterpret_cast<uintptr_t>(a.arr[st.arg])) & 15) return false;
  auto geom = [&](const TileOp& op, const TileVal& t, MoveGeom& g) {
    const int32_t* ext = a.shape[op.arg];
    if (ext[3] % vn) return false;  // rows of whole 16-byte vectors
    int64_t astride[kTileRank], run = 1;
    for (int d = kTileRank - 1; d >= 0; --d) {
      astride[d] = run;
      run *= ext[d];
    }
    g = MoveGeom{};
    g.row = astride[2];
    g.ext_r = ext[2];
    g.ext_c = ext[3];
    for (int d = 0; d < kTileRank; ++d) {
      const int cb = op.coord_bid[d];
      // leading dims: tile extent 1; every Block's coordinate must lie inside the array
      if (d < 2 && (cb >= 0 ? a.grid[cb] > ext[d] : op.coord[d] >= ext[d])) return false;
      const int64_t step = static_cast<int64_t>(t.shape[d]);
      if (cb >= 0) {
        g.mult[cb] += step * astride[d];
        if (d == 2) g.r_mult[cb] = static_cast<int32_t>(step);
        if (d == 3) g.c_mult[cb] = static_cast<int32_t>(step);
      } else {
        g.cst += op.coord[d] * step * astride[d];
        if (d == 2) g.r_cst = op.coord[d] * step;
        if (d == 3) g.c_cst = op.coord[d] * step;
      }
    }
    return true;
  };
  if (!geom(ld, v, m.g_in) || !geom(st, o, m.g_out)) return false;
  m.in = a.arr[ld.arg];
  m.out = a.arr[st.arg];
  m.R = R;
  m.C = C;
  m.lc = lc;
  m.lo = lo;
  m.sp = sp;
  m.bid0_begin = a.bid0_begin;
  return true;
}

}  // namespace

cudaError_t launch_tile(const TileArgs& a, cudaStream_t stream) {
  const int64_t gx = a.bid0_end - a.bid0_begin;
  if (gx <= 0) return cudaSuccess;
  if (gx > 0x7fffffff || a.grid[1] > 65535 || a.grid[2] > 65535) return cudaErrorInvalidValue;
  {
    MoveArgs m;
    bool transpose = false;
    int eb = 4;
    if (plan_move(a, m, transpose, eb)) {
      const size_t msmem = static_cast<size_t>(m.R) * m.sp * sizeof(float);
      PdlLaunch launch(dim3(static_cast<unsigned>(gx), static_cast<unsigned>(a.grid[1]),
                            static_cast<unsigned>(a.grid[2])),
                       dim3(kTileThreads), msmem, stream);
      if (eb == 4) return transpose ? launch(tile_move<4, true>, m) : launch(tile_move<4, false>, m);
      if (eb == 2) return transpose ? launch(tile_move<2, true>, m) : launch(tile_move<2, false>, m);
      return transpose ? launch(tile_move<1, true>, m) : launch(tile_move<1, false>, m);
    }
  }
  // 128 threads for programs of small tiles whose rows (in the row-only
  // variant) divide 128 columns
  bool small = true, tiny = true;
  for (int v = 0; v < kTileMaxVals; ++v)
    if (a.vals[v].numel > 0) {
      small = small && a.vals[v].numel <= 4096 && (!a.rows || 128 % a.vals[v].shape[3] == 0);
      tiny = tiny && a.vals[v].numel <= 2048 && (!a.rows || 64 % a.vals[v].shape[3] == 0);
    }
  const int th = tiny ? 64 : small ? 128 : kTileThreads;
  const size_t smem = static_cast<size_t>(a.smem_floats) * sizeof(float);
  if (smem > 48 * 1024) {
    // the opt-in to more than 48 KiB is per device; set it to the family's maximum once
    int dev = 0;
    cudaGetDevice(&dev);
    static std::atomic<uint64_t> attr_devices{0};
    const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
    if (!(attr_devices.load(std::memory_order_relaxed) & bit)) {
      for (auto k : {tile_program<true, 256>, tile_program<false, 256>, tile_program<true, 128>,
                     tile_program<false, 128>, tile_program<true, 64>, tile_program<false, 64>}) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kTileSmemFloats * static_cast<int>(sizeof(float)));
        if (e != cudaSuccess) return e;
      }
      attr_devices.fetch_or(bit, std::memory_order_relaxed);
    }
  }
  PdlLaunch launch(dim3(static_cast<unsigned>(gx), static_cast<unsigned>(a.grid[1]), static_cast<unsigned>(a.grid[2])),
                   dim3(th), smem, stream);
  if (th == 64) return a.rows ? launch(tile_program<true, 64>, a) : launch(tile_program<false, 64>, a);
  if (th == 128) return a.rows ? launch(tile_program<true, 128>, a) : launch(tile_program<false, 128>, a);
  return a.rows ? launch(tile_program<true, 256>, a) : launch(tile_program<false, 256>, a);
}

}  // namespace dev
}  // namespace xt
