// Tile programs: any Block program the dedicated families do not take.
//
// A program that is one row-tile load and one store of that tile, unchanged
// or transposed, runs the data-movement kernel below.  Every other tile
// program runs a kernel generated for it (codegen.cpp: one CTA per Block,
// each tile value in a shared-memory slot, the ops in order with every shape,
// offset and coordinate a constant of the source) with these semantics:
//   load / store  tile (coordinates x tile dims) of a global array, row-major;
//                 elements past the array edge load 0 and are not stored
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

#include "../codegen.h"
#include "../kernels.h"
#include "pdl.cuh"

namespace xt {
namespace dev {
namespace {

// Data-movement CTA width: the transpose of [8, 2048, 2048] f32 in 32 x 64
// tiles measured 5250 GB/s with 64 threads, 6048 with 128 and 5090 with 256
// (128: four 16-byte loads in flight per thread and up to 16 CTAs per SM).
constexpr int kTileThreads = 128;

// ---------------------------------------------------------------------------
// Pure data movement: the program is one row-tile load and one store of that
// tile, unchanged or transposed (a permute folded into the store), with both
// arrays of one element type.  This kernel takes the tile geometry
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
  MoveArgs m;
  bool transpose = false;
  int eb = 4;
  if (plan_move(a, m, transpose, eb)) {
    const size_t msmem = static_cast<size_t>(m.R) * m.sp * sizeof(float);
    PdlLaunch launch(dim3(static_cast<unsigned>(gx), static_cast<unsigned>(a.grid[1]), static_cast<unsigned>(a.grid[2])),
                     dim3(kTileThreads), msmem, stream);
    if (eb == 4) return transpose ? launch(tile_move<4, true>, m) : launch(tile_move<4, false>, m);
    if (eb == 2) return transpose ? launch(tile_move<2, true>, m) : launch(tile_move<2, false>, m);
    return transpose ? launch(tile_move<1, true>, m) : launch(tile_move<1, false>, m);
  }
  return jit::launch_tile(a, stream);
}

}  // namespace dev
}  // namespace xt
