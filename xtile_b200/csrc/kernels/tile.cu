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
//                 two dims, XTOps.cpp:318-327).
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

__device__ __forceinline__ int slot(const TileVal& v, const int (&i)[kTileRank]) {
  return v.offset + i[0] * v.stride[0] + i[1] * v.stride[1] + i[2] * v.stride[2] + i[3];
}

__device__ __forceinline__ float wrap_i8(float x) {
  return static_cast<float>(static_cast<int8_t>(static_cast<int>(x)));
}

__global__ void __launch_bounds__(kTileThreads) tile_program(const __grid_constant__ TileArgs p) {
  extern __shared__ float sm[];
  griddep_launch_dependents();
  griddep_wait();
  const int64_t bid[3] = {p.bid0_begin + blockIdx.x, blockIdx.y, blockIdx.z};
  for (int o = 0; o < p.n_ops; ++o) {
    const TileOp& op = p.ops[o];
    switch (op.kind) {
      case kTLoad:
      case kTStore: {
        const bool load = op.kind == kTLoad;
        const TileVal& v = p.vals[load ? op.dst : op.a];
        const int32_t(&as)[kTileRank] = p.shape[op.arg];
        int64_t start[kTileRank];
#pragma unroll
        for (int d = 0; d < kTileRank; ++d)
          start[d] = (op.coord_bid[d] >= 0 ? bid[op.coord_bid[d]] : op.coord[d]) * static_cast<int64_t>(v.shape[d]);
        for (int e = threadIdx.x; e < v.numel; e += kTileThreads) {
          int i[kTileRank];
          unravel(e, v.shape, i);
          bool in = true;
          int64_t off = 0;
#pragma unroll
          for (int d = 0; d < kTileRank; ++d) {
            const int64_t g = start[d] + i[d];
            in = in && g < as[d];
            off = off * as[d] + g;
          }
          if (load)
            sm[slot(v, i)] = in ? load_elem(p.arr[op.arg], p.elem[op.arg], off) : 0.0f;
          else if (in)
            store_elem(p.arr[op.arg], p.elem[op.arg], off, sm[slot(v, i)]);
        }
        break;
      }
      case kTConst: {
        const TileVal& d = p.vals[op.dst];
        for (int e = threadIdx.x; e < d.numel; e += kTileThreads) {
          int i[kTileRank];
          unravel(e, d.shape, i);
          sm[slot(d, i)] = op.value;
        }
        break;
      }
      case kTUnary: {
        const TileVal &d = p.vals[op.dst], &a = p.vals[op.a];
        for (int e = threadIdx.x; e < d.numel; e += kTileThreads) {
          int i[kTileRank];
          unravel(e, d.shape, i);
          sm[slot(d, i)] = unary_op(op.code, sm[slot(a, i)]);
        }
        break;
      }
      case kTBinary: {
        const TileVal &d = p.vals[op.dst], &a = p.vals[op.a], &b = p.vals[op.b];
        for (int e = threadIdx.x; e < d.numel; e += kTileThreads) {
          int i[kTileRank], ia[kTileRank], ib[kTileRank];
          unravel(e, d.shape, i);
#pragma unroll
          for (int k = 0; k < kTileRank; ++k) {
            ia[k] = a.shape[k] == 1 ? 0 : i[k];
            ib[k] = b.shape[k] == 1 ? 0 : i[k];
          }
          float r = binary_op(op.code, sm[slot(a, ia)], sm[slot(b, ib)]);
          sm[slot(d, i)] = d.i8 ? wrap_i8(r) : r;
        }
        break;
      }
      case kTReduce: {
        const TileVal &d = p.vals[op.dst], &a = p.vals[op.a];
        const int n = a.shape[op.axis];
        const int step = a.stride[op.axis];
        for (int e = threadIdx.x; e < d.numel; e += kTileThreads) {
          int i[kTileRank];
          unravel(e, d.shape, i);
          const float* src = sm + slot(a, i);  // the reduced dim's index is 0 in i
          float r;
          if (op.code == 0) {
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
          sm[slot(d, i)] = r;
        }
        break;
      }
      case kTReshape: {
        const TileVal &d = p.vals[op.dst], &a = p.vals[op.a];
        for (int e = threadIdx.x; e < d.numel; e += kTileThreads) {
          int i[kTileRank], j[kTileRank];
          unravel(e, d.shape, i);
          unravel(e, a.shape, j);
          sm[slot(d, i)] = sm[slot(a, j)];
        }
        break;
      }
      case kTPermute: {
        const TileVal &d = p.vals[op.dst], &a = p.vals[op.a];
        for (int e = threadIdx.x; e < d.numel; e += kTileThreads) {
          int i[kTileRank], j[kTileRank];
          unravel(e, d.shape, i);
#pragma unroll
          for (int k = 0; k < kTileRank; ++k) j[op.perm[k]] = i[k];
          sm[slot(d, i)] = sm[slot(a, j)];
        }
        break;
      }
      default:
        break;
    }
    __syncthreads();
  }
}

}  // namespace

cudaError_t launch_tile(const TileArgs& a, cudaStream_t stream) {
  const int64_t gx = a.bid0_end - a.bid0_begin;
  if (gx <= 0) return cudaSuccess;
  if (gx > 0x7fffffff || a.grid[1] > 65535 || a.grid[2] > 65535) return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(a.smem_floats) * sizeof(float);
  if (smem > 48 * 1024) {
    // the opt-in to more than 48 KiB is per device; set it to the family's maximum once
    int dev = 0;
    cudaGetDevice(&dev);
    static std::atomic<uint64_t> attr_devices{0};
    const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
    if (!(attr_devices.load(std::memory_order_relaxed) & bit)) {
      cudaError_t e = cudaFuncSetAttribute(tile_program, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kTileSmemFloats * static_cast<int>(sizeof(float)));
      if (e != cudaSuccess) return e;
      attr_devices.fetch_or(bit, std::memory_order_relaxed);
    }
  }
  return PdlLaunch(dim3(static_cast<unsigned>(gx), static_cast<unsigned>(a.grid[1]), static_cast<unsigned>(a.grid[2])),
                   dim3(kTileThreads), smem, stream)(tile_program, a);
}

}  // namespace dev
}  // namespace xt
