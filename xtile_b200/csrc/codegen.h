// Kernels generated per Block program (ew, rows and tile families),
// compiled at run time with NVRTC for sm_100a.
//
// The planner turns an elementwise or row program into a short register
// program (plan.h: Instr).  Instead of interpreting it on the GPU, the host
// writes it out as straight-line CUDA C++ -- each value a register, each op
// the op_math.cuh function applied in place -- compiles it once per program
// and device, and launches the cubin.  Programs are cached by their code,
// element types and shapes, so a program compiles once per process.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "kernels.h"

namespace xt {
namespace jit {

// CUDA source of the ew kernels for a program (its code, element types and
// broadcast flags): ``xt_ew_v`` (4 * kEwVec elements per thread and pass, for
// aligned arrays) and ``xt_ew_s`` (one element per thread, any alignment).
std::string ew_source(const dev::EwArgs& a);
// CUDA source of the rows kernels for a program of rows of ``a.cols``
// columns: ``xt_rows_v`` (float4 accesses, cols % 4 == 0 on 16-byte aligned
// rows) and ``xt_rows_s`` (element accesses).
std::string rows_source(const dev::RowArgs& a);
// Whether a rows program runs the one-warp-per-row kernels: rows of at most
// 2048 columns whose live rows a lane holds in at most 160 values.  Others
// run ``xt_rows_cv`` / ``xt_rows_cs`` (rows_cta_source): one CTA of
// ``tpr`` threads per row (row_cta_threads in plan.h), block reductions.
bool rows_fit(const dev::RowArgs& a);
std::string rows_cta_source(const dev::RowArgs& a, int tpr);
// The source a launch of the rows program compiles (one of the two above).
std::string rows_kernel_source(const dev::RowArgs& a);

// CUDA source of the tile-program kernels for ``a`` run by ``threads``
// threads per CTA: ``xt_tile_v`` (accesses whose rows are whole 4-element
// groups move 4 elements at a time; every array 16-byte aligned) and
// ``xt_tile_s`` (element accesses).
std::string tile_source(const dev::TileArgs& a, int threads);
// The CTA width for a tile program by its largest tile: 128 threads up to
// 4096 elements, 256 up to 8192, 512 up to 16384, else 1024 (column sums of
// 64 x 32 tiles: 4391 GB/s with 64 threads, 5979 with 128, 5124 with 256;
// large tiles hold an SM alone and need the loads of many threads in flight).
int tile_threads(const dev::TileArgs& a);
// Shared memory (floats) of the tile kernel for ``a`` at ``threads``
// threads: the planned slots, then one double per thread for the partial
// results of reductions when the program reduces.
int tile_smem_floats(const dev::TileArgs& a, int threads);

// Compiles ``source`` with NVRTC for sm_100a; returns the cubin.  Throws
// xt::Error (kCudaError) with NVRTC's log on failure or when NVRTC cannot be
// loaded.  Needs no GPU.
std::string compile(const std::string& source);

// Launches the generated ew / rows kernels for ``a`` on ``stream`` (compiling
// and loading them on first use on the current device).
cudaError_t launch_ew(const dev::EwArgs& a, cudaStream_t stream);
cudaError_t launch_rows(const dev::RowArgs& a, cudaStream_t stream);
cudaError_t launch_tile(const dev::TileArgs& a, cudaStream_t stream);

constexpr int kEwVec = 2;          // float4 groups per thread and pass in xt_ew_v
constexpr int kEwThreads = 256;
constexpr int kRowsPerCta = 4;     // one warp per row

}  // namespace jit
}  // namespace xt
