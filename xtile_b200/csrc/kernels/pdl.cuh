// Programmatic dependent launch (PDL) for back-to-back Block programs.
//
// Every kernel of this backend is launched with programmatic stream
// serialization: the next launch on the stream may be scheduled while this
// one drains, so its CTAs are placed and finish their set-up (barrier init,
// TMEM allocation, tensor-map prefetch) during the previous grid's tail
// instead of after a full launch gap.  Stream order for memory is unchanged:
// each kernel executes griddep_wait() before its first global-memory access,
// and that wait returns only once the preceding grid has completed and its
// writes are visible.  Without a programmatic predecessor (the first launch,
// a launch after a copy or a library kernel) the wait returns at once.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

namespace xt {
namespace dev {

// Blocks until the preceding grid on the stream has completed and flushed.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Allows the next grid on the stream to be scheduled.  It takes effect once
// every CTA of this grid has issued it or exited, i.e. once no CTA of this
// grid is still waiting for an SM.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Fetches [p, p + bytes) into L2 (16-byte aligned address, size a multiple of
// 16).  L2 is the point of coherence, so this may run before griddep_wait():
// a later load still sees every store the previous grid makes to those lines.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
               : "memory");
}

// Launch attributes: programmatic serialization, plus an optional cluster.
struct PdlLaunch {
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attrs[2];

  PdlLaunch(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster_x = 1) {
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
    if (cluster_x > 1) {
      attrs[1].id = cudaLaunchAttributeClusterDimension;
      attrs[1].val.clusterDim.x = static_cast<unsigned>(cluster_x);
      attrs[1].val.clusterDim.y = 1;
      attrs[1].val.clusterDim.z = 1;
      cfg.numAttrs = 2;
    }
    cfg.attrs = attrs;
  }

  template <class... KArgs, class... Args>
  cudaError_t operator()(void (*kernel)(KArgs...), Args&&... args) {
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  }
};

}  // namespace dev
}  // namespace xt
