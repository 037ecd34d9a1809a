// xt_matmul_launch_noalloc: launching a matmul program without allocating
// device memory.
//
// xt_launch gives the tensor-core GEMM a small workspace (the error word its
// bounded waits write) that it allocates with cudaMalloc on the first launch
// on each device.  Some callers cannot allow that: engines that reserve all
// device memory up front and hand out pieces from their own pool (a serving
// process that has claimed most of HBM at start-up), plugin interfaces whose
// enqueue step must not allocate, and latency-critical paths that cannot pay
// for the implicit device synchronisation of cudaMalloc.  For them this entry
// point keeps the GEMM's scratch in a file-scope __device__ array instead.
//
// Limits and rules:
//  * the scratch array holds kScratchBytes (256) bytes; the GEMM uses one
//    32-bit error word of it, and a launch needing more is rejected;
//  * every GPU that loads libxt_b200.so holds the array until the process
//    exits;
//  * the first call on a device resolves the array's device address with
//    cudaGetSymbolAddress (with that device current); make that first call
//    before any stream capture.  The address is kept for the process's
//    lifetime: after cudaDeviceReset on a device it is stale, so do not call
//    this entry point on a device that has been reset;
//  * all calls share the array and it keeps the last call's contents: each
//    call clears the error word on its stream before the kernel runs, and
//    calls whose kernels overlap on the GPU race on that word;
//  * the error word is not reported back (use xt_launch + xt_device_error
//    when a bounded-wait timeout must be observed).
#include <cuda_runtime.h>

#include <memory>
#include <mutex>
#include <string>

#include "../../include/xt_b200.h"
#include "kernels.h"
#include "plan.h"

namespace xt {
std::shared_ptr<Plan> module_plan(const xt_module* module, const char* func);
int record_error(int code, const std::string& msg);
}  // namespace xt

namespace {

constexpr size_t kScratchBytes = 256;
constexpr size_t kGemmScratchBytes = sizeof(uint32_t);  // the error word
static_assert(kGemmScratchBytes <= kScratchBytes, "the GEMM's scratch must fit the static array");
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint32_t g_scratch[kScratchBytes / sizeof(uint32_t)];

std::mutex g_mu;
uint32_t* g_scratch_addr[kMaxDevices] = {};

// Device address of g_scratch on the current device, resolved once per
// device.  The symbol name is a host-side stand-in; only this address may be
// handed to a kernel.
int scratch_address(int device, uint32_t** out) {
  if (device < 0 || device >= kMaxDevices)
    return xt::record_error(XT_EARGUMENT, "xt_matmul_launch_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess)
      return xt::record_error(XT_ECUDA, std::string("xt_matmul_launch_noalloc: cudaGetSymbolAddress: ") +
                                            cudaGetErrorString(e));
    g_scratch_addr[device] = static_cast<uint32_t*>(p);
  }
  *out = g_scratch_addr[device];
  return XT_OK;
}

}  // namespace

extern "C" int xt_matmul_launch_noalloc(const xt_module* module, const char* func, void* const* args,
                                        int n_args, int64_t bid0_begin, int64_t bid0_end, void* stream) {
  using namespace xt;
  if (!module) return record_error(XT_EARGUMENT, "xt_matmul_launch_noalloc: null module");
  std::shared_ptr<Plan> p;
  try {
    p = module_plan(module, func);
  } catch (const Error& e) {
    return record_error(e.category == kArgumentError ? XT_EARGUMENT : XT_EUNSUPPORTED,
                        std::string("xt_matmul_launch_noalloc: ") + e.what());
  }
  if (p->family != Family::Gemm)
    return record_error(XT_EUNSUPPORTED, "xt_matmul_launch_noalloc: @" + p->func + " maps onto the '" +
                                             family_name(p->family) + "' family; only matmul programs");
  if (n_args != static_cast<int>(p->arg_types.size()))
    return record_error(XT_EARGUMENT, "xt_matmul_launch_noalloc: @" + p->func + " takes " +
                                          std::to_string(p->arg_types.size()) + " arrays, got " +
                                          std::to_string(n_args));
  for (int i = 0; i < n_args; ++i) {
    if (!args || !args[i])
      return record_error(XT_EARGUMENT, "xt_matmul_launch_noalloc: array %" + p->arg_names[i] + " is null");
    if (reinterpret_cast<uintptr_t>(args[i]) & 15)
      return record_error(XT_EARGUMENT,
                          "xt_matmul_launch_noalloc: array %" + p->arg_names[i] + " is not 16-byte aligned");
  }
  const int64_t g0 = p->grid[0];
  const int64_t b0 = bid0_end <= 0 ? 0 : bid0_begin;
  const int64_t b1 = bid0_end <= 0 ? g0 : bid0_end;
  if (b0 < 0 || b1 > g0 || b0 > b1)
    return record_error(XT_EARGUMENT, "xt_matmul_launch_noalloc: bid0 range [" + std::to_string(b0) + ", " +
                                          std::to_string(b1) + ") is outside the grid's [0, " +
                                          std::to_string(g0) + ")");
  if (b0 == b1) return XT_OK;

  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess)
    return record_error(XT_ECUDA, std::string("xt_matmul_launch_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
  uint32_t* scratch = nullptr;
  int st = scratch_address(device, &scratch);
  if (st != XT_OK) return st;
  // the same arguments xt_launch builds (SM budget included); only the error
  // word's home differs
  dev::GemmArgs a{};
  st = gemm_launch_args(*p, args, b0, b1, scratch, "xt_matmul_launch_noalloc", &a);
  if (st != XT_OK) return st;
  if (a.M <= 0) return XT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(scratch, 0, kGemmScratchBytes, s);
  if (e != cudaSuccess)
    return record_error(XT_ECUDA, std::string("xt_matmul_launch_noalloc: clearing scratch: ") + cudaGetErrorString(e));
  e = dev::launch_gemm(a, s);
  if (e != cudaSuccess)
    return record_error(XT_ECUDA, std::string("xt_matmul_launch_noalloc: gemm kernel launch: ") + cudaGetErrorString(e));
  return XT_OK;
}
