/* C ABI of the B200 xtile backend (libxt_b200.so).
 *
 * The reference exposes its compiler to Python through one nanobind module,
 * ``_xtile`` (python/XTModule.cpp:210-231): parse, seven pass thunks,
 * _parse_module and _module_asm, with MLIR modules owned by PyCapsules.  This
 * header is the same surface as plain C: an opaque module handle, the same
 * pass names, and -- new, since the reference cannot execute anything --
 * planning and launching a module's Block program on a B200.
 *
 * Conventions
 *  - Every call returns an int status: XT_OK (0) or one of the XT_E* codes.
 *    The message of the last failure on the calling thread is returned by
 *    xt_last_error() (replaces the exceptions raised at
 *    python/XTModule.cpp:119 (parse), :41,50 (type) and :135-148 (passes)).
 *  - Device buffers are borrowed: the caller allocates them (any allocator),
 *    keeps them alive until the launch's stream has finished, and owns the
 *    results, which are written in place (xt.store into a mutable Array).
 *  - Arrays are dense row-major with the exact shape and element type of the
 *    kernel's memref arguments; device pointers must be 16-byte aligned.
 *  - Launches are asynchronous on the given CUDA stream (NULL: legacy default
 *    stream) on the device current on the calling thread.  xt_launch may be
 *    called from several threads, one device per thread.
 */
#ifndef XT_B200_H
#define XT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct xt_module xt_module;

enum {
  XT_OK = 0,
  XT_EPARSE = 1,       /* text is not valid xt (reference: ValueError) */
  XT_EVERIFY = 2,      /* an op verifier failed (reference: parse fails) */
  XT_EPASS = 3,        /* a stage failed (reference: RuntimeError) */
  XT_EUNSUPPORTED = 4, /* no B200 kernel family implements the program */
  XT_EARGUMENT = 5,    /* bad argument to a call (count, null, range) */
  XT_ECUDA = 6,        /* a CUDA runtime / driver call failed */
  XT_ETYPE = 7,        /* wrong handle type (reference: TypeError) */
  XT_EDEVICE = 8       /* a kernel reported an error word (bounded wait ran out) */
};

/* Kernel families a Block program maps onto.  XT_FAMILY_TILE runs any other
 * Block program (reshape / transpose / permute, reductions along any axis,
 * broadcasting binaries, tensor constants) one CTA per Block in shared memory. */
enum { XT_FAMILY_EW = 1, XT_FAMILY_ROWS = 2, XT_FAMILY_GEMM = 3, XT_FAMILY_CONV = 4, XT_FAMILY_TILE = 5 };

typedef struct xt_plan_info {
  int family;           /* XT_FAMILY_* */
  int n_args;           /* memref arguments of the function, in signature order */
  int64_t grid[3];      /* xt.grid */
  int64_t bid0_extent;  /* grid[0]: the range xt_launch's bid0 bounds select from */
  int64_t m, n, k;      /* gemm/conv: covered GEMM extents; ew: elements; rows: rows, cols */
  double flops;         /* algorithmic FLOPs of one full launch (0 for ew/rows) */
  double bytes;         /* algorithmic bytes moved by one full launch */
} xt_plan_info;

/* Message of the last failed call on this thread ("" if none). */
const char* xt_last_error(void);

/* Parses and verifies xt text (a ``module { ... }`` or bare func.func ops).
 * Replaces parseModule, python/XTModule.cpp:112-126. */
int xt_parse(const char* text, xt_module** out);

/* Frees a module (the capsule destructor, python/XTModule.cpp:88-100). */
void xt_module_free(xt_module* module);

/* Prints the module at its current stage into a malloc'ed string the caller
 * frees with xt_string_free.  Replaces _module_asm, python/XTModule.cpp:228-230. */
int xt_module_asm(const xt_module* module, char** out_text);
void xt_string_free(char* text);

/* Runs one stage in place.  ``pass`` is one of the reference's names:
 * "xt_serialize", "xt_to_nova", "nova_optimize", "nova_threading",
 * "nova_barrier", "nova_allocate", "nova_to_x1" (python/XTModule.cpp:153-206,
 * pipeline order xtile/__init__.py:160-168).  xt_serialize unrolls the grid
 * for the dump (lib/xt/XTSerialize.cpp semantics); the later stages annotate
 * the B200 kernel plan.  Launching never depends on the stage. */
int xt_run_pass(xt_module* module, const char* pass);

/* Canonicalizes the module in place: xt.add(x, 0), xt.add(0, x) and
 * xt.sub(x, 0) with 0 a splat zero constant fold to x, and side-effect-free
 * ops left unused are erased.  Replaces MLIR's --canonicalize with the xt
 * dialect's patterns (lib/xt/XTOps.cpp:395-449), which the reference's
 * xt-opt runs (xt-opt/xt-opt.cpp:18-33; test/xt/canonicalize.mlir). */
int xt_canonicalize(xt_module* module);

/* Number of functions and the name of function ``index``. */
int xt_num_funcs(const xt_module* module, int* out_count);
int xt_func_name(const xt_module* module, int index, const char** out_name);

/* Element types of memref arguments. */
enum { XT_ELEM_F32 = 0, XT_ELEM_BF16 = 1, XT_ELEM_I8 = 2, XT_ELEM_OTHER = 3 };

typedef struct xt_arg_info {
  const char* name;     /* argument name without '%' (valid while the module lives) */
  int is_memref;        /* 0 for tensor / scalar arguments (not launchable) */
  int elem;             /* XT_ELEM_* */
  int rank;
  int64_t shape[8];
} xt_arg_info;

/* Arguments of ``func`` (NULL: the first function), in signature order: the
 * arrays xt_launch expects.  Mirrors the memref signature the DSL prints
 * (reference xtile/dsl.py:491-495). */
int xt_func_num_args(const xt_module* module, const char* func, int* out_count);
int xt_func_arg(const xt_module* module, const char* func, int index, xt_arg_info* out);

/* Maps function ``func`` (NULL: the first one) onto a kernel family. */
int xt_plan(const xt_module* module, const char* func, xt_plan_info* out);

/* Runs the Block program of ``func`` (NULL: the first) for the Blocks with
 * bid0 in [bid0_begin, bid0_end) -- all Blocks when bid0_end <= 0 -- on
 * ``stream``.  ``args`` holds one device pointer per memref argument in
 * signature order, ``n_args`` of them.  Used by one process per GPU to split
 * a Grid along bid0.  Allocates a small per-device workspace (error word,
 * scheduler counters) with cudaMalloc on the first launch on each device. */
int xt_launch(const xt_module* module, const char* func, void* const* args, int n_args,
              int64_t bid0_begin, int64_t bid0_end, void* stream);

/* Reads and clears the error word the kernels on the current device set when
 * a bounded wait runs out (0: none).  Synchronizes the device. */
int xt_device_error(uint32_t* out_code);

/* No counterpart in the reference.  Caps the SMs that the persistent kernels
 * (gemm and conv families) of later launches from the calling thread occupy;
 * 0 (the default) means all SMs.  A launch that runs beside a communication
 * kernel (an NCCL gather of the previous step's rows, say) leaves the other
 * SMs to it, so the two overlap instead of queueing behind each other.  The
 * GEMM rounds the budget down to an even number (its CTAs come in pairs). */
int xt_set_sm_budget(int sms);

/* No counterpart in the reference.  Elementwise, row and tile programs
 * (other than those the dedicated add, softmax and data-movement kernels
 * run) run in kernels generated for the program and compiled at their first
 * launch with NVRTC for sm_100a.
 * xt_generated_source gives that CUDA source for ``func`` (NULL: the first)
 * in a malloc'ed string (free with xt_string_free); XT_EUNSUPPORTED for
 * programs that run a compiled kernel.  xt_compile_generated compiles such a
 * source as a launch would and reports the cubin's size; it needs NVRTC but
 * no GPU. */
int xt_generated_source(const xt_module* module, const char* func, char** out_text);
int xt_compile_generated(const char* source, size_t* out_cubin_bytes);

/* No counterpart in the reference.  Sets how long a pipeline wait (TMA data,
 * MMA completion, accumulator hand-off) of the gemm and conv kernels that the
 * calling thread launches later may take before the kernel gives up: it then
 * records a code in the error word (read with xt_device_error: 0x101-0x103
 * gemm, 0x201-0x203 conv), stops every role, lets issued copies and MMAs
 * land, frees its tensor memory and returns, leaving the context usable.
 * ``ns`` 0 restores the default (about 2 s); at most 60 s.  Every wait takes
 * at least a few tens of microseconds before it can give up, whatever the
 * limit.  Teardown drains keep their own limits.  Used to test the failure
 * path; production keeps the default. */
int xt_set_wait_limit_ns(uint64_t ns);

/* No counterpart in the reference.  CUDA IPC for row gathers without a
 * collective: xt_ipc_export gives the 64-byte handle of the device allocation
 * holding ``ptr`` and ptr's byte offset in it; xt_ipc_open maps such an
 * allocation of another process of the node into this one on the current
 * device (*base: the mapping's base address; accesses go over NVLink), and
 * xt_ipc_close unmaps it.  A process passes base + offset to xt_launch as an
 * output array, and its kernel's stores land in the exporting GPU's array. */
int xt_ipc_export(const void* ptr, unsigned char* handle64, uint64_t* offset);
int xt_ipc_open(const unsigned char* handle64, void** base);
int xt_ipc_close(void* base);

/* No counterpart in the reference.  Launches a matmul program (the gemm
 * family only; other families are rejected) exactly like xt_launch, but
 * without allocating device memory: for callers that cannot call cudaMalloc,
 * such as engines that reserve all device memory up front, plugin enqueue
 * paths that must not allocate, or latency-critical paths that cannot absorb
 * cudaMalloc's implicit synchronisation.  The GEMM's scratch (its 4-byte error
 * word) lives in a 256-byte static __device__ array that every GPU loading
 * this library holds until exit; a launch needing more scratch is rejected.
 * The launch arguments (bid0 range, SM budget of xt_set_sm_budget) are built
 * by the same code as xt_launch's.  The first call on a device resolves that
 * array's address (make it before any stream capture); the address is kept,
 * so the entry point must not be used on a device after cudaDeviceReset.  All
 * calls share the array: each call clears the error word on its stream first,
 * calls whose kernels overlap on the GPU race on it, and the word is not
 * reported back. */
int xt_matmul_launch_noalloc(const xt_module* module, const char* func, void* const* args, int n_args,
                             int64_t bid0_begin, int64_t bid0_end, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XT_B200_H */
