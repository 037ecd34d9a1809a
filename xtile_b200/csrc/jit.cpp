// Run-time compilation and launch of the generated ew / rows / tile kernels
// (codegen.h): NVRTC, loaded with dlopen from the CUDA toolkit, compiles a
// program's source to an sm_100a cubin; the driver API (resolved through the
// runtime's entry-point query, so the library needs no link against
// libcuda) loads it once per device and launches it with programmatic
// dependent launch, like every other kernel of this library.
//
// A missing NVRTC is an error at the first launch of a generated program
// (with the reason); there is no fallback.
#include <cuda.h>
#include <dlfcn.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "codegen.h"
#include "ir.h"

namespace xt {
namespace jit {
namespace {

// ------------------------------------------------------------------ NVRTC
typedef int (*CreateFn)(void**, const char*, const char*, int, const char* const*, const char* const*);
typedef int (*CompileFn)(void*, int, const char* const*);
typedef int (*SizeFn)(void*, size_t*);
typedef int (*GetFn)(void*, char*);
typedef int (*DestroyFn)(void**);
typedef const char* (*ErrStrFn)(int);
typedef int (*VersionFn)(int*, int*);

struct Nvrtc {
  CreateFn create = nullptr;
  CompileFn compile = nullptr;
  SizeFn cubin_size = nullptr, log_size = nullptr;
  GetFn cubin = nullptr, log = nullptr;
  DestroyFn destroy = nullptr;
  ErrStrFn err = nullptr;
  VersionFn version = nullptr;
  std::string why;  // empty when loaded
};

const Nvrtc& nvrtc() {
  static Nvrtc n = [] {
    Nvrtc r;
    std::vector<std::string> names;
    if (const char* home = std::getenv("CUDA_HOME")) names.push_back(std::string(home) + "/lib64/libnvrtc.so.12");
    names.push_back("/usr/local/cuda/lib64/libnvrtc.so.12");
    names.push_back("libnvrtc.so.12");
    names.push_back("libnvrtc.so");
    void* h = nullptr;
    for (const std::string& n : names)
      if ((h = dlopen(n.c_str(), RTLD_NOW | RTLD_LOCAL)) != nullptr) break;
    if (!h) {
      r.why = "NVRTC (libnvrtc.so.12) could not be loaded: set CUDA_HOME to the CUDA toolkit";
      return r;
    }
    r.create = reinterpret_cast<CreateFn>(dlsym(h, "nvrtcCreateProgram"));
    r.compile = reinterpret_cast<CompileFn>(dlsym(h, "nvrtcCompileProgram"));
    r.cubin_size = reinterpret_cast<SizeFn>(dlsym(h, "nvrtcGetCUBINSize"));
    r.cubin = reinterpret_cast<GetFn>(dlsym(h, "nvrtcGetCUBIN"));
    r.log_size = reinterpret_cast<SizeFn>(dlsym(h, "nvrtcGetProgramLogSize"));
    r.log = reinterpret_cast<GetFn>(dlsym(h, "nvrtcGetProgramLog"));
    r.destroy = reinterpret_cast<DestroyFn>(dlsym(h, "nvrtcDestroyProgram"));
    r.err = reinterpret_cast<ErrStrFn>(dlsym(h, "nvrtcGetErrorString"));
    r.version = reinterpret_cast<VersionFn>(dlsym(h, "nvrtcVersion"));
    if (!r.create || !r.compile || !r.cubin_size || !r.cubin || !r.log_size || !r.log || !r.destroy || !r.err)
      r.why = "NVRTC is missing an entry point";
    return r;
  }();
  return n;
}

// ------------------------------------------------------------------ driver
typedef CUresult (*ModuleLoadDataFn)(CUmodule*, const void*);
typedef CUresult (*ModuleGetFunctionFn)(CUfunction*, CUmodule, const char*);
typedef CUresult (*LaunchKernelExFn)(const CUlaunchConfig*, CUfunction, void**, void**);
typedef CUresult (*GetErrorStringFn)(CUresult, const char**);
typedef CUresult (*FuncSetAttributeFn)(CUfunction, CUfunction_attribute, int);

template <class F>
F driver_fn(const char* name) {
  void* f = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &f, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<F>(f);
}

struct Driver {
  ModuleLoadDataFn load = driver_fn<ModuleLoadDataFn>("cuModuleLoadData");
  ModuleGetFunctionFn get = driver_fn<ModuleGetFunctionFn>("cuModuleGetFunction");
  LaunchKernelExFn launch = driver_fn<LaunchKernelExFn>("cuLaunchKernelEx");
  GetErrorStringFn err = driver_fn<GetErrorStringFn>("cuGetErrorString");
  FuncSetAttributeFn set_attr = driver_fn<FuncSetAttributeFn>("cuFuncSetAttribute");
};

const Driver& driver() {
  static Driver d;
  return d;
}

std::string cu_error(CUresult r) {
  const char* s = nullptr;
  if (driver().err) driver().err(r, &s);
  return s ? s : ("CUresult " + std::to_string(static_cast<int>(r)));
}

// ------------------------------------------------------------------ disk cache
// Compiled cubins persist across processes in a directory: XT_JIT_CACHE_DIR,
// else $XDG_CACHE_HOME/xtile_b200, else ~/.cache/xtile_b200; XT_JIT_CACHE=0
// turns the cache off.  A file is named by two independent 64-bit hashes of
// the source, the NVRTC version and the compile options, and starts with the
// lengths of that key and of the cubin, which a read checks; it is written,
// checked, to a temporary name
// and renamed, so processes that compile the same program at once (ranks)
// each see a whole file.  Any failure to read or write the cache only means
// a compile.
std::string cache_dir() {
  static const std::string dir = [] {
    const char* off = std::getenv("XT_JIT_CACHE");
    if (off && std::strcmp(off, "0") == 0) return std::string();
    if (const char* d = std::getenv("XT_JIT_CACHE_DIR")) return std::string(d);
    if (const char* x = std::getenv("XDG_CACHE_HOME")) return std::string(x) + "/xtile_b200";
    if (const char* h = std::getenv("HOME")) return std::string(h) + "/.cache/xtile_b200";
    return std::string();
  }();
  return dir;
}

// FNV-1a over ``s`` from ``h``
uint64_t fnv1a(const std::string& s, uint64_t h) {
  for (unsigned char c : s) {
    h ^= c;
    h *= 1099511628211ull;
  }
  return h;
}

bool make_dirs(const std::string& dir) {
  for (size_t i = 1; i <= dir.size(); ++i)
    if (i == dir.size() || dir[i] == '/') {
      const std::string part = dir.substr(0, i);
      if (mkdir(part.c_str(), 0755) != 0 && errno != EEXIST) return false;
    }
  return true;
}

std::string cached_compile(const std::string& source);

// ------------------------------------------------------------------ cache
struct Program {
  std::string cubin;
  std::map<int, CUmodule> modules;                          // per device
  std::map<std::pair<int, std::string>, CUfunction> fns;    // (device, kernel name)
};

std::mutex g_mu;
std::unordered_map<std::string, std::unique_ptr<Program>> g_programs;

// The fixed part of a program's launch arguments: what its generated source
// depends on (the family, the register code, and ``extra``: element types,
// broadcast flags, row width).
std::string key_of(char family, const Instr* code, int n_code, const std::string& extra) {
  std::string k(1, family);
  k.append(reinterpret_cast<const char*>(code), sizeof(Instr) * static_cast<size_t>(n_code));
  k += extra;
  return k;
}

// Kernel ``name`` of the program (``key``; ``make`` writes its source) on
// the current device, compiled and loaded on first use.  ``smem``: the
// dynamic shared memory its launches use, opted into above 48 KiB when the
// function is loaded.
template <class Make>
CUfunction function(const std::string& key, Make make, const char* name, int smem = 0) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) throw Error(kCudaError, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_programs.find(key);
  if (it == g_programs.end()) {
    auto p = std::make_unique<Program>();
    p->cubin = cached_compile(make());
    it = g_programs.emplace(key, std::move(p)).first;
  }
  Program& p = *it->second;
  auto f = p.fns.find({dev, name});
  if (f != p.fns.end()) return f->second;
  const Driver& d = driver();
  if (!d.load || !d.get || !d.launch) throw Error(kCudaError, "the CUDA driver lacks cuModuleLoadData / cuLaunchKernelEx");
  // the device's primary context, current on this thread, receives the module
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) throw Error(kCudaError, std::string("context set-up: ") + cudaGetErrorString(e));
  auto m = p.modules.find(dev);
  if (m == p.modules.end()) {
    CUmodule mod = nullptr;
    CUresult r = d.load(&mod, p.cubin.data());
    if (r != CUDA_SUCCESS) throw Error(kCudaError, "loading a generated kernel: " + cu_error(r));
    m = p.modules.emplace(dev, mod).first;
  }
  CUfunction fn = nullptr;
  CUresult r = d.get(&fn, m->second, name);
  if (r != CUDA_SUCCESS) throw Error(kCudaError, std::string("generated kernel ") + name + ": " + cu_error(r));
  if (smem > 48 * 1024) {
    if (!d.set_attr) throw Error(kCudaError, "the CUDA driver lacks cuFuncSetAttribute");
    r = d.set_attr(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, smem);
    if (r != CUDA_SUCCESS) throw Error(kCudaError, std::string("generated kernel ") + name + " shared memory: " + cu_error(r));
  }
  p.fns[{dev, name}] = fn;
  return fn;
}

cudaError_t launch(CUfunction fn, dim3 grid, unsigned block, cudaStream_t stream, void* params, unsigned smem = 0) {
  CUlaunchAttribute attr[1];
  attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr[0].value.programmaticStreamSerializationAllowed = 1;
  CUlaunchConfig cfg{};
  cfg.gridDimX = grid.x;
  cfg.gridDimY = grid.y;
  cfg.gridDimZ = grid.z;
  cfg.blockDimX = block;
  cfg.blockDimY = cfg.blockDimZ = 1;
  cfg.sharedMemBytes = smem;
  cfg.hStream = reinterpret_cast<CUstream>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {params};
  CUresult r = driver().launch(&cfg, fn, args, nullptr);
  if (r != CUDA_SUCCESS) throw Error(kCudaError, "launching a generated kernel: " + cu_error(r));
  return cudaSuccess;
}

unsigned grid_of(int64_t items, int per_block) {
  int64_t b = (items + per_block - 1) / per_block;
  if (b < 1) b = 1;
  if (b > 0x7fffffff) b = 0x7fffffff;
  return static_cast<unsigned>(b);
}

// kernel parameter blocks: the layout of XtEwArgs / XtRowArgs in the source
struct EwParams {
  const void* in[kMaxSlots];
  void* out[kMaxSlots];
  int64_t begin, end, period;
};
struct RowParams {
  const float* in[kMaxSlots];
  float* out[kMaxSlots];
  int64_t row_begin, row_end;
};
struct TileParams {
  void* arr[kTileMaxArgs];
  int64_t bid0_begin;
};

// Everything a tile program's source depends on, field by field (its ops,
// values, array element types and shapes, grid and CTA width).
std::string tile_key(const dev::TileArgs& a, int th) {
  std::string k(1, 't');
  auto put = [&](int64_t v) { k.append(reinterpret_cast<const char*>(&v), sizeof v); };
  put(th);
  put(a.n_ops);
  put(a.smem_floats);
  for (int i = 0; i < 3; ++i) put(a.grid[i]);
  for (int i = 0; i < kTileMaxArgs; ++i) {
    put(a.elem[i]);
    for (int d = 0; d < kTileRank; ++d) put(a.shape[i][d]);
  }
  for (int v = 0; v < kTileMaxVals; ++v) {
    const TileVal& t = a.vals[v];
    for (int d = 0; d < kTileRank; ++d) put((static_cast<int64_t>(t.shape[d]) << 32) | static_cast<uint32_t>(t.stride[d]));
    put((static_cast<int64_t>(t.offset) << 32) | static_cast<uint32_t>(t.numel));
    put(t.i8);
  }
  for (int o = 0; o < a.n_ops; ++o) {
    const TileOp& t = a.ops[o];
    const int64_t fields[7] = {t.kind, t.code, t.dst, t.a, t.b, t.arg, t.axis};
    int64_t packed = 0;
    for (int f = 0; f < 7; ++f) packed |= fields[f] << (8 * f);
    put(packed);
    for (int d = 0; d < kTileRank; ++d)
      put(static_cast<int64_t>(t.perm[d]) | (static_cast<int64_t>(t.coord_bid[d]) & 0xff) << 8 |
          static_cast<int64_t>(t.coord[d]) << 16);
    uint32_t bits;
    std::memcpy(&bits, &t.value, sizeof bits);
    put(bits);
  }
  return k;
}

}  // namespace

std::string compile(const std::string& source) {
  const Nvrtc& n = nvrtc();
  if (!n.why.empty()) throw Error(kCudaError, n.why);
  void* prog = nullptr;
  int st = n.create(&prog, source.c_str(), "xt_generated.cu", 0, nullptr, nullptr);
  if (st != 0) throw Error(kCudaError, std::string("nvrtcCreateProgram: ") + n.err(st));
  const char* opts[] = {"-arch=sm_100a", "-std=c++17", "-lineinfo"};
  st = n.compile(prog, 3, opts);
  std::string log;
  size_t log_n = 0;
  if (n.log_size(prog, &log_n) == 0 && log_n > 1) {
    log.resize(log_n);
    n.log(prog, &log[0]);
  }
  if (st != 0) {
    n.destroy(&prog);
    throw Error(kCudaError, std::string("NVRTC failed on a generated kernel: ") + n.err(st) + "\n" + log);
  }
  size_t size = 0;
  n.cubin_size(prog, &size);
  std::string cubin(size, '\0');
  n.cubin(prog, &cubin[0]);
  n.destroy(&prog);
  return cubin;
}

namespace {

std::string cached_compile(const std::string& source) {
  const std::string dir = cache_dir();
  if (dir.empty()) return compile(source);
  const Nvrtc& n = nvrtc();
  int major = 0, minor = 0;
  if (n.version) n.version(&major, &minor);
  const std::string key = source + "\n// nvrtc " + std::to_string(major) + "." + std::to_string(minor) +
                          " -arch=sm_100a -std=c++17 -lineinfo";
  char name[48];
  std::snprintf(name, sizeof name, "%016llx%016llx.cubin",
                static_cast<unsigned long long>(fnv1a(key, 14695981039346656037ull)),
                static_cast<unsigned long long>(fnv1a(key, 0x9e3779b97f4a7c15ull)));
  const std::string path = dir + "/" + name;
  {
    std::ifstream in(path, std::ios::binary);
    uint64_t len[2] = {0, 0};
    if (in && in.read(reinterpret_cast<char*>(len), sizeof len) && len[0] == key.size() && len[1] > 0) {
      std::string cubin((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
      if (cubin.size() == len[1]) return cubin;
    }
  }
  std::string cubin = compile(source);
  if (make_dirs(dir)) {
    const std::string tmp = path + ".tmp." + std::to_string(getpid());
    bool ok = false;
    {
      std::ofstream out(tmp, std::ios::binary | std::ios::trunc);
      const uint64_t len[2] = {key.size(), cubin.size()};
      out.write(reinterpret_cast<const char*>(len), sizeof len);
      out.write(cubin.data(), static_cast<std::streamsize>(cubin.size()));
      out.flush();
      ok = out.good();
    }
    if (!ok || std::rename(tmp.c_str(), path.c_str()) != 0) std::remove(tmp.c_str());
  }
  return cubin;
}

}  // namespace

cudaError_t launch_ew(const dev::EwArgs& a, cudaStream_t stream) {
  const int64_t n = a.end - a.begin;
  if (n <= 0) return cudaSuccess;
  std::string extra;
  for (int k = 0; k < kMaxSlots; ++k) {
    extra += static_cast<char>(k < a.n_in ? a.in_elem[k] : 255);
    extra += static_cast<char>(k < a.n_in ? a.in_bcast[k] : 0);
    extra += static_cast<char>(k < a.n_out ? a.out_elem[k] : 255);
  }
  const std::string key = key_of('e', a.code, a.n_code, extra);
  // the vector kernel: a range starting at a multiple of 4 elements, arrays
  // aligned to 4 elements of their type, broadcast rows a multiple of 4 long
  bool v4 = a.begin % 4 == 0 && a.bcast_period % 4 == 0;
  for (int k = 0; k < a.n_in && v4; ++k)
    v4 = reinterpret_cast<uintptr_t>(a.in[k]) % (a.in_elem[k] == dev::kF32 ? 16 : a.in_elem[k] == dev::kBF16 ? 8 : 4) == 0;
  for (int k = 0; k < a.n_out && v4; ++k)
    v4 = reinterpret_cast<uintptr_t>(a.out[k]) % (a.out_elem[k] == dev::kF32 ? 16 : a.out_elem[k] == dev::kBF16 ? 8 : 4) == 0;
  EwParams p{};
  for (int k = 0; k < kMaxSlots; ++k) {
    p.in[k] = a.in[k];
    p.out[k] = a.out[k];
  }
  p.begin = a.begin;
  p.end = a.end;
  p.period = a.bcast_period > 0 ? a.bcast_period : 1;
  if (v4) {
    const int64_t groups = n / (4 * kEwVec);
    CUfunction f = function(key, [&] { return ew_source(a); }, "xt_ew_v");
    return launch(f, dim3(grid_of(groups > 0 ? groups : 1, kEwThreads)), kEwThreads, stream, &p);
  }
  CUfunction f = function(key, [&] { return ew_source(a); }, "xt_ew_s");
  return launch(f, dim3(grid_of(n, kEwThreads)), kEwThreads, stream, &p);
}

cudaError_t launch_rows(const dev::RowArgs& a, cudaStream_t stream) {
  const int64_t rows = a.row_end - a.row_begin;
  if (rows <= 0) return cudaSuccess;
  std::string extra(reinterpret_cast<const char*>(&a.cols), sizeof a.cols);
  extra += static_cast<char>(a.n_vregs);
  for (int k = 0; k < kMaxSlots; ++k) {
    extra += static_cast<char>(a.in_scalar[k]);
    extra += static_cast<char>(a.out_scalar[k]);
  }
  const bool warp = rows_fit(a);
  const int tpr = warp ? 32 : row_cta_threads(a.cols, std::max(a.n_vregs, 1));
  if (!tpr) throw Error(kUnsupported, "the row program's live rows exceed a CTA's registers");
  const std::string key = key_of(warp ? 'r' : 'R', a.code, a.n_code, extra);
  bool vec = a.cols % 4 == 0;
  for (int k = 0; k < kMaxSlots && vec; ++k) {
    if (a.in[k] && !a.in_scalar[k]) vec = (reinterpret_cast<uintptr_t>(a.in[k]) & 15) == 0;
    if (vec && a.out[k] && !a.out_scalar[k]) vec = (reinterpret_cast<uintptr_t>(a.out[k]) & 15) == 0;
  }
  RowParams p{};
  for (int k = 0; k < kMaxSlots; ++k) {
    p.in[k] = a.in[k];
    p.out[k] = a.out[k];
  }
  p.row_begin = a.row_begin;
  p.row_end = a.row_end;
  if (!warp) {
    CUfunction f = function(key, [&] { return rows_cta_source(a, tpr); }, vec ? "xt_rows_cv" : "xt_rows_cs");
    return launch(f, dim3(grid_of(rows, 1)), tpr, stream, &p);
  }
  CUfunction f = function(key, [&] { return rows_source(a); }, vec ? "xt_rows_v" : "xt_rows_s");
  return launch(f, dim3(grid_of(rows, kRowsPerCta)), 32 * kRowsPerCta, stream, &p);
}

cudaError_t launch_tile(const dev::TileArgs& a, cudaStream_t stream) {
  const int64_t gx = a.bid0_end - a.bid0_begin;
  if (gx <= 0) return cudaSuccess;
  if (gx > 0x7fffffff || a.grid[1] > 65535 || a.grid[2] > 65535) return cudaErrorInvalidValue;
  const int th = tile_threads(a);
  const std::string key = tile_key(a, th);
  // the aligned kernel: every array 16-byte aligned
  bool aligned = true;
  for (int i = 0; i < kTileMaxArgs; ++i) aligned = aligned && (reinterpret_cast<uintptr_t>(a.arr[i]) & 15) == 0;
  TileParams p{};
  for (int i = 0; i < kTileMaxArgs; ++i) p.arr[i] = a.arr[i];
  p.bid0_begin = a.bid0_begin;
  const int smem = tile_smem_floats(a, th) * static_cast<int>(sizeof(float));
  CUfunction f = function(key, [&] { return tile_source(a, th); }, aligned ? "xt_tile_v" : "xt_tile_s", smem);
  return launch(f, dim3(static_cast<unsigned>(gx), static_cast<unsigned>(a.grid[1]), static_cast<unsigned>(a.grid[2])),
                th, stream, &p, static_cast<unsigned>(smem));
}

}  // namespace jit
}  // namespace xt
