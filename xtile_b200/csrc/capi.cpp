// C ABI of libxt_b200.so (include/xt_b200.h): module handles, stage dumps,
// planning and launching.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>

#include "../../include/xt_b200.h"
#include "codegen.h"
#include "ir.h"
#include "kernels.h"
#include "plan.h"

struct xt_module {
  std::unique_ptr<xt::Module> source;     // as parsed and verified
  std::unique_ptr<xt::Module> unrolled;   // after the xt_serialize stage
  int stage = 0;                          // stages run so far (0..7)
  mutable std::mutex mu;
  mutable std::map<std::string, std::shared_ptr<xt::Plan>> plans;
  mutable std::map<std::string, std::string> plan_errors;
};

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int fail(const xt::Error& e) {
  static const int kMap[] = {0, XT_EPARSE, XT_EVERIFY, XT_EPASS, XT_EUNSUPPORTED, XT_EARGUMENT, XT_ECUDA, XT_ETYPE};
  int code = (e.category >= 1 && e.category <= 7) ? kMap[e.category] : XT_EPASS;
  return fail(code, e.what());
}

const char* kPasses[] = {"xt_serialize", "xt_to_nova", "nova_optimize", "nova_threading",
                         "nova_barrier", "nova_allocate", "nova_to_x1"};

const xt::Func* find_func(const xt_module* m, const char* name) {
  if (m->source->funcs.empty()) return nullptr;
  if (!name) return &m->source->funcs[0];
  for (const xt::Func& f : m->source->funcs)
    if (f.name == name) return &f;
  return nullptr;
}

// Plans are computed once per function and cached on the module.
std::shared_ptr<xt::Plan> get_plan(const xt_module* m, const xt::Func& f) {
  std::lock_guard<std::mutex> lock(m->mu);
  auto it = m->plans.find(f.name);
  if (it != m->plans.end()) return it->second;
  auto e = m->plan_errors.find(f.name);
  if (e != m->plan_errors.end()) throw xt::Error(xt::kUnsupported, e->second);
  try {
    auto p = std::make_shared<xt::Plan>(xt::make_plan(*m->source, f));
    m->plans[f.name] = p;
    return p;
  } catch (const xt::Error& err) {
    m->plan_errors[f.name] = err.what();
    throw;
  }
}

// Per-device workspace: the error word the kernels' bounded waits write.
struct Workspace {
  uint32_t* error_word = nullptr;
};

std::mutex g_ws_mu;
std::map<int, Workspace> g_ws;

cudaError_t workspace(int device, Workspace** out) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  auto it = g_ws.find(device);
  if (it == g_ws.end()) {
    Workspace w;
    cudaError_t e = cudaMalloc(&w.error_word, 256);
    if (e != cudaSuccess) return e;
    e = cudaMemset(w.error_word, 0, 256);
    if (e != cudaSuccess) return e;
    it = g_ws.emplace(device, w).first;
  }
  *out = &it->second;
  return cudaSuccess;
}

uint8_t elem_code(xt::Elem e) {
  switch (e) {
    case xt::Elem::BF16: return xt::dev::kBF16;
    case xt::Elem::I8: return xt::dev::kI8;
    default: return xt::dev::kF32;
  }
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(XT_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int64_t clamp64(int64_t v, int64_t lo, int64_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

// SM budget of the persistent (gemm, conv) kernels launched by this thread.
thread_local int t_sm_budget = 0;

// Pipeline wait limit of the gemm and conv kernels launched by this thread,
// in nanoseconds (0: the kernels' default of about 2 s).  Kernels count SM
// cycles; at the B200's 1.9-2.0 GHz SM clock a nanosecond is 2 cycles.
thread_local uint64_t t_wait_limit_ns = 0;

uint64_t wait_limit_cycles() { return t_wait_limit_ns * 2; }

}  // namespace

namespace xt {

// Launch arguments of the GEMM of plan ``p`` for the Blocks with bid0 in
// [b0, b1) (a sub-range selects a contiguous slab of output rows), with the
// calling thread's SM budget and ``error_word`` as the kernel's error word.
// ``who`` prefixes error messages.  A range holding no rows gives out->M == 0.
int gemm_launch_args(const Plan& p, void* const* args, int64_t b0, int64_t b1, uint32_t* error_word,
                     const char* who, dev::GemmArgs* out) {
  const GemmPlan& g = p.gemm;
  dev::GemmArgs a{};
  a.A = args[g.a_arg];
  a.B = args[g.b_arg];
  a.C = args[g.c_arg];
  a.acc = g.acc_arg >= 0 ? static_cast<const float*>(args[g.acc_arg]) : nullptr;
  a.N = g.N;
  a.K = g.K;
  a.lda = g.lda;
  a.ldb = g.ldb;
  a.ldc = g.ldc;
  a.ab_elem = elem_code(g.ab_elem);
  a.c_elem = elem_code(g.c_elem);
  a.n_epi = static_cast<int>(g.epi.size());
  if (a.n_epi > 4) return fail(XT_EUNSUPPORTED, std::string(who) + ": at most 4 epilogue steps are supported");
  for (int i = 0; i < a.n_epi; ++i) {
    a.epi_kind[i] = g.epi[i].kind;
    a.epi_ptr[i] = static_cast<const float*>(args[g.epi[i].arg]);
  }
  a.error_word = error_word;
  a.max_sms = t_sm_budget;
  a.wait_limit_cycles = wait_limit_cycles();
  if (b0 == 0 && b1 == p.grid[0]) {
    a.m_begin = 0;
    a.M = g.M;
  } else {
    if (g.m_axis != 0)
      return fail(XT_EARGUMENT, std::string(who) + ": output rows of @" + p.func + " are not indexed by xt.bid(0)");
    const int64_t r0 = clamp64(b0 * g.tm, 0, g.M), r1 = clamp64(b1 * g.tm, 0, g.M);
    a.m_begin = r0;
    a.M = r1 - r0;
  }
  *out = a;
  return XT_OK;
}

}  // namespace xt

namespace {

// Launch arguments of an ew / rows plan; ``args`` null leaves the pointers
// null (the generated source depends only on the rest).
xt::dev::EwArgs ew_args_of(const xt::EwPlan& e, void* const* args) {
  xt::dev::EwArgs a{};
  for (int i = 0; i < e.n_in; ++i) {
    a.in[i] = args ? args[e.in_arg[i]] : nullptr;
    a.in_elem[i] = elem_code(e.in_elem[i]);
    a.in_bcast[i] = e.in_bcast[i] ? 1 : 0;
  }
  a.bcast_period = e.bcast_period;
  for (int i = 0; i < e.n_out; ++i) {
    a.out[i] = args ? args[e.out_arg[i]] : nullptr;
    a.out_elem[i] = elem_code(e.out_elem[i]);
  }
  a.n_in = e.n_in;
  a.n_out = e.n_out;
  a.n_code = static_cast<int>(e.code.size());
  for (size_t i = 0; i < e.code.size(); ++i) a.code[i] = e.code[i];
  a.begin = 0;
  a.end = e.numel;
  return a;
}

xt::dev::RowArgs row_args_of(const xt::RowPlan& r, void* const* args) {
  xt::dev::RowArgs a{};
  for (int i = 0; i < r.n_in; ++i) {
    a.in[i] = args ? static_cast<const float*>(args[r.in_arg[i]]) : nullptr;
    a.in_scalar[i] = r.in_is_scalar[i];
  }
  for (int i = 0; i < r.n_out; ++i) {
    a.out[i] = args ? static_cast<float*>(args[r.out_arg[i]]) : nullptr;
    a.out_scalar[i] = r.out_is_scalar[i];
  }
  a.n_code = static_cast<int>(r.code.size());
  for (size_t i = 0; i < r.code.size(); ++i) a.code[i] = r.code[i];
  a.n_vregs = r.n_vregs;
  a.n_sregs = r.n_sregs;
  a.cols = r.cols;
  a.softmax = r.softmax;
  a.row_begin = 0;
  a.row_end = r.rows;
  return a;
}

// Launch arguments of a tile plan (every Block of the grid); ``args`` null
// leaves the pointers null.
xt::dev::TileArgs tile_args_of(const xt::Plan& p, void* const* args) {
  const xt::TilePlan& t = p.tile;
  xt::dev::TileArgs a{};
  for (int i = 0; i < t.n_args; ++i) {
    a.arr[i] = args ? args[t.arg[i]] : nullptr;
    a.elem[i] = elem_code(t.arg_elem[i]);
    for (int d = 0; d < xt::kTileRank; ++d) a.shape[i][d] = t.arg_shape[i][d];
  }
  for (size_t i = 0; i < t.vals.size(); ++i) a.vals[i] = t.vals[i];
  for (size_t i = 0; i < t.ops.size(); ++i) a.ops[i] = t.ops[i];
  a.n_ops = static_cast<int>(t.ops.size());
  a.smem_floats = t.smem_floats;
  for (int k = 0; k < 3; ++k) a.grid[k] = p.grid[k];
  a.bid0_begin = 0;
  a.bid0_end = p.grid[0];
  return a;
}

int launch_plan(const xt::Plan& p, void* const* args, int64_t b0, int64_t b1, cudaStream_t stream) {
  using namespace xt;
  const int64_t g0 = p.grid[0];
  const bool full = b0 == 0 && b1 == g0;
  int device = 0;
  cudaGetDevice(&device);
  switch (p.family) {
    case Family::Ew: {
      const EwPlan& e = p.ew;
      dev::EwArgs a = ew_args_of(e, args);
      if (full) {
        a.begin = 0;
        a.end = e.numel;
      } else {
        if (e.bid0_span == 0)
          return fail(XT_EARGUMENT, "xt_launch: xt.bid(0) of @" + p.func +
                                        " does not select contiguous rows, so the grid cannot be split along it");
        a.begin = clamp64(b0 * e.bid0_span, 0, e.numel);
        a.end = clamp64(b1 * e.bid0_span, 0, e.numel);
      }
      cudaError_t err = dev::launch_ew(a, stream);
      return err == cudaSuccess ? XT_OK : cuda_fail(err, "ew kernel launch");
    }
    case Family::Rows: {
      const RowPlan& r = p.rows;
      dev::RowArgs a = row_args_of(r, args);
      if (full) {
        a.row_begin = 0;
        a.row_end = r.rows;
      } else {
        if (r.row_axis != 0)
          return fail(XT_EARGUMENT, "xt_launch: rows of @" + p.func + " are not indexed by xt.bid(0)");
        a.row_begin = clamp64(b0 * r.tile_rows, 0, r.rows);
        a.row_end = clamp64(b1 * r.tile_rows, 0, r.rows);
      }
      cudaError_t err = dev::launch_rows(a, stream);
      return err == cudaSuccess ? XT_OK : cuda_fail(err, "rows kernel launch");
    }
    case Family::Gemm: {
      Workspace* ws = nullptr;
      cudaError_t err = workspace(device, &ws);
      if (err != cudaSuccess) return cuda_fail(err, "workspace allocation");
      dev::GemmArgs a{};
      int st = xt::gemm_launch_args(p, args, b0, b1, ws->error_word, "xt_launch", &a);
      if (st != XT_OK) return st;
      if (a.M <= 0) return XT_OK;
      err = dev::launch_gemm(a, stream);
      return err == cudaSuccess ? XT_OK : cuda_fail(err, "gemm kernel launch");
    }
    case Family::Conv: {
      const ConvPlan& c = p.conv;
      Workspace* ws = nullptr;
      cudaError_t err = workspace(device, &ws);
      if (err != cudaSuccess) return cuda_fail(err, "workspace allocation");
      dev::ConvArgs a{};
      a.in = args[c.in_arg];
      a.filt = args[c.filt_arg];
      a.out = static_cast<float*>(args[c.out_arg]);
      a.N = c.N;
      a.H = c.H;
      a.W = c.W;
      a.C = c.C;
      a.KH = c.KH;
      a.KW = c.KW;
      a.KO = c.KO;
      a.OH = c.OH;
      a.OW = c.OW;
      a.out_h = c.out_h;
      a.out_w = c.out_w;
      a.out_c = c.out_c;
      a.pad_t = c.pad_t;
      a.pad_l = c.pad_l;
      a.dil_h = c.dil_h;
      a.dil_w = c.dil_w;
      a.elem = elem_code(c.elem);
      a.error_word = ws->error_word;
      a.max_sms = t_sm_budget;
      a.wait_limit_cycles = wait_limit_cycles();
      if (full) {
        a.n_begin = 0;
        a.ON = c.ON;
      } else {
        if (c.n_axis != 0)
          return fail(XT_EARGUMENT, "xt_launch: images of @" + p.func + " are not indexed by xt.bid(0)");
        int64_t n0 = clamp64(b0 * c.tb, 0, c.ON), n1 = clamp64(b1 * c.tb, 0, c.ON);
        a.n_begin = n0;
        a.ON = n1 - n0;
      }
      if (a.ON <= 0) return XT_OK;
      err = dev::launch_conv(a, stream);
      return err == cudaSuccess ? XT_OK : cuda_fail(err, "conv kernel launch");
    }
    case Family::Tile: {
      dev::TileArgs a = tile_args_of(p, args);
      a.bid0_begin = clamp64(b0, 0, g0);
      a.bid0_end = clamp64(b1, 0, g0);
      if (a.bid0_end <= a.bid0_begin) return XT_OK;
      cudaError_t err = dev::launch_tile(a, stream);
      return err == cudaSuccess ? XT_OK : cuda_fail(err, "tile kernel launch");
    }
  }
  return fail(XT_EUNSUPPORTED, "unknown kernel family");
}

}  // namespace

namespace xt {

// Plan of ``func`` (NULL: the first function) for launchers outside this
// file; throws Error on a missing function or an unsupported program.
std::shared_ptr<Plan> module_plan(const xt_module* module, const char* func) {
  const Func* f = find_func(module, func);
  if (!f) throw Error(kArgumentError, std::string("no function @") + (func ? func : "(first)"));
  return get_plan(module, *f);
}

// Records ``msg`` as the calling thread's last error and returns ``code``.
int record_error(int code, const std::string& msg) { return fail(code, msg); }

}  // namespace xt

extern "C" {

const char* xt_last_error(void) { return g_last_error.c_str(); }

int xt_parse(const char* text, xt_module** out) {
  if (!text || !out) return fail(XT_EARGUMENT, "xt_parse: null argument");
  try {
    auto mod = xt::parse_module(text);
    xt::verify_module(*mod);
    auto* m = new xt_module();
    m->source = std::move(mod);
    *out = m;
    return XT_OK;
  } catch (const xt::Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail(XT_EPARSE, e.what());
  }
}

void xt_module_free(xt_module* module) { delete module; }

int xt_module_asm(const xt_module* module, char** out_text) {
  if (!module || !out_text) return fail(XT_EARGUMENT, "xt_module_asm: null argument");
  try {
    std::string text;
    if (module->stage == 1 && module->unrolled) {
      text = xt::print_module(*module->unrolled);
    } else {
      text = xt::print_module(*module->source);
    }
    if (module->stage >= 2) {
      std::string plans;
      for (const xt::Func& f : module->source->funcs) {
        try {
          plans += xt::describe_plan(*get_plan(module, f), module->stage);
        } catch (const xt::Error& e) {
          plans += "  // b200 @" + f.name + ": no kernel family: " + e.what() + "\n";
        }
      }
      text.insert(text.rfind('}'), plans);
    }
    char* buf = static_cast<char*>(std::malloc(text.size() + 1));
    if (!buf) return fail(XT_EARGUMENT, "xt_module_asm: out of host memory");
    std::memcpy(buf, text.c_str(), text.size() + 1);
    *out_text = buf;
    return XT_OK;
  } catch (const xt::Error& e) {
    return fail(e);
  }
}

void xt_string_free(char* text) { std::free(text); }

int xt_run_pass(xt_module* module, const char* pass) {
  if (!module || !pass) return fail(XT_EARGUMENT, "xt_run_pass: null argument");
  int index = -1;
  for (int i = 0; i < 7; ++i)
    if (std::strcmp(pass, kPasses[i]) == 0) index = i;
  if (index < 0) return fail(XT_EARGUMENT, std::string("xt_run_pass: unknown pass '") + pass + "'");
  try {
    if (index == 0) module->unrolled = xt::serialize_module(*module->source);
    module->stage = index + 1 > module->stage ? index + 1 : module->stage;
    return XT_OK;
  } catch (const xt::Error& e) {
    return fail(e);
  }
}

int xt_canonicalize(xt_module* module) {
  if (!module) return fail(XT_EARGUMENT, "xt_canonicalize: null argument");
  try {
    std::lock_guard<std::mutex> lock(module->mu);
    xt::canonicalize_module(*module->source);
    xt::verify_module(*module->source);
    module->plans.clear();  // plans describe the program as it was
    module->plan_errors.clear();
    if (module->unrolled) module->unrolled = xt::serialize_module(*module->source);
    return XT_OK;
  } catch (const xt::Error& e) {
    return fail(e);
  }
}

int xt_num_funcs(const xt_module* module, int* out_count) {
  if (!module || !out_count) return fail(XT_EARGUMENT, "xt_num_funcs: null argument");
  *out_count = static_cast<int>(module->source->funcs.size());
  return XT_OK;
}

int xt_func_name(const xt_module* module, int index, const char** out_name) {
  if (!module || !out_name) return fail(XT_EARGUMENT, "xt_func_name: null argument");
  if (index < 0 || index >= static_cast<int>(module->source->funcs.size()))
    return fail(XT_EARGUMENT, "xt_func_name: index out of range");
  *out_name = module->source->funcs[index].name.c_str();
  return XT_OK;
}

int xt_func_num_args(const xt_module* module, const char* func, int* out_count) {
  if (!module || !out_count) return fail(XT_EARGUMENT, "xt_func_num_args: null argument");
  const xt::Func* f = find_func(module, func);
  if (!f) return fail(XT_EARGUMENT, std::string("xt_func_num_args: no function @") + (func ? func : "(first)"));
  *out_count = static_cast<int>(f->args.size());
  return XT_OK;
}

int xt_func_arg(const xt_module* module, const char* func, int index, xt_arg_info* out) {
  if (!module || !out) return fail(XT_EARGUMENT, "xt_func_arg: null argument");
  const xt::Func* f = find_func(module, func);
  if (!f) return fail(XT_EARGUMENT, std::string("xt_func_arg: no function @") + (func ? func : "(first)"));
  if (index < 0 || index >= static_cast<int>(f->args.size()))
    return fail(XT_EARGUMENT, "xt_func_arg: index out of range");
  const xt::Value& v = module->source->value(f->args[index]);
  std::memset(out, 0, sizeof(*out));
  out->name = v.name.c_str();
  out->is_memref = v.type.kind == xt::Type::MemRef;
  out->elem = v.type.elem == xt::Elem::F32 ? XT_ELEM_F32
              : v.type.elem == xt::Elem::BF16 ? XT_ELEM_BF16
              : v.type.elem == xt::Elem::I8 ? XT_ELEM_I8 : XT_ELEM_OTHER;
  out->rank = v.type.rank();
  if (out->rank > 8) return fail(XT_EUNSUPPORTED, "xt_func_arg: rank above 8");
  for (int i = 0; i < out->rank; ++i) out->shape[i] = v.type.shape[i];
  return XT_OK;
}

int xt_plan(const xt_module* module, const char* func, xt_plan_info* out) {
  if (!module || !out) return fail(XT_EARGUMENT, "xt_plan: null argument");
  const xt::Func* f = find_func(module, func);
  if (!f) return fail(XT_EARGUMENT, std::string("xt_plan: no function @") + (func ? func : "(first)"));
  try {
    auto p = get_plan(module, *f);
    std::memset(out, 0, sizeof(*out));
    out->family = static_cast<int>(p->family);
    out->n_args = static_cast<int>(p->arg_types.size());
    for (int i = 0; i < 3; ++i) out->grid[i] = p->grid[i];
    out->bid0_extent = p->grid[0];
    switch (p->family) {
      case xt::Family::Ew: {
        out->m = p->ew.numel;
        double bytes = 0, row_bytes = 0;
        for (int i = 0; i < p->ew.n_in; ++i)
          (p->ew.in_bcast[i] ? row_bytes : bytes) += xt::elem_bytes(p->ew.in_elem[i]);
        for (int i = 0; i < p->ew.n_out; ++i) bytes += xt::elem_bytes(p->ew.out_elem[i]);
        // a broadcast row is read once
        out->bytes = bytes * static_cast<double>(p->ew.numel) + row_bytes * static_cast<double>(p->ew.bcast_period);
        break;
      }
      case xt::Family::Rows: {
        out->m = p->rows.rows;
        out->n = p->rows.cols;
        double per_row = 0;
        for (int i = 0; i < p->rows.n_in; ++i) per_row += p->rows.in_is_scalar[i] ? 4 : 4.0 * p->rows.cols;
        for (int i = 0; i < p->rows.n_out; ++i) per_row += p->rows.out_is_scalar[i] ? 4 : 4.0 * p->rows.cols;
        out->bytes = per_row * static_cast<double>(p->rows.rows);
        break;
      }
      case xt::Family::Gemm: {
        const xt::GemmPlan& g = p->gemm;
        out->m = g.M;
        out->n = g.N;
        out->k = g.K;
        out->flops = 2.0 * g.M * g.N * g.K;
        const double ab = xt::elem_bytes(g.ab_elem);
        out->bytes = ab * (g.M * g.K + g.K * g.N) + xt::elem_bytes(g.c_elem) * double(g.M) * g.N;
        break;
      }
      case xt::Family::Conv: {
        const xt::ConvPlan& c = p->conv;
        out->m = c.ON * c.OH * c.OW;
        out->n = c.OC;
        out->k = c.KH * c.KW * c.C;
        out->flops = 2.0 * out->m * out->n * out->k;
        const double eb = xt::elem_bytes(c.elem);
        out->bytes = eb * (double(c.N) * c.H * c.W * c.C + double(c.KH) * c.KW * c.C * c.KO) + 4.0 * out->m * c.OC;
        break;
      }
      case xt::Family::Tile: {
        // every Block's loaded and stored tiles, as the program addresses them
        const xt::TilePlan& t = p->tile;
        double per_block = 0;
        for (const xt::TileOp& op : t.ops) {
          if (op.kind != xt::kTLoad && op.kind != xt::kTStore) continue;
          const xt::TileVal& v = t.vals[op.kind == xt::kTLoad ? op.dst : op.a];
          per_block += xt::elem_bytes(t.arg_elem[op.arg]) * static_cast<double>(v.numel);
        }
        out->bytes = per_block * static_cast<double>(p->grid[0] * p->grid[1] * p->grid[2]);
        break;
      }
    }
    return XT_OK;
  } catch (const xt::Error& e) {
    return fail(e);
  }
}

int xt_launch(const xt_module* module, const char* func, void* const* args, int n_args, int64_t bid0_begin,
              int64_t bid0_end, void* stream) {
  if (!module) return fail(XT_EARGUMENT, "xt_launch: null module");
  const xt::Func* f = find_func(module, func);
  if (!f) return fail(XT_EARGUMENT, std::string("xt_launch: no function @") + (func ? func : "(first)"));
  try {
    auto p = get_plan(module, *f);
    if (n_args != static_cast<int>(p->arg_types.size()))
      return fail(XT_EARGUMENT, "xt_launch: @" + p->func + " takes " + std::to_string(p->arg_types.size()) +
                                    " arrays, got " + std::to_string(n_args));
    for (int i = 0; i < n_args; ++i) {
      if (!args || !args[i]) return fail(XT_EARGUMENT, "xt_launch: array %" + p->arg_names[i] + " is null");
      if (reinterpret_cast<uintptr_t>(args[i]) & 15)
        return fail(XT_EARGUMENT, "xt_launch: array %" + p->arg_names[i] + " is not 16-byte aligned");
    }
    const int64_t g0 = p->grid[0];
    int64_t b0 = bid0_end <= 0 ? 0 : bid0_begin;
    int64_t b1 = bid0_end <= 0 ? g0 : bid0_end;
    if (b0 < 0 || b1 > g0 || b0 > b1)
      return fail(XT_EARGUMENT, "xt_launch: bid0 range [" + std::to_string(b0) + ", " + std::to_string(b1) +
                                    ") is outside the grid's [0, " + std::to_string(g0) + ")");
    if (b0 == b1) return XT_OK;
    return launch_plan(*p, args, b0, b1, static_cast<cudaStream_t>(stream));
  } catch (const xt::Error& e) {
    return fail(e);
  }
}

int xt_device_error(uint32_t* out_code) {
  if (!out_code) return fail(XT_EARGUMENT, "xt_device_error: null argument");
  int device = 0;
  cudaGetDevice(&device);
  Workspace* ws = nullptr;
  cudaError_t e = workspace(device, &ws);
  if (e != cudaSuccess) return cuda_fail(e, "workspace allocation");
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "device synchronize");
  uint32_t code = 0;
  e = cudaMemcpy(&code, ws->error_word, sizeof code, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "error word read");
  if (code) cudaMemset(ws->error_word, 0, sizeof code);
  *out_code = code;
  return XT_OK;
}

typedef CUresult (*MemGetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int xt_ipc_export(const void* ptr, unsigned char* handle64, uint64_t* offset) {
  if (!ptr || !handle64 || !offset) return fail(XT_EARGUMENT, "xt_ipc_export: null argument");
  static MemGetAddressRangeFn range = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<MemGetAddressRangeFn>(nullptr);
    return reinterpret_cast<MemGetAddressRangeFn>(f);
  }();
  if (!range) return fail(XT_ECUDA, "xt_ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(XT_EARGUMENT, "xt_ipc_export: pointer is not device memory");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(XT_ECUDA, std::string("xt_ipc_export: ") + cudaGetErrorString(e));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle64, &h, sizeof h);
  *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return XT_OK;
}

int xt_ipc_open(const unsigned char* handle64, void** base) {
  if (!handle64 || !base) return fail(XT_EARGUMENT, "xt_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof h);
  cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(XT_ECUDA, std::string("xt_ipc_open: ") + cudaGetErrorString(e));
  return XT_OK;
}

int xt_ipc_close(void* base) {
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return fail(XT_ECUDA, std::string("xt_ipc_close: ") + cudaGetErrorString(e));
  return XT_OK;
}

int xt_set_sm_budget(int sms) {
  if (sms < 0) return fail(XT_EARGUMENT, "xt_set_sm_budget: negative SM count");
  t_sm_budget = sms;
  return XT_OK;
}

int xt_generated_source(const xt_module* module, const char* func, char** out_text) {
  if (!module || !out_text) return fail(XT_EARGUMENT, "xt_generated_source: null argument");
  const xt::Func* f = find_func(module, func);
  if (!f) return fail(XT_EARGUMENT, std::string("xt_generated_source: no function @") + (func ? func : "(first)"));
  try {
    auto p = get_plan(module, *f);
    std::string text;
    if (p->family == xt::Family::Ew)
      text = xt::jit::ew_source(ew_args_of(p->ew, nullptr));
    else if (p->family == xt::Family::Rows && (!p->rows.softmax || p->rows.cols > 2048 || p->rows.cols % 4 != 0))
      text = xt::jit::rows_kernel_source(row_args_of(p->rows, nullptr));
    else if (p->family == xt::Family::Tile) {
      const xt::dev::TileArgs a = tile_args_of(*p, nullptr);
      text = xt::jit::tile_source(a, xt::jit::tile_threads(a));
    }
    else
      return fail(XT_EUNSUPPORTED, "xt_generated_source: @" + p->func + " runs a compiled kernel ('" +
                                       xt::family_name(p->family) + "' family)");
    char* buf = static_cast<char*>(std::malloc(text.size() + 1));
    if (!buf) return fail(XT_EARGUMENT, "xt_generated_source: out of host memory");
    std::memcpy(buf, text.c_str(), text.size() + 1);
    *out_text = buf;
    return XT_OK;
  } catch (const xt::Error& e) {
    return fail(e);
  }
}

int xt_compile_generated(const char* source, size_t* out_cubin_bytes) {
  if (!source || !out_cubin_bytes) return fail(XT_EARGUMENT, "xt_compile_generated: null argument");
  try {
    *out_cubin_bytes = xt::jit::compile(source).size();
    return XT_OK;
  } catch (const xt::Error& e) {
    return fail(e);
  }
}

int xt_set_wait_limit_ns(uint64_t ns) {
  if (ns > 60ull * 1000000000ull) return fail(XT_EARGUMENT, "xt_set_wait_limit_ns: more than 60 s");
  t_wait_limit_ns = ns;
  return XT_OK;
}

}  // extern "C"
