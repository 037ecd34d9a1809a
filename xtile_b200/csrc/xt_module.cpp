// The ``_xtile`` Python extension: the reference's native module surface
// (python/XTModule.cpp:210-231: parse, xt_to_nova, xt_serialize,
// nova_optimize, nova_allocate, nova_threading, nova_barrier, nova_to_x1,
// _parse_module, _module_asm) over the C ABI of libxt_b200.so, plus plan and
// launch.
//
// Modules travel as PyCapsules named "xtile.b200.module" whose destructor
// frees the handle (the reference's capsule owns its MLIRContext the same
// way, python/XTModule.cpp:82-110).  Objects carrying the capsule in a
// ``_CAPIPtr`` attribute are accepted too (python/XTModule.cpp:36-52).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/xt_b200.h"

namespace py = pybind11;

namespace {

constexpr const char* kCapsuleName = "xtile.b200.module";

[[noreturn]] void raise_status(int status, const char* context) {
  std::string msg = xt_last_error();
  switch (status) {
    case XT_EPARSE:
    case XT_EVERIFY:
      throw py::value_error(std::string("failed to parse test module\n") + msg);
    case XT_ETYPE:
      throw py::type_error(msg);
    case XT_EARGUMENT:
      throw py::value_error(msg);
    default:
      throw std::runtime_error(std::string(context) + ": " + msg);
  }
}

xt_module* unwrap(py::handle obj) {
  py::object cap = py::reinterpret_borrow<py::object>(obj);
  if (!PyCapsule_CheckExact(cap.ptr())) {
    if (!py::hasattr(obj, "_CAPIPtr")) throw py::type_error("expected an xtile module object");
    cap = obj.attr("_CAPIPtr");
  }
  if (!PyCapsule_IsValid(cap.ptr(), kCapsuleName)) throw py::type_error("expected an xtile module object");
  return static_cast<xt_module*>(PyCapsule_GetPointer(cap.ptr(), kCapsuleName));
}

py::object parse(const std::string& text) {
  xt_module* m = nullptr;
  int st = xt_parse(text.c_str(), &m);
  if (st != XT_OK) raise_status(st, "parse");
  PyObject* cap = PyCapsule_New(m, kCapsuleName, [](PyObject* c) {
    xt_module_free(static_cast<xt_module*>(PyCapsule_GetPointer(c, kCapsuleName)));
  });
  if (!cap) {
    xt_module_free(m);
    throw py::error_already_set();
  }
  return py::reinterpret_steal<py::object>(cap);
}

py::object run_pass(py::object module, const char* name) {
  int st = xt_run_pass(unwrap(module), name);
  if (st != XT_OK) raise_status(st, (std::string("xtile.") + name).c_str());
  return module;
}

std::string module_asm(py::object module) {
  char* text = nullptr;
  int st = xt_module_asm(unwrap(module), &text);
  if (st != XT_OK) raise_status(st, "_module_asm");
  std::string s(text);
  xt_string_free(text);
  return s;
}

py::dict plan(py::object module, py::object func) {
  std::string name;
  const char* fname = nullptr;
  if (!func.is_none()) {
    name = func.cast<std::string>();
    fname = name.c_str();
  }
  xt_plan_info info;
  int st = xt_plan(unwrap(module), fname, &info);
  if (st != XT_OK) raise_status(st, "plan");
  static const char* kFamilies[] = {"", "ew", "rows", "gemm", "conv", "tile"};
  py::dict d;
  d["family"] = kFamilies[info.family];
  d["n_args"] = info.n_args;
  d["grid"] = py::make_tuple(info.grid[0], info.grid[1], info.grid[2]);
  d["m"] = info.m;
  d["n"] = info.n;
  d["k"] = info.k;
  d["flops"] = info.flops;
  d["bytes"] = info.bytes;
  return d;
}

void launch(py::object module, const std::vector<uintptr_t>& ptrs, int64_t bid0_begin, int64_t bid0_end,
            uintptr_t stream, py::object func) {
  std::string name;
  const char* fname = nullptr;
  if (!func.is_none()) {
    name = func.cast<std::string>();
    fname = name.c_str();
  }
  std::vector<void*> args(ptrs.size());
  for (size_t i = 0; i < ptrs.size(); ++i) args[i] = reinterpret_cast<void*>(ptrs[i]);
  xt_module* m = unwrap(module);
  int st;
  {
    py::gil_scoped_release nogil;
    st = xt_launch(m, fname, args.data(), static_cast<int>(args.size()), bid0_begin, bid0_end,
                   reinterpret_cast<void*>(stream));
  }
  if (st != XT_OK) raise_status(st, "launch");
}

std::vector<std::string> func_names(py::object module) {
  xt_module* m = unwrap(module);
  int n = 0;
  xt_num_funcs(m, &n);
  std::vector<std::string> out;
  for (int i = 0; i < n; ++i) {
    const char* s = nullptr;
    xt_func_name(m, i, &s);
    out.emplace_back(s);
  }
  return out;
}

py::list func_args(py::object module, py::object func) {
  std::string name;
  const char* fname = nullptr;
  if (!func.is_none()) {
    name = func.cast<std::string>();
    fname = name.c_str();
  }
  xt_module* m = unwrap(module);
  int n = 0;
  int st = xt_func_num_args(m, fname, &n);
  if (st != XT_OK) raise_status(st, "func_args");
  static const char* kElems[] = {"f32", "bf16", "i8", "other"};
  py::list out;
  for (int i = 0; i < n; ++i) {
    xt_arg_info a;
    st = xt_func_arg(m, fname, i, &a);
    if (st != XT_OK) raise_status(st, "func_args");
    py::tuple shape(a.rank);
    for (int k = 0; k < a.rank; ++k) shape[k] = a.shape[k];
    out.append(py::make_tuple(a.name, bool(a.is_memref), kElems[a.elem], shape));
  }
  return out;
}

uint32_t device_error() {
  uint32_t code = 0;
  int st = xt_device_error(&code);
  if (st != XT_OK) raise_status(st, "device_error");
  return code;
}

}  // namespace

PYBIND11_MODULE(_xtile, m) {
  m.doc() = "B200 backend of the xtile tile DSL (C ABI: include/xt_b200.h)";
  m.def("parse", &parse, py::arg("asm"), "Parse and verify xt text into a module capsule.");
  m.def("_parse_module", &parse, py::arg("asm"));
  m.def("_module_asm", &module_asm, py::arg("module"));
  for (const char* name : {"xt_serialize", "xt_to_nova", "nova_optimize", "nova_threading", "nova_barrier",
                           "nova_allocate", "nova_to_x1"}) {
    std::string n(name);
    m.def(
        name, [n](py::object module) { return run_pass(module, n.c_str()); }, py::arg("module"),
        ("Run the " + n + " stage in place and return the module.").c_str());
  }
  m.def(
      "canonicalize",
      [](py::object module) {
        int st = xt_canonicalize(unwrap(module));
        if (st != XT_OK) raise_status(st, "xtile.canonicalize");
        return module;
      },
      py::arg("module"), "Fold x + 0 / x - 0 and erase unused side-effect-free ops, in place.");
  m.def("plan", &plan, py::arg("module"), py::arg("func") = py::none());
  m.def(
      "ipc_export",
      [](uintptr_t ptr) {
        unsigned char h[64];
        uint64_t off = 0;
        if (xt_ipc_export(reinterpret_cast<const void*>(ptr), h, &off) != XT_OK)
          throw std::runtime_error(xt_last_error());
        return py::make_tuple(py::bytes(reinterpret_cast<const char*>(h), 64), off);
      },
      py::arg("ptr"));
  m.def(
      "ipc_open",
      [](py::bytes handle) {
        std::string h = handle;
        if (h.size() != 64) throw std::invalid_argument("ipc_open: handle must be 64 bytes");
        void* base = nullptr;
        if (xt_ipc_open(reinterpret_cast<const unsigned char*>(h.data()), &base) != XT_OK)
          throw std::runtime_error(xt_last_error());
        return reinterpret_cast<uintptr_t>(base);
      },
      py::arg("handle"));
  m.def(
      "ipc_close",
      [](uintptr_t base) {
        if (xt_ipc_close(reinterpret_cast<void*>(base)) != XT_OK) throw std::runtime_error(xt_last_error());
      },
      py::arg("base"));
  m.def(
      "set_sm_budget",
      [](int sms) {
        if (xt_set_sm_budget(sms) != XT_OK) throw std::invalid_argument(xt_last_error());
      },
      py::arg("sms"));
  m.def(
      "generated_source",
      [](py::object module, py::object func) {
        std::string name;
        if (!func.is_none()) name = func.cast<std::string>();
        char* text = nullptr;
        int st = xt_generated_source(unwrap(module), func.is_none() ? nullptr : name.c_str(), &text);
        if (st != XT_OK) raise_status(st, "generated_source");
        std::string s(text);
        xt_string_free(text);
        return s;
      },
      py::arg("module"), py::arg("func") = py::none());
  m.def(
      "compile_generated",
      [](const std::string& source) {
        size_t n = 0;
        int st = xt_compile_generated(source.c_str(), &n);
        if (st != XT_OK) raise_status(st, "compile_generated");
        return n;
      },
      py::arg("source"));
  m.def(
      "set_wait_limit_ns",
      [](uint64_t ns) {
        if (xt_set_wait_limit_ns(ns) != XT_OK) throw std::invalid_argument(xt_last_error());
      },
      py::arg("ns"));
  m.def("launch", &launch, py::arg("module"), py::arg("ptrs"), py::arg("bid0_begin"), py::arg("bid0_end"),
        py::arg("stream"), py::arg("func") = py::none());
  m.def("func_names", &func_names, py::arg("module"));
  m.def("func_args", &func_args, py::arg("module"), py::arg("func") = py::none());
  m.def("device_error", &device_error);
}
