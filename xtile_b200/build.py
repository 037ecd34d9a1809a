"""Builds the native parts of xtile_b200 in-tree.

* ``libxt_b200.so``  -- the C ABI (include/xt_b200.h): parser, verifier,
  planner and the sm_100a kernels (nvcc, -gencode arch=compute_100a,code=sm_100a);
* ``_xtile*.so``     -- the Python extension (pybind11) over that library.

Objects go to ``xtile_b200/_build``; a source is recompiled when it or any
header it can include is newer than its object.

    python xtile_b200/build.py [--force]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB = PKG / "libxt_b200.so"


def ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


EXT = PKG / f"_xtile{ext_suffix()}"


def _headers() -> list[Path]:
    return list(CSRC.rglob("*.h")) + list(CSRC.rglob("*.cuh")) + list((ROOT / "include").glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def _compile(src: Path, force: bool, deps: list[Path]) -> Path:
    obj = BUILD / (src.relative_to(CSRC).as_posix().replace("/", "_") + ".o")
    if force or _stale(obj, src, deps):
        inc = [f"-I{CSRC}", f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}", f"-I{BUILD}"]
        if src.suffix == ".cu":
            cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                   "--expt-relaxed-constexpr", *inc, "-c", str(src), "-o", str(obj)]
        else:
            cmd = ["g++", "-O2", "-fPIC", "-std=c++17", "-Wall", "-Wno-unused-function", *inc,
                   "-c", str(src), "-o", str(obj)]
        _run(cmd)
    return obj


def _embed_op_math() -> None:
    """Writes op_math.cuh's text as a C++ string literal into the build
    directory: codegen.cpp puts it at the top of every generated kernel, so
    the generated kernels and the compiled ones share one definition of each
    element op.  Rewritten only when the text changes (keeps objects fresh)."""
    text = (CSRC / "kernels" / "op_math.cuh").read_text()
    if ")XTOPS\"" in text:
        raise RuntimeError("op_math.cuh may not contain the string literal's delimiter")
    inc = BUILD / "op_math_src.inc"
    body = 'R"XTOPS(' + text + ')XTOPS"\n'
    if not inc.exists() or inc.read_text() != body:
        inc.write_text(body)


def build(force: bool = False, verbose: bool = False) -> None:
    BUILD.mkdir(exist_ok=True)
    _embed_op_math()
    deps = _headers()
    lib_srcs = [p for p in sorted(CSRC.rglob("*.cpp")) if p.name != "xt_module.cpp"]
    lib_srcs += sorted(CSRC.rglob("*.cu"))
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        objs = list(pool.map(lambda s: _compile(s, force, deps), lib_srcs))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-ldl",
              "-lrt", "-lpthread"])
        if verbose:
            print("linked", LIB)

    # the Python extension
    import pybind11

    src = CSRC / "xt_module.cpp"
    obj = BUILD / "xt_module.o"
    if force or _stale(obj, src, deps):
        py_inc = sysconfig.get_paths()["include"]
        _run(["g++", "-O2", "-fPIC", "-std=c++17", f"-I{pybind11.get_include()}", f"-I{py_inc}",
              f"-I{CSRC}", f"-I{ROOT / 'include'}", "-c", str(src), "-o", str(obj)])
    if force or not EXT.exists() or obj.stat().st_mtime > EXT.stat().st_mtime \
            or LIB.stat().st_mtime > EXT.stat().st_mtime:
        _run(["g++", "-shared", "-o", str(EXT), str(obj), f"-L{PKG}", "-lxt_b200",
              "-Wl,-rpath,$ORIGIN"])
        if verbose:
            print("linked", EXT)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    build(force=args.force, verbose=True)


if __name__ == "__main__":
    main()
