"""The reference's own front-end artefacts, run unchanged against this package.

Needs a checkout of the reference (sjjeong94/xtile): the directory named by
``XTILE_REFERENCE``, else a ``reference`` directory beside this repository.
Skipped when neither exists (the GPU boxes have none).

* ``kernels/add.py``, ``softmax.py``, ``matmul.py`` and ``conv2d.py`` run
  as-is (their ``main()``, with this repository's ``xtile`` first on the path)
  and must write their eight stage files; the DSL text each writes
  (``0_xt.mlir``) must equal, byte for byte, what the reference's own tracer
  writes for the same script (the reference's DSL run in place behind a
  stand-in ``xtile`` module, as its ``test/python/matmul_cli.py`` stands one
  in);
* ``test/xt/*.mlir`` go through ``python -m xtile_b200.xt_opt`` with each
  file's ``RUN:`` flags, and the output is checked against the file's
  ``CHECK`` / ``ERR`` lines by the small FileCheck below.  ``to_nova.mlir``
  checks the NPU (nova) lowering, which this backend replaces with the B200
  plan: it must run, its CHECK lines are not applied.
"""
from __future__ import annotations

import contextlib
import importlib.util
import io
import os
import re
import runpy
import sys
import types
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _reference() -> Path | None:
    cand = os.environ.get("XTILE_REFERENCE")
    path = Path(cand) if cand else ROOT.parent / "reference"
    return path if (path / "xtile" / "dsl.py").exists() and (path / "kernels").is_dir() else None


REF = _reference()
pytestmark = pytest.mark.skipif(REF is None, reason="no checkout of the reference (set XTILE_REFERENCE)")


# --------------------------------------------------------------------------- FileCheck
def _pattern(text: str, env: dict) -> re.Pattern:
    """A FileCheck pattern as a regex: {{re}}, [[VAR:re]] defines, [[VAR]] uses;
    runs of horizontal whitespace match any run."""
    out, pos = [], 0
    token = re.compile(r"\{\{(.*?)\}\}|\[\[(\w+):(.*?)\]\]|\[\[(\w+)\]\]")
    for m in token.finditer(text):
        out.append(r"[ \t]+".join(re.escape(p) for p in re.split(r"[ \t]+", text[pos:m.start()])))
        if m.group(1) is not None:
            out.append(f"(?:{m.group(1)})")
        elif m.group(2) is not None:
            out.append(f"(?P<{m.group(2)}>{m.group(3)})")
        else:
            if m.group(4) not in env:
                raise AssertionError(f"FileCheck: undefined variable {m.group(4)}")
            out.append(re.escape(env[m.group(4)]))
        pos = m.end()
    out.append(r"[ \t]+".join(re.escape(p) for p in re.split(r"[ \t]+", text[pos:])))
    return re.compile("".join(out))


def filecheck(output: str, check_file: str, prefix: str = "CHECK") -> None:
    """Applies the PREFIX, PREFIX-LABEL and PREFIX-NOT lines of ``check_file``
    to ``output`` in order (each match within one line, as FileCheck does)."""
    lines = output.splitlines()
    directive = re.compile(rf"//\s*{prefix}(-LABEL|-NOT)?:\s?(.*)$")
    env: dict = {}
    line_no, col = 0, 0
    pending_not: list[tuple[str, int]] = []
    for ln in check_file.splitlines():
        m = directive.search(ln)
        if not m:
            continue
        kind, text = m.group(1) or "", m.group(2).rstrip()
        if kind == "-NOT":
            pending_not.append((text, line_no))
            continue
        pat = _pattern(text, env)
        found = None
        for i in range(line_no, len(lines)):
            hit = pat.search(lines[i], col if i == line_no else 0)
            if hit:
                found = (i, hit)
                break
        assert found, f"{prefix}{kind}: {text!r} not found after output line {line_no + 1}"
        i, hit = found
        for not_text, start in pending_not:  # nothing between the previous match and this one
            npat = _pattern(not_text, env)
            for j in range(start, i + 1):
                assert not npat.search(lines[j]), f"{prefix}-NOT: {not_text!r} found on output line {j + 1}"
        pending_not = []
        env.update({k: v for k, v in hit.groupdict().items() if v is not None})
        line_no, col = i, hit.end()
    for not_text, start in pending_not:
        npat = _pattern(not_text, env)
        for j in range(start, len(lines)):
            assert not npat.search(lines[j]), f"{prefix}-NOT: {not_text!r} found on output line {j + 1}"


def test_filecheck_itself():
    out = "a %1 = op(%0)\nb %2 = op(%1)\nc done\n"
    filecheck(out, "// CHECK: %[[X:.*]] = op(%0)\n// CHECK-NOT: done\n// CHECK: op(%[[X]])\n// CHECK: done")
    with pytest.raises(AssertionError):
        filecheck(out, "// CHECK: %[[X:.*]] = op(%0)\n// CHECK: op(%[[X]]5)")
    with pytest.raises(AssertionError):
        filecheck(out, "// CHECK-NOT: op(%1)\n// CHECK: done")


# --------------------------------------------------------------------------- lit inputs
def _run_xt_opt(flags: list[str], path: Path) -> tuple[int, str, str]:
    from xtile_b200 import xt_opt

    out, err = io.StringIO(), io.StringIO()
    with contextlib.redirect_stdout(out), contextlib.redirect_stderr(err):
        rc = xt_opt.main([*flags, str(path)])
    return rc, out.getvalue(), err.getvalue()


def _run_line(path: Path) -> str:
    return next(ln for ln in path.read_text().splitlines() if "RUN:" in ln)


@pytest.mark.parametrize("name", ["parse", "serialize", "canonicalize", "invalid", "serialize_invalid"])
def test_lit_file_through_xt_opt(name):
    path = REF / "test" / "xt" / f"{name}.mlir"
    run = _run_line(path)
    flags = [f for f in re.findall(r"--[\w-]+", run.split("|")[0])]
    expect_failure = re.search(r"RUN:\s*not\s", run) is not None
    prefix = re.search(r"--check-prefix=(\w+)", run)
    rc, out, err = _run_xt_opt(flags, path)
    if expect_failure:
        assert rc != 0
        filecheck(out + err, path.read_text(), prefix.group(1) if prefix else "CHECK")  # 2>&1
    else:
        assert rc == 0, err
        filecheck(out, path.read_text(), prefix.group(1) if prefix else "CHECK")


def test_to_nova_lit_file_runs():
    path = REF / "test" / "xt" / "to_nova.mlir"
    flags = re.findall(r"--[\w-]+", _run_line(path).split("|")[0])
    rc, out, err = _run_xt_opt(flags, path)
    assert rc == 0, err
    assert "// b200 @" in out  # the B200 plan stands where the nova lowering was


# --------------------------------------------------------------------------- kernels/*.py as-is
def _reference_xtile_stub():
    """A stand-in ``xtile`` built on the reference's own tracer: ``convert``
    returns the text, every stage returns its input, ``save_*`` write it."""
    spec = importlib.util.spec_from_file_location("xtile_reference_dsl_artefacts", REF / "xtile" / "dsl.py")
    dsl = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = dsl
    spec.loader.exec_module(dsl)
    stub = types.ModuleType("xtile")
    for k in dir(dsl):
        if not k.startswith("_"):
            setattr(stub, k, getattr(dsl, k))
    stub.cdiv = lambda a, b: (a + b - 1) // b
    stub.convert = lambda fn, *, args, grid, double_buffering=False: dsl.convert(
        fn, args=args, grid=grid, double_buffering=double_buffering, parse_module=lambda s: s)

    def save_ir(ir, path):
        with open(path, "wt") as f:
            f.write(str(ir))

    stub.save_ir = save_ir
    stages = ("xt_serialize", "xt_to_nova", "nova_optimize", "nova_threading", "nova_barrier",
              "nova_allocate", "nova_to_x1")
    for s in stages:
        setattr(stub, s, lambda ir: ir)

    def save_compile_results(ir, save_dir):
        os.makedirs(save_dir, exist_ok=True)
        save_ir(ir, os.path.join(save_dir, "0_xt.mlir"))
        for i, s in enumerate(stages, start=1):
            save_ir(ir, os.path.join(save_dir, f"{i}_{s}.mlir"))

    stub.save_compile_results = save_compile_results
    return stub


def _run_kernel_script(name: str, workdir: Path, xtile_module) -> Path:
    saved = sys.modules.get("xtile")
    sys.modules["xtile"] = xtile_module
    cwd = os.getcwd()
    os.chdir(workdir)
    try:
        g = runpy.run_path(str(REF / "kernels" / f"{name}.py"), run_name=f"reference_kernels_{name}")
        with contextlib.redirect_stdout(io.StringIO()):
            g["main"]([])
    finally:
        os.chdir(cwd)
        if saved is None:
            sys.modules.pop("xtile", None)
        else:
            sys.modules["xtile"] = saved
    dirs = [p for p in (workdir / "compiled" / name).iterdir() if p.is_dir()]
    assert len(dirs) == 1
    return dirs[0]


@pytest.mark.parametrize("name", ["add", "softmax", "matmul", "conv2d"])
def test_reference_kernel_script_runs_as_is(name, tmp_path):
    import xtile

    ours = _run_kernel_script(name, tmp_path / "ours", xtile) if (tmp_path / "ours").mkdir() is None else None
    theirs = _run_kernel_script(name, tmp_path / "ref", _reference_xtile_stub()) \
        if (tmp_path / "ref").mkdir() is None else None
    files = sorted(p.name for p in ours.iterdir())
    assert files == ["0_xt.mlir", "1_xt_serialize.mlir", "2_xt_to_nova.mlir", "3_nova_optimize.mlir",
                     "4_nova_threading.mlir", "5_nova_barrier.mlir", "6_nova_allocate.mlir", "7_nova_to_x1.mlir"]
    # the traced program is the reference tracer's, byte for byte
    assert (ours / "0_xt.mlir").read_text() == (theirs / "0_xt.mlir").read_text()
    # the serialize stage unrolled the grid; the later stages carry the B200 plan
    assert "xt.get_tile_block_id" not in (ours / "1_xt_serialize.mlir").read_text()
    assert "// b200 @" in (ours / "7_nova_to_x1.mlir").read_text()
    # and the Block program is one a B200 kernel family runs
    assert xtile.parse((ours / "0_xt.mlir").read_text()).plan()["family"] in ("ew", "rows", "gemm", "conv")
