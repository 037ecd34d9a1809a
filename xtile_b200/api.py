"""Compiler-facing API: modules, stages and stage dumps.

Mirrors the reference package facade (``xtile/__init__.py`` of
sjjeong94/xtile): ``parse`` wraps bare ``func.func`` text in a module and keeps
the DSL text for display (``:74-82,113-115``); every stage wrapper runs in
place, clears the display override and returns the *same* ``Module`` object
(``:104-157``); ``compile`` runs the seven stages in order (``:160-168``);
``save_compile_results`` writes the eight stage files (``:186-205``).

On this backend the stage names are kept so existing scripts run unchanged,
but only ``xt_serialize`` transforms the printed IR (grid unrolling, as the
reference does); the later stages annotate the B200 kernel plan (kernel
family, warp roles, mbarrier pipeline, shared memory / TMEM budget) instead of
emitting NPU commands.
"""
from __future__ import annotations

import os
from typing import Any

from . import dsl
from ._native import native as _native

_STAGES = ("xt_serialize", "xt_to_nova", "nova_optimize", "nova_threading", "nova_barrier",
           "nova_allocate", "nova_to_x1")


def cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def _wrap_module_asm(asm: str) -> tuple[str, str | None]:
    text = asm.strip()
    if text.startswith("module"):
        return text, None
    body = "\n".join(f"  {line}" if line else line for line in text.splitlines())
    return f"module {{\n{body}\n}}", text


class Module:
    """A parsed xt module; owns the native handle (a capsule)."""

    def __init__(self, raw_module: Any, display_asm: str | None = None, source_asm: str | None = None) -> None:
        self._raw_module = raw_module
        self._display_asm = display_asm
        self._source_asm = source_asm

    @property
    def _CAPIPtr(self):
        return self._raw_module

    def __str__(self) -> str:
        if self._display_asm is not None:
            return self._display_asm
        return _native._module_asm(self._raw_module)

    def _clear_display_override(self) -> None:
        self._display_asm = None

    # -- B200 additions -----------------------------------------------------
    @property
    def source_text(self) -> str:
        """The text this module was parsed from, unchanged (for a converted
        kernel: the DSL's own xt text).  Stages never alter it."""
        if self._source_asm is None:
            raise ValueError("module has no source text (it was not created by xtile.parse)")
        return self._source_asm

    def func_names(self) -> list[str]:
        return list(_native.func_names(self._raw_module))

    def plan(self, func: str | None = None) -> dict:
        """Kernel family and algorithmic work of ``func`` (default: first)."""
        return dict(_native.plan(self._raw_module, func))

    def arguments(self, func: str | None = None) -> list[tuple[str, bool, str, tuple]]:
        """``(name, is_memref, elem, shape)`` per argument, in launch order."""
        return [tuple(a) for a in _native.func_args(self._raw_module, func)]


def parse(asm: str) -> Module:
    wrapped, display = _wrap_module_asm(asm)
    return Module(_native.parse(wrapped), display_asm=display, source_asm=asm)


def _run_stage(name: str, module: Any):
    raw = module._CAPIPtr if isinstance(module, Module) else module
    result = getattr(_native, name)(raw)
    if isinstance(module, Module):
        module._clear_display_override()
        return module
    return result


def xt_serialize(module: Any):
    return _run_stage("xt_serialize", module)


def xt_to_nova(module: Any):
    return _run_stage("xt_to_nova", module)


def nova_optimize(module: Any):
    return _run_stage("nova_optimize", module)


def nova_threading(module: Any):
    return _run_stage("nova_threading", module)


def nova_barrier(module: Any):
    return _run_stage("nova_barrier", module)


def nova_allocate(module: Any):
    return _run_stage("nova_allocate", module)


def nova_to_x1(module: Any):
    return _run_stage("nova_to_x1", module)


def canonicalize(module: Any):
    """The xt dialect's canonicalization (``xt-opt --canonicalize`` of the
    reference): ``x + 0``, ``0 + x`` and ``x - 0`` fold to ``x``
    (``lib/xt/XTOps.cpp:395-449``) and unused side-effect-free ops are erased.
    In place; returns the same module."""
    return _run_stage("canonicalize", module)


def compile(module: Any):  # noqa: A001 - the reference's name
    for name in _STAGES:
        module = _run_stage(name, module)
    return module


def convert(kernel_fn, *, args, grid, double_buffering=False) -> Module:
    return dsl.convert(kernel_fn, args=args, grid=grid, double_buffering=double_buffering,
                       parse_module=parse)


def save_ir(ir: object, save_path: str) -> None:
    with open(save_path, "wt") as f:
        f.write(str(ir))


def save_compile_results(ir: object, save_dir: str) -> None:
    os.makedirs(save_dir, exist_ok=True)
    save_ir(ir, os.path.join(save_dir, "0_xt.mlir"))
    for i, name in enumerate(_STAGES, start=1):
        ir = _run_stage(name, ir)
        save_ir(ir, os.path.join(save_dir, f"{i}_{name}.mlir"))
    print("compiled kernel ->", save_dir)


def _module_asm(module: Any) -> str:
    raw = module._CAPIPtr if isinstance(module, Module) else module
    return _native._module_asm(raw)


def _parse_module(asm: str) -> Module:
    return parse(asm)
