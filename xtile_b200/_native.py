"""Loads the native extension ``_xtile`` (over ``libxt_b200.so``).

There is no pure-Python fallback: without the extension nothing can be parsed
or launched, and importing the package fails with the build command to run.
"""
from __future__ import annotations

import importlib

try:
    native = importlib.import_module("xtile_b200._xtile")
except ImportError as exc:  # pragma: no cover - exercised only on an unbuilt tree
    raise ImportError(
        "the xtile_b200 native extension is not built; run `python xtile_b200/build.py` "
        f"(or __graft_entry__.build()) first: {exc}") from exc
