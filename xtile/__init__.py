"""``import xtile as xt`` compatibility package: the reference's import name.

Everything comes from ``xtile_b200`` (the B200 backend); ``xtile.dsl`` and the
native module ``xtile._xtile`` resolve to the backend's tracer and extension,
the names the reference's package exposes (``xtile/__init__.py:45-71``).
"""
import sys as _sys

import xtile_b200 as _b200
from xtile_b200 import *  # noqa: F401,F403
from xtile_b200 import __all__ as _all
from xtile_b200 import _module_asm, _parse_module  # noqa: F401
from xtile_b200 import dsl  # noqa: F401
from xtile_b200._native import native as _native

_sys.modules.setdefault("xtile._xtile", _native)
_sys.modules.setdefault("xtile.dsl", dsl)
__all__ = list(_all)
__version__ = "0.1.0+b200"
del _b200
