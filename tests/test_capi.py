"""The C ABI library loads and exports every function include/*.h declares,
and its host-only calls work through ctypes (no GPU needed)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "xtile_b200" / "libxt_b200.so"


def declared_functions():
    names = []
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[\w]+\s*\*?\s*(xt_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("xt_parse", "xt_module_free", "xt_module_asm", "xt_run_pass", "xt_plan",
                     "xt_launch", "xt_last_error"):
        assert required in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports(name):
    lib = ctypes.CDLL(str(LIB))
    assert hasattr(lib, name), f"{name} is declared in include/ but not exported"


def test_parse_and_print_through_c_abi():
    lib = ctypes.CDLL(str(LIB))
    lib.xt_last_error.restype = ctypes.c_char_p
    mod = ctypes.c_void_p()
    text = b"""func.func @k(%a: memref<64x64xf32>, %b: memref<64x64xf32>) attributes {xt.grid = array<i32: 2, 1, 1>} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %x = xt.load(%a, %bid#0, %zero) : (memref<64x64xf32>, i32, i32) -> tensor<32x64xf32>
  %e = xt.exp(%x) : tensor<32x64xf32> -> tensor<32x64xf32>
  xt.store(%e, %b, %bid#0, %zero) : (tensor<32x64xf32>, memref<64x64xf32>, i32, i32) -> ()
  func.return
}"""
    assert lib.xt_parse(text, ctypes.byref(mod)) == 0
    out = ctypes.c_char_p()
    assert lib.xt_run_pass(mod, b"xt_to_nova") == 0
    assert lib.xt_module_asm(mod, ctypes.byref(out)) == 0
    asm = out.value.decode()
    lib.xt_string_free(out)
    assert "family ew" in asm
    assert lib.xt_run_pass(mod, b"no_such_pass") == 5          # XT_EARGUMENT
    assert b"unknown pass" in lib.xt_last_error()
    lib.xt_module_free(mod)
    bad = ctypes.c_void_p()
    assert lib.xt_parse(b"func.func @k() {\n xt.nope() : () -> ()\n}", ctypes.byref(bad)) == 1
    assert b"custom op 'xt.nope' is unknown" in lib.xt_last_error()


def test_host_side_argument_checks_of_new_entry_points():
    lib = ctypes.CDLL(str(LIB))
    lib.xt_last_error.restype = ctypes.c_char_p
    assert lib.xt_set_sm_budget(-1) == 5                       # XT_EARGUMENT
    assert b"negative" in lib.xt_last_error()
    assert lib.xt_set_sm_budget(0) == 0
    handle = (ctypes.c_ubyte * 64)()
    offset = ctypes.c_uint64()
    assert lib.xt_ipc_export(None, handle, ctypes.byref(offset)) == 5
    base = ctypes.c_void_p()
    assert lib.xt_ipc_open(None, ctypes.byref(base)) == 5
