"""xt_matmul_launch_noalloc through the C ABI (ctypes), against the CPU oracle
and against the ordinary entry point xt_launch.

The no-allocation entry point serves callers that cannot call cudaMalloc
(engines that own all device memory, plugin enqueue paths that must not
allocate, latency-critical paths that cannot absorb cudaMalloc's implicit
synchronisation).  It must compute what the ordinary entry point computes:
two calls in a row check that the shared static scratch is reset between
calls, a bid0 sub-range must write exactly its rows, and its very first call
on a device (the one that resolves the scratch array's address) is checked in
a fresh process.  Tolerance: the bf16 matmul bar of the other GPU tests
(max|gpu - ref| / max|ref| <= 1e-2).  This file is collected last.
"""
import ctypes
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import xtile_b200.dsl as dsl
from oracle import xt_oracle

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
M, N, K, TM, TN, TK = 384, 512, 256, 128, 128, 64


def _lib():
    lib = ctypes.CDLL(str(ROOT / "xtile_b200" / "libxt_b200.so"))
    launch_args = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
    lib.xt_parse.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
    lib.xt_launch.argtypes = launch_args
    lib.xt_matmul_launch_noalloc.argtypes = launch_args
    lib.xt_module_free.argtypes = [ctypes.c_void_p]
    lib.xt_set_sm_budget.argtypes = [ctypes.c_int]
    lib.xt_last_error.restype = ctypes.c_char_p
    return lib


@dsl.kernel
def matmul_kloop(lhs, rhs, out, tm, tn, tk, ksteps):
    i, j = dsl.bid(0), dsl.bid(1)
    acc = None
    for k in range(ksteps):
        p = dsl.matmul(dsl.load(lhs, index=(i, k), shape=(tm, tk)),
                       dsl.load(rhs, index=(k, j), shape=(tk, tn), shared=1))
        acc = p if acc is None else acc + p
    dsl.store(out, index=(i, j), tile=acc)


def _text():
    A = dsl.Array
    return dsl.trace_text(matmul_kloop, args=(A((M, K), dsl.bfloat16), A((K, N), dsl.bfloat16),
                                              A((M, N), dsl.float32), TM, TN, TK, K // TK),
                          grid=(M // TM, N // TN, 1), double_buffering=True)


def _inputs(seed):
    gen = torch.Generator().manual_seed(seed)
    a = (torch.randn(M, K, generator=gen) / 16).to(torch.bfloat16)
    b = (torch.randn(K, N, generator=gen) / 16).to(torch.bfloat16)
    return a, b


def _oracle(text, a, b):
    ref = np.zeros((M, N), np.float32)
    xt_oracle.run(text, [a.view(torch.uint16).numpy(), b.view(torch.uint16).numpy(), ref])
    return ref


def _close(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) <= 1e-2


def _noalloc(lib, mod, a, b, out, lo=0, hi=0):
    stream = ctypes.c_void_p(torch.cuda.current_stream(out.device).cuda_stream)
    ptrs = (ctypes.c_void_p * 3)(a.data_ptr(), b.data_ptr(), out.data_ptr())
    return lib.xt_matmul_launch_noalloc(mod, None, ptrs, 3, lo, hi, stream)


def test_noalloc_matches_oracle_and_launch_on_consecutive_calls():
    lib = _lib()
    text = _text()
    mod = ctypes.c_void_p()
    assert lib.xt_parse(text.encode(), ctypes.byref(mod)) == 0, lib.xt_last_error()
    dev = torch.device("cuda:0")
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    try:
        for seed in (11, 12):  # two calls in a row: the shared scratch is reset by each call
            a, b = _inputs(seed)
            ad, bd = a.to(dev), b.to(dev)
            out = torch.full((M, N), float("nan"), device=dev)
            assert _noalloc(lib, mod, ad, bd, out) == 0, lib.xt_last_error()
            ref_launch = torch.full((M, N), float("nan"), device=dev)
            ptrs = (ctypes.c_void_p * 3)(ad.data_ptr(), bd.data_ptr(), ref_launch.data_ptr())
            assert lib.xt_launch(mod, None, ptrs, 3, 0, 0, stream) == 0, lib.xt_last_error()
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            assert not np.isnan(got).any()
            _close(got, _oracle(text, a, b))
            _close(got, ref_launch.cpu().numpy())
    finally:
        lib.xt_module_free(mod)


def test_noalloc_bid0_subrange_writes_only_its_rows():
    lib = _lib()
    text = _text()
    mod = ctypes.c_void_p()
    assert lib.xt_parse(text.encode(), ctypes.byref(mod)) == 0, lib.xt_last_error()
    dev = torch.device("cuda:0")
    try:
        a, b = _inputs(13)
        out = torch.full((M, N), float("nan"), device=dev)
        assert _noalloc(lib, mod, a.to(dev), b.to(dev), out, 1, 2) == 0, lib.xt_last_error()  # Blocks bid0 = 1
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        _close(got[TM:2 * TM], _oracle(text, a, b)[TM:2 * TM])
        assert np.isnan(got[:TM]).all() and np.isnan(got[2 * TM:]).all()
        assert _noalloc(lib, mod, a.to(dev), b.to(dev), out, 2, 9) == 5   # XT_EARGUMENT: past the grid
        assert b"outside the grid" in lib.xt_last_error()
    finally:
        lib.xt_module_free(mod)


def test_noalloc_under_an_sm_budget():
    # the SM cap of xt_set_sm_budget applies to this entry point as to xt_launch
    lib = _lib()
    text = _text()
    mod = ctypes.c_void_p()
    assert lib.xt_parse(text.encode(), ctypes.byref(mod)) == 0, lib.xt_last_error()
    dev = torch.device("cuda:0")
    try:
        a, b = _inputs(14)
        out = torch.full((M, N), float("nan"), device=dev)
        assert lib.xt_set_sm_budget(16) == 0
        try:
            assert _noalloc(lib, mod, a.to(dev), b.to(dev), out) == 0, lib.xt_last_error()
        finally:
            lib.xt_set_sm_budget(0)
        torch.cuda.synchronize()
        _close(out.cpu().numpy(), _oracle(text, a, b))
    finally:
        lib.xt_module_free(mod)


FIRST_CALL = r"""
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from tests import test_zz_no_alloc as t
lib = t._lib()
text = t._text()
mod = ctypes.c_void_p()
assert lib.xt_parse(text.encode(), ctypes.byref(mod)) == 0
a, b = t._inputs(15)
out = torch.full((t.M, t.N), float("nan"), device="cuda:0")
# the first GEMM call of this process on the device: resolves the scratch address
assert t._noalloc(lib, mod, a.cuda(), b.cuda(), out) == 0, lib.xt_last_error()
torch.cuda.synchronize()
t._close(out.cpu().numpy(), t._oracle(text, a, b))
lib.xt_module_free(mod)
print("first call ok")
"""


def test_noalloc_first_call_in_a_fresh_process():
    res = subprocess.run([sys.executable, "-c", FIRST_CALL, str(ROOT)], cwd=ROOT, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    assert "first call ok" in res.stdout


def test_noalloc_rejects_other_families():
    lib = _lib()

    @dsl.kernel
    def add_rows(lhs, rhs, out, trow, col):
        i = dsl.bid(0)
        dsl.store(out, index=(i, 0), tile=dsl.load(lhs, index=(i, 0), shape=(trow, col))
                  + dsl.load(rhs, index=(i, 0), shape=(trow, col)))

    A = dsl.Array
    text = dsl.trace_text(add_rows, args=(A((64, 64), dsl.float32),) * 3 + (32, 64), grid=(2, 1, 1),
                          double_buffering=False)
    mod = ctypes.c_void_p()
    assert lib.xt_parse(text.encode(), ctypes.byref(mod)) == 0
    x = torch.zeros(64, 64, device="cuda:0")
    ptrs = (ctypes.c_void_p * 3)(x.data_ptr(), x.data_ptr(), x.data_ptr())
    try:
        assert lib.xt_matmul_launch_noalloc(mod, None, ptrs, 3, 0, 0, None) == 4   # XT_EUNSUPPORTED
        assert b"only matmul programs" in lib.xt_last_error()
    finally:
        lib.xt_module_free(mod)
