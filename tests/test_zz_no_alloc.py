"""xt_matmul_launch_noalloc against xt_launch, through the C ABI (ctypes).

The no-allocation entry point serves callers that cannot call cudaMalloc
(engines that own all device memory, plugin enqueue paths that must not
allocate, latency-critical paths that cannot absorb cudaMalloc's implicit
synchronisation).  It must compute what the ordinary entry point computes;
two calls in a row check that the shared static scratch is reset between
calls.  Tolerance: the bf16 matmul bar of the other GPU tests (relative 1e-2).
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import xtile_b200.dsl as dsl

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _lib():
    lib = ctypes.CDLL(str(ROOT / "xtile_b200" / "libxt_b200.so"))
    launch_args = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
    lib.xt_parse.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
    lib.xt_launch.argtypes = launch_args
    lib.xt_matmul_launch_noalloc.argtypes = launch_args
    lib.xt_module_free.argtypes = [ctypes.c_void_p]
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


def _close(got, ref):
    got = got.double().cpu().numpy()
    ref = ref.double().cpu().numpy()
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) <= 1e-2


def test_noalloc_matches_launch_on_consecutive_calls():
    lib = _lib()
    M, N, K = 384, 512, 256
    A = dsl.Array
    text = dsl.trace_text(matmul_kloop, args=(A((M, K), dsl.bfloat16), A((K, N), dsl.bfloat16),
                                              A((M, N), dsl.float32), 128, 128, 64, K // 64),
                          grid=(M // 128, N // 128, 1), double_buffering=True)
    mod = ctypes.c_void_p()
    assert lib.xt_parse(text.encode(), ctypes.byref(mod)) == 0, lib.xt_last_error()
    dev = torch.device("cuda:0")
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    gen = torch.Generator().manual_seed(11)
    try:
        for _ in range(2):
            a = (torch.randn(M, K, generator=gen) / 16).to(torch.bfloat16).to(dev)
            b = (torch.randn(K, N, generator=gen) / 16).to(torch.bfloat16).to(dev)
            ref = torch.full((M, N), float("nan"), device=dev)
            out = torch.full((M, N), float("nan"), device=dev)
            ptrs = (ctypes.c_void_p * 3)(a.data_ptr(), b.data_ptr(), ref.data_ptr())
            assert lib.xt_launch(mod, None, ptrs, 3, 0, 0, stream) == 0, lib.xt_last_error()
            ptrs = (ctypes.c_void_p * 3)(a.data_ptr(), b.data_ptr(), out.data_ptr())
            assert lib.xt_matmul_launch_noalloc(mod, None, ptrs, 3, 0, 0, stream) == 0, lib.xt_last_error()
            torch.cuda.synchronize()
            assert not torch.isnan(out).any()
            _close(out, ref)
    finally:
        lib.xt_module_free(mod)


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
