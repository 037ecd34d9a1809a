"""The tensor-core kernels' bounded waits run out on a GPU, and the context
stays usable.

A GEMM with a long K (512 x 512 x 65536 bf16: one 256 x 256 tile per CTA
pair, about 0.4 ms of MMAs per tile) is launched with a pipeline wait limit of
1 us (``xtile.wait_limit``).  The epilogue warps' wait for the first
accumulator (the whole tile's MMAs) runs out, so the kernel records an error
code -- kErrEpilogue (0x103), or kErrProducer / kErrMma (0x101 / 0x102) if a
pipeline wait ran out first -- stops every role, lets its copies and MMAs
land, frees its tensor memory and returns.  ``device_error()`` reads the code
and clears it.  With the default limit the same launch must then match the
CPU oracle (bf16 tolerance: max|d| / max|ref| <= 1e-2) and leave no error.
No fault, trap or endless loop is involved: the kernel returns on its own.
"""
import numpy as np
import pytest
import torch

import xtile as xt
from oracle import xt_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None
M, N, K, TM, TN = 512, 512, 65536, 128, 128


@xt.kernel
def matmul_long_k(lhs, rhs, out, tm, tn, tk):
    i, j = xt.bid(0), xt.bid(1)
    a = xt.load(lhs, index=(i, 0), shape=(tm, tk))
    b = xt.load(rhs, index=(0, j), shape=(tk, tn), shared=1)
    xt.store(out, index=(i, j), tile=xt.matmul(a, b))


def test_gemm_wait_runs_out_then_recovers():
    g = torch.Generator().manual_seed(31)
    a = (torch.randn(M, K, generator=g) / 256).to(torch.bfloat16)
    b = (torch.randn(K, N, generator=g) / 256).to(torch.bfloat16)
    A = xt.Array
    mod = xt.convert(matmul_long_k, args=(A((M, K), xt.bfloat16), A((K, N), xt.bfloat16), A((M, N), xt.float32),
                                          TM, TN, K), grid=(M // TM, N // TN, 1))
    assert mod.plan()["family"] == "gemm"
    ad, bd = a.to(DEV), b.to(DEV)
    out = torch.zeros(M, N, device=DEV)
    assert xt.device_error() == 0

    with xt.wait_limit(1000):
        xt.launch(mod, ad, bd, out)
    torch.cuda.synchronize()  # the kernel returned by itself
    code = xt.device_error()
    assert code in (0x101, 0x102, 0x103), hex(code)
    assert xt.device_error() == 0  # read and cleared

    out.fill_(float("nan"))
    xt.launch(mod, ad, bd, out)  # default limit
    torch.cuda.synchronize()
    assert xt.device_error() == 0
    blocks = [(0, 0, 0), (3, 1, 0), (1, 3, 0), (2, 2, 0)]
    ref = np.full((M, N), np.nan, np.float32)
    xt_oracle.run(mod.source_text, [a.view(torch.uint16).numpy(), b.view(torch.uint16).numpy(), ref],
                  blocks=blocks)
    got = out.cpu().numpy()
    assert not np.isnan(got).any()
    mask = ~np.isnan(ref)
    d = np.abs(got[mask].astype(np.float64) - ref[mask])
    assert d.max() / np.abs(ref[mask]).max() <= 1e-2


def test_wait_limit_is_validated_and_restored():
    from xtile_b200._native import native

    with pytest.raises(ValueError):
        native.set_wait_limit_ns(61 * 10 ** 9)
    with xt.wait_limit(5000):
        pass
    native.set_wait_limit_ns(0)
