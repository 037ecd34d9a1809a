"""Back-to-back dependent launches.

Every kernel of this backend is launched with programmatic dependent launch:
the next launch on a stream may be scheduled while the previous one drains,
and each kernel waits for its predecessor before touching global memory.
These tests launch chains in which each kernel reads the previous kernel's
output, with no host synchronisation in between, and compare the results with
the same chains run with a synchronisation after every launch.  The kernels
are deterministic, so the comparison is bit for bit; each iteration uses
different inputs, so a read that ran ahead of its producer would see the
previous iteration's values and fail.
"""
import pytest
import torch

import xtile as xt
from tests.test_gpu_kernels import add_tiles, conv2d_tiles, matmul_i8, softmax_rows

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


def gen(seed):
    return torch.Generator().manual_seed(seed)


@pytest.fixture(autouse=True)
def no_device_errors():
    yield
    assert xt.device_error() == 0


def test_add_ping_pong_reads_each_predecessor():
    g = gen(11)
    x = torch.rand(1024, 1024, generator=g) - 0.5
    b = torch.rand(1024, 1024, generator=g) * 1e-3
    bufs = [x.to(DEV), torch.empty(1024, 1024, device=DEV)]
    bd = b.to(DEV)
    m = xt.run(add_tiles, args=(bufs[0], bd, bufs[1], 32, 64), grid=(32, 16, 1))
    torch.cuda.synchronize()
    bufs[0].copy_(x.to(DEV))
    for k in range(64):
        xt.launch(m, bufs[k % 2], bd, bufs[(k + 1) % 2])
    ref = x.clone()
    for _ in range(64):
        ref = ref + b
    assert torch.equal(bufs[0].cpu(), ref)


def test_chain_across_kernel_families_without_syncs():
    g = gen(12)
    M, N, K, iters = 1024, 64, 128, 4
    a = [torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8).to(DEV) for _ in range(iters)]
    b = torch.randint(-128, 128, (K, N), generator=g, dtype=torch.int8).to(DEV)
    scale = (torch.rand(1, N, generator=g) * 1e-4).to(DEV)
    bias = (torch.rand(1, N, generator=g) * 16 - 8).to(DEV)
    f = torch.randint(-16, 16, (3, 3, 64, 64), generator=g, dtype=torch.int8).to(DEV)
    r = torch.rand(M, N, generator=g).to(DEV)
    q = torch.zeros(M, N, dtype=torch.int8, device=DEV)  # GEMM out, conv in as NHWC [1,16,64,64]
    y = torch.empty(1, 16, 64, 64, device=DEV)  # conv out
    s = torch.empty(M, N, device=DEV)  # softmax out
    t = torch.empty(M, N, device=DEV)  # add out
    qi, yr = q.view(1, 16, 64, 64), y.view(M, N)
    m_g = xt.run(matmul_i8, args=(a[0], b, q, scale, bias, 64, 64, K), grid=(M // 64, N // 64, 1))
    m_c = xt.run(conv2d_tiles, args=(qi, f, y, 16, 64, 64, 64, 3, 3, 1, 1, 1, 1), grid=(1, 1, 1))
    m_s = xt.run(softmax_rows, args=(yr, s, 1, N), grid=(M, 1, 1))
    m_a = xt.run(add_tiles, args=(s, r, t, 32, 64), grid=(M // 32, 1, 1))
    assert [m.plan()["family"] for m in (m_g, m_c, m_s, m_a)] == ["gemm", "conv", "rows", "ew"]

    def chain(k, sync):
        for launch in (lambda: xt.launch(m_g, a[k], b, q, scale, bias), lambda: xt.launch(m_c, qi, f, y),
                       lambda: xt.launch(m_s, yr, s), lambda: xt.launch(m_a, s, r, t)):
            launch()
            if sync:
                torch.cuda.synchronize()
        return t.clone()

    ref = [chain(k, True) for k in range(iters)]
    torch.cuda.synchronize()
    got = [chain(k, False) for k in range(iters)]
    torch.cuda.synchronize()
    assert not torch.equal(ref[0], ref[1])
    for k in range(iters):
        assert torch.equal(got[k], ref[k]), f"iteration {k}"
