"""GPU parity: every kernel family against the CPU oracle, through the public
API (xtile.launch -> _xtile -> libxt_b200.so C ABI -> sm_100a kernels).

Tolerances (fixed up front):
* f32 add/sub/mul, int8 matmul with its f32 epilogue: bit-exact;
* row softmax: max elementwise |gpu - ref| / ref <= 1e-5;
* bf16 matmul / conv (f32 accumulation): max|gpu - ref| / max|ref| <= 1e-2
  and |gpu - ref| <= 1e-2 |ref| + 1e-2 rms(ref) per element.
Full-size configurations are checked on a seeded sample of Blocks.
"""
import numpy as np
import pytest
import torch

import xtile as xt
from oracle import xt_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


def gen(seed):
    return torch.Generator().manual_seed(seed)


def host(t):
    t = t.detach().cpu()
    return t.view(torch.uint16).numpy() if t.dtype == torch.bfloat16 else t.numpy()


def oracle(module, arrays, blocks=None):
    outs = [host(a).copy() for a in arrays]
    xt_oracle.run(module.source_text, outs, blocks=blocks)
    return outs


def bf16_close(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.max(np.abs(ref))
    rms = np.sqrt(np.mean(ref ** 2))
    assert np.max(np.abs(got - ref)) / scale <= 1e-2
    assert np.all(np.abs(got - ref) <= 1e-2 * np.abs(ref) + 1e-2 * rms)


@pytest.fixture(autouse=True)
def no_device_errors():
    yield
    assert xt.device_error() == 0


# ------------------------------------------------------------------- add
@xt.kernel
def add_tiles(lhs, rhs, out, th, tw):
    i, j = xt.bid(0), xt.bid(1)
    a = xt.load(lhs, index=(i, j), shape=(th, tw))
    b = xt.load(rhs, index=(i, j), shape=(th, tw))
    xt.store(out, index=(i, j), tile=a + b)


@xt.kernel
def add_rows(lhs, rhs, out, trow, col):
    i = xt.bid(0)
    a = xt.load(lhs, index=(i, 0), shape=(trow, col))
    b = xt.load(rhs, index=(i, 0), shape=(trow, col))
    xt.store(out, index=(i, 0), tile=a + b)


def test_add_config1_bit_exact():
    g = gen(0)
    a = torch.rand(2048, 2048, generator=g) * 2 - 1
    b = torch.rand(2048, 2048, generator=g) * 2 - 1
    c = torch.empty(2048, 2048, device=DEV)
    m = xt.run(add_tiles, args=(a.to(DEV), b.to(DEV), c, 32, 64), grid=(64, 32, 1))
    ref = oracle(m, [a, b, torch.zeros(2048, 2048)])[2]
    assert np.array_equal(host(c).view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("shape,trow", [((128, 128), 64), ((101, 37), 64), ((7, 3), 4)])
def test_add_rows_ragged(shape, trow):
    g = gen(1)
    a = torch.randn(*shape, generator=g)
    b = torch.randn(*shape, generator=g)
    c = torch.full(shape, float("nan"), device=DEV)
    grid = ((shape[0] + trow - 1) // trow, 1, 1)
    m = xt.run(add_rows, args=(a.to(DEV), b.to(DEV), c, trow, shape[1]), grid=grid)
    ref = oracle(m, [a, b, torch.zeros(shape)])[2]
    assert np.array_equal(host(c).view(np.uint32), ref.view(np.uint32))


def test_add_subnormals_and_specials_bit_exact():
    vals = torch.tensor([1e-45, -1e-45, 1e-38, float("inf"), -float("inf"), 0.0, -0.0, 3.0e38])
    a = vals.repeat(16, 1)
    b = vals.flip(0).repeat(16, 1)
    c = torch.empty(16, 8, device=DEV)
    m = xt.run(add_rows, args=(a.to(DEV), b.to(DEV), c, 16, 8), grid=(1, 1, 1))
    ref = oracle(m, [a, b, torch.zeros(16, 8)])[2]
    got = host(c)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    mask = ~np.isnan(ref)
    assert np.array_equal(got[mask].view(np.uint32), ref[mask].view(np.uint32))


@xt.kernel
def ew_mixed(x, y, out, out2, trow, col):
    i = xt.bid(0)
    a = xt.load(x, index=(i, 0), shape=(trow, col))
    b = xt.load(y, index=(i, 0), shape=(trow, col))
    t = xt.exp(a) * b - a
    xt.store(out, index=(i, 0), tile=t)
    xt.store(out2, index=(i, 0), tile=xt.sigmoid(t) + xt.tanh(b))


def test_ew_generated_program():
    g = gen(2)
    a = torch.randn(300, 50, generator=g)
    b = torch.randn(300, 50, generator=g)
    c = torch.empty(300, 50, device=DEV)
    d = torch.empty(300, 50, device=DEV)
    m = xt.run(ew_mixed, args=(a.to(DEV), b.to(DEV), c, d, 100, 50), grid=(3, 1, 1))
    assert m.plan()["family"] == "ew"
    ref = oracle(m, [a, b, torch.zeros(300, 50), torch.zeros(300, 50)])
    np.testing.assert_allclose(host(c), ref[2], rtol=2e-6, atol=1e-6)
    np.testing.assert_allclose(host(d), ref[3], rtol=2e-6, atol=1e-6)


@xt.kernel
def ew_int8(q, r, y, yq, trow, col):
    i = xt.bid(0)
    a = xt.astype(xt.load(q, index=(i, 0), shape=(trow, col)), dtype=xt.float32)
    b = xt.load(r, index=(i, 0), shape=(trow, col))
    t = a * b + a
    xt.store(y, index=(i, 0), tile=t)
    xt.store(yq, index=(i, 0), tile=xt.astype(t, dtype=xt.int8))


def test_ew_generated_int8_casts_tail_and_shards_bit_exact():
    # 7 x 13 = 91 elements: 22 groups of four (4-byte int8 and 16-byte f32
    # accesses) and a tail of 3; a bid0 shard starting at element 13 runs the
    # element-at-a-time kernel.  ftoi rounds half to even and saturates.
    g = gen(29)
    q = torch.randint(-128, 128, (7, 13), generator=g, dtype=torch.int8)
    r = torch.randn(7, 13, generator=g) * 3
    y = torch.empty(7, 13, device=DEV)
    yq = torch.zeros(7, 13, dtype=torch.int8, device=DEV)
    m = xt.run(ew_int8, args=(q.to(DEV), r.to(DEV), y, yq, 1, 13), grid=(7, 1, 1))
    assert m.plan()["family"] == "ew"
    ref = oracle(m, [q, r, torch.zeros(7, 13), torch.zeros(7, 13, dtype=torch.int8)])
    assert np.array_equal(host(y).view(np.uint32), ref[2].view(np.uint32))
    assert np.array_equal(host(yq), ref[3])
    y2 = torch.full((7, 13), float("nan"), device=DEV)
    yq2 = torch.zeros(7, 13, dtype=torch.int8, device=DEV)
    for lo, hi in [(0, 1), (1, 7)]:
        xt.launch(m, q.to(DEV), r.to(DEV), y2, yq2, bid0_range=(lo, hi))
    assert torch.equal(y, y2) and torch.equal(yq, yq2)


@xt.kernel
def ew_copy(x, y, trow, col):
    i = xt.bid(0)
    xt.store(y, index=(i, 0), tile=xt.load(x, index=(i, 0), shape=(trow, col)))


@pytest.mark.parametrize("shape,trow", [((64, 200), 16), ((9, 35), 3)])
def test_ew_bf16_copy_bit_exact(shape, trow):
    # bf16 through the generated ew kernel: 8-byte groups of four; 9 x 35 = 315
    # elements leave a 3-element tail, and its bid0 shard starting at element
    # 105 takes the element-at-a-time kernel; values pass through f32 and come back
    # bit for bit
    x = torch.randn(*shape, generator=gen(31)).to(torch.bfloat16)
    y = torch.zeros(*shape, dtype=torch.bfloat16, device=DEV)
    m = xt.run(ew_copy, args=(x.to(DEV), y, trow, shape[1]), grid=(shape[0] // trow, 1, 1))
    assert m.plan()["family"] == "ew"
    assert torch.equal(y.cpu(), x)
    y2 = torch.zeros(*shape, dtype=torch.bfloat16, device=DEV)
    g0 = shape[0] // trow
    for lo, hi in [(0, 1), (1, g0)]:
        xt.launch(m, x.to(DEV), y2, bid0_range=(lo, hi))
    assert torch.equal(y2.cpu(), x)


# --------------------------------------------------------------- softmax
@xt.kernel
def softmax_rows(inp, out, trow, col):
    i = xt.bid(0)
    x = xt.load(inp, index=(i, 0), shape=(trow, col))
    x = x - xt.max(x, axis=-1)
    x = xt.exp(x)
    xt.store(out, index=(i, 0), tile=x / xt.sum(x, axis=-1))


def softmax_case(rows, cols, trow, seed, blocks=None):
    x = torch.randn(rows, cols, generator=gen(seed)) * 4
    y = torch.empty(rows, cols, device=DEV)
    grid = ((rows + trow - 1) // trow, 1, 1)
    m = xt.run(softmax_rows, args=(x.to(DEV), y, trow, cols), grid=grid)
    ref = oracle(m, [x, torch.zeros(rows, cols)], blocks=blocks)[1]
    return host(y), ref


def test_softmax_config2():
    blocks = [(b, 0, 0) for b in np.random.default_rng(1).choice(8192, 512, replace=False)]
    got, ref = softmax_case(8192, 1024, 1, 1, blocks)
    rows = [b[0] for b in blocks]
    assert np.max(np.abs(got[rows] - ref[rows]) / ref[rows]) <= 1e-5
    np.testing.assert_allclose(got.sum(axis=1), 1.0, rtol=1e-5)


@pytest.mark.parametrize("rows,cols,trow", [(128, 128, 64), (100, 37, 64), (9, 2048, 4), (33, 100, 8)])
def test_softmax_shapes(rows, cols, trow):
    got, ref = softmax_case(rows, cols, trow, 3)
    assert np.max(np.abs(got - ref) / ref) <= 1e-5


@xt.kernel
def row_stats(x, y, mx, trow, col):
    i = xt.bid(0)
    t = xt.load(x, index=(i, 0), shape=(trow, col))
    m = xt.max(t, axis=1)
    xt.store(y, index=(i, 0), tile=(t - m) * (t - m))
    xt.store(mx, index=(i, 0), tile=xt.reciprocal(xt.sum(t, axis=1)))


@pytest.mark.parametrize("rows,cols", [(96, 200), (64, 1024), (50, 37), (33, 128), (40, 2048), (20, 1531)])
def test_row_program_generated(rows, cols):
    # cols a multiple of 4: float4 accesses; 37 and 1531 columns: element
    # accesses with a guard per element (partial last chunk of every row)
    x = torch.randn(rows, cols, generator=gen(4)) + 3
    y = torch.empty(rows, cols, device=DEV)
    mx = torch.empty(rows, 1, device=DEV)
    m = xt.run(row_stats, args=(x.to(DEV), y, mx, 32, cols), grid=((rows + 31) // 32, 1, 1))
    assert m.plan()["family"] == "rows"
    ref = oracle(m, [x, torch.zeros(rows, cols), torch.zeros(rows, 1)])
    np.testing.assert_array_equal(host(y), ref[1])
    np.testing.assert_allclose(host(mx), ref[2], rtol=1e-5)


@pytest.mark.parametrize("rows,cols", [(40, 3000), (24, 8192), (10, 6000), (9, 4097)])
def test_row_program_wide_rows_one_cta_per_row(rows, cols):
    # rows wider than 2048 columns run one CTA per row (128 to 1024 threads,
    # block reductions through shared memory); 3000 and 6000 columns: a
    # partial last chunk; 4097: element accesses.  (This program keeps three
    # rows live: 8192 columns is the widest a CTA holds.)
    x = torch.randn(rows, cols, generator=gen(5)) + 3
    y = torch.empty(rows, cols, device=DEV)
    mx = torch.empty(rows, 1, device=DEV)
    m = xt.run(row_stats, args=(x.to(DEV), y, mx, 8, cols), grid=((rows + 7) // 8, 1, 1))
    assert m.plan()["family"] == "rows"
    ref = oracle(m, [x, torch.zeros(rows, cols), torch.zeros(rows, 1)])
    np.testing.assert_array_equal(host(y), ref[1])
    np.testing.assert_allclose(host(mx), ref[2], rtol=1e-5)
    assert xt.device_error() == 0


@pytest.mark.parametrize("rows,cols", [(16, 8192), (6, 32768), (12, 5001)])
def test_softmax_wide_rows_and_shards(rows, cols):
    # kernels/softmax.py's program on rows wider than the dedicated kernel
    # takes (2048): the generated one-CTA-per-row kernel; a bid0 split into
    # two launches gives the same rows
    got, ref = softmax_case(rows, cols, 1, 7)
    assert np.max(np.abs(got - ref) / ref) <= 1e-5
    x = torch.randn(rows, cols, generator=gen(7)) * 4
    y2 = torch.full((rows, cols), float("nan"), device=DEV)
    m = xt.convert(softmax_rows, args=(xt.Array((rows, cols), xt.float32), xt.Array((rows, cols), xt.float32), 1, cols),
                   grid=(rows, 1, 1))
    assert m.plan()["family"] == "rows"
    for lo, hi in [(0, rows // 2), (rows // 2, rows)]:
        xt.launch(m, x.to(DEV), y2, bid0_range=(lo, hi))
    np.testing.assert_array_equal(host(y2), got)


# ---------------------------------------------------------------- matmul
@xt.kernel
def matmul_kloop(lhs, rhs, out, tm, tn, tk, ksteps):
    i, j = xt.bid(0), xt.bid(1)
    acc = None
    for k in range(ksteps):
        p = xt.matmul(xt.load(lhs, index=(i, k), shape=(tm, tk)),
                      xt.load(rhs, index=(k, j), shape=(tk, tn), shared=1))
        acc = p if acc is None else acc + p
    xt.store(out, index=(i, j), tile=acc)


@xt.kernel
def matmul_single(lhs, rhs, out, tm, tn, tk):
    i, j = xt.bid(0), xt.bid(1)
    a = xt.load(lhs, index=(i, 0), shape=(tm, tk))
    b = xt.load(rhs, index=(0, j), shape=(tk, tn), shared=1)
    xt.store(out, index=(i, j), tile=xt.matmul(a, b))


def bf16_inputs(m, n, k, seed, scale=None):
    g = gen(seed)
    s = scale if scale is not None else 1.0 / np.sqrt(k)
    a = (torch.randn(m, k, generator=g) * s).to(torch.bfloat16)
    b = (torch.randn(k, n, generator=g) * s).to(torch.bfloat16)
    return a, b


def test_matmul_bf16_kloop_small():
    a, b = bf16_inputs(256, 256, 512, 5)
    c = torch.empty(256, 256, device=DEV)
    m = xt.run(matmul_kloop, args=(a.to(DEV), b.to(DEV), c, 128, 128, 64, 8), grid=(2, 2, 1))
    assert m.plan()["family"] == "gemm"
    ref = oracle(m, [a, b, torch.zeros(256, 256)])[2]
    bf16_close(host(c), ref)


@pytest.mark.parametrize("mnk,tile", [((300, 200, 96), (128, 128, 96)), ((128, 520, 64), (128, 256, 64)),
                                      ((64, 64, 8), (64, 64, 8)),
                                      # 3 k-blocks per tile, 320 tiles: tiles share pipeline groups
                                      # and most CTAs end inside a group
                                      ((5120, 2048, 192), (128, 256, 192)),
                                      # 80 pair tiles on 74 pairs: the last 6 split into column halves
                                      ((2560, 2048, 128), (128, 256, 128)),
                                      ((2523, 1944, 96), (128, 256, 96))])
def test_matmul_bf16_ragged(mnk, tile):
    M, N, K = mnk
    tm, tn, tk = tile
    a, b = bf16_inputs(M, N, K, 6)
    c = torch.full((M, N), float("nan"), device=DEV)
    grid = ((M + tm - 1) // tm, (N + tn - 1) // tn, 1)
    m = xt.run(matmul_single, args=(a.to(DEV), b.to(DEV), c, tm, tn, tk), grid=grid)
    ref = oracle(m, [a, b, torch.zeros(M, N)])[2]
    bf16_close(host(c), ref)


def test_matmul_config3_sampled():
    a, b = bf16_inputs(4096, 4096, 4096, 2, scale=1.0 / 64)
    c = torch.empty(4096, 4096, device=DEV)
    m = xt.run(matmul_kloop, args=(a.to(DEV), b.to(DEV), c, 128, 128, 64, 64), grid=(32, 32, 1))
    rng = np.random.default_rng(2)
    blocks = [(int(x), int(y), 0) for x, y in zip(rng.integers(0, 32, 12), rng.integers(0, 32, 12))]
    blocks += [(0, 0, 0), (31, 31, 0), (0, 31, 0), (31, 0, 0)]
    ref = oracle(m, [a, b, torch.zeros(4096, 4096)], blocks=blocks)[2]
    got = host(c)
    for x, y, _ in blocks:
        sl = (slice(x * 128, x * 128 + 128), slice(y * 128, y * 128 + 128))
        bf16_close(got[sl], ref[sl])


def test_matmul_bid0_shards_match_full_launch():
    a, b = bf16_inputs(2048, 1024, 1024, 7)
    full = torch.empty(2048, 1024, device=DEV)
    parts = torch.full((2048, 1024), float("nan"), device=DEV)
    m = xt.run(matmul_single, args=(a.to(DEV), b.to(DEV), full, 256, 128, 1024), grid=(8, 8, 1))
    for lo, hi in [(0, 3), (3, 4), (4, 8)]:
        xt.launch(m, a.to(DEV), b.to(DEV), parts, bid0_range=(lo, hi))
    assert torch.equal(full, parts)


def test_matmul_config5_shards_full_size():
    """Config 5 at full size (A bf16 [32768,8192] x B bf16 [8192,8192], seed 4,
    256x128 Blocks, grid (128,64)), built exactly as bench.py builds it.

    * the bid0 splits bench.py uses (equal shares over 2, 4 and 8 ranks, and the
      peer-gather split that gives rank 0 a larger share) each reproduce a
      full launch bit for bit;
    * three seeded Blocks in every one of the 8 equal shards (its first and
      last bid0 and one inside: 768 rows per shard) against the oracle;
    * the full rows on both sides of every shard boundary against float64 dot
      products of the same bf16 inputs.
    """
    import bench

    w = bench.build_workload("sharded_matmul", bench.load_dsl(), torch, 1, 0)
    m = xt.parse(w["text"])
    a_h, b_h = w["inputs"]
    a, b = a_h.to(DEV), b_h.to(DEV)
    M, N = w["out_shape"]
    grid0 = m.plan()["grid"][0]
    full = torch.empty(M, N, device=DEV)
    xt.launch(m, a, b, full)
    parts = torch.empty(M, N, device=DEV)
    splits = [(world, None) for world in (2, 4, 8)]
    splits += [(world, bench.gather_root_share(world, 2.0 * M * N * 8192, M * N * 4.0)) for world in (4, 8)]
    bounds = set()
    for world, share in splits:
        parts.fill_(float("nan"))
        for r in range(world):
            lo, hi = bench.bid0_share(grid0, world, r, share)
            xt.launch(m, a, b, parts, bid0_range=(lo, hi))
            bounds.add(lo)
        assert torch.equal(full, parts), (world, share)
    del parts

    rng = np.random.default_rng(4)
    blocks = []
    for s in range(8):
        lo, hi = bench.bid0_share(grid0, 8, s)
        for x in (lo, int(rng.integers(lo + 1, hi - 1)), hi - 1):
            blocks.append((x, int(rng.integers(0, 64)), 0))
    ref = oracle(m, [a_h, b_h, torch.zeros(M, N)], blocks=blocks)[2]
    got = host(full)
    for x, y, _ in blocks:
        sl = (slice(x * 256, x * 256 + 256), slice(y * 128, y * 128 + 128))
        bf16_close(got[sl], ref[sl])

    rows = sorted({r for lo in bounds if lo > 0 for r in (lo * 256 - 1, lo * 256)})
    a64 = a_h[rows].double().numpy()
    b64 = b_h.double().numpy()
    bf16_close(got[rows], a64 @ b64)
    torch.cuda.empty_cache()


@xt.kernel
def matmul_i8(lhs, rhs, res, scale, bias, tm, tn, tk):
    i, j = xt.bid(0), xt.bid(1)
    a = xt.load(lhs, index=(i, 0), shape=(tm, tk))
    b = xt.load(rhs, index=(0, j), shape=(tk, tn), shared=1)
    s = xt.load(scale, index=(0, j), shape=(1, tn), shared=1)
    c = xt.load(bias, index=(0, j), shape=(1, tn), shared=1)
    t = xt.matmul(a, b)
    t = t * s + c
    xt.store(res, index=(i, j), tile=xt.astype(t, dtype=xt.int8))


@pytest.mark.parametrize("m_,n_,k_", [(128, 128, 256), (1024, 512, 256), (192, 320, 128)])
def test_matmul_int8_epilogue_bit_exact(m_, n_, k_):
    g = gen(8)
    a = torch.randint(-128, 128, (m_, k_), generator=g, dtype=torch.int8)
    b = torch.randint(-128, 128, (k_, n_), generator=g, dtype=torch.int8)
    s = torch.rand(1, n_, generator=g) * 1e-4
    bias = torch.rand(1, n_, generator=g) * 16 - 8
    c = torch.zeros(m_, n_, dtype=torch.int8, device=DEV)
    grid = ((m_ + 63) // 64, (n_ + 63) // 64, 1)
    m = xt.run(matmul_i8, args=(a.to(DEV), b.to(DEV), c, s.to(DEV), bias.to(DEV), 64, 64, k_), grid=grid)
    ref = oracle(m, [a, b, torch.zeros(m_, n_, dtype=torch.int8), s, bias])[2]
    assert np.array_equal(host(c), ref)


@xt.kernel
def mma_chain(a, b, acc_in, acc_out, tm, tn, tk, ksteps):
    i, j = xt.bid(0), xt.bid(1)
    acc = xt.load(acc_in, index=(i, j), shape=(tm, tn))
    for k in range(ksteps):
        acc = xt.mma(xt.load(a, index=(i, k), shape=(tm, tk)), xt.load(b, index=(k, j), shape=(tk, tn)), acc)
    xt.store(acc_out, index=(i, j), tile=acc)


def test_mma_int8_accumulator_bit_exact():
    g = gen(9)
    a = torch.randint(-20, 20, (256, 256), generator=g, dtype=torch.int8)
    b = torch.randint(-20, 20, (256, 256), generator=g, dtype=torch.int8)
    acc = torch.randint(-1000, 1000, (256, 256), generator=g).float()
    out = torch.empty(256, 256, device=DEV)
    m = xt.run(mma_chain, args=(a.to(DEV), b.to(DEV), acc.to(DEV), out, 128, 128, 128, 2), grid=(2, 2, 1))
    ref = oracle(m, [a, b, acc, torch.zeros(256, 256)])[3]
    assert np.array_equal(host(out), ref)


def test_launch_rejects_bad_arguments():
    a, b = bf16_inputs(256, 256, 64, 10)
    c = torch.empty(256, 256, device=DEV)
    m = xt.run(matmul_single, args=(a.to(DEV), b.to(DEV), c, 128, 128, 64), grid=(2, 2, 1))
    with pytest.raises(TypeError, match="must be bf16"):
        xt.launch(m, a.float().to(DEV), b.to(DEV), c)
    with pytest.raises(ValueError, match="shape"):
        xt.launch(m, a[:128].to(DEV), b.to(DEV), c)
    with pytest.raises(ValueError, match="expects 3 arrays"):
        xt.launch(m, a.to(DEV), b.to(DEV))
    with pytest.raises(ValueError, match="outside the grid"):
        xt.launch(m, a.to(DEV), b.to(DEV), c, bid0_range=(0, 5))


# ------------------------------------------------------------------ conv
@xt.kernel
def conv2d_tiles(inp, filt, out, tile_h, tile_w, cin, cout, kh, kw, ph, pw, dh, dw):
    n, h, w = xt.bid(0), xt.bid(1), xt.bid(2)
    f = xt.load(filt, index=(0, 0, 0, 0), shape=(kh, kw, cin, cout), shared=2)
    y = xt.load_conv2d(inp, f, index=(n, h, w, 0), shape=(1, tile_h, tile_w, cout), group=1,
                       pad=(ph, pw, ph, pw), stride=(1, 1), dilation=(dh, dw))
    xt.store(out, index=(n, h, w, 0), tile=y)


def conv_case(shape, kshape, tile, dtype, seed, pad=None, dil=(1, 1), blocks=None):
    n, h, w, c = shape
    kh, kw, _, ko = kshape
    th, tw = tile
    g = gen(seed)
    if dtype == torch.int8:
        x = torch.randint(-16, 16, shape, generator=g, dtype=torch.int8)
        f = torch.randint(-16, 16, kshape, generator=g, dtype=torch.int8)
    else:
        x = (torch.randn(*shape, generator=g) * 0.1).to(dtype)
        f = (torch.randn(*kshape, generator=g) * 0.1).to(dtype)
    ph, pw = pad if pad is not None else (kh // 2, kw // 2)
    out = torch.full((n, h, w, ko), float("nan"), device=DEV)
    grid = (n, (h + th - 1) // th, (w + tw - 1) // tw)
    m = xt.run(conv2d_tiles, args=(x.to(DEV), f.to(DEV), out, th, tw, c, ko, kh, kw, ph, pw, *dil), grid=grid)
    assert m.plan()["family"] == "conv"
    ref = oracle(m, [x, f, torch.zeros(n, h, w, ko)], blocks=blocks)[2]
    return host(out), ref


def test_conv_config4_bf16_sampled():
    blocks = [(b, hb, 0) for b in (0, 13, 31) for hb in range(7)]
    got, ref = conv_case((32, 56, 56, 64), (3, 3, 64, 64), (8, 56), torch.bfloat16, 3, blocks=blocks)
    for b in (0, 13, 31):
        bf16_close(got[b], ref[b])


@pytest.mark.parametrize("shape,kshape,tile,pad,dil", [
    ((2, 9, 70, 64), (3, 3, 64, 32), (3, 35), None, (1, 1)),     # two W tiles, odd H, ragged tiles
    ((1, 16, 16, 96), (5, 5, 96, 64), (16, 16), (2, 2), (1, 1)),  # channel chunk past C (zero-filled)
    ((1, 12, 20, 64), (3, 3, 64, 128), (4, 20), (2, 2), (2, 2)),  # dilation 2, 128 output channels
    ((1, 20, 300, 64), (3, 3, 64, 64), (10, 100), None, (1, 1)),  # window kernel, 4 column strips
    ((2, 10, 30, 128), (3, 3, 128, 64), (5, 30), None, (1, 1)),   # window kernel, 2 channel chunks
    ((1, 9, 9, 64), (1, 1, 64, 256), (9, 9), (0, 0), (1, 1)),     # 1x1, 256 output channels
    ((1, 16, 16, 32), (5, 5, 32, 32), (16, 16), (2, 2), (1, 1)),  # window kernel, any-tap loop
    ((3, 16, 16, 32), (5, 5, 32, 32), (16, 16), (2, 2), (1, 1)),  # 5 stacked taps, 4 shifted rows
    ((1, 12, 20, 64), (3, 3, 64, 64), (4, 20), (2, 2), (2, 2)),   # stacked taps with dilation 2
    ((3, 17, 45, 64), (3, 3, 64, 64), (6, 45), None, (1, 1)),     # window kernel, odd sizes
    ((1, 14, 33, 64), (5, 3, 64, 64), (5, 33), (2, 1), (2, 1)),   # 5 x 3 filter, dilation 2 in H
    ((1, 12, 20, 64), (3, 3, 64, 64), (4, 22), (2, 2), (1, 1)),   # pad 2: output wider than the input
])
def test_conv_bf16_shapes(shape, kshape, tile, pad, dil):
    got, ref = conv_case(shape, kshape, tile, torch.bfloat16, 4, pad=pad, dil=dil)
    bf16_close(got, ref)


@pytest.mark.parametrize("sms,shape,dtype", [
    (8, (6, 20, 30, 64), torch.bfloat16),    # 6 strips x 3 tiles on 8 CTAs: 2 waves and a partial one
    (6, (5, 17, 45, 64), torch.bfloat16),    # odd sizes
    (4, (3, 16, 32, 64), torch.int8),        # int8, exact
])
def test_conv_window_several_waves(sms, shape, dtype):
    # Few CTAs (an SM budget): each CTA runs several tiles through its window
    # ring and both accumulators, the last wave partial.
    n, h, w, c = shape
    g = gen(9)
    if dtype == torch.int8:
        x = torch.randint(-16, 16, shape, generator=g, dtype=torch.int8)
        f = torch.randint(-16, 16, (3, 3, c, 64), generator=g, dtype=torch.int8)
    else:
        x = (torch.randn(*shape, generator=g) * 0.1).to(dtype)
        f = (torch.randn(3, 3, c, 64, generator=g) * 0.1).to(dtype)
    out = torch.full((n, h, w, 64), float("nan"), device=DEV)
    with xt.sm_budget(sms):
        m = xt.run(conv2d_tiles, args=(x.to(DEV), f.to(DEV), out, h, w, c, 64, 3, 3, 1, 1, 1, 1), grid=(n, 1, 1))
    assert m.plan()["family"] == "conv"
    ref = oracle(m, [x, f, torch.zeros(n, h, w, 64)])[2]
    got = host(out)
    if dtype == torch.int8:
        assert np.array_equal(got, ref)
    else:
        bf16_close(got, ref)


def test_conv_int8_two_images_bit_exact():
    # two images, stacked taps with kind::i8
    got, ref = conv_case((2, 16, 32, 128), (3, 3, 128, 64), (16, 32), torch.int8, 8)
    assert np.array_equal(got, ref)


def test_conv_int8_kernels_conv2d_pattern_bit_exact():
    # kernels/conv2d.py defaults: n=1, 32x64 image, cin=128, cout=64, 3x3, tile 32x64
    got, ref = conv_case((1, 32, 64, 128), (3, 3, 128, 64), (32, 64), torch.int8, 5)
    assert np.array_equal(got, ref)


def test_conv_bid0_shards_match_full_launch():
    g = gen(6)
    x = (torch.randn(8, 14, 14, 64, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    f = (torch.randn(3, 3, 64, 64, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    full = torch.empty(8, 14, 14, 64, device=DEV)
    parts = torch.full((8, 14, 14, 64), float("nan"), device=DEV)
    m = xt.run(conv2d_tiles, args=(x, f, full, 7, 14, 64, 64, 3, 3, 1, 1, 1, 1), grid=(8, 2, 1))
    for lo, hi in [(0, 3), (3, 8)]:
        xt.launch(m, x, f, parts, bid0_range=(lo, hi))
    assert torch.equal(full, parts)
