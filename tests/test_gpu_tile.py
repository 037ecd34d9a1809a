"""GPU parity of the tile family against the CPU oracle, through the public API.

Tolerances: bit-exact for everything but f32 sums (f64 accumulation in both,
in different orders, then one rounding to f32: |gpu - ref| <= 1e-6 |ref| + 1e-6).
"""
import numpy as np
import pytest
import torch

import xtile as xt
from oracle import xt_oracle
from tests.test_tile import col_sums, transpose3

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None
A = xt.Array
f32 = xt.float32


def gen(seed):
    return torch.Generator().manual_seed(seed)


def host(t):
    return t.detach().cpu().numpy()


def oracle(module, arrays):
    outs = [np.array(host(a)) for a in arrays]
    xt_oracle.run(module.source_text, outs)
    return outs


@pytest.fixture(autouse=True)
def no_device_errors():
    yield
    assert xt.device_error() == 0


def test_transpose_rank3_ragged_bit_exact():
    x = torch.randn(2, 96, 200, generator=gen(1))
    y = torch.full((2, 200, 96), float("nan"), device=DEV)
    m = xt.run(transpose3, args=(x.to(DEV), y, 32, 64), grid=(2, 3, 4))
    assert m.plan()["family"] == "tile"
    ref = oracle(m, [x, torch.zeros(2, 200, 96)])[1]
    assert np.array_equal(host(y), ref)
    assert np.array_equal(ref, np.swapaxes(host(x), 1, 2))


def test_transpose_bid0_shards_match_full_launch():
    x = torch.randn(4, 64, 64, generator=gen(2)).to(DEV)
    full = torch.empty(4, 64, 64, device=DEV)
    parts = torch.full((4, 64, 64), float("nan"), device=DEV)
    m = xt.run(transpose3, args=(x, full, 32, 32), grid=(4, 2, 2))
    for lo, hi in [(0, 1), (1, 3), (3, 4)]:
        xt.launch(m, x, parts, bid0_range=(lo, hi))
    assert torch.equal(full, parts)


@xt.kernel
def reshape_tiles(x, y, tm, tn):
    i, j = xt.bid(0), xt.bid(1)
    t = xt.load(x, index=(i, j), shape=(tm, tn))
    xt.store(y, index=(i, j), tile=xt.reshape(t, shape=(tn, tm)))


def test_reshape_bit_exact():
    x = torch.randn(64, 128, generator=gen(3))
    y = torch.empty(128, 64, device=DEV)
    m = xt.run(reshape_tiles, args=(x.to(DEV), y, 16, 32), grid=(4, 4, 1))
    assert m.plan()["family"] == "tile"
    ref = oracle(m, [x, torch.zeros(128, 64)])[1]
    assert np.array_equal(host(y), ref)


@xt.kernel
def col_stats(x, s, mx, tm, tn):
    i, j = xt.bid(0), xt.bid(1)
    t = xt.load(x, index=(i, j), shape=(tm, tn))
    xt.store(s, index=(i, j), tile=xt.sum(t, axis=0))
    xt.store(mx, index=(i, j), tile=xt.max(t, axis=0))


def test_axis0_reductions():
    x = torch.randn(256, 96, generator=gen(4)) * 3
    s = torch.empty(4, 96, device=DEV)
    mx = torch.empty(4, 96, device=DEV)
    m = xt.run(col_stats, args=(x.to(DEV), s, mx, 64, 32), grid=(4, 3, 1))
    assert m.plan()["family"] == "tile"
    _, ref_s, ref_m = oracle(m, [x, torch.zeros(4, 96), torch.zeros(4, 96)])
    assert np.array_equal(host(mx), ref_m)
    got = host(s)
    assert np.all(np.abs(got - ref_s) <= 1e-6 * np.abs(ref_s) + 1e-6)


def test_axis0_sums_ragged_tiles():
    # 100 rows in tiles of 64: the second tile's rows past the edge load zero
    x = torch.randn(100, 40, generator=gen(5))
    y = torch.empty(2, 40, device=DEV)
    m = xt.run(col_sums, args=(x.to(DEV), y, 64, 40), grid=(2, 1, 1))
    ref = oracle(m, [x, torch.zeros(2, 40)])[1]
    got = host(y)
    assert np.all(np.abs(got - ref) <= 1e-6 * np.abs(ref) + 1e-6)


@xt.kernel
def row_vector_ops(x, v, y, tm, tn):
    i = xt.bid(0)
    t = xt.load(x, index=(i, 0), shape=(tm, tn))
    r = xt.load(v, index=(0, 0), shape=(1, tn), shared=1)
    xt.store(y, index=(i, 0), tile=xt.sigmoid(t * r - r))


@pytest.mark.parametrize("rows,cols,tm", [(128, 64, 32), (96, 37, 32), (64, 512, 8)])
def test_row_vector_broadcast_runs_elementwise(rows, cols, tm):
    # a [1, C] row broadcast over the rows is an elementwise program (the row
    # is element i mod C of the flat map); 37 columns take the one-element
    # kernel, 64 and 512 the vectorised one; a bid0 split matches
    x = torch.randn(rows, cols, generator=gen(6))
    v = torch.randn(1, cols, generator=gen(7))
    y = torch.empty(rows, cols, device=DEV)
    m = xt.run(row_vector_ops, args=(x.to(DEV), v.to(DEV), y, tm, cols), grid=(rows // tm, 1, 1))
    assert m.plan()["family"] == "ew"
    ref = oracle(m, [x, v, torch.zeros(rows, cols)])[2]
    # sigmoid: CUDA expf against numpy's f64 exp, within a few ulp
    np.testing.assert_allclose(host(y), ref, rtol=1e-6, atol=1e-7)
    y2 = torch.full((rows, cols), float("nan"), device=DEV)
    g0 = rows // tm
    for lo, hi in [(0, 1), (1, g0)]:
        xt.launch(m, x.to(DEV), v.to(DEV), y2, bid0_range=(lo, hi))
    assert torch.equal(y, y2)


@xt.kernel
def col_vector_ops(x, c, y, tm, tn):
    i, j = xt.bid(0), xt.bid(1)
    t = xt.load(x, index=(i, j), shape=(tm, tn))
    s = xt.load(c, index=(i, 0), shape=(tm, 1))
    xt.store(y, index=(i, j), tile=xt.sigmoid(t * s - s))


@pytest.mark.parametrize("rows,cols,tm,tn", [(128, 128, 32, 64), (128, 256, 32, 128), (64, 512, 16, 256),
                                             (96, 1024, 8, 512)])
def test_column_vector_broadcast_tile_cta_widths(rows, cols, tm, tn):
    # a (tm, 1) column broadcast over tiles narrower than a row is a tile
    # program; its generated kernel runs 128 threads for the 2048- and
    # 4096-element tiles (32x64, 32x128, 16x256, 8x512: one or several rows
    # per warp)
    x = torch.randn(rows, cols, generator=gen(6))
    c = torch.randn(rows, 1, generator=gen(7))
    y = torch.empty(rows, cols, device=DEV)
    m = xt.run(col_vector_ops, args=(x.to(DEV), c.to(DEV), y, tm, tn), grid=(rows // tm, cols // tn, 1))
    assert m.plan()["family"] == "tile"
    ref = oracle(m, [x, c, torch.zeros(rows, cols)])[2]
    np.testing.assert_allclose(host(y), ref, rtol=1e-6, atol=1e-7)


def _text_case(body_op: str, out_shape: str, result_tensor: str):
    return f"""func.func @p(%x: memref<4x3x5xf32>, %y: memref<{out_shape}xf32>) attributes {{xt.grid = array<i32: 2, 1, 1>}} {{
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %t = xt.load(%x, %bid#0, %zero, %zero) : (memref<4x3x5xf32>, i32, i32, i32) -> tensor<2x3x5xf32>
  {body_op}
  xt.store(%u, %y, %bid#0, %zero, %zero) : ({result_tensor}, memref<{out_shape}xf32>, i32, i32, i32) -> ()
  func.return
}}"""


def test_permute_bit_exact():
    text = _text_case("%u = xt.permute(%t) {permutation = [2, 0, 1]} : tensor<2x3x5xf32> -> tensor<5x2x3xf32>",
                      "10x2x3", "tensor<5x2x3xf32>")
    m = xt.parse(text)
    assert m.plan()["family"] == "tile"
    x = torch.randn(4, 3, 5, generator=gen(8))
    y = torch.empty(10, 2, 3, device=DEV)
    xt.launch(m, x.to(DEV), y)
    ref = oracle(m, [x, torch.zeros(10, 2, 3)])[1]
    assert np.array_equal(host(y), ref)


def test_splat_constant_bit_exact():
    text = _text_case("%c = arith.constant dense<1.250000e-01> : tensor<2x3x5xf32>\n"
                      "  %u = xt.mul(%t, %c) : tensor<2x3x5xf32>, tensor<2x3x5xf32> -> tensor<2x3x5xf32>",
                      "4x3x5", "tensor<2x3x5xf32>")
    m = xt.parse(text)
    assert m.plan()["family"] == "tile"
    x = torch.randn(4, 3, 5, generator=gen(9))
    y = torch.empty(4, 3, 5, device=DEV)
    xt.launch(m, x.to(DEV), y)
    ref = oracle(m, [x, torch.zeros(4, 3, 5)])[1]
    assert np.array_equal(host(y), ref)


@xt.kernel
def i8_wrap(a, b, y, tm, tn):
    i, j = xt.bid(0), xt.bid(1)
    s = xt.load(a, index=(i, j), shape=(tm, tn)) + xt.load(b, index=(0, j), shape=(1, tn))
    xt.store(y, index=(i, j), tile=s * s)


def test_int8_arithmetic_wraps_bit_exact():
    g = gen(10)
    a = torch.randint(-128, 128, (64, 64), generator=g, dtype=torch.int8)
    b = torch.randint(-128, 128, (1, 64), generator=g, dtype=torch.int8)
    y = torch.zeros(64, 64, dtype=torch.int8, device=DEV)
    m = xt.run(i8_wrap, args=(a.to(DEV), b.to(DEV), y, 16, 32), grid=(4, 2, 1))
    assert m.plan()["family"] == "tile"
    ref = oracle(m, [a, b, torch.zeros(64, 64, dtype=torch.int8)])[2]
    assert np.array_equal(host(y), ref)


def test_rank4_permute_leading_dims():
    # rank-4 tiles with non-unit leading dims: rows unravel into three indices
    text = """func.func @r(%x: memref<4x6x10x12xf32>, %y: memref<4x10x6x12xf32>) attributes {xt.grid = array<i32: 2, 1, 2>} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %t = xt.load(%x, %bid#0, %zero, %bid#2, %zero) : (memref<4x6x10x12xf32>, i32, i32, i32, i32) -> tensor<2x6x5x12xf32>
  %p = xt.permute(%t) {permutation = [0, 2, 1, 3]} : tensor<2x6x5x12xf32> -> tensor<2x5x6x12xf32>
  %u = xt.mul(%p, %p) : tensor<2x5x6x12xf32>, tensor<2x5x6x12xf32> -> tensor<2x5x6x12xf32>
  xt.store(%u, %y, %bid#0, %bid#2, %zero, %zero) : (tensor<2x5x6x12xf32>, memref<4x10x6x12xf32>, i32, i32, i32, i32) -> ()
  func.return
}"""
    m = xt.parse(text)
    assert m.plan()["family"] == "tile"
    x = torch.randn(4, 6, 10, 12, generator=gen(11))
    y = torch.full((4, 10, 6, 12), float("nan"), device=DEV)
    xt.launch(m, x.to(DEV), y)
    ref = oracle(m, [x, torch.zeros(4, 10, 6, 12)])[1]
    assert np.array_equal(host(y), ref)
    xh = host(x)
    assert np.array_equal(ref, np.transpose(xh, (0, 2, 1, 3)) ** 2)


def test_bf16_transpose_round_trip_bit_exact():
    # bf16 loads widen exactly to f32 and stores round back: a transpose moves bits unchanged
    x = torch.randn(2, 40, 70, generator=gen(14)).to(torch.bfloat16)
    y = torch.zeros(2, 70, 40, dtype=torch.bfloat16, device=DEV)
    m = xt.run(transpose3, args=(x.to(DEV), y, 16, 32), grid=(2, 3, 3))
    assert m.plan()["family"] == "tile"
    assert torch.equal(y.cpu(), x.transpose(1, 2))


@xt.kernel
def rank1_scale(x, y, t):
    i = xt.bid(0)
    v = xt.load(x, index=(i,), shape=(t,))
    xt.store(y, index=(i,), tile=v * v)


def test_rank1_ragged_stores_are_clipped():
    # 1000 elements in tiles of 96: the last tile runs past the end; nothing past it is written
    x = torch.randn(1000, generator=gen(12))
    y = torch.full((1000,), float("nan"), device=DEV)
    m = xt.run(rank1_scale, args=(x.to(DEV), y, 96), grid=(11, 1, 1))
    ref = oracle(m, [x, torch.zeros(1000)])[1]
    assert np.array_equal(host(y), ref)


def test_permute_general_path_rank3_ragged():
    text = """func.func @p(%x: memref<5x7x9xf32>, %y: memref<9x5x7xf32>) attributes {xt.grid = array<i32: 2, 1, 1>} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %t = xt.load(%x, %bid#0, %zero, %zero) : (memref<5x7x9xf32>, i32, i32, i32) -> tensor<3x7x9xf32>
  %u = xt.permute(%t) {permutation = [2, 0, 1]} : tensor<3x7x9xf32> -> tensor<9x3x7xf32>
  xt.store(%u, %y, %zero, %bid#0, %zero) : (tensor<9x3x7xf32>, memref<9x5x7xf32>, i32, i32, i32) -> ()
  func.return
}"""
    m = xt.parse(text)
    x = torch.randn(5, 7, 9, generator=gen(13))
    y = torch.full((9, 5, 7), float("nan"), device=DEV)
    xt.launch(m, x.to(DEV), y)
    ref = oracle(m, [x, torch.zeros(9, 5, 7)])[1]
    assert np.array_equal(host(y), ref)
    assert np.array_equal(ref, np.transpose(host(x), (2, 0, 1)))


# Grids of thousands of Blocks, with ragged edge tiles and bid0 shards: every
# CTA of the launch sees its own Block coordinates, tile starts past 2^16
# elements, and edge tiles clipped in rows and in float4 columns.

def test_large_grid_transpose_ragged_edges_bit_exact():
    # grid (6, 33, 16) = 3168 Blocks; the last row tile holds 8 of 16 rows
    # and the last column tile 20 of 32
    x = torch.randn(6, 520, 500, generator=gen(21))
    y = torch.full((6, 500, 520), float("nan"), device=DEV)
    m = xt.run(transpose3, args=(x.to(DEV), y, 16, 32), grid=(6, 33, 16))
    assert torch.equal(y.cpu(), x.transpose(1, 2))


def test_large_grid_transpose_bid0_shards_match_full_launch():
    # grid (160, 4, 4) launched whole and as the shards [0, 150) and [150, 160)
    x = torch.randn(160, 64, 128, generator=gen(22)).to(DEV)
    full = torch.empty(160, 128, 64, device=DEV)
    parts = torch.full((160, 128, 64), float("nan"), device=DEV)
    m = xt.run(transpose3, args=(x, full, 16, 32), grid=(160, 4, 4))
    assert torch.equal(full, x.transpose(1, 2))
    for lo, hi in [(0, 150), (150, 160)]:
        xt.launch(m, x, parts, bid0_range=(lo, hi))
    assert torch.equal(full, parts)


def test_large_grid_axis0_reductions():
    # 64 x 32 tiles over [4096, 1024]: grid (64, 32) = 2048 Blocks
    x = torch.randn(4096, 1024, generator=gen(23)) * 3
    s = torch.empty(64, 1024, device=DEV)
    mx = torch.empty(64, 1024, device=DEV)
    m = xt.run(col_stats, args=(x.to(DEV), s, mx, 64, 32), grid=(64, 32, 1))
    xr = x.view(64, 64, 1024).double()
    assert torch.equal(mx.cpu(), x.view(64, 64, 1024).amax(dim=1))
    ref = xr.sum(dim=1).float().numpy()
    got = host(s)
    assert np.all(np.abs(got - ref) <= 1e-6 * np.abs(ref) + 1e-6)


def test_large_grid_rank4_permute_general_path():
    # rank-4 tiles with a non-unit leading dim on a grid
    # of (40, 1, 80) = 3200 Blocks
    text = """func.func @r(%x: memref<80x6x320x12xf32>, %y: memref<80x320x6x12xf32>) attributes {xt.grid = array<i32: 40, 1, 80>} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %t = xt.load(%x, %bid#0, %zero, %bid#2, %zero) : (memref<80x6x320x12xf32>, i32, i32, i32, i32) -> tensor<2x6x4x12xf32>
  %p = xt.permute(%t) {permutation = [0, 2, 1, 3]} : tensor<2x6x4x12xf32> -> tensor<2x4x6x12xf32>
  %u = xt.mul(%p, %p) : tensor<2x4x6x12xf32>, tensor<2x4x6x12xf32> -> tensor<2x4x6x12xf32>
  xt.store(%u, %y, %bid#0, %bid#2, %zero, %zero) : (tensor<2x4x6x12xf32>, memref<80x320x6x12xf32>, i32, i32, i32, i32) -> ()
  func.return
}"""
    m = xt.parse(text)
    assert m.plan()["family"] == "tile"
    x = torch.randn(80, 6, 320, 12, generator=gen(24))
    y = torch.full((80, 320, 6, 12), float("nan"), device=DEV)
    xt.launch(m, x.to(DEV), y)
    assert torch.equal(y.cpu(), x.permute(0, 2, 1, 3) ** 2)


def test_permute_used_twice_and_permute_chains_bit_exact():
    # the transposed tile feeds a store and a multiply (not folded into the
    # store); a second program transposes twice (the first permute feeds the
    # second, which is folded into the store)
    from tests.test_tile import transpose_twice_used

    x = torch.randn(2, 96, 200, generator=gen(25))
    y = torch.full((2, 200, 96), float("nan"), device=DEV)
    z = torch.full((2, 200, 96), float("nan"), device=DEV)
    xt.run(transpose_twice_used, args=(x.to(DEV), y, z, 32, 64), grid=(2, 3, 4))
    xt_ = x.transpose(1, 2)
    assert torch.equal(y.cpu(), xt_)
    assert torch.equal(z.cpu(), xt_ * xt_)
    text = """func.func @pp(%x: memref<4x6x8xf32>, %y: memref<4x6x8xf32>) attributes {xt.grid = array<i32: 2, 1, 1>} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %t = xt.load(%x, %bid#0, %zero, %zero) : (memref<4x6x8xf32>, i32, i32, i32) -> tensor<2x6x8xf32>
  %u = xt.permute(%t) {permutation = [2, 0, 1]} : tensor<2x6x8xf32> -> tensor<8x2x6xf32>
  %v = xt.permute(%u) {permutation = [1, 2, 0]} : tensor<8x2x6xf32> -> tensor<2x6x8xf32>
  xt.store(%v, %y, %bid#0, %zero, %zero) : (tensor<2x6x8xf32>, memref<4x6x8xf32>, i32, i32, i32) -> ()
  func.return
}"""
    m = xt.parse(text)
    xs = torch.randn(4, 6, 8, generator=gen(26))
    ys = torch.full((4, 6, 8), float("nan"), device=DEV)
    xt.launch(m, xs.to(DEV), ys)
    assert torch.equal(ys.cpu(), xs)


@xt.kernel
def swap_tiles(x, y, tm, tn):
    i, j = xt.bid(0), xt.bid(1)
    xt.store(y, index=(j, i), tile=xt.load(x, index=(i, j), shape=(tm, tn)))


def test_tile_copy_to_swapped_coordinates_ragged():
    # a plain load + store (the data-movement path without a transpose): the
    # tile at (i, j) of x lands at (j, i) of y; edge tiles load zeros past x's
    # edge and are clipped at y's
    x = torch.randn(90, 188, generator=gen(27))
    y = torch.full((90, 188), float("nan"), device=DEV)
    m = xt.run(swap_tiles, args=(x.to(DEV), y, 16, 32), grid=(6, 6, 1))
    ref = oracle(m, [x, torch.full((90, 188), float("nan"))])[1]
    assert np.array_equal(host(y), ref, equal_nan=True)


@pytest.mark.parametrize("dtype,shape,tile", [
    (torch.bfloat16, (4, 64, 128), (32, 64)),
    (torch.bfloat16, (3, 104, 120), (16, 32)),   # ragged rows and columns (whole 16-byte vectors)
    (torch.int8, (2, 64, 192), (32, 64)),
    (torch.int8, (2, 80, 176), (32, 32)),        # ragged rows and columns
])
def test_data_movement_transpose_bf16_int8_bit_exact(dtype, shape, tile):
    # 16-byte vectors of 8 bf16 or 16 int8 elements; the values pass through
    # f32 in shared memory and come back bit for bit
    g = gen(28)
    if dtype == torch.int8:
        x = torch.randint(-128, 128, shape, generator=g, dtype=torch.int8)
    else:
        x = torch.randn(*shape, generator=g).to(dtype)
    y = torch.zeros(shape[0], shape[2], shape[1], dtype=dtype, device=DEV)
    tm, tn = tile
    grid = (shape[0], -(-shape[1] // tm), -(-shape[2] // tn))
    xt.run(transpose3, args=(x.to(DEV), y, tm, tn), grid=grid)
    assert torch.equal(y.cpu(), x.transpose(1, 2))


@xt.kernel
def row_stats_tiles(x, s, mx, tm, tn):
    i, j = xt.bid(0), xt.bid(1)
    t = xt.load(x, index=(i, j), shape=(tm, tn))
    xt.store(s, index=(i, j), tile=xt.sum(t, axis=1))
    xt.store(mx, index=(i, j), tile=xt.max(t, axis=1))


def test_tile_reductions_both_axes_with_nans():
    # 16 x 64 tiles reduced along each axis; a NaN in a column or row makes
    # its max NaN and its sum NaN, as in the oracle
    x = torch.randn(128, 256, generator=gen(30)) * 2
    x[5, 7] = float("nan")
    x[70, 200] = float("nan")
    s = torch.empty(128, 4, device=DEV)
    mx = torch.empty(128, 4, device=DEV)
    m = xt.run(row_stats_tiles, args=(x.to(DEV), s, mx, 16, 64), grid=(8, 4, 1))
    assert m.plan()["family"] == "tile"
    _, ref_s, ref_m = oracle(m, [x, torch.zeros(128, 4), torch.zeros(128, 4)])
    assert np.array_equal(host(mx), ref_m, equal_nan=True)
    got = host(s)
    assert np.array_equal(np.isnan(got), np.isnan(ref_s))
    ok = ~np.isnan(ref_s)
    assert np.all(np.abs(got[ok] - ref_s[ok]) <= 1e-6 * np.abs(ref_s[ok]) + 1e-6)
    cs = torch.empty(8, 256, device=DEV)
    cm = torch.empty(8, 256, device=DEV)
    m = xt.run(col_stats, args=(x.to(DEV), cs, cm, 16, 64), grid=(8, 4, 1))
    _, ref_s, ref_m = oracle(m, [x, torch.zeros(8, 256), torch.zeros(8, 256)])
    assert np.array_equal(host(cm), ref_m, equal_nan=True)
    got = host(cs)
    ok = ~np.isnan(ref_s)
    assert np.array_equal(np.isnan(got), ~ok)
    assert np.all(np.abs(got[ok] - ref_s[ok]) <= 1e-6 * np.abs(ref_s[ok]) + 1e-6)
