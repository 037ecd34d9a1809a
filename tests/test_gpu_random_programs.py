"""Seeded random Block programs against the CPU oracle, through the public API.

Each program loads two [R, C] f32 arrays in (tm, tn) tiles and a [1, C] row,
applies 2-5 random ops (unary sigmoid / tanh / sin / cos / exp of a bounded
value, binary + - * between tiles, with the broadcast row, or with a per-row
sum or max reduced from a tile) and stores one or two results.  Depending on
the ops and tiles the planner picks the ew, rows or tile family, so one set
of seeds covers the three kinds of generated kernel: register programs,
shared-memory slots with in-place reuse, broadcast rows, reductions and
partial tiles.
A program beyond every family's limits (live rows, tile count) is refused by
the planner and its seed skipped.  Tolerance: |gpu - ref| <= 1e-4 |ref| + 1e-4 (transcendentals within a few
ulp of numpy's float64 ones, sums in another order); a wrong index, slot or
lane would be off by O(1).

With ``wide``, 24 more seeds use full rows of 3000, 4097 or 8192 columns,
which row programs run one CTA per row.

A second generator (``random_tile_program``) aims at the tile family:
column and row broadcasts, reductions along either axis combined back by
broadcasting, and tiles ragged along the rows; it covers the generated tile
kernel's single-pass runs of elementwise ops, its reductions split over
threads and its slot reuse.
"""
import numpy as np
import pytest
import torch

import xtile as xt
from oracle import xt_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None

UNARY = [xt.sigmoid, xt.tanh, xt.sin, xt.cos]


def random_program(seed, wide=False):
    """``wide``: full rows of 3000, 4097 or 8192 columns (row programs too wide
    for a warp, which run one CTA per row)."""
    rng = np.random.default_rng(seed)
    R, C = [(64, 64), (96, 128), (128, 256), (40, 72)][rng.integers(4)]
    if wide:
        R, C = [(16, 3000), (8, 4097), (12, 8192)][rng.integers(3)]
    tn = C if (wide or rng.random() < 0.5) else C // 2
    tm = [1, 8, 16][rng.integers(3)] if tn == C else [8, 16][rng.integers(2)]
    ops = []
    for _ in range(int(rng.integers(2, 6))):
        r = rng.random()
        if r < 0.35:
            ops.append(("unary", int(rng.integers(len(UNARY))), bool(rng.random() < 0.3)))
        elif r < 0.7:
            ops.append(("binary", int(rng.integers(3)), int(rng.integers(3))))
        elif r < 0.85 and tn != C:
            # (full-row programs skip the broadcast row: with per-row reductions they are row programs)
            ops.append(("row", int(rng.integers(3)), 0))
        else:
            ops.append(("reduce", int(rng.integers(2)), int(rng.integers(3))))
    two_stores = bool(rng.random() < 0.4)

    full_rows = tn == C

    @xt.kernel
    def prog(x, y, v, out, out2, tm, tn):
        # full-row tiles are indexed (i, 0), as row programs index them
        i, j = xt.bid(0), (0 if full_rows else xt.bid(1))
        vals = [xt.load(x, index=(i, j), shape=(tm, tn)), xt.load(y, index=(i, j), shape=(tm, tn))]
        row = None
        for kind, a, b in ops:
            t = vals[-1]
            if kind == "unary":
                u = UNARY[a](t)
                vals.append(xt.exp(u) if b else u)
            elif kind == "binary":
                o = vals[-2] if len(vals) > 1 else t
                vals.append([t + o, t - o, t * o][a])
            elif kind == "row":
                if row is None:
                    row = xt.load(v, index=(0, j), shape=(1, tn))
                vals.append([t + row, t - row, t * row][a])
            else:
                s = xt.sum(t, axis=1) if a == 0 else xt.max(t, axis=1)
                vals.append([t + s, t - s, t * s][b])
        xt.store(out, index=(i, j), tile=vals[-1])
        if two_stores:
            xt.store(out2, index=(i, j), tile=vals[-2])
        else:
            xt.store(out2, index=(i, j), tile=vals[0])

    return prog, R, C, tm, tn


@pytest.mark.parametrize("seed,wide", [(s, False) for s in range(36)] + [(s, True) for s in range(24)])
def test_random_program_matches_oracle(seed, wide):
    prog, R, C, tm, tn = random_program(seed, wide)
    g = torch.Generator().manual_seed(100 + seed)
    x = torch.randn(R, C, generator=g)
    y = torch.randn(R, C, generator=g)
    v = torch.randn(1, C, generator=g)
    out = torch.full((R, C), float("nan"), device=DEV)
    out2 = torch.full((R, C), float("nan"), device=DEV)
    grid = (-(-R // tm), C // tn, 1)
    A, F = xt.Array, xt.float32
    m = xt.convert(prog, args=(A((R, C), F), A((R, C), F), A((1, C), F), A((R, C), F), A((R, C), F), tm, tn),
                   grid=grid, double_buffering=True)
    try:
        m.plan()
    except RuntimeError as e:  # beyond every family's limits (live rows, tile count): refused loudly
        pytest.skip(str(e)[:120])
    xt.launch(m, x.to(DEV), y.to(DEV), v.to(DEV), out, out2)
    refs = [np.zeros((R, C), np.float32), np.zeros((R, C), np.float32)]
    arrays = [x.numpy(), y.numpy(), v.numpy(), refs[0], refs[1]]
    xt_oracle.run(m.source_text, arrays)
    # A row sum of C values of magnitude up to 1 can reach C; summed in
    # another order than the oracle's it moves by a few ulps of C, and a
    # later subtraction that cancels back to values of order 1 (t - sum,
    # then minus the row max) keeps that absolute error: wide rows add four
    # ulps of C (about 1e-3 at 4097 columns) to the absolute bar.
    atol = 1e-4 + (4 * float(np.spacing(np.float32(C))) if wide else 0.0)
    for got, ref in ((out, arrays[3]), (out2, arrays[4])):
        got = got.cpu().numpy()
        assert np.all(np.isfinite(got) == np.isfinite(ref)), m.plan()["family"]
        ok = np.isfinite(ref)
        assert np.all(np.abs(got[ok] - ref[ok]) <= 1e-4 * np.abs(ref[ok]) + atol), m.plan()["family"]
    assert xt.device_error() == 0


def random_tile_program(seed):
    """A seeded Block program for the tile family: (tm, tn) tiles of [R, C]
    arrays (ragged along the rows for R = 40), 2-6 ops among unary ops,
    binaries between the last two values, a (tm, 1) column or (1, tn) row
    broadcast, and reductions along axis 0 or 1 combined back by
    broadcasting (2-4 ops: a program holds at most 16 tiles); one or two
    stores."""
    rng = np.random.default_rng(1000 + seed)
    R, C = [(64, 64), (96, 128), (128, 256), (40, 72)][rng.integers(4)]
    tn = [C, C // 2, C // 4][rng.integers(3)]
    tm = [8, 16, 32][rng.integers(3)]
    ops = []
    for _ in range(int(rng.integers(2, 5))):
        r = rng.random()
        if r < 0.25:
            ops.append(("unary", int(rng.integers(len(UNARY)))))
        elif r < 0.45:
            ops.append(("binary", int(rng.integers(3))))
        elif r < 0.6:
            ops.append(("col", int(rng.integers(3))))
        elif r < 0.7:
            ops.append(("row", int(rng.integers(3))))
        else:
            ops.append(("reduce", int(rng.integers(2)), int(rng.integers(2)), int(rng.integers(3))))
    two_stores = bool(rng.random() < 0.5)

    @xt.kernel
    def prog(x, y, v, col, out, out2, tm, tn):
        i, j = xt.bid(0), xt.bid(1)
        vals = [xt.load(x, index=(i, j), shape=(tm, tn)), xt.load(y, index=(i, j), shape=(tm, tn))]
        c = r = None  # the column and row, loaded once
        for op in ops:
            t = vals[-1]
            if op[0] == "unary":
                vals.append(UNARY[op[1]](t))
            elif op[0] == "binary":
                o = vals[-2]
                vals.append([t + o, t - o, t * o][op[1]])
            elif op[0] == "col":
                if c is None:
                    c = xt.load(col, index=(i, 0), shape=(tm, 1))
                vals.append([t + c, t - c, t * c][op[1]])
            elif op[0] == "row":
                if r is None:
                    r = xt.load(v, index=(0, j), shape=(1, tn))
                vals.append([t + r, t - r, t * r][op[1]])
            else:
                _, axis, fn, comb = op
                s = xt.sum(t, axis=axis) if fn == 0 else xt.max(t, axis=axis)
                vals.append([t + s, t - s, t * s][comb])
        xt.store(out, index=(i, j), tile=vals[-1])
        xt.store(out2, index=(i, j), tile=vals[-2] if two_stores else vals[0])

    return prog, R, C, tm, tn


def tile_program_module(seed):
    prog, R, C, tm, tn = random_tile_program(seed)
    A, F = xt.Array, xt.float32
    m = xt.convert(prog, args=(A((R, C), F), A((R, C), F), A((1, C), F), A((R, 1), F), A((R, C), F), A((R, C), F),
                               tm, tn), grid=(-(-R // tm), C // tn, 1), double_buffering=True)
    return m, R, C


@pytest.mark.parametrize("seed", range(48))
def test_random_tile_program_matches_oracle(seed):
    m, R, C = tile_program_module(seed)
    try:
        m.plan()
    except RuntimeError as e:  # beyond every family's limits: refused loudly
        pytest.skip(str(e)[:120])
    g = torch.Generator().manual_seed(2000 + seed)
    x = torch.randn(R, C, generator=g)
    y = torch.randn(R, C, generator=g)
    v = torch.randn(1, C, generator=g)
    col = torch.randn(R, 1, generator=g)
    out = torch.full((R, C), float("nan"), device=DEV)
    out2 = torch.full((R, C), float("nan"), device=DEV)
    xt.launch(m, x.to(DEV), y.to(DEV), v.to(DEV), col.to(DEV), out, out2)
    arrays = [x.numpy(), y.numpy(), v.numpy(), col.numpy(), np.zeros((R, C), np.float32), np.zeros((R, C), np.float32)]
    xt_oracle.run(m.source_text, arrays)
    for got, ref in ((out, arrays[4]), (out2, arrays[5])):
        got = got.cpu().numpy()
        assert np.all(np.isfinite(got) == np.isfinite(ref)), m.plan()["family"]
        ok = np.isfinite(ref)
        assert np.all(np.abs(got[ok] - ref[ok]) <= 1e-4 * np.abs(ref[ok]) + 1e-4), m.plan()["family"]
    assert xt.device_error() == 0
