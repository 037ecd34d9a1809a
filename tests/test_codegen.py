"""The per-program kernels of the ew, rows and tile families, generated and
compiled for sm_100a on the CPU (NVRTC needs no GPU).

Every elementwise, row or tile program among the 36 seeded random programs
of the GPU parity test, row programs of several widths, the tile programs of
the tile GPU tests and programs with bf16 / int8 arrays and casts must
produce source that NVRTC compiles for sm_100a.  What the kernels compute is
checked on a GPU against the oracle (``tests/test_gpu_random_programs.py``,
``tests/test_gpu_kernels.py``, ``tests/test_gpu_tile.py``).
"""
import pytest

import xtile as xt
from tests.test_gpu_random_programs import random_program, tile_program_module
from xtile_b200._native import native

A = xt.Array


def generated(mod):
    return native.generated_source(mod._CAPIPtr)


def compiles(mod):
    return native.compile_generated(generated(mod)) > 0


@pytest.mark.parametrize("seed,wide", [(s, False) for s in range(36)] + [(s, True) for s in range(24)])
def test_random_program_compiles(seed, wide):
    prog, R, C, tm, tn = random_program(seed, wide)
    F = xt.float32
    m = xt.convert(prog, args=(A((R, C), F), A((R, C), F), A((1, C), F), A((R, C), F), A((R, C), F), tm, tn),
                   grid=(-(-R // tm), C // tn, 1), double_buffering=True)
    try:
        fam = m.plan()["family"]
    except RuntimeError:
        pytest.skip("beyond every family's limits")
    if fam not in ("ew", "rows", "tile"):
        with pytest.raises(RuntimeError, match="runs a compiled kernel"):
            generated(m)
        return
    src = generated(m)
    assert "switch" not in src.split("xt_warp_sum")[-1]  # straight-line code: nothing dispatched per element
    assert compiles(m)


@xt.kernel
def casts(x, y, out, out2, trow, col):
    i = xt.bid(0)
    a = xt.load(x, index=(i, 0), shape=(trow, col))
    b = xt.load(y, index=(i, 0), shape=(trow, col))
    t = xt.astype(a, dtype=xt.float32) * b
    xt.store(out, index=(i, 0), tile=xt.astype(t, dtype=xt.int8))
    xt.store(out2, index=(i, 0), tile=xt.silu(t))


@xt.kernel
def bf16_copy(x, out, trow, col):
    # bf16 tiles are moved, not computed on, in elementwise programs
    i = xt.bid(0)
    xt.store(out, index=(i, 0), tile=xt.load(x, index=(i, 0), shape=(trow, col)))


def test_int8_and_bf16_programs_compile():
    m = xt.convert(casts, args=(A((64, 48), xt.int8), A((64, 48), xt.float32), A((64, 48), xt.int8),
                                A((64, 48), xt.float32), 16, 48), grid=(4, 1, 1))
    assert m.plan()["family"] == "ew"
    src = generated(m)
    for fn in ("xt_ld4_i8", "xt_st4_i8", "xt_itof", "xt_ftoi", "xt_silu"):
        assert fn in src
    assert compiles(m)
    B = xt.bfloat16
    m = xt.convert(bf16_copy, args=(A((64, 48), B), A((64, 48), B), 16, 48), grid=(4, 1, 1))
    assert m.plan()["family"] == "ew"
    src = generated(m)
    assert "xt_ld4_bf16" in src and "xt_st4_bf16" in src
    assert compiles(m)


@xt.kernel
def row_stats(x, s, y, trow, col):
    i = xt.bid(0)
    t = xt.load(x, index=(i, 0), shape=(trow, col))
    c = xt.load(s, index=(i, 0), shape=(trow, 1))
    m = xt.max(t, axis=1) * c
    xt.store(y, index=(i, 0), tile=xt.exp(t - m) * xt.reciprocal(xt.sum(t, axis=1)))


@pytest.mark.parametrize("cols", [16, 37, 1024, 2048, 3000, 8192, 16384])
def test_row_programs_compile_for_any_width(cols):
    # up to 2048 columns one warp per row; wider rows one CTA per row
    F = xt.float32
    m = xt.convert(row_stats, args=(A((64, cols), F), A((64, 1), F), A((64, cols), F), 2, cols), grid=(32, 1, 1))
    assert m.plan()["family"] == "rows"
    src = generated(m)
    kernels = ("xt_rows_v", "xt_rows_s") if cols <= 2048 else ("xt_rows_cv", "xt_rows_cs", "xt_cta_max")
    assert f"#define XT_COLS {cols}" in src and all(k in src for k in kernels)
    assert compiles(m)


def test_row_programs_beyond_a_cta_are_refused_loudly():
    # two live rows of 32768 columns exceed a CTA's registers (1024 threads,
    # 32 values each) and their tiles exceed 192 KiB of shared memory: the
    # planner refuses the program with both reasons
    F = xt.float32
    m = xt.convert(row_stats, args=(A((64, 32768), F), A((64, 1), F), A((64, 32768), F), 2, 32768), grid=(32, 1, 1))
    with pytest.raises(RuntimeError, match="exceed a CTA's registers"):
        m.plan()


def test_wide_softmax_runs_a_generated_kernel():
    @xt.kernel
    def softmax_rows(inp, out, trow, col):
        i = xt.bid(0)
        x = xt.load(inp, index=(i, 0), shape=(trow, col))
        x = x - xt.max(x, axis=-1)
        x = xt.exp(x)
        xt.store(out, index=(i, 0), tile=x / xt.sum(x, axis=-1))

    F = xt.float32
    m = xt.convert(softmax_rows, args=(A((64, 32768), F), A((64, 32768), F), 1, 32768), grid=(64, 1, 1))
    assert m.plan()["family"] == "rows"
    src = generated(m)
    assert "#define XT_TPR 1024" in src and "xt_cta_sum" in src
    assert compiles(m)


def test_softmax_keeps_its_dedicated_kernel():
    @xt.kernel
    def softmax_rows(inp, out, trow, col):
        i = xt.bid(0)
        x = xt.load(inp, index=(i, 0), shape=(trow, col))
        x = x - xt.max(x, axis=-1)
        x = xt.exp(x)
        xt.store(out, index=(i, 0), tile=x / xt.sum(x, axis=-1))

    F = xt.float32
    m = xt.convert(softmax_rows, args=(A((64, 1024), F), A((64, 1024), F), 1, 1024), grid=(64, 1, 1))
    with pytest.raises(RuntimeError, match="runs a compiled kernel"):
        generated(m)


def test_compile_errors_carry_the_log():
    with pytest.raises(RuntimeError, match="(?s)NVRTC failed.*not_a_function.*undefined"):
        native.compile_generated("extern \"C\" __global__ void k() { not_a_function(); }")


import tests.test_gpu_tile as tile_cases  # noqa: E402

RANK4_PERMUTE = """func.func @r(%x: memref<4x6x10x12xf32>, %y: memref<4x10x6x12xf32>) attributes {xt.grid = array<i32: 2, 1, 2>} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %t = xt.load(%x, %bid#0, %zero, %bid#2, %zero) : (memref<4x6x10x12xf32>, i32, i32, i32, i32) -> tensor<2x6x5x12xf32>
  %p = xt.permute(%t) {permutation = [0, 2, 1, 3]} : tensor<2x6x5x12xf32> -> tensor<2x5x6x12xf32>
  %u = xt.mul(%p, %p) : tensor<2x5x6x12xf32>, tensor<2x5x6x12xf32> -> tensor<2x5x6x12xf32>
  xt.store(%u, %y, %bid#0, %bid#2, %zero, %zero) : (tensor<2x5x6x12xf32>, memref<4x10x6x12xf32>, i32, i32, i32, i32) -> ()
  func.return
}"""


@pytest.mark.parametrize("case", ["col_stats", "col_vector_ops", "wide", "i8_wrap", "row_stats_tiles", "rank4"])
def test_tile_programs_compile(case):
    F, I8 = xt.float32, xt.int8
    if case == "col_stats":
        # column sums and maxima: 64 x 32 tiles, 128-thread CTAs, float4
        # loads into unpadded rows, each column's 64 rows split over four
        # threads
        m = xt.convert(tile_cases.col_stats, args=(A((16384, 2048), F), A((256, 2048), F), A((256, 2048), F), 64, 32),
                       grid=(256, 64, 1))
        want = ("xt_ld4_f32_kept", "xt_st4_f32", "static_cast<double>", "__launch_bounds__(128)", "xt_red_f64[part",
                "*reinterpret_cast<float4*>(xt_sm + 0 + q * 32 + c) = v[u]")
    elif case == "col_vector_ops":
        m = xt.convert(tile_cases.col_vector_ops, args=(A((96, 1024), F), A((96, 1), F), A((96, 1024), F), 8, 512),
                       grid=(12, 2, 1))
        want = ("xt_sigmoid", "__launch_bounds__(128)")  # 4096-element tiles
    elif case == "wide":
        # 8192-element tiles: 256-thread CTAs
        m = xt.convert(tile_cases.col_vector_ops, args=(A((96, 1024), F), A((96, 1), F), A((96, 1024), F), 16, 512),
                       grid=(6, 2, 1))
        want = ("__launch_bounds__(256)",)
    elif case == "i8_wrap":
        m = xt.convert(tile_cases.i8_wrap, args=(A((64, 96), I8), A((1, 96), I8), A((64, 96), I8), 32, 48),
                       grid=(2, 2, 1))
        want = ("xt_wrap_i8", "xt_ld4_i8", "xt_st4_i8")
    elif case == "row_stats_tiles":
        # a ragged edge along both dims: limits computed per Block
        m = xt.convert(tile_cases.row_stats_tiles, args=(A((100, 70), F), A((100, 3), F), A((100, 3), F), 32, 32),
                       grid=(4, 3, 1))
        want = ("const int l", "xt_max_nan")
    else:
        # rank-4 tiles with leading dims above 1: rows unravel into (i0, i1, i2)
        m = xt.parse(RANK4_PERMUTE)
        want = ("xt_ld1_f32", "i0 = q / 30", "xt_mul")
    assert m.plan()["family"] == "tile"
    src = generated(m)
    for w in want:
        assert w in src, w
    assert "switch" not in src.split("xt_warp_sum")[-1]
    assert compiles(m)


@pytest.mark.parametrize("seed", range(48))
def test_random_tile_program_compiles(seed):
    m, _, _ = tile_program_module(seed)
    try:
        fam = m.plan()["family"]
    except RuntimeError:
        pytest.skip("beyond every family's limits")
    if fam not in ("ew", "rows", "tile"):
        pytest.skip(f"runs the compiled {fam} kernel")
    assert compiles(m)


def test_elementwise_ops_share_one_pass():
    # load, load, (t * c - c), sigmoid, store: the three elementwise ops run
    # as one pass with their intermediate results in registers, four columns
    # (a float4) per step; the two loads need no barrier between them: two
    # barriers in all
    F = xt.float32
    m = xt.convert(tile_cases.col_vector_ops, args=(A((16384, 2048), F), A((16384, 1), F), A((16384, 2048), F), 32, 64),
                   grid=(512, 32, 1))
    body = generated(m).split("template <bool V>")[1]
    assert "ops 2-4: one pass, 4 columns per step" in body
    assert body.count("__syncthreads") == 2
    assert compiles(m)
