"""The per-program kernels of the ew and rows families, generated and compiled
for sm_100a on the CPU (NVRTC needs no GPU).

Every elementwise or row program among the 36 seeded random programs of the
GPU parity test, row programs of several widths and programs with
bf16 / int8 arrays and casts must produce source that NVRTC compiles for
sm_100a.  What the kernels compute is checked on a GPU against the oracle
(``tests/test_gpu_random_programs.py``, ``tests/test_gpu_kernels.py``).
"""
import pytest

import xtile as xt
from tests.test_gpu_random_programs import random_program
from xtile_b200._native import native

A = xt.Array


def generated(mod):
    return native.generated_source(mod._CAPIPtr)


def compiles(mod):
    return native.compile_generated(generated(mod)) > 0


@pytest.mark.parametrize("seed", range(36))
def test_random_program_compiles(seed):
    prog, R, C, tm, tn = random_program(seed)
    F = xt.float32
    m = xt.convert(prog, args=(A((R, C), F), A((R, C), F), A((1, C), F), A((R, C), F), A((R, C), F), tm, tn),
                   grid=(-(-R // tm), C // tn, 1), double_buffering=True)
    try:
        fam = m.plan()["family"]
    except RuntimeError:
        pytest.skip("beyond every family's limits")
    if fam not in ("ew", "rows"):
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


@pytest.mark.parametrize("cols", [16, 37, 1024, 2048])
def test_row_programs_compile_for_any_width(cols):
    F = xt.float32
    m = xt.convert(row_stats, args=(A((64, cols), F), A((64, 1), F), A((64, cols), F), 2, cols), grid=(32, 1, 1))
    assert m.plan()["family"] == "rows"
    src = generated(m)
    assert f"#define XT_COLS {cols}" in src and "xt_rows_v" in src and "xt_rows_s" in src
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
