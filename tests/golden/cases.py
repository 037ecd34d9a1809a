"""Block programs whose xt text is pinned against the reference tracer.

``build_cases(xt)`` takes a DSL namespace -- either the reference tracer
(``xtile/dsl.py`` of sjjeong94/xtile, loaded in place by ``make_golden.py``)
or this repository's ``xtile_b200.dsl`` -- and returns
``[(name, kernel, args, grid, double_buffering), ...]``.

The programs are the four workload patterns of the reference (``kernels/add.py``,
``kernels/softmax.py``, ``kernels/matmul.py``, ``kernels/conv2d.py``) at the
shapes of the benchmark configurations where the reference dtypes allow it,
plus the cases of the reference's ``test/python/dsl_convert.py``.  Each kernel
body is written here from the published DSL surface, not copied.
"""
from __future__ import annotations


def build_cases(xt):
    cases = []

    def add_case(name, fn, args, grid, db=True):
        cases.append((name, fn, args, grid, db))

    f32, i8 = xt.float32, xt.int8
    A = xt.Array

    # --- elementwise add: row-slab tiles (kernels/add.py) and 32x64 tiles ---
    @xt.kernel
    def add_rows(lhs, rhs, out, trow, col):
        i = xt.bid(0)
        a = xt.load(lhs, index=(i, 0), shape=(trow, col))
        b = xt.load(rhs, index=(i, 0), shape=(trow, col))
        xt.store(out, index=(i, 0), tile=a + b)

    add_case("add_rows_128x128", add_rows,
             (A((128, 128), f32), A((128, 128), f32), A((128, 128), f32), 64, 128), (2, 1, 1))

    @xt.kernel
    def add_tiles(lhs, rhs, out, th, tw):
        i = xt.bid(0)
        j = xt.bid(1)
        a = xt.load(lhs, index=(i, j), shape=(th, tw))
        b = xt.load(rhs, index=(i, j), shape=(th, tw))
        xt.store(out, index=(i, j), tile=a + b)

    add_case("add_tiles_2048_32x64", add_tiles,
             (A((2048, 2048), f32), A((2048, 2048), f32), A((2048, 2048), f32), 32, 64),
             (64, 32, 1))

    # --- row softmax (kernels/softmax.py: max-subtract, exp, sum, divide) ---
    @xt.kernel
    def softmax_rows(inp, out, trow, col):
        i = xt.bid(0)
        x = xt.load(inp, index=(i, 0), shape=(trow, col))
        x = x - xt.max(x, axis=-1)
        x = xt.exp(x)
        s = xt.sum(x, axis=-1)
        x = x / s
        xt.store(out, index=(i, 0), tile=x)

    add_case("softmax_8192x1024_row1", softmax_rows,
             (A((8192, 1024), f32), A((8192, 1024), f32), 1, 1024), (8192, 1, 1))
    add_case("softmax_128x128_row64", softmax_rows,
             (A((128, 128), f32), A((128, 128), f32), 64, 128), (2, 1, 1))

    # --- int8 matmul with scale/bias and int8 result (kernels/matmul.py) ---
    @xt.kernel
    def matmul_i8(lhs, rhs, res, scale, bias, tm, tn, tk):
        i = xt.bid(0)
        j = xt.bid(1)
        a = xt.load(lhs, index=(i, 0), shape=(tm, tk))
        b = xt.load(rhs, index=(0, j), shape=(tk, tn), shared=1)
        s = xt.load(scale, index=(0, j), shape=(1, tn), shared=1)
        c = xt.load(bias, index=(0, j), shape=(1, tn), shared=1)
        t = xt.matmul(a, b)
        t = t * s + c
        t = xt.astype(t, dtype=xt.int8)
        xt.store(res, index=(i, j), tile=t)

    add_case("matmul_i8_128x128x256", matmul_i8,
             (A((128, 256), i8), A((256, 128), i8), A((128, 128), i8),
              A((1, 128), f32), A((1, 128), f32), 64, 64, 256), (2, 2, 1))
    add_case("matmul_i8_1024x512x256", matmul_i8,
             (A((1024, 256), i8), A((256, 512), i8), A((1024, 512), i8),
              A((1, 512), f32), A((1, 512), f32), 64, 64, 256), (16, 8, 1))

    # --- K-looped matmul (block tile 128x128, K-step 64); f32 here because the
    # reference DSL has no bfloat16 ---
    @xt.kernel
    def matmul_kloop(lhs, rhs, out, tm, tn, tk, ksteps):
        i = xt.bid(0)
        j = xt.bid(1)
        acc = None
        for k in range(ksteps):
            a = xt.load(lhs, index=(i, k), shape=(tm, tk))
            b = xt.load(rhs, index=(k, j), shape=(tk, tn))
            p = xt.matmul(a, b)
            acc = p if acc is None else acc + p
        xt.store(out, index=(i, j), tile=acc)

    add_case("matmul_kloop_f32_512", matmul_kloop,
             (A((512, 512), f32), A((512, 512), f32), A((512, 512), f32), 128, 128, 64, 8),
             (4, 4, 1))

    # --- int8 conv2d with a shared=2 filter (kernels/conv2d.py) ---
    @xt.kernel
    def conv2d_i8(inp, filt, out, tile_h, tile_w, cin, cout, kh, kw):
        n = xt.bid(0)
        h = xt.bid(1)
        w = xt.bid(2)
        f = xt.load(filt, index=(0, 0, 0, 0), shape=(kh, kw, cin, cout), shared=2)
        y = xt.load_conv2d(inp, f, index=(n, h, w, 0), shape=(1, tile_h, tile_w, cout),
                           group=1, pad=(kh // 2, kw // 2, kh // 2, kw // 2),
                           stride=(1, 1), dilation=(1, 1))
        xt.store(out, index=(n, h, w, 0), tile=y)

    add_case("conv2d_i8_1x32x64x128x64", conv2d_i8,
             (A((1, 32, 64, 128), i8), A((3, 3, 128, 64), i8), A((1, 32, 64, 64), f32),
              32, 64, 128, 64, 3, 3), (1, 1, 1))
    add_case("conv2d_i8_32x56x56x64_t8x56", conv2d_i8,
             (A((32, 56, 56, 64), i8), A((3, 3, 64, 64), i8), A((32, 56, 56, 64), f32),
              8, 56, 64, 64, 3, 3), (32, 7, 1))

    # --- the reference's dsl_convert.py cases ---
    @xt.kernel
    def rowwise_softmax(x, y):
        i = xt.bid(0)
        t = xt.load(x, index=(i, 0), shape=(64, 64))
        r = xt.max(t)
        t = t - r
        t = xt.exp(t)
        r = xt.sum(t)
        r = xt.reciprocal(r)
        t = t * r
        xt.store(y, index=(i, 0), tile=t)

    add_case("rowwise_softmax", rowwise_softmax,
             (A((128, 64), f32), A((128, 64), f32)), (2, 1, 1))

    @xt.kernel
    def divide_kernel(x, y, z):
        tile = xt.load(x, index=(0, 0), shape=(8, 8))
        denom = xt.load(y, index=(0, 0), shape=(8, 1))
        xt.store(z, index=(0, 0), tile=tile / denom)

    add_case("divide", divide_kernel, (A((8, 8), f32), A((8, 1), f32), A((8, 8), f32)),
             (1, 1, 1), False)

    @xt.kernel
    def unary_and_shape(x, y, z, t_in, t_out):
        tile = xt.load(x, index=(0, 0), shape=(8, 8))
        tile = xt.silu(xt.tanh(xt.sigmoid(xt.rsqrt(xt.sin(xt.cos(tile))))))
        xt.store(y, index=(0, 0), tile=tile)
        xt.store(z, index=(0, 0), tile=xt.reshape(tile, shape=(4, 16)))
        t3 = xt.transpose(xt.load(t_in, index=(0, 0, 0), shape=(2, 3, 4)))
        xt.store(t_out, index=(0, 0, 0), tile=t3)

    add_case("unary_and_shape", unary_and_shape,
             (A((8, 8), f32), A((8, 8), f32), A((4, 16), f32), A((2, 3, 4), f32),
              A((2, 4, 3), f32)), (1, 1, 1), False)

    @xt.kernel
    def compute_mma(a, b, acc_src, acc_dst):
        a_t = xt.load(a, index=(0, 0), shape=(16, 32))
        b_t = xt.load(b, index=(0, 0), shape=(32, 8))
        acc = xt.load(acc_src, index=(0, 0), shape=(16, 8))
        xt.store(acc_dst, index=(0, 0), tile=xt.mma(a_t, b_t, acc))

    add_case("mma", compute_mma,
             (A((16, 32), i8), A((32, 8), i8), A((16, 8), f32), A((16, 8), f32)), (1, 1, 1), False)

    @xt.kernel
    def column_reduce(x, y):
        tile = xt.load(x, index=(0, 0), shape=(8, 8))
        xt.store(y, index=(0, 0), tile=xt.sum(tile, axis=0))

    add_case("column_reduce", column_reduce, (A((8, 8), f32), A((1, 8), f32)), (1, 1, 1), False)

    # constants other than zero, an argument that is both loaded and stored,
    # an unused array argument and repeated value stems
    @xt.kernel
    def mixed(buf, other, unused, out):
        a = xt.load(buf, index=(1, 2), shape=(4, 4))
        b = xt.load(other, index=(3, 2), shape=(4, 4))
        c = (a + b) + (a - b)
        xt.store(buf, index=(0, 0), tile=c * c)
        xt.store(out, index=(2, 1), tile=xt.exp(c))

    add_case("mixed_args_constants", mixed,
             (A((16, 16), f32), A((16, 16), f32), A((4, 4), f32), A((16, 16), f32)), (1, 1, 1))

    return cases
