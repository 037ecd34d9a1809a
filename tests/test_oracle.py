"""The CPU oracle against the reference's known answers and independent math.

The reference holds no numeric golden vectors; what it does pin is the
structure the oracle restates:

* tile coordinate -> element start (``test/xt/to_nova.mlir:143-144``);
* conv halo slices and pads at interior / top-left / bottom-right tiles
  (``test/xt/to_nova.mlir:149-156``);
* serialize (grid walk) order (``test/xt/serialize.mlir:55-76``).

The numeric cases then check the interpreter against formulas written
independently here (numpy / torch), on small seeded inputs.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import xt_oracle as xo
from tests.golden.cases import build_cases
import xtile_b200.dsl as xt


def test_tile_start_pins():
    # to_nova.mlir:143-144: load (0, 2) and store (1, 2) of 16x16 tiles
    assert xo.tile_start((0, 2), (16, 16)) == (0, 32)
    assert xo.tile_start((1, 2), (16, 16)) == (16, 32)


@pytest.mark.parametrize("idx,start,size,pads", [
    # (h/w tile index) -> load start, load size, conv pad [top, left, bottom, right]
    ((1, 1), (31, 63), (34, 66), (0, 0, 0, 0)),   # to_nova.mlir:149-150
    ((0, 0), (0, 0), (33, 65), (1, 1, 0, 0)),     # to_nova.mlir:151-152
    ((2, 2), (63, 127), (33, 65), (0, 0, 1, 1)),  # to_nova.mlir:153-154
])
def test_conv_slice_pins(idx, start, size, pads):
    hs = xo.conv_spatial_slice(96, idx[0], 32, 3, 1, 1, 1)
    ws = xo.conv_spatial_slice(192, idx[1], 64, 3, 1, 1, 1)
    assert (hs[0], ws[0]) == start
    assert (hs[1], ws[1]) == size
    assert (hs[2], ws[2], hs[3], ws[3]) == pads


def test_serialize_order_pin():
    # serialize.mlir:55-76: (x, y) = (0,0), (1,0), (0,1), (1,1)
    assert xo.serialize_order((2, 2, 1)) == [(0, 0, 0), (1, 0, 0), (0, 1, 0), (1, 1, 0)]
    assert xo.serialize_order((2, 1, 2))[1] == (1, 0, 0)


def _text(name):
    for n, fn, args, grid, db in build_cases(xt):
        if n == name:
            return xt.trace_text(fn, args=args, grid=grid, double_buffering=db)
    raise KeyError(name)


def test_add_exact():
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (128, 128)).astype(np.float32)
    b = rng.uniform(-1, 1, (128, 128)).astype(np.float32)
    c = np.zeros_like(a)
    xo.run(_text("add_rows_128x128"), [a, b, c])
    assert np.array_equal(c.view(np.uint32), (a + b).view(np.uint32))


def test_softmax_matches_formula():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((128, 128)) * 4).astype(np.float32)
    y = np.zeros_like(x)
    xo.run(_text("softmax_128x128_row64"), [x, y])
    x64 = x.astype(np.float64)
    e = np.exp(x64 - x64.max(axis=1, keepdims=True))
    ref = e / e.sum(axis=1, keepdims=True)
    assert np.max(np.abs(y - ref) / ref) < 1e-5   # f32 rounding of x - max, then exp


def test_int8_matmul_epilogue():
    rng = np.random.default_rng(2)
    a = rng.integers(-128, 128, (128, 256), dtype=np.int8)
    b = rng.integers(-128, 128, (256, 128), dtype=np.int8)
    s = rng.uniform(0, 1e-4, (1, 128)).astype(np.float32)
    bias = rng.uniform(-8, 8, (1, 128)).astype(np.float32)
    c = np.zeros((128, 128), np.int8)
    xo.run(_text("matmul_i8_128x128x256"), [a, b, c, s, bias])
    acc = (a.astype(np.int64) @ b.astype(np.int64)).astype(np.float32)
    t = (acc * s).astype(np.float32) + bias
    ref = np.clip(np.rint(t), -128, 127).astype(np.int8)
    assert np.array_equal(c, ref)


def test_kloop_matmul():
    rng = np.random.default_rng(3)
    a = rng.standard_normal((512, 512)).astype(np.float32)
    b = rng.standard_normal((512, 512)).astype(np.float32)
    c = np.zeros((512, 512), np.float32)
    xo.run(_text("matmul_kloop_f32_512"), [a, b, c])
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert np.max(np.abs(c - ref)) / np.max(np.abs(ref)) < 1e-5


def test_conv_int8_matches_torch():
    rng = np.random.default_rng(4)
    x = rng.integers(-8, 8, (1, 32, 64, 128), dtype=np.int8)
    f = rng.integers(-8, 8, (3, 3, 128, 64), dtype=np.int8)
    y = np.zeros((1, 32, 64, 64), np.float32)
    xo.run(_text("conv2d_i8_1x32x64x128x64"), [x, f, y])
    xt_ = torch.from_numpy(x.astype(np.float64)).permute(0, 3, 1, 2)
    ft = torch.from_numpy(f.astype(np.float64)).permute(3, 2, 0, 1)
    ref = torch.nn.functional.conv2d(xt_, ft, padding=1).permute(0, 2, 3, 1).numpy()
    assert np.array_equal(y, ref.astype(np.float32))


def test_conv_tiled_edges_match_torch():
    # 56x56 image in 8x56 tiles: the bottom tiles' halo reaches past the image
    rng = np.random.default_rng(5)
    x = rng.integers(-4, 4, (32, 56, 56, 64), dtype=np.int8)
    f = rng.integers(-4, 4, (3, 3, 64, 64), dtype=np.int8)
    y = np.zeros((32, 56, 56, 64), np.float32)
    blocks = [(n, h, 0) for n in (0, 31) for h in range(7)]
    xo.run(_text("conv2d_i8_32x56x56x64_t8x56"), [x, f, y], blocks=blocks)
    xt_ = torch.from_numpy(x[[0, 31]].astype(np.float64)).permute(0, 3, 1, 2)
    ft = torch.from_numpy(f.astype(np.float64)).permute(3, 2, 0, 1)
    ref = torch.nn.functional.conv2d(xt_, ft, padding=1).permute(0, 2, 3, 1).numpy()
    assert np.array_equal(y[[0, 31]], ref.astype(np.float32))


def test_bf16_round_trip():
    x = np.array([1.0, -2.5, 3.14159, 1e-3, np.float32(1.00390625)], np.float32)
    bits = xo.f32_to_bf16(x)
    back = xo.bf16_to_f32(bits)
    ref = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(back, ref)


def test_ftoi_rounding():
    x = np.array([0.5, 1.5, 2.5, -0.5, -1.5, 126.6, 200.0, -300.0, np.nan], np.float32)
    assert xo.ftoi_i8(x).tolist() == [0, 2, 2, 0, -2, 127, 127, -128, 0]


def test_partial_tile_clips():
    # rows 0..99 in 64-row tiles: the second tile reaches past the edge
    @xt.kernel
    def add_rows(lhs, rhs, out, trow, col):
        i = xt.bid(0)
        xt.store(out, index=(i, 0), tile=xt.load(lhs, index=(i, 0), shape=(trow, col))
                 + xt.load(rhs, index=(i, 0), shape=(trow, col)))

    A = xt.Array
    text = xt.trace_text(add_rows, args=(A((100, 16), xt.float32), A((100, 16), xt.float32),
                                         A((100, 16), xt.float32), 64, 16),
                         grid=(2, 1, 1), double_buffering=True)
    a = np.ones((100, 16), np.float32)
    c = np.zeros_like(a)
    xo.run(text, [a, a, c])
    assert np.all(c == 2)


def test_lit_syntax_parses():
    text = """
    module {
      func.func @serialize_grid(%src: memref<128x16xf32>, %dst: memref<128x16xf32>) attributes {xt.grid = array<i32: 2, 2, 1>} {
        %bid0:3 = xt.get_tile_block_id : i32, i32, i32
        %bid1:3 = xt.get_tile_block_id : i32, i32, i32
        %0 = xt.load(%src, %bid0#0, %bid1#1) : (memref<128x16xf32>, i32, i32) -> tensor<16x16xf32>
        %1 = xt.exp(%0) : tensor<16x16xf32> -> tensor<16x16xf32>
        xt.store(%1, %dst, %bid1#0, %bid0#1) : (tensor<16x16xf32>, memref<128x16xf32>, i32, i32) -> ()
        func.return
      }
    }
    """
    src = np.random.default_rng(6).standard_normal((128, 16)).astype(np.float32)
    dst = np.zeros_like(src)
    xo.run(text, [src, dst])
    assert np.allclose(dst[:32], np.exp(src[:32]))
    assert np.all(dst[32:] == 0)


# --------------------------------------------------------------------------
# The product's C++ parse + print must not change a program.  The GPU parity
# tests feed the oracle the DSL's own text (``Module.source_text``) while the
# kernels run from the C++ parse of that text; these cases show that the two
# readings are the same program, op by op with every attribute, so a misread
# attribute in the C++ parser (a conv pad, a shared level, an epilogue
# constant) cannot hide behind a re-printed text.
# --------------------------------------------------------------------------
def _bf16_programs():
    A, bf, f32 = xt.Array, xt.bfloat16, xt.float32

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
    def conv2d_bf16(inp, filt, out, th, tw, cin, cout):
        n, h, w = xt.bid(0), xt.bid(1), xt.bid(2)
        f = xt.load(filt, index=(0, 0, 0, 0), shape=(3, 3, cin, cout), shared=2)
        y = xt.load_conv2d(inp, f, index=(n, h, w, 0), shape=(1, th, tw, cout), group=1,
                           pad=(1, 1, 1, 1), stride=(1, 1), dilation=(1, 1))
        xt.store(out, index=(n, h, w, 0), tile=y)

    return {
        "matmul_4096_bf16": xt.trace_text(
            matmul_kloop, args=(A((4096, 4096), bf), A((4096, 4096), bf), A((4096, 4096), f32), 128, 128, 64, 64),
            grid=(32, 32, 1), double_buffering=True),
        "sharded_matmul_bf16": xt.trace_text(
            matmul_kloop, args=(A((32768, 8192), bf), A((8192, 8192), bf), A((32768, 8192), f32), 256, 128,
                                8192, 1), grid=(128, 64, 1), double_buffering=True),
        "conv2d_bf16_32x56x56x64": xt.trace_text(
            conv2d_bf16, args=(A((32, 56, 56, 64), bf), A((3, 3, 64, 64), bf), A((32, 56, 56, 64), f32),
                               8, 56, 64, 64), grid=(32, 7, 1), double_buffering=True),
    }


def _roundtrip_cases():
    golden = Path(__file__).resolve().parent / "golden" / "dsl_text"
    cases = [(p.stem, p.read_text()) for p in sorted(golden.glob("*.mlir"))]
    return cases + sorted(_bf16_programs().items())


@pytest.mark.parametrize("name,text", _roundtrip_cases(), ids=[c[0] for c in _roundtrip_cases()])
def test_cpp_parse_print_preserves_program(name, text):
    import xtile_b200 as b200

    printed = b200._module_asm(b200.parse(text))
    want = xo.parse_module(text)
    got = xo.parse_module(printed)
    assert len(got) == len(want)
    for fg, fw in zip(got, want):
        assert (fg.name, fg.args, fg.grid) == (fw.name, fw.args, fw.grid)
        assert len(fg.ops) == len(fw.ops)
        for og, ow in zip(fg.ops, fw.ops):
            assert og == ow, f"{name}: {og} != {ow}"


def test_roundtrip_comparison_sees_a_changed_attribute():
    # a planted change in the oracle's input (a conv pad) must show up in the comparison
    text = _bf16_programs()["conv2d_bf16_32x56x56x64"]
    planted = text.replace("pad = array<i64: 1, 1, 1, 1>", "pad = array<i64: 1, 0, 1, 1>")
    assert planted != text
    assert xo.parse_module(planted) != xo.parse_module(text)


def test_module_source_text_is_the_dsl_text():
    import xtile_b200 as b200

    text = _bf16_programs()["matmul_4096_bf16"]
    m = b200.parse(text)
    b200.compile(m)  # stages change the printed module, never the source text
    assert m.source_text == text
    assert str(m) != text
