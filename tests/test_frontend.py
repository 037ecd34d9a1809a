"""Parser, verifier, stage dumps and planner of the native front end (CPU).

The verifier cases restate the reference's ``test/xt/invalid.mlir`` (one
program per ``// -----`` split, each expecting the reference's diagnostic) and
``test/xt/serialize_invalid.mlir``; the serialize cases restate the order and
``shared`` reuse pinned by ``test/xt/serialize.mlir:55-127`` and the checks of
``test/python/serialize.py``; the stage-object identity checks follow
``test/python/dsl_convert.py:45-47`` and ``test/python/compile.py:33-35``.
"""
import re

import pytest

import xtile as xt
import xtile_b200.dsl as dsl
from tests.golden.cases import build_cases

INVALID = [
    ("func.func @f(%a: memref<2048xf32>) {\n %z = arith.constant 0 : i32\n"
     " %0 = xt.load(%a, %z, %z) : (memref<2048xf32>, i32, i32) -> tensor<16xf32>\n func.return\n}",
     "coordinate count must match tensor rank"),
    ("func.func @f(%a: memref<2048x16xf32>) {\n %z = arith.constant 0 : i32\n"
     " %0 = xt.load(%a, %z, %z) : (memref<2048x16xf32>, i32, i32) -> tensor<16x16xi32>\n func.return\n}",
     "requires matching memref/tensor element types"),
    ("func.func @f(%a: tensor<16x32xf32>, %b: tensor<16x8xf32>) {\n"
     " %0 = xt.matmul(%a, %b) : tensor<16x32xf32>, tensor<16x8xf32> -> tensor<16x8xf32>\n func.return\n}",
     "matmul requires lhs inner dimension to match rhs outer dimension"),
    ("func.func @f(%a: tensor<16x32xf32>, %b: tensor<32x8xi8>, %c: tensor<16x8xf32>) {\n"
     " %0 = xt.mma(%a, %b, %c) : tensor<16x32xf32>, tensor<32x8xi8>, tensor<16x8xf32> -> tensor<16x8xf32>\n"
     " func.return\n}", "mma requires i8 input tensors"),
    ("func.func @f(%a: tensor<16x32xi8>, %b: tensor<32x8xi8>, %c: tensor<16x8xi32>) {\n"
     " %0 = xt.mma(%a, %b, %c) : tensor<16x32xi8>, tensor<32x8xi8>, tensor<16x8xi32> -> tensor<16x8xi32>\n"
     " func.return\n}", "mma requires f32 or bf16 accumulator and result tensors"),
    ("func.func @f(%a: memref<256x512xi8>) {\n %z = arith.constant 0 : i32\n"
     " %0 = xt.load(%a, %z, %z) {shared = 3 : i64} : (memref<256x512xi8>, i32, i32) -> tensor<256x64xi8>\n"
     " func.return\n}", "shared attribute must be 0, 1, or 2"),
    ("func.func @f(%a: tensor<16x16xf32>, %b: tensor<8x16xf32>) -> tensor<16x16xf32> {\n"
     " %0 = xt.add(%a, %b) : tensor<16x16xf32>, tensor<8x16xf32> -> tensor<16x16xf32>\n"
     " func.return %0 : tensor<16x16xf32>\n}", "operands are not broadcast-compatible with result tensor type"),
    ("func.func @f(%a: memref<1x34x66x128xi8>, %b: tensor<3x3x64x64xi8>) -> tensor<1x32x64x32xf32> {\n"
     " %c0 = arith.constant 0 : i32\n"
     " %0 = xt.load_conv2d(%a, %b, %c0, %c0, %c0, %c0) {dilation = array<i64: 1, 1>, group = 1 : i64, "
     "pad = array<i64: 1, 1, 1, 1>, stride = array<i64: 1, 1>} : (memref<1x34x66x128xi8>, "
     "tensor<3x3x64x64xi8>, i32, i32, i32, i32) -> tensor<1x32x64x32xf32>\n"
     " func.return %0 : tensor<1x32x64x32xf32>\n}",
     "load_conv2d requires source and filter channel dimensions to match"),
    ("func.func @f(%a: memref<1x34x66x128xi8>, %b: tensor<3x3x128x64xi8>) -> tensor<1x32x64x32xf32> {\n"
     " %c0 = arith.constant 0 : i32\n"
     " %0 = xt.load_conv2d(%a, %b, %c0, %c0, %c0, %c0) {dilation = array<i64: 1, 1>, group = 0 : i64, "
     "pad = array<i64: 1, 1, 1, 1>, stride = array<i64: 1, 1>} : (memref<1x34x66x128xi8>, "
     "tensor<3x3x128x64xi8>, i32, i32, i32, i32) -> tensor<1x32x64x32xf32>\n"
     " func.return %0 : tensor<1x32x64x32xf32>\n}", "group attribute must be positive"),
    ("func.func @f(%a: tensor<16x16xf32>) -> tensor<8x1xf32> {\n"
     " %0 = xt.reduce_sum(%a) {axis = 1 : i64} : tensor<16x16xf32> -> tensor<8x1xf32>\n"
     " func.return %0 : tensor<8x1xf32>\n}",
     "reduce result shape must match input shape except for the reduced dimension, which must be 1"),
    ("func.func @f(%a: tensor<16x16xf32>) -> tensor<16x1xf32> {\n"
     " %0 = xt.reduce_sum(%a) {axis = 2 : i64} : tensor<16x16xf32> -> tensor<16x1xf32>\n"
     " func.return %0 : tensor<16x1xf32>\n}", r"axis must be in range \[-rank, rank\)"),
    ("func.func @f(%a: tensor<64x16xf32>) -> tensor<2x16x16xf32> {\n"
     " %0 = xt.reshape(%a) : tensor<64x16xf32> -> tensor<2x16x16xf32>\n"
     " func.return %0 : tensor<2x16x16xf32>\n}",
     "reshape requires operand and result to have the same number of elements"),
    ("func.func @f(%a: tensor<2x32x16xf32>) -> tensor<2x32x16xf32> {\n"
     " %0 = xt.transpose(%a) : tensor<2x32x16xf32> -> tensor<2x32x16xf32>\n"
     " func.return %0 : tensor<2x32x16xf32>\n}", "transpose result shape must preserve dim 0 and swap dims 1 and 2"),
    ("func.func @f(%a: tensor<2x3x5xf32>) -> tensor<2x5x3xf32> {\n"
     " %0 = xt.permute(%a) {permutation = [2, 0, 1]} : tensor<2x3x5xf32> -> tensor<2x5x3xf32>\n"
     " func.return %0 : tensor<2x5x3xf32>\n}",
     "permute result shape must match the input shape reordered by permutation"),
    ("func.func @f(%a: tensor<2x3x5xf32>) -> tensor<5x2x3xf32> {\n"
     " %0 = xt.permute(%a) {permutation = [2, 0, 0]} : tensor<2x3x5xf32> -> tensor<5x2x3xf32>\n"
     " func.return %0 : tensor<5x2x3xf32>\n}", "permutation attribute must contain each dimension exactly once"),
    ("func.func @f() attributes {xt.grid = array<i32: 32, 8>} {\n func.return\n}",
     "xt.grid must have exactly 3 entries"),
    ("module attributes {xt.grid = array<i32: 1, 1, 1>} {\n}", "xt.grid is only valid on func.func operations"),
    ("func.func @f(%a: tensor<5x16xf32>) {\n %0 = xt.itof(%a) : tensor<5x16xf32> -> tensor<5x16xf32>\n"
     " func.return\n}", "'xt.itof' op requires integer input and floating-point result element types"),
    ("func.func @f(%a: tensor<5x16xi8>) {\n %0 = xt.ftoi(%a) : tensor<5x16xi8> -> tensor<5x16xi8>\n"
     " func.return\n}", "'xt.ftoi' op requires floating-point input and integer result element types"),
    ("func.func @f(%a: tensor<16x16xf32>) {\n xt.free(%a) : tensor<16x16xf32>\n func.return\n}",
     "custom op 'xt.free' is unknown"),
]


@pytest.mark.parametrize("text,message", INVALID, ids=[m[:40] for _, m in INVALID])
def test_invalid_programs_are_rejected(text, message):
    with pytest.raises(ValueError, match="failed to parse test module") as info:
        xt.parse(text)
    assert re.search(message, str(info.value)), str(info.value)


def test_valid_lit_syntax_round_trips():
    text = """
    module {
      func.func @generic_tile_ops(%arg0: memref<2048x16xf32>, %arg1: memref<2048x16xf32>) {
        %bid:3 = xt.get_tile_block_id : i32, i32, i32
        %zero = arith.constant 0 : i32
        %0 = xt.load(%arg0, %bid#0, %zero) : (memref<2048x16xf32>, i32, i32) -> tensor<16x16xf32>
        %1 = xt.exp(%0) : tensor<16x16xf32> -> tensor<16x16xf32>
        %2 = xt.add(%1, %1) : tensor<16x16xf32>, tensor<16x16xf32> -> tensor<16x16xf32>
        xt.store(%2, %arg1, %bid#0, %zero) : (tensor<16x16xf32>, memref<2048x16xf32>, i32, i32) -> ()
        func.return
      }
      func.func @generic_permute(%arg0: tensor<2x3x5xf32>) -> tensor<5x2x3xf32> {
        %0 = xt.permute(%arg0) {permutation = [2, 0, 1]} : tensor<2x3x5xf32> -> tensor<5x2x3xf32>
        func.return %0 : tensor<5x2x3xf32>
      }
      func.func @kernel_with_grid() attributes {xt.grid = array<i32: 32, 8, 1>} {
        func.return
      }
    }
    """
    m = xt.parse(text)
    printed = xt._module_asm(m)
    assert "xt.permute(%arg0) {permutation = [2, 0, 1]}" in printed
    assert "func.func @kernel_with_grid() attributes {xt.grid = array<i32: 32, 8, 1>}" in printed
    again = xt._module_asm(xt.parse(printed))
    assert again == printed
    assert m.func_names() == ["generic_tile_ops", "generic_permute", "kernel_with_grid"]


SERIALIZE_SRC = """
module {
  func.func @serialize_shared_x(%src: memref<128x16xf32>, %dst: memref<128x16xf32>) attributes {xt.grid = array<i32: 2, 2, 1>} {
    %bid:3 = xt.get_tile_block_id : i32, i32, i32
    %0 = xt.load(%src, %bid#0, %bid#1) {shared = 1 : i64} : (memref<128x16xf32>, i32, i32) -> tensor<16x16xf32>
    xt.store(%0, %dst, %bid#0, %bid#1) : (tensor<16x16xf32>, memref<128x16xf32>, i32, i32) -> ()
    func.return
  }
}
"""


def test_serialize_unrolls_with_reference_reuse():
    # serialize.mlir:78-84: one load per y value, reused by both x blocks
    m = xt.parse(SERIALIZE_SRC)
    assert xt.xt_serialize(m) is m
    text = xt._module_asm(m)
    assert "xt.get_tile_block_id" not in text
    loads = [ln for ln in text.splitlines() if "xt.load(" in ln]
    stores = [ln for ln in text.splitlines() if "xt.store(" in ln]
    assert len(loads) == 2 and len(stores) == 4
    first = loads[0].split("=")[0].strip()
    assert stores[0].startswith(f"    xt.store({first},") and stores[1].startswith(f"    xt.store({first},")


def test_serialize_grid_order():
    # serialize.mlir:55-76: blocks (x, y) in order (0,0) (1,0) (0,1) (1,1)
    src = SERIALIZE_SRC.replace(" {shared = 1 : i64}", "")
    m = xt.parse(src)
    xt.xt_serialize(m)
    consts = re.findall(r"arith.constant (\d+) : i32", xt._module_asm(m))
    assert [tuple(map(int, consts[i:i + 3])) for i in range(0, 12, 3)] == [
        (0, 0, 0), (1, 0, 0), (0, 1, 0), (1, 1, 0)]
    assert len(re.findall("arith.constant 0 : i32", xt._module_asm(m))) >= 2


@pytest.mark.parametrize("text,message", [
    (SERIALIZE_SRC.replace(" attributes {xt.grid = array<i32: 2, 2, 1>}", ""),
     "xt-serialize requires func.func xt.grid attribute"),
    ("func.func @non_void(%src: memref<128x16xf32>) -> i32 attributes {xt.grid = array<i32: 1, 1, 1>} {\n"
     "  %bid:3 = xt.get_tile_block_id : i32, i32, i32\n  func.return %bid#0 : i32\n}",
     "xt-serialize only supports void functions"),
    ("func.func @multi_block(%flag: i1) attributes {xt.grid = array<i32: 1, 1, 1>} {\n"
     "  cf.cond_br %flag, ^bb1, ^bb2\n^bb1:\n  func.return\n^bb2:\n  func.return\n}",
     "xt-serialize only supports single-block functions"),
])
def test_serialize_invalid(text, message):
    # serialize_invalid.mlir; stage failures raise RuntimeError
    # (python/XTModule.cpp:135-148)
    m = xt.parse(text)
    with pytest.raises(RuntimeError, match=message):
        xt.xt_serialize(m)


def test_stages_keep_module_identity_and_dump(tmp_path):
    names = {c[0]: c for c in build_cases(dsl)}
    _, fn, args, grid, db = names["matmul_i8_128x128x256"]
    m = xt.convert(fn, args=args, grid=grid, double_buffering=db)
    assert xt.compile(m) is m
    text = str(m)
    assert "family gemm" in text and "-> i8 (round half even, saturate)" in text
    m2 = xt.convert(fn, args=args, grid=grid, double_buffering=db)
    xt.save_compile_results(m2, str(tmp_path / "out"))
    files = sorted(p.name for p in (tmp_path / "out").iterdir())
    assert files == ["0_xt.mlir", "1_xt_serialize.mlir", "2_xt_to_nova.mlir", "3_nova_optimize.mlir",
                     "4_nova_threading.mlir", "5_nova_barrier.mlir", "6_nova_allocate.mlir",
                     "7_nova_to_x1.mlir"]


PLANS = {
    "add_rows_128x128": "ew",
    "add_tiles_2048_32x64": "ew",
    "softmax_8192x1024_row1": "rows",
    "softmax_128x128_row64": "rows",
    "rowwise_softmax": "rows",
    "matmul_i8_128x128x256": "gemm",
    "matmul_i8_1024x512x256": "gemm",
}


@pytest.mark.parametrize("name,family", sorted(PLANS.items()))
def test_plan_families(name, family):
    case = {c[0]: c for c in build_cases(dsl)}[name]
    _, fn, args, grid, db = case
    m = xt.convert(fn, args=args, grid=grid, double_buffering=db)
    assert m.plan()["family"] == family


def test_plan_work_figures():
    case = {c[0]: c for c in build_cases(dsl)}["add_tiles_2048_32x64"]
    m = xt.convert(case[1], args=case[2], grid=case[3], double_buffering=case[4])
    assert m.plan()["bytes"] == 3 * 2048 * 2048 * 4          # 50,331,648 B
    case = {c[0]: c for c in build_cases(dsl)}["softmax_8192x1024_row1"]
    m = xt.convert(case[1], args=case[2], grid=case[3], double_buffering=case[4])
    assert m.plan()["bytes"] == 2 * 8192 * 1024 * 4          # 67,108,864 B


def test_unsupported_programs_explain_why():
    case = {c[0]: c for c in build_cases(dsl)}["matmul_kloop_f32_512"]
    m = xt.convert(case[1], args=case[2], grid=case[3], double_buffering=case[4])
    with pytest.raises(RuntimeError, match="bf16 or i8 operands"):
        m.plan()
    # a column reduction is no elementwise map or row program: the tile family takes it
    case = {c[0]: c for c in build_cases(dsl)}["column_reduce"]
    m = xt.convert(case[1], args=case[2], grid=case[3], double_buffering=case[4])
    assert m.plan()["family"] == "tile"

    # every Block of a (4, 1, 1) grid storing the same tile: no family can run it
    # without the result depending on Block order
    @xt.kernel
    def same_tile(x, y):
        t = xt.load(x, index=(xt.bid(0), 0), shape=(8, 8))
        xt.store(y, index=(0, 0), tile=xt.sum(t, axis=0))

    m = xt.convert(same_tile, args=(xt.Array((32, 8), xt.float32), xt.Array((1, 8), xt.float32)), grid=(4, 1, 1))
    with pytest.raises(RuntimeError, match="no B200 kernel family.*would store the same tile"):
        m.plan()


# --- the planner's register programs, evaluated on the CPU -------------------
import numpy as np  # noqa: E402

from oracle import xt_oracle  # noqa: E402

_UNARY = {"exp": np.exp, "cos": np.cos, "sin": np.sin, "recip": lambda x: np.float32(1) / x,
          "rsqrt": lambda x: np.float32(1) / np.sqrt(x), "tanh": np.tanh,
          "sigmoid": lambda x: np.float32(1) / (np.float32(1) + np.exp(-x)),
          "silu": lambda x: x / (np.float32(1) + np.exp(-x)), "itof": lambda x: x,
          "ftoi": lambda x: xt_oracle.ftoi_i8(x).astype(np.float32)}
_BINARY = {"add": np.add, "sub": np.subtract, "mul": np.multiply,
           "bcast_add": np.add, "bcast_sub": np.subtract, "bcast_mul": np.multiply}


def run_register_program(module, arrays):
    """Evaluates the ew/rows register program of the stage dump with numpy."""
    xt.nova_optimize(module)
    names = [a[0] for a in module.arguments()]
    mem = dict(zip(names, arrays))
    regs = {}
    for line in xt._module_asm(module).splitlines():
        m = re.match(r"\s*//\s{5}(\w+) = (\w+) (.*)$", line)
        s = re.match(r"\s*//\s{5}(store|store_scalar) %(\w+) <- (\w+)$", line)
        if s:
            dst = mem[s.group(2)]
            dst[...] = regs[s.group(3)].astype(dst.dtype)
        elif m:
            dst, op, rest = m.groups()
            ops = [o.strip() for o in rest.split(",")]
            if op in ("load", "load_scalar"):
                regs[dst] = mem[ops[0].lstrip("%")].astype(np.float32)
            elif op == "rowmax":
                regs[dst] = regs[ops[0]].max(axis=1, keepdims=True)
            elif op == "rowsum":
                regs[dst] = regs[ops[0]].astype(np.float64).sum(axis=1, keepdims=True).astype(np.float32)
            elif op in _BINARY:
                regs[dst] = _BINARY[op](regs[ops[0]], regs[ops[1]]).astype(np.float32)
            else:
                regs[dst] = _UNARY[op](regs[ops[0]]).astype(np.float32)


def test_ew_register_program_matches_oracle():
    @dsl.kernel
    def ew_mixed(x, y, out, out2, trow, col):
        i = xt.bid(0)
        a = xt.load(x, index=(i, 0), shape=(trow, col))
        b = xt.load(y, index=(i, 0), shape=(trow, col))
        t = xt.exp(a) * b - a
        xt.store(out, index=(i, 0), tile=t)
        xt.store(out2, index=(i, 0), tile=xt.sigmoid(t) + xt.tanh(b))

    A = xt.Array
    m = xt.convert(ew_mixed, args=(A((30, 5), xt.float32),) * 4 + (10, 5), grid=(3, 1, 1))
    rng = np.random.default_rng(0)
    a = rng.standard_normal((30, 5)).astype(np.float32)
    b = rng.standard_normal((30, 5)).astype(np.float32)
    got = [a, b, np.zeros_like(a), np.zeros_like(a)]
    run_register_program(m, got)
    ref = [a, b, np.zeros_like(a), np.zeros_like(a)]
    xt_oracle.run(m.source_text, ref)
    np.testing.assert_allclose(got[2], ref[2], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(got[3], ref[3], rtol=1e-6, atol=1e-6)


def test_rows_register_program_matches_oracle():
    @dsl.kernel
    def row_stats(x, y, mx, trow, col):
        i = xt.bid(0)
        t = xt.load(x, index=(i, 0), shape=(trow, col))
        m = xt.max(t, axis=1)
        xt.store(y, index=(i, 0), tile=(t - m) * (t - m))
        xt.store(mx, index=(i, 0), tile=xt.reciprocal(xt.sum(t, axis=1)))

    A = xt.Array
    m = xt.convert(row_stats, args=(A((12, 7), xt.float32), A((12, 7), xt.float32), A((12, 1), xt.float32),
                                    4, 7), grid=(3, 1, 1))
    x = np.random.default_rng(1).standard_normal((12, 7)).astype(np.float32) + 3
    got = [x, np.zeros_like(x), np.zeros((12, 1), np.float32)]
    run_register_program(m, got)
    ref = [x, np.zeros_like(x), np.zeros((12, 1), np.float32)]
    xt_oracle.run(m.source_text, ref)
    np.testing.assert_array_equal(got[1], ref[1])
    np.testing.assert_allclose(got[2], ref[2], rtol=1e-6)
