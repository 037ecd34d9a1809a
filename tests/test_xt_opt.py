"""The xt-opt style command-line driver (``python -m xtile_b200.xt_opt``)."""
import io
import sys

from xtile_b200 import xt_opt

GOOD = """func.func @ok(%arg0: tensor<64x16xf32>) -> tensor<64x16xf32> {
  %0 = xt.reshape(%arg0) : tensor<64x16xf32> -> tensor<2x32x16xf32>
  %1 = xt.transpose(%0) : tensor<2x32x16xf32> -> tensor<2x16x32xf32>
  %2 = xt.reshape(%1) : tensor<2x16x32xf32> -> tensor<64x16xf32>
  return %2 : tensor<64x16xf32>
}
"""
BAD = """func.func @bad(%arg0: tensor<2x32x16xf32>) -> tensor<2x32x16xf32> {
  %0 = xt.transpose(%arg0) : tensor<2x32x16xf32> -> tensor<2x32x16xf32>
  return %0 : tensor<2x32x16xf32>
}
"""
GRID = """func.func @g(%x: memref<8x8xf32>, %y: memref<8x8xf32>) attributes {xt.grid = array<i32: 2, 1, 1>} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %t = xt.load(%x, %bid#0, %zero) : (memref<8x8xf32>, i32, i32) -> tensor<4x8xf32>
  xt.store(%t, %y, %bid#0, %zero) : (tensor<4x8xf32>, memref<8x8xf32>, i32, i32) -> ()
  func.return
}
"""


def run(tmp_path, text, *flags):
    path = tmp_path / "in.mlir"
    path.write_text(text)
    out, err = io.StringIO(), io.StringIO()
    old = sys.stdout, sys.stderr
    sys.stdout, sys.stderr = out, err
    try:
        rc = xt_opt.main([*flags, str(path)])
    finally:
        sys.stdout, sys.stderr = old
    return rc, out.getvalue(), err.getvalue(), str(path)


def test_parse_and_print(tmp_path):
    rc, out, err, _ = run(tmp_path, GOOD)
    assert rc == 0 and not err
    assert "xt.transpose(%0) : tensor<2x32x16xf32> -> tensor<2x16x32xf32>" in out


def test_split_input_file_reports_each_part(tmp_path):
    rc, out, err, path = run(tmp_path, GOOD + "\n// -----\n\n" + BAD, "--split-input-file")
    assert rc == 1
    assert "func.func @ok" in out and "@bad" not in out
    # the bad transpose is line 11 of the file
    assert f"{path}:11: error: 'xt.transpose' op transpose result shape must preserve dim 0" in err


def test_serialize_unrolls_the_grid(tmp_path):
    rc, out, _, _ = run(tmp_path, GRID, "--xt-serialize")
    assert rc == 0
    # both Blocks' ops, with their block ids as constants
    assert out.count("xt.load") == 2 and out.count("xt.store") == 2
    assert "xt.get_tile_block_id" not in out and "arith.constant 1 : i32" in out


def test_plan_is_appended(tmp_path):
    rc, out, _, _ = run(tmp_path, GRID, "--plan")
    assert rc == 0 and '// plan @g: {"family": "ew"' in out


ZEROS = """func.func @z(%a: tensor<16x16xf32>, %b: tensor<16x1xf32>) -> tensor<16x16xf32> {
  %zero = arith.constant dense<0.0> : tensor<16x16xf32>
  %izero = arith.constant dense<0> : tensor<16x16xf32>
  %0 = xt.add(%zero, %a) : tensor<16x16xf32>, tensor<16x16xf32> -> tensor<16x16xf32>
  %1 = xt.sub(%0, %izero) : tensor<16x16xf32>, tensor<16x16xf32> -> tensor<16x16xf32>
  %2 = xt.sub(%zero, %1) : tensor<16x16xf32>, tensor<16x16xf32> -> tensor<16x16xf32>
  %3 = xt.add(%b, %zero) : tensor<16x1xf32>, tensor<16x16xf32> -> tensor<16x16xf32>
  %4 = xt.mul(%2, %3) : tensor<16x16xf32>, tensor<16x16xf32> -> tensor<16x16xf32>
  %5 = xt.exp(%a) : tensor<16x16xf32> -> tensor<16x16xf32>
  return %4 : tensor<16x16xf32>
}
"""


def test_canonicalize_folds_zero_operands(tmp_path):
    # lib/xt/XTOps.cpp:395-449: 0 + x and x - 0 fold; 0 - x does not; a fold
    # whose operand has another type than the result (a broadcast) is kept;
    # the unused exp and the constants left unused are erased
    rc, out, err, _ = run(tmp_path, ZEROS, "--canonicalize", "--keep-names")
    assert rc == 0, err
    assert "xt.sub(%zero, %a)" in out
    assert "xt.add(%b, %zero)" in out
    assert "xt.exp" not in out and "%izero" not in out
    assert out.count("xt.add") == 1 and out.count("xt.sub") == 1
