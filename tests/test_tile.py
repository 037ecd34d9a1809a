"""The tile family's planner, on the CPU: which Block programs it takes, the
shared-memory layout it gives their tiles, and what it rejects."""
import pytest

import xtile as xt

A = xt.Array
f32 = xt.float32


@xt.kernel
def transpose3(x, y, tm, tn):
    b, i, j = xt.bid(0), xt.bid(1), xt.bid(2)
    t = xt.load(x, index=(b, i, j), shape=(1, tm, tn))
    xt.store(y, index=(b, j, i), tile=xt.transpose(t))


@xt.kernel
def col_sums(x, y, tm, tn):
    i, j = xt.bid(0), xt.bid(1)
    t = xt.load(x, index=(i, j), shape=(tm, tn))
    xt.store(y, index=(i, j), tile=xt.sum(t, axis=0))


def test_transpose_plans_as_a_tile_program():
    m = xt.convert(transpose3, args=(A((2, 96, 200), f32), A((2, 200, 96), f32), 32, 64), grid=(2, 3, 4))
    p = m.plan()
    assert p["family"] == "tile"
    # every Block loads and stores one 32x64 f32 tile
    assert p["bytes"] == 2 * 3 * 4 * 2 * 32 * 64 * 4


def test_column_sums_plan_as_a_tile_program():
    m = xt.convert(col_sums, args=(A((256, 96), f32), A((4, 96), f32), 64, 32), grid=(4, 3, 1))
    assert m.plan()["family"] == "tile"


def test_stage_dump_describes_the_tile_plan():
    m = xt.convert(col_sums, args=(A((256, 96), f32), A((4, 96), f32), 64, 32), grid=(4, 3, 1))
    text = str(xt.xt_to_nova(xt.xt_serialize(m)))
    assert "family tile" in text and "one CTA per Block" in text


def test_tiles_beyond_shared_memory_are_rejected():
    # 2 x 256 x 512 f32 tiles = 1 MiB: more than one Block's shared memory
    m = xt.convert(col_sums, args=(A((512, 512), f32), A((2, 512), f32), 256, 512), grid=(2, 1, 1))
    with pytest.raises(RuntimeError, match="192 KiB of shared memory"):
        m.plan()


def test_permute_must_match_its_result_shape():
    text = """func.func @p(%x: memref<2x3x5xf32>, %y: memref<5x2x3xf32>) attributes {xt.grid = array<i32: 1, 1, 1>} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %t = xt.load(%x, %zero, %zero, %zero) : (memref<2x3x5xf32>, i32, i32, i32) -> tensor<2x3x5xf32>
  %u = xt.permute(%t) {permutation = [2, 0, 1]} : tensor<2x3x5xf32> -> tensor<5x2x3xf32>
  xt.store(%u, %y, %zero, %zero, %zero) : (tensor<5x2x3xf32>, memref<5x2x3xf32>, i32, i32, i32) -> ()
  func.return
}"""
    assert xt.parse(text).plan()["family"] == "tile"


@xt.kernel
def transpose_twice_used(x, y, z, tm, tn):
    b, i, j = xt.bid(0), xt.bid(1), xt.bid(2)
    t = xt.transpose(xt.load(x, index=(b, i, j), shape=(1, tm, tn)))
    xt.store(y, index=(b, j, i), tile=t)
    xt.store(z, index=(b, j, i), tile=t * t)


def test_a_permute_feeding_only_a_store_is_folded_into_it():
    # load + transpose + store plans as two tile ops: the store reads the
    # loaded tile through the transposed strides
    m = xt.convert(transpose3, args=(A((2, 96, 200), f32), A((2, 200, 96), f32), 32, 64), grid=(2, 3, 4))
    assert "2 tile ops" in str(xt.xt_to_nova(xt.xt_serialize(m)))
    # a transposed tile that is also multiplied keeps its permute op
    m = xt.convert(transpose_twice_used, args=(A((2, 96, 200), f32), A((2, 200, 96), f32), A((2, 200, 96), f32),
                                               32, 64), grid=(2, 3, 4))
    assert "5 tile ops" in str(xt.xt_to_nova(xt.xt_serialize(m)))
