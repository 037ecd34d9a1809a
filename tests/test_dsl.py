"""The tracer's text against fixtures produced by the reference tracer.

``tests/golden/dsl_text/*.mlir`` were written by ``tests/golden/make_golden.py``
running the reference's ``xtile/dsl.py`` in place; the text is the interface
between the DSL and every compiler stage, so it must match byte for byte
(the exact-text check of the reference's ``test/python/dsl_convert.py:25-43``
is one of these cases).
"""
from pathlib import Path

import pytest

import xtile_b200.dsl as xt
from tests.golden.cases import build_cases

GOLDEN = Path(__file__).resolve().parent / "golden" / "dsl_text"
CASES = build_cases(xt)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_text_matches_reference(case):
    name, fn, args, grid, db = case
    text = xt.trace_text(fn, args=args, grid=grid, double_buffering=db)
    assert text == (GOLDEN / f"{name}.mlir").read_text().rstrip("\n")


def test_every_fixture_has_a_case():
    assert {p.stem for p in GOLDEN.glob("*.mlir")} == {c[0] for c in CASES}


def _convert(fn, args, grid=(1, 1, 1)):
    return xt.trace_text(fn, args=args, grid=grid, double_buffering=False)


def test_outside_trace_raises():
    with pytest.raises(RuntimeError, match="xt.bid may only be used"):
        xt.bid(0)
    with pytest.raises(RuntimeError, match="xt.max may only be used"):
        xt.max(None)
    with pytest.raises(RuntimeError, match="xt.exp may only be used"):
        xt.exp(None)


def test_argument_errors():
    A = xt.Array
    with pytest.raises(TypeError):
        A((0, 4), xt.float32)
    with pytest.raises(TypeError):
        A([4, 4], xt.float32)

    @xt.kernel
    def k(x, y):
        t = xt.load(x, index=(0, 0), shape=(4, 4))
        xt.store(y, index=(0, 0), tile=t / 2)

    with pytest.raises(TypeError, match="truediv currently requires a tensor rhs"):
        _convert(k, (A((4, 4), xt.float32), A((4, 4), xt.float32)))

    @xt.kernel
    def bad_shared(x):
        xt.load(x, index=(0, 0), shape=(4, 4), shared=3)

    with pytest.raises(ValueError, match="shared must be 0, 1, 2, or None"):
        _convert(bad_shared, (A((4, 4), xt.float32),))

    @xt.kernel
    def bad_bcast(x, y):
        a = xt.load(x, index=(0, 0), shape=(4, 4))
        b = xt.load(y, index=(0, 0), shape=(2, 4))
        a + b

    with pytest.raises(ValueError, match="rowwise-broadcast-compatible"):
        _convert(bad_bcast, (A((4, 4), xt.float32), A((4, 4), xt.float32)))

    @xt.kernel
    def returns(x):
        return 1

    with pytest.raises(ValueError, match="must not return a value"):
        _convert(returns, (A((4, 4), xt.float32),))

    with pytest.raises(ValueError, match="grid must be a 3-tuple"):
        xt.trace_text(returns, args=(A((4, 4), xt.float32),), grid=(1, 1),
                      double_buffering=False)
    with pytest.raises(ValueError, match="args must match"):
        _convert(returns, ())
    with pytest.raises(TypeError, match="decorated with @xt.kernel"):
        xt.trace_text(lambda x: None, args=(1,), grid=(1, 1, 1), double_buffering=False)


def test_bfloat16_extension():
    A = xt.Array

    @xt.kernel
    def mm(a, b, c):
        x = xt.load(a, index=(xt.bid(0), 0), shape=(128, 64))
        y = xt.load(b, index=(0, xt.bid(1)), shape=(64, 128), shared=1)
        xt.store(c, index=(xt.bid(0), xt.bid(1)), tile=xt.matmul(x, y))

    text = _convert(mm, (A((256, 64), xt.bfloat16), A((64, 256), xt.bfloat16),
                         A((256, 256), xt.float32)), grid=(2, 2, 1))
    assert "tensor<128x64xbf16>, tensor<64x128xbf16> -> tensor<128x128xf32>" in text

    @xt.kernel
    def mixed(a, b, c):
        x = xt.load(a, index=(0, 0), shape=(4, 4))
        y = xt.load(b, index=(0, 0), shape=(4, 4))
        xt.store(c, index=(0, 0), tile=xt.matmul(x, y))

    with pytest.raises(TypeError, match="matching dtypes or int8"):
        _convert(mixed, (A((4, 4), xt.bfloat16), A((4, 4), xt.int8), A((4, 4), xt.float32)))
