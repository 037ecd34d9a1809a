"""xtile tile DSL: traces one Block program and prints it as xt-dialect text.

A kernel is a Python function written from the point of view of one Block.
``convert`` runs it once with symbolic arguments; every ``xt.*`` call appends a
record to the active trace, and the trace is then printed as one
``func.func`` in the xt dialect.  The printed text is an interface shared with
the reference compiler (sjjeong94/xtile), so its spelling is kept identical:

* value names and their stems (``%x``, ``%row_max``, ``%shifted`` ...) and the
  ``%stem2``/``%stem3`` numbering -- reference ``xtile/dsl.py:692-695``;
* argument naming (``input``/``inputN`` for arrays that are only loaded,
  ``output``/``outputN`` for arrays that are only stored) --
  ``xtile/dsl.py:670-690``;
* constants listed once, sorted by value, ``%zero`` for 0 --
  ``xtile/dsl.py:664-668,506-509``;
* one line per op in the formats of ``xtile/dsl.py:511-620``.

Extensions over the reference surface (none of them changes the text of a
float32/int8 program):

* ``bfloat16`` dtype (mlir name ``bf16``);
* ``matmul`` of two bfloat16 tiles yields float32 (fp32 accumulation), the
  same rule the reference applies to int8 (``xtile/dsl.py:369-374``);
* ``load_conv2d`` accepts bfloat16 source and filter (result float32), next
  to int8 (``xtile/dsl.py:284-285``).
"""
from __future__ import annotations

import inspect
from dataclasses import dataclass
from typing import Callable, Iterable


# --------------------------------------------------------------------------
# dtypes and global arrays
# --------------------------------------------------------------------------
@dataclass(frozen=True)
class DType:
    name: str
    mlir_name: str


float32 = DType(name="float32", mlir_name="f32")
int8 = DType(name="int8", mlir_name="i8")
bfloat16 = DType(name="bfloat16", mlir_name="bf16")


@dataclass(frozen=True)
class Array:
    """A global-memory array: static shape and dtype (row-major, contiguous)."""

    shape: tuple[int, ...]
    dtype: DType

    def __post_init__(self) -> None:
        if not isinstance(self.shape, tuple) or not self.shape:
            raise TypeError("shape must be a non-empty tuple of integers")
        for dim in self.shape:
            if not isinstance(dim, int) or dim <= 0:
                raise TypeError("shape must contain positive integers")
        if not isinstance(self.dtype, DType):
            raise TypeError("dtype must be an xtile dtype")

    @property
    def ndim(self) -> int:
        return len(self.shape)


class KernelFunction:
    """The object ``@xt.kernel`` returns; ``convert`` only accepts these."""

    def __init__(self, fn: Callable[..., object]) -> None:
        self.fn = fn
        self.__name__ = fn.__name__
        self.__doc__ = fn.__doc__
        self.__wrapped__ = fn


def kernel(fn: Callable[..., object]) -> KernelFunction:
    return KernelFunction(fn)


# --------------------------------------------------------------------------
# symbolic values seen by the kernel body while it is traced
# --------------------------------------------------------------------------
@dataclass(frozen=True)
class KernelArg:
    index: int
    python_name: str
    array: Array


@dataclass(frozen=True)
class BlockId:
    dim: int


@dataclass(frozen=True)
class ConstantIndex:
    value: int


@dataclass(frozen=True)
class TensorValue:
    """A tile produced inside the Block program."""

    ssa_name: str
    shape: tuple[int, ...]
    dtype: DType

    def __add__(self, other: object) -> "TensorValue":
        return add(self, other)  # type: ignore[arg-type]

    def __sub__(self, other: object) -> "TensorValue":
        return sub(self, other)  # type: ignore[arg-type]

    def __mul__(self, other: object) -> "TensorValue":
        return mul(self, other)  # type: ignore[arg-type]

    def __truediv__(self, other: object) -> "TensorValue":
        return truediv(self, other)


Index = tuple  # tuple[BlockId | ConstantIndex, ...]


@dataclass(frozen=True)
class Record:
    """One traced operation.

    ``form`` selects the printed layout: load, load_conv2d, store, reduce,
    unary (also casts, reshape, transpose), binary (also matmul), ternary.
    """

    form: str
    op: str
    result: TensorValue | None = None
    operands: tuple[TensorValue, ...] = ()
    array: KernelArg | None = None
    index: Index = ()
    shared: int | None = None
    axis: int = 0
    conv: tuple[int, tuple[int, ...], tuple[int, ...], tuple[int, ...]] | None = None


# stems of the SSA names each op gets (reference xtile/dsl.py:315-357,622-644)
_UNARY_STEMS = {
    "exp": "exp",
    "cos": "cos",
    "sin": "sin",
    "reciprocal": "inv_sum",
    "rsqrt": "rsqrt",
    "sigmoid": "sigmoid",
    "tanh": "tanh",
    "silu": "silu",
}
_BINARY_STEMS = {"add": "sum", "sub": "shifted", "mul": "normalized"}
_REDUCE_OPS = {"max": ("xt.reduce_max", "row_max"), "sum": ("xt.reduce_sum", "row_sum")}


def _type_str(kind: str, shape: Iterable[int], dtype: DType) -> str:
    return f"{kind}<{'x'.join(str(d) for d in shape)}x{dtype.mlir_name}>"


def _tensor_type(shape: Iterable[int], dtype: DType) -> str:
    return _type_str("tensor", shape, dtype)


def _memref_type(array: Array) -> str:
    return _type_str("memref", array.shape, array.dtype)


def _count(shape: Iterable[int]) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


class Trace:
    """State of one ``convert`` call: arguments, records and name counters."""

    def __init__(self, kernel_fn: KernelFunction, args: tuple, grid: tuple,
                 double_buffering: bool) -> None:
        if len(grid) != 3 or any(not isinstance(g, int) or g <= 0 for g in grid):
            raise ValueError("grid must be a 3-tuple of positive integers")
        params = list(inspect.signature(kernel_fn.fn).parameters.values())
        if len(params) != len(args):
            raise ValueError("convert args must match the kernel signature")
        self.name = kernel_fn.fn.__name__
        self.grid = tuple(grid)
        self.double_buffering = double_buffering
        self.params: list[KernelArg | int] = []
        for i, (param, arg) in enumerate(zip(params, args)):
            if isinstance(arg, Array):
                self.params.append(KernelArg(i, param.name, arg))
            elif isinstance(arg, int):
                self.params.append(arg)
            else:
                raise TypeError("convert args must be xt.Array values or integers")
        self.records: list[Record] = []
        self.uses_bid = False
        self.loads = [0] * len(args)
        self.stores = [0] * len(args)
        self.counters: dict[str, int] = {}
        self.constants: dict[int, str] = {}

    # -- naming -------------------------------------------------------------
    def fresh(self, stem: str) -> str:
        n = self.counters.get(stem, 0) + 1
        self.counters[stem] = n
        return f"%{stem}" if n == 1 else f"%{stem}{n}"

    def value(self, stem: str, shape: tuple, dtype: DType) -> TensorValue:
        return TensorValue(self.fresh(stem), tuple(shape), dtype)

    # -- argument checks ----------------------------------------------------
    @staticmethod
    def need_arg(array: object) -> KernelArg:
        if not isinstance(array, KernelArg):
            raise TypeError("xtile load/store expect kernel arguments")
        return array

    @staticmethod
    def need_tile(value: object) -> TensorValue:
        if not isinstance(value, TensorValue):
            raise TypeError("xtile operation expects a tensor value")
        return value

    @staticmethod
    def need_shape(shape: object) -> tuple:
        if (not isinstance(shape, tuple) or not shape
                or any(not isinstance(d, int) or d <= 0 for d in shape)):
            raise TypeError("shape must be a tuple of positive integers")
        return shape

    @staticmethod
    def need_ints(name: str, value: object, length: int, positive: bool) -> tuple:
        if not isinstance(value, tuple) or len(value) != length:
            raise TypeError(f"{name} must be a tuple of {length} integers")
        for item in value:
            if not isinstance(item, int):
                raise TypeError(f"{name} must be a tuple of {length} integers")
            if positive and item <= 0:
                raise ValueError(f"{name} values must be positive")
            if not positive and item < 0:
                raise ValueError(f"{name} values must be non-negative")
        return value

    def index(self, index: object) -> Index:
        if not isinstance(index, tuple) or not index:
            raise TypeError("index must be a non-empty tuple of values")
        out = []
        for item in index:
            if isinstance(item, BlockId):
                out.append(item)
            elif isinstance(item, int):
                if item not in self.constants:
                    self.constants[item] = "%zero" if item == 0 else self.fresh(f"c{item}")
                out.append(ConstantIndex(item))
            else:
                raise TypeError("index values must be xt.bid(...) results or integers")
        return tuple(out)

    # -- ops ----------------------------------------------------------------
    def bid(self, dim: int) -> BlockId:
        if dim not in (0, 1, 2):
            raise ValueError("xt.bid only supports dimensions 0, 1, and 2")
        self.uses_bid = True
        return BlockId(dim)

    def load(self, array, index, shape, shared) -> TensorValue:
        arg = self.need_arg(array)
        idx = self.index(index)
        self.need_shape(shape)
        if shared is not None and shared not in (0, 1, 2):
            raise ValueError("shared must be 0, 1, 2, or None")
        if arg.array.ndim != len(shape):
            raise ValueError("xt.load requires shape rank to match the source array rank")
        if len(idx) != len(shape):
            raise ValueError("xt.load requires index rank to match the source array rank")
        result = self.value("x", shape, arg.array.dtype)
        self.records.append(Record("load", "xt.load", result, array=arg, index=idx, shared=shared))
        self.loads[arg.index] += 1
        return result

    def load_conv2d(self, array, filt, index, shape, group, pad, stride, dilation) -> TensorValue:
        arg = self.need_arg(array)
        filt = self.need_tile(filt)
        idx = self.index(index)
        self.need_shape(shape)
        self.need_ints("pad", pad, 4, positive=False)
        self.need_ints("stride", stride, 2, positive=True)
        self.need_ints("dilation", dilation, 2, positive=True)
        if group <= 0:
            raise ValueError("xt.load_conv2d requires group to be positive")
        if arg.array.ndim != 4:
            raise ValueError("xt.load_conv2d requires a rank-4 source memref")
        if len(filt.shape) != 4:
            raise ValueError("xt.load_conv2d requires a rank-4 filter tensor")
        if len(idx) != 4 or len(shape) != 4:
            raise ValueError("xt.load_conv2d requires rank-4 index and result shape tuples")
        src_dtype = arg.array.dtype
        if src_dtype != filt.dtype or src_dtype not in (int8, bfloat16):
            raise TypeError("xt.load_conv2d currently requires int8 source/filter "
                            "(bfloat16 source/filter is also accepted)")
        if arg.array.shape[3] != filt.shape[2]:
            raise ValueError("xt.load_conv2d requires source/filter channel dimensions to match")
        if shape[3] > filt.shape[3]:
            raise ValueError("xt.load_conv2d result channel dimension must not exceed "
                             "filter output channels")
        result = self.value("load_conv", shape, float32)
        self.records.append(Record("load_conv2d", "xt.load_conv2d", result, (filt,), arg, idx,
                                   conv=(group, tuple(pad), tuple(stride), tuple(dilation))))
        self.loads[arg.index] += 1
        return result

    def store(self, array, index, tile) -> None:
        arg = self.need_arg(array)
        idx = self.index(index)
        if not isinstance(tile, TensorValue):
            raise TypeError("xt.store expects a tensor value")
        if arg.array.ndim != len(tile.shape):
            raise ValueError("xt.store requires tile rank to match the destination array rank")
        if len(idx) != len(tile.shape):
            raise ValueError("xt.store requires index rank to match the destination array rank")
        self.records.append(Record("store", "xt.store", None, (tile,), arg, idx))
        self.stores[arg.index] += 1

    def reduce(self, kind: str, value, axis: int) -> TensorValue:
        op, stem = _REDUCE_OPS[kind]
        value = self.need_tile(value)
        if len(value.shape) != 2:
            raise ValueError("xt.max and xt.sum currently support rank-2 tensors only")
        if not isinstance(axis, int):
            raise TypeError("axis must be an integer")
        rank = len(value.shape)
        if axis < -rank or axis >= rank:
            raise ValueError("axis must be in range [-rank, rank)")
        axis %= rank
        shape = list(value.shape)
        shape[axis] = 1
        result = self.value(stem, tuple(shape), value.dtype)
        self.records.append(Record("reduce", op, result, (value,), axis=axis))
        return result

    def unary(self, kind: str, value) -> TensorValue:
        value = self.need_tile(value)
        result = self.value(_UNARY_STEMS[kind], value.shape, value.dtype)
        self.records.append(Record("unary", f"xt.{kind}", result, (value,)))
        return result

    def binary(self, kind: str, lhs, rhs) -> TensorValue:
        lhs = self.need_tile(lhs)
        rhs = self.need_tile(rhs)
        if lhs.dtype != rhs.dtype:
            raise TypeError("binary xtile ops require matching dtypes")
        # equal shapes, or rhs broadcast along its size-1 dims (reference
        # xtile/dsl.py:754-759); the result takes the lhs shape
        ok = lhs.shape == rhs.shape or (
            len(lhs.shape) == len(rhs.shape)
            and all(r in (1, l) for l, r in zip(lhs.shape, rhs.shape)))
        if not ok:
            raise ValueError("binary xtile ops require equal or rowwise-broadcast-compatible shapes")
        result = self.value(_BINARY_STEMS[kind], lhs.shape, lhs.dtype)
        self.records.append(Record("binary", f"xt.{kind}", result, (lhs, rhs)))
        return result

    def truediv(self, lhs, rhs) -> TensorValue:
        # division is spelled mul(lhs, reciprocal(rhs)) (reference xtile/dsl.py:354-357)
        self.need_tile(lhs)
        self.need_tile(rhs)
        return self.binary("mul", lhs, self.unary("reciprocal", rhs))

    def matmul(self, lhs, rhs) -> TensorValue:
        lhs = self.need_tile(lhs)
        rhs = self.need_tile(rhs)
        if len(lhs.shape) != 2 or len(rhs.shape) != 2:
            raise ValueError("xt.matmul currently supports rank-2 tensors only")
        if lhs.shape[1] != rhs.shape[0]:
            raise ValueError("xt.matmul requires lhs inner dimension to match rhs outer dimension")
        if lhs.dtype == rhs.dtype and lhs.dtype in (int8, bfloat16):
            dtype = float32          # int8 (reference) and bfloat16 (extension) accumulate in f32
        elif lhs.dtype == rhs.dtype:
            dtype = lhs.dtype
        else:
            raise TypeError("xt.matmul requires matching dtypes or int8 inputs")
        result = self.value("matmul", (lhs.shape[0], rhs.shape[1]), dtype)
        self.records.append(Record("binary", "xt.matmul", result, (lhs, rhs)))
        return result

    def astype(self, value, dtype) -> TensorValue:
        value = self.need_tile(value)
        if not isinstance(dtype, DType):
            raise TypeError("xt.astype requires an xtile dtype")
        if value.dtype == dtype:
            return value
        if (value.dtype, dtype) == (int8, float32):
            op = "xt.itof"
        elif (value.dtype, dtype) == (float32, int8):
            op = "xt.ftoi"
        else:
            raise TypeError("xt.astype only supports int8<->float32 conversions")
        result = self.value("cast", value.shape, dtype)
        self.records.append(Record("unary", op, result, (value,)))
        return result

    def reshape(self, value, shape) -> TensorValue:
        value = self.need_tile(value)
        self.need_shape(shape)
        if _count(value.shape) != _count(shape):
            raise ValueError("xt.reshape requires the same number of elements")
        result = self.value("reshape", shape, value.dtype)
        self.records.append(Record("unary", "xt.reshape", result, (value,)))
        return result

    def transpose(self, value) -> TensorValue:
        value = self.need_tile(value)
        if len(value.shape) != 3:
            raise ValueError("xt.transpose currently supports rank-3 tensors only")
        a, b, c = value.shape
        result = self.value("transpose", (a, c, b), value.dtype)
        self.records.append(Record("unary", "xt.transpose", result, (value,)))
        return result

    def mma(self, lhs, rhs, acc) -> TensorValue:
        lhs, rhs, acc = (self.need_tile(v) for v in (lhs, rhs, acc))
        if len(lhs.shape) != 2 or len(rhs.shape) != 2 or len(acc.shape) != 2:
            raise ValueError("xt.mma currently supports rank-2 tensors only")
        if lhs.dtype != int8 or rhs.dtype != int8:
            raise TypeError("xt.mma requires int8 lhs and rhs tensors")
        if acc.dtype != float32:
            raise TypeError("xt.mma currently requires a float32 accumulator")
        if lhs.shape[1] != rhs.shape[0]:
            raise ValueError("xt.mma requires lhs inner dimension to match rhs outer dimension")
        if acc.shape != (lhs.shape[0], rhs.shape[1]):
            raise ValueError("xt.mma accumulator shape must match the matmul result shape")
        result = self.value("mma", acc.shape, acc.dtype)
        self.records.append(Record("ternary", "xt.mma", result, (lhs, rhs, acc)))
        return result

    # -- printing -----------------------------------------------------------
    def arg_names(self) -> dict[int, str]:
        names: dict[int, str] = {}
        n_in = n_out = 0
        for p in self.params:
            if not isinstance(p, KernelArg):
                continue
            loads, stores = self.loads[p.index], self.stores[p.index]
            if loads and not stores:
                n_in += 1
                names[p.index] = "input" if n_in == 1 else f"input{n_in}"
            elif stores and not loads:
                n_out += 1
                names[p.index] = "output" if n_out == 1 else f"output{n_out}"
            else:
                names[p.index] = p.python_name
        return names

    def index_text(self, index: Index) -> str:
        parts = []
        for item in index:
            if isinstance(item, BlockId):
                parts.append(f"%bid#{item.dim}")
            else:
                parts.append("%zero" if item.value == 0 else f"%c{item.value}")
        return ", ".join(parts)

    def record_text(self, r: Record, names: dict[int, str]) -> str:
        coords = ", ".join(["i32"] * len(r.index))
        if r.form == "load":
            attr = f" {{shared = {r.shared} : i64}}" if r.shared in (1, 2) else ""
            return (f"{r.result.ssa_name} = xt.load(%{names[r.array.index]}, "
                    f"{self.index_text(r.index)}){attr} : ({_memref_type(r.array.array)}, "
                    f"{coords}) -> {_tensor_type(r.result.shape, r.result.dtype)}")
        if r.form == "load_conv2d":
            group, pad, stride, dilation = r.conv
            filt = r.operands[0]
            attrs = (f"dilation = array<i64: {', '.join(map(str, dilation))}>, "
                     f"group = {group} : i64, "
                     f"pad = array<i64: {', '.join(map(str, pad))}>, "
                     f"stride = array<i64: {', '.join(map(str, stride))}>")
            return (f"{r.result.ssa_name} = xt.load_conv2d(%{names[r.array.index]}, "
                    f"{filt.ssa_name}, {self.index_text(r.index)}) {{{attrs}}} : "
                    f"({_memref_type(r.array.array)}, {_tensor_type(filt.shape, filt.dtype)}, "
                    f"{coords}) -> {_tensor_type(r.result.shape, r.result.dtype)}")
        if r.form == "store":
            tile = r.operands[0]
            return (f"xt.store({tile.ssa_name}, %{names[r.array.index]}, "
                    f"{self.index_text(r.index)}) : ({_tensor_type(tile.shape, tile.dtype)}, "
                    f"{_memref_type(r.array.array)}, {coords}) -> ()")
        operands = ", ".join(v.ssa_name for v in r.operands)
        result_type = _tensor_type(r.result.shape, r.result.dtype)
        operand_types = ", ".join(_tensor_type(v.shape, v.dtype) for v in r.operands)
        if r.form == "reduce":
            return (f"{r.result.ssa_name} = {r.op}({operands}) {{axis = {r.axis} : i64}} : "
                    f"{operand_types} -> {result_type}")
        return f"{r.result.ssa_name} = {r.op}({operands}) : {operand_types} -> {result_type}"

    def text(self) -> str:
        names = self.arg_names()
        signature = ", ".join(
            f"%{names[p.index]}: {_memref_type(p.array)}"
            for p in self.params if isinstance(p, KernelArg))
        attrs = [f"xt.grid = array<i32: {', '.join(map(str, self.grid))}>"]
        if self.double_buffering:
            attrs.append("xt.double_buffering = 1 : i32")
        lines = [f"func.func @{self.name}({signature}) attributes {{{', '.join(attrs)}}} {{"]
        if self.uses_bid:
            lines.append("  %bid:3 = xt.get_tile_block_id : i32, i32, i32")
        if self.constants:
            for value in sorted(self.constants):
                lines.append(f"  {self.constants[value]} = arith.constant {value} : i32")
            lines.append("")
        lines.extend("  " + self.record_text(r, names) for r in self.records)
        lines.append("  func.return")
        lines.append("}")
        return "\n".join(lines)


# --------------------------------------------------------------------------
# public DSL functions (valid only while ``convert`` runs a kernel body)
# --------------------------------------------------------------------------
_ACTIVE: Trace | None = None


def _active(public_name: str) -> Trace:
    if _ACTIVE is None:
        raise RuntimeError(f"xt.{public_name} may only be used while converting a kernel")
    return _ACTIVE


def bid(dim: int) -> BlockId:
    return _active("bid").bid(dim)


def load(array: KernelArg, *, index: tuple, shape: tuple, shared: int | None = None) -> TensorValue:
    return _active("load").load(array, index, shape, shared)


def load_conv2d(array: KernelArg, filter_value: TensorValue, *, index: tuple, shape: tuple,
                group: int = 1, pad: tuple, stride: tuple, dilation: tuple) -> TensorValue:
    return _active("load_conv2d").load_conv2d(array, filter_value, index, shape,
                                              group, pad, stride, dilation)


def store(array: KernelArg, *, index: tuple, tile: TensorValue) -> None:
    _active("store").store(array, index, tile)


def max(input_value: TensorValue, axis: int = -1) -> TensorValue:  # noqa: A001
    return _active("max").reduce("max", input_value, axis)


def sum(input_value: TensorValue, axis: int = -1) -> TensorValue:  # noqa: A001
    return _active("sum").reduce("sum", input_value, axis)


def _make_unary(kind: str) -> Callable[[TensorValue], TensorValue]:
    def fn(input_value: TensorValue) -> TensorValue:
        return _active(kind).unary(kind, input_value)
    fn.__name__ = kind
    fn.__qualname__ = kind
    fn.__doc__ = f"Elementwise {kind} of a tile (emits xt.{kind})."
    return fn


exp = _make_unary("exp")
cos = _make_unary("cos")
sin = _make_unary("sin")
reciprocal = _make_unary("reciprocal")
rsqrt = _make_unary("rsqrt")
sigmoid = _make_unary("sigmoid")
tanh = _make_unary("tanh")
silu = _make_unary("silu")


def add(lhs: TensorValue, rhs: TensorValue) -> TensorValue:
    return _active("add").binary("add", lhs, rhs)


def sub(lhs: TensorValue, rhs: TensorValue) -> TensorValue:
    return _active("sub").binary("sub", lhs, rhs)


def mul(lhs: TensorValue, rhs: TensorValue) -> TensorValue:
    return _active("mul").binary("mul", lhs, rhs)


def truediv(lhs: TensorValue, rhs: object) -> TensorValue:
    trace = _active("truediv")
    if not isinstance(rhs, TensorValue):
        raise TypeError("xt.truediv currently requires a tensor rhs")
    return trace.truediv(lhs, rhs)


def matmul(lhs: TensorValue, rhs: TensorValue) -> TensorValue:
    return _active("matmul").matmul(lhs, rhs)


def astype(input_value: TensorValue, *, dtype: DType) -> TensorValue:
    return _active("astype").astype(input_value, dtype)


def reshape(input_value: TensorValue, *, shape: tuple) -> TensorValue:
    return _active("reshape").reshape(input_value, shape)


def transpose(input_value: TensorValue) -> TensorValue:
    return _active("transpose").transpose(input_value)


def mma(lhs: TensorValue, rhs: TensorValue, acc: TensorValue) -> TensorValue:
    return _active("mma").mma(lhs, rhs, acc)


def trace_text(kernel_fn: KernelFunction, *, args: tuple, grid: tuple,
               double_buffering: bool) -> str:
    """Run the kernel body once and return its xt-dialect text."""
    global _ACTIVE
    if not isinstance(kernel_fn, KernelFunction):
        raise TypeError("xt.convert expects a function decorated with @xt.kernel")
    trace = Trace(kernel_fn, args, grid, double_buffering)
    outer, _ACTIVE = _ACTIVE, trace
    try:
        returned = kernel_fn.fn(*(p for p in trace.params))
    finally:
        _ACTIVE = outer
    if returned is not None:
        raise ValueError("xt.kernel functions must not return a value")
    return trace.text()


def convert(kernel_fn: KernelFunction, *, args: tuple, grid: tuple, double_buffering: bool,
            parse_module: Callable[[str], object]) -> object:
    """Trace ``kernel_fn`` and hand its text to ``parse_module`` (reference
    ``xtile/dsl.py:1001-1029``)."""
    return parse_module(trace_text(kernel_fn, args=args, grid=grid,
                                   double_buffering=double_buffering))
