"""CPU oracle for xt Block programs -- TEST INFRASTRUCTURE ONLY.

This module is the checker the parity tests, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg compare the B200 kernels against.  It is never
part of the product path: the ``xtile_b200`` package does not import it.

What it restates
----------------
The reference (sjjeong94/xtile) compiles Block programs to NPU command IR and
executes nothing, so there is no reference CPU loop lowering to build.  This
file interprets the xt program the way the reference's passes define it:

* the grid is walked z-outer, y, x-inner -- ``lib/xt/XTSerialize.cpp:68-84``;
* a tile coordinate ``i`` of a tile dimension ``t`` starts at element ``i*t``
  -- ``lib/xt/XTToNova.cpp:82-101`` (``:98``);
* ``load_conv2d`` loads the halo slice of ``computeConv2DSpatialSlice``
  (``lib/xt/XTToNova.cpp:103-142``) and convolves it with the slice's pads
  (``:353-437``), i.e. zero padding outside the source image;
* binary ops broadcast size-1 dims (``lib/xt/XTOps.cpp:104-120``); division is
  ``mul(x, reciprocal(y))`` (``xtile/dsl.py:354-357``); reductions keep the
  reduced dim as 1 (``lib/xt/XTOps.cpp:274-299``);
* ``matmul`` multiplies exactly and rounds once to f32; the scale/bias written
  as ``t * s + b`` stays two f32 roundings (``lib/nova/NovaOptimize.cpp:126-296``
  folds them into the matmul epilogue without changing their order).

Deviations from the reference, all deliberate:

* every load reads the tile its index names.  The reference's serialize pass
  reuses a ``shared=k`` load across blocks keyed by ``(op, k==2 ? 0 : y, z)``
  (``XTSerialize.cpp:86-99``), which only differs when a program breaks the
  ``shared`` contract;
* tiles reaching past an array edge read zeros and their out-of-range part is
  not stored (the reference has no partial tiles);
* ``ftoi`` rounds half to even and saturates to the int8 range, NaN -> 0
  (the reference leaves the rounding unspecified);
* unary ops the reference never lowers (cos, sin, rsqrt, sigmoid, tanh, silu)
  use their mathematical definitions in f32.

Parity status: numeric parity is UNPINNED -- the reference computes no numbers
and its tests hold no numeric golden vectors.  The structural semantics above
are pinned by the reference's own known answers (tile offsets and conv halo
slices of ``test/xt/to_nova.mlir:143-156``, grid order of
``test/xt/serialize.mlir:55-76``) in ``tests/test_oracle.py``.

Arrays are numpy arrays: float32, int8, and bfloat16 carried as uint16 bit
patterns.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field

import numpy as np

# --------------------------------------------------------------------------
# types
# --------------------------------------------------------------------------
_TYPE_RE = re.compile(r"(tensor|memref)<((?:\d+x)*)(f32|bf16|i8|i32|f16)>")


@dataclass
class OType:
    kind: str                  # "tensor" | "memref" | "i32" | "index"
    shape: tuple = ()
    elem: str = "i32"


def parse_type(text: str) -> OType:
    text = text.strip()
    m = _TYPE_RE.fullmatch(text)
    if m:
        dims = tuple(int(d) for d in m.group(2).split("x") if d)
        return OType(m.group(1), dims, m.group(3))
    if text in ("i32", "index", "i64", "i1"):
        return OType(text)
    raise ValueError(f"oracle: unsupported type {text!r}")


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest, ties to even) as uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


_NP_DTYPE = {"f32": np.float32, "i8": np.int8, "bf16": np.uint16, "i32": np.int32}


# --------------------------------------------------------------------------
# program representation and parser (independent of the product's parser)
# --------------------------------------------------------------------------
@dataclass
class OOp:
    name: str
    results: list
    operands: list
    attrs: dict
    types_in: list
    type_out: OType | None


@dataclass
class OFunc:
    name: str
    args: list                              # [(name, OType)]
    grid: tuple = (1, 1, 1)
    ops: list = field(default_factory=list)

    @property
    def memref_args(self):
        return [(n, t) for n, t in self.args if t.kind == "memref"]


def _split_top(text: str) -> list[str]:
    parts, depth, cur = [], 0, []
    for ch in text:
        if ch in "<([{":
            depth += 1
        elif ch in ">)]}":
            depth -= 1
        if ch == "," and depth == 0:
            parts.append("".join(cur).strip())
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        parts.append("".join(cur).strip())
    return parts


def _parse_attrs(text: str) -> dict:
    attrs = {}
    for item in _split_top(text):
        key, _, val = item.partition("=")
        key, val = key.strip(), val.strip()
        m = re.fullmatch(r"array<i\d+:\s*(.*)>", val)
        if m:
            attrs[key] = tuple(int(v) for v in m.group(1).split(",") if v.strip())
            continue
        m = re.fullmatch(r"\[(.*)\]", val)
        if m:
            attrs[key] = tuple(int(v) for v in m.group(1).split(",") if v.strip())
            continue
        m = re.fullmatch(r"(-?\d+)\s*:\s*i\d+", val)
        if m:
            attrs[key] = int(m.group(1))
            continue
        attrs[key] = val
    return attrs


_FUNC_RE = re.compile(r"func\.func\s+@(\w+)\((.*?)\)\s*(?:->\s*(\(.*?\)|[^{]*?))?\s*"
                      r"(?:attributes\s*\{(.*)\})?\s*\{\s*$")


def parse_module(text: str) -> list[OFunc]:
    """Parse xt text (DSL output or the lit-test syntax) into OFunc objects."""
    lines = [ln.split("//")[0].rstrip() for ln in text.splitlines()]
    funcs: list[OFunc] = []
    cur: OFunc | None = None
    for ln in lines:
        s = ln.strip()
        if not s or s.startswith("module") or s == "}":
            if s == "}" and cur is not None:
                funcs.append(cur)
                cur = None
            continue
        if s.startswith("func.func"):
            m = _FUNC_RE.match(s)
            if not m:
                raise ValueError(f"oracle: cannot parse function header: {s}")
            args = []
            for a in _split_top(m.group(2)):
                n, _, t = a.partition(":")
                args.append((n.strip().lstrip("%"), parse_type(t)))
            cur = OFunc(m.group(1), args)
            if m.group(4):
                g = _parse_attrs(m.group(4)).get("xt.grid")
                if g is not None:
                    cur.grid = tuple(g)
            continue
        if cur is None:
            continue
        if s.startswith("func.return") or s.startswith("return"):
            continue
        cur.ops.append(_parse_op(s))
    if cur is not None:
        funcs.append(cur)
    return funcs


def _parse_op(s: str) -> OOp:
    results: list = []
    if "=" in s.split("(")[0]:
        lhs, _, s = s.partition("=")
        lhs = lhs.strip()
        m = re.fullmatch(r"%([\w.]+):(\d+)", lhs)
        if m:
            results = [f"%{m.group(1)}#{i}" for i in range(int(m.group(2)))]
        else:
            results = [lhs]
        s = s.strip()
    m = re.match(r"([\w.]+)", s)
    name = m.group(1)
    rest = s[m.end():].strip()
    if name == "arith.constant":
        val, _, typ = rest.rpartition(":")
        t = parse_type(typ)
        val = val.strip()
        dm = re.fullmatch(r"dense<(.*)>", val)
        value = float(dm.group(1)) if dm else int(val)
        return OOp(name, results, [], {"value": value}, [], t)
    if name == "xt.get_tile_block_id":
        return OOp(name, results, [], {}, [], None)
    operands: list = []
    if rest.startswith("("):
        depth = 0
        for i, ch in enumerate(rest):
            depth += ch == "("
            depth -= ch == ")"
            if depth == 0:
                operands = [o.strip() for o in rest[1:i].split(",") if o.strip()]
                rest = rest[i + 1:].strip()
                break
    attrs = {}
    if rest.startswith("{"):
        depth = 0
        for i, ch in enumerate(rest):
            depth += ch == "{"
            depth -= ch == "}"
            if depth == 0:
                attrs = _parse_attrs(rest[1:i])
                rest = rest[i + 1:].strip()
                break
    sig = rest.lstrip(":").strip()
    ins, _, out = sig.rpartition("->")
    ins = ins.strip()
    if ins.startswith("(") and ins.endswith(")"):
        ins = ins[1:-1]
    types_in = [parse_type(t) for t in _split_top(ins)]
    out = out.strip()
    type_out = None if out == "()" else parse_type(out)
    return OOp(name, results, operands, attrs, types_in, type_out)


# --------------------------------------------------------------------------
# semantics
# --------------------------------------------------------------------------
def serialize_order(grid: tuple) -> list[tuple[int, int, int]]:
    """Blocks in the reference's serialize order: z outer, y, x inner
    (``lib/xt/XTSerialize.cpp:68-70``)."""
    gx, gy, gz = grid
    return [(x, y, z) for z in range(gz) for y in range(gy) for x in range(gx)]


def tile_start(index: tuple, tile_shape: tuple) -> tuple:
    """Element start of a tile: index * tile dim (``XTToNova.cpp:98``)."""
    return tuple(i * d for i, d in zip(index, tile_shape))


def conv_spatial_slice(source_dim, result_index, result_dim, kernel_dim, pad_before,
                       stride, dilation):
    """Halo slice of one spatial dim -- restates ``computeConv2DSpatialSlice``
    (``lib/xt/XTToNova.cpp:110-142``).  Returns (load_start, load_size,
    conv_pad_before, conv_pad_after)."""
    result_start = result_index * result_dim
    receptive = (result_dim - 1) * stride + dilation * (kernel_dim - 1) + 1
    ideal_start = result_start * stride - pad_before
    ideal_end = ideal_start + receptive
    load_start = max(ideal_start, 0)
    pad_b = load_start - ideal_start
    load_end = min(load_start + (receptive - pad_b), source_dim)
    load_size = load_end - load_start
    pad_a = ideal_end - load_end
    if load_size <= 0 or pad_a < 0:
        raise ValueError("oracle: load_conv2d slice is empty")
    return load_start, load_size, pad_b, pad_a


def _read_tile(arr: np.ndarray, start: tuple, shape: tuple) -> np.ndarray:
    """Copy a tile; the part past the array edge reads zero."""
    out = np.zeros(shape, dtype=arr.dtype)
    src, dst = [], []
    for s, n, lim in zip(start, shape, arr.shape):
        lo, hi = max(s, 0), min(s + n, lim)
        if hi <= lo:
            return out
        src.append(slice(lo, hi))
        dst.append(slice(lo - s, hi - s))
    out[tuple(dst)] = arr[tuple(src)]
    return out


def _write_tile(arr: np.ndarray, start: tuple, tile: np.ndarray) -> None:
    src, dst = [], []
    for s, n, lim in zip(start, tile.shape, arr.shape):
        lo, hi = max(s, 0), min(s + n, lim)
        if hi <= lo:
            return
        dst.append(slice(lo, hi))
        src.append(slice(lo - s, hi - s))
    arr[tuple(dst)] = tile[tuple(src)]


def _as_compute(x: np.ndarray, elem: str) -> np.ndarray:
    """Tile values as the interpreter holds them: f32 for f32/bf16, int for i8."""
    if elem == "bf16":
        return bf16_to_f32(x)
    return x


def _to_storage(x: np.ndarray, elem: str) -> np.ndarray:
    if elem == "bf16":
        return f32_to_bf16(x.astype(np.float32))
    return x.astype(_NP_DTYPE[elem])


def ftoi_i8(x: np.ndarray) -> np.ndarray:
    """f32 -> int8: round half to even, saturate, NaN -> 0 (B200 choice)."""
    x = np.asarray(x, dtype=np.float32)
    r = np.rint(np.nan_to_num(x, nan=0.0, posinf=127.0, neginf=-128.0))
    return np.clip(r, -128, 127).astype(np.int8)


def _matmul(a: np.ndarray, b: np.ndarray, ea: str, eb: str) -> np.ndarray:
    if ea == "i8" and eb == "i8":
        return (a.astype(np.int64) @ b.astype(np.int64)).astype(np.float32)
    return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)


def _conv(src_slice: np.ndarray, filt: np.ndarray, pads, stride, dilation, out_shape) -> np.ndarray:
    """Direct conv of an NHWC slice with HWIO filter, exact accumulation."""
    n, oh, ow, oc = out_shape
    kh, kw, cin, _ = filt.shape
    pt, pl, pb, pr = pads
    x = np.pad(src_slice.astype(np.float64), ((0, 0), (pt, pb), (pl, pr), (0, 0)))
    f = filt.astype(np.float64)[..., :oc]
    out = np.zeros((n, oh, ow, oc), dtype=np.float64)
    sh, sw = stride
    dh, dw = dilation
    for r in range(kh):
        for s in range(kw):
            patch = x[:, r * dh: r * dh + (oh - 1) * sh + 1: sh,
                      s * dw: s * dw + (ow - 1) * sw + 1: sw, :]
            out += patch.reshape(-1, cin) .dot(f[r, s]).reshape(n, oh, ow, oc)
    return out.astype(np.float32)


_UNARY = {
    "xt.exp": lambda x: np.exp(x),
    "xt.cos": lambda x: np.cos(x),
    "xt.sin": lambda x: np.sin(x),
    "xt.reciprocal": lambda x: np.float32(1.0) / x,
    "xt.rsqrt": lambda x: np.float32(1.0) / np.sqrt(x),
    "xt.sigmoid": lambda x: (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32),
    "xt.tanh": lambda x: np.tanh(x),
    "xt.silu": lambda x: (x.astype(np.float64) / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32),
}


class Interpreter:
    """Executes one function over (a subset of) its grid on numpy arrays."""

    def __init__(self, func: OFunc):
        self.func = func

    def run(self, arrays: list[np.ndarray], blocks=None) -> None:
        memrefs = self.func.memref_args
        if len(arrays) != len(memrefs):
            raise ValueError(f"oracle: expected {len(memrefs)} arrays, got {len(arrays)}")
        for (name, t), a in zip(memrefs, arrays):
            if tuple(a.shape) != t.shape or a.dtype != _NP_DTYPE[t.elem]:
                raise ValueError(f"oracle: array %{name} must be {t.shape} {t.elem}")
        self.mem = {f"%{n}": a for (n, _), a in zip(memrefs, arrays)}
        self.elem = {f"%{n}": t.elem for n, t in self.func.args}
        order = serialize_order(self.func.grid) if blocks is None else blocks
        for block in order:
            self.run_block(block)

    def run_block(self, block: tuple) -> None:
        env: dict = {}
        elem = dict(self.elem)
        for op in self.func.ops:
            self.step(op, env, elem, block)

    def coord(self, env, name):
        return int(env[name])

    def step(self, op: OOp, env: dict, elem: dict, block: tuple) -> None:
        n = op.name
        if n == "xt.get_tile_block_id":
            for i, r in enumerate(op.results):
                env[r] = block[i]
            return
        if n == "arith.constant":
            v = op.attrs["value"]
            if op.type_out.kind == "tensor":
                env[op.results[0]] = np.full(op.type_out.shape, v, dtype=np.float32)
                elem[op.results[0]] = op.type_out.elem
            else:
                env[op.results[0]] = int(v)
            return
        if n == "xt.load":
            src = op.operands[0]
            t = op.type_out
            idx = tuple(self.coord(env, c) for c in op.operands[1:])
            tile = _read_tile(self.mem[src], tile_start(idx, t.shape), t.shape)
            env[op.results[0]] = _as_compute(tile, t.elem)
            elem[op.results[0]] = t.elem
            return
        if n == "xt.store":
            val, dst = op.operands[0], op.operands[1]
            idx = tuple(self.coord(env, c) for c in op.operands[2:])
            tile = env[val]
            _write_tile(self.mem[dst], tile_start(idx, tile.shape), _to_storage(tile, self.elem[dst]))
            return
        if n == "xt.load_conv2d":
            self.load_conv2d(op, env, elem)
            return
        args = [env[o] for o in op.operands]
        t = op.type_out
        res = op.results[0]
        elem[res] = t.elem
        if n in ("xt.add", "xt.sub", "xt.mul"):
            a, b = args
            fn = {"xt.add": np.add, "xt.sub": np.subtract, "xt.mul": np.multiply}[n]
            if t.elem == "i8":
                r = fn(a.astype(np.int32), b.astype(np.int32)).astype(np.int8)
            else:
                r = fn(a.astype(np.float32), b.astype(np.float32))
            env[res] = np.broadcast_to(r, t.shape).astype(r.dtype)
        elif n in _UNARY:
            with np.errstate(all="ignore"):
                env[res] = _UNARY[n](args[0].astype(np.float32)).astype(np.float32)
        elif n in ("xt.reduce_max", "xt.reduce_sum"):
            axis = op.attrs["axis"]
            x = args[0]
            if n == "xt.reduce_max":
                env[res] = np.max(x, axis=axis, keepdims=True)
            else:
                env[res] = np.sum(x.astype(np.float64), axis=axis, keepdims=True).astype(np.float32)
        elif n == "xt.matmul":
            ea, eb = elem[op.operands[0]], elem[op.operands[1]]
            env[res] = _matmul(args[0], args[1], ea, eb)
        elif n == "xt.mma":
            ea, eb = elem[op.operands[0]], elem[op.operands[1]]
            env[res] = (args[2].astype(np.float32) + _matmul(args[0], args[1], ea, eb)).astype(np.float32)
        elif n == "xt.itof":
            env[res] = args[0].astype(np.float32)
        elif n == "xt.ftoi":
            env[res] = ftoi_i8(args[0])
        elif n == "xt.reshape":
            env[res] = args[0].reshape(t.shape)
        elif n == "xt.transpose":
            env[res] = np.ascontiguousarray(np.swapaxes(args[0], 1, 2))
        elif n == "xt.permute":
            env[res] = np.ascontiguousarray(np.transpose(args[0], op.attrs["permutation"]))
        else:
            raise ValueError(f"oracle: unsupported op {n}")

    def load_conv2d(self, op: OOp, env: dict, elem: dict) -> None:
        src = self.mem[op.operands[0]]
        src_elem = self.elem[op.operands[0]]
        filt = env[op.operands[1]]
        ib, ih, iw, ic = (self.coord(env, c) for c in op.operands[2:6])
        out_shape = op.type_out.shape
        kh, kw, cin, _ = filt.shape
        pad = op.attrs["pad"]
        stride = op.attrs["stride"]
        dilation = op.attrs["dilation"]
        hs = conv_spatial_slice(src.shape[1], ih, out_shape[1], kh, pad[0], stride[0], dilation[0])
        ws = conv_spatial_slice(src.shape[2], iw, out_shape[2], kw, pad[1], stride[1], dilation[1])
        start = (ib * out_shape[0], hs[0], ws[0], ic * cin)
        shape = (out_shape[0], hs[1], ws[1], cin)
        slab = _as_compute(_read_tile(src, start, shape), src_elem)
        env[op.results[0]] = _conv(slab, filt, (hs[2], ws[2], hs[3], ws[3]), stride, dilation,
                                   out_shape)
        elem[op.results[0]] = "f32"


def run(text: str, arrays: list[np.ndarray], func: str | None = None, blocks=None) -> None:
    """Interpret the (first or named) function of ``text`` in place on ``arrays``."""
    funcs = parse_module(text)
    f = funcs[0] if func is None else next(fn for fn in funcs if fn.name == func)
    Interpreter(f).run(arrays, blocks=blocks)
