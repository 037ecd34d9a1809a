"""Launching Block programs on B200 GPUs.

The reference cannot execute a program; this is the new part of the
interface.  ``launch`` runs a converted/parsed module on torch CUDA tensors
(one per memref argument, in signature order), writing the stored arrays in
place -- the DSL's ``xt.store`` into a mutable Array.  ``bid0_range`` runs
only the Blocks whose ``xt.bid(0)`` lies in ``[lo, hi)``: one process per GPU
passes its own range to split a Grid across GPUs.

Tensors must be contiguous, on one CUDA device, with exactly the memref's
shape and dtype (float32 / bfloat16 / int8), 16-byte aligned.  The launch is
asynchronous on ``stream`` (default: torch's current stream of that device).
"""
from __future__ import annotations

from typing import Sequence

from . import dsl
from ._native import native as _native
from .api import Module, convert

_TORCH_DTYPES = None


def _dtype_map():
    global _TORCH_DTYPES
    if _TORCH_DTYPES is None:
        import torch

        _TORCH_DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "i8": torch.int8}
    return _TORCH_DTYPES


def _signature(module: Module, func: str | None):
    cache = module.__dict__.setdefault("_launch_sig", {})
    sig = cache.get(func)
    if sig is None:
        dtypes = _dtype_map()
        sig = cache[func] = [(name, is_memref, elem, tuple(shape), dtypes.get(elem))
                             for name, is_memref, elem, shape in module.arguments(func)]
    return sig


class PeerArray:
    """An array in another GPU's memory, mapped into this process over NVLink.

    ``export_array(t)`` on the owning process gives a picklable handle;
    ``PeerArray.open(handle, shape, dtype)`` maps it here.  ``launch`` takes a
    PeerArray wherever it takes a tensor: the kernel reads or writes the
    owner's memory directly (the sharded matmul stores its rows straight into
    rank 0's output this way, with no separate gather).
    """

    def __init__(self, base: int, offset: int, shape: tuple, dtype) -> None:
        self._base = base
        self.ptr = base + offset
        self.shape = tuple(shape)
        self.dtype = dtype

    @classmethod
    def open(cls, handle: tuple, shape: tuple, dtype) -> "PeerArray":
        blob, offset = handle
        return cls(int(_native.ipc_open(blob)), int(offset), shape, dtype)

    def data_ptr(self) -> int:
        return self.ptr

    def close(self) -> None:
        if self._base:
            _native.ipc_close(self._base)
            self._base = 0


def export_array(t) -> tuple:
    """Picklable CUDA IPC handle of tensor ``t`` for ``PeerArray.open``."""
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("export_array: a contiguous CUDA tensor is required")
    blob, offset = _native.ipc_export(t.data_ptr())
    return bytes(blob), int(offset)


def _check_arrays(module: Module, arrays: Sequence, func: str | None):
    import torch

    sig = _signature(module, func)
    if len(arrays) != len(sig):
        raise ValueError(f"launch expects {len(sig)} arrays "
                         f"({', '.join('%' + s[0] for s in sig)}), got {len(arrays)}")
    device = None
    for t, (name, is_memref, elem, shape, dtype) in zip(arrays, sig):
        if not is_memref:
            raise TypeError(f"argument %{name} is not a memref; only memref kernels can be launched")
        if isinstance(t, PeerArray):
            if dtype is None or t.dtype != dtype:
                raise TypeError(f"array %{name} must be {elem}, got {t.dtype}")
            if t.shape != shape:
                raise ValueError(f"array %{name} must have shape {shape}, got {t.shape}")
            continue
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"array %{name} must be a torch tensor, got {type(t).__name__}")
        if not t.is_cuda:
            raise ValueError(f"array %{name} must be a CUDA tensor")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError(f"array %{name} is on {t.device}, expected {device}")
        if dtype is None or t.dtype != dtype:
            raise TypeError(f"array %{name} must be {elem}, got {t.dtype}")
        if t.shape != shape:
            raise ValueError(f"array %{name} must have shape {shape}, got {tuple(t.shape)}")
        if not t.is_contiguous():
            raise ValueError(f"array %{name} must be contiguous (row-major)")
    if device is None:
        raise ValueError("launch needs at least one local CUDA tensor to pick the device")
    return device


def launch(module: Module, *arrays, func: str | None = None, stream=None,
           bid0_range: tuple[int, int] | None = None) -> None:
    """Run the Block program of ``func`` (default: the first) over its grid."""
    import torch

    device = _check_arrays(module, arrays, func)
    if stream is None:
        stream = torch.cuda.current_stream(device)
    handle = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
    lo, hi = (0, 0) if bid0_range is None else bid0_range
    if bid0_range is not None and hi <= lo:
        return
    ptrs = [t.data_ptr() for t in arrays]
    if torch.cuda.current_device() == device.index:
        _native.launch(module._CAPIPtr, ptrs, int(lo), int(hi), int(handle), func)
    else:
        with torch.cuda.device(device):
            _native.launch(module._CAPIPtr, ptrs, int(lo), int(hi), int(handle), func)


def run(kernel_fn: dsl.KernelFunction, *, args: tuple, grid: tuple, double_buffering: bool = False,
        stream=None, bid0_range: tuple[int, int] | None = None) -> Module:
    """Trace ``kernel_fn`` with tensors standing in for Arrays, then launch it.

    ``args`` mixes torch tensors (one per Array parameter) and ints (compile
    time constants), in the kernel's parameter order.  Returns the module, so
    a caller can launch it again without re-tracing.
    """
    import torch

    elems = {torch.float32: dsl.float32, torch.bfloat16: dsl.bfloat16, torch.int8: dsl.int8}
    trace_args, tensors = [], []
    for a in args:
        if isinstance(a, torch.Tensor):
            if a.dtype not in elems:
                raise TypeError(f"unsupported tensor dtype {a.dtype}")
            trace_args.append(dsl.Array(shape=tuple(int(d) for d in a.shape), dtype=elems[a.dtype]))
            tensors.append(a)
        else:
            trace_args.append(a)
    module = convert(kernel_fn, args=tuple(trace_args), grid=grid, double_buffering=double_buffering)
    launch(module, *tensors, stream=stream, bid0_range=bid0_range)
    return module


def device_error() -> int:
    """Reads and clears the current device's kernel error word (0: none)."""
    return int(_native.device_error())


class wait_limit:
    """Limits how long a pipeline wait of the gemm and conv kernels launched
    by this thread inside a ``with`` block may take, in nanoseconds, before
    the kernel gives up, records an error code (``device_error()``), drains
    and returns.  For testing the failure path; the default is about 2 s."""

    def __init__(self, ns: int) -> None:
        self.ns = int(ns)

    def __enter__(self) -> "wait_limit":
        _native.set_wait_limit_ns(self.ns)
        return self

    def __exit__(self, *exc) -> None:
        _native.set_wait_limit_ns(0)


class sm_budget:
    """Caps the SMs the persistent kernels (gemm, conv) launched by this
    thread occupy, for the duration of a ``with`` block (0: all SMs).

    Used when a launch runs beside a communication kernel, e.g. the NCCL
    gather of the previous step's rows: the kernel leaves the other SMs to the
    collective so the two overlap instead of queueing behind each other.
    """

    def __init__(self, sms: int) -> None:
        self.sms = int(sms)

    def __enter__(self) -> "sm_budget":
        _native.set_sm_budget(self.sms)
        return self

    def __exit__(self, *exc) -> None:
        _native.set_sm_budget(0)
