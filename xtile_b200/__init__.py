"""xtile_b200: a B200-native execution backend for the xtile tile DSL.

The DSL surface is the reference's (``xtile`` of sjjeong94/xtile): write a
Block program with ``xt.bid``/``xt.load``/``xt.store`` and tile ops, convert
it, and -- new here -- launch it on a B200 with ``launch``/``run``.  The
package ``xtile`` at the repository root re-exports this one under the
reference's import name, so ``import xtile as xt`` scripts run unchanged.
"""
from .dsl import (
    Array,
    DType,
    add,
    astype,
    bfloat16,
    bid,
    cos,
    exp,
    float32,
    int8,
    kernel,
    load,
    load_conv2d,
    matmul,
    max,
    mma,
    mul,
    reciprocal,
    reshape,
    rsqrt,
    sigmoid,
    silu,
    sin,
    store,
    sub,
    sum,
    tanh,
    transpose,
    truediv,
)
from .api import (
    Module,
    _module_asm,
    _parse_module,
    canonicalize,
    cdiv,
    compile,
    convert,
    nova_allocate,
    nova_barrier,
    nova_optimize,
    nova_threading,
    nova_to_x1,
    parse,
    save_compile_results,
    save_ir,
    xt_serialize,
    xt_to_nova,
)
from .runtime import PeerArray, device_error, export_array, launch, run, sm_budget, wait_limit

__all__ = [
    "Array", "DType", "Module", "PeerArray", "add", "astype", "bfloat16", "bid", "canonicalize", "cdiv", "compile",
    "convert",
    "cos", "device_error", "exp", "export_array", "float32", "int8", "kernel", "launch", "load", "load_conv2d",
    "matmul", "max", "mma", "mul", "nova_allocate", "nova_barrier", "nova_optimize",
    "nova_threading", "nova_to_x1", "parse", "reciprocal", "reshape", "rsqrt", "run",
    "save_compile_results", "save_ir", "sigmoid", "silu", "sin", "sm_budget", "store", "sub", "sum", "tanh",
    "transpose", "truediv", "wait_limit", "xt_serialize", "xt_to_nova",
]
