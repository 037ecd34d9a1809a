"""Benchmark of the B200 xtile backend (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl b200|reference]

Workloads are the BASELINE configurations (synthetic, seeded inputs):

  add             fp32 [2048,2048] + [2048,2048], 32x64 Block tiles, grid (64,32)
  softmax         fp32 [8192,1024] row softmax, 1x1024 Block tiles, grid (8192,)
  matmul          bf16 4096^3, fp32 out, 128x128 Block tiles, K-step 64, grid (32,32)
  conv2d          NHWC bf16 [32,56,56,64] * [3,3,64,64], pad 1, fp32 out
  sharded_matmul  bf16 [32768,8192] x [8192,8192], fp32 out, 256x128 Block tiles,
                  grid (128,64) split along bid0 across ranks, output rows
                  gathered to rank 0 over NVLink by peer stores from the GEMM
                  (--gather nccl: an NCCL gather; the default workload)
  transpose, silu, row_center, row_bias
                  not BASELINE configurations: the data-movement kernel and the
                  generated ew and rows kernels on f32 programs over 128 MiB
  matmul_i8       not a BASELINE configuration: the reference's int8
                  kernels/matmul.py program (scale, bias, int8 out) at 8192^3
  col_sums        not a BASELINE configuration: a generated tile kernel
                  (column sums of 64 x 32 tiles of a 128 MiB f32 array)
  softmax_wide    not a BASELINE configuration: kernels/softmax.py's program on
                  [4096, 8192] (a generated kernel, one CTA per row)
  col_bias        not a BASELINE configuration: a generated tile kernel whose
                  elementwise ops run as one pass (sigmoid(t * c - c), c a
                  column broadcast over 32 x 64 tiles)

A step is one launch of the workload's Block program over its whole Grid
(for sharded_matmul: every rank's share plus the gather).  ``value`` is the
whole-job throughput with inputs resident in HBM; ``e2e`` repeats the step
through the public ``xtile.launch`` API with pinned host inputs copied in and
the result copied out inside the timed region.  ``--impl reference`` times the
reference path on the host CPU instead: the reference (sjjeong94/xtile)
executes nothing, so its arm is the CPU oracle restating its semantics
(``oracle/xt_oracle.py``) on a bounded sample of the workload.

On one GPU the default line also carries ``per_config`` (BASELINE
configurations 1-4) and ``generated`` (one workload of each kind of kernel
generated per program: silu, row_center, softmax_wide, col_bias), each timed,
put against its roofline and checked against the oracle on sampled Blocks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "TFLOP/s (matmul/conv) & HBM GB/s (add/softmax) vs B200 peak, 1–8 GPUs"
L2_BYTES = 126 * 2 ** 20
OPS_UNITS = ("TFLOP/s", "TOP/s")  # tensor-core work counted in multiply-add ops (bf16 / int8)


def launch_arrays(w: dict, ins: list, out) -> list:
    """The program's arrays in signature order: the output sits at w["out_pos"] (last by default)."""
    pos = w.get("out_pos", len(ins))
    return [*ins[:pos], out, *ins[pos:]]
# SMs the sharded GEMM leaves to the NCCL gather it overlaps, and NCCL's
# channel cap.  On 2 B200s, 16 free SMs did not let the gather's kernels run
# beside the GEMM at all (it waited for the GEMM to finish); 32 did.
GATHER_SMS = 32
GATHER_CHANNELS = 16
# Rank 0's share of the sharded GEMM when the other ranks store their rows into
# its memory: rank 0's NVLink ingress, not compute, bounds the step at 4 and 8
# GPUs, and rank 0's own rows never cross NVLink.  The share balances rank 0's
# compute against that ingress using two rates measured on B200s: the rows the
# other ranks' kernels deliver into rank 0 while it computes (640-680 GB/s at
# 4 and 8 GPUs) and the single-GPU rate of this GEMM (about 1450 TFLOP/s).
PEER_INGEST_GBS = 680.0
SHARDED_GEMM_TFLOPS = 1450.0
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM bytes per launch of the dominant kernel from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum), summarised in profiles/.
# ncu flushes the caches before the capture, so output bytes still in L2 when
# the kernel ends are not in these figures (they are written back later).
NCU_TRAFFIC_BYTES: dict[str, float] = {
    "matmul": 89_688_320 + 40_005_376,
    "conv2d": 12_960_768 + 2_304,
    "add": 33_561_088 + 10_496,
    "softmax": 33_566_464 + 343_552,
    "sharded_matmul": 6_210_000_000 + 1_060_000_000,
    "transpose": 134_243_200 + 82_835_968,
    "matmul_i8": 215_210_496 + 55_281_408,
    "silu": 134_240_512 + 84_709_376,
    "row_center": 134_223_360 + 78_821_120,
    "col_sums": 134_223_360 + 4_445_056,
    "col_bias": 134_317_056 + 81_739_648,
    "softmax_wide": 134_230_784 + 77_903_104,
}


# ---------------------------------------------------------------- workloads
def build_workload(name: str, xt, torch, world: int, rank: int):
    """The workload ``name``: its Block program's xt text and seeded host inputs.

    ``xt`` is the DSL namespace (``xtile_b200/dsl.py``, which is pure Python):
    the text is traced here without the native library, so the reference arm
    can use it too.  ``work`` is the algorithmic work of one full launch
    (bytes for HBM-bound programs, FLOP or int8 ops for the tensor-core ones),
    from the configuration's own formula.
    """
    g = torch.Generator().manual_seed
    A = xt.Array
    if name == "add":
        @xt.kernel
        def add_tiles(lhs, rhs, out, th, tw):
            i, j = xt.bid(0), xt.bid(1)
            a = xt.load(lhs, index=(i, j), shape=(th, tw))
            b = xt.load(rhs, index=(i, j), shape=(th, tw))
            xt.store(out, index=(i, j), tile=a + b)

        gen = g(0)
        a = torch.rand(2048, 2048, generator=gen) * 2 - 1
        b = torch.rand(2048, 2048, generator=gen) * 2 - 1
        args = (A((2048, 2048), xt.float32),) * 3
        text = xt.trace_text(add_tiles, args=(*args, 32, 64), grid=(64, 32, 1), double_buffering=True)
        return dict(text=text, inputs=[a, b], out_shape=(2048, 2048), out_dtype=torch.float32,
                    unit="GB/s", dtype="f32", work=3 * 2048 * 2048 * 4,
                    config={"workload": "add", "shape": [2048, 2048], "block_tile": [32, 64],
                            "grid": [64, 32, 1]})
    if name in ("softmax", "softmax_wide"):
        @xt.kernel
        def softmax_rows(inp, out, trow, col):
            i = xt.bid(0)
            x = xt.load(inp, index=(i, 0), shape=(trow, col))
            x = x - xt.max(x, axis=-1)
            x = xt.exp(x)
            xt.store(out, index=(i, 0), tile=x / xt.sum(x, axis=-1))

        if name == "softmax_wide":
            # not a BASELINE configuration: the same program on rows wider
            # than the dedicated kernel takes (a generated kernel, one CTA
            # per row)
            R, C = 4096, 8192
            x = torch.randn(R, C, generator=g(12)) * 4
            F = xt.float32
            text = xt.trace_text(softmax_rows, args=(A((R, C), F), A((R, C), F), 1, C), grid=(R, 1, 1),
                                 double_buffering=True)
            return dict(text=text, inputs=[x], out_shape=(R, C), out_dtype=torch.float32, unit="GB/s", dtype="f32",
                        work=2 * R * C * 4, tolerance="softmax",
                        config={"workload": name, "shape": [R, C], "block_tile": [1, C], "grid": [R, 1, 1]})
        x = torch.randn(8192, 1024, generator=g(1)) * 4
        text = xt.trace_text(softmax_rows, args=(A((8192, 1024), xt.float32), A((8192, 1024), xt.float32),
                                                 1, 1024), grid=(8192, 1, 1), double_buffering=True)
        return dict(text=text, inputs=[x], out_shape=(8192, 1024), out_dtype=torch.float32,
                    unit="GB/s", dtype="f32", work=2 * 8192 * 1024 * 4, tolerance="softmax",
                    config={"workload": "softmax", "shape": [8192, 1024], "block_tile": [1, 1024],
                            "grid": [8192, 1, 1]})
    if name in ("matmul", "sharded_matmul"):
        if name == "matmul":
            M = N = K = 4096
            tm, tn, tk, seed = 128, 128, 64, 2
        else:
            M, N, K = 32768, 8192, 8192
            tm, tn, tk, seed = 256, 128, K, 4

        @xt.kernel
        def matmul_kloop(lhs, rhs, out, tm, tn, tk, ksteps):
            i, j = xt.bid(0), xt.bid(1)
            acc = None
            for k in range(ksteps):
                p = xt.matmul(xt.load(lhs, index=(i, k), shape=(tm, tk)),
                              xt.load(rhs, index=(k, j), shape=(tk, tn), shared=1))
                acc = p if acc is None else acc + p
            xt.store(out, index=(i, j), tile=acc)

        gen = g(seed)
        s = 1.0 / (K ** 0.5)
        a = (torch.randn(M, K, generator=gen) * s).to(torch.bfloat16)
        b = (torch.randn(K, N, generator=gen) * s).to(torch.bfloat16)
        grid = (M // tm, N // tn, 1)
        text = xt.trace_text(matmul_kloop, args=(A((M, K), xt.bfloat16), A((K, N), xt.bfloat16),
                                                 A((M, N), xt.float32), tm, tn, tk, K // tk),
                             grid=grid, double_buffering=True)
        cfg = {"workload": name, "M": M, "N": N, "K": K, "block_tile": [tm, tn], "k_step": tk,
               "grid": list(grid)}
        if name == "sharded_matmul":
            cfg["parallelism"] = ("one GPU, the whole Grid" if world == 1 else
                                  f"bid0 split over {world} GPUs, NCCL gather of C rows to rank 0")
        return dict(text=text, inputs=[a, b], out_shape=(M, N), out_dtype=torch.float32,
                    unit="TFLOP/s", dtype="bf16", config=cfg, sharded=name == "sharded_matmul", work=2 * M * N * K)
    if name == "conv2d":
        @xt.kernel
        def conv2d_bf16(inp, filt, out, tile_h, tile_w, cin, cout, kh, kw):
            n, h, w = xt.bid(0), xt.bid(1), xt.bid(2)
            f = xt.load(filt, index=(0, 0, 0, 0), shape=(kh, kw, cin, cout), shared=2)
            y = xt.load_conv2d(inp, f, index=(n, h, w, 0), shape=(1, tile_h, tile_w, cout), group=1,
                               pad=(kh // 2, kw // 2, kh // 2, kw // 2), stride=(1, 1), dilation=(1, 1))
            xt.store(out, index=(n, h, w, 0), tile=y)

        gen = g(3)
        x = (torch.randn(32, 56, 56, 64, generator=gen) * 0.1).to(torch.bfloat16)
        f = (torch.randn(3, 3, 64, 64, generator=gen) * 0.1).to(torch.bfloat16)
        text = xt.trace_text(conv2d_bf16, args=(A((32, 56, 56, 64), xt.bfloat16), A((3, 3, 64, 64), xt.bfloat16),
                                                A((32, 56, 56, 64), xt.float32), 8, 56, 64, 64, 3, 3),
                             grid=(32, 7, 1), double_buffering=True)
        # implicit GEMM: M = 32*56*56 output pixels, N = 64 channels, K = 3*3*64
        return dict(text=text, inputs=[x, f], out_shape=(32, 56, 56, 64), out_dtype=torch.float32,
                    unit="TFLOP/s", dtype="bf16", work=2 * (32 * 56 * 56) * 64 * (3 * 3 * 64),
                    config={"workload": "conv2d", "input": [32, 56, 56, 64], "filter": [3, 3, 64, 64],
                            "pad": 1, "block_tile": [1, 8, 56, 64], "grid": [32, 7, 1]})
    if name == "transpose":
        # not a BASELINE configuration: the tile family on an HBM-bound program
        @xt.kernel
        def transpose3(inp, out, tm, tn):
            b, i, j = xt.bid(0), xt.bid(1), xt.bid(2)
            t = xt.load(inp, index=(b, i, j), shape=(1, tm, tn))
            xt.store(out, index=(b, j, i), tile=xt.transpose(t))

        x = torch.randn(8, 2048, 2048, generator=g(5))
        text = xt.trace_text(transpose3, args=(A((8, 2048, 2048), xt.float32), A((8, 2048, 2048), xt.float32),
                                               32, 64), grid=(8, 64, 32), double_buffering=True)
        return dict(text=text, inputs=[x], out_shape=(8, 2048, 2048), out_dtype=torch.float32,
                    unit="GB/s", dtype="f32", work=2 * 8 * 2048 * 2048 * 4,
                    config={"workload": "transpose", "shape": [8, 2048, 2048], "block_tile": [1, 32, 64],
                            "grid": [8, 64, 32]})
    if name == "matmul_i8":
        # not a BASELINE configuration: the reference's kernels/matmul.py
        # Block program as written (int8 A, B; 64 x 64 Blocks over the whole K;
        # t * scale + bias; int8 result) at 8192^3 on the int8 tensor cores
        @xt.kernel
        def matmul_kernel(lhs, rhs, res, scale, bias, tm, tn, tk):
            bid_x, bid_y = xt.bid(0), xt.bid(1)
            lhs_tile = xt.load(lhs, index=(bid_x, 0), shape=(tm, tk))
            rhs_tile = xt.load(rhs, index=(0, bid_y), shape=(tk, tn), shared=1)
            s_tile = xt.load(scale, index=(0, bid_y), shape=(1, tn), shared=1)
            b_tile = xt.load(bias, index=(0, bid_y), shape=(1, tn), shared=1)
            t = xt.matmul(lhs_tile, rhs_tile)
            t = t * s_tile + b_tile
            xt.store(res, index=(bid_x, bid_y), tile=xt.astype(t, dtype=xt.int8))

        M = N = K = 8192
        gen = g(8)
        a = torch.randint(-128, 128, (M, K), generator=gen, dtype=torch.int8)
        b = torch.randint(-128, 128, (K, N), generator=gen, dtype=torch.int8)
        s = torch.rand(1, N, generator=gen) * 1e-5
        bias = torch.rand(1, N, generator=gen) * 16 - 8
        I8, F = xt.int8, xt.float32
        text = xt.trace_text(matmul_kernel, args=(A((M, K), I8), A((K, N), I8), A((M, N), I8), A((1, N), F),
                                                  A((1, N), F), 64, 64, K), grid=(M // 64, N // 64, 1),
                             double_buffering=True)
        return dict(text=text, inputs=[a, b, s, bias], out_pos=2, out_shape=(M, N), out_dtype=torch.int8,
                    unit="TOP/s", dtype="int8", work=2 * M * N * K,
                    config={"workload": name, "M": M, "N": N, "K": K, "block_tile": [64, 64], "k_step": K,
                            "grid": [M // 64, N // 64, 1], "epilogue": "t * scale + bias, int8 (round half even, saturate)"})
    if name in ("silu", "row_center", "row_bias"):
        # not BASELINE configurations: the generated ew and rows kernels
        # on HBM-bound f32 programs over 128 MiB arrays (row_bias: a
        # broadcast row, which the ew kernel reads as element i mod C)
        R, C = (32768, 1024) if name == "row_center" else (16384, 2048)
        x = torch.randn(R, C, generator=g(6))
        F = xt.float32
        if name == "silu":
            @xt.kernel
            def silu_rows(inp, out, trow, col):
                i = xt.bid(0)
                t = xt.load(inp, index=(i, 0), shape=(trow, col))
                xt.store(out, index=(i, 0), tile=t * xt.sigmoid(t))

            text = xt.trace_text(silu_rows, args=(A((R, C), F), A((R, C), F), 16, C), grid=(R // 16, 1, 1),
                                 double_buffering=True)
            inputs, tile, grid, work = [x], [16, C], [R // 16, 1, 1], 2 * R * C * 4
            tol = "transcendental"
        elif name == "row_center":
            @xt.kernel
            def row_center(inp, out, trow, col):
                i = xt.bid(0)
                t = xt.load(inp, index=(i, 0), shape=(trow, col))
                m = xt.max(t, axis=1)
                xt.store(out, index=(i, 0), tile=(t - m) * (t - m))

            text = xt.trace_text(row_center, args=(A((R, C), F), A((R, C), F), 1, C), grid=(R, 1, 1),
                                 double_buffering=True)
            inputs, tile, grid, work = [x], [1, C], [R, 1, 1], 2 * R * C * 4
            tol = "bit-exact"
        else:
            @xt.kernel
            def row_bias(inp, vec, out, tm, tn):
                i, j = xt.bid(0), xt.bid(1)
                t = xt.load(inp, index=(i, j), shape=(tm, tn))
                r = xt.load(vec, index=(0, j), shape=(1, tn), shared=1)
                xt.store(out, index=(i, j), tile=t * r + r)

            v = torch.randn(1, C, generator=g(7))
            text = xt.trace_text(row_bias, args=(A((R, C), F), A((1, C), F), A((R, C), F), 32, 256),
                                 grid=(R // 32, C // 256, 1), double_buffering=True)
            # the broadcast row is read once
            inputs, tile, grid, work = [x, v], [32, 256], [R // 32, C // 256, 1], (2 * R * C + C) * 4
            tol = "bit-exact"
        return dict(text=text, inputs=inputs, work=work, tolerance=tol, out_shape=(R, C), out_dtype=torch.float32, unit="GB/s", dtype="f32",
                    config={"workload": name, "shape": [R, C], "block_tile": tile, "grid": grid})
    if name == "col_sums":
        # not a BASELINE configuration: a tile program (column sums of 64 x 32
        # tiles, float64 accumulation) over a 128 MiB f32 array
        @xt.kernel
        def col_sums(x, out, tm, tn):
            i, j = xt.bid(0), xt.bid(1)
            t = xt.load(x, index=(i, j), shape=(tm, tn))
            xt.store(out, index=(i, j), tile=xt.sum(t, axis=0))

        R, C, tm, tn = 16384, 2048, 64, 32
        x = torch.randn(R, C, generator=g(9))
        text = xt.trace_text(col_sums, args=(A((R, C), xt.float32), A((R // tm, C), xt.float32), tm, tn),
                             grid=(R // tm, C // tn, 1), double_buffering=True)
        return dict(text=text, inputs=[x], work=(R * C + R // tm * C) * 4, tolerance="sum", out_shape=(R // tm, C),
                    out_dtype=torch.float32, unit="GB/s", dtype="f32",
                    config={"workload": name, "shape": [R, C], "block_tile": [tm, tn], "grid": [R // tm, C // tn, 1]})
    if name == "col_bias":
        # not a BASELINE configuration: a tile program whose elementwise ops
        # run as one pass (sigmoid(t * c - c), c a (32, 1) column of a [R, 1]
        # array) over a 128 MiB f32 array
        @xt.kernel
        def col_bias(x, c, out, tm, tn):
            i, j = xt.bid(0), xt.bid(1)
            t = xt.load(x, index=(i, j), shape=(tm, tn))
            s = xt.load(c, index=(i, 0), shape=(tm, 1))
            xt.store(out, index=(i, j), tile=xt.sigmoid(t * s - s))

        R, C, tm, tn = 16384, 2048, 32, 64
        x = torch.randn(R, C, generator=g(10))
        col = torch.randn(R, 1, generator=g(11))
        F = xt.float32
        text = xt.trace_text(col_bias, args=(A((R, C), F), A((R, 1), F), A((R, C), F), tm, tn),
                             grid=(R // tm, C // tn, 1), double_buffering=True)
        # bytes of every Block's tiles: each of the C / tn Blocks of a row of
        # tiles loads its (32, 1) column (from L2 after the first)
        return dict(text=text, inputs=[x, col], work=(2 * R * C + R * (C // tn)) * 4, tolerance="transcendental",
                    out_shape=(R, C), out_dtype=torch.float32, unit="GB/s", dtype="f32",
                    config={"workload": name, "shape": [R, C], "block_tile": [tm, tn], "grid": [R // tm, C // tn, 1]})
    raise SystemExit(f"unknown workload {name}")


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clocks, power and clock-event (throttle) reasons during the timed region.

    NVML is read from a thread every 10 ms, so even a timed region of a few tens
    of milliseconds gets samples; without NVML, ``nvidia-smi -lms 50`` is used.
    Reading is all either does: no clock or power setting is changed.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvmlClocksEventReason*)
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpu_id: str):
        self.gpu = gpu_id
        self.proc = None
        self.thread = None
        self.rows: list[tuple[float, float, float, int]] = []
        self.file = None

    def _nvml_loop(self, nvml, handle, stop):
        max_sm = float(nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM))
        while not stop.is_set():
            try:
                sm = float(nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM))
                reasons = int(nvml.nvmlDeviceGetCurrentClocksEventReasons(handle))
                power = nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                self.rows.append((sm, max_sm, power, reasons))
            except Exception:  # noqa: BLE001 - a failed read just drops the sample
                pass
            stop.wait(0.01)

    def __enter__(self):
        import threading
        try:
            import pynvml as nvml
            nvml.nvmlInit()
            handle = nvml.nvmlDeviceGetHandleByUUID(self.gpu)
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._nvml_loop, args=(nvml, handle, self.stop), daemon=True)
            self.thread.start()
            t0 = time.monotonic()
            while not self.rows and time.monotonic() - t0 < 5.0:
                time.sleep(0.005)
            return self
        except Exception:  # noqa: BLE001 - no NVML: fall back to nvidia-smi
            self.thread = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        # nvidia-smi takes a while to start (longer with 8 GPUs visible): wait
        # for its first row, so the samples cover the timed region that follows
        t0 = time.monotonic()
        while self.proc is not None and time.monotonic() - t0 < 10.0:
            if self.proc.poll() is not None or os.path.getsize(self.file.name) > 0:
                break
            time.sleep(0.02)
        time.sleep(0.06)
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        if self.file is not None:
            self.file.flush()
            for line in Path(self.file.name).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    bits = 0
                    for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                        "sw_power_cap"), parts[5:9]):
                        if v.lower() == "active":
                            bits |= self.REASON_BITS[name]
                    power = float(parts[3]) if parts[3][:1].isdigit() else 0.0
                    rows.append((float(parts[1]), float(parts[2]), power, bits))
            os.unlink(self.file.name)
        else:
            rows = list(self.rows)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        reasons = sorted({n for r in rows for n, bit in self.REASON_BITS.items() if r[3] & bit})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_min_mhz": min(r[0] for r in rows),
                "sm_max_mhz": rows[0][1], "reasons": reasons, "samples": len(rows),
                "power_w_max": max(r[2] for r in rows),
                "source": "nvml, 10 ms" if self.file is None else "nvidia-smi, 50 ms"}


# ---------------------------------------------------------------- helpers
def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except ValueError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def oracle_arrays(w: dict, torch) -> list:
    """The workload's arrays as the oracle takes them (numpy, bf16 as uint16 bits), output zeroed."""
    import numpy as np

    arrays = [t.view(torch.uint16).numpy() if t.dtype == torch.bfloat16 else t.numpy() for t in w["inputs"]]
    out = np.zeros(w["out_shape"], dtype=np.int8 if w["out_dtype"] == torch.int8 else np.float32)
    arrays.insert(w.get("out_pos", len(arrays)), out)
    return arrays


def load_dsl():
    """``xtile_b200/dsl.py`` loaded by path: the tracer is pure Python, and
    importing the package would load the native library."""
    import importlib.util

    name = "xt_bench_dsl"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, ROOT / "xtile_b200" / "dsl.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def oracle_rate(w: dict, done: int, secs: float, n_blocks: int) -> float:
    """Throughput in the workload's unit of ``done`` Blocks in ``secs``."""
    scale = 1e12 if w["unit"] in OPS_UNITS else 1e9
    return w["work"] / n_blocks * done / secs / scale


def cpu_baseline(w: dict, torch, budget_s: float = 12.0) -> dict:
    """Times the CPU oracle on a bounded sample of the workload's Blocks, on
    every host core (one process per core, Blocks split between them)."""
    from oracle.parallel import BlockTimer

    with BlockTimer(w["text"], oracle_arrays(w, torch)) as timer:
        timer.sample(min(2.0, budget_s / 6))  # first touch of the mapped inputs
        done, secs = timer.sample(budget_s)
        n, procs = timer.n_blocks, timer.procs
    return {"value": oracle_rate(w, done, secs, n), "unit": w["unit"], "cores": procs, "kind": "port",
            "sample": f"{done} Blocks ({done / n:.3g} of the Grid's {n}) in {secs:.1f} s; numpy oracle, "
                      f"{procs} processes with one BLAS thread each"}


def bid0_share(grid0: int, world: int, rank: int, root_share: float | None = None) -> tuple[int, int]:
    """Blocks [lo, hi) along bid0 that ``rank`` of ``world`` computes.

    Contiguous ranges in rank order.  With ``root_share`` None every rank gets
    an equal range; otherwise rank 0 gets that fraction of the Grid (at least
    one Block, leaving at least one per other rank) and the other ranks split
    the rest equally.
    """
    if root_share is None or world == 1:
        return rank * grid0 // world, (rank + 1) * grid0 // world
    if grid0 < world:
        raise ValueError(f"grid0={grid0} has fewer Blocks than the {world} ranks")
    b0 = min(grid0 - (world - 1), max(1, round(root_share * grid0)))
    if rank == 0:
        return 0, b0
    rest = grid0 - b0
    return b0 + (rank - 1) * rest // (world - 1), b0 + rank * rest // (world - 1)


def gather_root_share(world: int, flops: float, out_bytes: float, tflops: float = SHARDED_GEMM_TFLOPS,
                      ingest_gbs: float = PEER_INGEST_GBS) -> float:
    """Rank 0's fraction of the Grid when rank 0 receives every other rank's rows.

    Rank 0 computes f of the work (time f*T) while it takes in (1 - f) of the
    output (time (1 - f)*R); each other rank computes (1 - f)/(world - 1) of
    it.  The step ends when the slowest of the three does; with
    m = max(R, T/(world - 1)) the best f is m / (T + m).
    """
    if world == 1:
        return 1.0
    t = flops / (tflops * 1e12)
    r = out_bytes / (ingest_gbs * 1e9)
    m = max(r, t / (world - 1))
    return m / (t + m)


def gather_step_ms(f: float, world: int, t_ms: float, r_ms: float, slabs: int = 0) -> float:
    """Modelled step time with rank 0 computing a fraction ``f`` of the Grid.

    ``t_ms``: the whole GEMM on one GPU; ``r_ms``: rank 0 taking in the whole
    output.  Rank 0 computes f*T.  The other ranks' rows reach rank 0 at the
    ingest rate: during their GEMM (stores from the epilogue, ``slabs`` 0),
    or (copy engines, ``slabs`` S) only once a rank's first slab is done, and
    the last slab's copy follows the rank's last GEMM slab.
    """
    if world == 1:
        return t_ms
    other = (1 - f) * t_ms / (world - 1)
    if slabs <= 0:
        return max(f * t_ms, (1 - f) * r_ms, other)
    return max(f * t_ms, other / slabs + (1 - f) * r_ms, other + (1 - f) * r_ms / slabs)


def plan_root_blocks(grid0: int, world: int, t_ms: float, r_ms: float, slabs: int = 0) -> int:
    """Rank 0's Block count minimising ``gather_step_ms`` (each other rank keeps at least one Block)."""
    best = min(range(1, grid0 - (world - 1) + 1),
               key=lambda b: gather_step_ms(b / grid0, world, t_ms, r_ms, slabs))
    return best


def nccl_gather(out, rows_per_rank, world, rank, dist):
    if world == 1:
        return
    mine = out[rank * rows_per_rank:(rank + 1) * rows_per_rank]
    if rank == 0:
        dist.gather(mine, gather_list=[out[r * rows_per_rank:(r + 1) * rows_per_rank] for r in range(world)], dst=0)
    else:
        dist.gather(mine, dst=0)


def roofline_line(plan: dict, share: float, kernel_ms: float, peaks: dict, peak_kind: str,
                  int8: bool = False) -> dict:
    """The ``roofline`` object for one launch of ``share`` of the Grid taking ``kernel_ms``.

    ``int8``: the work is int8 tensor-core ops, whose dense rate is twice the
    bf16 rate; the tensor peaks are the measured bf16 ones doubled, and the
    unit is TOP/s.

    The binding roofline is the one whose floor (work / peak) is longer: a
    TFLOP/s workload below the ridge point (FLOP per byte < tensor peak / HBM
    peak) is bound by HBM, not by the tensor pipe.  The denominator is the
    burst peak: every workload here is timed alone, over a few tens of
    milliseconds.  For tensor-bound launches of a millisecond or more the
    fraction of the sustained GEMM peak (a seconds-long cuBLAS loop under the
    1000 W power cap) is given beside it, for steps long enough to reach the cap.
    """
    launch_bytes = plan["bytes"] * share
    launch_flops = plan["flops"] * share
    secs = kernel_ms * 1e-3
    if int8:
        peaks = {**peaks, "bf16_tflops": 2 * peaks["bf16_tflops"]}
        if "bf16_tflops_sustained" in peaks:
            peaks["bf16_tflops_sustained"] = 2 * peaks["bf16_tflops_sustained"]
    hbm_floor = launch_bytes / (peaks["hbm_gbs"] * 1e9)
    tensor_floor = launch_flops / (peaks["bf16_tflops"] * 1e12)
    bound = "hbm" if hbm_floor >= tensor_floor else "tensor"
    out = {"bound": bound}
    if bound == "hbm":
        achieved, peak, unit = launch_bytes / secs / 1e9, peaks["hbm_gbs"], "GB/s"
    else:
        achieved, peak, unit = launch_flops / secs / 1e12, peaks["bf16_tflops"], "TOP/s" if int8 else "TFLOP/s"
    kind = f"{peak_kind} (burst)" + (", int8 = 2 x bf16" if int8 and bound == "tensor" else "")
    extra = {}
    if launch_flops > 0:  # the non-binding roofline's fraction, for reference
        if bound == "hbm":
            extra["tensor_frac"] = round(launch_flops / secs / 1e12 / peaks["bf16_tflops"], 4)
        else:
            extra["hbm_frac"] = round(launch_bytes / secs / 1e9 / peaks["hbm_gbs"], 4)
    if bound == "tensor" and kernel_ms >= 1.0 and "bf16_tflops_sustained" in peaks:
        extra["frac_sustained"] = round(achieved / peaks["bf16_tflops_sustained"], 4)
    out.update({"achieved": round(achieved, 2), "peak": peak, "unit": unit, "frac": round(achieved / peak, 4),
                "peak_kind": kind, "traffic": None, "kernel_ms": round(kernel_ms, 4), **extra})
    return out


# ---------------------------------------------------------------- checks
TOLERANCES = {
    "bit-exact": "bit-exact",
    "softmax": "|d|/ref <= 1e-5",
    "transcendental": "|d| <= 1e-5 |ref| + 1e-6",
    "sum": "|d| <= 1e-6 |ref| + 1e-6",
    "bf16": "max|d|/max|ref| <= 1e-2 and |d| <= 1e-2|ref| + 1e-2 rms(ref)",
}


def tolerance_of(w: dict) -> str:
    """The parity bar of a workload's path: exact f32 arithmetic (add, sub,
    mul, max, data movement) bit-exact; the row softmax 1e-5 relative per
    element; programs with f32 transcendentals (their CUDA math functions
    against the oracle's float64 ones) 1e-5 relative plus 1e-6; tile sums
    (float64 accumulation in another order than numpy's) 1e-6 relative plus
    1e-6; bf16
    tensor-core work with f32 accumulation 1e-2 of the output's scale."""
    return w.get("tolerance", "bf16" if w["dtype"] == "bf16" else "bit-exact")


def close_enough(got, ref, tol: str) -> dict:
    """Compares ``got`` with the oracle's ``ref`` at tolerance ``tol`` (TOLERANCES)."""
    import numpy as np

    got = np.asarray(got)
    ref = np.asarray(ref)
    g, r = got.astype(np.float64), ref.astype(np.float64)
    d = np.abs(g - r)
    if tol == "bf16":
        scale = float(np.max(np.abs(r))) or 1.0
        rms = float(np.sqrt(np.mean(r * r)))
        ok = bool(d.max() / scale <= 1e-2 and np.all(d <= 1e-2 * np.abs(r) + 1e-2 * rms))
        return {"ok": ok, "max_rel": float(d.max() / scale), "tolerance": TOLERANCES[tol]}
    if tol == "softmax":
        rel = float(np.max(d / r))
        return {"ok": bool(np.all(r > 0) and rel <= 1e-5), "max_rel": rel, "tolerance": TOLERANCES[tol]}
    if tol in ("transcendental", "sum"):
        rtol, atol = (1e-5, 1e-6) if tol == "transcendental" else (1e-6, 1e-6)
        ok = bool(np.all(np.isfinite(g) == np.isfinite(r)))
        fin = np.isfinite(r)
        ok = ok and bool(np.all(d[fin] <= rtol * np.abs(r[fin]) + atol))
        rel = float(np.max(d[fin] / np.maximum(np.abs(r[fin]), 1e-30))) if fin.any() else 0.0
        return {"ok": ok, "max_rel": rel, "tolerance": TOLERANCES[tol]}
    same = bool(np.array_equal(got.view(np.uint32), ref.view(np.uint32)))
    return {"ok": same, "max_rel": 0.0 if same else float(np.max(d)), "tolerance": TOLERANCES["bit-exact"]}


def sample_check(w: dict, out, torch, n_blocks: int = 8, seed: int = 0, blocks=None) -> dict:
    """Checks a seeded sample of the Grid's Blocks of the device output ``out``
    against the CPU oracle run on those Blocks only (the oracle reads the DSL's
    own text).  Entries the sampled Blocks do not store are not compared."""
    import numpy as np
    from oracle import xt_oracle

    func = xt_oracle.parse_module(w["text"])[0]
    order = xt_oracle.serialize_order(func.grid)
    if blocks is None:
        rng = np.random.default_rng(seed)
        picks = sorted(rng.choice(len(order), size=min(n_blocks, len(order)), replace=False))
        blocks = [order[i] for i in picks]
    arrays = oracle_arrays(w, torch)
    pos = w.get("out_pos", len(w["inputs"]))
    if arrays[pos].dtype != np.float32:
        raise ValueError("sample_check compares f32 outputs")
    arrays[pos][...] = np.nan  # marks what the sampled Blocks do not store
    xt_oracle.run(w["text"], arrays, blocks=blocks)
    ref = arrays[pos]
    mask = ~np.isnan(ref)
    got = out.cpu().numpy()[mask]
    res = close_enough(got, ref[mask], tolerance_of(w))
    return {"ok": res["ok"], "blocks": len(blocks), "values": int(mask.sum()), "max_rel": res["max_rel"],
            "tolerance": res["tolerance"], "seed": seed}


def gather_check(w: dict, out, shares: list, rows_per_block: int, torch, per_shard: int = 3, seed: int = 0) -> dict:
    """The rows rank 0 gathered: ``per_shard`` seeded Blocks of every rank's
    bid0 range against the oracle, and the full rows on both sides of every
    boundary between two ranks' ranges against fp64 dot products."""
    import numpy as np
    from oracle import xt_oracle

    rng = np.random.default_rng(seed)
    gx, gy, gz = xt_oracle.parse_module(w["text"])[0].grid
    blocks = [(int(rng.integers(lo, hi)), int(rng.integers(0, gy)), int(rng.integers(0, gz)))
              for lo, hi in shares for _ in range(per_shard)]
    blk = sample_check(w, out, torch, blocks=blocks)
    rows = sorted({r for lo, _ in shares[1:] for r in (lo * rows_per_block - 1, lo * rows_per_block)})
    a, b = w["inputs"][0], w["inputs"][1]
    ref = (a[rows].double() @ b.double()).numpy()
    row = close_enough(out[rows].cpu().numpy(), ref, tolerance_of(w))
    return {"ok": bool(blk["ok"] and row["ok"]), "blocks": blk["blocks"], "block_max_rel": blk["max_rel"],
            "rows": len(rows), "row_max_rel": row["max_rel"], "max_rel": max(blk["max_rel"], row["max_rel"]),
            "tolerance": row["tolerance"], "seed": seed}


# ---------------------------------------------------------------- timing helpers
def capture_graph(step, steps: int, dev, torch):
    """``steps`` calls of ``step(i)`` captured in one CUDA graph, with the two
    timing events recorded inside it (so the interval is the launches on the
    device, not the host's graph-launch latency)."""
    g_begin = torch.cuda.Event(enable_timing=True, external=True)
    g_end = torch.cuda.Event(enable_timing=True, external=True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cap = torch.cuda.current_stream(dev)
        g_begin.record(cap)
        for i in range(steps):
            step(i)
        g_end.record(cap)
    graph.replay()
    torch.cuda.synchronize()
    return graph, g_begin, g_end


def rotating_sets(w: dict, dev, torch):
    """Device copies of the inputs and an output, repeated until the sets
    together exceed three times the 126 MB L2 (each launch then reads its
    inputs from HBM)."""
    inputs_dev = [t.to(dev) for t in w["inputs"]]
    out = torch.empty(w["out_shape"], dtype=w["out_dtype"], device=dev)
    ws_bytes = sum(t.numel() * t.element_size() for t in inputs_dev) + out.numel() * out.element_size()
    n_sets = 1 if ws_bytes > 3 * L2_BYTES else int(-(-3 * L2_BYTES // ws_bytes)) + 1
    sets = [(inputs_dev, out)] + [([t.clone() for t in inputs_dev], torch.empty_like(out))
                                  for _ in range(n_sets - 1)]
    return sets


def gpu_id_of(dev, torch) -> str:
    uuid = str(getattr(torch.cuda.get_device_properties(dev), "uuid", dev.index))
    return uuid if uuid.startswith("GPU-") or uuid.isdigit() else f"GPU-{uuid}"


PER_CONFIG = ("add", "softmax", "matmul", "conv2d")
# kernels generated per program (not BASELINE configurations), one of each
# kind: elementwise, rows (a CTA per row), tile (a fused elementwise run)
GENERATED = ("silu", "row_center", "softmax_wide", "col_bias")


def run_per_config(xt, torch, dev, peaks: dict, peak_kind: str, steps: int = 50, warmup: int = 5,
                   region_ms: float = 60.0, names=PER_CONFIG) -> dict:
    """BASELINE configurations 1-4 (or the workloads ``names``) on one GPU,
    each timed like the headline's graph mode (K launches in a CUDA graph over rotating buffer sets, events
    inside the graph), replayed for about ``region_ms`` with the clocks
    sampled, then checked on a seeded sample of Blocks against the oracle.

    The region is a burst as long as the headline's (tens of milliseconds),
    so the burst peaks are the denominators; a region of a few hundred
    milliseconds of the 4096^3 GEMM already meets the 1000 W cap (measured:
    1432 MHz median SM clock over 300 ms, 0.89 of the sustained GEMM peak)."""
    out = {}
    for name in names:
        w = build_workload(name, load_dsl(), torch, 1, 0)
        mod = xt.parse(w["text"])
        plan = mod.plan()
        sets = rotating_sets(w, dev, torch)
        n_sets = len(sets)

        def step(i, sets=sets, mod=mod, w=w):
            ins, o = sets[i % len(sets)]
            xt.launch(mod, *launch_arrays(w, ins, o))

        for i in range(warmup):
            step(i)
        torch.cuda.synchronize()
        graph, g_begin, g_end = capture_graph(step, steps, dev, torch)
        one = g_begin.elapsed_time(g_end)
        replays = max(3, int(region_ms / max(one, 1e-3)))
        times = []
        with ClockSampler(gpu_id_of(dev, torch)) as clocks:
            for _ in range(replays):
                graph.replay()
                torch.cuda.synchronize()
                times.append(g_begin.elapsed_time(g_end))
        del graph
        ms = statistics.fmean(times) / steps
        scale = 1e12 if w["unit"] in OPS_UNITS else 1e9
        roof = roofline_line(plan, 1.0, ms, peaks, peak_kind)
        roof["traffic"] = NCU_TRAFFIC_BYTES.get(name)
        out[name] = {"value": round(w["work"] / (ms * 1e-3) / scale, 3), "unit": w["unit"],
                     "ms_per_launch": round(ms, 5), "launches": steps * replays, "roofline": roof,
                     "clocks": clocks.summary(), "l2": f"{n_sets} rotating input/output sets",
                     "timing": "CUDA-graph replay of K launches, events recorded inside the graph",
                     "parity": sample_check(w, sets[0][1], torch), "config": w["config"]}
        del sets
        torch.cuda.empty_cache()
    return out


def _cudart(torch):
    """torch's CUDA runtime (the same primary contexts), for plain copies."""
    import ctypes
    import glob

    base = Path(torch.__file__).resolve().parent
    for pat in ("../nvidia/cuda_runtime/lib/libcudart.so*", "lib/libcudart*.so*"):
        hits = sorted(glob.glob(str(base / pat)))
        if hits:
            lib = ctypes.CDLL(hits[0])
            lib.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                            ctypes.c_void_p]
            return lib
    return None


def measure_ingest(torch, dev, dist, rank: int, src, target, rows: tuple, flag, gemm_send, reps: int = 3) -> dict:
    """Rate at which rank 0 takes in rows over NVLink while every other rank
    sends its rows [rows[0], rows[1]) at once, measured on rank 0 between two
    all-reduces that bracket the transfer (rank 0's interval covers every
    sender, so no maximum over ranks is needed).  Two senders:

    * ``gemm_stores``: ``gemm_send()`` launches the sharded GEMM for this
      rank's Blocks with rank 0's array as its output, so the rows go out as
      the GEMM's epilogue stores them (128-byte TMA row segments) while it
      computes; when the GEMM itself takes longer than the transfer (two
      GPUs) this is a lower bound on the store rate;
    * ``copy_engines``: one cudaMemcpyAsync per rank, device to peer device.
    """
    lo, hi = rows
    n_cols = src.shape[1]
    nbytes = (hi - lo) * n_cols * 4
    total = torch.tensor([float(nbytes if rank else 0)], device=dev)
    dist.all_reduce(total)
    cudart = _cudart(torch)
    stream = torch.cuda.current_stream(dev)
    res = {}
    for how in ("gemm_stores", "copy_engines"):
        if how == "copy_engines" and cudart is None:
            continue
        best = None
        for _ in range(reps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            dist.all_reduce(flag)
            e0.record(stream)
            if rank != 0 and hi > lo:
                if how == "gemm_stores":
                    gemm_send()
                else:
                    off = lo * n_cols * 4
                    rc = cudart.cudaMemcpyAsync(target.data_ptr() + off, src.data_ptr() + off, nbytes, 4,
                                                stream.cuda_stream)
                    if rc != 0:
                        raise RuntimeError(f"cudaMemcpyAsync to rank 0 failed: {rc}")
            dist.all_reduce(flag)
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        t = torch.tensor([best], device=dev)
        dist.broadcast(t, src=0)
        res[how] = round(total.item() / (t.item() * 1e-3) / 1e9, 1)
    res["bytes"] = int(total.item())
    res["how"] = ("rank 0 times, between two all-reduces, every other rank sending its equal share of the "
                  "output rows at once; best of %d" % reps)
    return res


# ---------------------------------------------------------------- main
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="sharded_matmul",
                    choices=["add", "softmax", "matmul", "conv2d", "sharded_matmul", "transpose", "silu",
                             "row_center", "row_bias", "matmul_i8", "col_sums", "col_bias", "softmax_wide"])
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "torch"],
                    help="b200: this backend; reference: the reference's CPU path; torch: the vendor library "
                         "(cuBLAS, cuDNN) through PyTorch on one GPU, for context")
    ap.add_argument("--gather", default="auto", choices=["auto", "peer", "dma", "nccl"],
                    help="sharded_matmul on N>1 GPUs: ranks store their rows straight into rank 0's output "
                         "over NVLink from the GEMM (peer), compute slabs locally and push each to rank 0 with "
                         "the copy engines (dma), or compute locally and gather with NCCL; auto: peer on 2 GPUs, "
                         "dma on more (rank 0's NVLink ingress binds from 3 GPUs on; the copy engines fill it, measured "
                         "778 GB/s, and the slabs let rank 0 keep a smaller share)")
    ap.add_argument("--slabs", type=int, default=6,
                    help="dma gather: slabs per rank (each slab's copy overlaps the next slab's GEMM)")
    ap.add_argument("--root-share", type=float, default=None,
                    help="peer gather: rank 0's fraction of the Grid (default: balanced against its NVLink ingress)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip configurations 1-4 and the generated-kernel workloads beside the default "
                         "(sharded_matmul) line on one GPU")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gather == "auto":
        args.gather = "peer" if world <= 2 else "dma"
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch

    if args.impl == "reference":
        run_reference(args, world, rank, torch)
        return
    if args.impl == "torch":
        if rank == 0:
            run_torch_library(args, torch)
        return

    import xtile as xt

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # NCCL runs one CTA per channel: keep them within the SMs the GEMM leaves
        # free, so the gather of step i really runs beside the GEMM of step i + 1
        os.environ.setdefault("NCCL_MAX_NCHANNELS", str(GATHER_CHANNELS))
        os.environ.setdefault("NCCL_MAX_P2P_NCHANNELS", str(GATHER_CHANNELS))
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    w = build_workload(args.workload, load_dsl(), torch, world, rank)
    mod = xt.parse(w["text"])
    plan = mod.plan()
    plan_work = plan["flops"] if w["unit"] in OPS_UNITS else plan["bytes"]
    if abs(plan_work - w["work"]) > 1e-9 * w["work"]:
        raise SystemExit(f"bench: the planner's work {plan_work} differs from the configuration's {w['work']}")
    grid0 = plan["grid"][0]
    sharded = w.get("sharded", False)
    if world > 1 and not sharded:
        # not a sharded configuration: every rank runs an independent replica
        w["config"]["parallelism"] = f"{world} independent replicas"
    if sharded and (grid0 % world or w["out_shape"][0] % grid0):
        raise SystemExit(f"bench: grid0={grid0} does not split evenly over {world} ranks")
    # peer and dma: rank 0's output arrays are mapped into every rank (CUDA IPC)
    peer = sharded and world > 1 and args.gather in ("peer", "dma")
    dma = peer and args.gather == "dma"
    # equal ranges: compute-only scaling (output left in place) and the NCCL gather
    even_lo, even_hi = bid0_share(grid0, world, rank) if sharded else (0, grid0)
    rows_per_block = w["out_shape"][0] // grid0
    rows_per_rank = w["out_shape"][0] // world if sharded else 0

    # device-resident inputs; rotate enough sets to defeat the 126 MB L2
    if sharded:
        # two output buffers: step i + 1 computes into one while step i's rows
        # are still being gathered out of the other
        inputs_dev = [t.to(dev) for t in w["inputs"]]
        out = torch.empty(w["out_shape"], dtype=w["out_dtype"], device=dev)
        sets = [(inputs_dev, out), (inputs_dev, torch.empty_like(out))]
    else:
        sets = rotating_sets(w, dev, torch)
    n_sets = len(sets)
    stream = torch.cuda.current_stream(dev)
    comm = torch.cuda.Stream(dev) if sharded else None
    # peer gather: every rank's kernel stores its rows into rank 0's output
    # arrays (mapped over NVLink with CUDA IPC); a one-element all-reduce per
    # step is the GPU-side barrier after which rank 0 holds all rows
    targets = [o for _, o in sets]
    flag = torch.zeros(1, device=dev)
    if peer:
        handles = [xt.export_array(o) for o in targets] if rank == 0 else None
        box = [handles]
        dist.broadcast_object_list(box, src=0)
        if rank != 0:
            targets = [xt.PeerArray.open(h, tuple(w["out_shape"]), w["out_dtype"]) for h in box[0]]

    # ---- row gather: rank 0's share of the Grid from rates measured here.
    # T: the whole GEMM on one GPU (every rank times its equal share; the
    # slowest share times N).  R: rank 0 taking in the whole output from all
    # other ranks at once, at the measured rate of the sender this run uses
    # (the GEMM's own stores, or the copy engines).
    rates = None
    root_share = None
    if peer:
        for i in range(2):  # warm the GEMM's tensor maps and clocks
            xt.launch(mod, *launch_arrays(w, sets[0][0], sets[0][1]), bid0_range=(even_lo, even_hi))
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for i in range(3):
            xt.launch(mod, *launch_arrays(w, sets[0][0], sets[0][1]), bid0_range=(even_lo, even_hi))
        c1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([c0.elapsed_time(c1) / 3], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gemm_ms = t.item() * world
        src = sets[1][1]  # a local buffer of the output's shape (rank 0's is never sent)
        rows = (even_lo * rows_per_block, even_hi * rows_per_block)
        ingest = measure_ingest(torch, dev, dist, rank, src, targets[0], rows, flag, lambda: xt.launch(
            mod, *launch_arrays(w, sets[0][0], targets[0]), bid0_range=(even_lo, even_hi)))
        out_bytes = w["out_shape"][0] * w["out_shape"][1] * 4
        tflops = plan["flops"] / (gemm_ms * 1e-3) / 1e12
        rates = {"gemm_tflops_1gpu": round(tflops, 1), "gemm_ms_1gpu": round(gemm_ms, 4), "ingest_gbs": ingest}
        # the ingest rate of the sender this run uses
        how = "copy_engines" if dma else "gemm_stores"
        rates["sender"] = how
        r_ms = out_bytes / (ingest[how] * 1e9) * 1e3
        n_slabs = args.slabs if dma else 0
        root_share = args.root_share if args.root_share is not None else (
            plan_root_blocks(grid0, world, gemm_ms, r_ms, n_slabs) / grid0)
        rates["bound_ms"] = round(gemm_ms * r_ms / (gemm_ms + r_ms), 4)  # T*R/(T+R): no split does better
        rates["bound_note"] = ("T*R/(T+R): T the one-GPU GEMM, R rank 0 taking in the whole output at the "
                               f"measured ingest rate of the sender used ({how})")
    lo, hi = bid0_share(grid0, world, rank, root_share) if sharded else (0, grid0)
    shares = [bid0_share(grid0, world, r, root_share) for r in range(world)] if sharded else [(0, grid0)]
    if peer:
        b0 = shares[0][1]
        how = (f"the other ranks compute {args.slabs} slabs each locally and push each finished slab into rank 0's "
               f"output over NVLink with one cudaMemcpyAsync (copy engines, CUDA IPC)" if dma else
               "each rank's kernel stores its C rows into rank 0's output over NVLink (CUDA IPC)")
        w["config"]["parallelism"] = (f"bid0 split over {world} GPUs, rank 0 {b0} of {grid0} Blocks, the others "
                                      f"{(grid0 - b0) // (world - 1)}-{-(-(grid0 - b0) // (world - 1))}; {how}")
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    computed = [torch.cuda.Event() for _ in range(n_sets)]
    gathered = [torch.cuda.Event() for _ in range(n_sets)]
    # dma gather: this rank's bid0 range in slabs, one event per slab
    slabs = [(lo + k * (hi - lo) // args.slabs, lo + (k + 1) * (hi - lo) // args.slabs)
             for k in range(max(1, args.slabs))] if dma and rank != 0 else []
    slabs = [s for s in slabs if s[1] > s[0]]
    slab_done = [torch.cuda.Event() for _ in slabs]
    cudart = _cudart(torch) if dma else None
    row_bytes = w["out_shape"][1] * 4

    def push_slab(o, tgt, a, b):
        off = a * rows_per_block * row_bytes
        rc = cudart.cudaMemcpyAsync(tgt.data_ptr() + off, o.data_ptr() + off, (b - a) * rows_per_block * row_bytes,
                                    4, comm.cuda_stream)  # cudaMemcpyDefault: device to peer device
        if rc != 0:
            raise RuntimeError(f"cudaMemcpyAsync of a slab to rank 0 failed: {rc}")

    def step(i, rng=(lo, hi)):
        ins, o = sets[i % n_sets]
        xt.launch(mod, *launch_arrays(w, ins, o), bid0_range=rng)

    def sharded_step(i, start=None, end=None):
        if dma and rank != 0:
            # GEMM slab by slab into the local output; the copy engines push
            # each finished slab to rank 0 while the next slab computes
            ins, o = sets[i % n_sets]
            if i >= n_sets:
                stream.wait_event(gathered[i % n_sets])  # that step's pushes have read o
            if start is not None:
                start.record(stream)
            for (a, b), ev in zip(slabs, slab_done):
                xt.launch(mod, *launch_arrays(w, ins, o), bid0_range=(a, b))
                ev.record(stream)
                comm.wait_event(ev)
                push_slab(o, targets[i % n_sets], a, b)
            if end is not None:
                end.record(stream)
            gathered[i % n_sets].record(comm)
            stream.wait_event(gathered[i % n_sets])  # every row has reached rank 0 ...
            dist.all_reduce(flag)  # ... before the step's barrier
            return
        if peer:
            ins, o = sets[i % n_sets][0], targets[i % n_sets]
            if start is not None:
                start.record(stream)
            xt.launch(mod, *launch_arrays(w, ins, o), bid0_range=(lo, hi))
            if end is not None:
                end.record(stream)
            dist.all_reduce(flag)
            return
        # compute on the default stream, gather on the communication stream:
        # the gather of step i overlaps the compute of step i + 1
        ins, o = sets[i % n_sets]
        if i >= n_sets:
            stream.wait_event(gathered[i % n_sets])  # that gather has read o
        if start is not None:
            start.record(stream)
        with xt.sm_budget(sms - GATHER_SMS if world > 1 else 0):
            xt.launch(mod, *launch_arrays(w, ins, o), bid0_range=(lo, hi))
        if end is not None:
            end.record(stream)
        computed[i % n_sets].record(stream)
        comm.wait_event(computed[i % n_sets])
        with torch.cuda.stream(comm):
            nccl_gather(o, rows_per_rank, world, rank, dist)
        gathered[i % n_sets].record(comm)

    for i in range(args.warmup):
        if sharded:
            sharded_step(i)
        else:
            step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()

    # ---- timed region: K steps.  Microsecond-scale steps are captured once in
    # a CUDA graph and replayed, so host launch overhead does not starve the
    # GPU; the millisecond-scale sharded step (with its NCCL gather) launches
    # eagerly with per-launch events, its gather on a second stream.
    use_graph = not sharded
    graph = None
    # In graph mode the two timing events are nodes of the graph itself
    # (external events), so the measured interval is the K launches on the
    # device and not the host's graph-launch latency.  (Event nodes between
    # the launches would add gaps of their own, so there are none.)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if use_graph:
        graph, g_begin, g_end = capture_graph(step, args.steps, dev, torch)
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id_of(dev, torch)) as clocks:
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        t_begin.record(stream)
        if use_graph:
            graph.replay()
        else:
            for i in range(args.steps):
                sharded_step(i, starts[i], ends[i])
            stream.wait_stream(comm)  # every gather is inside the timed region
        t_end.record(stream)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
    if use_graph:
        total_ms = g_begin.elapsed_time(g_end)
        kernel_ms = total_ms / args.steps
    else:
        total_ms = t_begin.elapsed_time(t_end)
        kernel_ms = statistics.fmean(s.elapsed_time(e) for s, e in zip(starts, ends))
    del graph
    # this repository's kernels launched in the timed region, summed over ranks
    # (a rank pushing slabs launches one GEMM per slab)
    launches = args.steps * (len(slabs) if dma and rank != 0 else 1)
    if dist:
        t = torch.tensor([total_ms, kernel_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, kernel_ms = t.tolist()
        n = torch.tensor([float(launches)], device=dev)
        dist.all_reduce(n)
        launches = int(n.item())
    clock = clocks.summary()
    err = xt.device_error()

    # ---- correctness of what the timed steps produced (after the timed
    # region): a seeded sample of Blocks against the oracle; on N GPUs, rank 0
    # checks the rows it gathered from every rank (the others wait at the
    # next barrier)
    parity = None
    last_out = sets[(args.steps - 1) % n_sets][1]
    if w["out_dtype"] == torch.float32:
        if world == 1:
            parity = sample_check(w, last_out, torch)
        elif sharded and rank == 0:
            parity = gather_check(w, last_out, shares, rows_per_block, torch)
    if dist:
        dist.barrier()

    # ---- compute-only timing (sharded: no gather), for the scaling report
    compute = None
    if sharded and world > 1:
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        dist.barrier()
        c0.record(stream)
        for i in range(args.steps):
            step(i, (even_lo, even_hi))
        c1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([c0.elapsed_time(c1) / args.steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        compute = t.item()

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        host_in = [t.pin_memory() for t in w["inputs"]]
        if sharded:
            host_in[0] = host_in[0][lo * rows_per_block:hi * rows_per_block]
        host_out = torch.empty(w["out_shape"] if (rank == 0 or not sharded) else (0,), dtype=w["out_dtype"]).pin_memory()
        ins, o = sets[0]
        h2d = sum(t.numel() * t.element_size() for t in host_in)
        d2h = host_out.numel() * host_out.element_size()
        e_steps = max(3, min(args.steps, 10))
        e_note = "one stream: each step's copies in, launch and copy out in sequence"
        # One GPU: a three-stage pipeline over two buffer sets.  One stream only
        # copies inputs in, one only launches, one only copies results out, so
        # step j + 1's host-to-device copies run while step j's result is copied
        # back (PCIe carries both directions at once).  Events per buffer set
        # keep a copy-in from overwriting inputs a kernel still reads and a
        # kernel from overwriting a result still being copied out.  Every step
        # moves all of its inputs in and its whole result out.
        # The same pipeline on N GPUs when the rows reach rank 0 without a
        # collective (peer and dma modes; the launch stores straight into rank
        # 0's output): every rank copies its inputs in and launches, rank 0
        # copies the whole result out.  A second one-element all-reduce before
        # each launch keeps every rank from writing an output set of rank 0's
        # before rank 0 has copied that set's previous result out.
        e_streams = [torch.cuda.Stream(dev) for _ in range(3)] if (world == 1 or peer or not sharded) else None
        if e_streams:
            e_note = ("three streams (copy in, launch, copy out) over two buffer sets: step j+1's "
                      "host-to-device copies overlap step j's device-to-host copy")
            if peer:
                e_note += ("; on N GPUs every rank's launch stores into rank 0's output (with --gather dma "
                           "too: the GEMM's own stores), rank 0 copies the whole result out, two one-element "
                           "all-reduces per step order the sets")
                e_sets = [(ins, targets[0]), ([torch.empty_like(t) for t in ins], targets[1])]
            else:
                e_sets = [sets[0], ([torch.empty_like(t) for t in ins], torch.empty_like(o))]
            host_outs = [host_out, torch.empty_like(host_out).pin_memory()]
            ev_in, ev_k, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))
            flag2 = torch.zeros(1, device=dev)

        def e2e_step_pipe(j):
            b = j % 2
            e_ins, e_o = e_sets[b]
            s_in, s_k, s_out = e_streams
            with torch.cuda.stream(s_in):
                if j >= 2:
                    s_in.wait_event(ev_k[b])  # step j - 2's kernel has read these inputs
                if sharded:
                    e_ins[0][lo * rows_per_block:hi * rows_per_block].copy_(host_in[0], non_blocking=True)
                    e_ins[1].copy_(host_in[1], non_blocking=True)
                else:
                    for d, h in zip(e_ins, host_in):
                        d.copy_(h, non_blocking=True)
                ev_in[b].record(s_in)
            with torch.cuda.stream(s_k):
                s_k.wait_event(ev_in[b])
                if j >= 2 and host_outs[b].numel():
                    s_k.wait_event(ev_out[b])  # step j - 2's result has been copied out
                if peer and j >= 2:
                    dist.all_reduce(flag2)  # ... on rank 0, before any rank writes set b again
                xt.launch(mod, *launch_arrays(w, e_ins, e_o), bid0_range=(lo, hi))
                if peer:
                    dist.all_reduce(flag)  # every rank's rows are in rank 0's set b
                ev_k[b].record(s_k)
            if host_outs[b].numel():
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_k[b])
                    host_outs[b].copy_(e_o, non_blocking=True)
                    ev_out[b].record(s_out)

        def e2e_step():
            if sharded:
                ins[0][lo * rows_per_block:hi * rows_per_block].copy_(host_in[0], non_blocking=True)
                ins[1].copy_(host_in[1], non_blocking=True)
            else:
                for d, h in zip(ins, host_in):
                    d.copy_(h, non_blocking=True)
            if peer:
                xt.launch(mod, *launch_arrays(w, ins, targets[0]), bid0_range=(lo, hi))
                dist.all_reduce(flag)
            else:
                xt.launch(mod, *launch_arrays(w, ins, o), bid0_range=(lo, hi))
                if sharded:
                    nccl_gather(o, rows_per_rank, world, rank, dist)
            if host_out.numel():
                host_out.copy_(o, non_blocking=True)

        if e_streams:
            e2e_step_pipe(0)
            e2e_step_pipe(1)
        else:
            e2e_step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if e_streams:
            for es in e_streams:
                es.wait_stream(stream)
            for j in range(2, 2 + e_steps):
                e2e_step_pipe(j)
            for es in e_streams:
                stream.wait_stream(es)
        else:
            for _ in range(e_steps):
                e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / e_steps
        if dist:
            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = t.item()
        e2e = (e_ms, h2d, d2h, e_note)

    if dist:
        dist.barrier()
    if peer and rank != 0:
        for t in targets:
            t.close()
    if rank != 0:
        dist.destroy_process_group()
        return

    # ---- report
    peaks, peak_kind = load_peaks()
    work = w["work"]
    scale = 1e12 if w["unit"] in OPS_UNITS else 1e9
    job_units = work if (sharded or world == 1) else work * world
    ms_per_step = total_ms / args.steps
    value = job_units / (ms_per_step * 1e-3) / scale
    roofline = roofline_line(plan, (hi - lo) / grid0, kernel_ms, peaks, peak_kind, int8=w["unit"] == "TOP/s")
    roofline["traffic"] = NCU_TRAFFIC_BYTES.get(args.workload)
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": w["unit"],
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong" if sharded else "weak",
        "vs_baseline": None,
        "dtype": w["dtype"],
        "data": "synthetic (seeded torch.Generator inputs of the BASELINE shapes)",
        "config": {**w["config"], "l2": f"{n_sets} rotating input/output sets" if n_sets > 1
                   else "working set larger than L2",
                   "timing": ("CUDA-graph replay of K launches, events recorded inside the graph"
                              if not sharded else "eager launches, events around each launch" if world == 1 else
                              ("eager launches; slabs pushed into rank 0's output by the copy engines, "
                               "one-element all-reduce per step" if dma else
                               "eager launches; rows stored into rank 0's output over NVLink, one-element "
                               "all-reduce per step" if peer else
                               "eager launches; step i's NCCL gather overlaps step i+1's compute"))},
        "roofline": roofline,
        "clocks": clock,
        "gpu_launches": launches,
        "device_error": err,
    }
    if compute is not None:
        line["compute_only"] = {"ms_per_step": round(compute, 4),
                                "value": round(work / (compute * 1e-3) / scale, 3)}
        line["gather"] = {"ms_per_step": round(ms_per_step - compute, 4),
                          "bytes": (w["out_shape"][0] - (hi - lo) * rows_per_block) * w["out_shape"][1] * 4}
    if parity is not None:
        line["parity" if world == 1 else "gather_check"] = parity
    if rates is not None:
        # which term of the step model binds at this split: rank 0's own share,
        # rank 0's ingress of the others' rows, or another rank's share
        f = shares[0][1] / grid0
        t_ms, r_ms = rates["gemm_ms_1gpu"], w["out_shape"][0] * w["out_shape"][1] * 4 / (
            rates["ingest_gbs"][rates["sender"]] * 1e9) * 1e3
        n_sl = args.slabs if dma else 0
        other = (1 - f) * t_ms / (world - 1)
        terms = {"rank 0's own share of the GEMM": f * t_ms,
                 "rank 0's NVLink ingress of the other ranks' rows": (other / n_sl if n_sl else 0.0) + (1 - f) * r_ms,
                 "the other ranks' shares of the GEMM": other + ((1 - f) * r_ms / n_sl if n_sl else 0.0)}
        rates["model_ms"] = {k: round(v, 4) for k, v in terms.items()}
        rates["model_step_ms"] = round(gather_step_ms(f, world, t_ms, r_ms, n_sl), 4)
        rates["limiter"] = max(terms, key=terms.get)
        rates["efficiency_vs_bound"] = round(rates["bound_ms"] / ms_per_step, 4)
        line["gather_rates"] = rates
    if e2e is not None:
        e_ms, h2d, d2h, e_note = e2e
        line["e2e"] = {"value": round(job_units / (e_ms * 1e-3) / scale, 3), "unit": w["unit"],
                       "ms_per_step": round(e_ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                       "pipelining": e_note}
    if world == 1 and args.workload == "sharded_matmul" and not args.no_per_config:
        # BASELINE configurations 1-4, one GPU each, beside the headline; then
        # one workload of each kind of generated kernel
        line["per_config"] = run_per_config(xt, torch, dev, peaks, peak_kind)
        line["generated"] = run_per_config(xt, torch, dev, peaks, peak_kind, names=GENERATED)
    if not args.no_cpu and world == 1:  # the host-core baseline is a 1-GPU figure
        line["cpu_baseline"] = cpu_baseline(w, torch)
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def run_torch_library(args, torch) -> None:
    """Times the workload through PyTorch's CUDA libraries on one GPU, for context.

    add and softmax run torch's own kernels, matmul cuBLAS (``torch.mm`` with
    an f32 output), conv2d cuDNN on channels-last bf16 tensors (its output is
    bf16, half the bytes of this backend's f32 output).  The same inputs,
    rotating buffer sets and graph-replay timing as the b200 arm.
    """
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = build_workload(args.workload, load_dsl(), torch, 1, 0)
    name = args.workload
    ins = [t.to(dev) for t in w["inputs"]]
    if name == "conv2d":
        x, f = ins
        ins = [x.permute(0, 3, 1, 2), f.permute(3, 2, 0, 1).contiguous(memory_format=torch.channels_last)]
    ws = sum(t.numel() * t.element_size() for t in ins) + 2 * torch.Size(w["out_shape"]).numel() * 4
    n_sets = 1 if ws > 3 * L2_BYTES else int(-(-3 * L2_BYTES // ws)) + 1
    sets = [ins] + [[t.clone(memory_format=torch.preserve_format) for t in ins] for _ in range(n_sets - 1)]
    outs = [torch.empty(w["out_shape"], dtype=torch.float32, device=dev) for _ in range(n_sets)]
    if name == "add":
        lib = "torch.add (out=)"
        fn = lambda i: torch.add(*sets[i % n_sets], out=outs[i % n_sets])  # noqa: E731
    elif name in ("softmax", "softmax_wide"):
        lib = "torch.softmax"
        fn = lambda i: torch.softmax(sets[i % n_sets][0], -1)  # noqa: E731
    elif name in ("matmul", "sharded_matmul"):
        lib = "cuBLAS via torch.mm(out_dtype=float32, out=)"
        fn = lambda i: torch.mm(*sets[i % n_sets], out_dtype=torch.float32, out=outs[i % n_sets])  # noqa: E731
    elif name == "transpose":
        lib = "torch copy_ of a transposed view"
        fn = lambda i: outs[i % n_sets].copy_(sets[i % n_sets][0].transpose(1, 2))  # noqa: E731
    elif name == "matmul_i8":
        lib = "torch._int_mm (cuBLASLt int8) + f32 scale/bias + int8 cast"

        def fn(i):
            a, b, sc, bi = sets[i % n_sets]
            t = torch._int_mm(a, b).float().mul_(sc).add_(bi)
            return t.round_().clamp_(-128, 127).to(torch.int8)
    elif name == "silu":
        lib = "torch.nn.functional.silu"
        fn = lambda i: torch.nn.functional.silu(sets[i % n_sets][0], inplace=False)  # noqa: E731
    elif name == "row_center":
        lib = "torch: (x - x.amax(1, keepdim=True)) ** 2 (three kernels)"
        fn = lambda i: (sets[i % n_sets][0] - sets[i % n_sets][0].amax(1, keepdim=True)).square_()  # noqa: E731
    elif name == "row_bias":
        lib = "torch.addcmul(r, x, r, out=)"
        fn = lambda i: torch.addcmul(sets[i % n_sets][1], sets[i % n_sets][0], sets[i % n_sets][1],  # noqa: E731
                                     out=outs[i % n_sets])
    elif name == "col_bias":
        lib = "torch: sigmoid(x * c - c) (three kernels)"
        fn = lambda i: torch.sigmoid((sets[i % n_sets][0] * sets[i % n_sets][1]).sub_(sets[i % n_sets][1]))  # noqa: E731
    elif name == "col_sums":
        lib = "torch.sum over the 64-row tiles (f32 accumulation, out=)"
        fn = lambda i: torch.sum(sets[i % n_sets][0].view(256, 64, 2048), dim=1, out=outs[i % n_sets])  # noqa: E731
    else:
        lib = "cuDNN via torch.nn.functional.conv2d, channels-last bf16 in, bf16 out"
        fn = lambda i: torch.nn.functional.conv2d(sets[i % n_sets][0], sets[i % n_sets][1], padding=1)  # noqa: E731
    for i in range(args.warmup):
        fn(i)
    torch.cuda.synchronize()
    g_begin = torch.cuda.Event(enable_timing=True, external=True)
    g_end = torch.cuda.Event(enable_timing=True, external=True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cap = torch.cuda.current_stream(dev)
        g_begin.record(cap)
        for i in range(args.steps):
            fn(i)
        g_end.record(cap)
    graph.replay()
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    ms = g_begin.elapsed_time(g_end) / args.steps
    work = w["work"]
    scale = 1e12 if w["unit"] in OPS_UNITS else 1e9
    print(json.dumps({"metric": METRIC, "impl": "torch", "library": lib, "value": round(work / (ms * 1e-3) / scale, 3),
                      "unit": w["unit"], "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(ms, 4), "higher_is_better": True,
                      "config": {**w["config"], "l2": f"{n_sets} rotating input/output sets"}}), flush=True)


def run_reference(args, world: int, rank: int, torch) -> None:
    """Reference arm: the CPU oracle (the reference executes nothing itself).

    Self-contained: the Block program is traced by the pure-Python DSL and the
    work comes from the configuration's formula, so no library of this
    repository is loaded.  Every host core in the affinity mask is used,
    whatever ``OMP_NUM_THREADS`` torchrun sets.
    """
    if rank != 0:
        return
    from oracle.parallel import BlockTimer

    w = build_workload(args.workload, load_dsl(), torch, 1, 0)
    budget = max(1.0, 60.0 / (args.warmup + args.steps))
    samples = []
    with BlockTimer(w["text"], oracle_arrays(w, torch)) as timer:
        for i in range(args.warmup + args.steps):
            done, secs = timer.sample(budget)
            if i >= args.warmup:
                samples.append((done, secs))
        n, procs = timer.n_blocks, timer.procs
    value = statistics.fmean(oracle_rate(w, d, s, n) for d, s in samples)
    done = sum(d for d, _ in samples)
    secs = sum(s for _, s in samples)
    line = {
        "metric": METRIC, "impl": "reference", "value": round(value, 6), "unit": w["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong" if w.get("sharded") else "weak", "vs_baseline": None, "dtype": w["dtype"],
        "data": "synthetic (seeded torch.Generator inputs of the BASELINE shapes)", "config": w["config"],
        "cpu_baseline": {"value": round(value, 6), "unit": w["unit"], "cores": procs, "kind": "port",
                         "sample": f"{args.steps} steps of about {budget:.1f} s: {done} Blocks of the Grid's {n} "
                                   f"in {secs:.1f} s; numpy oracle, {procs} processes with one BLAS thread each"},
        "e2e": {"value": round(value, 6), "unit": w["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference (sjjeong94/xtile) compiles to NPU command IR and executes nothing; this arm "
                "times the CPU oracle that restates its semantics on a bounded sample of Blocks",
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
