"""Host-side pieces of ``bench.py``: the roofline object and the clock summary.

These run on the CPU; the timings themselves need a B200 (``bench.py``).
"""
import json
import subprocess
import sys
from pathlib import Path

import pytest

import bench

ROOT = Path(__file__).resolve().parents[1]

PEAKS = {"hbm_gbs": 6544.7, "bf16_tflops": 1634.5, "bf16_tflops_sustained": 1385.9}


def test_matmul_is_tensor_bound_against_the_burst_peak():
    plan = {"flops": 2.0 * 4096 ** 3, "bytes": 134_217_728.0}
    r = bench.roofline_line(plan, 1.0, 0.1, PEAKS, "measured")
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s" and r["peak"] == 1634.5
    assert abs(r["achieved"] - plan["flops"] / 1e-4 / 1e12) < 0.01
    assert abs(r["frac"] - r["achieved"] / 1634.5) < 1e-4
    assert "hbm_frac" in r and "frac_burst" not in r and r["peak_kind"] == "measured (burst)"


def test_conv_below_the_ridge_is_hbm_bound():
    plan = {"flops": 7_398_752_256.0, "bytes": 38_608_896.0}
    r = bench.roofline_line(plan, 1.0, 0.014, PEAKS, "measured")
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["peak"] == 6544.7
    assert abs(r["achieved"] - 38_608_896.0 / 14e-6 / 1e9) < 0.01
    assert abs(r["tensor_frac"] - plan["flops"] / 14e-6 / 1e12 / 1634.5) < 1e-4


def test_elementwise_has_no_tensor_fraction():
    r = bench.roofline_line({"flops": 0.0, "bytes": 50_331_648.0}, 1.0, 0.009, PEAKS, "measured")
    assert r["bound"] == "hbm" and "tensor_frac" not in r and "hbm_frac" not in r


def test_long_tensor_launches_also_report_the_sustained_fraction():
    plan = {"flops": 2.0 * 32768 * 8192 * 8192, "bytes": 1.6e9}
    r = bench.roofline_line(plan, 1.0, 3.2, PEAKS, "measured")
    assert r["bound"] == "tensor" and r["peak"] == 1634.5 and r["peak_kind"] == "measured (burst)"
    assert abs(r["frac_sustained"] - r["achieved"] / 1385.9) < 1e-4
    # a share of the Grid scales the work, not the time
    half = bench.roofline_line(plan, 0.5, 3.2, PEAKS, "measured")
    assert abs(half["achieved"] - r["achieved"] / 2) < 0.02


def test_clock_summary_from_nvml_samples():
    c = bench.ClockSampler("GPU-test")
    c.rows = [(1965.0, 1965.0, 700.0, 0), (1800.0, 1965.0, 990.0, 0x4), (1965.0, 1965.0, 800.0, 0)]
    s = c.summary()
    assert s["sm_mhz"] == 1965.0 and s["sm_min_mhz"] == 1800.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"] and s["power_w_max"] == 990.0


def test_clock_summary_without_samples_is_marked_unavailable():
    assert bench.ClockSampler("GPU-test").summary()["reasons"] == ["unavailable"]


def test_int8_roofline_doubles_the_tensor_peak():
    # int8 ops are measured against twice the bf16 peaks, in TOP/s
    plan = {"flops": 2.0 * 8192 ** 3, "bytes": 3 * 8192 ** 2}
    r = bench.roofline_line(plan, 1.0, 0.332, PEAKS, "measured", int8=True)
    assert r["bound"] == "tensor" and r["unit"] == "TOP/s"
    assert r["peak"] == 2 * PEAKS["bf16_tflops"]
    assert abs(r["frac"] - plan["flops"] / 0.332e-3 / 1e12 / (2 * PEAKS["bf16_tflops"])) < 1e-3
    assert "int8 = 2 x bf16" in r["peak_kind"]


def test_launch_arrays_places_the_output():
    # kernels/matmul.py takes (lhs, rhs, res, scale, bias): the output third
    assert bench.launch_arrays({"out_pos": 2}, ["a", "b", "s", "t"], "o") == ["a", "b", "o", "s", "t"]
    assert bench.launch_arrays({}, ["a", "b"], "o") == ["a", "b", "o"]


def test_extra_workloads_plan_onto_their_families():
    import torch
    import xtile as xt
    fams = {name: xt.parse(bench.build_workload(name, bench.load_dsl(), torch, 1, 0)["text"]).plan()["family"]
            for name in ("silu", "row_center", "row_bias", "transpose", "matmul_i8", "col_sums", "col_bias",
                         "softmax_wide")}
    assert fams == {"silu": "ew", "row_center": "rows", "row_bias": "ew", "transpose": "tile", "matmul_i8": "gemm",
                    "col_sums": "tile", "col_bias": "tile", "softmax_wide": "rows"}


@pytest.mark.parametrize("name", ["add", "softmax", "matmul", "conv2d", "sharded_matmul", "transpose", "silu",
                                  "row_center", "row_bias", "matmul_i8", "col_sums", "col_bias", "softmax_wide"])
def test_configuration_work_matches_the_plan(name):
    # the reference arm takes the work from the configuration's formula; the
    # planner must count the same bytes / FLOP for the GPU arm
    import torch
    import xtile as xt
    w = bench.build_workload(name, bench.load_dsl(), torch, 1, 0)
    plan = xt.parse(w["text"]).plan()
    assert (plan["flops"] if w["unit"] in bench.OPS_UNITS else plan["bytes"]) == w["work"]


def test_reference_arm_loads_no_library_of_this_repository(tmp_path):
    # the reference arm traces with the pure-Python DSL and times the oracle:
    # neither the _xtile extension nor libxt_b200.so may be mapped
    code = (
        "import sys, io, contextlib, json\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'add', '--steps', '1', '--warmup', '1']\n"
        "import bench\n"
        "buf = io.StringIO()\n"
        "with contextlib.redirect_stdout(buf):\n"
        "    bench.main()\n"
        "line = json.loads(buf.getvalue().strip().splitlines()[-1])\n"
        "maps = open('/proc/self/maps').read()\n"
        "print(json.dumps({'line': line, 'so': [m for m in ('libxt_b200', '_xtile') if m in maps],\n"
        "                  'mods': [m for m in sys.modules if m.startswith(('xtile', 'xtile_b200'))]}))\n")
    res = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    assert out["so"] == [] and out["mods"] == []
    line = out["line"]
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "GB/s"
    assert line["cpu_baseline"]["cores"] >= 1 and line["e2e"]["h2d_bytes_per_step"] == 0


def _small_matmul_workload(torch):
    dsl = bench.load_dsl()
    A = dsl.Array

    @dsl.kernel
    def matmul_rows(lhs, rhs, out, tm, tn, tk):
        i, j = dsl.bid(0), dsl.bid(1)
        a = dsl.load(lhs, index=(i, 0), shape=(tm, tk))
        b = dsl.load(rhs, index=(0, j), shape=(tk, tn), shared=1)
        dsl.store(out, index=(i, j), tile=dsl.matmul(a, b))

    M, N, K = 64, 48, 32
    g = torch.Generator().manual_seed(3)
    a = (torch.randn(M, K, generator=g) / 4).to(torch.bfloat16)
    b = (torch.randn(K, N, generator=g) / 4).to(torch.bfloat16)
    text = dsl.trace_text(matmul_rows, args=(A((M, K), dsl.bfloat16), A((K, N), dsl.bfloat16), A((M, N), dsl.float32),
                                             8, 16, K), grid=(8, 3, 1), double_buffering=True)
    w = dict(text=text, inputs=[a, b], out_shape=(M, N), out_dtype=torch.float32, unit="TFLOP/s", dtype="bf16",
             work=2 * M * N * K)
    full = (a.double() @ b.double()).float()
    return w, full


def test_sample_check_passes_the_right_output_and_catches_a_planted_error():
    import torch
    w, full = _small_matmul_workload(torch)
    c = bench.sample_check(w, full, torch, n_blocks=24)
    assert c["ok"] and c["blocks"] == 24 and c["values"] == 64 * 48
    bad = full.clone()
    bad[13, 7] += 1.0  # a wrong value in a sampled Block
    assert not bench.sample_check(w, bad, torch, n_blocks=24)["ok"]


def test_gather_check_covers_every_shard_and_the_boundary_rows():
    import torch
    w, full = _small_matmul_workload(torch)
    shares = [bench.bid0_share(8, 3, r, 0.5) for r in range(3)]
    c = bench.gather_check(w, full, shares, 8, torch)
    assert c["ok"] and c["blocks"] == 9 and c["rows"] == 4
    bad = full.clone()
    bad[shares[1][0] * 8, 40] -= 0.5  # first row of rank 1's range
    assert not bench.gather_check(w, bad, shares, 8, torch)["ok"]


def test_close_enough_modes():
    import numpy as np
    x = np.array([0.25, 0.5], np.float32)
    assert bench.close_enough(x, x.copy(), "softmax")["ok"]
    assert not bench.close_enough(x, x * (1 + 1e-4), "softmax")["ok"]
    y = np.array([-1.5, 2.0], np.float32)
    assert not bench.close_enough(y, np.nextafter(y, np.inf), "bit-exact")["ok"]  # add: one ulp is a failure
    assert bench.close_enough(y, np.nextafter(y, np.inf), "transcendental")["ok"]  # silu: one ulp is fine
    assert not bench.close_enough(y, y * 1.001, "transcendental")["ok"]
    assert bench.close_enough(y * 1.001, y, "bf16")["ok"]
    assert bench.tolerance_of({"dtype": "bf16"}) == "bf16" and bench.tolerance_of({"dtype": "f32"}) == "bit-exact"
