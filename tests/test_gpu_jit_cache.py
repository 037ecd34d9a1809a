"""The on-disk cache of generated kernels, in fresh processes on a GPU.

A first launch of a generated program compiles it with NVRTC and writes the
cubin to the cache directory; a second process finds it there and computes
the same result; a damaged file is compiled again; XT_JIT_CACHE=0 writes
nothing.  Each run is a subprocess so that the in-process program cache does
not hide the disk.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import xtile as xt

@xt.kernel
def prog(x, y, trow, col):
    i = xt.bid(0)
    t = xt.load(x, index=(i, 0), shape=(trow, col))
    xt.store(y, index=(i, 0), tile=xt.tanh(t) * t + t)

x = torch.linspace(-3, 3, 64 * 96, device="cuda").reshape(64, 96)
y = torch.empty_like(x)
m = xt.run(prog, args=(x, y, 16, 96), grid=(4, 1, 1))
assert m.plan()["family"] == "ew"
torch.cuda.synchronize()
torch.save(y.cpu(), sys.argv[2])
"""


def run(tmp_path, tag, **env):
    out = tmp_path / f"{tag}.pt"
    e = dict(os.environ, **env)
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), str(out)], env=e, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    import torch
    return torch.load(out)


def test_cubins_persist_across_processes(tmp_path):
    import torch
    cache = tmp_path / "cache"
    first = run(tmp_path, "first", XT_JIT_CACHE_DIR=str(cache))
    files = sorted(cache.glob("*.cubin"))
    assert files and not list(cache.glob("*.tmp.*"))
    stamp = {f: f.stat().st_mtime_ns for f in files}
    second = run(tmp_path, "second", XT_JIT_CACHE_DIR=str(cache))
    assert torch.equal(first, second)
    assert {f: f.stat().st_mtime_ns for f in sorted(cache.glob("*.cubin"))} == stamp  # read, not rewritten
    # a damaged file (cut short) is compiled again and replaced
    f = files[0]
    f.write_bytes(f.read_bytes()[:100])
    third = run(tmp_path, "third", XT_JIT_CACHE_DIR=str(cache))
    assert torch.equal(first, third)
    assert f.stat().st_size > 100


def test_cache_off_writes_nothing(tmp_path):
    cache = tmp_path / "cache"
    run(tmp_path, "off", XT_JIT_CACHE="0", XT_JIT_CACHE_DIR=str(cache))
    assert not cache.exists()
