"""The CPU oracle timed on every host core -- TEST INFRASTRUCTURE ONLY.

``bench.py``'s CPU baseline (``cpu_baseline`` and the ``--impl reference``
arm) times the oracle of ``xt_oracle.py`` -- the CPU restatement of the
reference's semantics -- on a bounded sample of a workload's Blocks.  xtile
Blocks are independent (the reference's README, "Blocks are logically
independent"), so the baseline runs them in parallel: one worker process per
host core, each with a single BLAS thread, each taking its own slice of a
seeded random permutation of the Grid.  The arrays live in files under a
temporary directory, memory-mapped shared by every worker (a worker's stores
land in the one output mapping, as the Blocks' stores would).

Workers are started with ``spawn`` (never ``fork``), so a caller that has
already used CUDA can start them safely.  The product path never imports
this module.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import shutil
import tempfile
import time

import numpy as np


def host_cores() -> int:
    """Cores this process may run on (its affinity mask), not the machine's count."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - not Linux
        return os.cpu_count() or 1


def _serve(rank: int, procs: int, text: str, func: str | None, paths: list[str], seed: int,
           cmd_q, res_q) -> None:
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(1)  # parallelism is across Blocks: one BLAS thread per process
    except ImportError:  # pragma: no cover - the environment variables below still apply
        pass
    from oracle import xt_oracle

    funcs = xt_oracle.parse_module(text)
    f = funcs[0] if func is None else next(fn for fn in funcs if fn.name == func)
    arrays = [np.load(p, mmap_mode="r+") for p in paths]
    interp = xt_oracle.Interpreter(f)
    interp.run(arrays, blocks=[])  # binds the arrays
    order = xt_oracle.serialize_order(f.grid)
    picks = np.random.default_rng(seed).permutation(len(order))[rank::procs]
    pos = 0
    res_q.put(("ready", rank, 0, 0.0))
    while True:
        cmd = cmd_q.get()
        if cmd is None:
            break
        budget_s, start_at = cmd
        while time.time() < start_at:  # every worker starts its sample at the same moment
            time.sleep(0.0002)
        t0 = time.perf_counter()
        done = 0
        while len(picks) and time.perf_counter() - t0 < budget_s:
            interp.run_block(order[picks[pos % len(picks)]])
            pos += 1
            done += 1
        res_q.put(("done", rank, done, time.perf_counter() - t0))


class BlockTimer:
    """Worker pool timing the oracle on samples of one function's Blocks.

    ``arrays`` are numpy arrays in the function's memref order (bf16 as uint16
    bit patterns), inputs filled and outputs allocated.  ``sample(budget_s)``
    runs every worker for about ``budget_s`` seconds of Blocks and returns
    ``(blocks_done, seconds)`` with seconds the longest worker's time.
    """

    def __init__(self, text: str, arrays: list[np.ndarray], procs: int | None = None, seed: int = 0,
                 func: str | None = None, start_timeout_s: float = 300.0) -> None:
        from oracle import xt_oracle

        funcs = xt_oracle.parse_module(text)
        f = funcs[0] if func is None else next(fn for fn in funcs if fn.name == func)
        self.n_blocks = len(xt_oracle.serialize_order(f.grid))
        self.procs = max(1, min(procs or host_cores(), self.n_blocks))
        self.text, self.func, self.seed = text, func, seed
        self.arrays = arrays
        self.start_timeout_s = start_timeout_s
        self.dir = None
        self.workers: list = []

    def __enter__(self) -> "BlockTimer":
        self.dir = tempfile.mkdtemp(prefix="xt_oracle_")
        paths = []
        for i, a in enumerate(self.arrays):
            p = os.path.join(self.dir, f"a{i}.npy")
            m = np.lib.format.open_memmap(p, mode="w+", dtype=a.dtype, shape=a.shape)
            if np.any(a):
                m[...] = a
            m.flush()
            del m
            paths.append(p)
        ctx = mp.get_context("spawn")
        self.res_q = ctx.Queue()
        self.cmd_qs = [ctx.Queue() for _ in range(self.procs)]
        saved = {k: os.environ.get(k) for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")}
        os.environ.update(OMP_NUM_THREADS="1", OPENBLAS_NUM_THREADS="1", MKL_NUM_THREADS="1")
        try:
            for r in range(self.procs):
                p = ctx.Process(target=_serve, args=(r, self.procs, self.text, self.func, paths, self.seed,
                                                     self.cmd_qs[r], self.res_q), daemon=True)
                p.start()
                self.workers.append(p)
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
        for _ in range(self.procs):
            self.res_q.get(timeout=self.start_timeout_s)
        return self

    def sample(self, budget_s: float) -> tuple[int, float]:
        start_at = time.time() + 0.05
        for q in self.cmd_qs:
            q.put((budget_s, start_at))
        done, secs = 0, 0.0
        for _ in range(self.procs):
            _, _, d, dt = self.res_q.get(timeout=budget_s + self.start_timeout_s)
            done += d
            secs = max(secs, dt)
        return done, secs

    def __exit__(self, *exc) -> None:
        for q in self.cmd_qs:
            q.put(None)
        for p in self.workers:
            p.join(timeout=10)
            if p.is_alive():
                p.terminate()
        if self.dir:
            shutil.rmtree(self.dir, ignore_errors=True)
