"""World-size-2 runs of the bid0 sharding on the CPU (gloo backend).

Each rank computes its share of a matmul Grid's Blocks - the share
``bench.bid0_share`` gives it, the one ``bench.py`` launches on that rank's
GPU - with the reference interpreter standing in for the kernel; the shares
are gathered to rank 0 with the benchmark's own gather and rank 0 compares
with a single-process run of the whole Grid.  This covers the partition
arithmetic, the gather and the order of the collectives; the kernels
themselves are covered by the GPU tests.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
import xtile_b200 as xt
from oracle import xt_oracle


@xt.kernel
def matmul_rows(lhs, rhs, out, tm, tn, tk):
    i, j = xt.bid(0), xt.bid(1)
    a = xt.load(lhs, index=(i, 0), shape=(tm, tk))
    b = xt.load(rhs, index=(0, j), shape=(tk, tn), shared=1)
    xt.store(out, index=(i, j), tile=xt.matmul(a, b))


M, N, K, TM, TN = 64, 32, 16, 8, 16
GRID = (M // TM, N // TN, 1)


def inputs():
    rng = np.random.default_rng(11)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((K, N)).astype(np.float32)
    return xt_oracle.f32_to_bf16(a), xt_oracle.f32_to_bf16(b)  # bf16 bit patterns


def module_text():
    A = xt.Array
    mod = xt.convert(matmul_rows, args=(A((M, K), xt.bfloat16), A((K, N), xt.bfloat16), A((M, N), xt.float32),
                                        TM, TN, K), grid=GRID)
    return str(mod)


def shard_worker(rank, world, port, text):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a, b = inputs()
        out = np.full((M, N), np.nan, dtype=np.float32)
        lo, hi = bench.bid0_share(GRID[0], world, rank)
        blocks = [(i, j, 0) for i in range(lo, hi) for j in range(GRID[1])]
        xt_oracle.run(text, [a, b, out], blocks=blocks)
        out_t = torch.from_numpy(out)
        bench.nccl_gather(out_t, M // world, world, rank, dist)
        if rank == 0:
            ref = np.zeros((M, N), dtype=np.float32)
            xt_oracle.run(text, [a, b, ref])
            assert np.array_equal(out_t.numpy(), ref), "gathered shards differ from the single-rank result"
            # each rank computed exactly its own rows
            assert (hi - lo) * TM == M // world
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2])
def test_bid0_shards_gathered_to_rank0(world):
    text = module_text()
    mp.start_processes(shard_worker, args=(world, free_port(), text), nprocs=world, join=True, start_method="spawn")


def test_bid0_share_partitions_the_grid():
    for grid0 in (1, 7, 128):
        for world in (1, 2, 3, 8):
            spans = [bench.bid0_share(grid0, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == grid0
            assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))


def test_bid0_share_with_root_share_partitions_the_grid():
    for grid0 in (8, 13, 128):
        for world in (2, 3, 8):
            if grid0 < world:
                continue
            for f in (0.0, 0.1, 0.342, 0.9, 1.0):
                spans = [bench.bid0_share(grid0, world, r, f) for r in range(world)]
                assert spans[0][0] == 0 and spans[-1][1] == grid0
                assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))
                assert all(hi > lo for lo, hi in spans)  # every rank gets at least one Block
                sizes = [hi - lo for lo, hi in spans[1:]]
                assert max(sizes) - min(sizes) <= 1  # the other ranks split the rest evenly


def test_gather_root_share_balances_compute_and_ingress():
    flops, out_bytes = 2.0 * 32768 * 8192 * 8192, 32768 * 8192 * 4
    assert bench.gather_root_share(1, flops, out_bytes) == 1.0
    # two GPUs: rank 1's compute, not rank 0's ingress, bounds the step
    assert abs(bench.gather_root_share(2, flops, out_bytes) - 0.5) < 1e-12
    for world in (4, 8):
        f = bench.gather_root_share(world, flops, out_bytes)
        t = flops / (bench.SHARDED_GEMM_TFLOPS * 1e12)
        r = out_bytes / (bench.PEER_INGEST_GBS * 1e9)
        # rank 0's compute equals its ingress, and the other ranks finish first
        assert abs(f * t - (1 - f) * r) < 1e-12
        assert (1 - f) / (world - 1) * t <= f * t
    # slower links give rank 0 more of the Grid
    assert bench.gather_root_share(8, flops, out_bytes, ingest_gbs=300.0) > bench.gather_root_share(8, flops, out_bytes)


# ---------------------------------------------------------------------------
# Failure detection on the host (gloo ranks, no GPU): a rank that never joins,
# and a rank that leaves between steps.  The surviving rank must end with an
# error within a bounded time, never hang.
# ---------------------------------------------------------------------------
def never_joins_worker(rank, world, port, result_q):
    import datetime
    import time

    if rank == 1:
        return  # this rank never joins the process group
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
        result_q.put(("joined", time.monotonic() - t0))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - the error itself is what is checked
        result_q.put((type(e).__name__, time.monotonic() - t0))


def test_rank_that_never_joins_ends_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=never_joins_worker, args=(r, 2, free_port(), q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, secs = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert kind != "joined"
    assert secs < 60


def leaves_between_steps_worker(rank, world, port, result_q):
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)  # step 0: both ranks
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)  # step 1: the peer is gone
        result_q.put(("completed", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001
        result_q.put((type(e).__name__, time.monotonic() - t0))


def test_rank_that_leaves_between_steps_fails_the_next_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=leaves_between_steps_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, secs = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
    assert kind != "completed"
    assert secs < 60


def test_plan_root_blocks_minimises_the_step_model():
    # one-GPU GEMM 3.18 ms, rank 0 ingesting the whole output in 1.42 ms
    t, r = 3.18, 1.42
    for world, slabs in ((2, 0), (4, 0), (8, 0), (4, 4), (8, 4)):
        b0 = bench.plan_root_blocks(128, world, t, r, slabs)
        best = bench.gather_step_ms(b0 / 128, world, t, r, slabs)
        assert all(bench.gather_step_ms(b / 128, world, t, r, slabs) >= best - 1e-12 for b in range(1, 128 - world + 2))
    # copy-engine slabs: more ranks finish their first slab sooner, so 8 GPUs model faster than 4
    s4 = bench.gather_step_ms(bench.plan_root_blocks(128, 4, t, r, 4) / 128, 4, t, r, 4)
    s8 = bench.gather_step_ms(bench.plan_root_blocks(128, 8, t, r, 4) / 128, 8, t, r, 4)
    assert s8 < s4
    # with stores from the GEMM itself the bound is T*R/(T+R) at any world >= 3
    s = bench.gather_step_ms(bench.plan_root_blocks(128, 8, t, r, 0) / 128, 8, t, r, 0)
    assert s >= t * r / (t + r) - 1e-9


def heartbeat_worker(rank, world, port, result_q):
    import datetime

    from xtile_b200 import ranks

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    hb = ranks.Heartbeat(rank, world)
    t = torch.ones(4)
    for step in range(3):
        if rank == 1 and step == 1:
            os._exit(0)  # leaves between steps, before announcing step 1
        hb.beat(step)
        try:
            hb.wait_all(step, deadline_s=2.0)
        except ranks.PeerLost as e:
            result_q.put(("lost", step, str(e)))
            return  # the survivor stops before launching the step's collective
        dist.all_reduce(t)
    result_q.put(("done", 3, ""))


def test_heartbeat_notices_a_rank_that_left_before_the_next_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=heartbeat_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, step, msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
    assert kind == "lost" and step == 1 and "ranks [1]" in msg
