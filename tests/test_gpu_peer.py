"""Row gather over NVLink without a collective (two GPUs, one process each).

Rank 0 exports its output array (CUDA IPC); rank 1 maps it as an
``xt.PeerArray`` and launches its bid0 share of a matmul Grid with that
array as the output, so its kernel's stores land in rank 0's memory.  After a
one-element all-reduce (the GPU-side barrier) rank 0's array must match the
CPU oracle on every Block (bf16 tolerance: max|d|/max|ref| <= 1e-2 and
|d| <= 1e-2 |ref| + 1e-2 rms(ref)) and equal a single-GPU launch of the whole
Grid bit for bit.  Skipped with fewer than two GPUs.
"""
import datetime
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


M, N, K, TM, TN = 1024, 768, 320, 128, 256


def worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(21)
        a = (torch.randn(M, K, generator=g) / K ** 0.5).to(torch.bfloat16).to(dev)
        b = (torch.randn(K, N, generator=g) / K ** 0.5).to(torch.bfloat16).to(dev)
        A = xt.Array
        mod = xt.convert(matmul_rows, args=(A((M, K), xt.bfloat16), A((K, N), xt.bfloat16), A((M, N), xt.float32),
                                            TM, TN, K), grid=(M // TM, N // TN, 1))
        out = torch.full((M, N), float("nan"), device=dev)
        box = [xt.export_array(out) if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        target = out if rank == 0 else xt.PeerArray.open(box[0], (M, N), torch.float32)
        lo, hi = bench.bid0_share(M // TM, world, rank)
        xt.launch(mod, a, b, target, bid0_range=(lo, hi))
        flag = torch.zeros(1, device=dev)
        dist.all_reduce(flag)  # every rank's rows are in rank 0's array
        torch.cuda.synchronize()
        if rank == 0:
            host = [a.cpu().view(torch.uint16).numpy(), b.cpu().view(torch.uint16).numpy(),
                    np.zeros((M, N), np.float32)]
            xt_oracle.run(mod.source_text, host)
            got = out.cpu().numpy().astype(np.float64)
            ref = host[2].astype(np.float64)
            rms = np.sqrt(np.mean(ref ** 2))
            assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) <= 1e-2
            assert np.all(np.abs(got - ref) <= 1e-2 * np.abs(ref) + 1e-2 * rms)
            one = torch.empty(M, N, device=dev)
            xt.launch(mod, a, b, one)
            torch.cuda.synchronize()
            assert torch.equal(out, one), "rows stored over NVLink differ from a single-GPU launch"
        dist.barrier()
        if rank != 0:
            target.close()
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_rows_stored_into_rank0_over_nvlink():
    mp.start_processes(worker, args=(2, free_port()), nprocs=2, join=True, start_method="spawn")


def leave_worker(rank, world, port):
    # a rank leaves between steps; the other learns of it through the
    # heartbeat before launching the next collective, reads the communicator's
    # asynchronous error and aborts the communicator with nothing in flight
    from xtile_b200 import ranks

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    ranks.init_nccl(dev, timeout_s=20.0, blocking=False, rank=rank, world_size=world)
    hb = ranks.Heartbeat(rank, world)
    t = torch.ones(4, device=dev)
    for step in range(3):
        if rank == 1 and step == 1:
            torch.cuda.synchronize()
            os._exit(0)
        hb.beat(step)
        try:
            hb.wait_all(step, deadline_s=3.0)
        except ranks.PeerLost:
            assert step == 1
            try:
                ranks.check(dev)  # the peer's exit may already show as a remote error
            except RuntimeError:
                pass
            ranks.abort(dev)
            return
        dist.all_reduce(t)
        torch.cuda.synchronize()
        assert t[0].item() == 2 ** (step + 1)
    raise AssertionError("the lost rank went unnoticed")


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_rank_leaving_between_steps_is_noticed_on_the_host():
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=leave_worker, args=(r, 2, port)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.terminate()
    assert codes == [0, 0], codes
