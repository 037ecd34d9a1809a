"""One process per GPU: the NCCL process group of a Grid split along bid0,
with failure detection on the host.

The reference has no runtime and no collectives; this is the control side of
the multi-GPU path (a bid0 range per GPU, rows gathered to rank 0):

* ``init_nccl`` creates the process group with a *non-blocking* NCCL
  communicator (``ncclCommInitRankConfig`` with ``blocking = 0``) and a short
  timeout, so no host call waits on a peer for longer than that;
* ``Heartbeat`` lets every rank tell the others, through the process group's
  store, that it has reached a step before any collective of that step is
  launched.  A rank that left between steps is noticed on the host before its
  peers launch a kernel that would wait for it;
* ``check`` reads the communicator's asynchronous error
  (``ncclCommGetAsyncError``) and ``abort`` tears the communicator down
  (``ncclCommAbort``); both are host calls with nothing of ours in flight.

Ranks leave only between steps; a step's kernels and collectives are never
abandoned half-way.
"""
from __future__ import annotations

import datetime


class PeerLost(RuntimeError):
    """A peer did not reach a step within the heartbeat deadline."""


def init_nccl(device, timeout_s: float = 30.0, blocking: bool = False, rank: int | None = None,
              world_size: int | None = None):
    """NCCL process group for ``device``; ``rank`` and ``world_size`` default
    to the environment's (torchrun sets them).  Returns the group."""
    import torch.distributed as dist
    from torch._C._distributed_c10d import ProcessGroupNCCL

    opts = ProcessGroupNCCL.Options()
    opts.config.blocking = blocking
    kw = {} if rank is None else {"rank": rank, "world_size": world_size}
    dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=timeout_s),
                            pg_options=opts, **kw)
    return dist.group.WORLD


def _nccl_backend(group, device):
    import torch.distributed as dist

    group = group or dist.group.WORLD
    return group._get_backend(device)


def check(device, group=None) -> None:
    """Raises RuntimeError if the communicator reports an asynchronous error."""
    err = _nccl_backend(group, device).get_error()
    if str(err) not in ("ErrorType.SUCCESS", "SUCCESS", "0"):
        raise RuntimeError(f"NCCL communicator error: {err}")


def abort(device, group=None) -> None:
    """Aborts the NCCL communicator (no collective of this rank may be in flight)."""
    _nccl_backend(group, device).abort()


class Heartbeat:
    """Per-step presence of every rank, through the process group's store."""

    def __init__(self, rank: int, world: int, store=None, prefix: str = "xt/alive") -> None:
        import torch.distributed as dist

        self.rank, self.world = rank, world
        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.prefix = prefix

    def beat(self, step: int) -> None:
        self.store.set(f"{self.prefix}/{step}/{self.rank}", "1")

    def wait_all(self, step: int, deadline_s: float) -> None:
        """Returns once every rank has reached ``step``; raises PeerLost after
        ``deadline_s`` seconds otherwise."""
        keys = [f"{self.prefix}/{step}/{r}" for r in range(self.world)]
        try:
            self.store.wait(keys, datetime.timedelta(seconds=deadline_s))
        except Exception as e:  # noqa: BLE001 - the store raises its own timeout types
            missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
            raise PeerLost(f"ranks {missing} did not reach step {step} within {deadline_s} s") from e
