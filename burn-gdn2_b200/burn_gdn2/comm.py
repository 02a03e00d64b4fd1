"""Process-group set-up and the deadline-bounded all-reduce of the head-sharded
layer (multi-GPU plumbing; the reference has no distributed code).

The one collective of a sharded layer is the all-reduce of the row-parallel
o_proj partials.  A rank that dies or stalls between steps must not leave the
other ranks waiting forever, so:

* ``init_process_group`` creates NCCL communicators non-blocking
  (``ncclCommInitRankConfig`` with ``blocking = 0``) under the group's
  timeout, which also bounds every later collective (torch's NCCL watchdog
  aborts the communicator once it passes);
* ``all_reduce_deadline`` issues the all-reduce asynchronously, polls it
  against a deadline on the host and, when the deadline passes, aborts the
  process group and raises ``CollectiveTimeout``, a bounded error the caller
  can act on.

Failure is detected on the host only: no kernel waits on another rank.
"""
from __future__ import annotations

import time
from datetime import timedelta


class CollectiveTimeout(RuntimeError):
    """A collective did not complete before its deadline; the group was aborted."""


def init_process_group(backend: str, timeout_s: float = 60.0, device=None):
    """torch.distributed.init_process_group with a bounded timeout; NCCL
    communicators are initialised non-blocking.  Rank, world size and the
    rendezvous address come from the environment (RANK, WORLD_SIZE,
    MASTER_ADDR, MASTER_PORT)."""
    import torch.distributed as dist

    kw = dict(timeout=timedelta(seconds=timeout_s))
    if backend == "nccl":
        from torch.distributed import ProcessGroupNCCL

        opts = ProcessGroupNCCL.Options()
        opts.config.blocking = 0
        kw["pg_options"] = opts
        if device is not None:
            kw["device_id"] = device
    dist.init_process_group(backend, **kw)


def abort(group=None):
    """Abort the (default) process group's communicators so that no
    collective of this rank keeps waiting on a peer."""
    import torch.distributed as dist

    pg = group if group is not None else dist.distributed_c10d._get_default_group()
    try:
        pg.abort()
    except (AttributeError, RuntimeError, NotImplementedError):
        dist.distributed_c10d._abort_process_group(group)


def all_reduce_deadline(t, deadline_s: float, group=None, poll_s: float = 1e-3):
    """In-place sum all-reduce of `t` that completes or raises
    CollectiveTimeout within about `deadline_s` seconds.  Errors the backend
    reports (a peer's connection closed) propagate as they are."""
    import torch.distributed as dist

    work = dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group, async_op=True)
    end = time.monotonic() + deadline_s
    while not work.is_completed():
        if time.monotonic() > end:
            abort(group)
            raise CollectiveTimeout(f"all_reduce of {tuple(t.shape)} did not complete within {deadline_s} s; "
                                    "process group aborted")
        time.sleep(poll_s)
    work.wait()
    return t
