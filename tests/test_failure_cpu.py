"""Failure handling of the multi-rank path, on the host (gloo, CPU ranks, no
GPU): a rank that stalls or exits between steps makes the other ranks' next
all-reduce of the o_proj partials end with a bounded error
(burn_gdn2.comm.all_reduce_deadline) instead of waiting forever, and a rank
that never joins makes the others' process-group set-up fail within its
timeout."""
import os
import socket
import sys
import time

import pytest
import torch.multiprocessing as mp

PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "burn-gdn2_b200")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _report(q, item):
    """Put `item` and flush the queue's feeder thread (the worker leaves with
    os._exit, which would otherwise drop it)."""
    q.put(item)
    q.close()
    q.join_thread()


def _env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, PKG)


def _step_worker(rank, world, port, mode, q):
    """Step 0: every rank joins the all-reduce.  Then the last rank stalls
    (sleeps past the others' deadline) or exits; the others run step 1 with
    a 2 s deadline and report how it ended."""
    _env(rank, world, port)
    import torch
    from burn_gdn2 import comm

    comm.init_process_group("gloo", timeout_s=30)
    t = torch.ones(8)
    comm.all_reduce_deadline(t, 20.0)
    ok0 = bool((t == world).all())
    if rank == world - 1:
        _report(q, (rank, "left", ok0, 0.0))
        if mode == "stall":
            time.sleep(6.0)
        os._exit(0)  # leaves between steps, with nothing in flight
    t0 = time.monotonic()
    try:
        comm.all_reduce_deadline(torch.ones(8), 2.0)
        how = "completed"
    except comm.CollectiveTimeout:
        how = "timeout"
    except Exception as e:  # the backend saw the peer's connection close
        how = "error:" + type(e).__name__
    _report(q, (rank, how, ok0, time.monotonic() - t0))
    os._exit(0)


@pytest.mark.parametrize("mode", ["stall", "exit"])
@pytest.mark.parametrize("world", [2, 3])
def test_rank_failure_between_steps_is_a_bounded_error(mode, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_step_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=30)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = {r[0]: r[1:] for r in res}
    assert all(ok0 for _, ok0, _ in res.values()), res
    for rank in range(world - 1):
        how, _, elapsed = res[rank]
        assert how == "timeout" or how.startswith("error:"), res
        assert elapsed < 15.0, res


def _init_worker(rank, world, port, q):
    _env(rank, world, port)
    from burn_gdn2 import comm

    t0 = time.monotonic()
    try:
        comm.init_process_group("gloo", timeout_s=3)
        how = "joined"
    except Exception as e:
        how = "error:" + type(e).__name__
    _report(q, (how, time.monotonic() - t0))
    os._exit(0)


def test_rank_that_never_joins_fails_set_up_within_timeout():
    """World size 2, only rank 0 starts: its rendezvous gives up within the
    3 s group timeout (plus the store's own retry slack)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_init_worker, args=(0, 2, _free_port(), q))
    p.start()
    how, elapsed = q.get(timeout=120)
    p.join(timeout=30)
    if p.is_alive():
        p.kill()
    assert how.startswith("error:"), how
    assert elapsed < 60.0, elapsed
