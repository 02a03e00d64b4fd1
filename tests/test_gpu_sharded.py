"""GPU parity of the head-sharded layer: ShardedGatedDeltaNet2 on the CUDA
path (per-rank GatedDeltaNet2 shards, the overlapped chunk-mode
forward_train with its all-reduce of the o_proj partials, and the stateful
forward) against the unsharded layer on the same weights and inputs.

Two forms: two gloo ranks that share one GPU (the collective moves the CUDA
tensors through the host; runs wherever one GPU is), and two NCCL ranks on
two GPUs (skipped with fewer).  No kernel of one rank waits on another rank."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from helpers import assert_close_normwise

PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "burn-gdn2_b200")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, backend, cfgd, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, PKG)
    import torch.distributed as dist
    import burn_gdn2 as bg
    from burn_gdn2 import comm, sharding

    dev = torch.device("cuda", rank if backend == "nccl" else 0)
    torch.cuda.set_device(dev)
    comm.init_process_group(backend, timeout_s=60, device=dev if backend == "nccl" else None)
    try:
        cfg = bg.Gdn2Config(mode=bg.Gdn2Mode.Chunk, chunk_size=64, **cfgd)
        full = bg.GatedDeltaNet2.new(cfg, device=dev, dtype=torch.bfloat16, seed=31)
        m = sharding.ShardedGatedDeltaNet2(cfg, full.export_weights(), device=dev, dtype=torch.bfloat16)
        g = torch.Generator(device=dev).manual_seed(32)
        x = torch.randn(2, 200, cfg.hidden_size, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
        y = m.forward_train(x)  # chunk mode: the overlapped ranges
        y2, _ = m.forward(x[:, :9], None, True)  # T <= 64: the fused recurrent kernel, one all-reduce
        torch.cuda.synchronize()
        if rank == 0:
            ref = full.forward_train(x)
            ref2, _ = full.forward(x[:, :9], None, True)
            torch.cuda.synchronize()
            f = lambda t: t.float().cpu().numpy()
            q.put((f(y), f(ref), f(y2), f(ref2), len(m.pop_allreduce_ms())))
    finally:
        dist.destroy_process_group()


def _run(world, backend, cfgd):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, backend, cfgd, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    y, ref, y2, ref2, ncalls = res
    assert ncalls == 2
    # Whole-layer bf16 criterion, tightened to 1e-2: each rank's o_proj partial is a bf16 tensor before the sum
    # (as in any bf16 tensor-parallel layer), so an output entry that is a cancellation between the ranks'
    # partials carries their rounding, and no per-element relative bound holds for it.
    assert_close_normwise(y, ref, 1e-2, what="sharded forward_train")
    assert_close_normwise(y2, ref2, 1e-2, what="sharded forward")


CFGS = [dict(hidden_size=512, num_heads=4, head_dim=128),
        dict(hidden_size=512, num_heads=2, head_dim=128, num_v_heads=4, min_decay=0.9, allow_neg_eigval=True)]


@pytest.mark.gpu
@pytest.mark.parametrize("cfgd", CFGS)
def test_sharded_layer_matches_unsharded_two_ranks_one_gpu(cfgd):
    _run(2, "gloo", cfgd)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("cfgd", CFGS[:1])
def test_sharded_layer_matches_unsharded_nccl_two_gpus(cfgd):
    _run(2, "nccl", cfgd)
