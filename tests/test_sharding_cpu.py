"""CPU, world_size 2, 4 and 8 over gloo: head sharding of one layer.  Each rank runs
the oracle layer on its shard of the weights; the all-reduce (sum) of the
row-parallel o_proj partials must equal the unsharded layer (forward_train
and a stateful forward), including GVA groups."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import gdn2_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cfgd, seed, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "burn-gdn2_b200"))
        from burn_gdn2 import sharding
        cfg = O.Gdn2Config(**cfgd)
        W = O.init_weights(cfg, seed=seed)
        lcfg = sharding.shard_config(cfg, world)
        lw = sharding.shard_weights(W, cfg, rank, world)
        layer = O.Gdn2Layer(lcfg, lw, np.float64)
        x = np.random.default_rng(seed + 1).standard_normal((2, 70, cfgd["hidden_size"]))
        part = torch.tensor(layer.forward_train(x))
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
        part2, _ = layer.forward(x[:, :5], None, True)
        part2 = torch.tensor(part2)
        dist.all_reduce(part2, op=dist.ReduceOp.SUM)
        if rank == 0:
            full = O.Gdn2Layer(cfg, W, np.float64)
            ref = full.forward_train(x)
            ref2, _ = full.forward(x[:, :5], None, True)
            q.put((float(np.abs(part.numpy() - ref).max()), float(np.abs(part2.numpy() - ref2).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cfgd,world", [
    (dict(hidden_size=64, num_heads=4, head_dim=16, mode="chunk"), 2),
    (dict(hidden_size=64, num_heads=2, head_dim=16, num_v_heads=4, expand_v=2.0, mode="chunk", min_decay=0.9,
          allow_neg_eigval=True), 2),
    (dict(hidden_size=64, num_heads=4, head_dim=16, mode="chunk"), 4),
    (dict(hidden_size=128, num_heads=8, head_dim=16, mode="chunk"), 8),  # the bench's widest split (N = 8)
])
def test_head_sharded_layer_matches_unsharded(cfgd, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfgd, 3, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    d1, d2 = q.get(timeout=10)
    assert d1 < 1e-10 and d2 < 1e-10, (d1, d2)
