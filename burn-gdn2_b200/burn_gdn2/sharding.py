"""Head sharding of one GDN-2 layer over ranks (multi-GPU, one process per GPU).

(batch x value-head) recurrence chains are independent, so a layer splits by
heads with no communication inside the recurrence: rank r of N owns key heads
[r H/N, (r+1) H/N) and the matching value heads (whole GVA groups, value head
h*rep + j follows key head h, src/module.rs:457-468).  Column-parallel:
q, k, b, f_proj_1 (key channels), v, w, g_proj_1 (value channels), A_log,
dt_bias, decay_factors and the conv weights / caches / state.  Replicated:
f_proj_0, g_proj_0, o_norm_w.  Row-parallel: o_proj, whose partial outputs are
summed by one all-reduce (NCCL over NVLink on B200) per layer call.
"""
from __future__ import annotations

import dataclasses

import numpy as np


def shard_config(cfg, world: int):
    """The per-rank config: num_heads / N key heads, num_v_heads / N value
    heads; everything else unchanged (the per-rank layer sees a smaller
    model of the same head shape)."""
    h, hv = cfg.num_heads, (cfg.num_v_heads if cfg.num_v_heads is not None else cfg.num_heads)
    if h % world:
        raise ValueError(f"num_heads={h} is not divisible by the {world} ranks")
    local = dataclasses.replace(cfg, num_heads=h // world,
                                num_v_heads=None if cfg.num_v_heads is None else hv // world)
    return local


def shard_weights(weights: dict, cfg, rank: int, world: int) -> dict:
    """Slice the layer weights ([in, out] burn layout) for `rank` of `world`."""
    h, hk = cfg.num_heads, cfg.head_dim
    hv = cfg.num_v_heads if cfg.num_v_heads is not None else h
    vh = int(np.float32(hk) * np.float32(cfg.expand_v))
    kd, vd = h * hk, hv * vh
    kk = slice(rank * kd // world, (rank + 1) * kd // world)
    vv = slice(rank * vd // world, (rank + 1) * vd // world)
    hh = slice(rank * h // world, (rank + 1) * h // world)
    out = {}
    for name, w in weights.items():
        w = np.asarray(w) if not hasattr(w, "detach") else w
        if name in ("q_proj", "k_proj", "b_proj", "f_proj_1"):
            out[name] = w[:, kk]
        elif name in ("v_proj", "w_proj", "g_proj_1_w"):
            out[name] = w[:, vv]
        elif name == "g_proj_1_b":
            out[name] = w[vv]
        elif name in ("q_conv_w", "k_conv_w", "dt_bias"):
            out[name] = w[kk]
        elif name == "v_conv_w":
            out[name] = w[vv]
        elif name in ("A_log", "decay_factors"):
            out[name] = w[hh]
        elif name == "o_proj":
            out[name] = w[vv, :]
        else:  # f_proj_0, g_proj_0, o_norm_w
            out[name] = w
    return out


class ShardedGatedDeltaNet2:
    """One layer split by heads over a torch.distributed process group.

    Each rank holds a GatedDeltaNet2 of H/N key heads (and HV/N value heads)
    built from `shard_weights`; `forward_train` / `forward` return the full
    output after one all-reduce (sum) of the row-parallel o_proj partials.
    Every all-reduce is bracketed by CUDA events on the current stream and
    nothing waits on them here, so a timed loop of layer calls never stalls
    the host; `pop_allreduce_ms()` (after the caller has synchronised) returns
    the all-reduce time of each call since the last pop, so it can be
    reported separately.
    """

    def __init__(self, cfg, weights: dict, group=None, device="cuda", dtype=None, **kw):
        import torch
        import torch.distributed as dist

        from .module import GatedDeltaNet2

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.config = cfg
        self.local = GatedDeltaNet2(shard_config(cfg, self.world), shard_weights(weights, cfg, self.rank, self.world),
                                    device=device, dtype=dtype or torch.float32, **kw)
        self._events = []

    def _reduce(self, y):
        import torch

        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        self.dist.all_reduce(y, op=self.dist.ReduceOp.SUM, group=self.group)
        e1.record()
        self._events.append((e0, e1))
        return y

    def pop_allreduce_ms(self):
        """All-reduce times (ms) of the calls since the last pop, oldest
        first.  Call after the work has completed (e.g. after
        torch.cuda.synchronize()); it does not wait itself."""
        out = [e0.elapsed_time(e1) for e0, e1 in self._events]
        self._events = []
        return out

    def forward_train(self, x):
        return self._reduce(self.local.forward_train(x))

    def forward(self, x, state=None, update_state=True):
        y, state = self.local.forward(x, state, update_state)
        return self._reduce(y), state
