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
    output after the all-reduce (sum) of the row-parallel o_proj partials.

    `forward_train` in chunk mode overlaps that all-reduce with the
    recurrence: after the projections of the whole sequence, the chunk core
    runs over `overlap_segments` consecutive token ranges (whole chunks, the
    state carried from one to the next, which is the same recurrence as one
    call), and as each range completes, its o_proj GEMM and its all-reduce
    run on a side stream while the core walks the next range.  Only the last
    range's o_proj and all-reduce are exposed.  `reserve_sms` > 0 leaves that
    many SMs to the side stream while the core runs (gdn2_set_reserved_sms);
    with 2 and 4 B200s it made no measurable difference, so it is 0 by
    default.

    Every all-reduce is bracketed by CUDA events on the stream it runs on and
    nothing waits on them here, so a timed loop of layer calls never stalls
    the host; `pop_allreduce_ms()` (after the caller has synchronised) returns
    the all-reduce time of each call since the last pop (summed over its
    ranges), so it can be reported separately.
    """

    def __init__(self, cfg, weights: dict, group=None, device="cuda", dtype=None, overlap_segments: int = 4,
                 reserve_sms: int = 0, **kw):
        import torch
        import torch.distributed as dist

        from .module import GatedDeltaNet2

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.config = cfg
        self.overlap_segments = int(overlap_segments)
        self.reserve_sms = int(reserve_sms)
        self.local = GatedDeltaNet2(shard_config(cfg, self.world), shard_weights(weights, cfg, self.rank, self.world),
                                    device=device, dtype=dtype or torch.float32, **kw)
        self._events = []
        self._side = None

    def _reduce(self, y):
        import torch

        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        self.dist.all_reduce(y, op=self.dist.ReduceOp.SUM, group=self.group)
        e1.record()
        self._events.append([(e0, e1)])
        return y

    def _forward_train_overlapped(self, x):
        """Chunk-mode forward_train with the o_proj all-reduce overlapped
        with the recurrence (see the class docstring)."""
        import dataclasses as dc

        import torch

        from ._lib import LIB

        m = self.local
        C = m.config.chunk_size
        B, T, D = x.shape
        h, hk, hv, vh = m._dims
        nch = (T + C - 1) // C
        seg = -(-nch // self.overlap_segments) * C  # tokens per range, whole chunks
        p, _ = m.project(x, None)
        state = torch.zeros(B, hv, hk, vh, dtype=torch.float32, device=x.device)
        y = torch.empty(B, T, D, dtype=x.dtype, device=x.device)
        main = torch.cuda.current_stream(x.device)
        if self._side is None:
            self._side = torch.cuda.Stream(device=x.device)
        side = self._side
        side.wait_stream(main)  # y and the weights exist before the side stream writes or reads them
        evs = []
        prev = LIB.gdn2_set_reserved_sms(self.reserve_sms) if self.reserve_sms else None
        try:
            for t0 in range(0, T, seg):
                t1 = min(T, t0 + seg)
                ps = dc.replace(p, q=p.q[:, :, t0:t1], k=p.k[:, :, t0:t1], v=p.v[:, :, t0:t1], g=p.g[:, :, t0:t1],
                                b=p.b[:, :, t0:t1], w=p.w[:, :, t0:t1], gate=p.gate[:, t0:t1])
                normed = m._chunk_core(ps, state)
                done = torch.cuda.Event()
                done.record(main)
                with torch.cuda.stream(side):
                    side.wait_event(done)
                    normed.record_stream(side)
                    part = m._out_proj(normed)  # [B, t1 - t0, D], contiguous
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(side)
                    self.dist.all_reduce(part, op=self.dist.ReduceOp.SUM, group=self.group)
                    e1.record(side)
                    evs.append((e0, e1))
                    y[:, t0:t1].copy_(part)
        finally:
            if prev is not None:
                LIB.gdn2_set_reserved_sms(prev)
        main.wait_stream(side)
        self._events.append(evs)
        return y

    def _overlap_applies(self, x):
        from .config import Gdn2Mode

        return (self.overlap_segments > 1 and self.world > 1 and Gdn2Mode(self.local.config.mode) == Gdn2Mode.Chunk
                and x.is_cuda and x.shape[1] >= 2 * self.local.config.chunk_size)

    def pop_allreduce_ms(self):
        """All-reduce times (ms) of the calls since the last pop, oldest
        first.  Call after the work has completed (e.g. after
        torch.cuda.synchronize()); it does not wait itself."""
        out = [sum(e0.elapsed_time(e1) for e0, e1 in call) for call in self._events]
        self._events = []
        return out

    def forward_train(self, x):
        if self._overlap_applies(x):
            return self._forward_train_overlapped(x)
        return self._reduce(self.local.forward_train(x))

    def forward(self, x, state=None, update_state=True):
        y, state = self.local.forward(x, state, update_state)
        return self._reduce(y), state
