#!/usr/bin/env python3
"""Benchmark of the GDN-2 token-mixer hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one pass of the chunked forward core (kernels (1) chunk-intra +
(2) chunk-inter with the fused SiLU-gated RMS-norm epilogue) over one batch
of BASELINE config 2: hidden 2048 = 16 value heads x K = V = 128, B = 8,
T = 4096, chunk 64, bf16 inputs / f32 state and accumulation.  Inputs are
seeded synthetic tensors with the module's value laws (L2-normalised q/k,
sigmoid gates, g = -A dt with A in [1,16], dt in [1e-3, 0.1]); they are
1.2 GB per step, larger than the 126 MB L2, so no flush is needed.

Printed (rank 0, one JSON line): tokens/s of the device-resident core
(`value`), the same through the C ABI from pinned host buffers (`e2e`),
the roofline of the dominant kernel, the decode step of BASELINE config 3
(B = 256, one token, state [256,16,128,128] f32) as `decode`, the config-2
layer (`layer`: projections + core + o_proj, against the tensor-core peak),
the config-2 core in f32 (`f32`), the core's backward over a config-2 batch
(`backward`) and one training step of the config-2 layer (`layer_train_step`), BASELINE configs 4 and 5 (`other_configs`:
their chunk cores, and config 5 as its head-sharded layer over the N ranks),
the CPU baseline (numpy restatement of the crate's tensor path on the host
cores) and SM clocks sampled during the timed region.

Multi-GPU (torchrun, one rank per GPU): (batch x value-head) chains are
independent, so each rank runs its own partition of config-2 chains
(weak scaling, no collective in the timed region); the value is the sum of
all ranks' tokens over the slowest rank's device time.
"""
import argparse
import ctypes
import json
import math
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "burn-gdn2_b200"))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]), "src": "measured"}
    except Exception:
        return dict(PEAKS_FALLBACK, src="fallback")


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
CFG2 = dict(B=8, HV=16, H=16, T=4096, K=128, V=128, chunk=64)
CFG3 = dict(B=256, HV=16, H=16, K=128, V=128)


def core_bytes_per_token_head(K, V, esize):
    """Algorithmic HBM bytes per token per value head of the chunk core:
    q, k, b, v, w, gate read and out written at the input dtype, g in f32
    (the state read/write once per (b, hv) is amortised and excluded)."""
    return 3 * K * esize + 4 * K + 4 * V * esize


def core_flops_per_token_head(K, V, C):
    return (6 * C * C * K + 4 * C * C * V + 6 * C * K * V) / C


def make_inputs(torch, B, HV, T, K, V, dtype, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)

    def nrm(*s):
        return torch.randn(*s, generator=g, device=device, dtype=torch.float32)

    def uni(lo, hi, *s):
        return torch.rand(*s, generator=g, device=device, dtype=torch.float32) * (hi - lo) + lo

    q = nrm(B, T, HV, K)
    q = q / q.norm(dim=-1, keepdim=True)
    k = nrm(B, T, HV, K)
    k = k / k.norm(dim=-1, keepdim=True)
    A = torch.exp(uni(0.0, math.log(16.0), B, T, HV, K))
    dt = torch.exp(uni(math.log(1e-3), math.log(0.1), B, T, HV, K))
    gl = (-A * dt).contiguous()
    b = torch.sigmoid(nrm(B, T, HV, K))
    v = nrm(B, T, HV, V)
    w = torch.sigmoid(nrm(B, T, HV, V))
    gate = nrm(B, T, HV, V)
    cast = lambda t: t.to(dtype).contiguous()
    return dict(q=cast(q), k=cast(k), v=cast(v), g=gl, b=cast(b), w=cast(w), gate=cast(gate))


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled through NVML
    every ~5 ms on a background thread during the timed region (the same
    counters `nvidia-smi --query-gpu=clocks.sm,clocks_event_reasons.*`
    reports; read-only)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, index):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._th = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self._mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return

        def loop():
            while not self._stop.is_set():
                try:
                    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((sm, rs))
                except Exception:
                    pass
                time.sleep(0.005)

        self._th = threading.Thread(target=loop, daemon=True)
        self._th.start()

    def stop(self):
        if self._th is None:
            return None
        self._stop.set()
        self._th.join()
        if not self.samples:
            return None
        sm = sorted(s for s, _ in self.samples)
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": self._mx, "reasons": reasons,
                "samples": len(self.samples), "source": "nvml"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def measure_core(torch, bg, ops, env, args, dtype, precision, with_e2e, clocks=False):
    """BASELINE config 2 chunk core (intra + inter + fused gated RMS norm) in `dtype` with `precision`
    intermediates: device-resident value, per-kernel split, and (with_e2e) the same step through the C ABI
    from pinned host buffers with the host <-> device copies inside the timed region."""
    dev, stream, rank, world = env["dev"], env["stream"], env["rank"], env["world"]
    barrier, max_over_ranks = env["barrier"], env["max_over_ranks"]
    c = CFG2
    B, HV, T, K, V = c["B"], c["HV"], c["T"], c["K"], c["V"]
    x = make_inputs(torch, B, HV, T, K, V, dtype, dev, seed=1000 + rank)
    view = lambda t: t.permute(0, 2, 1, 3)  # [B,T,HV,D] storage -> [B,HV,T,D] view
    state = torch.zeros(B, HV, K, V, dtype=torch.float32, device=dev)
    out = torch.empty(B, T, HV, V, dtype=dtype, device=dev)
    onw = torch.ones(V, dtype=torch.float32, device=dev)
    a = ops.chunk_args(view(x["q"]), view(x["k"]), view(x["v"]), view(x["g"]), view(x["b"]), view(x["w"]), state,
                       view(out), K ** -0.5, c["chunk"], num_heads=c["H"], gate=view(x["gate"]),
                       o_norm_weight=onw, norm_eps=1e-5, precision=precision)
    ws = ops.chunk_workspace(a, dev)
    sh = ctypes.c_void_p(stream.cuda_stream)
    wsp, wsn = ctypes.c_void_p(ws.data_ptr()), ws.numel()
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def step(e0=None, e1=None, e2=None):
        state.zero_()
        if e0 is not None:
            e0.record(stream)
        bg._lib.check(bg.LIB.gdn2_chunk_intra(ctypes.byref(a), wsp, wsn, sh))
        if e1 is not None:
            e1.record(stream)
        bg._lib.check(bg.LIB.gdn2_chunk_inter(ctypes.byref(a), wsp, wsn, sh))
        if e2 is not None:
            e2.record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(env["local"]) if (clocks and rank == 0) else None
    if sampler:
        sampler.start()
    evs = [(ev(), ev(), ev()) for _ in range(args.steps)]
    t_start, t_end = ev(), ev()
    t_start.record(stream)
    for e in evs:
        step(*e)
    t_end.record(stream)
    torch.cuda.synchronize()
    res = {"clocks": sampler.stop() if sampler else None}
    barrier()
    ms = max_over_ranks(t_start.elapsed_time(t_end) / args.steps)
    intra_ms = sum(e0.elapsed_time(e1) for e0, e1, _ in evs) / args.steps
    inter_ms = sum(e1.elapsed_time(e2) for _, e1, e2 in evs) / args.steps
    tokens = B * T
    esize = 2 if dtype == torch.bfloat16 else 4
    alg_bytes = core_bytes_per_token_head(K, V, esize) * tokens * HV
    flops = core_flops_per_token_head(K, V, c["chunk"]) * tokens * HV
    res.update(value=tokens * world / (ms / 1e3), ms=ms, intra_ms=intra_ms, inter_ms=inter_ms, alg_bytes=alg_bytes,
               flops=flops, tokens=tokens)
    if not with_e2e:
        return res

    # ---- e2e through the C ABI from pinned host buffers ----
    # Batch entries are independent chains, so the step is pipelined by batch
    # entry: entry i + 1 is copied in (copy stream) while entry i computes
    # (one gdn2_chunk_fwd call on its slice) and entry i - 1 is copied out.
    host = {n: t.cpu().pin_memory() for n, t in x.items()}
    dbuf = {n: torch.empty_like(t) for n, t in x.items()}
    hout = torch.empty(out.shape, dtype=dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = hout.numel() * hout.element_size()
    slice_args = [ops.chunk_args(view(dbuf["q"][i:i + 1]), view(dbuf["k"][i:i + 1]), view(dbuf["v"][i:i + 1]),
                                 view(dbuf["g"][i:i + 1]), view(dbuf["b"][i:i + 1]), view(dbuf["w"][i:i + 1]),
                                 state[i:i + 1], view(out[i:i + 1]), K ** -0.5, c["chunk"], num_heads=c["H"],
                                 gate=view(dbuf["gate"][i:i + 1]), o_norm_weight=onw, norm_eps=1e-5,
                                 precision=precision)
                  for i in range(B)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def e2e_step():
        start = torch.cuda.Event()
        start.record(stream)
        s_in.wait_event(start)
        s_out.wait_event(start)
        copied = []
        for i in range(B):
            with torch.cuda.stream(s_in):
                for n in host:
                    dbuf[n][i].copy_(host[n][i], non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_in)
                copied.append(e)
        for i in range(B):
            stream.wait_event(copied[i])
            state[i].zero_()
            bg._lib.check(bg.LIB.gdn2_chunk_fwd(ctypes.byref(slice_args[i]), wsp, wsn, sh))
            e = torch.cuda.Event()
            e.record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(e)
                hout[i].copy_(out[i], non_blocking=True)
        end = torch.cuda.Event()
        end.record(s_out)
        stream.wait_event(end)

    e2e_steps = max(2, min(args.steps, 5))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    s0, s1 = ev(), ev()
    s0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    s1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s0.elapsed_time(s1) / e2e_steps)
    res["e2e"] = {"value": tokens * world / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                  "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms}
    del host, dbuf
    return res


def core_line(res, peaks, dtype_name, precision):
    """Summary of one measure_core result: tokens/s, ms, the per-kernel split and the HBM roofline of the chunk
    core (algorithmic bytes over the two kernels' CUDA-event time)."""
    core_ms = res["intra_ms"] + res["inter_ms"]
    achieved = res["alg_bytes"] / (core_ms / 1e3) / 1e9
    out = {"value": res["value"], "unit": "tokens/s", "ms_per_step": res["ms"], "dtype": dtype_name,
           "precision": precision,
           "kernels_ms": {"chunk_intra": res["intra_ms"], "chunk_inter_plus_epilogue": res["inter_ms"]},
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": achieved / peaks["hbm_gbs"], "alg_bytes_per_step": res["alg_bytes"],
                        "tc_frac": res["flops"] / (core_ms / 1e3) / (peaks["bf16_tflops"] * 1e12)}}
    if "e2e" in res:
        out["e2e"] = res["e2e"]
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist
    import burn_gdn2 as bg
    from burn_gdn2 import comm, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # NCCL communicators created non-blocking, every collective bounded by the group timeout
        comm.init_process_group("nccl", timeout_s=120, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream(dev)
    env = dict(dev=dev, stream=stream, rank=rank, world=world, local=local, barrier=barrier,
               max_over_ranks=max_over_ranks)
    peaks = load_peaks()
    head_dt = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    head = measure_core(torch, bg, ops, env, args, head_dt, "f32", with_e2e=True, clocks=True)
    # the other input dtype with f32-grade intermediates, and the opt-in bf16-intermediate path
    other_dt = torch.float32 if head_dt == torch.bfloat16 else torch.bfloat16
    other = None if args.core_only else measure_core(torch, bg, ops, env, args, other_dt, "f32", with_e2e=True)
    fast = None if args.core_only else measure_core(torch, bg, ops, env, args, torch.bfloat16, "bf16",
                                                    with_e2e=False)

    # ---- decode step, BASELINE config 3 (one token, B = 256, state from a T = 512 prefill) ----
    decode = run_decode(torch, bg, ops, dev, stream, args, rank, max_over_ranks, world)
    # ---- whole layer forward_train (projections on cuBLAS + the core) ----
    layer = run_layer(torch, bg, dev, stream, args, max_over_ranks, world) if not args.core_only else None
    backward = run_backward(torch, bg, dev, max_over_ranks, rank) if not args.core_only else None
    layer_train = run_layer_train(torch, bg, dev, max_over_ranks) if not args.core_only else None
    layer_fast = (run_layer(torch, bg, dev, stream, args, max_over_ranks, world, precision="bf16")
                  if not args.core_only else None)
    # ---- N > 1: one config-2 layer split by heads, o_proj all-reduce timed apart ----
    layer_tp = run_layer_sharded(torch, bg, dev, stream, max_over_ranks, world) if world > 1 else None
    # ---- BASELINE configs 1, 4 and 5 ----
    others = None
    if not args.core_only:
        others = {"cfg1_layer": run_cfg1(torch, bg, dev, stream, max_over_ranks, world),
                  "cfg4_core": run_core_cfg(torch, bg, ops, dev, stream, CFG4, "config 4", max_over_ranks, world,
                                            seed=4000 + 10 * rank),
                  "cfg4_core_bf16_intermediates": run_core_cfg(torch, bg, ops, dev, stream, CFG4, "config 4",
                                                               max_over_ranks, world, seed=4000 + 10 * rank,
                                                               precision="bf16"),
                  "cfg5_core": run_core_cfg(torch, bg, ops, dev, stream, CFG5, "config 5", max_over_ranks, world,
                                            seed=5000 + 10 * rank),
                  # the config-2 core split by heads over the N ranks (strong scaling; no collective)
                  "cfg2_core_head_split": (run_core_cfg(torch, bg, ops, dev, stream,
                                                        dict(CFG2, H=16 // world, HV=16 // world, negeig=False,
                                                             min_decay=None), "config 2", max_over_ranks, world,
                                                        seed=2000 + 10 * rank, strong=True)
                                           if 16 % world == 0 else None),
                  # the config-5 layer split by heads over the N ranks (strong scaling, all-reduce timed apart)
                  "cfg5_layer_head_sharded": run_layer_cfg5(torch, bg, dev, stream, max_over_ranks, world)}

    c = CFG2
    B, HV, T, K, V = c["B"], c["HV"], c["T"], c["K"], c["V"]
    hl = core_line(head, peaks, args.dtype, "f32")
    dom_name = "chunk_inter" if head["inter_ms"] >= head["intra_ms"] else "chunk_intra"
    result = None
    if rank == 0:
        result = {
            "metric": "chunk-fwd tokens/s (H2048,T4096); decode tok/s @B256; % TC/HBM roofline",
            "value": head["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": args.dtype, "data": "synthetic (seeded, module value laws)",
            "config": {"workload": f"BASELINE config 2 chunked forward core: B={B} (per rank), T=4096, HV=16, "
                                   f"K=V=128, chunk 64, {args.dtype} inputs, f32-grade intermediates, f32 state, "
                                   "fused gated RMS-norm epilogue",
                       "global_batch": B * world, "seq_len": T, "parallelism": f"chains x{world} (no collective)",
                       "l2": f"inputs {head['alg_bytes'] / 1e9:.2f} GB/step > 126 MB L2, no flush"},
            "e2e": head["e2e"],
            "roofline": dict(hl["roofline"], kernel="chunk core (intra + inter + epilogue) per step",
                             # DRAM bytes per step from the ncu capture, scaled by the batch (linear in B)
                             traffic=(lambda t: None if t is None else t * B / 8)(
                                 ncu_traffic(f"chunk_core_x3_{args.dtype}_cfg2")),
                             peak_src=peaks["src"]),
            "kernels_ms": dict(hl["kernels_ms"], dominant=dom_name),
            "precision": "f32-grade intermediates (split bf16 operand pairs on tcgen05, f32 accumulation)",
            ("bf16" if other_dt == torch.bfloat16 else "f32"): core_line(other, peaks,
                                                                         "bf16" if other_dt == torch.bfloat16
                                                                         else "f32", "f32") if other else None,
            "bf16_intermediates": core_line(fast, peaks, "bf16", "bf16") if fast else None,
            "decode": decode,
            "layer": layer,
            "layer_bf16_intermediates": layer_fast,
            "layer_head_sharded": layer_tp,
            "backward": backward,
            "layer_train_step": layer_train,
            "other_configs": others,
            "gpu_launches": 2 * args.steps,
            "clocks": head["clocks"],
        }
    if world > 1:
        dist.destroy_process_group()
    return result


def ncu_traffic(key):
    """DRAM bytes per step measured by ncu (profiles/roofline_traffic.txt)."""
    try:
        for line in open(os.path.join(ROOT, "profiles", "roofline_traffic.txt")):
            k, _, v = line.partition("=")
            if k.strip() == key:
                return float(v.split()[0])
    except OSError:
        pass
    return None


def run_layer(torch, bg, dev, stream, args, max_over_ranks, world, precision="f32"):
    """GatedDeltaNet2.forward_train at BASELINE config 2 (hidden 2048,
    16 x 128 heads, chunk 64, bf16, B=8, T=4096): tokens/s and the fraction
    of the dense bf16 tensor-core peak the whole layer reaches, with the
    core's intermediates at `precision`."""
    c = CFG2
    cfg = bg.Gdn2Config(hidden_size=2048, num_heads=16, head_dim=128, mode=bg.Gdn2Mode.Chunk, chunk_size=64)
    m = bg.GatedDeltaNet2.new(cfg, device=dev, dtype=torch.bfloat16, seed=0, precision=precision)
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(c["B"], c["T"], 2048, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    for _ in range(2):
        m.forward_train(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 5
    e0.record(stream)
    for _ in range(n):
        m.forward_train(x)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / n)
    D, kd, vd, vh = 2048, 16 * 128, 16 * 128, 128
    tokens = c["B"] * c["T"]
    # q, k, b (D x KD); v, w (D x VD); f_proj_0, g_proj_0 (D x vh); f_proj_1 (vh x KD);
    # g_proj_1 (vh x VD); o_proj (VD x D)  -> 52.4 MFLOP per token
    proj_flops = 2 * tokens * (3 * D * kd + 2 * D * vd + 2 * D * vh + vh * kd + vh * vd + vd * D)
    core_flops = core_flops_per_token_head(128, 128, 64) * tokens * 16
    peaks = load_peaks()
    flops = proj_flops + core_flops
    return {"value": tokens * world / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "precision": precision,
            "workload": f"GatedDeltaNet2.forward_train, BASELINE config 2 (D=2048, 16x128 heads, B={c['B']}, T=4096, bf16)",
            "tflops": flops / (ms / 1e3) / 1e12, "tc_frac": flops / (ms / 1e3) / (peaks["bf16_tflops"] * 1e12),
            "flops_per_step": flops}


def run_layer_train(torch, bg, dev, max_over_ranks):
    """One training step of the config-2 layer (hidden 2048, 16 x 128 heads, bf16, B = 8, T = 4096):
    GatedDeltaNet2.forward_train_autograd, a mean-square loss, backward to every weight and the input
    (torch autograd; the recurrence on the chunked forward and gdn2_recurrent_bwd kernels)."""
    c = CFG2
    cfg = bg.Gdn2Config(hidden_size=2048, num_heads=16, head_dim=128, mode=bg.Gdn2Mode.Chunk, chunk_size=64)
    m = bg.GatedDeltaNet2.new(cfg, device=dev, dtype=torch.bfloat16, seed=0)
    m.requires_grad_(True)
    g = torch.Generator(device=dev).manual_seed(12)
    x = torch.randn(c["B"], c["T"], 2048, generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)

    def step():
        for t in m.parameters().values():
            t.grad = None
        x.grad = None
        m.forward_train_autograd(x).float().square().mean().backward()

    step()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 2
    e0.record(st)
    for _ in range(n):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / n)
    m.requires_grad_(False)
    return {"workload": f"GatedDeltaNet2 training step (forward_train_autograd + backward), BASELINE config 2 "
                        f"(D=2048, 16x128 heads, B={c['B']}, T=4096, bf16)",
            "ms_per_step": round(ms, 3), "tokens_per_s": c["B"] * c["T"] / (ms / 1e3)}


def run_layer_sharded(torch, bg, dev, stream, max_over_ranks, world):
    """BASELINE config 2 layer (16 heads) split by heads over the N ranks
    (strong scaling of one layer): forward_train time per step (max over
    ranks) and the NCCL all-reduce of the o_proj partials [B,T,2048] bf16,
    timed separately."""
    from burn_gdn2 import sharding
    c = CFG2
    cfg = bg.Gdn2Config(hidden_size=2048, num_heads=16, head_dim=128, mode=bg.Gdn2Mode.Chunk, chunk_size=64)
    full = bg.GatedDeltaNet2.new(cfg, device=dev, dtype=torch.bfloat16, seed=0)
    W = full.export_weights()
    del full
    m = sharding.ShardedGatedDeltaNet2(cfg, W, device=dev, dtype=torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(c["B"], c["T"], 2048, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    ms, ar_ms, local_ms = time_sharded(torch, m, x, stream, max_over_ranks, n=5)
    nbytes = c["B"] * c["T"] * 2048 * 2
    return {"value": c["B"] * c["T"] / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "scaling": "strong",
            "workload": f"GatedDeltaNet2.forward_train, BASELINE config 2, 16 heads split over {world} GPUs",
            "allreduce_ms": ar_ms, "allreduce_bytes": nbytes,
            "allreduce_busbw_gbs": 2 * (world - 1) / world * nbytes / (ar_ms / 1e3) / 1e9,
            **overlap_fields(ms, ar_ms, local_ms, m.overlap_segments),
            "parity_vs_unsharded": sharded_parity(torch, bg, sharding, dev, world)}


def time_sharded(torch, m, x, stream, max_over_ranks, n):
    """Sharded forward_train per step (max over ranks), its all-reduce time
    (summed over the overlapped ranges) and the same rank's local layer alone
    (no collective, one core call): the step minus the local layer is the
    all-reduce time left exposed."""
    ev = lambda: torch.cuda.Event(enable_timing=True)
    for _ in range(2):
        m.forward_train(x)
        m.local.forward_train(x)
    torch.cuda.synchronize()
    m.pop_allreduce_ms()
    e0, e1, e2 = ev(), ev(), ev()
    e0.record(stream)
    for _ in range(n):
        m.forward_train(x)
    e1.record(stream)
    for _ in range(n):
        m.local.forward_train(x)
    e2.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / n)
    local_ms = max_over_ranks(e1.elapsed_time(e2) / n)
    ar_ms = max_over_ranks(sum(m.pop_allreduce_ms()) / n)
    return ms, ar_ms, local_ms


def overlap_fields(ms, ar_ms, local_ms, segments):
    exposed = max(0.0, ms - local_ms)
    return {"local_layer_ms": local_ms, "exposed_allreduce_ms": exposed, "overlap_segments": segments,
            "allreduce_hidden_frac": max(0.0, 1.0 - exposed / ar_ms) if ar_ms > 0 else None}


def sharded_parity(torch, bg, sharding, dev, world):
    """ShardedGatedDeltaNet2 (NCCL all-reduce, overlapped forward_train) vs the unsharded layer on rank 0, both
    on the CUDA path: a bf16 layer of 8 x 128 heads, hidden 1024, B = 2, T = 320 (five chunks over the ranges),
    checked by the whole-layer criterion of the tests (relative Frobenius error <= 1e-2, max |d| <= 2.5e-2 of the
    reference's max magnitude: the ranks' o_proj partials are bf16 before their sum)."""
    import torch.distributed as dist
    cfg = bg.Gdn2Config(hidden_size=1024, num_heads=8, head_dim=128, mode=bg.Gdn2Mode.Chunk, chunk_size=64)
    full = bg.GatedDeltaNet2.new(cfg, device=dev, dtype=torch.bfloat16, seed=21)
    W = full.export_weights()
    m = sharding.ShardedGatedDeltaNet2(cfg, W, device=dev, dtype=torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(22)
    x = torch.randn(2, 320, 1024, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    y = m.forward_train(x).float()
    ref = full.forward_train(x).float()
    torch.cuda.synchronize()
    rel = float((y - ref).norm() / ref.norm())
    worst = float((y - ref).abs().max() / ref.abs().max())
    ok = torch.tensor([1.0 if rel <= 1e-2 and worst <= 2.5e-2 else 0.0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    return {"workload": "bf16 layer, hidden 1024, 8 x 128 heads, B=2, T=320, chunk mode", "ranks": world,
            "rel_fro": rel, "max_abs_err_over_max_ref": worst, "pass": bool(ok.item() == 1.0)}


def layer_flops(tokens, D, H, K, HV, V, C):
    """Dense FLOPs of one forward_train: the seven input projections (one concatenated GEMM: q, k, b with
    D x H.K, v, w with D x HV.V, f / gate down-projections D x V), the two up-projections (V x H.K,
    V x HV.V), o_proj (HV.V x D), and the chunk core."""
    kd, vd = H * K, HV * V
    proj = 2 * tokens * (3 * D * kd + 2 * D * vd + 2 * D * V + V * kd + V * vd + vd * D)
    return proj + core_flops_per_token_head(K, V, C) * tokens * HV


def run_layer_cfg5(torch, bg, dev, stream, max_over_ranks, world):
    """BASELINE config 5 (hidden 4096, 32 x 128 heads, B = 2, T = 65536, bf16) as the head-sharded layer of
    its definition: at N = 1 the whole layer, at N > 1 the layer split by heads over the N ranks (strong
    scaling of one layer) with the one NCCL all-reduce of the o_proj partials [B, T, 4096] timed apart."""
    B, T, D, H, K = 2, 65536, 4096, 32, 128
    cfg = bg.Gdn2Config(hidden_size=D, num_heads=H, head_dim=K, mode=bg.Gdn2Mode.Chunk, chunk_size=64)
    full = bg.GatedDeltaNet2.new(cfg, device=dev, dtype=torch.bfloat16, seed=7)
    if world > 1:
        from burn_gdn2 import sharding
        W = full.export_weights()
        del full
        m = sharding.ShardedGatedDeltaNet2(cfg, W, device=dev, dtype=torch.bfloat16)
        del W
    else:
        m = full
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(B, T, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    n = 3
    if world > 1:
        ms, ar_ms, local_ms = time_sharded(torch, m, x, stream, max_over_ranks, n)
    else:
        for _ in range(2):
            m.forward_train(x)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            m.forward_train(x)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / n)
    flops = layer_flops(B * T, D, H, K, H, K, 64)
    out = {"value": B * T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "scaling": "strong",
           "workload": f"GatedDeltaNet2.forward_train, BASELINE config 5 (D=4096, 32x128 heads, B=2, T=65536, bf16), "
                       f"heads split over {world} GPU(s)",
           "tc_frac_of_all_gpus": flops / (ms / 1e3) / (load_peaks()["bf16_tflops"] * 1e12 * world)}
    if world > 1:
        nbytes = B * T * D * 2
        out.update({"allreduce_ms": ar_ms, "allreduce_bytes": nbytes,
                    "allreduce_busbw_gbs": 2 * (world - 1) / world * nbytes / (ar_ms / 1e3) / 1e9,
                    **overlap_fields(ms, ar_ms, local_ms, m.overlap_segments)})
    del m, x
    return out


# BASELINE configs 4 (GVA: 8 key heads grouped over 16 value heads, V = 256, neg-eig b in [0, 2], min_decay 0.9)
# and 5 (long context, 32 heads), chunk core only (bf16), measured beside the headline so the path each one
# takes and its roofline fraction are on record.
CFG4 = dict(B=4, H=8, HV=16, T=8192, K=128, V=256, chunk=64, negeig=True, min_decay=0.9)
CFG5 = dict(B=2, H=32, HV=32, T=65536, K=128, V=128, chunk=64, negeig=False, min_decay=None)


def run_core_cfg(torch, bg, ops, dev, stream, c, name, max_over_ranks, world, seed, precision="f32", strong=False):
    """Chunk core (intra + inter + fused epilogue) at one BASELINE config:
    tokens/s, ms/step and the fraction of the measured HBM copy bandwidth
    its algorithmic bytes reach.  Key-side inputs (q, k, g, b) have H heads
    and are read grouped (value head hv uses key head hv // (HV / H)).
    strong: `c` is this rank's share of one job split by heads over the
    ranks (tokens/s counts the job's B x T tokens once)."""
    B, H, HV, T, K, V = c["B"], c["H"], c["HV"], c["T"], c["K"], c["V"]
    xk = make_inputs(torch, B, H, T, K, K, torch.bfloat16, dev, seed=seed)
    xv = make_inputs(torch, B, HV, T, V, V, torch.bfloat16, dev, seed=seed + 1)
    b = xk["b"]
    if c["negeig"]:
        b = (b.float() * 2.0).to(torch.bfloat16)
    g = xk["g"]
    if c["min_decay"] is not None:  # the module's remap with decay factors 2: log(sigmoid(2) (1 - m) e^g + m)
        g = torch.log((1.0 / (1.0 + math.exp(-2.0))) * (1.0 - c["min_decay"]) * torch.exp(g) + c["min_decay"])
    view = lambda t: t.permute(0, 2, 1, 3)
    state = torch.zeros(B, HV, K, V, dtype=torch.float32, device=dev)
    out = torch.empty(B, T, HV, V, dtype=torch.bfloat16, device=dev)
    onw = torch.ones(V, dtype=torch.float32, device=dev)
    a = ops.chunk_args(view(xk["q"]), view(xk["k"]), view(xv["v"]), view(g.contiguous()), view(b), view(xv["w"]),
                       state, view(out), K ** -0.5, c["chunk"], num_heads=H, grouped=H < HV, gate=view(xv["gate"]),
                       o_norm_weight=onw, norm_eps=1e-5, precision=precision)
    ws = ops.chunk_workspace(a, dev)
    sh = ctypes.c_void_p(stream.cuda_stream)
    run = lambda: bg._lib.check(bg.LIB.gdn2_chunk_fwd(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), ws.numel(), sh))
    run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 3
    e0.record(stream)
    for _ in range(n):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / n)
    del ws, xk, xv
    # algorithmic bytes per value head: the key-side reads count once per value head, as the kernels read them
    alg = core_bytes_per_token_head(K, V, 2) * B * T * HV
    peaks = load_peaks()
    if precision == "bf16":
        path = ("tensor cores, bf16 intermediates (k_intra_tc + k_inter_tc)" if V <= 128 else
                "tensor cores, bf16 intermediates (k_intra_tc; k_inter_tc over two 128-column slices per chain, a "
                "2-CTA cluster exchanging the gated RMS norm's row sums)")
    else:
        path = ("tensor cores, f32-grade intermediates (k_intra_x3 + k_inter_x3)" if V <= 128 else
                "tensor cores, f32-grade intermediates (k_intra_x3 with U in two 128-column halves; k_inter_x3 over "
                "two 128-column slices per chain, a 2-CTA cluster exchanging the gated RMS norm's row sums)")
    return {"value": B * T * (1 if strong else world) / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "precision": precision, "scaling": "strong" if strong else "weak",
            "workload": (f"BASELINE {name} chunk core, {H * world} key / {HV * world} value heads split over {world} "
                         f"GPU(s): B={B}, T={T}, H={H}, HV={HV} per rank, K={K}, V={V}, bf16" if strong else
                         f"BASELINE {name} chunk core: B={B} (per rank), T={T}, H={H}, HV={HV}, K={K}, V={V}, bf16"),
            "path": path,
            "roofline": {"bound": "hbm", "achieved": alg / (ms / 1e3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": alg / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]}}


def run_backward(torch, bg, dev, max_over_ranks, rank):
    """The core's backward (gdn2_recurrent_bwd) over one config-2 batch per rank: B = 8, HV = 16, T = 4096,
    K = V = 128, bf16 inputs and output gradient, an initial state, f32 gradients of q, k, v, g, b, w and the
    state.  Arithmetic: per token and head the kernel runs two forward steps (5 K V flops each: decay, erase
    product, rank-1 update) and one adjoint step (19 K V flops), 29 K V in all, on the f32 CUDA cores."""
    c = CFG2
    B, HV, T, K, V = c["B"], c["HV"], c["T"], c["K"], c["V"]
    gen = torch.Generator(device=dev).manual_seed(6000 + rank)
    rn = lambda *s: torch.randn(*s, generator=gen, device=dev)
    ru = lambda *s: torch.rand(*s, generator=gen, device=dev)
    bf = torch.bfloat16
    q = torch.nn.functional.normalize(rn(B, HV, T, K), dim=-1).to(bf)
    k = torch.nn.functional.normalize(rn(B, HV, T, K), dim=-1).to(bf)
    v, w, b = rn(B, HV, T, V).to(bf), ru(B, HV, T, V).to(bf), ru(B, HV, T, K).to(bf)
    g = -0.14 * ru(B, HV, T, K) - 0.01
    dout, h0 = rn(B, HV, T, V).to(bf), 0.1 * rn(B, HV, K, V)
    run = lambda: bg.recurrent_backward(q, k, v, g, b, w, h0, K ** -0.5, dout, None)
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 3
    e0.record(st)
    for _ in range(n):
        run()
    e1.record(st)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / n)
    flops = 29.0 * K * V * B * HV * T
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    peak = sms * 128 * 2 * 1.965e9 / 1e12  # f32 FMA lanes x 2 flops x max SM clock (nominal, not measured)
    return {"workload": f"core backward, config 2 per rank: B={B}, HV={HV}, T={T}, K=V={K}, bf16 inputs, "
                        "f32 gradients", "ms": round(ms, 3), "tokens_per_s": B * T / (ms / 1e3),
            "tflops_f32": round(flops / (ms / 1e3) / 1e12, 2), "f32_simt_peak_tflops_nominal": round(peak, 1),
            "frac_of_nominal_f32": round(flops / (ms / 1e3) / 1e12 / peak, 3)}


def run_decode(torch, bg, ops, dev, stream, args, rank, max_over_ranks, world):
    """GatedDeltaNet2 (hidden 2048, 16 x 128 heads, f32) prefills a seeded N(0,1) sequence of
    T = 512 for B = 256 (the chunked path), then the decode kernel (3) runs 128 one-token steps from that state and
    those conv caches, in place, with the fused short-conv + L2 prologue (raw projections of seeded N(0,1) tokens
    through the layer's own weights) and the gated RMS-norm epilogue.  Also the whole layer's decode step
    (projections + kernel + o_proj) through GatedDeltaNet2.forward."""
    c = CFG3
    B, HV, H, K, V = c["B"], c["HV"], c["H"], c["K"], c["V"]
    D = H * K
    cfg = bg.Gdn2Config(hidden_size=D, num_heads=H, head_dim=K, mode=bg.Gdn2Mode.Chunk, chunk_size=64)
    m = bg.GatedDeltaNet2.new(cfg, device=dev, dtype=torch.float32, seed=3)
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    xp = torch.randn(B, 512, D, generator=gen, device=dev, dtype=torch.float32)
    _, st = m.forward(xp, None, True)
    del xp
    torch.cuda.synchronize()
    kd, vd = H * K, HV * V
    xt = torch.randn(B, 1, D, generator=gen, device=dev, dtype=torch.float32)
    # the raw projections and gates of one seeded token through the layer's own weights (src/module.rs:400-476)
    qr, kr, vr = m.q_proj.forward(xt), m.k_proj.forward(xt), m.v_proj.forward(xt)
    f = m.f_proj_1.forward(m.f_proj_0.forward(xt))
    g = -torch.exp(m.a_log).repeat_interleave(K).view(1, 1, kd) * torch.nn.functional.softplus(f + m.dt_bias)
    b = torch.sigmoid(m.b_proj.forward(xt))
    w = torch.sigmoid(m.w_proj.forward(xt))
    gate = m.g_proj_1.forward(m.g_proj_0.forward(xt))
    S = st.recurrent
    cq, ck, cv = st.conv_q, st.conv_k, st.conv_v
    cw = [m.q_conv_w, m.k_conv_w, m.v_conv_w]
    out = torch.empty(B, 1, HV, V, device=dev)
    to4 = lambda t, n, d: t.reshape(B, 1, n, d).permute(0, 2, 1, 3)
    a = ops.recurrent_args(to4(qr, H, K), to4(kr, H, K), to4(vr, HV, V), to4(g.contiguous(), H, K), to4(b, H, K),
                           to4(w, HV, V), S, out.permute(0, 2, 1, 3), K ** -0.5, num_heads=H, grouped=True,
                           prologue=1, conv_w=cw, conv_in=(cq, ck, cv), conv_out=(cq, ck, cv),
                           gate=to4(gate.contiguous(), HV, V), o_norm_weight=m.o_norm_weight, norm_eps=1e-5)
    sh = ctypes.c_void_p(stream.cuda_stream)
    run = lambda: bg._lib.check(bg.LIB.gdn2_recurrent_fwd(ctypes.byref(a), sh))
    for _ in range(max(3, args.warmup)):
        run()
    torch.cuda.synchronize()
    steps = 128  # 128 decode steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    # the whole layer's decode step from the same state: projections (cuBLAS) + kernel (3) + o_proj
    for _ in range(3):
        m.forward(xt, st, True)
    torch.cuda.synchronize()
    n = 16
    e0.record(stream)
    for _ in range(n):
        m.forward(xt, st, True)
    e1.record(stream)
    torch.cuda.synchronize()
    layer_ms = max_over_ranks(e0.elapsed_time(e1) / n)
    # the same layer step replayed from a CUDA graph (the state advances in place on every replay)
    xin = xt.clone()
    gc = bg.GraphedCall(lambda t: m.forward(t, st, True)[0], xin, warmup=1)
    for _ in range(3):
        gc.replay()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(n):
        gc.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    layer_graphed_ms = max_over_ranks(e0.elapsed_time(e1) / n)
    del gc
    state_bytes = 2 * B * HV * K * V * 4
    vec_bytes = B * 1 * (3 * kd + 4 * vd) * 4 + B * HV * V * 4 + 2 * B * 3 * (2 * kd + vd) * 4
    peaks = load_peaks()
    gbs = (state_bytes + vec_bytes) / (ms / 1e3) / 1e9
    return {"value": B * world / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "workload": "BASELINE config 3 decode step: B=256 (per rank), HV=16, K=V=128, state f32 in place, "
                        "initialised by a seeded T=512 prefill through GatedDeltaNet2.forward, fused short-conv + "
                        "L2 prologue and gated RMS-norm epilogue",
            "layer_decode_ms_per_step": layer_ms, "layer_decode_tokens_per_s": B * world / (layer_ms / 1e3),
            "layer_decode_graphed_ms_per_step": layer_graphed_ms,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "bytes_per_step": state_bytes + vec_bytes,
                         "traffic": ncu_traffic("decode_cfg3")}}


def run_cfg1(torch, bg, dev, stream, max_over_ranks, world):
    """BASELINE config 1 on the GPU: hidden 256, 4 x 64 heads, Chunk mode, f32, x [1, 1024, 256] ~ N(0,1) seed 0,
    weights seeded 0: forward_train, and a T = 1024 prefill followed by one decode token with Gdn2State."""
    cfg = bg.Gdn2Config(hidden_size=256, num_heads=4, head_dim=64, mode=bg.Gdn2Mode.Chunk, chunk_size=64)
    m = bg.GatedDeltaNet2.new(cfg, device=dev, dtype=torch.float32, seed=0)
    gen = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(1, 1025, 256, generator=gen, device=dev, dtype=torch.float32)

    def prefill_decode():
        _, st = m.forward(x[:, :1024], None, True)
        return m.forward(x[:, 1024:], st, True)

    out = {}
    for name, fn in (("forward_train", lambda: m.forward_train(x[:, :1024])), ("prefill_1024_then_decode_1",
                                                                             prefill_decode)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 10
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        out[name + "_ms"] = max_over_ranks(e0.elapsed_time(e1) / n)
    # the same forward_train replayed from a CUDA graph (GraphedCall: one graph launch instead of ~20 kernels)
    xin = x[:, :1024].contiguous()
    gc = bg.GraphedCall(m.forward_train, xin)
    for _ in range(3):
        gc.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 20
    e0.record(stream)
    for _ in range(n):
        gc.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    out["forward_train_graphed_ms"] = max_over_ranks(e0.elapsed_time(e1) / n)
    del gc
    out["workload"] = ("BASELINE config 1: GatedDeltaNet2 hidden 256, 4 x 64 heads, Chunk, f32, B=1, T=1024 "
                       "(eager, and replayed from a CUDA graph)")
    out["forward_train_tokens_per_s"] = 1024 * world / (out["forward_train_ms"] / 1e3)
    out["forward_train_graphed_tokens_per_s"] = 1024 * world / (out["forward_train_graphed_ms"] / 1e3)
    return out


# ---------------------------------------------------------------------------
# CPU baseline: numpy restatement of the crate's tensor path (oracle)
# ---------------------------------------------------------------------------
def _blas_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(n[0]) if n else os.cpu_count()
    except Exception:
        return os.cpu_count()


def cpu_sample_step(O, np, arr, s0):
    """One step of the CPU port: chunk_wy_forward + rms_norm_gate_per_head over one sequence (B = 1 of
    config 2's B = 8, full T = 4096, 16 value heads, K = V = 128, f32).  Returns seconds."""
    c = CFG2
    t0 = time.perf_counter()
    o, _ = O.chunk_wy_forward(arr["q"], arr["k"], arr["v"], arr["g"], arr["b"], arr["w"], s0, c["K"] ** -0.5,
                              c["chunk"])
    O.rms_norm_gate_per_head(o.transpose(0, 2, 1, 3), arr["gate"], np.ones(c["V"], np.float32), 1e-5)
    return time.perf_counter() - t0


def _cpu_sample_inputs():
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import gdn2_oracle as O

    c = CFG2
    arr = O.make_core_inputs(1, c["HV"], c["T"], c["K"], c["V"], seed=3, dtype=np.float32)
    return O, np, arr, np.zeros((1, c["HV"], c["K"], c["V"]), np.float32)


CPU_SAMPLE = ("numpy (OpenBLAS) restatement of the crate's f32 tensor path (chunk_wy_forward + rms_norm_gate, the "
              "same op sequence as its NdArray backend): one sequence of BASELINE config 2 per step (B=1 of 8, "
              "T=4096, HV=16, K=V=128, chunk 64); tokens/s scales linearly in B")


def cpu_baseline(budget_s=10.0):
    O, np, arr, s0 = _cpu_sample_inputs()
    times = []
    while sum(times) < budget_s or len(times) < 2:
        times.append(cpu_sample_step(O, np, arr, s0))
    el = sum(times)
    out = {"value": len(times) * CFG2["T"] / el, "unit": "tokens/s", "cores": _blas_threads(), "kind": "port",
           "sample": f"{CPU_SAMPLE}; {len(times)} steps in {el:.1f} s"}
    out["cfg1"] = cpu_baseline_cfg1()
    return out


def cpu_baseline_cfg1():
    """BASELINE config 1 in full on the CPU port: forward_train of x [1, 1024, 256] and a T = 1024 prefill
    followed by one decode token (Gdn2State), f32, weights seeded 0."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import gdn2_oracle as O

    cfg = O.Gdn2Config(hidden_size=256, num_heads=4, head_dim=64, mode="chunk", chunk_size=64)
    layer = O.Gdn2Layer(cfg, O.init_weights(cfg, seed=0), np.float32)
    x = np.random.default_rng(0).standard_normal((1, 1025, 256)).astype(np.float32)
    t0 = time.perf_counter()
    layer.forward_train(x[:, :1024])
    t1 = time.perf_counter()
    _, st = layer.forward(x[:, :1024], None, True)
    layer.forward(x[:, 1024:], st, True)
    t2 = time.perf_counter()
    return {"forward_train_ms": (t1 - t0) * 1e3, "prefill_1024_then_decode_1_ms": (t2 - t1) * 1e3,
            "forward_train_tokens_per_s": 1024 / (t1 - t0), "cores": _blas_threads(), "kind": "port",
            "workload": "BASELINE config 1 in full (hidden 256, 4 x 64 heads, Chunk, f32, B=1, T=1024)"}


def run_reference(args):
    """The reference arm: the crate's f32 tensor path, restated in numpy (the crate itself is Rust and cannot be
    built here), timed on the host cores.  One step = one sequence of config 2 (B = 1 of 8, full T = 4096);
    ms_per_step is that step's own measured time."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    O, np, arr, s0 = _cpu_sample_inputs()
    for _ in range(args.warmup):
        cpu_sample_step(O, np, arr, s0)
    times = [cpu_sample_step(O, np, arr, s0) for _ in range(args.steps)]
    ms = sum(times) / len(times) * 1e3
    value = CFG2["T"] / (ms / 1e3)
    return {"impl": "reference", "metric": "chunk-fwd tokens/s (H2048,T4096); decode tok/s @B256; % TC/HBM roofline",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, module value laws)",
            "config": {"workload": "BASELINE config 2 chunked forward core, one sequence per step (B=1 of 8, "
                                   "T=4096, HV=16, K=V=128, chunk 64, f32)",
                       "global_batch": 1, "seq_len": CFG2["T"], "parallelism": "host cores (OpenBLAS threads)"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": _blas_threads(), "kind": "port",
                             "sample": f"{CPU_SAMPLE}; {args.steps} steps of {ms:.0f} ms"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--dtype", default="f32", choices=["bf16", "f32"],
                    help="input dtype of the headline line (f32: the reference's own arithmetic)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--core-only", action="store_true", help="skip the side measurements (other dtype, layer, configs)")
    ap.add_argument("--batch", type=int, default=None,
                    help="batch of config 2 (default 8, the BASELINE value); smaller for profiling captures")
    args = ap.parse_args()
    if args.batch:
        CFG2["B"] = args.batch
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        res = run_reference(args)
    else:
        res = run_ours(args)
        if res is not None and int(os.environ.get("WORLD_SIZE", "1")) == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline()
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
