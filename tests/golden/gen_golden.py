#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle to the reference.

The reference crate (sehaxe/burn-gdn2 v0.5.1) ships its own Python
transcription of the layer, ``tests/gen_reference.py`` (class
``Gdn2Reference``: projections, replicate-padded short conv, L2 norm,
per-token gated-delta scan, SiLU-gated RMS norm, o_proj).  Its tests compare
the crate against that transcription at 5e-4 (tests/bit_exact.rs:11).

This script imports that file from a checkout of the reference (it is not
vendored here), runs it exactly as its own ``main()`` does — seed 1337, one
layer, cases ``T = 2**(i % 6) + (i % 7)`` drawn in order — and stores the
weights (burn ``[in, out]`` layout, like its ``ref_data.bin`` writer) and the
first N (x, y) pairs as ``.npz``.  Two extra fixture sets patch the module
constants before building the layer (allow_neg_eigval on; a K=64 head
config with longer sequences that reach the crate's chunk path).

Usage: python tests/golden/gen_golden.py <reference checkout>   (or GDN2_REFERENCE_ROOT=<checkout>)
Runs on CPU in a few seconds.  The GPU box never runs it.
"""
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(ref_root):
    path = os.path.join(ref_root, "tests", "gen_reference.py")
    spec = importlib.util.spec_from_file_location("gen_reference", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def dump(mod, name, n_cases, seq_fn, patch):
    for k, v in patch.items():
        setattr(mod, k, v)
    # derived constants of the reference module (gen_reference.py:32-34)
    mod.KD = mod.H * mod.HK
    mod.V_HEAD = int(mod.HK * mod.EXPAND_V)
    mod.VD = mod.HV * mod.V_HEAD
    torch.manual_seed(1337)
    layer = mod.Gdn2Reference()
    layer.eval()
    out = {
        "D": mod.D, "H": mod.H, "HK": mod.HK, "HV": mod.HV, "EXPAND_V": mod.EXPAND_V,
        "USE_SHORT_CONV": int(mod.USE_SHORT_CONV), "ALLOW_NEG_EIGVAL": int(mod.ALLOW_NEG_EIGVAL),
        "EPS": mod.EPS, "n_cases": n_cases,
    }
    t = lambda x: x.detach().cpu().contiguous().numpy().astype(np.float32)
    out["q_proj"] = t(layer.q_proj.weight.t())
    out["k_proj"] = t(layer.k_proj.weight.t())
    out["v_proj"] = t(layer.v_proj.weight.t())
    out["f_proj_0"] = t(layer.f_proj[0].weight.t())
    out["f_proj_1"] = t(layer.f_proj[1].weight.t())
    out["b_proj"] = t(layer.b_proj.weight.t())
    out["w_proj"] = t(layer.w_proj.weight.t())
    out["g_proj_0"] = t(layer.g_proj[0].weight.t())
    out["g_proj_1_w"] = t(layer.g_proj[1].weight.t())
    out["g_proj_1_b"] = t(layer.g_proj[1].bias)
    out["A_log"] = t(layer.A_log)
    out["dt_bias"] = t(layer.dt_bias)
    out["o_norm_w"] = t(layer.o_norm_w)
    out["o_proj"] = t(layer.o_proj.weight.t())
    out["q_conv_w"] = t(layer.q_conv_w.reshape(mod.KD, 4))
    out["k_conv_w"] = t(layer.k_conv_w.reshape(mod.KD, 4))
    out["v_conv_w"] = t(layer.v_conv_w.reshape(mod.VD, 4))
    with torch.no_grad():
        for i in range(n_cases):
            T = seq_fn(i)
            x = torch.randn(1, T, mod.D)
            y = layer.forward(x)
            out[f"x_{i:03d}"] = t(x)
            out[f"y_{i:03d}"] = t(y)
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {n_cases} cases")


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GDN2_REFERENCE_ROOT")
    if not ref_root:
        sys.exit("usage: gen_golden.py <reference checkout> (or set GDN2_REFERENCE_ROOT)")
    base = dict(D=64, H=4, HK=16, HV=4, EXPAND_V=1.5, USE_SHORT_CONV=True, ALLOW_NEG_EIGVAL=False)
    # 1) the reference's own fixture stream (first 42 of its 1000 cases:
    #    every combination of i % 6 and i % 7, T in 2..70)
    mod = load_reference(ref_root)
    dump(mod, "ref_d64.npz", 42, lambda i: 2 ** (i % 6) + (i % 7), base)
    # 2) negative eigenvalues (b *= 2, gen_reference.py:121-122)
    mod = load_reference(ref_root)
    dump(mod, "ref_d64_negeig.npz", 12, lambda i: 2 ** (i % 6) + (i % 7), dict(base, ALLOW_NEG_EIGVAL=True))
    # 3) K = V = 64 heads (BASELINE config-1 head shape) and sequences of
    #    65..200 tokens, which the crate routes through chunk_wy_forward
    mod = load_reference(ref_root)
    dump(mod, "ref_d256_k64.npz", 4, lambda i: (65, 128, 130, 200)[i],
         dict(D=256, H=4, HK=64, HV=4, EXPAND_V=1.0, USE_SHORT_CONV=True, ALLOW_NEG_EIGVAL=False))


if __name__ == "__main__":
    main()
