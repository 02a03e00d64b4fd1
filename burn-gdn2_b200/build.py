#!/usr/bin/env python3
"""Build libgdn2_b200.so (all sm_100a kernels + the C ABI of include/gdn2.h).

    python burn-gdn2_b200/build.py [--force] [--verbose]

Each ``csrc/*.cu`` is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/``, then linked
into ``burn_gdn2/libgdn2_b200.so`` next to the Python host package, so the
library travels with the source tree.  Objects are rebuilt when the source,
a header, or the flags change.
"""
import argparse
import concurrent.futures as cf
import hashlib
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "burn_gdn2", "libgdn2_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def _digest(paths, extra):
    h = hashlib.sha256()
    for p in sorted(paths):
        with open(p, "rb") as f:
            h.update(f.read())
    h.update(" ".join(extra).encode())
    return h.hexdigest()[:16]


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(INCLUDE, "gdn2.h"))
    jobs = []
    for src in sources:
        path = os.path.join(CSRC, src)
        tag = _digest([path] + headers, ARCH + CFLAGS)
        obj = os.path.join(BUILD, f"{src[:-3]}.{tag}.o")
        jobs.append((path, obj))

    def compile_one(job):
        path, obj = job
        if os.path.exists(obj) and not force:
            return obj, None
        cmd = [NVCC, *ARCH, *CFLAGS, "-c", path, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {path}:\n{r.stdout}\n{r.stderr}")
        return obj, (r.stdout + r.stderr) if verbose else None

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(compile_one, jobs))
    for _, log in results:
        if log:
            print(log)
    objs = [o for o, _ in results]
    link_tag = _digest(objs, ["link"])
    stamp = LIB + ".stamp"
    if force or not os.path.exists(LIB) or not os.path.exists(stamp) or open(stamp).read() != link_tag:
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        with open(stamp, "w") as f:
            f.write(link_tag)
    # drop objects of older source revisions
    keep = set(objs)
    for f in os.listdir(BUILD):
        p = os.path.join(BUILD, f)
        if f.endswith(".o") and p not in keep:
            os.remove(p)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
