"""The bench's arithmetic and its reference arm, on CPU.

* Algorithmic bytes and FLOPs per token per value head of the chunk core,
  against the figures of the hot-path scope table's measurement section:
  config 2 bf16 2304 B and 180 224 FLOP, config 2 f32 4096 B, config 4
  3328 B and 311 296 FLOP.
* `bench.py --impl reference` prints one JSON line with the keys the
  driver reads (the reference arm times the CPU restatement; no GPU).
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


@pytest.mark.parametrize("K, V, esize, C, nbytes, flops", [
    (128, 128, 2, 64, 2304, 180224),   # config 2, bf16
    (128, 128, 4, 64, 4096, 180224),   # config 2, f32
    (128, 256, 2, 64, 3328, 311296),   # config 4, bf16
    (64, 64, 4, 64, 2048, 65536),      # config 1, f32
])
def test_core_bytes_and_flops_per_token_head(K, V, esize, C, nbytes, flops):
    assert bench.core_bytes_per_token_head(K, V, esize) == nbytes
    assert bench.core_flops_per_token_head(K, V, C) == flops


def test_reference_arm_json_line():
    import time

    t0 = time.monotonic()
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                        "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    wall = time.monotonic() - t0
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.strip().splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "dtype", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["warmup"] >= 3
    # the line's own per-step time is measured, so its steps fit inside the run
    assert d["ms_per_step"] * (d["steps"] + d["warmup"]) / 1e3 < wall
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
