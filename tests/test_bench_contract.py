"""bench.py's command-line contract, on the CPU: the reference arm (the reference's own CPU
matmul) prints one JSON line with the metric, unit, cpu_baseline and e2e keys the driver reads;
it names the workloads it does not time; and the B200 arm refuses to run without a B200
instead of falling back to anything."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(*args, timeout=300):
    return subprocess.run([sys.executable, "bench.py", *args], cwd=REPO, timeout=timeout,
                          stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)


def json_line(out: str) -> dict:
    lines = [l for l in out.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    r = run("--impl", "reference", "--steps", "2", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    d = json_line(r.stdout)
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["steps"] == 2
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("reference", "port")
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


@pytest.mark.parametrize("workload", ["tp_decode", "sweep", "prefill", "attention", "sgemm"])
def test_reference_arm_names_what_it_does_not_time(workload):
    r = run("--impl", "reference", "--workload", workload, "--steps", "2", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    d = json_line(r.stdout)
    assert d["impl"] == "reference" and d["unavailable"]


def test_warmup_below_three_is_refused():
    r = run("--steps", "2", "--warmup", "2")
    assert r.returncode != 0 and "--warmup must be >= 3" in r.stderr


def _gpu_visible() -> bool:
    r = subprocess.run([sys.executable, "-c",
                        "import torch, sys; sys.exit(0 if torch.cuda.is_available() else 1)"],
                       capture_output=True)
    return r.returncode == 0


@pytest.mark.skipif(_gpu_visible(), reason="a GPU is present")
def test_b200_arm_refuses_without_a_b200():
    r = run("--steps", "2", "--warmup", "3")
    assert r.returncode != 0
    assert "needs an sm_100 (B200) GPU" in r.stderr


def test_algorithmic_bytes_match_the_workload_definitions():
    # The roofline numerators: one 4096 x 4096 int8 GEMV at m = 1 (weights + scales + A + C)
    # and the 7B chain's 225 products (32 layers of wq, wk, wv, wo, w1, w3, w2 and the
    # classifier), whose int8 weights alone are 6,607,077,376 bytes.
    sys.path.insert(0, REPO)
    import bench
    assert bench.algorithmic_bytes(4096, 4096) == 16_826_368
    shapes = bench.chain_shapes()
    assert len(shapes) == 225
    assert sum(k * n for _, k, n, _ in shapes) == 6_607_077_376
    assert [name for name, _, _, row in shapes if row][:2] == ["wo0", "w20"]
    assert sum(1 for *_, row in shapes if row) == 64
