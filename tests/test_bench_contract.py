"""The benchmark's result line, checked on the CPU.

``bench.py --impl reference`` (the reference's CPU path on the host cores)
runs anywhere, so its JSON line is checked here key by key against the
contract both arms share.  The device arm needs a B200: without one it must
fail loudly and print no result line (no CPU fallback).
"""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args, timeout=240):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                          cwd=ROOT, capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    p = _run("--impl", "reference", "--steps", "1", "--warmup", "0")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, p.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert d["unit"] == "TOPS" and d["scaling"] == "weak"
    assert "workload" in d["config"] and d["config"]["M"] == 2048
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_device_arm_without_a_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        return  # the device arm itself is exercised on the GPU box
    p = _run("--steps", "1", "--warmup", "0", timeout=120)
    assert p.returncode != 0
    assert not any(ln.lstrip().startswith("{") for ln in p.stdout.splitlines())
