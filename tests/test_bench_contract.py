"""bench.py's reference arm (the CPU implementation of the path, timed on the
host) prints one JSON line with the keys the measurement contract needs, and
the bench refuses fewer than 3 warm-up steps.  CPU only."""
from __future__ import annotations

import json
import subprocess
import sys

from conftest import ROOT


def _run(*args, timeout=600):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    r = _run("--impl", "reference", "--steps", "3", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "dtype", "data", "config"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["steps"] == 3 and d["warmup"] == 3
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("reference", "port") and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_bench_refuses_short_warmup():
    r = _run("--impl", "reference", "--steps", "3", "--warmup", "1", timeout=120)
    assert r.returncode != 0
    assert "warmup" in r.stderr
