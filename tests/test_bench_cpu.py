"""The benchmark's command line on CPU: the reference arm (the reference's
layer step on torch's CPU operators, and config 1 on ``F.embedding_bag``)
prints one JSON line with the contract's keys and the step counts it ran,
and option combinations that make no sense are refused before any work."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*args, timeout=600):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, capture_output=True,
                          text=True, timeout=timeout)


@pytest.mark.parametrize("workload,unit", [("c2", "tokens/s"), ("c1", "GB/s")])
def test_reference_arm_prints_the_contract_line(workload, unit):
    r = _bench("--impl", "reference", "--workload", workload, "--steps", "2", "--warmup", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["value"] > 0 and d["unit"] == unit
    assert d["steps"] == 2 and d["warmup"] == 1 and d["dtype"] == "bf16"
    assert d["config"]["workload"].startswith(workload)
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] == os.cpu_count() and cb["value"] == d["value"]
    assert cb["steps"] == 2 and cb["warmup"] == 1


def test_owner_exchange_needs_the_optimizer_step():
    r = _bench("--grad-exchange", "owner", timeout=120)
    assert r.returncode == 2
    assert "--optimizer sgd" in r.stderr
