"""bench.py's reference arm prints one JSON line with the contract's keys (CPU)."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--layers", "2"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the same workload description as the B200 arm's line
    sys.path.insert(0, str(ROOT))
    import bench

    assert d["config"] == bench.bench_config(1, 2)
    # the steps it reports are the whole decode steps it timed
    assert d["steps"] == d["cpu_baseline"]["steps"] == 1


def test_redistribute_cpu_baseline_and_single_gpu_line():
    """The redistribute microbench's CPU leg (the oracle on one edge) and its N=1 answer."""
    sys.path.insert(0, str(ROOT))
    import bench

    cb = bench.redistribute_cpu_baseline(2, tokens=16, budget_s=0.5)
    assert cb["kind"] == "port" and cb["unit"] == "GB/s" and cb["value"] > 0 and cb["cores"] >= 1
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--redistribute"], capture_output=True, text=True,
                         timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][0])
    assert d["metric"] == bench.REDIST_METRIC and "unavailable" in d
