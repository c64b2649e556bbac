"""bench.py contract checks that need no GPU: the reference arm's JSON line, the B200 arm
failing loudly without a device, and the clock-sample summary."""

from __future__ import annotations

import json
import subprocess
import sys

import pytest

from tests.conftest import REPO


def _run(*args, timeout=240):
    return subprocess.run([sys.executable, str(REPO / "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=str(REPO))


def test_reference_arm_prints_one_contract_line():
    r = _run("--impl", "reference", "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "plans/s" and d["value"] > 0
    assert d["config"]["workload"]
    assert set(d["cpu_baseline"]) >= {"value", "unit", "cores", "kind", "sample"}
    # The reference's own ICEMSolver.solve when its package is installed, else the labelled port.
    want_kind = "reference" if (REPO / "baseline" / "_ref" / "lewm" / "jepa.py").is_file() else "port"
    assert d["cpu_baseline"]["kind"] == want_kind
    # Same config keys as the B200 arm's line.
    sys.path.insert(0, str(REPO))
    import bench

    assert d["config"] == bench.bench_config(d["n_gpus"])
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]


def test_b200_arm_fails_loudly_without_a_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = _run("--steps", "1", "--warmup", "3", timeout=120)
    assert r.returncode != 0
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{") and '"value"' in ln]


def test_clock_summary_reports_median_and_every_reason():
    sys.path.insert(0, str(REPO))
    import bench

    cs = bench.ClockSampler(0)
    no = {n: False for n in cs.REASONS}
    cs.rows = [(1965.0, 1965.0, dict(no)), (1900.0, 1965.0, dict(no, sw_power_cap=True)),
               (1800.0, 1965.0, dict(no, hw_slowdown=True))]
    s = cs.summary()
    assert s["sm_mhz"] == 1900.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]
