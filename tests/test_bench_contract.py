"""The bench.py output contract, on the CPU.

`python bench.py --impl reference` (the reference arm: the oracle port timed on
the host cores) must print one JSON line with the metric, value, unit and the
cpu_baseline / e2e objects; `--warmup` below 3 is refused; every workload has a
metric, and the DRAM-traffic table in profiles/ parses for the workloads it
lists.
"""

from __future__ import annotations

import json
import subprocess
import sys

import pytest

from conftest import ROOT


def _run(*args: str, timeout: float = 240) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                          text=True, timeout=timeout, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    # the default workload, as the reference arm is run; a bounded oracle sample per step
    res = _run("--impl", "reference", "--steps", "1", "--warmup", "3", "--ref-step-seconds", "0.2")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better",
                "dtype", "data", "config", "cpu_baseline", "e2e", "vs_baseline"):
        assert key in d, key
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    assert "workload" in d["config"]
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["unit"] == d["unit"] and cpu["kind"] == "port"
    assert cpu["cores"] >= 1 and cpu["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_warmup_below_three_is_refused():
    res = _run("--impl", "reference", "--steps", "1", "--warmup", "2", timeout=120)
    assert res.returncode != 0
    assert "--warmup" in res.stderr


def test_every_workload_has_a_metric_and_traffic_parses():
    sys.path.insert(0, str(ROOT))
    import bench

    for name, w in bench.WORKLOADS.items():
        metric, unit, hib = bench.metric_of(w)
        assert metric and unit
        assert hib is (w.kind != "head_call")  # latency: lower is better
        assert bench.config_of(w, 1)["workload"]
    rows = [ln for ln in (ROOT / "profiles" / "traffic.md").read_text().splitlines()
            if ln.startswith("| ") and not ln.startswith("| workload") and "---" not in ln]
    assert rows
    for row in rows:
        name = row.strip("|").split("|")[0].strip()
        assert name in bench.WORKLOADS, name
        assert bench.load_traffic(bench.WORKLOADS[name]) > 0


def test_side_workloads_are_known_and_the_default_is_the_headline():
    sys.path.insert(0, str(ROOT))
    import bench

    assert all(name in bench.WORKLOADS for name in bench.SIDE_WORKLOADS)
    assert "long_prefill" not in bench.SIDE_WORKLOADS
    kinds = {bench.WORKLOADS[n].kind for n in bench.SIDE_WORKLOADS}
    assert kinds <= set(bench.RUNNERS)
