"""The benchmark's reference arm (`bench.py --impl reference`) on the host.

The arm times the oracle port of the reference search (search.rs:1175-1391) on
host threads; it needs no GPU, so its JSON line is checked here against the
benchmark contract: the same metric and unit as the engine arm, `impl`,
a `cpu_baseline` describing the run, an `e2e` object with no copies, and
recall@10 of its own index.  Configuration 0 keeps it to seconds.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=e,
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    return [json.loads(l) for l in res.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_line_at_configuration_0():
    (line,) = _run(["--impl", "reference", "--config", "0", "--steps", "2", "--warmup", "1"])
    assert line["impl"] == "reference"
    assert line["metric"].startswith("IVF-PQ queries/sec at recall@10")
    assert line["unit"] == "queries/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 2 and line["warmup"] == 1
    assert line["config"]["workload"] == "c0_ivfpq_n1e5_d96"
    assert 0.0 < line["recall_at_10"] <= 1.0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "queries/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_of_a_device_generated_configuration_is_unavailable():
    (line,) = _run(["--impl", "reference", "--config", "4", "--steps", "1", "--warmup", "1"])
    assert line["impl"] == "reference" and "unavailable" in line


def test_reference_arm_runs_on_rank_0_only():
    assert _run(["--impl", "reference", "--config", "0", "--steps", "1", "--warmup", "1"], {"RANK": "1"}) == []
