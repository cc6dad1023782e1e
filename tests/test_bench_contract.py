"""CPU: the parts of bench.py that run without a GPU — the clock-log parser
and the reference arm (`--impl reference`, the reference's CPU path timed on
a bounded sample), whose JSON line the round's driver reads."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import bench

ROOT = Path(__file__).resolve().parents[1]


def test_clock_summary_parses_nvidia_smi_lines():
    s = bench.ClockSampler(0)
    s.lines = [
        "0, 1965, 1965, 650.25, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1635, 1965, 998.10, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1650, 1965, 997.00, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, [N/A], 1965, 997.00, 0x0, Not Active, Not Active, Not Active, Not Active",  # unreadable sample
        "garbage",
    ]
    out = s.summary()
    assert out == {"sm_mhz": 1650.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    s.lines = ["0, 1200, 1965, 700.0, 0x0000000000000048, Not Active, Active, Not Active, Not Active"]
    assert s.summary()["reasons"] == ["hw_thermal_slowdown"]
    s.lines = []
    assert s.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def _run_bench(*args: str, env_extra: dict | None = None) -> subprocess.CompletedProcess:
    env = dict(os.environ, **(env_extra or {}))
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=600, cwd=ROOT, env=env)


def test_reference_arm_other_ranks_exit_quietly():
    out = _run_bench("--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0",
                     env_extra={"RANK": "1", "WORLD_SIZE": "2"})
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == ""


def test_reference_arm_json_line():
    out = _run_bench("--impl", "reference", "--steps", "1", "--warmup", "0")
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 1, 0)
    assert line["vs_baseline"] is None and line["data"] == "synthetic"
    assert line["config"]["workload"] == bench.WORKLOAD
    assert abs(line["ms_per_step"] - 1e3 * bench.S_TOTAL * bench.DEPTH / line["value"]) < 1e-6 * line["ms_per_step"]
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == line["value"] and cb["unit"] == line["unit"]
    assert cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
