"""bench.py's reference arm on the CPU: the JSON line it prints carries the keys
the benchmark contract names, and ranks other than 0 print nothing and exit 0.

The reference arm times the reference's own host implementation (the oracle's
build of it when present, else the C restatement), so it needs no GPU."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run_bench(*args, env_extra=None):
    env = dict(os.environ, MPK_REF_STEP_BUDGET_S="0.1")
    env.update(env_extra or {})
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return out.stdout


def _check_reference_line(line, unit):
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in line, key
    assert line["unit"] == unit and line["value"] > 0
    assert line["warmup"] >= 3
    assert line["e2e"] == {"value": line["value"], "unit": unit, "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == line["value"]
    assert "workload" in line["config"]


@pytest.mark.parametrize("workload,unit", [("dense_projection", "TFLOPS"), ("codec", "GB/s")])
def test_reference_arm_prints_one_contract_line(workload, unit):
    lines = [ln for ln in _run_bench("--impl", "reference", "--workload", workload, "--steps", "1",
                                     "--warmup", "1").splitlines() if ln.strip()]
    assert len(lines) == 1
    _check_reference_line(json.loads(lines[0]), unit)


def test_reference_arm_other_ranks_print_nothing():
    out = _run_bench("--impl", "reference", "--steps", "1",
                     env_extra={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert out.strip() == ""
