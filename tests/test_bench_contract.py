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


def test_reference_line_names_its_sample_and_the_gpu_arms_config():
    """The reference arm's step is one timed row sample: the line says so
    (extrapolated, sample rows and seconds, ms_per_step = the sample's time, so that
    steps x ms_per_step is the time the arm spent), and its config is the GPU arm's."""
    import argparse

    sys.path.insert(0, ROOT)
    import bench

    line = json.loads(_run_bench("--impl", "reference", "--steps", "2", "--warmup", "1").strip())
    assert line["extrapolated"] is True and line["sample_rows"] >= 1 and line["sample_s"] > 0
    assert abs(line["ms_per_step"] - 1e3 * line["sample_s"]) < 1.0
    assert line["full_step_ms_extrapolated"] > line["ms_per_step"]
    want = bench.workload_config(argparse.Namespace(workload="dense_projection", scaling="strong"), 1)
    assert line["config"] == want


@pytest.mark.parametrize("workload,world,rows,cols", [
    ("dense_projection", 8, 512, 12288), ("dense_projection", 4, 1024, 12288), ("tall_skinny", 8, 16384, 2048),
    ("wide", 8, 2048, 3584), ("square", 8, 2048, 16384), ("dense_projection", 1, 4096, 12288)])
def test_strong_scaling_slabs(workload, world, rows, cols):
    """Strong scaling cuts the workload's global GEMM: M-row slabs, or 32-column
    multiples of N for the wide shape; every rank's slab has the same size."""
    import argparse

    sys.path.insert(0, ROOT)
    import bench

    a = argparse.Namespace(workload=workload, scaling="strong")
    M, N, K, _, _ = bench.WORKLOADS[workload]
    for r in range(world):
        rr, cc, kk, mt, nt, shards, mode, _ = bench.layout(a, world, r)
        assert (rr, cc, kk, mt, nt) == (rows, cols, K, M, N)
        assert cc % 32 == 0
    cfg = bench.workload_config(a, world)
    assert cfg["M_per_gpu"] == rows and cfg["N_per_gpu"] == cols and cfg["M_total"] == M
    weak = bench.layout(argparse.Namespace(workload=workload, scaling="weak"), world, world - 1)
    assert weak[:5] == (M, N, K, M * world, N)
