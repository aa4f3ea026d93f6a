"""Host-side parts of bench.py that need no GPU: the reference arm's JSON
line (the CPU path of the reference, timed on the host cores), its rank-0-only
rule under torchrun, the warm-up floor, the clock-sample summary and the
sweep summary."""

import json
import os
import subprocess
import sys

import pytest

from tests.conftest import REPO

import bench  # noqa: E402  (repo root is on sys.path via conftest)


def run_bench(*args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(REPO / "bench.py"), *args], capture_output=True, text=True,
                          env=env, timeout=300)


def test_reference_arm_json_line():
    proc = run_bench("--impl", "reference", "--steps", "3", "--warmup", "3", "--size", "512")
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "TFLOP/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    assert (line["steps"], line["warmup"], line["n_gpus"]) == (3, 3, 1)
    assert line["config"]["workload"] == "square_512"
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s",
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_prints_on_rank_zero_only():
    proc = run_bench("--impl", "reference", "--steps", "3", "--warmup", "3", "--size", "256",
                     env_extra={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert proc.stdout.strip() == ""


def test_warmup_floor():
    proc = run_bench("--impl", "reference", "--steps", "3", "--warmup", "2")
    assert proc.returncode == 2
    assert "--warmup must be >= 3" in proc.stderr


def test_clock_summary_uses_loaded_samples():
    s = bench.ClockSampler(0)
    idle = "0, 120, 1965, 198.5, 0x1, Not Active, Not Active, Not Active, Not Active"
    s.lines = [idle, idle] + [
        f"0, {mhz}, 1965, {w}, 0x4, Not Active, Not Active, Not Active, Active"
        for mhz, w in ((1100, 990.0), (1050, 1001.0), (1200, 985.0))]
    out = s.summary()
    assert out["samples"] == 5 and out["samples_under_load"] == 3
    assert out["sm_mhz"] == 1100 and out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"]


def test_clock_summary_without_samples():
    s = bench.ClockSampler(0)
    s.lines = ["garbage", "0, N/A, 1965"]
    assert s.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_sweep_summary_geomeans():
    rows = [{"tag": "qwen3_4b:q:1", "ratio_to_cublaslt": 2.0, "shape_auto_ratio_to_cublaslt": 2.0},
            {"tag": "qwen3_4b:q:8", "ratio_to_cublaslt": 0.5, "shape_auto_ratio_to_cublaslt": 1.0},
            {"tag": "square", "ratio_to_cublaslt": 0.1}]
    out = bench.sweep_summary(rows)
    assert out["qwen_shapes"] == 2
    assert out["qwen_geomean_ratio_auto"] == pytest.approx(1.0)
    assert out["qwen_shapes_at_or_above_1"] == 1
    assert out["qwen_geomean_ratio_shape_auto"] == pytest.approx(2 ** 0.5, rel=1e-3)
    assert out["qwen_shapes_at_or_above_1_shape_auto"] == 2
