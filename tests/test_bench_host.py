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
    rows = [{"tag": "qwen3_4b.q_proj", "shape": "1x4096x2560", "ratio_to_cublaslt": 2.0,
             "shape_auto_ratio_to_cublaslt": 2.0, "roofline_frac": 0.5, "status": "pass"},
            {"tag": "qwen3_4b.q_proj", "shape": "512x4096x2560", "ratio_to_cublaslt": 0.5,
             "shape_auto_ratio_to_cublaslt": 1.0, "roofline_frac": 0.3, "status": "pass"},
            {"tag": "square", "shape": "1024x1024x1024", "ratio_to_cublaslt": 0.1, "tflops": 100.0,
             "roofline_frac": 0.1, "status": "fail"}]
    out = bench.sweep_summary(rows)
    assert out["qwen_shapes"] == 2
    assert out["qwen_geomean_ratio_auto"] == pytest.approx(1.0)
    assert out["qwen_shapes_at_or_above_1"] == 1
    assert out["qwen_geomean_ratio_shape_auto"] == pytest.approx(2 ** 0.5, rel=1e-3)
    assert out["qwen_shapes_at_or_above_1_shape_auto"] == 2
    assert out["ratio_by_layer"] == {"q_proj": [2.0, 0.5]}
    assert out["hbm_frac_m_le_128"] == {"q_proj": [0.5]}
    assert out["square_ratio"] == {"1024x1024x1024": 0.1}
    assert out["gate_failures"] == ["1024x1024x1024"]


def test_full_sweep_summary_fits_a_short_result_line(monkeypatch):
    # The driver reads the last stdout line: the summary of the full sweep
    # (every square, ragged and Qwen shape) must keep that line short.
    rows = []
    for m, n, k, tag in ([(s, s, s, "square") for s in bench.SQUARE]
                         + [(m, n, k, "ragged") for (m, n, k) in bench.RAGGED]
                         + [(m, n, k, f"qwen3_4b.{layer}") for layer, (k, n) in bench.QWEN_LAYERS.items()
                            for m in bench.QWEN_M]
                         + [(m, *bench.QWEN_LAYERS[layer][::-1], f"unseen.{layer}") for layer in bench.UNSEEN_LAYERS
                            for m in bench.UNSEEN_M]):
        rows.append({"tag": tag, "shape": f"{m}x{n}x{k}", "ratio_to_cublaslt": 0.987,
                     "shape_auto_ratio_to_cublaslt": 0.991, "roofline_frac": 0.812, "tflops": 1234.5,
                     "status": "pass"})
    out = bench.sweep_summary(rows)
    assert out["shapes"] == len(rows) and out["qwen_shapes"] == 48
    assert out["unseen_shapes"] == 24       # 12 unseen rows + the Qwen rows at M = 8, 16, 64
    assert len(json.dumps(out)) < 2500


def test_reference_arm_under_torchrun_times_the_tp_workload():
    # Under torchrun, N = 1 included, both arms run the tensor-parallel MLP.
    proc = run_bench("--impl", "reference", "--steps", "3", "--warmup", "3",
                     env_extra={"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0"})
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["config"]["workload"] == "tp_mlp"
    assert line["config"]["gemms"] == ["8192x28672x8192", "8192x8192x28672"]
    assert line["scaling"] == "strong" and line["value"] > 0
    assert "A rows 0.." in line["cpu_baseline"]["sample"]


def fake_sweep(monkeypatch, policy_loaded=True):
    """bench.sweep() with the GPU parts replaced: checks how the per-shape rows
    are assembled (timings, ratios, error metrics, shape_auto columns)."""
    import torch

    import llm_hgemm.dispatch
    import llm_hgemm.ops

    tiny = (torch.zeros(2, 2, dtype=torch.float16),) * 3
    calls = {"n": 0}       # timing calls since the shape's inputs were made

    def fake_sets(m, n, k, device):
        calls["n"] = 0
        return [tiny]

    def fake_timing(fn, sets):
        base = 10.0 + calls["n"]         # auto 10, cuBLASLt 11, shape_auto 12 us
        calls["n"] += 1
        return {"median_us": base, "p95_us": base + 1.0, "min_us": base - 1.0, "eager_median_us": base + 2.0}

    monkeypatch.setattr(bench, "make_sets", fake_sets)

    monkeypatch.setattr(bench, "median_launch_us", fake_timing)
    errors = {"max_abs_error": 1e-3, "mean_abs_error": 1e-4, "max_rel_error": 0.5,
              "relative_l2_error": 2e-4, "nan_count": 0, "inf_count": 0}
    monkeypatch.setattr(bench, "gpu_reference_metrics", lambda out, a, b: dict(errors, passed=True))
    monkeypatch.setattr(bench, "gpu_reference_check", lambda out, a, b: True)
    monkeypatch.setattr(bench, "load_policy", lambda: policy_loaded)
    monkeypatch.setattr(llm_hgemm.ops, "_hgemm_out", lambda *a, **k: None)
    monkeypatch.setattr(llm_hgemm.ops, "resolved_config", lambda a, b, impl: ("tc_persistent_128x256", 1))
    monkeypatch.setattr(llm_hgemm.dispatch, "last_selected", lambda: "auto")
    peaks = {"bf16_tflops": 1651.8, "hbm_gbs": 6493.7, "bf16_tflops_sustained": 1372.7}
    return bench.sweep(peaks, quick=True), peaks


def test_sweep_rows_without_gpu(monkeypatch):
    rows, _ = fake_sweep(monkeypatch)
    assert rows and all(r["status"] == "pass" for r in rows)
    r = next(r for r in rows if r["tag"].startswith("qwen3_4b"))
    # auto timed first, cuBLASLt second, shape_auto third for a Qwen shape.
    assert (r["median_us"], r["p95_us"], r["min_us"]) == (10.0, 11.0, 9.0)
    assert (r["cublaslt_us"], r["cublaslt_p95_us"], r["cublaslt_min_us"]) == (11.0, 12.0, 10.0)
    assert r["ratio_to_cublaslt"] == pytest.approx(1.1)
    assert r["shape_auto_us"] == 12.0 and r["shape_auto_status"] == "pass"
    assert r["errors"]["relative_l2_error"] == 2e-4 and "passed" not in r["errors"]
    squares = [r for r in rows if r["tag"] == "square"]
    assert [r["shape"] for r in squares] == ["1024x1024x1024", "2048x2048x2048", "4096x4096x4096"]
    assert all("shape_auto_us" not in r for r in squares)


def test_sweep_csv_and_manifest(monkeypatch, tmp_path):
    import csv

    rows, peaks = fake_sweep(monkeypatch)
    env = {"timestamp": "2026-01-01T00:00:00Z", "git_sha": "abc", "gpu": "NVIDIA B200", "sm": "10.0",
           "driver": "580.159", "cuda": "12.8", "torch": "2.11.0", "code_fingerprint": "f" * 64, "seed": 2026}
    path = tmp_path / "sweep.csv"
    bench.write_csv(rows, path, env, peaks)
    with path.open() as f:
        reader = csv.DictReader(f)
        assert reader.fieldnames == bench.CSV_FIELDS
        out = list(reader)
    tuned = sum(r["tag"].startswith(("qwen3_4b", "unseen")) for r in rows)
    assert len(out) == 2 * len(rows) + tuned         # auto + cuBLASLt, + shape_auto on Qwen / unseen shapes
    auto = [r for r in out if r["provider"] == "auto"]
    assert all(r["status"] == "pass" and r["relative_l2_error"] == "0.0002" for r in auto)
    assert {r["provider"] for r in out} == {"auto", "shape_auto", "cublaslt"}
    first = out[0]
    m, n, k = int(first["M"]), int(first["N"]), int(first["K"])
    assert float(first["tflops"]) == pytest.approx(2 * m * n * k / float(first["median_us"]) / 1e6, rel=1e-3)
    assert first["gpu"] == "NVIDIA B200" and first["layout"] == "row-major/row-major"
    manifest = json.loads((tmp_path / "sweep.csv.manifest.json").read_text())
    assert manifest["environment"]["code_fingerprint"] == "f" * 64
    assert manifest["benchmark"]["launches_per_sample"] == 10
    assert manifest["peaks"]["bf16_tflops"] == 1651.8


@pytest.mark.parametrize("case", ["auto:64x64", "auto:0x64x64", ":64x64x64"])
def test_profile_driver_rejects_malformed_cases(case):
    proc = subprocess.run([sys.executable, str(REPO / "llm-tensorcore-hgemm_b200" / "profile_one.py"),
                           "--case", "auto:64x64x64", "--case", case], capture_output=True, text=True, timeout=300)
    assert proc.returncode == 2, proc.stderr[-1000:]
    assert "expected IMPL:MxNxK" in proc.stderr


def test_profile_driver_rejects_f32_output_for_the_comparator():
    proc = subprocess.run([sys.executable, str(REPO / "llm-tensorcore-hgemm_b200" / "profile_one.py"),
                           "--m", "64", "--n", "64", "--k", "64", "--f32-out", "--provider", "cublaslt"],
                          capture_output=True, text=True, timeout=300)
    assert proc.returncode == 2, proc.stderr[-1000:]
    assert "--f32-out applies to this library's kernels only" in proc.stderr
