"""SM100 exact-shape policy tooling: measure, select, validate.

Counterpart of the reference's offline tuner and validator
(benchmarks/tune_dispatch.py:12-57, benchmarks/report_v7.py:14-97), re-targeted
to this library's configurations. The rules are the reference's:

* every (shape, provider) is measured in at least ``runs`` independent runs;
* a candidate whose run-to-run variation ((max - min) / median) exceeds
  ``max_variation`` (default 10 %) is not eligible;
* ``best_custom`` is the fastest eligible configuration;
* ``best_available`` is ``best_custom`` only when it beats the baseline by at
  least ``min_gain`` (default 5 %) in every run, else the baseline.

The baseline is this library's ``auto`` heuristic: cuBLASLt is a benchmark
comparator here, not a dispatch target. Validation re-measures ``shape_auto``
under the policy in a fresh run (never the tuning measurements) against the
cuBLASLt comparator and checks that every shape dispatched to its entry.

    python -m llm_hgemm.tune measure --shapes qwen3_4b --output tune_runs.json
    python -m llm_hgemm.tune select --inputs tune_runs.json --output configs/sm100_dispatch.json
    python -m llm_hgemm.tune validate --dispatch configs/sm100_dispatch.json --output summary.json
"""

from __future__ import annotations

import argparse
import json
import math
import statistics
from pathlib import Path

from .dispatch import CUSTOM_PROVIDERS, SCHEMA_VERSION, TARGET_SM
from .provenance import code_fingerprint, file_sha256

BASELINE = "auto"

# Qwen3-4B linears (K, N) and token counts: the reference's LLM shape set at
# the token counts the benchmark sweeps (decode 1 .. 128, prefill 512 .. 8192).
QWEN3_4B_LAYERS = {"q_proj": (2560, 4096), "k_proj": (2560, 1024), "o_proj": (4096, 2560),
                   "gate_proj": (2560, 9728), "down_proj": (9728, 2560), "lm_head": (2560, 151936)}
QWEN3_4B_M = (1, 8, 16, 64, 128, 512, 2048, 8192)


def variation(values: list[float]) -> float:
    """Run-to-run spread: (max - min) / median."""
    med = statistics.median(values)
    return (max(values) - min(values)) / med if med > 0 else math.inf


# Shapes the table was not tuned on: the reference's unseen-shape validation
# (M in {2, 8, 16, 64, 256} x the q, o, gate/up and down linears,
# results/raw/v7_unseen_20260929_053349/unseen_comparison.csv:2-21 of the
# reference) and the M = 4 rows of its Qwen3-4B trace (configs/qwen3_shapes.csv).
UNSEEN_LAYERS = {"q_proj": (2560, 4096), "o_proj": (4096, 2560), "gate_proj": (2560, 9728),
                 "down_proj": (9728, 2560)}
UNSEEN_M = (2, 4, 8, 16, 64, 256)


def shape_set(name: str) -> list[tuple[int, int, int]]:
    """Named shape sets, or a JSON file holding [[M, N, K], ...]."""
    if name == "qwen3_4b":
        return [(m, n, k) for (k, n) in QWEN3_4B_LAYERS.values() for m in QWEN3_4B_M]
    if name == "unseen":
        return [(m, n, k) for (k, n) in UNSEEN_LAYERS.values() for m in UNSEEN_M]
    if name == "square":
        return [(s, s, s) for s in (1024, 2048, 4096, 8192)]
    return [tuple(int(v) for v in item) for item in json.loads(Path(name).read_text())]


# ------------------------------------------------------------------ timing --

def _environment() -> dict:
    import torch

    from .dispatch import policy

    pol = policy()
    return {"gpu": torch.cuda.get_device_name(0), "sm": TARGET_SM,
            "capability": list(torch.cuda.get_device_capability(0)),
            "torch": torch.__version__, "torch_cuda": torch.version.cuda,
            "code_fingerprint": code_fingerprint(),
            "dispatch_sha256": pol["table_sha256"] if pol else None,
            "dispatch_strategy": pol["strategy"] if pol else None}


def _time_us(fn_for_set, sets, samples: int, per_sample: int = 10) -> float:
    """Median microseconds per launch: `per_sample` launches over the rotating
    input sets replayed as one CUDA graph, `samples` times (CUDA events)."""
    import torch

    stream = torch.cuda.current_stream()
    for i in range(20):
        fn_for_set(sets[i % len(sets)])
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
        for j in range(per_sample):
            fn_for_set(sets[j % len(sets)])
    stream.wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    out = []
    for _ in range(samples):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        graph.replay()
        e.record(stream)
        e.synchronize()
        out.append(s.elapsed_time(e) * 1000.0 / per_sample)
    del graph
    return statistics.median(out)


def _input_sets(m: int, n: int, k: int, seed: int):
    """Seeded input sets whose total size exceeds L2 (126 MB), so that launches
    read their operands from HBM as a model's layers do."""
    import torch

    per_set = 2 * (m * k + k * n + m * n)
    count = max(2, min(16, math.ceil(256e6 / per_set)))
    g = torch.Generator(device="cuda").manual_seed(seed)
    sets = []
    for _ in range(count):
        a = (torch.randn((m, k), generator=g, device="cuda", dtype=torch.float32) * 0.1).half()
        b = (torch.randn((k, n), generator=g, device="cuda", dtype=torch.float32) * 0.1).half()
        sets.append((a, b, torch.empty((m, n), device="cuda", dtype=torch.float16)))
    return sets


def measure(shapes, providers, runs: int = 3, samples: int = 20, seed: int = 2026) -> dict:
    """Times every provider on every shape in `runs` independent runs (the
    input sets are rebuilt and the order rotated between runs)."""
    import torch

    from . import _comparators
    from .ops import _hgemm_out

    results = {}
    for r in range(runs):
        for (m, n, k) in shapes:
            sets = _input_sets(m, n, k, seed + r)
            order = list(providers[r % len(providers):]) + list(providers[:r % len(providers)])
            for prov in order:
                if prov == "cublaslt":
                    fn = lambda s: _comparators.cublaslt_out(s[0], s[1], s[2])  # noqa: E731
                else:
                    fn = lambda s, p=prov: _hgemm_out(s[0], s[1], s[2], implementation=p)  # noqa: E731
                us = _time_us(fn, sets, samples)
                results.setdefault(f"{m}x{n}x{k}:{prov}", []).append(us)
            del sets
            torch.cuda.empty_cache()
    rows = []
    for key, us in results.items():
        shape, prov = key.split(":")
        m, n, k = (int(v) for v in shape.split("x"))
        rows.append({"M": m, "N": n, "K": k, "provider": prov, "us": us})
    return {"environment": _environment(), "runs": runs, "samples": samples, "results": rows}


# --------------------------------------------------------------- selection --

def select(measurements: list[dict], *, min_gain: float = 0.05, max_variation: float = 0.10,
           providers=CUSTOM_PROVIDERS) -> list[dict]:
    """Policy entries from measurement payloads (all must come from the same
    code and environment, measured on direct providers, not a policy)."""
    if not 0 <= min_gain < 1 or max_variation < 0:
        raise ValueError("invalid thresholds")
    envs = [m["environment"] for m in measurements]
    if any(e.get("dispatch_sha256") for e in envs):
        raise ValueError("tune using direct providers, not an existing policy")
    if len({(e["code_fingerprint"], e["gpu"], e["torch"], e["torch_cuda"]) for e in envs}) != 1:
        raise ValueError("measurements come from different code or environments")
    times: dict[tuple, list[float]] = {}
    for payload in measurements:
        for row in payload["results"]:
            times.setdefault((row["M"], row["N"], row["K"], row["provider"]), []).extend(row["us"])
    entries = []
    for shape in sorted({key[:3] for key in times}):
        base = times.get((*shape, BASELINE))
        if base is None:
            raise ValueError(f"missing baseline measurement: {shape}")
        candidates = []
        for prov in providers:
            values = times.get((*shape, prov))
            if values and len(values) >= 3 and variation(values) <= max_variation:
                candidates.append((statistics.median(values), prov, values))
        candidates.sort()
        best_custom = candidates[0][1] if candidates else BASELINE
        best_available = BASELINE
        if candidates and variation(base) <= max_variation:
            med, prov, values = candidates[0]
            # Run i of the candidate against run i of the baseline.
            if all(c <= b * (1.0 - min_gain) for c, b in zip(values, base)):
                best_available = prov
        entries.append({"M": shape[0], "N": shape[1], "K": shape[2],
                        "best_custom": best_custom, "best_available": best_available,
                        "custom_covered": bool(candidates),
                        "custom_median_us": candidates[0][0] if candidates else None,
                        "baseline_median_us": statistics.median(base),
                        "baseline_variation": variation(base)})
    return entries


def policy_payload(entries: list[dict], environment: dict, *, min_gain: float, max_variation: float,
                   sources: list[str]) -> dict:
    return {"schema_version": SCHEMA_VERSION, "gpu": environment["gpu"], "sm": TARGET_SM,
            "cuda": environment["torch_cuda"], "torch": environment["torch"],
            "code_fingerprint": environment["code_fingerprint"], "baseline": BASELINE,
            "min_gain": min_gain, "max_variation": max_variation, "entries": entries,
            "sources": sources}


# -------------------------------------------------------------- validation --

def validate(dispatch: Path, runs: int = 3, samples: int = 20, seed: int = 7,
             strategy: str = "best_available", extra_shapes=None) -> dict:
    """Re-measures ``shape_auto`` under the table (``best_available``: what
    ``configure_dispatch`` loads by default) against the cuBLASLt comparator
    on every policy shape, with input seeds the tuner does not use, and checks
    each dispatch hit its policy entry; with ``extra_shapes``, also the shapes
    the table holds no entry for (:func:`validate_unseen`). (The reference validates its custom
    kernels alone, ``best_custom``, because its baseline is cuBLASLt; here the
    baseline ``auto`` is this library's own kernels too.)"""
    from .dispatch import configure_dispatch, selected_implementation

    policy = json.loads(Path(dispatch).read_text())
    configure_dispatch(dispatch, strategy=strategy)
    shapes = [(e["M"], e["N"], e["K"]) for e in policy["entries"]]
    wanted = {(e["M"], e["N"], e["K"]): e[strategy] for e in policy["entries"]}
    payload = measure(shapes, ["shape_auto", "cublaslt"], runs=runs, samples=samples, seed=seed + 1000)
    times = {}
    for row in payload["results"]:
        times[(row["M"], row["N"], row["K"], row["provider"])] = row["us"]
    details, ratios, stable = [], [], True
    import torch

    for shape in shapes:
        m, n, k = shape
        a = torch.empty((m, k), device="cuda", dtype=torch.float16)
        b = torch.empty((k, n), device="cuda", dtype=torch.float16)
        chosen = selected_implementation(a, b, "shape_auto")
        if chosen != wanted[shape]:
            raise ValueError(f"shape_auto selected {chosen} for {shape}, policy says {wanted[shape]}")
        custom = times[(*shape, "shape_auto")]
        base = times[(*shape, "cublaslt")]
        ratio = statistics.median(base) / statistics.median(custom)
        ratios.append(ratio)
        shape_stable = max(variation(custom), variation(base)) <= policy["max_variation"]
        stable = stable and shape_stable
        details.append({"M": m, "N": n, "K": k, "implementation": chosen,
                        "custom_median_us": statistics.median(custom),
                        "cublaslt_median_us": statistics.median(base), "ratio_to_cublaslt": ratio,
                        "custom_variation": variation(custom), "baseline_variation": variation(base),
                        "stable": shape_stable})
    configure_dispatch(None)
    summary = {"dispatch_sha256": file_sha256(dispatch), "strategy": strategy,
               "environment": payload["environment"], "shape_count": len(shapes),
               "custom_geomean_percent_of_cublaslt": 100.0 * math.exp(statistics.mean(math.log(r) for r in ratios)),
               "validation_stability_passed": stable, "details": details}
    if extra_shapes:
        summary["unseen"] = validate_unseen(dispatch, extra_shapes, runs=runs, samples=samples, seed=seed,
                                            strategy=strategy)
    return summary


def validate_unseen(dispatch: Path, shapes, runs: int = 3, samples: int = 20, seed: int = 7,
                    strategy: str = "best_available") -> dict:
    """Shapes the table holds no entry for (the reference's unseen-shape
    check): ``shape_auto`` under the table, ``auto`` and the cuBLASLt
    comparator, timed as in :func:`validate`, and each result of
    ``shape_auto`` gated with the reference's limits against its FP32 product
    (``llm_hgemm.reference``, the reference's report gate) on seeded inputs."""
    import torch

    from . import reference
    from .dispatch import configure_dispatch, selected_implementation
    from .ops import hgemm

    configure_dispatch(dispatch, strategy=strategy)
    try:
        payload = measure(shapes, ["shape_auto", "auto", "cublaslt"], runs=runs, samples=samples, seed=seed + 2000)
        times = {(r["M"], r["N"], r["K"], r["provider"]): r["us"] for r in payload["results"]}
        details = []
        for (m, n, k) in shapes:
            g = torch.Generator(device="cuda").manual_seed(seed + m + n + k)
            a = (torch.randn((m, k), generator=g, device="cuda", dtype=torch.float32) * 0.1).half()
            b = (torch.randn((k, n), generator=g, device="cuda", dtype=torch.float32) * 0.1).half()
            chosen = selected_implementation(a, b, "shape_auto")
            metrics = reference.error_metrics(hgemm(a, b, implementation="shape_auto"),
                                              reference.torch_reference(a, b))
            lt = statistics.median(times[(m, n, k, "cublaslt")])
            details.append({"M": m, "N": n, "K": k, "implementation": chosen,
                            "shape_auto_median_us": statistics.median(times[(m, n, k, "shape_auto")]),
                            "auto_median_us": statistics.median(times[(m, n, k, "auto")]),
                            "cublaslt_median_us": lt,
                            "shape_auto_ratio_to_cublaslt": lt / statistics.median(times[(m, n, k, "shape_auto")]),
                            "auto_ratio_to_cublaslt": lt / statistics.median(times[(m, n, k, "auto")]),
                            "gate_passed": bool(reference.correctness_passed(metrics)),
                            "max_abs_error": metrics["max_abs_error"],
                            "relative_l2_error": metrics["relative_l2_error"]})
    finally:
        configure_dispatch(None)

    def geo(key):
        return 100.0 * math.exp(statistics.mean(math.log(d[key]) for d in details))

    return {"shape_count": len(details),
            "shape_auto_geomean_percent_of_cublaslt": geo("shape_auto_ratio_to_cublaslt"),
            "auto_geomean_percent_of_cublaslt": geo("auto_ratio_to_cublaslt"),
            "at_or_above_cublaslt": sum(d["shape_auto_ratio_to_cublaslt"] >= 1.0 for d in details),
            "all_gates_passed": all(d["gate_passed"] for d in details), "details": details}


# --------------------------------------------------------------------- CLI --

def main(argv=None) -> None:
    p = argparse.ArgumentParser(prog="python -m llm_hgemm.tune", description=__doc__.splitlines()[0])
    sub = p.add_subparsers(dest="cmd", required=True)
    pm = sub.add_parser("measure")
    pm.add_argument("--shapes", default="qwen3_4b")
    pm.add_argument("--providers", nargs="+", default=list(CUSTOM_PROVIDERS) + [BASELINE])
    pm.add_argument("--runs", type=int, default=3)
    pm.add_argument("--samples", type=int, default=20)
    pm.add_argument("--output", type=Path, required=True)
    ps = sub.add_parser("select")
    ps.add_argument("--inputs", nargs="+", type=Path, required=True)
    ps.add_argument("--output", type=Path, required=True)
    ps.add_argument("--min-gain", type=float, default=0.05)
    ps.add_argument("--max-variation", type=float, default=0.10)
    pv = sub.add_parser("validate")
    pv.add_argument("--dispatch", type=Path, required=True)
    pv.add_argument("--runs", type=int, default=3)
    pv.add_argument("--strategy", default="best_available", choices=("best_available", "best_custom"))
    pv.add_argument("--output", type=Path, required=True)
    pv.add_argument("--unseen", default=None,
                    help="also validate a shape set the table was not tuned on (e.g. 'unseen')")
    args = p.parse_args(argv)

    if args.cmd == "measure":
        if args.runs < 3:
            raise SystemExit("at least 3 runs per shape and provider")
        payload = measure(shape_set(args.shapes), args.providers, runs=args.runs, samples=args.samples)
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(json.dumps(payload, indent=1))
    elif args.cmd == "select":
        measurements = [json.loads(path.read_text()) for path in args.inputs]
        entries = select(measurements, min_gain=args.min_gain, max_variation=args.max_variation)
        payload = policy_payload(entries, measurements[0]["environment"], min_gain=args.min_gain,
                                 max_variation=args.max_variation, sources=[p.name for p in args.inputs])
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(json.dumps(payload, indent=2))
        print(json.dumps({"entries": len(entries),
                          "custom_over_baseline": sum(e["best_available"] != BASELINE for e in entries)}))
    else:
        extra = None
        if args.unseen:
            tuned = {(e["M"], e["N"], e["K"]) for e in json.loads(args.dispatch.read_text())["entries"]}
            extra = [s for s in shape_set(args.unseen) if s not in tuned]
        summary = validate(args.dispatch, runs=args.runs, strategy=args.strategy, extra_shapes=extra)
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(json.dumps(summary, indent=2))
        brief = {k: summary[k] for k in ("shape_count", "custom_geomean_percent_of_cublaslt",
                                         "validation_stability_passed")}
        if "unseen" in summary:
            brief["unseen"] = {k: v for k, v in summary["unseen"].items() if k != "details"}
        print(json.dumps(brief))


if __name__ == "__main__":
    main()
