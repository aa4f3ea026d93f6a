"""Generates the golden fixtures that pin oracle/reference.py.

Run in the build container, where the reference checkout is mounted:

    python tests/golden/make_golden.py <path of the reference checkout>

It loads the reference's own ``llm_hgemm/reference.py`` by file path (a plain
``import llm_hgemm`` would need the reference's compiled extension) and, for
the shapes its tests use, stores seeded CPU inputs and the reference
``torch_reference`` output (hgemm_golden.npz), plus the reference
``error_metrics`` of perturbed outputs (metrics_golden.json). The GPU box
never needs the reference: tests read only the committed fixtures.
"""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# Shapes of the reference tests: tests/test_correctness.py:24-33,
# tests/test_boundaries.py:23-32, tests/test_v6_async.py:24-38,
# tests/test_v5_vectorized.py:20-30.
SHAPES = [
    (16, 16, 16), (32, 64, 48), (37, 53, 29), (128, 256, 64), (129, 77, 1003),
    (1, 1, 1), (15, 17, 31), (17, 33, 65), (127, 129, 63), (129, 257, 33),
    (1, 8, 8), (127, 136, 40), (128, 128, 96), (64, 64, 32), (128, 129, 32),
]
SEED = 2026


def load_reference(ref_root: Path):
    spec = importlib.util.spec_from_file_location(
        "ref_llm_hgemm_reference", ref_root / "llm_hgemm" / "reference.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <path of the reference checkout>")
    ref_root = Path(sys.argv[1])
    ref = load_reference(ref_root)
    torch.set_num_threads(1)
    arrays = {}
    gen = torch.Generator().manual_seed(SEED)
    for (m, n, k) in SHAPES:
        a = (torch.randn((m, k), generator=gen, dtype=torch.float32) * 0.1).half()
        b = (torch.randn((k, n), generator=gen, dtype=torch.float32) * 0.1).half()
        c = ref.torch_reference(a, b)
        tag = f"{m}x{n}x{k}"
        arrays[f"a_{tag}"] = a.numpy()
        arrays[f"b_{tag}"] = b.numpy()
        arrays[f"c_{tag}"] = c.numpy()
    # Input patterns of tests/test_correctness.py:60-76 on a 33x29x47 problem.
    a = ((torch.rand((33, 47), generator=gen) - 0.5) * 0.2).half()
    b = ((torch.rand((47, 29), generator=gen) - 0.5) * 0.2).half()
    arrays["a_uniform"], arrays["b_uniform"] = a.numpy(), b.numpy()
    arrays["c_uniform"] = ref.torch_reference(a, b).numpy()
    a = (torch.randn((33, 47), generator=gen) * 0.1).half()
    b = (torch.randn((47, 29), generator=gen) * 0.1).half()
    a[a.abs() < 0.12] = 0
    b[b.abs() < 0.12] = 0
    arrays["a_sparse"], arrays["b_sparse"] = a.numpy(), b.numpy()
    arrays["c_sparse"] = ref.torch_reference(a, b).numpy()
    np.savez_compressed(HERE / "hgemm_golden.npz", **arrays)

    # error_metrics / correctness_passed on perturbed outputs (the test
    # rebuilds the same perturbations with perturbations()).
    cases = []
    base = torch.from_numpy(arrays["c_129x77x1003"])
    for name, out in perturbations(base).items():
        metrics = ref.error_metrics(out, base)
        cases.append({"name": name, "metrics": metrics,
                      "passed": bool(ref.correctness_passed(metrics))})
    (HERE / "metrics_golden.json").write_text(json.dumps(
        {"base": "c_129x77x1003", "seed": SEED, "cases": cases}, indent=1) + "\n")
    print(f"wrote {len(arrays)} arrays and {len(cases)} metric cases")


def perturbations(base: torch.Tensor) -> dict:
    return {
        "identical": base.clone(),
        "plus_1e-3": (base.float() + 1e-3).half(),
        "scaled_1.01": (base.float() * 1.01).half(),
        "one_nan": base.clone().index_put_((torch.tensor([3]), torch.tensor([5])),
                                           torch.tensor(float("nan"), dtype=torch.float16)),
        "one_inf": base.clone().index_put_((torch.tensor([0]), torch.tensor([0])),
                                           torch.tensor(float("inf"), dtype=torch.float16)),
        "zeros": torch.zeros_like(base),
    }


if __name__ == "__main__":
    main()
