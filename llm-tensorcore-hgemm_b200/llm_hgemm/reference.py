"""Correctness gate of the HGEMM contract (reference llm_hgemm/reference.py:9-56).

Public API kept for drop-in users: ``torch_reference`` (FP32 matmul with TF32
disabled, then FP16 rounding), ``error_metrics`` and ``correctness_passed``
with the reference's limits (max-abs <= 5e-2, relative L2 <= 5e-3, no NaN/Inf).
Nothing in ``hgemm`` calls this module; it validates results, it does not
produce them.
"""

from __future__ import annotations

from contextlib import contextmanager

import torch

MAX_ABS_ERROR_LIMIT = 5e-2
RELATIVE_L2_ERROR_LIMIT = 5e-3


@contextmanager
def _tf32_disabled():
    previous = torch.backends.cuda.matmul.allow_tf32
    try:
        torch.backends.cuda.matmul.allow_tf32 = False
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = previous


@torch.no_grad()
def torch_reference(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """FP32 product of the FP16 inputs, rounded once to FP16."""
    with _tf32_disabled():
        return torch.mm(a.float(), b.float()).half()


@torch.no_grad()
def error_metrics(out: torch.Tensor, reference: torch.Tensor) -> dict[str, float | int]:
    out32 = out.float()
    ref32 = reference.float()
    diff = out32 - ref32
    absdiff = diff.abs()
    denom = ref32.abs().clamp_min(1e-6)
    ref_norm = torch.linalg.vector_norm(ref32).clamp_min(1e-12)
    return {
        "max_abs_error": float(absdiff.max().item()),
        "mean_abs_error": float(absdiff.mean().item()),
        "max_rel_error": float((absdiff / denom).max().item()),
        "relative_l2_error": float((torch.linalg.vector_norm(diff) / ref_norm).item()),
        "nan_count": int(torch.isnan(out32).sum().item()),
        "inf_count": int(torch.isinf(out32).sum().item()),
    }


def correctness_passed(metrics: dict[str, float | int]) -> bool:
    return (
        metrics["nan_count"] == 0
        and metrics["inf_count"] == 0
        and metrics["max_abs_error"] <= MAX_ABS_ERROR_LIMIT
        and metrics["relative_l2_error"] <= RELATIVE_L2_ERROR_LIMIT
    )
