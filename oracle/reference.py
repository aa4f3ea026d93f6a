"""Oracle for C[M,N] = A[M,K] @ B[K,N] (FP16 in, FP32 accumulate, FP16 out).

TEST INFRASTRUCTURE ONLY. This restates the reference's correctness oracle and
gate; it is the checker the tests, ``__graft_entry__.smoke()`` and the CPU
baseline of ``bench.py`` use, never part of the product path.

Reference algorithm (Qlunee/LLM-TensorCore-HGEMM):
  * ``torch_reference`` - llm_hgemm/reference.py:23-27: upcast both FP16
    operands to FP32, FP32 matrix product with TF32 disabled
    (reference.py:13-20), one round-to-nearest conversion to FP16.
  * ``error_metrics`` - reference.py:30-47: max / mean absolute error, max
    relative error with the denominator clamped at 1e-6, relative L2 error
    with the reference norm clamped at 1e-12, NaN and Inf counts of the output.
  * ``correctness_passed`` - reference.py:50-56 with the limits of
    reference.py:9-10: no NaN/Inf, max-abs <= 5e-2, relative L2 <= 5e-3.

Pinned: tests/golden/ holds inputs and outputs produced by the reference's own
``torch_reference`` / ``error_metrics`` (generated in the build container by
tests/golden/make_golden.py, which imports the reference file by path);
tests/test_oracle.py checks this module against them bit for bit.
"""

from __future__ import annotations

import torch

MAX_ABS_ERROR_LIMIT = 5e-2
RELATIVE_L2_ERROR_LIMIT = 5e-3


@torch.no_grad()
def torch_reference(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """FP32 matmul (TF32 off) of the FP16 operands, rounded once to FP16.

    Works for CPU tensors (the oracle proper) and for CUDA tensors (used only
    at sizes where a CPU FP32 GEMM would take minutes)."""
    saved = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        a32 = a.to(torch.float32)
        b32 = b.to(torch.float32)
        return torch.mm(a32, b32).to(torch.float16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = saved


@torch.no_grad()
def torch_reference_epilogue(a: torch.Tensor, b: torch.Tensor, epilogue: str = "none",
                             bias: torch.Tensor | None = None,
                             residual: torch.Tensor | None = None) -> torch.Tensor:
    """Oracle of the fused epilogues (an extension: the reference accepts only
    ``epilogue="none"``, csrc/dispatch.cpp:52). Every term is applied to the
    FP32 product of ``torch_reference`` and the result rounded once:

    * ``bias``: ``+ bias[j]``; ``residual``: ``+ residual[i, j]`` (FP16 operands
      widened to FP32), in that order;
    * ``silu_mul``: the product's columns are (gate, up) pairs 2j, 2j + 1 and
      output column j is ``silu(gate) * up`` (the SwiGLU of a Qwen3 MLP,
      ``down(silu(gate(x)) * up(x))``, without the intermediate roundings of
      the unfused layers).
    """
    terms = set() if epilogue == "none" else set(epilogue.split("+"))
    saved = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        acc = torch.mm(a.to(torch.float32), b.to(torch.float32))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = saved
    if "bias" in terms:
        acc = acc + bias.to(torch.float32)
    if "residual" in terms:
        acc = acc + residual.to(torch.float32)
    if "silu_mul" in terms:
        acc = torch.nn.functional.silu(acc[:, 0::2]) * acc[:, 1::2]
    return acc.to(torch.float16)


@torch.no_grad()
def error_metrics(out: torch.Tensor, reference: torch.Tensor) -> dict:
    o = out.to(torch.float32)
    r = reference.to(torch.float32)
    d = o - r
    ad = d.abs()
    return {
        "max_abs_error": float(ad.max().item()),
        "mean_abs_error": float(ad.mean().item()),
        "max_rel_error": float((ad / r.abs().clamp_min(1e-6)).max().item()),
        "relative_l2_error": float(
            (torch.linalg.vector_norm(d) / torch.linalg.vector_norm(r).clamp_min(1e-12)).item()),
        "nan_count": int(torch.isnan(o).sum().item()),
        "inf_count": int(torch.isinf(o).sum().item()),
    }


def correctness_passed(metrics: dict) -> bool:
    return (metrics["nan_count"] == 0 and metrics["inf_count"] == 0
            and metrics["max_abs_error"] <= MAX_ABS_ERROR_LIMIT
            and metrics["relative_l2_error"] <= RELATIVE_L2_ERROR_LIMIT)


def check(out: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> dict:
    """Gate ``out`` against the oracle computed on the CPU from the same inputs."""
    ref = torch_reference(a.detach().cpu(), b.detach().cpu())
    m = error_metrics(out.detach().cpu(), ref)
    m["passed"] = correctness_passed(m)
    return m


def stage_marker_inputs(m: int, n: int, k: int, block_k: int, device="cpu"):
    """Known-answer inputs after reference tests/test_v6_async.py:88-99.

    A is 0.125 everywhere; K-block t of B is filled with marker 2^(t mod 5)/16,
    so a missing, repeated or stale stage changes the exactly representable
    answer. Returns (a, b, expected value of every C element)."""
    a = torch.full((m, k), 0.125, dtype=torch.float16, device=device)
    b = torch.empty((k, n), dtype=torch.float16, device=device)
    total = 0.0
    for t in range((k + block_k - 1) // block_k):
        marker = float(2 ** (t % 5)) / 16.0
        rows = min(block_k, k - t * block_k)
        b[t * block_k: t * block_k + rows].fill_(marker)
        total += rows * 0.125 * marker
    return a, b, total
