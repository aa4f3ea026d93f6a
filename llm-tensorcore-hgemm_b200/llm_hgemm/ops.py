"""Public HGEMM entry points (reference llm_hgemm/ops.py:18-77).

``hgemm`` and ``_hgemm_out`` resolve ``shape_auto`` in Python, then call the
pybind11 module ``_C``, which checks the reference's contract and launches a
hand-written sm_100a kernel through the C ABI on the current CUDA stream.
There is no CPU or library fallback: without the built extension the import
fails.
"""

from __future__ import annotations

import torch

from .dispatch import last_selected, record_selected, selected_implementation

try:
    from . import _C
except ImportError as exc:  # the product path must not run without the kernels
    raise ImportError(
        "llm_hgemm._C is not built. Run `python build.py` in "
        "llm-tensorcore-hgemm_b200/ (or __graft_entry__.build()) first."
    ) from exc


def hgemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    implementation: str = "auto",
    epilogue: str = "none",
    bias: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
) -> torch.Tensor:
    """Row-major FP16 C = A @ B with FP32 accumulation (reference ops.py:18-30).

    ``epilogue`` (the reference accepts only ``"none"``) fuses terms into the
    GEMM's store, on the FP32 sum, with one FP16 rounding at the end:

    * ``"bias"``: ``+ bias[j]`` (FP16 ``[N]``);
    * ``"residual"``: ``+ residual[i, j]`` (FP16 ``[M, N]``, unit column
      stride; it may be the output of :func:`_hgemm_out` itself);
    * ``"bias+residual"``;
    * ``"silu_mul"`` / ``"bias+silu_mul"`` (SwiGLU): B's columns hold (gate,
      up) pairs ``2j, 2j + 1`` (see :func:`interleave_gate_up`) and the output
      is ``[M, N / 2]`` with ``C[:, j] = silu(g) * u``.
    """
    resolved = selected_implementation(a, b, implementation)
    output = _C.hgemm(a, b, resolved, epilogue, bias, residual)
    if implementation == "shape_auto":
        record_selected(resolved)
    return output


def _hgemm_out(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    *,
    implementation: str,
    epilogue: str = "none",
    bias: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
) -> torch.Tensor:
    """Benchmark seam writing into a preallocated ``out`` (reference ops.py:33-46)."""
    resolved = selected_implementation(a, b, implementation)
    _C.hgemm_out(a, b, out, resolved, epilogue, bias, residual)
    if implementation == "shape_auto":
        record_selected(resolved)
    return out


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``[K, 2I]`` operand for the ``silu_mul`` epilogue from the ``[K, I]``
    gate and up operands: column ``2j`` is ``gate[:, j]``, ``2j + 1`` is
    ``up[:, j]``."""
    if gate.shape != up.shape or gate.dim() != 2:
        raise ValueError("gate and up must be 2-D tensors of the same shape")
    return torch.stack((gate, up), dim=2).reshape(gate.shape[0], 2 * gate.shape[1]).contiguous()


def hgemm_f32_out(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, *,
                  implementation: str = "auto") -> torch.Tensor:
    """FP32-output GEMM (unrounded partial sums) for tensor-parallel K splits."""
    _C.hgemm_out_f32(a, b, out, implementation)
    return out


def available_providers() -> tuple[str, ...]:
    """Benchmark provider names (reference ops.py:49-69).

    ``torch`` is the plain ``torch.mm`` benchmark provider; every other name is
    an ``implementation=`` accepted by :func:`hgemm`. The cuBLASLt comparator
    is benchmark-only (``llm_hgemm.comparators``), not a provider.
    """
    return ("torch", "shape_auto", *_C.implementations())


def backend_info(implementation: str, shape: tuple[int, int, int] | None = None) -> dict[str, int]:
    """``{"algorithm_id", "workspace_bytes"}`` (reference ops.py:72-77).

    ``algorithm_id`` is -1 for every custom kernel, as in the reference. With
    ``shape=(M, N, K)`` the workspace is the one ``hgemm`` allocates for an
    aligned problem of that shape on the current device (stream-K partial
    tiles, split-K exchange slots; ``auto`` resolved first); without a shape,
    as in the reference's call form, it is 0."""
    if implementation == "torch":
        return {"algorithm_id": -1, "workspace_bytes": 0}
    if implementation == "shape_auto":
        implementation = last_selected()
    if shape is None:
        return dict(_C.backend_info(implementation))
    m, n, k = (int(v) for v in shape)
    return dict(_C.backend_info(implementation, m, n, k))


def resolved_config(a: torch.Tensor, b: torch.Tensor,
                    implementation: str = "auto") -> tuple[str, int]:
    """Kernel configuration and K-split count ``implementation`` launches for a, b."""
    name = selected_implementation(a, b, implementation)
    return tuple(_C.resolve(a, b, name))
