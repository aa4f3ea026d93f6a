"""Exact-shape dispatch policy for ``implementation="shape_auto"``
(reference llm_hgemm/dispatch.py:14-128), re-targeted to SM100.

A policy file maps exact (M, N, K) shapes to one of this library's kernel
configurations. ``configure_dispatch`` validates it once, off the hot path:
schema, torch and CUDA versions, the source fingerprint and the target SM
(10.0) must match, and devices are eligible only when both their name and
compute capability (10, 0) match. Per call, ``selected_implementation``
returns the requested name unchanged unless it is ``shape_auto``; then:

* inputs that break the contract -> ``auto`` (the C++ layer raises the error);
* no policy, or an ineligible device -> ``auto`` (the SM100 shape heuristic;
  the reference fell back to cuBLASLt, which is not a dispatch target here);
* a base address not 16-byte aligned -> ``auto`` (a table entry was tuned on
  aligned operands; ``auto`` stages such operands for TMA);
* otherwise the table entry for (M, N, K), else ``auto``.

The last selection is recorded per thread (``record_selected``/``last_selected``).
"""

from __future__ import annotations

import json
import threading
from pathlib import Path

import torch

from .provenance import code_fingerprint, file_sha256

CUSTOM_PROVIDERS = (
    "tc_persistent_128x256",
    "tc_persistent_128x128",
    "tc_splitk_128x128",
    "tc_swapab",
    "tc_generic_128x128",
    "tc_pair_256x256",
    "tc_splitk_128x256",
    "tc_streamk_128x256",
    "tc_streamk_swapab",
    "tc_pair_256x128",
    "tc_pair_128x256",
    "tc_pair_128x128",
    "tc_streamk_pair_256x256",
)
MISALIGNED_PROVIDER = "auto"
DEFAULT_PROVIDER = "auto"
SCHEMA_VERSION = 3
TARGET_SM = "10.0"
TARGET_CAPABILITY = (10, 0)

STRATEGIES = ("best_available", "best_custom")
_ALLOWED = set(CUSTOM_PROVIDERS) | {DEFAULT_PROVIDER}

_policy: dict | None = None
_local = threading.local()


def configure_dispatch(path: str | Path | None, *, strategy: str = "best_available") -> None:
    """Load (or with ``None`` clear) the exact-shape policy; raises ValueError."""
    global _policy

    if strategy not in STRATEGIES:
        raise ValueError(f"unknown dispatch strategy: {strategy}")
    if path is None:
        _policy = None
        return

    payload = json.loads(Path(path).read_text())
    if payload.get("schema_version") != SCHEMA_VERSION:
        raise ValueError(f"dispatch table requires schema_version={SCHEMA_VERSION}")
    if payload.get("torch") != torch.__version__:
        raise ValueError("dispatch table PyTorch version mismatch")
    if payload.get("cuda") != torch.version.cuda:
        raise ValueError("dispatch table CUDA version mismatch")
    if payload.get("code_fingerprint") != code_fingerprint():
        raise ValueError("dispatch table source/extension fingerprint mismatch")
    if str(payload.get("sm")) != TARGET_SM:
        raise ValueError("dispatch table must target SM100 (sm 10.0)")

    entries: dict[tuple[int, int, int], str] = {}
    for item in payload["entries"]:
        key = (int(item["M"]), int(item["N"]), int(item["K"]))
        if min(key) <= 0 or key in entries:
            raise ValueError(f"invalid/duplicate shape: {key}")
        for name in STRATEGIES:
            if item[name] not in _ALLOWED:
                raise ValueError(f"invalid provider: {item[name]}")
        entries[key] = item[strategy]

    eligible = {
        index
        for index in range(torch.cuda.device_count())
        if torch.cuda.get_device_name(index) == payload["gpu"]
        and torch.cuda.get_device_capability(index) == TARGET_CAPABILITY
    }
    _policy = {
        "strategy": strategy,
        "table_sha256": file_sha256(path),
        "entries": entries,
        "eligible_devices": eligible,
    }


def policy() -> dict | None:
    """The active policy (read-only view), or None."""
    return _policy


def _valid_contract(a: torch.Tensor, b: torch.Tensor) -> bool:
    return (
        a.is_cuda
        and b.is_cuda
        and a.device == b.device
        and a.dtype == torch.float16
        and b.dtype == torch.float16
        and a.ndim == 2
        and b.ndim == 2
        and a.is_contiguous()
        and b.is_contiguous()
        and a.shape[1] == b.shape[0]
        and min(a.shape[0], a.shape[1], b.shape[1]) > 0
    )


def selected_implementation(a: torch.Tensor, b: torch.Tensor, requested: str = "shape_auto") -> str:
    if requested != "shape_auto":
        return requested
    if not _valid_contract(a, b):
        return DEFAULT_PROVIDER
    pol = _policy
    if pol is None or a.device.index not in pol["eligible_devices"]:
        return DEFAULT_PROVIDER
    if a.data_ptr() % 16 or b.data_ptr() % 16:
        return MISALIGNED_PROVIDER
    return pol["entries"].get((a.shape[0], b.shape[1], a.shape[1]), DEFAULT_PROVIDER)


def record_selected(provider: str) -> None:
    _local.provider = provider


def last_selected() -> str:
    provider = getattr(_local, "provider", None)
    if provider is None:
        raise RuntimeError("shape_auto has not executed in this thread")
    return provider
