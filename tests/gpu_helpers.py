"""Shared helpers of the GPU parity tests."""

from __future__ import annotations

import torch

from oracle import reference as oracle

IMPLEMENTATIONS = [
    "auto",
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
]


def require_cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert torch.cuda.get_device_capability() == (10, 0), "GPU tests need an sm_100 GPU"


def seeded_inputs(m, n, k, seed=2026, device="cuda"):
    torch.manual_seed(seed)
    a = torch.randn((m, k), device=device, dtype=torch.float16) * 0.1
    b = torch.randn((k, n), device=device, dtype=torch.float16) * 0.1
    return a, b


def assert_gate(out, a, b):
    metrics = oracle.check(out, a, b)
    assert metrics["passed"], metrics
    return metrics
