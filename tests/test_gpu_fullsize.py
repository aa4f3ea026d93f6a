"""Parity at the benchmark's full sizes (square 8192 and
16384, ragged 8193, the Qwen3-4B lm_head at 8192 tokens, the tensor-parallel
up-projection on one GPU).

Two size-independent checks:
* exact known answer: the stage-marker inputs of the reference's
  tests/test_v6_async.py:88-99 scaled to the full K give an exactly
  representable result, so every element must match bit for bit;
* the oracle's gate (max-abs <= 5e-2, relative L2 <= 5e-3) against the FP32
  product computed on the GPU with TF32 off (what the reference's own
  benchmark does at these sizes, benchmarks/bench_square.py:193), on seeded
  random inputs."""

import pytest
import torch

from llm_hgemm import hgemm
from llm_hgemm.ops import _hgemm_out
from oracle import reference as oracle
from tests.gpu_helpers import require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    require_cuda()
    yield
    torch.cuda.empty_cache()


@pytest.mark.parametrize("impl", ["auto", "tc_persistent_128x256", "tc_pair_256x256", "tc_streamk_128x256"])
@pytest.mark.parametrize("size", [8192, 16384])
def test_fullsize_stage_markers_exact(impl, size):
    if size == 16384 and impl != "auto":
        pytest.skip("16384^3 runs once, through auto")
    a, b, value = oracle.stage_marker_inputs(size, size, size, 64, device="cuda")
    out = hgemm(a, b, implementation=impl)
    assert bool((out == value).all()), f"{impl} {size}^3: not every element equals {value}"


def gate_gpu(out, a, b):
    ref = oracle.torch_reference(a, b)        # FP32 on the GPU, TF32 off
    metrics = oracle.error_metrics(out, ref)
    assert oracle.correctness_passed(metrics), metrics


@pytest.mark.parametrize("shape,impl", [
    ((8192, 8192, 8192), "auto"),
    ((8193, 8193, 8192), "auto"),                 # ragged: operands staged
    ((8192, 151936, 2560), "auto"),               # Qwen3-4B lm_head, prefill
    ((16, 151936, 2560), "auto"),                 # lm_head, decode
    ((8192, 28672, 8192), "auto"),                # tensor-parallel up-projection, one GPU
    ((2048, 9728, 2560), "tc_pair_256x256"),      # the exact-shape table's entry
])
def test_fullsize_gate_against_gpu_fp32(shape, impl):
    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(2026)
    a = (torch.randn((m, k), generator=g, device="cuda") * 0.1).half()
    b = (torch.randn((k, n), generator=g, device="cuda") * 0.1).half()
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    _hgemm_out(a, b, out, implementation=impl)
    gate_gpu(out, a, b)


def test_fullsize_linearity():
    """hgemm(A1 + A2, B) equals hgemm(A1, B) + hgemm(A2, B) up to the FP16
    roundings of the three results (a property independent of any oracle)."""
    m = n = k = 8192
    g = torch.Generator(device="cuda").manual_seed(7)
    a1 = (torch.randn((m, k), generator=g, device="cuda") * 0.05).half()
    a2 = (torch.randn((m, k), generator=g, device="cuda") * 0.05).half()
    b = (torch.randn((k, n), generator=g, device="cuda") * 0.1).half()
    lhs = hgemm(a1 + a2, b).float()
    rhs = hgemm(a1, b).float() + hgemm(a2, b).float()
    d = lhs - rhs
    rel = (torch.linalg.vector_norm(d) / torch.linalg.vector_norm(rhs)).item()
    assert rel <= 5e-3 and d.abs().max().item() <= 5e-2, (rel, d.abs().max().item())
