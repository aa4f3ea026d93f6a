"""Parity of every kernel configuration with the oracle.

Shapes and input patterns of reference tests/test_correctness.py:10-75 and
tests/test_boundaries.py:10-41, plus the committed golden fixtures (inputs
and outputs of the reference's own torch_reference)."""

import pytest
import torch

from llm_hgemm import hgemm
from oracle import reference as oracle
from tests.golden.make_golden import SHAPES
from tests.gpu_helpers import IMPLEMENTATIONS, assert_gate, require_cuda, seeded_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
@pytest.mark.parametrize("shape", [(16, 16, 16), (32, 64, 48), (37, 53, 29), (128, 256, 64),
                                   (129, 77, 1003)])
def test_hgemm_backends(impl, shape):
    a, b = seeded_inputs(*shape, seed=2026)
    assert_gate(hgemm(a, b, implementation=impl), a, b)


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
@pytest.mark.parametrize("shape", [(1, 1, 1), (15, 17, 31), (17, 33, 65), (127, 129, 63),
                                   (129, 257, 33)])
def test_non_tile_aligned_shapes(impl, shape):
    a, b = seeded_inputs(*shape, seed=7)
    assert_gate(hgemm(a, b, implementation=impl), a, b)


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
@pytest.mark.parametrize("pattern", ["zeros", "uniform", "sparse"])
def test_input_patterns(impl, pattern):
    torch.manual_seed(2026)
    if pattern == "zeros":
        a = torch.zeros((33, 47), device="cuda", dtype=torch.float16)
        b = torch.zeros((47, 29), device="cuda", dtype=torch.float16)
    elif pattern == "uniform":
        a = (torch.rand((33, 47), device="cuda", dtype=torch.float16) - 0.5) * 0.2
        b = (torch.rand((47, 29), device="cuda", dtype=torch.float16) - 0.5) * 0.2
    else:
        a = torch.randn((33, 47), device="cuda", dtype=torch.float16) * 0.1
        b = torch.randn((47, 29), device="cuda", dtype=torch.float16) * 0.1
        a[a.abs() < 0.12] = 0
        b[b.abs() < 0.12] = 0
    out = hgemm(a, b, implementation=impl)
    assert_gate(out, a, b)
    if pattern == "zeros":
        assert torch.count_nonzero(out) == 0


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_golden_fixtures(golden, impl, shape):
    tag = "x".join(map(str, shape))
    a = torch.from_numpy(golden[f"a_{tag}"]).cuda()
    b = torch.from_numpy(golden[f"b_{tag}"]).cuda()
    expected = torch.from_numpy(golden[f"c_{tag}"])
    out = hgemm(a, b, implementation=impl).cpu()
    metrics = oracle.error_metrics(out, expected)
    assert oracle.correctness_passed(metrics), metrics


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
@pytest.mark.parametrize("shape", [(2048, 2048, 2048), (1, 4096, 2560), (16, 2560, 9728),
                                   (512, 1024, 2560), (300, 520, 2056), (2047, 1031, 777)])
def test_medium_shapes(impl, shape):
    a, b = seeded_inputs(*shape, seed=2026)
    assert_gate(hgemm(a, b, implementation=impl), a, b)
