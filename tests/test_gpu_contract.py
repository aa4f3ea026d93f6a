"""Contract errors and messages (reference tests/test_contract.py:16-66)."""

import pytest
import torch

from llm_hgemm import hgemm
from llm_hgemm.ops import _hgemm_out
from tests.gpu_helpers import require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()


def tensors(m=16, n=16, k=16):
    a = torch.randn((m, k), device="cuda", dtype=torch.float16)
    b = torch.randn((k, n), device="cuda", dtype=torch.float16)
    return a, b


def test_rejects_cpu_tensor():
    a = torch.randn((16, 16), dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        hgemm(a, a, implementation="auto")


def test_rejects_wrong_dtype():
    a = torch.randn((16, 16), device="cuda", dtype=torch.float32)
    b = torch.randn((16, 16), device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="float16"):
        hgemm(a, b, implementation="auto")


def test_rejects_k_mismatch():
    a, _ = tensors(m=8, n=9, k=7)
    b = torch.randn((6, 9), device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="K dimensions"):
        hgemm(a, b, implementation="tc_splitk_128x128")


def test_rejects_noncontiguous_input():
    a, b = tensors()
    with pytest.raises(RuntimeError, match="contiguous"):
        hgemm(a.t(), b, implementation="auto")


def test_rejects_zero_dimension():
    a = torch.empty((0, 16), device="cuda", dtype=torch.float16)
    b = torch.empty((16, 8), device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="positive"):
        hgemm(a, b, implementation="auto")


def test_rejects_three_dimensional():
    a = torch.randn((2, 16, 16), device="cuda", dtype=torch.float16)
    b = torch.randn((16, 16), device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="two-dimensional"):
        hgemm(a, b, implementation="auto")


def test_rejects_bad_output():
    a, b = tensors(m=8, n=9, k=7)
    out = torch.empty((8, 8), device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="out must have shape"):
        _hgemm_out(a, b, out, implementation="auto")


def test_rejects_unknown_implementation():
    a, b = tensors()
    with pytest.raises(RuntimeError, match="unknown implementation"):
        hgemm(a, b, implementation="not-a-kernel")


def test_cublaslt_is_not_a_dispatch_target():
    a, b = tensors()
    with pytest.raises(RuntimeError, match="unknown implementation"):
        hgemm(a, b, implementation="cublaslt")


def test_rejects_non_none_epilogue():
    a, b = tensors()
    with pytest.raises(RuntimeError, match="epilogue"):
        hgemm(a, b, implementation="auto", epilogue="bias")
