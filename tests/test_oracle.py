"""Pins the oracle (oracle/reference.py) to the reference's own outputs.

tests/golden/ was produced by the reference's llm_hgemm/reference.py
(torch_reference, error_metrics, correctness_passed); see make_golden.py."""

import json
import math

import numpy as np
import pytest
import torch

from oracle import reference as oracle
from tests.conftest import GOLDEN
from tests.golden.make_golden import SHAPES, perturbations


@pytest.fixture(autouse=True)
def single_thread():
    saved = torch.get_num_threads()
    torch.set_num_threads(1)
    yield
    torch.set_num_threads(saved)


def _impl(name):
    """The test-side oracle, or the package's public gate API (llm_hgemm.reference):
    both restate the reference's llm_hgemm/reference.py and both are pinned to the
    fixtures it generated."""
    if name == "oracle":
        return oracle
    from llm_hgemm import reference as public
    return public


IMPLS = ["oracle", "llm_hgemm.reference"]


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_oracle_matches_reference_outputs(golden, shape, impl):
    tag = "x".join(map(str, shape))
    a = torch.from_numpy(golden[f"a_{tag}"])
    b = torch.from_numpy(golden[f"b_{tag}"])
    expected = golden[f"c_{tag}"]
    out = _impl(impl).torch_reference(a, b).numpy()
    assert out.dtype == np.float16 and out.shape == expected.shape
    # Same FP32 GEMM then one FP16 rounding: bit-identical on the same CPU.
    np.testing.assert_array_equal(out.view(np.uint16), expected.view(np.uint16))


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("pattern", ["uniform", "sparse"])
def test_oracle_input_patterns(golden, pattern, impl):
    a = torch.from_numpy(golden[f"a_{pattern}"])
    b = torch.from_numpy(golden[f"b_{pattern}"])
    out = _impl(impl).torch_reference(a, b).numpy()
    np.testing.assert_array_equal(out.view(np.uint16), golden[f"c_{pattern}"].view(np.uint16))


def test_zero_inputs_give_zero():
    a = torch.zeros((33, 47), dtype=torch.float16)
    b = torch.zeros((47, 29), dtype=torch.float16)
    assert torch.count_nonzero(oracle.torch_reference(a, b)) == 0


@pytest.mark.parametrize("impl", IMPLS)
def test_error_metrics_match_reference(golden, impl):
    gate = _impl(impl)
    spec = json.loads((GOLDEN / "metrics_golden.json").read_text())
    base = torch.from_numpy(golden[spec["base"]])
    outs = perturbations(base)
    for case in spec["cases"]:
        metrics = gate.error_metrics(outs[case["name"]], base)
        for key, value in case["metrics"].items():
            got = metrics[key]
            if isinstance(value, float) and math.isnan(value):
                assert math.isnan(got), (case["name"], key)
            else:
                assert got == value, (case["name"], key, got, value)
        assert gate.correctness_passed(metrics) == case["passed"], case["name"]


def test_stage_marker_known_answer():
    # Reference tests/test_v6_async.py:88-99: 32-row K tiles with markers
    # 1,2,4,8,16 /16 and A = 0.125 give exactly 7.75.
    a, b, expected = oracle.stage_marker_inputs(129, 136, 160, 32)
    assert expected == 7.75
    out = oracle.torch_reference(a, b)
    assert torch.all(out == 7.75)


def test_gate_thresholds():
    assert oracle.MAX_ABS_ERROR_LIMIT == 5e-2
    assert oracle.RELATIVE_L2_ERROR_LIMIT == 5e-3


def test_public_gate_api_agrees_with_oracle(golden):
    from llm_hgemm import reference as public

    a = torch.from_numpy(golden["a_129x77x1003"])
    b = torch.from_numpy(golden["b_129x77x1003"])
    assert torch.equal(public.torch_reference(a, b), oracle.torch_reference(a, b))
    out = (oracle.torch_reference(a, b).float() * 1.001).half()
    assert public.error_metrics(out, oracle.torch_reference(a, b)) == \
        oracle.error_metrics(out, oracle.torch_reference(a, b))
