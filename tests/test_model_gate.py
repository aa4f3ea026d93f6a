"""The model-level logits gate on CPU (counterpart of the reference's
tests/test_integration_gate.py:40-57): both limits kept as they are, a
non-finite logit on either side fails, and a missing step or a shape
mismatch is an error rather than a pass."""

import importlib.util

import pytest
import torch

from tests.conftest import PKG


def load_model_check():
    spec = importlib.util.spec_from_file_location("model_check", PKG / "model_check.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


mc = load_model_check()


def test_identical_logits_pass():
    ref = torch.randn(4, 32)
    gate = mc.logits_gate([ref.clone(), ref.clone()], [ref, ref])
    assert gate["correctness"] == "pass"
    assert gate["logits_max_abs_error"] == 0.0
    assert gate["logits_max_relative_l2_error"] == 0.0
    assert [s["step"] for s in gate["logits_per_step_errors"]] == [0, 1]


def test_relative_gate_is_not_relaxed():
    ref = torch.ones(8)
    gate = mc.logits_gate([ref * 1.004], [ref])
    assert gate["correctness"] == "fail"
    assert gate["logits_max_abs_error"] < mc.MAX_LOGIT_ABS
    assert gate["logits_max_relative_l2_error"] > mc.MAX_LOGIT_REL_L2
    assert (mc.MAX_LOGIT_ABS, mc.MAX_LOGIT_REL_L2) == (0.05, 0.001)


def test_absolute_gate_is_kept():
    ref = torch.full((1000,), 10.0)
    out = ref.clone()
    out[0] += 0.06                     # relative L2 ~1.9e-4, max-abs over 0.05
    gate = mc.logits_gate([out], [ref])
    assert gate["logits_max_relative_l2_error"] < mc.MAX_LOGIT_REL_L2
    assert gate["correctness"] == "fail"


@pytest.mark.parametrize("value", [float("nan"), float("inf"), float("-inf")])
@pytest.mark.parametrize("side", ["actual", "expected"])
def test_nonfinite_logits_fail(value, side):
    ref = torch.ones(4, 8)
    bad = ref.clone()
    bad[1, 2] = value
    actual, expected = (bad, ref) if side == "actual" else (ref, bad)
    gate = mc.logits_gate([actual], [expected])
    assert gate["correctness"] == "fail"
    assert gate["logits_finite"] is False
    assert gate["logits_max_abs_error"] is None and gate["logits_max_relative_l2_error"] is None


def test_worst_step_decides():
    ref = torch.ones(16)
    gate = mc.logits_gate([ref.clone(), ref * 1.01], [ref, ref])
    assert gate["correctness"] == "fail"
    steps = gate["logits_per_step_errors"]
    assert steps[0]["relative_l2"] == 0.0 and steps[1]["relative_l2"] > mc.MAX_LOGIT_REL_L2


def test_missing_or_empty_trace_is_an_error():
    ref = torch.ones(4)
    with pytest.raises(ValueError):
        mc.logits_gate([], [])
    with pytest.raises(ValueError):
        mc.logits_gate([ref], [ref, ref])


def test_shape_mismatch_is_an_error():
    with pytest.raises(ValueError):
        mc.logits_gate([torch.ones(4, 8)], [torch.ones(4, 9)])
