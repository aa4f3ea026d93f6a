"""`auto`, `shape_auto` and the FrozenHgemmLinear adapter on the GPU
(reference tests/test_dispatch.py:9-15 re-specified, tests/test_v7.py)."""

import json

import pytest
import torch

from llm_hgemm import hgemm
from llm_hgemm.dispatch import configure_dispatch, last_selected, selected_implementation
from llm_hgemm.integration import FrozenHgemmLinear
from llm_hgemm.ops import _hgemm_out, backend_info, resolved_config
from llm_hgemm.provenance import code_fingerprint
from oracle import reference as oracle
from tests.gpu_helpers import assert_gate, require_cuda, seeded_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def reset_policy():
    require_cuda()
    configure_dispatch(None)
    yield
    configure_dispatch(None)


def policy_file(tmp_path, gpu=None):
    path = tmp_path / "dispatch.json"
    path.write_text(json.dumps({
        "schema_version": 3, "gpu": gpu or torch.cuda.get_device_name(),
        "cuda": torch.version.cuda, "torch": torch.__version__, "sm": "10.0",
        "code_fingerprint": code_fingerprint(),
        "entries": [{"M": 128, "N": 128, "K": 64, "best_available": "auto",
                     "best_custom": "tc_splitk_128x128"}],
    }))
    return path


@pytest.mark.parametrize("shape", [(64, 80, 48), (1, 4096, 2560), (512, 2560, 4096),
                                   (2048, 2048, 2048), (300, 520, 1000)])
def test_auto_matches_resolved_config_bitwise(shape):
    a, b = seeded_inputs(*shape)
    name, _ = resolved_config(a, b, "auto")
    assert name != "auto"
    auto = hgemm(a, b, implementation="auto")
    torch.testing.assert_close(auto, hgemm(a, b, implementation=name), rtol=0, atol=0)
    assert_gate(auto, a, b)


@pytest.mark.parametrize("strategy,expected", [("best_available", "auto"),
                                               ("best_custom", "tc_splitk_128x128")])
def test_strategy_selection(tmp_path, strategy, expected):
    configure_dispatch(policy_file(tmp_path), strategy=strategy)
    a, b = seeded_inputs(128, 128, 64)
    assert selected_implementation(a, b) == expected
    out = hgemm(a, b, implementation="shape_auto")
    assert last_selected() == expected
    assert_gate(out, a, b)
    assert backend_info("shape_auto") == backend_info(expected)


@pytest.mark.parametrize("strategy", ["best_available", "best_custom"])
@pytest.mark.parametrize("shape", [(127, 129, 63), (1, 136, 40), (65, 80, 48)])
def test_unknown_shape_uses_auto(tmp_path, strategy, shape):
    configure_dispatch(policy_file(tmp_path), strategy=strategy)
    a, b = seeded_inputs(*shape)
    assert selected_implementation(a, b) == "auto"
    assert_gate(hgemm(a, b, implementation="shape_auto"), a, b)


def test_misaligned_goes_auto(tmp_path):
    configure_dispatch(policy_file(tmp_path), strategy="best_custom")
    a, b = seeded_inputs(128, 128, 64)
    storage = torch.empty(a.numel() + 1, device="cuda", dtype=torch.float16)
    shifted = storage[1:].view_as(a)
    shifted.copy_(a)
    assert selected_implementation(shifted, b) == "auto"
    assert_gate(hgemm(shifted, b, implementation="shape_auto"), shifted, b)


def test_gpu_name_mismatch_falls_back(tmp_path):
    configure_dispatch(policy_file(tmp_path, gpu="different GPU"), strategy="best_custom")
    a, b = seeded_inputs(128, 128, 64)
    assert selected_implementation(a, b) == "auto"


def test_shape_auto_side_stream(tmp_path):
    configure_dispatch(policy_file(tmp_path), strategy="best_custom")
    a, b = seeded_inputs(128, 128, 64)
    out = torch.full((128, 128), float("nan"), device="cuda", dtype=torch.float16)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        returned = _hgemm_out(a, b, out, implementation="shape_auto")
    torch.cuda.current_stream().wait_stream(stream)
    assert returned is out
    assert_gate(out, a, b)


@pytest.mark.parametrize("shape", [(2, 64, 64), (3, 64), (64,)])
def test_adapter(tmp_path, shape):
    configure_dispatch(policy_file(tmp_path), strategy="best_custom")
    layer = torch.nn.Linear(64, 128, bias=False, device="cuda", dtype=torch.float16).eval()
    adapter = FrozenHgemmLinear(layer)
    x = torch.randn(shape, device="cuda", dtype=torch.float16) * 0.1
    with torch.inference_mode():
        actual, expected = adapter(x), layer(x)
    assert actual.shape == expected.shape
    assert oracle.correctness_passed(oracle.error_metrics(actual, expected))


def test_adapter_noncontiguous_and_empty():
    layer = torch.nn.Linear(64, 128, bias=False, device="cuda", dtype=torch.float16).eval()
    adapter = FrozenHgemmLinear(layer)
    inputs = [torch.randn((64, 3), device="cuda", dtype=torch.float16).T,
              torch.empty((0, 64), device="cuda", dtype=torch.float16)]
    with torch.inference_mode():
        for x in inputs:
            torch.testing.assert_close(adapter(x), layer(x), rtol=0, atol=0)


def test_training_rejected():
    layer = torch.nn.Linear(64, 128, bias=False, device="cuda", dtype=torch.float16)
    adapter = FrozenHgemmLinear(layer)
    with pytest.raises(RuntimeError, match="inference-only"):
        adapter(torch.randn((2, 64), device="cuda", dtype=torch.float16))


def test_changed_weight_rejected():
    layer = torch.nn.Linear(64, 128, bias=False, device="cuda", dtype=torch.float16)
    adapter = FrozenHgemmLinear(layer)
    with torch.no_grad():
        layer.weight.add_(1)
        with pytest.raises(RuntimeError, match="weights changed"):
            adapter(torch.randn((2, 64), device="cuda", dtype=torch.float16))
