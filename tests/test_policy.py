"""Exact-shape policy loading and selection logic (host only, no GPU).

Mirrors the policy checks of reference tests/test_v7.py:21-143 that do not
launch kernels: schema / version / fingerprint / SM validation, strategy
validation and the selection fallbacks."""

import json

import pytest
import torch

from llm_hgemm import dispatch
from llm_hgemm.dispatch import configure_dispatch, last_selected, selected_implementation
from llm_hgemm.provenance import code_fingerprint


@pytest.fixture(autouse=True)
def reset_policy():
    configure_dispatch(None)
    yield
    configure_dispatch(None)


def policy_payload(**overrides):
    payload = {
        "schema_version": 3, "gpu": "NVIDIA B200", "cuda": torch.version.cuda,
        "torch": torch.__version__, "sm": "10.0", "code_fingerprint": code_fingerprint(),
        "entries": [{"M": 128, "N": 128, "K": 64, "best_available": "auto",
                     "best_custom": "tc_splitk_128x128"}],
    }
    payload.update(overrides)
    return payload


def write(tmp_path, payload):
    path = tmp_path / "dispatch.json"
    path.write_text(json.dumps(payload))
    return path


def test_valid_policy_loads(tmp_path):
    configure_dispatch(write(tmp_path, policy_payload()), strategy="best_custom")
    pol = dispatch.policy()
    assert pol["entries"] == {(128, 128, 64): "tc_splitk_128x128"}
    assert pol["strategy"] == "best_custom"


@pytest.mark.parametrize("field,value,match", [
    ("schema_version", 2, "schema_version"),
    ("torch", "0.0", "PyTorch version"),
    ("cuda", "0.0", "CUDA version"),
    ("code_fingerprint", "stale", "fingerprint"),
    ("sm", "8.6", "SM100"),
])
def test_policy_rejected(tmp_path, field, value, match):
    with pytest.raises(ValueError, match=match):
        configure_dispatch(write(tmp_path, policy_payload(**{field: value})))


def test_invalid_provider_rejected(tmp_path):
    payload = policy_payload(entries=[{"M": 1, "N": 1, "K": 1, "best_available": "cublaslt",
                                       "best_custom": "auto"}])
    with pytest.raises(ValueError, match="invalid provider"):
        configure_dispatch(write(tmp_path, payload))


def test_duplicate_shape_rejected(tmp_path):
    entry = {"M": 1, "N": 1, "K": 1, "best_available": "auto", "best_custom": "auto"}
    with pytest.raises(ValueError, match="duplicate"):
        configure_dispatch(write(tmp_path, policy_payload(entries=[entry, entry])))


def test_invalid_strategy():
    with pytest.raises(ValueError, match="strategy"):
        configure_dispatch(None, strategy="invalid")


def test_explicit_names_pass_through():
    a = torch.zeros((4, 4), dtype=torch.float16)
    assert selected_implementation(a, a, "tc_swapab") == "tc_swapab"


def test_invalid_contract_goes_to_auto(tmp_path):
    configure_dispatch(write(tmp_path, policy_payload()), strategy="best_custom")
    a = torch.zeros((128, 64), dtype=torch.float16)   # CPU tensors break the contract
    b = torch.zeros((64, 128), dtype=torch.float16)
    assert selected_implementation(a, b) == "auto"


def test_last_selected_is_thread_local():
    import threading

    dispatch.record_selected("tc_swapab")
    seen = []

    def worker():
        try:
            last_selected()
        except RuntimeError as exc:
            seen.append(str(exc))

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert last_selected() == "tc_swapab"
    assert seen and "has not executed" in seen[0]
