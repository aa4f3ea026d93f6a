"""Policy tooling (llm_hgemm.tune): the selection rules of the reference's
offline tuner (benchmarks/tune_dispatch.py:12-57) on synthetic measurements,
and that a selected policy loads through configure_dispatch. CPU only."""

import json

import pytest
import torch

from llm_hgemm import dispatch, tune
from llm_hgemm.provenance import code_fingerprint


def env(**over):
    e = {"gpu": "NVIDIA B200", "sm": "10.0", "capability": [10, 0], "torch": torch.__version__,
         "torch_cuda": torch.version.cuda, "code_fingerprint": code_fingerprint(),
         "dispatch_sha256": None, "dispatch_strategy": None}
    e.update(over)
    return e


def payload(rows, **env_over):
    return {"environment": env(**env_over), "runs": 3, "samples": 20,
            "results": [{"M": m, "N": n, "K": k, "provider": p, "us": us} for (m, n, k, p, us) in rows]}


def test_variation():
    assert tune.variation([10.0, 10.0, 10.0]) == 0.0
    assert tune.variation([9.0, 10.0, 11.0]) == pytest.approx(0.2)


def test_fastest_stable_custom_and_min_gain():
    rows = [
        (16, 4096, 2560, "auto", [10.0, 10.1, 10.2]),
        (16, 4096, 2560, "tc_swapab", [9.0, 9.1, 9.2]),            # 10 % faster in every run
        (16, 4096, 2560, "tc_splitk_128x128", [7.0, 9.5, 8.0]),    # faster median, unstable
        (512, 1024, 2560, "auto", [10.0, 10.0, 10.0]),
        (512, 1024, 2560, "tc_swapab", [9.7, 9.8, 9.9]),           # < 5 % gain
    ]
    entries = {(e["M"], e["N"], e["K"]): e for e in tune.select([payload(rows)])}
    e1 = entries[(16, 4096, 2560)]
    assert e1["best_custom"] == "tc_swapab" and e1["best_available"] == "tc_swapab"
    e2 = entries[(512, 1024, 2560)]
    assert e2["best_custom"] == "tc_swapab" and e2["best_available"] == "auto"


def test_gain_must_hold_in_every_run():
    rows = [(1, 1024, 2560, "auto", [10.0, 10.0, 10.0]),
            (1, 1024, 2560, "tc_swapab", [9.0, 9.0, 9.6])]   # run 3 only 4 % faster
    (entry,) = tune.select([payload(rows)])
    assert entry["best_available"] == "auto"


def test_no_stable_candidate_falls_back_to_baseline():
    rows = [(1, 1024, 2560, "auto", [10.0, 10.0, 10.0]),
            (1, 1024, 2560, "tc_swapab", [5.0, 9.0, 13.0])]
    (entry,) = tune.select([payload(rows)])
    assert entry["best_custom"] == "auto" and not entry["custom_covered"]


def test_rejects_bad_inputs():
    rows = [(1, 1024, 2560, "tc_swapab", [9.0, 9.0, 9.0])]
    with pytest.raises(ValueError, match="baseline"):
        tune.select([payload(rows)])
    ok = [(1, 1024, 2560, "auto", [9.0, 9.0, 9.0])]
    with pytest.raises(ValueError, match="direct providers"):
        tune.select([payload(ok, dispatch_sha256="abc")])
    with pytest.raises(ValueError, match="different code"):
        tune.select([payload(ok), payload(ok, code_fingerprint="0" * 64)])
    with pytest.raises(ValueError, match="thresholds"):
        tune.select([payload(ok)], min_gain=1.5)


def test_selected_policy_loads(tmp_path):
    rows = [(16, 4096, 2560, "auto", [10.0, 10.0, 10.0]),
            (16, 4096, 2560, "tc_swapab", [8.0, 8.0, 8.0])]
    m = payload(rows)
    entries = tune.select([m])
    pol = tune.policy_payload(entries, m["environment"], min_gain=0.05, max_variation=0.10,
                              sources=["runs.json"])
    path = tmp_path / "sm100_dispatch.json"
    path.write_text(json.dumps(pol))
    try:
        dispatch.configure_dispatch(path, strategy="best_available")
        assert dispatch.policy()["entries"][(16, 4096, 2560)] == "tc_swapab"
    finally:
        dispatch.configure_dispatch(None)


def test_shape_sets(tmp_path):
    assert len(tune.shape_set("qwen3_4b")) == 48
    f = tmp_path / "shapes.json"
    f.write_text(json.dumps([[1, 2, 3]]))
    assert tune.shape_set(str(f)) == [(1, 2, 3)]


def test_unseen_shape_set_is_the_reference_unseen_check_plus_trace_m4():
    from llm_hgemm.tune import shape_set

    shapes = shape_set("unseen")
    assert len(shapes) == 24 and len(set(shapes)) == 24
    # The reference's 20 unseen shapes (M in {2, 8, 16, 64, 256} x four linears)...
    for m in (2, 8, 16, 64, 256):
        for (n, k) in ((2560, 4096), (2560, 9728), (4096, 2560), (9728, 2560)):
            assert (m, n, k) in shapes
    # ...and the M = 4 rows of its Qwen3-4B trace.
    assert {(4, 4096, 2560), (4, 2560, 4096), (4, 9728, 2560), (4, 2560, 9728)} <= set(shapes)
