"""The committed SM100 exact-shape table and its validation summary (CPU):
schema, the Qwen3-4B shape set it covers, provider names, and that the
validation summary describes this very table. Loading it also needs the
table to have been tuned on the current sources (its code fingerprint)."""

import json

import pytest

from tests.conftest import PKG

from llm_hgemm import dispatch, tune
from llm_hgemm.provenance import code_fingerprint, file_sha256

TABLE = PKG / "configs" / "sm100_dispatch.json"
VALIDATION = PKG / "configs" / "sm100_dispatch_validation.json"


def test_table_schema_and_coverage():
    table = json.loads(TABLE.read_text())
    assert table["schema_version"] == dispatch.SCHEMA_VERSION and str(table["sm"]) == dispatch.TARGET_SM
    assert table["baseline"] == "auto" and table["min_gain"] == 0.05 and table["max_variation"] == 0.10
    shapes = [(e["M"], e["N"], e["K"]) for e in table["entries"]]
    assert sorted(shapes) == sorted(tune.shape_set("qwen3_4b")) and len(shapes) == 48
    allowed = set(dispatch.CUSTOM_PROVIDERS) | {"auto"}
    for e in table["entries"]:
        assert e["best_available"] in allowed and e["best_custom"] in allowed
        # best_available is either the baseline or the measured best configuration.
        assert e["best_available"] in ("auto", e["best_custom"])


def test_validation_describes_this_table():
    table = json.loads(TABLE.read_text())
    summary = json.loads(VALIDATION.read_text())
    assert summary["dispatch_sha256"] == file_sha256(TABLE)
    assert summary["environment"]["code_fingerprint"] == table["code_fingerprint"]
    assert summary["shape_count"] == len(table["entries"]) == len(summary["details"])
    wanted = {(e["M"], e["N"], e["K"]): e[summary["strategy"]] for e in table["entries"]}
    for d in summary["details"]:
        assert wanted[(d["M"], d["N"], d["K"])] == d["implementation"]
        assert d["ratio_to_cublaslt"] == pytest.approx(d["cublaslt_median_us"] / d["custom_median_us"], rel=1e-6)


def test_table_loads_for_these_sources():
    table = json.loads(TABLE.read_text())
    if table["code_fingerprint"] != code_fingerprint():
        pytest.xfail("sources changed since the table was tuned: re-run llm_hgemm.tune on a B200")
    try:
        dispatch.configure_dispatch(TABLE)
        assert dispatch.policy()["table_sha256"] == file_sha256(TABLE)
    finally:
        dispatch.configure_dispatch(None)
