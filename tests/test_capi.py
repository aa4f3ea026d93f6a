"""The C-ABI library loads, exports every entry point its header declares,
and validates arguments before touching the GPU (no CUDA calls here)."""

import re

import pytest

from llm_hgemm import capi
from tests.conftest import REPO

HEADER = REPO / "include" / "hgemm_sm100.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hgemm_sm100_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "hgemm_sm100_run" in names and len(names) >= 8


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports(name):
    lib = capi.load()
    assert hasattr(lib, name), name


def test_config_names_round_trip():
    lib = capi.load()
    n = lib.hgemm_sm100_num_configs()
    assert n == 13
    for i in range(n):
        name = lib.hgemm_sm100_config_name(i).decode()
        assert lib.hgemm_sm100_config_from_name(name.encode()) == i
    assert lib.hgemm_sm100_config_name(n) is None
    assert lib.hgemm_sm100_config_from_name(b"cublaslt") == -1
    assert lib.hgemm_sm100_config_from_name(b"not-a-kernel") == -1


def test_header_enums_match_binding():
    text = HEADER.read_text()
    for const, value in [("HGEMM_SM100_CFG_AUTO", capi.CFG_AUTO),
                         ("HGEMM_SM100_CFG_SWAPAB", capi.CFG_SWAPAB),
                         ("HGEMM_SM100_CFG_GENERIC_128x128", capi.CFG_GENERIC_128x128),
                         ("HGEMM_SM100_ERR_PIPELINE_TIMEOUT", capi.ERR_PIPELINE_TIMEOUT),
                         ("HGEMM_SM100_FLAG_TEST_INJECT_TX", capi.FLAG_TEST_INJECT_TX)]:
        assert re.search(rf"\b{const}\s*=\s*{value}\b", text), const


def test_status_strings():
    assert capi.status_string(capi.OK) == "ok"
    assert "pipeline timeout" in capi.status_string(capi.ERR_PIPELINE_TIMEOUT)
    assert capi.status_string(capi.ERR_UNKNOWN_CONFIG) == "unknown implementation"


def test_workspace_is_zero():
    lib = capi.load()
    for cfg in range(lib.hgemm_sm100_num_configs()):
        assert lib.hgemm_sm100_workspace_bytes(cfg, 8192, 8192, 8192) == 0


@pytest.mark.parametrize("kwargs,expected", [
    (dict(a_ptr=0, b_ptr=16, c_ptr=16, m=1, n=1, k=1), capi.ERR_INVALID_ARGUMENT),
    (dict(a_ptr=16, b_ptr=16, c_ptr=16, m=0, n=1, k=1), capi.ERR_INVALID_ARGUMENT),
    (dict(a_ptr=16, b_ptr=16, c_ptr=16, m=4, n=4, k=4, lda=2), capi.ERR_INVALID_ARGUMENT),
    (dict(a_ptr=16, b_ptr=16, c_ptr=16, m=4, n=4, k=4, ldc=3), capi.ERR_INVALID_ARGUMENT),
    (dict(a_ptr=16, b_ptr=16, c_ptr=16, m=4, n=4, k=4, config=99), capi.ERR_UNKNOWN_CONFIG),
    (dict(a_ptr=16, b_ptr=16, c_ptr=16, m=4, n=4, k=4, split_k=17), capi.ERR_INVALID_ARGUMENT),
    (dict(a_ptr=16, b_ptr=16, c_ptr=16, m=2**31, n=4, k=4), capi.ERR_INVALID_ARGUMENT),
])
def test_run_rejects_bad_arguments(kwargs, expected):
    args = capi.make_args(**kwargs)
    assert capi.run(args) == expected
    rc, _, _ = capi.resolve(args)
    assert rc == expected
