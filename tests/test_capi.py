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
    assert n == 14
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


# --------------------------------------------------------- debug build --

@pytest.mark.parametrize("name", declared_functions())
def test_debug_library_exports(name):
    assert hasattr(capi.load(debug=True), name), name


def test_debug_build_flag_and_empty_record():
    assert capi.load().hgemm_sm100_debug_build() == 0
    assert capi.load(debug=True).hgemm_sm100_debug_build() == 1
    # A release build records nothing and touches no GPU.
    assert capi.debug_read(debug=False) == (capi.OK, 0, 0, 0)
    assert re.search(r"\bHGEMM_SM100_ERR_DEBUG_BOUNDS\s*=\s*9\b", HEADER.read_text())
    assert "debug bounds" in capi.status_string(capi.ERR_DEBUG_BOUNDS)


def _elements(base, rows, cols, ld, esize):
    """Byte addresses of every element of the matrix (a plain restatement)."""
    return {base + esize * (r * ld + c) for r in range(rows) for c in range(cols)}


@pytest.mark.parametrize("base,rows,cols,ld", [(4096, 3, 5, 7), (4098, 4, 9, 9), (4110, 2, 16, 21),
                                               (4096, 1, 1, 1), (4102, 5, 3, 8)])
def test_debug_vector_rule_matches_a_brute_force_restatement(base, rows, cols, ld):
    # The generic loader may load a 16-byte-aligned vector only when it holds
    # at least one element of its operand.
    elems = _elements(base, rows, cols, ld, 2)
    lo, hi = (min(elems) // 16 - 2) * 16, (max(elems) // 16 + 3) * 16
    for vec in range(lo, hi, 16):
        expect = any(vec <= e < vec + 16 for e in elems)
        assert capi.debug_vec_touches(vec, base, rows, cols, ld) == expect, vec
    assert not capi.debug_vec_touches(lo + 2, base, rows, cols, ld)      # unaligned vectors never pass


@pytest.mark.parametrize("esize", [2, 4])
def test_debug_span_rule_matches_a_brute_force_restatement(esize):
    base, rows, cols, ld = 8192, 3, 6, 10
    elems = _elements(base, rows, cols, ld, esize)
    for ptr in range(base - 4 * esize, base + esize * (rows * ld + 4)):
        for count in (1, 2, 4, 8):
            span = {ptr + esize * i for i in range(count)}
            same_row = (ptr - base) % esize == 0 and ptr >= base and \
                ((ptr - base) // esize) % ld + count <= ld
            expect = span <= elems and same_row
            assert capi.debug_span_in(ptr, count, base, rows, cols, ld, esize) == expect, (ptr, count)
