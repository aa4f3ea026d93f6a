"""The entry point that allocates nothing (hgemm_sm100_run_static_scratch).

Callers such as a plugin or FFI host that is handed only input/output pointers
and a stream, or a runtime that plans all of its device memory ahead of time,
cannot hand the library a workspace. This entry point takes its stream-K
scratch from a fixed static device buffer instead. These tests call it through
the C ABI, twice in a row on the same buffers, and check each result against
the regular entry point (hgemm_sm100_run with a workspace) with the gate the
other parity tests use; they also check that a problem needing more scratch
than the buffer holds is refused without touching the output.

Kept in a file that pytest collects last."""

import pytest
import torch

from llm_hgemm import capi
from oracle import reference as oracle
from tests.gpu_helpers import assert_gate, require_cuda, seeded_inputs

pytestmark = pytest.mark.gpu

# (M, N, K): swap-AB stream-K with a split tail (uses the scratch), and one
# without a split tail (needs none).
SHAPES = [(1, 19200, 2560), (16, 151936, 640), (128, 20000, 1000), (1, 9728, 2560)]


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()


def regular(a, b, cfg):
    m, k = a.shape
    n = b.shape[1]
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, config=cfg)
    need = capi.workspace_size(args)
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    if need:
        args.workspace, args.workspace_bytes = ws.data_ptr(), need
    assert capi.run(args, torch.cuda.current_stream().cuda_stream) == capi.OK
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_static_scratch_matches_regular_entry_twice(shape):
    m, n, k = shape
    a, b = seeded_inputs(m, n, k)
    expected = regular(a, b, capi.CFG_STREAMK_SWAPAB)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
        args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
                              config=capi.CFG_AUTO)
        assert capi.run_static_scratch(args, stream) == capi.OK, call
        torch.cuda.synchronize()
        metrics = oracle.error_metrics(out, expected)
        assert oracle.correctness_passed(metrics), (call, metrics)
        assert_gate(out, a, b)


def test_static_scratch_refuses_problems_beyond_its_buffer():
    # A 128x256 stream-K split tail needs one 128 KiB slot per SM: more than
    # the static buffer holds on a 148-SM GPU.
    m, n, k = 2048, 2560, 4096
    a, b = seeded_inputs(m, n, k)
    out = torch.full((m, n), 7.0, device="cuda", dtype=torch.float16)
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
                          config=capi.CFG_STREAMK_128x256)
    if capi.workspace_size(args) <= capi.STATIC_SCRATCH_BYTES:
        pytest.skip("this GPU's split tail fits the static buffer")
    rc = capi.run_static_scratch(args, torch.cuda.current_stream().cuda_stream)
    assert rc == capi.ERR_SCRATCH_LIMIT
    assert "static buffer" in capi.status_string(rc)
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)


def test_static_scratch_rejects_other_configs_and_unaligned_operands():
    m, n, k = 16, 4096, 2560
    a, b = seeded_inputs(m, n, k)
    out = torch.empty((m, n), device="cuda", dtype=torch.float16)
    stream = torch.cuda.current_stream().cuda_stream
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
                          config=capi.CFG_PERSISTENT_128x256)
    assert capi.run_static_scratch(args, stream) == capi.ERR_UNKNOWN_CONFIG
    args = capi.make_args(a.data_ptr() + 2, b.data_ptr(), out.data_ptr(), m, n, k - 1,
                          config=capi.CFG_AUTO)
    assert capi.run_static_scratch(args, stream) == capi.ERR_INVALID_ARGUMENT
