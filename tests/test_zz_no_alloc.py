"""The entry point that allocates nothing (hgemm_sm100_run_static_scratch).

Some hosts cannot hand this library a workspace: a plugin or FFI host that is
given only input/output pointers and a stream, or a runtime that plans all of
its device memory before it starts and must not call cudaMalloc (which can
synchronise the device) while it runs. This entry point takes the stream-K
scratch from a fixed static device buffer instead. These tests call it through
the C ABI, twice in a row on the same buffers, and check each result against
the regular entry point (hgemm_sm100_run with a workspace) with the gate the
other parity tests use; they also check that an explicit stream-K request
needing more scratch than the buffer holds is refused without touching the
output, while `auto` runs such a problem without scratch.

Kept in a file that pytest collects last."""

import pytest
import torch

from llm_hgemm import capi
from oracle import reference as oracle
from tests.gpu_helpers import assert_gate, require_cuda, seeded_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


def scratch_shapes():
    """(M, N, K, uses_scratch) from this GPU's SM count: swap-AB stream-K
    problems whose tile count leaves a partial last wave (a split tail, which
    needs the scratch), and one with fewer tiles than SMs (none needed)."""
    sms = _sms()
    return [
        (1, 128 * (sms + sms // 2), 2560, True),
        (16, 128 * (7 * sms + 3), 640, True),
        (128, 128 * (sms + 5) - 16, 1000, True),
        (1, 128 * (sms // 2), 2560, False),
    ]


def regular(a, b, cfg, *, n=None, ldb=None, ldc=None, epilogue=0, bias=None):
    """C through hgemm_sm100_run with the workspace it asks for."""
    m, k = a.shape
    n = b.shape[1] if n is None else n
    ldc = n if ldc is None else ldc
    out = torch.full((m, ldc), float("nan"), device="cuda", dtype=torch.float16)
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, ldb=ldb, ldc=ldc,
                          config=cfg, epilogue=epilogue,
                          bias_ptr=None if bias is None else bias.data_ptr())
    need = capi.workspace_size(args)
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    if need:
        args.workspace, args.workspace_bytes = ws.data_ptr(), need
    assert capi.run(args, torch.cuda.current_stream().cuda_stream) == capi.OK
    torch.cuda.synchronize()
    return out[:, :n]


def static_twice(a, b, expected, *, n=None, ldb=None, ldc=None, epilogue=0, bias=None, check=None):
    """Two calls in a row of the static-scratch entry point into fresh NaN
    outputs; each must pass the gate against `expected`."""
    m, k = a.shape
    n = b.shape[1] if n is None else n
    ldc = n if ldc is None else ldc
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full((m, ldc), float("nan"), device="cuda", dtype=torch.float16)
        args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, ldb=ldb, ldc=ldc,
                              config=capi.CFG_AUTO, epilogue=epilogue,
                              bias_ptr=None if bias is None else bias.data_ptr())
        assert capi.run_static_scratch(args, stream) == capi.OK, call
        torch.cuda.synchronize()
        got = out[:, :n]
        metrics = oracle.error_metrics(got, expected)
        assert oracle.correctness_passed(metrics), (call, metrics)
        if check is not None:
            check(got)


@pytest.mark.parametrize("case", range(4))
def test_static_scratch_matches_regular_entry_twice(case):
    m, n, k, uses = scratch_shapes()[case]
    a, b = seeded_inputs(m, n, k)
    probe = capi.make_args(a.data_ptr(), b.data_ptr(), 0, m, n, k, config=capi.CFG_STREAMK_SWAPAB)
    probe.c = a.data_ptr()   # any non-null pointer: workspace_size launches nothing
    need = capi.workspace_size(probe)
    assert (need > 0) == uses, need
    assert need <= capi.STATIC_SCRATCH_BYTES
    expected = regular(a, b, capi.CFG_STREAMK_SWAPAB)
    static_twice(a, b, expected, check=lambda got: assert_gate(got, a, b))


def test_static_scratch_ragged_c_and_padded_b():
    # Odd N: B lives in a padded [K, ldb] buffer (TMA-describable), C rows
    # have an odd pitch (no TMA store; direct stores).
    sms = _sms()
    m, n, k = 16, 128 * (sms + sms // 2) - 3, 1024
    ldb = (n + 7) // 8 * 8
    a, b_full = seeded_inputs(m, ldb, k)
    b = b_full[:, :n]
    expected = regular(a, b_full, capi.CFG_STREAMK_SWAPAB, n=n, ldb=ldb, ldc=n)
    static_twice(a, b_full, expected, n=n, ldb=ldb, ldc=n,
                 check=lambda got: assert_gate(got, a, b.contiguous()))


def test_static_scratch_bias_epilogue():
    sms = _sms()
    m, n, k = 8, 128 * (sms + sms // 2), 2560
    a, b = seeded_inputs(m, n, k)
    torch.manual_seed(7)
    bias = torch.randn(n, device="cuda", dtype=torch.float16)
    expected = regular(a, b, capi.CFG_STREAMK_SWAPAB, epilogue=capi.EPI_BIAS, bias=bias)

    def check(got):
        ref = oracle.torch_reference_epilogue(a.cpu(), b.cpu(), "bias", bias=bias.cpu())
        assert oracle.correctness_passed(oracle.error_metrics(got.cpu(), ref))

    static_twice(a, b, expected, epilogue=capi.EPI_BIAS, bias=bias, check=check)


def test_static_scratch_auto_runs_large_split_tail_without_scratch():
    # More 128x256 tiles than SMs with a partial last wave: the stream-K split
    # tail would need one 128 KiB slot per SM, more than the static buffer on
    # a 148-SM GPU. `auto` runs the problem with whole tiles instead.
    m, n, k = 2048, 2560, 4096
    a, b = seeded_inputs(m, n, k)
    expected = regular(a, b, capi.CFG_AUTO)
    static_twice(a, b, expected, check=lambda got: assert_gate(got, a, b))


def test_static_scratch_refuses_explicit_streamk_beyond_its_buffer():
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
