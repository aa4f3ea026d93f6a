"""The -DHGEMM_DEBUG build (libhgemm_sm100_debug.so): its device-side bounds
checks guard every global access whose address the kernels compute
themselves - the generic (no-TMA) tile loader, the operand-staging copies
and the epilogue's register stores. Here the debug library runs those paths
on ragged, misaligned and padded operands (with NaN guard bands around them,
as the pipeline tests do): every result must pass the oracle's gate, no check
may have failed (no recorded line, status word clear), and nothing outside
the matrices may change. The checks' own logic is tested on the CPU
(tests/test_capi.py)."""

import pytest
import torch

from llm_hgemm import capi
from oracle import reference as oracle
from tests.gpu_helpers import require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()
    assert capi.load(debug=True).hgemm_sm100_debug_build() == 1
    capi.debug_read(clear=True)
    capi.read_status(clear=True, debug=True)


def guarded(rows, cols, ld, offset, fill, seed=None):
    """A [rows x cols] FP16 view with pitch `ld` starting `offset` elements
    into a buffer that is `fill` everywhere else (guard band of 64 elements
    after the last row). With `seed`, the view holds randn * 0.1."""
    buf = torch.full((offset + rows * ld + 64,), fill, device="cuda", dtype=torch.float16)
    view = buf[offset:offset + rows * ld].view(rows, ld)[:, :cols]
    if seed is not None:
        g = torch.Generator(device="cuda").manual_seed(seed)
        view.copy_((torch.randn((rows, cols), generator=g, device="cuda") * 0.1).half())
    return buf, view


def run_debug(a, b, c, config, *, workspace=True, epilogue=0, bias=None, residual=None, f32=False):
    m, k = a.shape
    n = b.shape[1]
    args = capi.make_args(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k,
                          lda=a.stride(0), ldb=b.stride(0), ldc=c.stride(0), config=config,
                          flags=capi.FLAG_OUT_F32 if f32 else 0, epilogue=epilogue,
                          bias_ptr=None if bias is None else bias.data_ptr(),
                          residual_ptr=None if residual is None else residual.data_ptr(),
                          ldr=None if residual is None else residual.stride(0))
    keep = None
    if workspace:
        need = capi.workspace_size(args, debug=True)
        if need:
            keep = torch.empty(need, device="cuda", dtype=torch.uint8)
            args.workspace, args.workspace_bytes = keep.data_ptr(), need
    assert capi.run(args, torch.cuda.current_stream().cuda_stream, debug=True) == capi.OK
    torch.cuda.synchronize()
    del keep


def assert_clean():
    rc, line, i0, i1 = capi.debug_read(clear=True)
    assert rc == capi.OK and line == 0, f"bounds check failed at line {line} (indices {i0}, {i1})"
    rc, status = capi.read_status(clear=True, debug=True)
    assert rc == capi.OK and status == 0, capi.status_string(status)


# (M, N, K), element offsets of A, B, C and extra pitch (row padding).
CASES = [((70, 136, 72), (1, 0, 0), 0), ((129, 257, 200), (0, 1, 1), 3), ((300, 520, 1000), (3, 5, 7), 1),
         ((17, 1000, 333), (1, 1, 1), 5), ((1, 4099, 2561), (1, 3, 0), 0)]
CONFIGS = {"generic (no workspace)": (capi.CFG_GENERIC_128x128, False),
           "staged auto": (capi.CFG_AUTO, True),
           "staged persistent": (capi.CFG_PERSISTENT_128x256, True),
           "staged pair": (capi.CFG_PAIR_256x256, True),
           "staged split-K": (capi.CFG_SPLITK_128x128, True),
           "staged swap-AB": (capi.CFG_SWAPAB, True)}


@pytest.mark.parametrize("config", list(CONFIGS))
@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c[0])) + f"+{c[1]}")
def test_debug_build_generic_and_staged_paths(config, case):
    (m, n, k), (oa, ob, oc), pad = case
    cfg, workspace = CONFIGS[config]
    abuf, a = guarded(m, k, k + pad, oa, float("nan"), seed=1)
    bbuf, b = guarded(k, n, n + pad, ob, float("nan"), seed=2)
    cbuf, c = guarded(m, n, n + pad, oc, 7.0)
    before = cbuf.clone()
    run_debug(a, b, c, cfg, workspace=workspace)
    assert_clean()
    metrics = oracle.check(c.contiguous(), a.contiguous(), b.contiguous())
    assert metrics["passed"], metrics
    # Nothing outside C changed (guard band, row padding, the offset).
    mask = torch.ones_like(cbuf, dtype=torch.bool)
    mask[oc:oc + m * (n + pad)].view(m, n + pad)[:, :n] = False
    assert torch.equal(cbuf[mask], before[mask])


@pytest.mark.parametrize("epilogue", ["bias", "residual", "silu_mul"])
@pytest.mark.parametrize("cfg", [capi.CFG_GENERIC_128x128, capi.CFG_SWAPAB, capi.CFG_SPLITK_128x128])
def test_debug_build_epilogue_stores(epilogue, cfg):
    m, n, k = 37, 266, 300
    a = torch.randn((m, k), device="cuda", dtype=torch.float16) * 0.1
    b = torch.randn((k, n), device="cuda", dtype=torch.float16) * 0.1
    bias = torch.randn(n, device="cuda", dtype=torch.float16) * 0.1 if epilogue == "bias" else None
    residual = torch.randn((m, n), device="cuda", dtype=torch.float16) * 0.1 if epilogue == "residual" else None
    cols = n // 2 if epilogue == "silu_mul" else n
    cbuf, c = guarded(m, cols, cols + 1, 1, 7.0)      # odd pitch: register stores, element by element
    bits = {"bias": capi.EPI_BIAS, "residual": capi.EPI_RESIDUAL, "silu_mul": capi.EPI_SILU_MUL}[epilogue]
    run_debug(a, b, c, cfg, workspace=False, epilogue=bits, bias=bias, residual=residual)
    assert_clean()
    ref = oracle.torch_reference_epilogue(a.cpu(), b.cpu(), epilogue,
                                          bias=None if bias is None else bias.cpu(),
                                          residual=None if residual is None else residual.cpu())
    assert oracle.correctness_passed(oracle.error_metrics(c.cpu(), ref))


@pytest.mark.parametrize("cfg", [capi.CFG_GENERIC_128x128, capi.CFG_SWAPAB, capi.CFG_PERSISTENT_128x256])
def test_debug_build_fp32_output(cfg):
    m, n, k = 100, 264, 1000
    a = torch.randn((m, k), device="cuda", dtype=torch.float16) * 0.1
    b = torch.randn((k, n), device="cuda", dtype=torch.float16) * 0.1
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32)
    run_debug(a, b, out, cfg, workspace=False, f32=True)
    assert_clean()
    torch.testing.assert_close(out.cpu(), a.cpu().float() @ b.cpu().float(), rtol=1e-4, atol=1e-4)
