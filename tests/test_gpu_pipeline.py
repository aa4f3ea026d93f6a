"""Pipeline edge cases: exact stage-marker known answers for every ring
depth, explicit K splits, guard bands around the output, NaN-prefilled
outputs on a side stream, misaligned operands.

Counterparts of reference tests/test_v6_async.py:21-99 and
tests/test_v5_vectorized.py:40-76."""

import pytest
import torch

from llm_hgemm import capi, hgemm
from llm_hgemm.ops import _hgemm_out, backend_info
from oracle import reference as oracle
from tests.gpu_helpers import IMPLEMENTATIONS, assert_gate, require_cuda, seeded_inputs

pytestmark = pytest.mark.gpu

CONFIG_IDS = {
    "tc_persistent_128x256": capi.CFG_PERSISTENT_128x256,
    "tc_persistent_128x128": capi.CFG_PERSISTENT_128x128,
    "tc_splitk_128x128": capi.CFG_SPLITK_128x128,
    "tc_swapab": capi.CFG_SWAPAB,
    "tc_generic_128x128": capi.CFG_GENERIC_128x128,
    "tc_pair_256x256": capi.CFG_PAIR_256x256,
    "tc_splitk_128x256": capi.CFG_SPLITK_128x256,
    "tc_streamk_128x256": capi.CFG_STREAMK_128x256,
    "tc_streamk_swapab": capi.CFG_STREAMK_SWAPAB,
    "tc_pair_256x128": capi.CFG_PAIR_256x128,
    "tc_pair_128x256": capi.CFG_PAIR_128x256,
    "tc_pair_128x128": capi.CFG_PAIR_128x128,
    "tc_streamk_pair_256x256": capi.CFG_STREAMK_PAIR_256x256,
}


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()


def run_capi(a, b, out, config, split_k=0, flags=0, workspace=True):
    """Calls the C ABI with the workspace it asks for (staging, stream-K,
    split-K exchange), or with none."""
    m, k = a.shape
    n = b.shape[1]
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
                          config=config, split_k=split_k, flags=flags)
    need = capi.workspace_size(args) if workspace else 0
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    if need:
        args.workspace, args.workspace_bytes = ws.data_ptr(), need
    rc = capi.run(args, torch.cuda.current_stream().cuda_stream)
    assert rc == capi.OK, capi.status_string(rc)
    return out


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
def test_reference_stage_markers(impl):
    """Reference tests/test_v6_async.py:88-99 verbatim: exactly 7.75."""
    m, n, k = 129, 136, 160
    a, b, value = oracle.stage_marker_inputs(m, n, k, 32, device="cuda")
    out = hgemm(a, b, implementation=impl)
    torch.testing.assert_close(out, torch.full_like(out, value), rtol=0, atol=0)


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
@pytest.mark.parametrize("kblocks", [1, 2, 3, 4, 5, 6, 7, 9, 13])
@pytest.mark.parametrize("mn", [(129, 136), (8, 300), (256, 512)])
def test_stage_markers_every_ring_depth(impl, kblocks, mn):
    m, n = mn
    a, b, value = oracle.stage_marker_inputs(m, n, 64 * kblocks, 64, device="cuda")
    out = hgemm(a, b, implementation=impl)
    torch.testing.assert_close(out, torch.full_like(out, value), rtol=0, atol=0)


SPLIT_CONFIGS = ["tc_splitk_128x128", "tc_splitk_128x256", "tc_swapab", "tc_generic_128x128"]


@pytest.mark.parametrize("workspace", [True, False], ids=["l2_exchange", "dsmem_push"])
@pytest.mark.parametrize("config", SPLIT_CONFIGS)
@pytest.mark.parametrize("split", [1, 2, 3, 4, 5, 8, 16])
def test_explicit_split_k(config, split, workspace):
    m, n, k = (48, 384, 64 * 17) if config == "tc_swapab" else (200, 260, 64 * 17)
    a, b, value = oracle.stage_marker_inputs(m, n, k, 64, device="cuda")
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    run_capi(a, b, out, CONFIG_IDS[config], split_k=split, workspace=workspace)
    torch.testing.assert_close(out, torch.full_like(out, value), rtol=0, atol=0)
    a, b = seeded_inputs(m, n, k + 5)
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    run_capi(a, b, out, CONFIG_IDS[config], split_k=split, workspace=workspace)
    assert_gate(out, a, b)


@pytest.mark.parametrize("out_f32", [False, True], ids=["fp16", "fp32"])
@pytest.mark.parametrize("config", SPLIT_CONFIGS)
@pytest.mark.parametrize("split", [2, 3, 7, 16])
def test_split_transports_bitwise_equal(config, split, out_f32):
    """Both partial-tile transports sum the same FP32 partials in the same
    rank order: identical bits."""
    m, n, k = (40, 520, 64 * 19) if config == "tc_swapab" else (260, 520, 64 * 19)
    a, b = seeded_inputs(m, n, k)
    dtype = torch.float32 if out_f32 else torch.float16
    flags = capi.FLAG_OUT_F32 if out_f32 else 0
    via_l2 = torch.full((m, n), float("nan"), device="cuda", dtype=dtype)
    via_dsmem = torch.full((m, n), float("nan"), device="cuda", dtype=dtype)
    run_capi(a, b, via_l2, CONFIG_IDS[config], split_k=split, flags=flags, workspace=True)
    run_capi(a, b, via_dsmem, CONFIG_IDS[config], split_k=split, flags=flags, workspace=False)
    assert torch.equal(via_l2, via_dsmem)
    assert_gate(via_l2.half() if out_f32 else via_l2, a, b)


@pytest.mark.parametrize("config", list(CONFIG_IDS))
@pytest.mark.parametrize("shape", [(127, 129, 63), (200, 264, 520), (3, 1000, 300)])
def test_guard_bands_untouched(config, shape):
    m, n, k = shape
    a, b = seeded_inputs(m, n, k)
    pad = 4096
    buf = torch.full((pad + m * n + pad,), 1234.0, device="cuda", dtype=torch.float16)
    out = buf[pad:pad + m * n].view(m, n)
    run_capi(a, b, out, CONFIG_IDS[config])
    torch.cuda.synchronize()
    assert torch.all(buf[:pad] == 1234.0) and torch.all(buf[pad + m * n:] == 1234.0)
    assert_gate(out, a, b)


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
@pytest.mark.parametrize("shape", [(128, 128, 96), (127, 136, 40), (127, 129, 63)])
def test_non_default_stream_preallocated_nan(impl, shape):
    a, b = seeded_inputs(*shape)
    reference = oracle.torch_reference(a.cpu(), b.cpu())
    out = torch.full(shape[:2], float("nan"), device="cuda", dtype=torch.float16)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        returned = _hgemm_out(a, b, out, implementation=impl)
    torch.cuda.current_stream().wait_stream(stream)
    assert returned is out
    metrics = oracle.error_metrics(out.cpu(), reference)
    assert oracle.correctness_passed(metrics), metrics


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
@pytest.mark.parametrize("offset_a,offset_b", [(1, 0), (0, 1), (1, 1)])
def test_misaligned_storage(impl, offset_a, offset_b):
    torch.manual_seed(2026)
    m, n, k = 128, 128, 64
    a_storage = torch.randn(m * k + offset_a, device="cuda", dtype=torch.float16) * 0.1
    b_storage = torch.randn(k * n + offset_b, device="cuda", dtype=torch.float16) * 0.1
    a = a_storage[offset_a:].view(m, k)
    b = b_storage[offset_b:].view(k, n)
    assert a.data_ptr() % 16 == offset_a * 2 and b.data_ptr() % 16 == offset_b * 2
    assert_gate(hgemm(a, b, implementation=impl), a, b)


@pytest.mark.parametrize("config", list(CONFIG_IDS))
def test_misaligned_output(config):
    m, n, k = 70, 136, 72
    a, b = seeded_inputs(m, n, k)
    storage = torch.full((m * n + 1,), float("nan"), device="cuda", dtype=torch.float16)
    out = storage[1:].view(m, n)
    run_capi(a, b, out, CONFIG_IDS[config])
    assert_gate(out, a, b)


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
def test_provider_metadata(impl):
    assert backend_info(impl) == {"algorithm_id": -1, "workspace_bytes": 0}


@pytest.mark.parametrize("impl,shape", [
    ("tc_streamk_128x256", (2048, 2560, 4096)),     # split tail: partial slots + flags
    ("tc_streamk_swapab", (1, 151936, 2560)),
    ("tc_splitk_128x256", (256, 2560, 9728)),        # split-K exchange through the workspace
    ("auto", (2048, 2560, 4096)),
    ("auto", (1, 151936, 2560)),
    ("auto", (8192, 8192, 8192)),                    # whole tiles: none
    ("tc_persistent_128x256", (8192, 8192, 8192)),
])
def test_provider_metadata_per_shape(impl, shape):
    # backend_info with a shape reports the workspace hgemm allocates for an
    # aligned problem of that shape: the same bytes the C ABI asks for.
    m, n, k = shape
    a, b = seeded_inputs(m, n, k)
    out = torch.empty((m, n), device="cuda", dtype=torch.float16)
    cfg = capi.CFG_AUTO if impl == "auto" else CONFIG_IDS[impl]
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, config=cfg)
    info = backend_info(impl, (m, n, k))
    assert info["algorithm_id"] == -1
    assert info["workspace_bytes"] == capi.workspace_size(args)
    if impl.startswith("tc_streamk") or impl == "tc_splitk_128x256":
        assert info["workspace_bytes"] > 0


@pytest.mark.parametrize("config", list(CONFIG_IDS))
def test_fp32_output(config):
    m, n, k = 100, 264, 1000
    a, b = seeded_inputs(m, n, k)
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32)
    run_capi(a, b, out, CONFIG_IDS[config], flags=capi.FLAG_OUT_F32)
    ref = torch.mm(a.cpu().float(), b.cpu().float())
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-4, atol=1e-4)


def test_capi_matches_module_bitwise():
    a, b = seeded_inputs(300, 520, 1000)
    for name, cfg in CONFIG_IDS.items():
        out = torch.empty((300, 520), device="cuda", dtype=torch.float16)
        run_capi(a, b, out, cfg)
        assert torch.equal(out, hgemm(a, b, implementation=name)), name


STAGED_SHAPES = [(300, 1001, 517), (257, 129, 1003), (37, 53, 29), (1, 8193, 70), (513, 131, 264)]


@pytest.mark.parametrize("config", [c for c in CONFIG_IDS if c != "tc_generic_128x128"])
@pytest.mark.parametrize("shape", STAGED_SHAPES)
def test_staged_ragged_operands(config, shape):
    """Pitches that are not multiples of 8 halves: staged through the
    workspace into aligned copies, then the TMA configuration runs."""
    m, n, k = shape
    a, b = seeded_inputs(m, n, k)
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
                          config=CONFIG_IDS[config])
    need = capi.workspace_size(args)
    assert need > 0
    ws = torch.empty(need, device="cuda", dtype=torch.uint8)
    args.workspace, args.workspace_bytes = ws.data_ptr(), need
    rc, cfg, _ = capi.resolve(args)
    # Swap-AB configurations hand M beyond their range to the 128x256 kernels.
    remap = {"tc_swapab": capi.CFG_SPLITK_128x256, "tc_streamk_swapab": capi.CFG_STREAMK_128x256}
    assert rc == capi.OK and cfg in (CONFIG_IDS[config], remap.get(config))
    assert capi.run(args, torch.cuda.current_stream().cuda_stream) == capi.OK
    assert_gate(out, a, b)
    # Without a workspace the same call runs the generic (no-TMA) kernel.
    out2 = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    args2 = capi.make_args(a.data_ptr(), b.data_ptr(), out2.data_ptr(), m, n, k,
                           config=CONFIG_IDS[config])
    rc, cfg, _ = capi.resolve(args2)
    assert cfg == capi.CFG_GENERIC_128x128
    assert capi.run(args2, torch.cuda.current_stream().cuda_stream) == capi.OK
    assert_gate(out2, a, b)


@pytest.mark.parametrize("offsets", [(1, 0, 0), (0, 1, 0), (0, 0, 1), (1, 1, 1), (3, 5, 7)])
def test_staged_offset_views_through_api(offsets):
    """Offset (misaligned) views through the public API: staged, TMA path."""
    oa, ob, oc = offsets
    m, n, k = 200, 264, 520
    torch.manual_seed(5)
    sa = torch.randn(m * k + oa, device="cuda", dtype=torch.float16) * 0.1
    sb = torch.randn(k * n + ob, device="cuda", dtype=torch.float16) * 0.1
    sc = torch.full((m * n + oc,), float("nan"), device="cuda", dtype=torch.float16)
    a, b, out = sa[oa:].view(m, k), sb[ob:].view(k, n), sc[oc:].view(m, n)
    returned = _hgemm_out(a, b, out, implementation="auto")
    assert returned is out
    assert_gate(out, a, b)
    assert torch.all(torch.isnan(sc[:oc])) if oc else True


@pytest.mark.parametrize("shape", [(1, 1, 1), (37, 53, 29), (129, 130, 67), (200, 264, 520), (300, 7, 1000)])
@pytest.mark.parametrize("offsets", [(0, 0, 0), (1, 1, 1), (3, 5, 7)])
def test_generic_nan_guard_bands(shape, offsets):
    """The generic (no-TMA) kernel loads the 16-byte-aligned vectors around
    its operands' elements and shifts them into place: NaN before the first
    element, in the pitch padding of every row and after the last element
    must never reach the result, and no element outside C is written."""
    m, n, k = shape
    oa, ob, oc = offsets
    lda, ldb, ldc = k + 3, n + 5, n + 1
    a_ref, b_ref = seeded_inputs(m, n, k)
    nan = float("nan")
    sa = torch.full((oa + m * lda + 64,), nan, device="cuda", dtype=torch.float16)
    sb = torch.full((ob + k * ldb + 64,), nan, device="cuda", dtype=torch.float16)
    sc = torch.full((oc + m * ldc + 64,), nan, device="cuda", dtype=torch.float16)
    a = sa[oa:oa + m * lda].view(m, lda)
    b = sb[ob:ob + k * ldb].view(k, ldb)
    c = sc[oc:oc + m * ldc].view(m, ldc)
    a[:, :k].copy_(a_ref)
    b[:, :n].copy_(b_ref)
    args = capi.make_args(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, lda=lda, ldb=ldb, ldc=ldc,
                          config=capi.CFG_GENERIC_128x128)
    assert capi.run(args, torch.cuda.current_stream().cuda_stream) == capi.OK
    torch.cuda.synchronize()
    assert_gate(c[:, :n].contiguous(), a_ref, b_ref)
    assert torch.all(torch.isnan(c[:, n:])), "pitch padding of C written"
    assert torch.all(torch.isnan(sc[:oc])) and torch.all(torch.isnan(sc[oc + m * ldc:]))
