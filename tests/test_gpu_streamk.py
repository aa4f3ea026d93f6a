"""Stream-K configurations: whole tiles in waves, then the last (remainder +
one wave) tiles split into equal K ranges, one per CTA; a split tile is
finished by the CTA holding its last K block, which adds the FP32 partial of
the lower-numbered CTA.

Checks exactness (stage markers), the oracle gate over shapes with and
without a split tail (swap-AB and plain), run-to-run determinism, and
CUDA-graph replay (the readiness flags must be reset by every launch)."""

import pytest
import torch

from llm_hgemm import capi, hgemm
from llm_hgemm.ops import _hgemm_out, resolved_config
from oracle import reference as oracle
from tests.gpu_helpers import assert_gate, require_cuda, seeded_inputs

pytestmark = pytest.mark.gpu

SK_SHAPES = [
    # (M, N, K). Swap-AB tiles = ceil(N/128); plain tiles = ceil(M/128)*ceil(N/256).
    (1, 19200, 2560),      # swap: 150 tiles, split tail covers all
    (16, 151936, 2560),    # swap: 1187 tiles, 8 waves + split tail
    (100, 20000, 70),      # swap: 157 tiles, K = 2 blocks (ragged)
    (1, 9728, 2560),       # swap: 76 tiles < SMs, whole tiles only
    (2048, 2560, 4096),    # plain: 160 tiles, all split
    (4736, 1280, 1000),    # plain: 185 tiles, ragged K
    (8192, 5120, 640),     # plain: 1280 tiles, waves + split tail
    (300, 520, 2056),      # plain: 9 tiles < SMs, whole tiles only
]
CONFIGS = {"tc_streamk_128x256": capi.CFG_STREAMK_128x256,
           "tc_streamk_swapab": capi.CFG_STREAMK_SWAPAB,
           "tc_streamk_pair_256x256": capi.CFG_STREAMK_PAIR_256x256}


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()


def capi_run(a, b, out, cfg):
    m, k = a.shape
    n = b.shape[1]
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, config=cfg)
    need = capi.workspace_size(args)
    ws = torch.full((max(need, 1),), 0x5A, device="cuda", dtype=torch.uint8)  # garbage-filled
    args.workspace, args.workspace_bytes = ws.data_ptr(), need
    assert capi.run(args, torch.cuda.current_stream().cuda_stream) == capi.OK
    return need


@pytest.mark.parametrize("config", list(CONFIGS))
@pytest.mark.parametrize("shape", SK_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_streamk_gate_and_determinism(config, shape):
    m, n, k = shape
    if config == "tc_streamk_swapab" and m > 128:
        pytest.skip("swap-AB stream-K covers M <= 128")
    a, b = seeded_inputs(m, n, k)
    out1 = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    out2 = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    capi_run(a, b, out1, CONFIGS[config])
    capi_run(a, b, out2, CONFIGS[config])
    assert_gate(out1, a, b)
    assert torch.equal(out1, out2)


@pytest.mark.parametrize("config,mn", [
    ("tc_streamk_swapab", (1, 19200)), ("tc_streamk_swapab", (16, 151936)),
    ("tc_streamk_128x256", (2048, 2560)), ("tc_streamk_128x256", (8192, 5120)),
    ("tc_streamk_128x256", (4736, 1280)), ("tc_streamk_pair_256x256", (2048, 2560)),
    ("tc_streamk_pair_256x256", (8192, 5120)), ("tc_streamk_pair_256x256", (4736, 1280))])
@pytest.mark.parametrize("kblocks", [1, 2, 45])
def test_streamk_stage_markers(config, mn, kblocks):
    m, n = mn
    a, b, value = oracle.stage_marker_inputs(m, n, 64 * kblocks, 64, device="cuda")
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    need = capi_run(a, b, out, CONFIGS[config])
    assert need > 0   # a split tail (and its workspace) is planned
    torch.testing.assert_close(out, torch.full_like(out, value), rtol=0, atol=0)


@pytest.mark.parametrize("shape", [(1, 19200, 2560), (16, 151936, 640), (2048, 2560, 4096)])
def test_streamk_graph_replay(shape):
    """Replays of one captured launch reuse its epoch: each finisher must see
    the flags its own replay published, never the previous replay's."""
    m, n, k = shape
    a, b = seeded_inputs(m, n, k)
    out = torch.empty((m, n), device="cuda", dtype=torch.float16)
    cfg, _ = resolved_config(a, b, "auto")
    assert cfg.startswith("tc_streamk")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _hgemm_out(a, b, out, implementation="auto")
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _hgemm_out(a, b, out, implementation="auto")
    for seed in (1, 2, 3):
        torch.manual_seed(seed)
        a.copy_(torch.randn_like(a) * 0.1)
        b.copy_(torch.randn_like(b) * 0.1)
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert_gate(out, a, b)


# Few tiles (M <= 512): a cost model chooses among the tile kernels.
TILE_KERNELS = ("tc_swapab", "tc_splitk_128x256")


@pytest.mark.parametrize("shape,expected", [
    ((1, 151936, 2560), ("tc_streamk_swapab",)), ((16, 4096, 2560), ("tc_swapab",)),
    ((2048, 2560, 4096), ("tc_streamk_pair_256x256",)), ((512, 2560, 4096), TILE_KERNELS),
    ((512, 4096, 2560), TILE_KERNELS), ((512, 1024, 2560), TILE_KERNELS),
    ((200, 2560, 9728), TILE_KERNELS), ((8192, 8192, 1024), ("tc_pair_256x256",))])
def test_auto_picks_streamk_when_tiles_fill_the_sms(shape, expected):
    a, b = seeded_inputs(*shape)
    cfg, _ = resolved_config(a, b, "auto")
    assert cfg in expected, (shape, cfg)
    assert_gate(hgemm(a, b), a, b)


@pytest.mark.parametrize("shape", [(2048, 2560, 4096), (4096, 4096, 4096), (8192, 2560, 1000)])
def test_streamk_pair_graph_replay_and_single_launch(shape):
    """The CTA-pair stream-K configuration: a split tail is planned (workspace
    > 0), results pass the gate, match between two eager launches bitwise, and
    replays of one captured launch see their own flags."""
    m, n, k = shape
    a, b = seeded_inputs(m, n, k)
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    need = capi_run(a, b, out, capi.CFG_STREAMK_PAIR_256x256)
    assert need > 0
    assert_gate(out, a, b)
    out2 = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    capi_run(a, b, out2, capi.CFG_STREAMK_PAIR_256x256)
    assert torch.equal(out, out2)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _hgemm_out(a, b, out, implementation="tc_streamk_pair_256x256")
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _hgemm_out(a, b, out, implementation="tc_streamk_pair_256x256")
    for seed in (1, 2):
        torch.manual_seed(seed)
        a.copy_(torch.randn_like(a) * 0.1)
        b.copy_(torch.randn_like(b) * 0.1)
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert_gate(out, a, b)


@pytest.mark.parametrize("shape", [(8192, 2560, 4864), (2100, 2600, 1000), (4096, 8192, 3584)],
                         ids=lambda s: "x".join(map(str, s)))
def test_auto_fp32_output_takes_cta_pairs(shape):
    """FP32 output (the tensor-parallel partials) resolves to the CTA-pair kernels
    from one wave of tiles up, like FP16 output, and matches the FP32 product."""
    from llm_hgemm.ops import hgemm_f32_out

    m, n, k = shape
    a, b = seeded_inputs(m, n, k)
    out = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32)
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, flags=capi.FLAG_OUT_F32)
    rc, cfg, _ = capi.resolve(args)
    assert rc == capi.OK and cfg in (capi.CFG_PAIR_256x256, capi.CFG_STREAMK_PAIR_256x256), (shape, cfg)
    hgemm_f32_out(a, b, out, implementation="auto")
    assert not torch.backends.cuda.matmul.allow_tf32
    ref = a.float() @ b.float()
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
