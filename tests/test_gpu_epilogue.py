"""Fused epilogues (bias, residual, SwiGLU silu_mul) of every kernel
configuration against the oracle's FP32 composition
(oracle.reference.torch_reference_epilogue), gated with the reference's
limits (max-abs <= 5e-2, relative L2 <= 5e-3, reference llm_hgemm/reference.py:9-10).

The reference rejects every epilogue but "none" (csrc/dispatch.cpp:52,
tests/test_contract.py:63-66); these extend that argument, so the contract
tests below check the new error paths the same way."""

import pytest
import torch

from llm_hgemm import capi, hgemm
from llm_hgemm.ops import _hgemm_out, interleave_gate_up
from oracle import reference as oracle
from tests.gpu_helpers import IMPLEMENTATIONS, require_cuda, seeded_inputs
from tests.test_gpu_pipeline import CONFIG_IDS

pytestmark = pytest.mark.gpu

EPILOGUES = ["bias", "residual", "bias+residual", "silu_mul", "bias+silu_mul"]


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()


def operands(m, n, seed=11):
    g = torch.Generator(device="cuda").manual_seed(seed)
    bias = (torch.randn((n,), generator=g, device="cuda") * 0.1).half()
    residual = (torch.randn((m, n), generator=g, device="cuda") * 0.1).half()
    return bias, residual


def kwargs_for(epilogue, bias, residual):
    terms = epilogue.split("+")
    return {"bias": bias if "bias" in terms else None, "residual": residual if "residual" in terms else None}


def assert_epilogue_gate(out, a, b, epilogue, bias=None, residual=None):
    ref = oracle.torch_reference_epilogue(a, b, epilogue, bias, residual)
    assert out.shape == ref.shape
    metrics = oracle.error_metrics(out, ref)
    assert oracle.correctness_passed(metrics), metrics
    return metrics


@pytest.mark.parametrize("impl", IMPLEMENTATIONS)
@pytest.mark.parametrize("epilogue", EPILOGUES)
@pytest.mark.parametrize("shape", [(1, 2048, 2560), (16, 1024, 640), (37, 130, 200), (256, 512, 1024),
                                   (1000, 1536, 320)])
def test_epilogue_every_config(impl, epilogue, shape):
    m, n, k = shape
    a, b = seeded_inputs(m, n, k)
    bias, residual = operands(m, n)
    kw = kwargs_for(epilogue, bias, residual)
    out = hgemm(a, b, implementation=impl, epilogue=epilogue, **kw)
    assert_epilogue_gate(out, a, b, epilogue, **kw)


@pytest.mark.parametrize("impl", ["auto", "tc_persistent_128x256", "tc_pair_256x256", "tc_streamk_128x256"])
@pytest.mark.parametrize("epilogue", EPILOGUES)
def test_epilogue_many_tiles(impl, epilogue):
    """Several waves of tiles (persistent, pair and stream-K tails with their
    TMA-store epilogues)."""
    m, n, k = 2048, 4608, 1024
    a, b = seeded_inputs(m, n, k, seed=7)
    bias, residual = operands(m, n, seed=5)
    kw = kwargs_for(epilogue, bias, residual)
    out = hgemm(a, b, implementation=impl, epilogue=epilogue, **kw)
    assert_epilogue_gate(out, a, b, epilogue, **kw)


@pytest.mark.parametrize("workspace", [True, False], ids=["l2_exchange", "dsmem_push"])
@pytest.mark.parametrize("config", ["tc_splitk_128x128", "tc_splitk_128x256", "tc_swapab", "tc_generic_128x128"])
@pytest.mark.parametrize("split", [1, 3, 8])
@pytest.mark.parametrize("epilogue", ["bias+residual", "bias+silu_mul"])
def test_epilogue_explicit_split_k(config, split, workspace, epilogue):
    """The final writer of a split-K tile applies the epilogue once, after the
    fixed-order sum, for both partial-tile transports."""
    m, n, k = (48, 384, 64 * 17) if config == "tc_swapab" else (200, 260, 64 * 17)
    a, b = seeded_inputs(m, n, k)
    bias, residual = operands(m, n)
    kw = kwargs_for(epilogue, bias, residual)
    bits = sum({"bias": capi.EPI_BIAS, "residual": capi.EPI_RESIDUAL, "silu_mul": capi.EPI_SILU_MUL}[t]
               for t in epilogue.split("+"))
    cols = n // 2 if bits & capi.EPI_SILU_MUL else n
    out = torch.full((m, cols), float("nan"), device="cuda", dtype=torch.float16)
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, config=CONFIG_IDS[config],
                          split_k=split, epilogue=bits, bias_ptr=bias.data_ptr(),
                          residual_ptr=residual.data_ptr() if kw["residual"] is not None else None)
    need = capi.workspace_size(args) if workspace else 0
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    if need:
        args.workspace, args.workspace_bytes = ws.data_ptr(), need
    assert capi.run(args, torch.cuda.current_stream().cuda_stream) == capi.OK
    assert_epilogue_gate(out, a, b, epilogue, **kw)


@pytest.mark.parametrize("impl", ["auto", "tc_swapab", "tc_streamk_swapab", "tc_splitk_128x128",
                                  "tc_persistent_128x256", "tc_pair_256x128"])
def test_residual_in_place(impl):
    """residual may be the output itself: out = A @ B + out."""
    m, n, k = 96, 768, 512
    a, b = seeded_inputs(m, n, k)
    _, residual = operands(m, n)
    expect = oracle.torch_reference_epilogue(a, b, "residual", residual=residual)
    out = residual.clone()
    _hgemm_out(a, b, out, implementation=impl, epilogue="residual", residual=out)
    metrics = oracle.error_metrics(out, expect)
    assert oracle.correctness_passed(metrics), metrics


@pytest.mark.parametrize("impl", ["auto", "tc_swapab", "tc_persistent_128x128", "tc_generic_128x128"])
def test_unaligned_epilogue_operands(impl):
    """Bias at a 2-byte offset and a residual whose pitch is not a multiple of
    8 take the element-wise path."""
    m, n, k = 70, 264, 136
    a, b = seeded_inputs(m, n, k)
    g = torch.Generator(device="cuda").manual_seed(3)
    bias_buf = (torch.randn((n + 1,), generator=g, device="cuda") * 0.1).half()
    res_buf = (torch.randn((m, n + 3), generator=g, device="cuda") * 0.1).half()
    bias, residual = bias_buf[1:], res_buf[:, :n]
    out = hgemm(a, b, implementation=impl, epilogue="bias+residual", bias=bias, residual=residual)
    assert_epilogue_gate(out, a, b, "bias+residual", bias=bias, residual=residual)


def test_swiglu_matches_unfused_layers():
    """silu_mul over interleaved [gate | up] columns equals the unfused
    silu(x @ Wg) * (x @ Wu) of a Qwen3 MLP up to the unfused path's
    intermediate FP16 roundings."""
    m, k, inter = 64, 2560, 9728
    g = torch.Generator(device="cuda").manual_seed(2026)
    x = (torch.randn((m, k), generator=g, device="cuda") * 0.1).half()
    wg = (torch.randn((k, inter), generator=g, device="cuda") * 0.02).half()
    wu = (torch.randn((k, inter), generator=g, device="cuda") * 0.02).half()
    fused = hgemm(x, interleave_gate_up(wg, wu), epilogue="silu_mul")
    unfused = torch.nn.functional.silu(hgemm(x, wg).float()) * hgemm(x, wu).float()
    metrics = oracle.error_metrics(fused, unfused.half())
    assert oracle.correctness_passed(metrics), metrics


def test_epilogue_contract():
    a, b = seeded_inputs(32, 64, 48)
    bias, residual = operands(32, 64)
    with pytest.raises(RuntimeError, match="epilogue"):
        hgemm(a, b, epilogue="gelu")
    with pytest.raises(RuntimeError, match="epilogue"):
        hgemm(a, b, epilogue="bias+bias", bias=bias)
    with pytest.raises(RuntimeError, match="needs a bias"):
        hgemm(a, b, epilogue="bias")
    with pytest.raises(RuntimeError, match="needs a residual"):
        hgemm(a, b, epilogue="residual")
    with pytest.raises(RuntimeError, match="has no bias term"):
        hgemm(a, b, bias=bias)
    with pytest.raises(RuntimeError, match="does not combine"):
        hgemm(a, b, epilogue="residual+silu_mul", residual=residual)
    with pytest.raises(RuntimeError, match="bias must be a contiguous"):
        hgemm(a, b, epilogue="bias", bias=bias[:32])
    with pytest.raises(RuntimeError, match="bias must have dtype"):
        hgemm(a, b, epilogue="bias", bias=bias.float())
    with pytest.raises(RuntimeError, match="residual must be a"):
        hgemm(a, b, epilogue="residual", residual=residual.t().contiguous().t())
    a2, b2 = seeded_inputs(32, 63, 48)
    with pytest.raises(RuntimeError, match="even N"):
        hgemm(a2, b2, epilogue="silu_mul")
    out = torch.empty((32, 64), device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match=r"out must have shape \[32, 32\]"):
        _hgemm_out(a, b, out, implementation="auto", epilogue="silu_mul")
