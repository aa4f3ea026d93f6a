"""Model-level use of the adapter: a small random-init Qwen3 decoder with
every nn.Linear swapped for FrozenHgemmLinear (reference
benchmarks/bench_integration.py:92-119 qualifies one module at a time; here
all of them), prefill and cached decode against the stock model."""

import argparse
import importlib.util
import json
import os

import pytest
import torch

from tests.conftest import PKG
from tests.gpu_helpers import require_cuda

pytestmark = pytest.mark.gpu


def load_model_check():
    spec = importlib.util.spec_from_file_location("model_check", PKG / "model_check.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_small_qwen3_swapped_matches_stock():
    require_cuda()
    mc = load_model_check()
    from llm_hgemm.integration import FrozenHgemmLinear, swap_linears

    args = argparse.Namespace(vocab=1000, hidden=256, intermediate=704, layers=2, heads=4,
                              kv_heads=2, head_dim=64, context=64, seed=3)
    model = mc.build_model(args)
    g = torch.Generator(device="cuda").manual_seed(4)
    prompt = torch.randint(0, 1000, (1, 96), device="cuda", generator=g)
    dprompts = torch.randint(0, 1000, (4, 64), device="cuda", generator=g)
    dnext = torch.randint(0, 1000, (4, 1), device="cuda", generator=g)
    ref_pre, ref_dec, _, _ = mc.rollout(model, prompt, dprompts, dnext)
    n = swap_linears(model, "auto")
    assert n == 2 * 7 + 1              # q, k, v, o, gate, up, down per layer + lm_head
    out_pre, out_dec, _, _ = mc.rollout(model, prompt, dprompts, dnext)
    adapters = [m for m in model.modules() if isinstance(m, FrozenHgemmLinear)]
    assert all(m.last_backend == "auto" for m in adapters)
    for out, ref in ((out_pre, ref_pre), (out_dec, ref_dec)):
        gate = mc.logits_gate([out], [ref])        # the reference's limits: 0.05, 1e-3
        assert gate["correctness"] == "pass", gate


def test_small_qwen3_fused_projections_match_stock():
    """fuse_projections: one q|k|v GEMM per attention block, gate|up through
    the silu_mul epilogue, then every remaining linear swapped."""
    require_cuda()
    mc = load_model_check()
    from llm_hgemm.integration import FusedQKV, HgemmSwiGLU, fuse_projections, swap_linears

    args = argparse.Namespace(vocab=1000, hidden=256, intermediate=704, layers=2, heads=4,
                              kv_heads=2, head_dim=64, context=64, seed=3)
    model = mc.build_model(args)
    g = torch.Generator(device="cuda").manual_seed(4)
    prompt = torch.randint(0, 1000, (1, 96), device="cuda", generator=g)
    dprompts = torch.randint(0, 1000, (4, 64), device="cuda", generator=g)
    dnext = torch.randint(0, 1000, (4, 1), device="cuda", generator=g)
    ref_pre, ref_dec, _, _ = mc.rollout(model, prompt, dprompts, dnext)
    counts = fuse_projections(model, "auto")
    assert counts == {"qkv": 2, "mlp": 2}
    assert swap_linears(model, "auto") == 2 * 1 + 1     # o_proj per layer + lm_head
    fused = [m for m in model.modules() if isinstance(m, FusedQKV)]
    out_pre, out_dec, _, _ = mc.rollout(model, prompt, dprompts, dnext)
    # One q|k|v GEMM per block per forward; a rollout is seven forwards
    # (prefill, decode-context prefill, five decode steps).
    assert all(m.launches == 7 for m in fused), [m.launches for m in fused]
    assert all(m.last_backend == "auto" for m in model.modules() if isinstance(m, HgemmSwiGLU))
    for out, ref in ((out_pre, ref_pre), (out_dec, ref_dec)):
        gate = mc.logits_gate([out], [ref])        # the reference's limits: 0.05, 1e-3
        assert gate["correctness"] == "pass", gate


def test_qwen3_4b_full_model_logits():
    """the 36-layer random-init Qwen3-4B-architecture
    decoder, prefill 1 x 2048 and decode 16 x 1 at context 2048, every linear
    swapped (and, second copy, q|k|v and gate|up fused), against the stock
    model with the reference's logits gate (max-abs 0.05, relative L2 1e-3,
    benchmarks/bench_integration.py:132-133), and against the same weights
    run in FP32 beside the stock FP16 model (the FP16-propagation floor).

    Hard requirements: finite logits, max-abs within 0.05, and an error
    against the FP32 model no larger than 1.25x the stock cuBLAS model's (the
    kernels add no error beyond what every FP16 model has). The reference's
    relative-L2 gate is evaluated as it is and its outcome recorded: when it
    fails (as it did for the reference's own kernels) the test is marked
    xfail with the numbers. With HGEMM_MODEL_CHECK_OUT set, the full result
    is written there as JSON."""
    require_cuda()
    mc = load_model_check()
    res = mc.check(mc.parser().parse_args([]))
    out_path = os.environ.get("HGEMM_MODEL_CHECK_OUT")
    if out_path:
        with open(out_path, "w") as f:
            json.dump(res, f, indent=1)
    floor = res["fp32_floor"]
    variants = {"swapped": (res["prefill"], res["decode"], floor["hgemm_fp16"]),
                "fused": (res["fused_projections"]["prefill"], res["fused_projections"]["decode"],
                          floor["hgemm_fused_fp16"])}
    failed = []
    for name, (pre, dec, vs32) in variants.items():
        for step, gate in (("prefill", pre), ("decode", dec)):
            assert gate["logits_finite"], (name, step, gate)
            assert gate["logits_max_abs_error"] <= mc.MAX_LOGIT_ABS, (name, step, gate)
            ours, stock = vs32[step]["relative_l2"], floor["stock_fp16"][step]["relative_l2"]
            assert ours <= 1.25 * stock, (name, step, ours, stock)
            if gate["correctness"] != "pass":
                failed.append(f"{name} {step}: rel-L2 {gate['logits_max_relative_l2_error']:.2e} vs stock "
                              f"(stock FP16 vs FP32 {stock:.2e}, ours vs FP32 {ours:.2e})")
    if failed:
        pytest.xfail("reference logits gate (relative L2 1e-3) fails: " + "; ".join(failed))
