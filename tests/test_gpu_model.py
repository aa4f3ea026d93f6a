"""Model-level use of the adapter: a small random-init Qwen3 decoder with
every nn.Linear swapped for FrozenHgemmLinear (reference
benchmarks/bench_integration.py:92-119 qualifies one module at a time; here
all of them), prefill and cached decode against the stock model."""

import argparse
import importlib.util

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
        gate = mc.logits_gate([out], [ref], max_abs=0.05, max_rel_l2=0.01)
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
        gate = mc.logits_gate([out], [ref], max_abs=0.05, max_rel_l2=0.01)
        assert gate["correctness"] == "pass", gate
