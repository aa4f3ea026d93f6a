"""Model-level check: a random-init Qwen3-4B-architecture decoder with every
``nn.Linear`` swapped for ``FrozenHgemmLinear``, against the stock model.

Counterpart of the reference's model qualification
(benchmarks/bench_integration.py:18-119: prefill and cached decode rollouts,
``logits_gate`` with max-abs 0.05 and relative L2 0.001). No checkpoint is
available here, so the weights are the architecture's own random init
(normal, std 0.02) from a fixed seed; token ids are seeded random integers.

    python llm-tensorcore-hgemm_b200/model_check.py            # Qwen3-4B sizes
    python llm-tensorcore-hgemm_b200/model_check.py --layers 2 --hidden 256 ...

Prints one JSON line: for prefill (batch 1 x 2048 tokens, last-token logits)
and cached decode (batch 16, one token at context 2048), the logits gate of
the swapped model against the stock model and both models' device times. The
gate result is reported whether it passes or not. Unless ``--no-fused``, a
second copy of the model (same seed) with fused q|k|v and gate|up
projections (``fuse_projections``) is checked and timed the same way.

Unless ``--no-fp32``, the same seeded weights are also run as an FP32 model
(every operation in FP32, TF32 off): the logit error of the stock FP16 model
(cuBLAS) against it is the FP16-propagation floor, and the swapped and fused
models' errors against it are reported beside it. Two FP16 models whose GEMMs
round differently drift apart through 36 layers even when each GEMM is within
its own tolerance; the floor shows how far the stock FP16 model itself sits
from the FP32 result.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

import torch  # noqa: E402

MAX_LOGIT_ABS = 0.05        # reference benchmarks/bench_integration.py:132
MAX_LOGIT_REL_L2 = 0.001    # reference benchmarks/bench_integration.py:133


def logits_gate(actual: list[torch.Tensor], expected: list[torch.Tensor],
                max_abs: float = MAX_LOGIT_ABS, max_rel_l2: float = MAX_LOGIT_REL_L2) -> dict:
    """Largest max-abs and relative-L2 logit error over the rollout's steps
    (reference bench_integration.py:47-70): a missing or empty trace and a
    shape mismatch are errors, not passes; a non-finite logit on either side
    fails the gate and reports no error figures."""
    if not actual or len(actual) != len(expected):
        raise ValueError("empty or different-length logits traces")
    steps = []
    for i, (a, e) in enumerate(zip(actual, expected)):
        if a.shape != e.shape:
            raise ValueError(f"step {i}: logits shapes {tuple(a.shape)} and {tuple(e.shape)} differ")
        a32, e32 = a.float(), e.float()
        finite = bool(torch.isfinite(a32).all()) and bool(torch.isfinite(e32).all())
        err_abs = err_rel = None
        if finite:
            d = a32 - e32
            err_abs = float(d.abs().max())
            err_rel = float(torch.linalg.vector_norm(d) / torch.linalg.vector_norm(e32).clamp_min(1e-12))
        steps.append({"step": i, "finite": finite, "max_abs": err_abs, "relative_l2": err_rel})
    finite = all(s["finite"] for s in steps)
    worst_abs = max(s["max_abs"] for s in steps) if finite else None
    worst_rel = max(s["relative_l2"] for s in steps) if finite else None
    ok = finite and worst_abs <= max_abs and worst_rel <= max_rel_l2
    return {"correctness": "pass" if ok else "fail", "logits_finite": finite,
            "logits_max_abs_error": worst_abs, "logits_max_relative_l2_error": worst_rel,
            "logits_per_step_errors": steps,
            "max_abs_limit": max_abs, "max_relative_l2_limit": max_rel_l2}


def build_model(args):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(
        vocab_size=args.vocab, hidden_size=args.hidden, intermediate_size=args.intermediate,
        num_hidden_layers=args.layers, num_attention_heads=args.heads,
        num_key_value_heads=args.kv_heads, head_dim=args.head_dim, rms_norm_eps=1e-6,
        rope_theta=1_000_000.0, max_position_embeddings=max(40960, args.context + 16),
        tie_word_embeddings=True, attention_bias=False, initializer_range=0.02)
    torch.manual_seed(args.seed)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM(cfg).to(torch.float16).eval()
    return model


def timed(fn):
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    out = fn()
    e.record()
    e.synchronize()
    return out, s.elapsed_time(e)


@torch.inference_mode()
def rollout(model, prompt, decode_prompts, decode_next):
    """Last-token logits of a prefill, and decode-step logits for a batch of
    sequences after a cached prefill of `decode_prompts`, with their device
    times (milliseconds)."""
    pre, t_pre = timed(lambda: model(prompt, logits_to_keep=1).logits[:, -1].clone())
    cache = model(decode_prompts, use_cache=True, logits_to_keep=1).past_key_values
    torch.cuda.synchronize()
    # Five decode steps (the same next tokens, the cache growing by one each
    # time); the first step's logits are compared, the median step time kept.
    dec, times = None, []
    for _ in range(5):
        out, t = timed(lambda: model(decode_next, past_key_values=cache, use_cache=True,
                                     logits_to_keep=1).logits[:, -1].clone())
        dec = out if dec is None else dec
        times.append(t)
    del cache
    return pre, dec, t_pre, sorted(times)[len(times) // 2]


def fp32_rollout(args, prompt, decode_prompts, decode_next):
    """Rollout of the same seeded model in FP32 (weights upcast exactly from
    the FP16 init, TF32 off for matmuls and convolutions)."""
    model = build_model(args).float()
    saved = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        pre, dec, _, _ = rollout(model, prompt, decode_prompts, decode_next)
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = saved
    del model
    torch.cuda.empty_cache()
    return pre, dec


def errors_vs(actual: torch.Tensor, expected: torch.Tensor) -> dict:
    """Max-abs and relative-L2 error of one logits tensor against another."""
    g = logits_gate([actual], [expected])
    return {"max_abs": g["logits_max_abs_error"], "relative_l2": g["logits_max_relative_l2_error"]}


def check(args) -> dict:
    """Runs the model check described in the module docstring; returns the
    result dictionary (what ``main`` prints)."""
    from llm_hgemm.integration import FrozenHgemmLinear, HgemmSwiGLU, fuse_projections, swap_linears

    model = build_model(args)
    g = torch.Generator(device="cuda").manual_seed(args.seed + 1)
    prompt = torch.randint(0, args.vocab, (1, args.prefill_tokens), device="cuda", generator=g)
    decode_prompts = torch.randint(0, args.vocab, (args.decode_batch, args.context), device="cuda",
                                   generator=g)
    decode_next = torch.randint(0, args.vocab, (args.decode_batch, 1), device="cuda", generator=g)

    rollout(model, prompt, decode_prompts, decode_next)   # warm-up at full size
    ref_pre, ref_dec, t_pre_ref, t_dec_ref = rollout(model, prompt, decode_prompts, decode_next)

    swapped = swap_linears(model, args.implementation)
    adapters = [m for m in model.modules() if isinstance(m, FrozenHgemmLinear)]
    rollout(model, prompt, decode_prompts, decode_next)   # warm-up at full size
    out_pre, out_dec, t_pre, t_dec = rollout(model, prompt, decode_prompts, decode_next)
    backends = sorted({str(m.last_backend) for m in adapters})

    fused_result = None
    f_pre = f_dec = None
    if not args.no_fused:
        # The same seeded weights, with fused q|k|v and gate|up (silu_mul
        # epilogue) projections; the remaining linears through FrozenHgemmLinear.
        del model
        torch.cuda.empty_cache()
        model = build_model(args)
        counts = fuse_projections(model, args.implementation)
        counts["linears"] = swap_linears(model, args.implementation)
        rollout(model, prompt, decode_prompts, decode_next)   # warm-up at full size
        f_pre, f_dec, tf_pre, tf_dec = rollout(model, prompt, decode_prompts, decode_next)
        fused_backends = sorted({str(m.last_backend) for m in model.modules()
                                 if isinstance(m, (FrozenHgemmLinear, HgemmSwiGLU))})
        fused_result = {
            "fused": counts, "executed_backends": fused_backends,
            "prefill": {**logits_gate([f_pre], [ref_pre]), "hgemm_ms": round(tf_pre, 3)},
            "decode": {**logits_gate([f_dec], [ref_dec]), "hgemm_ms": round(tf_dec, 3)},
        }
    del model
    torch.cuda.empty_cache()

    floor = None
    if not args.no_fp32:
        p32, d32 = fp32_rollout(args, prompt, decode_prompts, decode_next)
        floor = {"reference": "the same seeded weights in FP32 (TF32 off)"}
        for name, (pre, dec) in (("stock_fp16", (ref_pre, ref_dec)), ("hgemm_fp16", (out_pre, out_dec)),
                                 ("hgemm_fused_fp16", (f_pre, f_dec))):
            if pre is not None:
                floor[name] = {"prefill": errors_vs(pre, p32), "decode": errors_vs(dec, d32)}

    return {
        "model": "Qwen3-4B architecture, random init (std 0.02), FP16",
        "layers": args.layers, "hidden": args.hidden, "vocab": args.vocab,
        "linears_swapped": swapped, "executed_backends": backends,
        "implementation": args.implementation,
        "prefill": {"tokens": args.prefill_tokens, **logits_gate([out_pre], [ref_pre]),
                    "stock_ms": round(t_pre_ref, 3), "hgemm_ms": round(t_pre, 3)},
        "decode": {"batch": args.decode_batch, "context": args.context,
                   **logits_gate([out_dec], [ref_dec]),
                   "stock_ms": round(t_dec_ref, 3), "hgemm_ms": round(t_dec, 3)},
        "fused_projections": fused_result,
        "fp32_floor": floor,
    }


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--layers", type=int, default=36)
    p.add_argument("--hidden", type=int, default=2560)
    p.add_argument("--intermediate", type=int, default=9728)
    p.add_argument("--heads", type=int, default=32)
    p.add_argument("--kv-heads", type=int, default=8)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--vocab", type=int, default=151936)
    p.add_argument("--prefill-tokens", type=int, default=2048)
    p.add_argument("--decode-batch", type=int, default=16)
    p.add_argument("--context", type=int, default=2048)
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--implementation", default="auto")
    p.add_argument("--no-fused", action="store_true",
                   help="skip the fused-projection variant (second model copy)")
    p.add_argument("--no-fp32", action="store_true",
                   help="skip the FP32 model (the FP16-propagation floor)")
    return p


def main() -> None:
    print(json.dumps(check(parser().parse_args())), flush=True)


if __name__ == "__main__":
    main()
