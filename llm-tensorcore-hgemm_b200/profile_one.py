"""Single-shape driver for Nsight Compute (reference benchmarks/profile_one.py:13-33).

    ncu --clock-control none -k regex:hgemm_ -s <warmup> -c 1 \
        python llm-tensorcore-hgemm_b200/profile_one.py --m 8192 --n 8192 --k 8192

Runs `--warmup` untimed launches and `--iters` launches of one implementation
on seeded inputs (randn*0.1, FP16) and exits; nothing is timed here.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

import torch  # noqa: E402

from llm_hgemm.ops import _hgemm_out, resolved_config  # noqa: E402


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--m", type=int, required=True)
    p.add_argument("--n", type=int, required=True)
    p.add_argument("--k", type=int, required=True)
    p.add_argument("--implementation", default="auto")
    p.add_argument("--provider", choices=["hgemm", "cublaslt"], default="hgemm",
                   help="cublaslt: the benchmark-only comparator on the same inputs")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--seed", type=int, default=2026)
    args = p.parse_args()
    torch.manual_seed(args.seed)
    a = torch.randn((args.m, args.k), device="cuda", dtype=torch.float16) * 0.1
    b = torch.randn((args.k, args.n), device="cuda", dtype=torch.float16) * 0.1
    c = torch.empty((args.m, args.n), device="cuda", dtype=torch.float16)
    if args.provider == "cublaslt":
        from llm_hgemm import _comparators

        for _ in range(args.warmup + args.iters):
            _comparators.cublaslt_out(a, b, c)
        torch.cuda.synchronize()
        print(f"profiled {args.m}x{args.n}x{args.k} cublaslt comparator")
        return
    cfg, split = resolved_config(a, b, args.implementation)
    for _ in range(args.warmup + args.iters):
        _hgemm_out(a, b, c, implementation=args.implementation)
    torch.cuda.synchronize()
    print(f"profiled {args.m}x{args.n}x{args.k} {args.implementation} -> {cfg} split_k={split}")


if __name__ == "__main__":
    main()
