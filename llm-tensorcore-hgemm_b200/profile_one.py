"""Single-shape driver for Nsight Compute (reference benchmarks/profile_one.py:13-33).

    ncu --clock-control none -k regex:hgemm_ -s <warmup> -c 1 \
        python llm-tensorcore-hgemm_b200/profile_one.py --m 8192 --n 8192 --k 8192

Runs `--warmup` untimed launches and `--iters` launches of one implementation
on seeded inputs (randn*0.1, FP16) and exits; nothing is timed here.

`--f32-out` runs the FP32-output GEMM (`hgemm_f32_out`, the tensor-parallel
partials) instead of the FP16 one.

With `--case IMPL:MxNxK` (repeatable) one process runs several shapes in turn,
each with its own inputs, `--warmup` + `--iters` launches (so one `ncu`
command captures every shipped configuration):

    python llm-tensorcore-hgemm_b200/profile_one.py --warmup 2 --iters 1 \
        --case tc_pair_128x128:512x4096x2560 --case tc_splitk_128x256:512x2560x4096
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
    p.add_argument("--m", type=int)
    p.add_argument("--n", type=int)
    p.add_argument("--k", type=int)
    p.add_argument("--case", action="append", default=[], metavar="IMPL:MxNxK",
                   help="implementation and shape; repeatable (replaces --m/--n/--k/--implementation)")
    p.add_argument("--implementation", default="auto")
    p.add_argument("--provider", choices=["hgemm", "cublaslt"], default="hgemm",
                   help="cublaslt: the benchmark-only comparator on the same inputs")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--seed", type=int, default=2026)
    p.add_argument("--f32-out", action="store_true", help="FP32 output (hgemm_f32_out)")
    args = p.parse_args()
    if args.f32_out and args.provider == "cublaslt":
        p.error("--f32-out applies to this library's kernels only")
    if args.case:
        cases = [parse_case(p, case) for case in args.case]   # all checked before any GPU work
        for impl, m, n, k in cases:
            run_one(m, n, k, impl, args.provider, args.warmup, args.iters, args.seed, args.f32_out)
        return
    if args.m is None or args.n is None or args.k is None:
        p.error("--m, --n and --k are required without --case")
    run_one(args.m, args.n, args.k, args.implementation, args.provider, args.warmup, args.iters, args.seed,
            args.f32_out)


def parse_case(parser: argparse.ArgumentParser, case: str) -> tuple[str, int, int, int]:
    """``IMPL:MxNxK`` -> (IMPL, M, N, K); a malformed case is a usage error."""
    impl, sep, shape = case.partition(":")
    dims = shape.lower().split("x")
    if not sep or not impl or len(dims) != 3 or not all(d.isdigit() and int(d) > 0 for d in dims):
        parser.error(f"--case {case!r}: expected IMPL:MxNxK with positive sizes")
    m, n, k = (int(d) for d in dims)
    return impl, m, n, k


def run_one(m: int, n: int, k: int, implementation: str, provider: str, warmup: int, iters: int,
            seed: int, f32_out: bool = False) -> None:
    torch.manual_seed(seed)
    a = torch.randn((m, k), device="cuda", dtype=torch.float16) * 0.1
    b = torch.randn((k, n), device="cuda", dtype=torch.float16) * 0.1
    c = torch.empty((m, n), device="cuda", dtype=torch.float32 if f32_out else torch.float16)
    if provider == "cublaslt":
        from llm_hgemm import _comparators

        for _ in range(warmup + iters):
            _comparators.cublaslt_out(a, b, c)
        torch.cuda.synchronize()
        print(f"profiled {m}x{n}x{k} cublaslt comparator")
        return
    if f32_out:
        from llm_hgemm.ops import hgemm_f32_out

        for _ in range(warmup + iters):
            hgemm_f32_out(a, b, c, implementation=implementation)
        torch.cuda.synchronize()
        print(f"profiled {m}x{n}x{k} {implementation} FP32 output")
    else:
        cfg, split = resolved_config(a, b, implementation)
        for _ in range(warmup + iters):
            _hgemm_out(a, b, c, implementation=implementation)
        torch.cuda.synchronize()
        print(f"profiled {m}x{n}x{k} {implementation} -> {cfg} split_k={split}")
    del a, b, c
    torch.cuda.empty_cache()   # the next case starts from an empty device pool


if __name__ == "__main__":
    main()
