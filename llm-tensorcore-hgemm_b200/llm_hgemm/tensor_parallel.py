"""Tensor-parallel MLP GEMMs over one node (one process per GPU, NCCL).

The reference is single-GPU; this is the multi-GPU configuration of the
hot path: large MLP GEMMs split where they shard naturally.

* Up-projection, column parallel: rank r holds W_up[:, r*N/G:(r+1)*N/G] and
  computes Y_r = X @ W_up_r with the same kernels; no communication, the
  output stays sharded on N.
* Down-projection, row parallel: rank r holds H[:, Kslice_r] and
  W_down[Kslice_r, :] and computes the FP32 partial P_r (the GEMM's FP32
  epilogue, no rounding); ``all_reduce(SUM)`` over NCCL adds the partials in
  FP32 and one conversion rounds the sum to FP16. That matches the oracle's
  FP32 accumulation followed by a single FP16 rounding.

Operands are always local to each GPU; data crosses NVLink only inside NCCL.
The GEMM callables are injectable so the partitioning and reduction logic
runs on CPU ranks (gloo) in tests.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


def shard_bounds(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, near-equal split of ``total`` (the first ``total % world``
    ranks get one more); raises when a rank would get nothing."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if total < world:
        raise ValueError(f"cannot split {total} over {world} ranks")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_columns(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    lo, hi = shard_bounds(w.shape[1], rank, world)
    return w[:, lo:hi].contiguous()


def shard_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    lo, hi = shard_bounds(w.shape[0], rank, world)
    return w[lo:hi].contiguous()


def _cuda_gemm(a, b, out):
    from .ops import _hgemm_out

    return _hgemm_out(a, b, out, implementation="auto")


def _cuda_gemm_f32(a, b, out):
    from .ops import hgemm_f32_out

    return hgemm_f32_out(a, b, out, implementation="auto")


@dataclass
class TensorParallelMLP:
    x: torch.Tensor          # [M, hidden] FP16, replicated
    w_up: torch.Tensor       # [hidden, inter/G] FP16, this rank's column shard
    h: torch.Tensor          # [M, inter/G] FP16, this rank's column shard of H
    w_down: torch.Tensor     # [inter/G, hidden] FP16, this rank's row shard
    rank: int = 0
    world: int = 1
    group: object = None
    gemm: Callable = _cuda_gemm
    gemm_f32: Callable = _cuda_gemm_f32
    inter_total: int | None = None

    def __post_init__(self):
        m = self.x.shape[0]
        if self.inter_total is None:
            # Every rank constructs the module, so this collective is matched.
            t = torch.tensor([self.w_up.shape[1]], dtype=torch.int64,
                             device=self.x.device if self.x.is_cuda else "cpu")
            if self.world > 1:
                dist.all_reduce(t, group=self.group)
            self.inter_total = int(t.item())
        self.y = torch.empty((m, self.w_up.shape[1]), device=self.x.device, dtype=torch.float16)
        self.partial = torch.empty((m, self.w_down.shape[1]), device=self.x.device,
                                   dtype=torch.float32)
        self.out = torch.empty((m, self.w_down.shape[1]), device=self.x.device,
                               dtype=torch.float16)

    @classmethod
    def synthetic(cls, rank: int, world: int, *, seed: int = 2026, device="cuda", m: int = 8192,
                  hidden: int = 8192, inter: int = 28672, **kwargs) -> "TensorParallelMLP":
        """Seeded identically on every rank (configs[4]: activations randn*0.1,
        weights randn*0.02), then sharded."""
        g = torch.Generator(device=device).manual_seed(seed)

        def rnd(shape, scale):
            return (torch.randn(shape, generator=g, device=device, dtype=torch.float32)
                    * scale).half()

        x = rnd((m, hidden), 0.1)
        w_up_full = rnd((hidden, inter), 0.02)
        w_up = shard_columns(w_up_full, rank, world)
        del w_up_full
        h_full = rnd((m, inter), 0.1)
        h = shard_columns(h_full, rank, world)
        del h_full
        w_down_full = rnd((inter, hidden), 0.02)
        w_down = shard_rows(w_down_full, rank, world)
        del w_down_full
        if torch.device(device).type == "cuda":
            torch.cuda.empty_cache()
        return cls(x, w_up, h, w_down, rank, world, inter_total=inter, **kwargs)

    # ---------------------------------------------------------------- steps
    def up(self) -> torch.Tensor:
        return self.gemm(self.x, self.w_up, self.y)

    def down(self) -> torch.Tensor:
        self.gemm_f32(self.h, self.w_down, self.partial)
        if self.world > 1:
            dist.all_reduce(self.partial, op=dist.ReduceOp.SUM, group=self.group)
        self.out.copy_(self.partial)          # the single FP16 rounding
        return self.out

    def step(self) -> None:
        self.up()
        self.down()

    def total_flops(self) -> float:
        """FLOPs of both full (unsharded) GEMMs; no communication."""
        m, hidden = self.x.shape
        return 2.0 * m * hidden * float(self.inter_total) * 2.0

    def time_gemms(self, steps: int, warmup: int) -> float:
        """Milliseconds per step of the two local GEMMs alone (CUDA events)."""
        for _ in range(warmup):
            self.gemm(self.x, self.w_up, self.y)
            self.gemm_f32(self.h, self.w_down, self.partial)
        torch.cuda.synchronize()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            self.gemm(self.x, self.w_up, self.y)
            self.gemm_f32(self.h, self.w_down, self.partial)
        e.record()
        e.synchronize()
        return s.elapsed_time(e) / steps

    def check(self, rows: int = 64) -> bool:
        """Checks sampled rows of this rank's up-proj shard and of the reduced
        down-proj output against FP32 (TF32 off) products of the same data,
        with the reference's gate (max-abs 5e-2, relative L2 5e-3)."""
        saved = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            self.step()
            idx = torch.arange(0, self.x.shape[0], max(1, self.x.shape[0] // rows),
                               device=self.x.device)[:rows]
            ref_y = (self.x[idx].float() @ self.w_up.float()).half()
            part = self.h[idx].float() @ self.w_down.float()
            if self.world > 1:
                dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
            ref_out = part.half()
        finally:
            torch.backends.cuda.matmul.allow_tf32 = saved

        def gate(out, ref):
            d = out.float() - ref.float()
            rel = torch.linalg.vector_norm(d) / torch.linalg.vector_norm(ref.float()).clamp_min(1e-12)
            return bool(torch.isfinite(out.float()).all()) and d.abs().max().item() <= 5e-2 \
                and rel.item() <= 5e-3

        return gate(self.y[idx], ref_y) and gate(self.out[idx], ref_out)
