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

* Down-projection, reduce-scatter (``down_scatter``): the same FP32 partials,
  but ``reduce_scatter`` leaves each rank only its share of the output rows,
  summed in FP32 and rounded once to an FP16 shard: half the bytes of the
  all-reduce cross NVLink and each rank rounds M / G rows. With ``chunks`` >
  1 the partial is computed in row blocks and block i is reduce-scattered on
  a side stream while block i + 1 is computed (NCCL overlaps the GEMM). Rank
  r then owns, of every block of M / chunks rows, the r-th 1 / G of it
  (:meth:`TensorParallelMLP.owned_rows`), stored block after block.

* Down-projection, fused GEMM + reduce-scatter (``down_p2p``): the FP32
  partial never lands in this GPU's memory as a whole. The GEMM's epilogue
  stores each output row straight into the receive buffer of the rank that
  owns it (peer stores over NVLink, tile by tile while later tiles compute;
  ``hgemm_sm100_run_scatter``); one NCCL barrier orders every rank's GEMM
  before the owners sum their G slots in rank order and round once
  (``hgemm_sm100_reduce_slots``). Receive buffers are this library's own
  device allocations, mapped into the peers through CUDA IPC, two per rank
  used alternately so a rank's next GEMM never overwrites slots its peer is
  still reducing. Rank r owns rows [r * M / G, (r + 1) * M / G).

Operands of the GEMMs are always local to each GPU; data crosses NVLink in
NCCL and, for ``down_p2p``, in the GEMM epilogue's stores (no kernel loads a
peer's memory). The GEMM callables are injectable so the partitioning and
reduction logic runs on CPU ranks (gloo) in tests.
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


class RowScatter:
    """Receive buffers of the fused GEMM + reduce-scatter for one process
    group: two local buffers of FP32 [G, rows_per_rank, cols] (allocated by
    the kernel library, shareable through CUDA IPC) and every peer's two,
    mapped here. Construction and :meth:`close` are collective."""

    def __init__(self, rows_per_rank: int, cols: int, rank: int, world: int, group=None):
        from . import capi

        if world > capi.MAX_RANKS:
            raise ValueError(f"at most {capi.MAX_RANKS} ranks")
        self.rows_per_rank, self.cols, self.rank, self.world, self.group = rows_per_rank, cols, rank, world, group
        nbytes = world * rows_per_rank * cols * 4
        # Two slot buffers (alternate steps) and the FP16 [M, cols] output
        # that the all-gather fills on every rank.
        self.local = [capi.alloc_shared(nbytes) for _ in range(2)]
        self.local.append(capi.alloc_shared(world * rows_per_rank * cols * 2))
        handles = [capi.ipc_handle(p) for p in self.local]
        gathered = [None] * world
        if world > 1:
            dist.all_gather_object(gathered, handles, group=group)
        else:
            gathered[0] = handles
        self.opened = []
        self.dest = []          # dest[b][q]: slot buffer b of rank q; dest[2][q]: output of rank q
        for b in range(3):
            row = []
            for q in range(world):
                if q == rank:
                    row.append(self.local[b])
                else:
                    ptr = capi.ipc_open(gathered[q][b])
                    self.opened.append(ptr)
                    row.append(ptr)
            self.dest.append(row)
        device = torch.device("cuda", torch.cuda.current_device())
        self.output = torch.as_tensor(capi.DeviceArray(self.local[2], (world * rows_per_rank, cols), "<f2"),
                                      device=device)
        self.steps = 0

    def close(self) -> None:
        from . import capi

        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)     # no peer still writes into our buffers
        for ptr in self.opened:
            capi.ipc_close(ptr)
        self.opened = []
        if self.world > 1:
            dist.barrier(group=self.group)     # every peer has unmapped them
        self.output = None
        for ptr in self.local:
            capi.free_shared(ptr)
        self.local = []


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
    down_mode: str = "all_reduce"     # or "p2p" (fused peer-memory path, CUDA only)

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
        """Row-parallel down-projection with the full FP16 output on every
        rank. ``down_mode`` "all_reduce": FP32 partial, NCCL all-reduce, one
        rounding; "p2p": the fused peer-memory path (:meth:`down_p2p` with
        the all-gather), the same value summed in rank order. With one rank
        the GEMM writes the FP16 output itself."""
        if self.world == 1:
            # One rank: nothing to reduce. The GEMM's own epilogue gives the
            # same value (the FP32 sum of the K blocks, rounded once).
            if self.out is getattr(getattr(self, "scatter", None), "output", None):
                self.out = torch.empty_like(self.out)
            return self.gemm(self.h, self.w_down, self.out)
        if self.down_mode == "p2p":
            self.out = self.down_p2p(gather=True)
            return self.out
        return self.down_all_reduce()

    def down_all_reduce(self) -> torch.Tensor:
        """FP32 partial, NCCL all-reduce (SUM), one FP16 rounding."""
        self.gemm_f32(self.h, self.w_down, self.partial)
        if self.world > 1:
            dist.all_reduce(self.partial, op=dist.ReduceOp.SUM, group=self.group)
        if self.out is getattr(getattr(self, "scatter", None), "output", None):
            self.out = torch.empty_like(self.out)       # leave the p2p output alone
        self.out.copy_(self.partial)          # the single FP16 rounding
        return self.out

    def owned_rows(self, chunks: int = 1) -> torch.Tensor:
        """Global output rows of this rank's :meth:`down_scatter` shard, in
        shard order."""
        m = self.x.shape[0]
        if chunks < 1 or m % (chunks * self.world) != 0:
            raise ValueError(f"M={m} must split into {chunks} blocks of {self.world} equal row groups")
        block, part = m // chunks, m // (chunks * self.world)
        return torch.cat([torch.arange(c * block + self.rank * part, c * block + (self.rank + 1) * part)
                          for c in range(chunks)])

    def down_scatter(self, chunks: int = 1) -> torch.Tensor:
        """Row-parallel down-projection with a reduce-scatter: returns this
        rank's FP16 [M / G, hidden] shard (rows :meth:`owned_rows`)."""
        m, hidden = self.partial.shape
        rows = self.owned_rows(chunks)          # validates the split
        block, part = m // chunks, rows.numel() // chunks
        if getattr(self, "shard_f32", None) is None or self.shard_f32.shape[0] != rows.numel():
            self.shard_f32 = torch.empty((rows.numel(), hidden), device=self.x.device, dtype=torch.float32)
            self.shard = torch.empty((rows.numel(), hidden), device=self.x.device, dtype=torch.float16)
        use_side = self.x.is_cuda and chunks > 1
        if use_side and getattr(self, "comm_stream", None) is None:
            self.comm_stream = torch.cuda.Stream(device=self.x.device)
        main = torch.cuda.current_stream(self.x.device) if self.x.is_cuda else None
        for c in range(chunks):
            lo, hi = c * block, (c + 1) * block
            self.gemm_f32(self.h[lo:hi], self.w_down, self.partial[lo:hi])
            dst, src = self.shard_f32[c * part:(c + 1) * part], self.partial[lo:hi]
            if self.world == 1:
                dst.copy_(src)
            elif use_side:
                self.comm_stream.wait_stream(main)
                with torch.cuda.stream(self.comm_stream):
                    dist.reduce_scatter_tensor(dst, src, op=dist.ReduceOp.SUM, group=self.group)
            else:
                dist.reduce_scatter_tensor(dst, src, op=dist.ReduceOp.SUM, group=self.group)
        if use_side:
            main.wait_stream(self.comm_stream)
        self.shard.copy_(self.shard_f32)      # the single FP16 rounding of the owned rows
        return self.shard

    def down_p2p(self, gather: bool = False, during_reduction: Callable | None = None) -> torch.Tensor:
        """Fused GEMM + reduce-scatter over peer memory: returns this rank's
        FP16 [M / G, hidden] shard (rows [r * M / G, (r + 1) * M / G)).

        With ``gather`` every owner also writes its reduced FP16 rows into all
        peers' output buffers (an all-gather over NVLink) and a second barrier
        completes them: the result is the full FP16 [M, hidden] output on
        every rank, the same value an FP32 all-reduce followed by one rounding
        gives (the slots are added in rank order). Its consumers run on this
        stream; the next call rewrites it.

        ``during_reduction``: work for the current stream (kernels with no
        data dependence on this projection) that runs while the slot
        reduction runs on a side stream."""
        from . import capi

        m, hidden = self.partial.shape
        k = self.h.shape[1]
        if m % self.world != 0:
            raise ValueError(f"M={m} must split into {self.world} equal row groups")
        rows = m // self.world
        if getattr(self, "scatter", None) is None:
            self.scatter = RowScatter(rows, hidden, self.rank, self.world, self.group)
            self.shard_p2p = torch.empty((rows, hidden), device=self.x.device, dtype=torch.float16)
            self._barrier_flag = torch.zeros(1, device=self.x.device, dtype=torch.int32)
        sc = self.scatter
        buf = sc.steps % 2
        stream = torch.cuda.current_stream(self.x.device).cuda_stream
        args = capi.make_args(self.h.data_ptr(), self.w_down.data_ptr(), sc.local[buf], m, hidden, k,
                              ldc=hidden, flags=capi.FLAG_OUT_F32)
        need = capi.workspace_size(args)
        if need:
            if getattr(self, "_p2p_ws", None) is None or self._p2p_ws.numel() < need:
                self._p2p_ws = torch.empty(need, device=self.x.device, dtype=torch.uint8)
            args.workspace, args.workspace_bytes = self._p2p_ws.data_ptr(), need
        rc = capi.run_scatter(args, capi.make_scatter(self.world, self.rank, rows, hidden, sc.dest[buf]), stream)
        if rc != capi.OK:
            raise RuntimeError(f"hgemm_sm100_run_scatter failed: {capi.status_string(rc)}")
        if self.world > 1:
            # Orders every rank's GEMM (its peer stores) before any owner reads.
            dist.all_reduce(self._barrier_flag, op=dist.ReduceOp.MAX, group=self.group)
        main = torch.cuda.current_stream(self.x.device)
        if during_reduction is not None:
            if getattr(self, "reduce_stream", None) is None:
                self.reduce_stream = torch.cuda.Stream(device=self.x.device)
            self.reduce_stream.wait_stream(main)
            stream = self.reduce_stream.cuda_stream
        if gather:
            offset = self.rank * rows * hidden * 2          # this rank's rows in every output
            outs = [sc.dest[2][q] + offset for q in range(self.world)]
            rc = capi.reduce_slots_gather(sc.local[buf], self.world, rows, hidden, hidden, outs, hidden, stream)
        else:
            rc = capi.reduce_slots(sc.local[buf], self.world, rows, hidden, hidden, self.shard_p2p.data_ptr(),
                                   hidden, stream)
        if rc != capi.OK:
            raise RuntimeError(f"hgemm_sm100_reduce_slots failed: {capi.status_string(rc)}")
        if during_reduction is not None:
            during_reduction()
            main.wait_stream(self.reduce_stream)
        sc.steps += 1
        if not gather:
            return self.shard_p2p
        if self.world > 1:
            # Every owner's rows have landed in every output.
            dist.all_reduce(self._barrier_flag, op=dist.ReduceOp.MAX, group=self.group)
        return sc.output

    def close(self) -> None:
        """Releases the peer mappings and receive buffers (collective)."""
        if getattr(self, "scatter", None) is not None:
            if self.out is self.scatter.output:
                self.out = self.out.clone()             # stream-ordered before the buffer is freed
            self.scatter.close()
            self.scatter = None

    def step(self) -> None:
        """One MLP step: the up-projection and the row-parallel
        down-projection. With several ranks on the fused peer-memory path
        (``down_mode`` "p2p", ``overlap`` on) the down-projection's exchange is
        overlapped with the up-projection, which needs no communication: the
        scatter GEMM runs first, then, after the barrier that orders every
        rank's stores, the owners' slot reduction and all-gather run on a side
        stream while the up-projection GEMM runs on the current stream; a
        second barrier completes the gathered output. The values are the same
        as ``up()`` then ``down()``."""
        if self.world > 1 and self.down_mode == "p2p" and getattr(self, "overlap", True) and self.x.is_cuda:
            self.out = self.down_p2p(gather=True, during_reduction=self.up)
            return
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
