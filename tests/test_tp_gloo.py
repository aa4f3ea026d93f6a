"""Tensor-parallel MLP partitioning and reduction on CPU ranks (gloo,
world_size 2 and 3), with an FP32 CPU stand-in for the partial GEMMs; plus
host-side failure detection: a rank that dies before the collective makes
its peer's collective fail instead of hanging."""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llm_hgemm.tensor_parallel import TensorParallelMLP, shard_bounds, shard_columns, shard_rows


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def cpu_gemm(a, b, out):
    return out.copy_((a.float() @ b.float()).half())


def cpu_gemm_f32(a, b, out):
    return out.copy_(a.float() @ b.float())


def _worker(rank, world, port, mode, results):
    try:
        from datetime import timedelta

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=20))
        torch.manual_seed(0)
        m, hidden, inter = 24, 40, 70
        mlp = TensorParallelMLP.synthetic(rank, world, seed=11, device="cpu", m=m,
                                          hidden=hidden, inter=inter,
                                          gemm=cpu_gemm, gemm_f32=cpu_gemm_f32)
        if mode == "die":
            if rank == 1:
                os._exit(3)      # leaves between steps, before any collective
            try:
                mlp.step()
                results[rank] = "no error"
            except Exception as exc:  # the peer's exit surfaces as an error
                results[rank] = f"error: {type(exc).__name__}"
            return
        mlp.step()
        # Full, unsharded products from the same seeds.
        g = torch.Generator().manual_seed(11)
        x = (torch.randn((m, hidden), generator=g) * 0.1).half()
        w_up = (torch.randn((hidden, inter), generator=g) * 0.02).half()
        h = (torch.randn((m, inter), generator=g) * 0.1).half()
        w_down = (torch.randn((inter, hidden), generator=g) * 0.02).half()
        lo, hi = shard_bounds(inter, rank, world)
        y_ref = (x.float() @ w_up.float()).half()[:, lo:hi]
        out_ref = (h.float() @ w_down.float()).half()
        ok_y = torch.equal(mlp.y, y_ref)
        d = (mlp.out.float() - out_ref.float()).abs().max().item()
        if mode == "scatter":
            # Reduce-scatter variants: each rank's FP16 shard holds exactly
            # its owned rows of the same FP32-summed, once-rounded output.
            for chunks in (1, 2):
                shard = mlp.down_scatter(chunks).clone()
                rows = mlp.owned_rows(chunks)
                assert shard.shape == (m // world, hidden)
                assert torch.equal(shard, mlp.out[rows]), chunks
                d = max(d, (shard.float() - out_ref[rows].float()).abs().max().item())
            owned = [None] * world
            dist.all_gather_object(owned, mlp.owned_rows(2).tolist())
            assert sorted(sum(owned, [])) == list(range(m))
        results[rank] = (ok_y, d, mlp.total_flops(), mlp.inter_total)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        results[rank] = traceback.format_exc()


def run_ranks(world, mode):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive(), "rank hung"
    return dict(results)


def test_shard_bounds_cover_exactly():
    for total, world in [(28672, 2), (28672, 8), (70, 3), (7, 7)]:
        spans = [shard_bounds(total, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
        sizes = [hi - lo for lo, hi in spans]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(3, 0, 4)


def test_shard_helpers():
    w = torch.arange(60.).view(6, 10)
    assert torch.equal(torch.cat([shard_columns(w, r, 3) for r in range(3)], 1), w)
    assert torch.equal(torch.cat([shard_rows(w, r, 4) for r in range(4)], 0), w)


@pytest.mark.parametrize("mode", ["ok", "scatter"])
@pytest.mark.parametrize("world", [2, 3])
def test_tp_mlp_matches_unsharded(world, mode):
    results = run_ranks(world, mode)
    assert len(results) == world
    for rank in range(world):
        res = results[rank]
        assert isinstance(res, tuple), res
        ok_y, max_diff, flops, inter = res
        assert ok_y, f"rank {rank} up-proj shard differs"
        assert max_diff <= 1e-3, max_diff
        assert inter == 70 and flops == 2.0 * 24 * 40 * 70 * 2


def test_dead_rank_fails_peer_collective():
    results = run_ranks(2, "die")
    assert results.get(0, "").startswith("error"), results


def test_single_rank_down_projection_needs_no_reduction():
    # One rank (torchrun N=1): the down-projection's GEMM writes the FP16
    # output itself; the value equals the FP32 partial rounded once.
    m, hidden, inter = 24, 40, 70
    mlp = TensorParallelMLP.synthetic(0, 1, seed=11, device="cpu", m=m, hidden=hidden, inter=inter,
                                      gemm=cpu_gemm, gemm_f32=cpu_gemm_f32, down_mode="p2p")
    mlp.step()
    ref = (mlp.h.float() @ mlp.w_down.float()).half()
    assert torch.equal(mlp.out, ref)
    assert torch.equal(mlp.y, (mlp.x.float() @ mlp.w_up.float()).half())
