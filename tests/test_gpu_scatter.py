"""Fused GEMM + reduce-scatter (tensor-parallel down-projection) through the
C ABI: hgemm_sm100_run_scatter writes each rank's FP32 partial rows into the
owners' receive buffers, hgemm_sm100_reduce_slots sums them.

On one GPU the ranks are emulated: G GEMMs (one per simulated rank, each with
its K shard and its own `rank`) scatter into G receive buffers that all live
on this GPU; nothing waits on anything, so this exercises every store path of
the scatter without a second GPU. The result must equal, bit for bit, the
FP32 partials of the plain FP32-output GEMM summed in rank order and rounded
once. The real multi-process version (CUDA IPC, NCCL barrier) runs when two
GPUs are present."""

import os
import socket
import traceback

import pytest
import torch

from llm_hgemm import capi
from llm_hgemm.ops import hgemm_f32_out
from oracle import reference as oracle
from tests.gpu_helpers import require_cuda
from tests.test_gpu_pipeline import CONFIG_IDS

pytestmark = pytest.mark.gpu

SCATTER_CONFIGS = ["auto", "tc_persistent_128x256", "tc_persistent_128x128", "tc_streamk_128x256",
                   "tc_pair_256x256", "tc_pair_128x128", "tc_splitk_128x128", "tc_swapab", "tc_generic_128x128"]


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()


def emulate(m, hidden, k_total, world, config, seed=5):
    g = torch.Generator(device="cuda").manual_seed(seed)
    h = (torch.randn((m, k_total), generator=g, device="cuda") * 0.1).half()
    w = (torch.randn((k_total, hidden), generator=g, device="cuda") * 0.02).half()
    rows = m // world
    ks = [(r * k_total // world, (r + 1) * k_total // world) for r in range(world)]
    recv = [torch.full((world, rows, hidden), float("nan"), device="cuda") for _ in range(world)]
    partials = []
    stream = torch.cuda.current_stream().cuda_stream
    cfg = 0 if config == "auto" else CONFIG_IDS[config]
    for r, (lo, hi) in enumerate(ks):
        hr, wr = h[:, lo:hi].contiguous(), w[lo:hi].contiguous()
        p = torch.empty((m, hidden), device="cuda")
        hgemm_f32_out(hr, wr, p, implementation=config)
        partials.append(p)
        args = capi.make_args(hr.data_ptr(), wr.data_ptr(), recv[r].data_ptr(), m, hidden, hi - lo,
                              config=cfg, flags=capi.FLAG_OUT_F32, ldc=hidden)
        need = capi.workspace_size(args)
        ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
        if need:
            args.workspace, args.workspace_bytes = ws.data_ptr(), need
        sc = capi.make_scatter(world, r, rows, hidden, [t.data_ptr() for t in recv])
        assert capi.run_scatter(args, sc, stream) == capi.OK
    shards = []
    for q in range(world):
        out = torch.full((rows, hidden), float("nan"), device="cuda", dtype=torch.float16)
        assert capi.reduce_slots(recv[q].data_ptr(), world, rows, hidden, hidden, out.data_ptr(), hidden,
                                 stream) == capi.OK
        shards.append(out)
    total = partials[0].clone()
    for p in partials[1:]:
        total += p
    return h, w, shards, total.half()


@pytest.mark.parametrize("config", SCATTER_CONFIGS)
@pytest.mark.parametrize("world,shape", [(2, (512, 768, 512)), (4, (1024, 390, 1024)), (8, (2048, 520, 4096))])
def test_emulated_scatter_equals_rank_order_sum(config, world, shape):
    m, hidden, k = shape
    h, w, shards, expect = emulate(m, hidden, k, world, config)
    rows = m // world
    for q, shard in enumerate(shards):
        assert torch.equal(shard, expect[q * rows:(q + 1) * rows]), (config, q)
    metrics = oracle.error_metrics(torch.cat(shards), oracle.torch_reference(h, w))
    assert oracle.correctness_passed(metrics), metrics


def test_emulated_scatter_auto_on_cta_pairs():
    """A row scatter whose K shard is long enough (4096 per rank here) runs on the
    CTA-pair kernel under `auto`, its rows leaving through the bulk-copy path."""
    m, hidden, k, world = 4096, 2560, 8192, 2
    args = capi.make_args(0x1000, 0x1000, 0x1000, m, hidden, k // world, flags=capi.FLAG_OUT_F32, ldc=hidden)
    rc, cfg, _ = capi.resolve(args)
    assert rc == capi.OK and cfg in (capi.CFG_PAIR_256x256, capi.CFG_STREAMK_PAIR_256x256), cfg
    h, w, shards, expect = emulate(m, hidden, k, world, "auto")
    rows = m // world
    for q, shard in enumerate(shards):
        assert torch.equal(shard, expect[q * rows:(q + 1) * rows]), q
    metrics = oracle.error_metrics(torch.cat(shards), oracle.torch_reference(h, w))
    assert oracle.correctness_passed(metrics), metrics


def test_reduce_slots_scalar_path():
    """Columns not a multiple of 4: the element-wise reduction."""
    g = torch.Generator(device="cuda").manual_seed(1)
    slots = torch.randn((3, 17, 30), generator=g, device="cuda")
    out = torch.empty((17, 29), device="cuda", dtype=torch.float16)
    assert capi.reduce_slots(slots.data_ptr(), 3, 17, 29, 30, out.data_ptr(), 29,
                             torch.cuda.current_stream().cuda_stream) == capi.OK
    expect = ((slots[0] + slots[1]) + slots[2])[:, :29].half()
    assert torch.equal(out, expect)


def test_scatter_contract():
    a = torch.zeros((64, 32), device="cuda", dtype=torch.float16)
    b = torch.zeros((32, 48), device="cuda", dtype=torch.float16)
    dst = torch.zeros((2, 32, 48), device="cuda")
    sc = capi.make_scatter(2, 0, 32, 48, [dst.data_ptr(), dst.data_ptr()])
    fp16 = capi.make_args(a.data_ptr(), b.data_ptr(), dst.data_ptr(), 64, 48, 32)
    assert capi.run_scatter(fp16, sc) == capi.ERR_INVALID_ARGUMENT          # needs FLAG_OUT_F32
    args = capi.make_args(a.data_ptr(), b.data_ptr(), dst.data_ptr(), 64, 48, 32, flags=capi.FLAG_OUT_F32)
    bad_rows = capi.make_scatter(2, 0, 30, 48, [dst.data_ptr(), dst.data_ptr()])
    assert capi.run_scatter(args, bad_rows) == capi.ERR_INVALID_ARGUMENT    # 2 * 30 != 64
    bad_rank = capi.make_scatter(2, 2, 32, 48, [dst.data_ptr(), dst.data_ptr()])
    assert capi.run_scatter(args, bad_rank) == capi.ERR_INVALID_ARGUMENT
    null_dest = capi.make_scatter(2, 0, 32, 48, [dst.data_ptr(), None])
    assert capi.run_scatter(args, null_dest) == capi.ERR_INVALID_ARGUMENT
    assert capi.reduce_slots(dst.data_ptr(), 9, 32, 48, 48, dst.data_ptr(), 48) == capi.ERR_INVALID_ARGUMENT


# ------------------------------------------------------ two real GPUs ----

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _p2p_worker(rank, world, port, results, shape=(1024, 768, 2048)):
    import torch.distributed as dist
    from datetime import timedelta

    from llm_hgemm.tensor_parallel import TensorParallelMLP

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        m, hidden, inter = shape
        mlp = TensorParallelMLP.synthetic(rank, world, seed=9, device=torch.device("cuda", rank), m=m,
                                          hidden=hidden, inter=inter)
        full = mlp.down_all_reduce().clone()
        ref = full[mlp.owned_rows(1).to(full.device)]
        worst = 0.0
        for _ in range(3):        # both receive buffers, then the first again
            shard = mlp.down_p2p().clone()
            worst = max(worst, (shard.float() - ref.float()).abs().max().item())
        # With the all-gather: the full output on every rank, as the step's
        # down-projection in "p2p" mode.
        mlp.down_mode = "p2p"
        for _ in range(3):
            out = mlp.down().clone()
            worst = max(worst, (out.float() - full.float()).abs().max().item())
        assert mlp.check()        # one more step, in "p2p" mode
        steps = mlp.scatter.steps
        mlp.close()
        dist.barrier()
        dist.destroy_process_group()
        results[rank] = (worst, steps)
    except Exception:
        results[rank] = traceback.format_exc()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("shape", [(1024, 768, 2048), (8192, 2560, 9728)], ids=["small", "qwen3_4b_mlp"])
def test_two_gpu_fused_reduce_scatter_matches_all_reduce(shape):
    """The small MLP runs the tile kernels; the Qwen3-4B MLP (K = 4864 per rank) the
    CTA-pair kernel with its bulk-copy row scatter across NVLink."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_p2p_worker, args=(r, 2, port, results, shape)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert not p.is_alive(), "rank hung"
    for r in range(2):
        res = results.get(r)
        assert isinstance(res, tuple), res
        worst, steps = res
        # Same FP32 partials; the rank-order sum and NCCL's sum may differ by
        # an FP32 rounding, which can move the FP16 result by one unit.
        assert worst <= 2e-3 and steps == 7, res
