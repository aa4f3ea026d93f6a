"""Failure detection on the GPU without a GPU fault.

Every mbarrier wait inside the kernels is bounded. The test-only flag
HGEMM_SM100_FLAG_TEST_INJECT_TX arms the first pipeline stage with 16 bytes
more than its TMA copies deliver, so that stage never completes: the consumer's
wait must run out after `timeout_ns`, record HGEMM_SM100_ERR_PIPELINE_TIMEOUT
in the status word, and every role of the CTA must drain and exit. The host
reads the status, and the context stays usable (a normal GEMM afterwards is
correct)."""

import pytest
import torch

from llm_hgemm import capi, hgemm
from tests.gpu_helpers import assert_gate, require_cuda, seeded_inputs

pytestmark = pytest.mark.gpu

TMA_CONFIGS = {
    "tc_persistent_128x256": (capi.CFG_PERSISTENT_128x256, (256, 512, 512)),
    "tc_persistent_128x128": (capi.CFG_PERSISTENT_128x128, (256, 256, 512)),
    "tc_pair_256x256": (capi.CFG_PAIR_256x256, (512, 512, 512)),
    "tc_pair_256x128": (capi.CFG_PAIR_256x128, (512, 512, 512)),
    "tc_pair_128x256": (capi.CFG_PAIR_128x256, (512, 512, 512)),
    "tc_pair_128x128": (capi.CFG_PAIR_128x128, (512, 512, 512)),
    "tc_splitk_128x128": (capi.CFG_SPLITK_128x128, (128, 256, 1024)),
    "tc_splitk_128x256": (capi.CFG_SPLITK_128x256, (128, 512, 1024)),
    "tc_swapab": (capi.CFG_SWAPAB, (16, 512, 1024)),
    "tc_streamk_128x256": (capi.CFG_STREAMK_128x256, (300, 520, 2056)),
    "tc_streamk_swapab": (capi.CFG_STREAMK_SWAPAB, (8, 1000, 3000)),
    "tc_streamk_pair_256x256": (capi.CFG_STREAMK_PAIR_256x256, (512, 512, 512)),
}


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    require_cuda()


@pytest.mark.parametrize("name", list(TMA_CONFIGS))
def test_injected_stall_times_out_and_context_survives(name):
    cfg, (m, n, k) = TMA_CONFIGS[name]
    a, b = seeded_inputs(m, n, k)
    out = torch.zeros((m, n), device="cuda", dtype=torch.float16)
    status = torch.zeros(1, device="cuda", dtype=torch.int32)
    stream = torch.cuda.current_stream().cuda_stream
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, config=cfg,
                          flags=capi.FLAG_TEST_INJECT_TX, status_ptr=status.data_ptr(),
                          timeout_ns=50_000_000)
    need = capi.workspace_size(args)
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    if need:
        args.workspace, args.workspace_bytes = ws.data_ptr(), need
    assert capi.run(args, stream) == capi.OK
    torch.cuda.synchronize()
    assert int(status.item()) == capi.ERR_PIPELINE_TIMEOUT
    # The context is intact: the same configuration now computes correctly.
    good = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float16)
    args_ok = capi.make_args(a.data_ptr(), b.data_ptr(), good.data_ptr(), m, n, k, config=cfg)
    if need:
        args_ok.workspace, args_ok.workspace_bytes = ws.data_ptr(), need
    assert capi.run(args_ok, stream) == capi.OK
    assert_gate(good, a, b)


def test_library_status_word():
    """Without a caller status pointer the library's own word records it."""
    rc, _ = capi.read_status(clear=True)
    assert rc == capi.OK
    m, n, k = 256, 512, 512
    a, b = seeded_inputs(m, n, k)
    out = torch.zeros((m, n), device="cuda", dtype=torch.float16)
    args = capi.make_args(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
                          config=capi.CFG_PERSISTENT_128x256, flags=capi.FLAG_TEST_INJECT_TX,
                          timeout_ns=50_000_000)
    assert capi.run(args, torch.cuda.current_stream().cuda_stream) == capi.OK
    rc, value = capi.read_status(clear=True)
    assert rc == capi.OK and value == capi.ERR_PIPELINE_TIMEOUT
    rc, value = capi.read_status(clear=False)
    assert value == 0
    assert_gate(hgemm(a, b), a, b)
