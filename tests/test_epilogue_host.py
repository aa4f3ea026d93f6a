"""Host-side pieces of the fused epilogues, on CPU: the interleaved gate/up
operand layout, the epilogue oracle against an explicit restatement, the
ctypes mirror of the C-ABI argument struct, and the SiLU detection of
fuse_projections."""

import ctypes

import torch

from llm_hgemm import capi
from llm_hgemm.integration import _is_silu
from llm_hgemm.ops import interleave_gate_up
from oracle import reference as oracle


def test_interleave_gate_up_layout():
    g = torch.arange(12, dtype=torch.float16).reshape(3, 4)
    u = -torch.arange(12, dtype=torch.float16).reshape(3, 4)
    b = interleave_gate_up(g, u)
    assert b.shape == (3, 8) and b.is_contiguous()
    assert torch.equal(b[:, 0::2], g) and torch.equal(b[:, 1::2], u)


def test_epilogue_oracle_matches_explicit_math():
    torch.manual_seed(0)
    a = (torch.randn(5, 7) * 0.5).half()
    b = (torch.randn(7, 6) * 0.5).half()
    bias = (torch.randn(6) * 0.1).half()
    res = (torch.randn(5, 6) * 0.1).half()
    acc = a.double() @ b.double()
    expect = (acc + bias.double() + res.double()).half()
    got = oracle.torch_reference_epilogue(a, b, "bias+residual", bias, res)
    assert (got.float() - expect.float()).abs().max() <= 1e-3
    g, u = acc[:, 0::2] + bias.double()[0::2], acc[:, 1::2] + bias.double()[1::2]
    expect = (g / (1 + torch.exp(-g)) * u).half()
    got = oracle.torch_reference_epilogue(a, b, "bias+silu_mul", bias)
    assert got.shape == (5, 3)
    assert (got.float() - expect.float()).abs().max() <= 1e-3
    assert torch.equal(oracle.torch_reference_epilogue(a, b), oracle.torch_reference(a, b))


def test_args_struct_layout():
    """Offsets of include/hgemm_sm100.h's HgemmSm100Args on x86-64."""
    A = capi.HgemmSm100Args
    assert ctypes.sizeof(A) == 152
    assert A.workspace_bytes.offset == 112
    assert A.epilogue.offset == 120 and A.bias.offset == 128
    assert A.residual.offset == 136 and A.ldr.offset == 144
    args = capi.make_args(1, 2, 3, 4, 10, 6, epilogue=capi.EPI_SILU_MUL)
    assert args.ldc == 5 and args.ldr == 10


def test_silu_detection():
    assert _is_silu(torch.nn.SiLU())
    assert not _is_silu(torch.nn.GELU())
    assert not _is_silu(None)
