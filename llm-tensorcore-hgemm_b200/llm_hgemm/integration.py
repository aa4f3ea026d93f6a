"""Inference-only adapter routing a bias-free FP16 ``nn.Linear`` through
``hgemm`` (reference llm_hgemm/integration.py:8-46).

The weight W[N, K] is packed once as a contiguous B = W^T [K, N]; an input
[..., K] is flattened to A [M, K]. As in the reference, a non-contiguous or
empty input takes ``F.linear`` (kept so that such inputs produce exactly the
stock layer's output), training or grad mode is rejected, and a weight
changed after construction (tracked through tensor versions) is rejected.

Fused projections (no reference counterpart; its model path runs one GEMM
per ``nn.Linear``): :func:`fuse_projections` gives each attention block one
GEMM over the concatenated q|k|v weights (:class:`FusedQKV`) and each SwiGLU
MLP one GEMM over interleaved gate/up weights whose ``silu_mul`` epilogue
writes ``silu(gate) * up`` directly (:class:`HgemmSwiGLU`), followed by the
down projection.
"""

import torch
import torch.nn.functional as F
from torch import nn

from .dispatch import last_selected
from .ops import hgemm, interleave_gate_up


class FrozenHgemmLinear(nn.Module):
    def __init__(self, linear: nn.Linear, implementation: str = "shape_auto"):
        super().__init__()
        if not isinstance(linear, nn.Linear) or linear.bias is not None:
            raise ValueError("requires a bias-free nn.Linear")
        if not linear.weight.is_cuda or linear.weight.dtype != torch.float16:
            raise ValueError("construct after moving FP16 model to CUDA")
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.implementation = implementation
        self.register_buffer("weight", linear.weight.detach())
        self.register_buffer("packed_weight", linear.weight.detach().t().contiguous())
        self._weight_version = self._version(self.weight)
        self._packed_version = self._version(self.packed_weight)
        self.last_backend = None
        self.eval()

    @staticmethod
    def _version(tensor):
        return None if torch.is_inference(tensor) else tensor._version

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.training or torch.is_grad_enabled():
            raise RuntimeError("FrozenHgemmLinear is inference-only")
        if (self._version(self.weight) != self._weight_version
                or self._version(self.packed_weight) != self._packed_version):
            raise RuntimeError("weights changed: rebuild the adapter")
        if x.ndim < 1 or x.shape[-1] != self.in_features:
            raise ValueError("invalid Linear input shape")
        if x.device != self.packed_weight.device or x.dtype != torch.float16:
            raise ValueError("input must be FP16 on the weight device")
        if not x.is_contiguous() or x.numel() == 0:
            self.last_backend = "torch"
            return F.linear(x, self.weight)
        y = hgemm(x.view(-1, self.in_features), self.packed_weight,
                  implementation=self.implementation)
        self.last_backend = (last_selected() if self.implementation == "shape_auto"
                             else self.implementation)
        return y.view(*x.shape[:-1], self.out_features)


def swap_linears(module: nn.Module, implementation: str = "shape_auto") -> int:
    """Replaces every bias-free FP16 CUDA ``nn.Linear`` below ``module`` with a
    ``FrozenHgemmLinear``; returns how many were swapped."""
    count = 0
    for name, child in list(module.named_children()):
        if (isinstance(child, nn.Linear) and child.bias is None and child.weight.is_cuda
                and child.weight.dtype == torch.float16):
            setattr(module, name, FrozenHgemmLinear(child, implementation))
            count += 1
        else:
            count += swap_linears(child, implementation)
    return count


def _check_linear(linear) -> None:
    if not isinstance(linear, nn.Linear) or linear.bias is not None:
        raise ValueError("requires bias-free nn.Linear projections")
    if not linear.weight.is_cuda or linear.weight.dtype != torch.float16:
        raise ValueError("construct after moving FP16 model to CUDA")


def _check_input(module, x: torch.Tensor, in_features: int, device) -> bool:
    """Common adapter checks; True when ``x`` takes the hgemm path."""
    if module.training or torch.is_grad_enabled():
        raise RuntimeError(f"{type(module).__name__} is inference-only")
    if x.ndim < 1 or x.shape[-1] != in_features:
        raise ValueError("invalid Linear input shape")
    if x.device != device or x.dtype != torch.float16:
        raise ValueError("input must be FP16 on the weight device")
    return x.is_contiguous() and x.numel() > 0


class FusedQKV(nn.Module):
    """One GEMM for the q, k and v projections of an attention block.

    ``packed_weight`` is [K, Nq + Nk + Nv] (the three W^T side by side). The
    block still calls ``q_proj(x)``, ``k_proj(x)``, ``v_proj(x)`` in turn:
    those become :class:`QKVSlice` views of this module. The first call with
    a given input tensor runs the GEMM; the other two calls with the same
    tensor object return column slices of that output: strided views (row
    pitch Nq + Nk + Nv) for q and k, which the block normalises into new
    tensors at once, and a contiguous copy for v, which a KV cache keeps (a
    view would keep the whole q|k|v output alive and make every later cache
    concatenation read it strided). The output is kept only until all three
    slices have been taken; a slice asked for twice, or for another tensor,
    runs the GEMM again. The three calls must see the input unchanged (the
    attention block makes them back to back).
    """

    def __init__(self, q: nn.Linear, k: nn.Linear, v: nn.Linear, implementation: str = "shape_auto"):
        super().__init__()
        for lin in (q, k, v):
            _check_linear(lin)
        if not q.in_features == k.in_features == v.in_features:
            raise ValueError("q, k, v projections must share in_features")
        self.in_features = q.in_features
        self.splits = (q.out_features, k.out_features, v.out_features)
        self.implementation = implementation
        self.register_buffer("weights", torch.cat([q.weight.detach(), k.weight.detach(), v.weight.detach()]))
        self.register_buffer("packed_weight", self.weights.t().contiguous())
        q_n, k_n, _ = self.splits
        self._bounds = ((0, q_n), (q_n, q_n + k_n), (q_n + k_n, sum(self.splits)))
        self._src = None
        self._out = None
        self._taken = set()
        self.launches = 0
        self.last_backend = None
        self.eval()

    def slice_of(self, x: torch.Tensor, which: int) -> torch.Tensor:
        lo, hi = self._bounds[which]
        if x is self._src and which not in self._taken:
            out = self._out[..., lo:hi]
            if which == 2:
                out = out.contiguous()
            self._taken.add(which)
            if len(self._taken) == 3:
                self._src = self._out = None
            return out
        if not _check_input(self, x, self.in_features, self.packed_weight.device):
            self.last_backend = "torch"
            return F.linear(x, self.weights[lo:hi])
        out = hgemm(x.view(-1, self.in_features), self.packed_weight, implementation=self.implementation)
        self.launches += 1
        self.last_backend = last_selected() if self.implementation == "shape_auto" else self.implementation
        self._src, self._out, self._taken = x, out.view(*x.shape[:-1], out.shape[-1]), {which}
        sliced = self._out[..., lo:hi]
        return sliced.contiguous() if which == 2 else sliced


class QKVSlice(nn.Module):
    """``q_proj`` / ``k_proj`` / ``v_proj`` stand-in reading its columns of the
    shared :class:`FusedQKV` output."""

    def __init__(self, fused: FusedQKV, which: int):
        super().__init__()
        self.which = which
        self.in_features = fused.in_features
        self.out_features = fused.splits[which]
        object.__setattr__(self, "_fused", fused)   # shared, registered once on the parent

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._fused.slice_of(x, self.which)


class HgemmSwiGLU(nn.Module):
    """SwiGLU MLP ``down(silu(gate(x)) * up(x))`` in two GEMM launches.

    The first GEMM multiplies by the interleaved [K, 2I] gate/up operand
    (column 2j = gate j, 2j + 1 = up j) with the ``silu_mul`` epilogue, so the
    [M, I] activation is written once, already gated; the second is the down
    projection. The stock module runs three GEMMs and two elementwise kernels
    and rounds the gate and up outputs to FP16 before the product."""

    def __init__(self, gate: nn.Linear, up: nn.Linear, down: nn.Linear, implementation: str = "shape_auto"):
        super().__init__()
        for lin in (gate, up, down):
            _check_linear(lin)
        if gate.weight.shape != up.weight.shape or down.in_features != gate.out_features:
            raise ValueError("gate/up/down shapes do not form an MLP")
        self.in_features = gate.in_features
        self.intermediate = gate.out_features
        self.out_features = down.out_features
        self.implementation = implementation
        self.register_buffer("gate_weight", gate.weight.detach())
        self.register_buffer("up_weight", up.weight.detach())
        self.register_buffer("down_weight", down.weight.detach())
        self.register_buffer("gate_up_packed", interleave_gate_up(gate.weight.detach().t(), up.weight.detach().t()))
        self.register_buffer("down_packed", down.weight.detach().t().contiguous())
        self.last_backend = None
        self.eval()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not _check_input(self, x, self.in_features, self.gate_up_packed.device):
            self.last_backend = "torch"
            h = F.silu(F.linear(x, self.gate_weight)) * F.linear(x, self.up_weight)
            return F.linear(h, self.down_weight)
        x2 = x.view(-1, self.in_features)
        h = hgemm(x2, self.gate_up_packed, implementation=self.implementation, epilogue="silu_mul")
        gate_backend = last_selected() if self.implementation == "shape_auto" else self.implementation
        y = hgemm(h, self.down_packed, implementation=self.implementation)
        self.last_backend = gate_backend
        return y.view(*x.shape[:-1], self.out_features)


def _is_silu(act) -> bool:
    t = torch.linspace(-6.0, 6.0, 25)
    try:
        return bool(torch.allclose(act(t), F.silu(t)))
    except Exception:   # not a plain elementwise callable
        return False


def fuse_projections(module: nn.Module, implementation: str = "shape_auto") -> dict:
    """Fuses the projections of every attention block (children ``q_proj``,
    ``k_proj``, ``v_proj``) and every SwiGLU MLP (children ``gate_proj``,
    ``up_proj``, ``down_proj`` with a SiLU ``act_fn``) below ``module``, in
    place. Run :func:`swap_linears` afterwards for the remaining linears.
    Returns ``{"qkv": blocks fused, "mlp": MLPs fused}``."""
    counts = {"qkv": 0, "mlp": 0}
    for name, child in list(module.named_children()):
        lins = [getattr(child, n, None) for n in ("q_proj", "k_proj", "v_proj")]
        if all(isinstance(lin, nn.Linear) for lin in lins):
            fused = FusedQKV(*lins, implementation=implementation)
            child.qkv_fused = fused
            for i, n in enumerate(("q_proj", "k_proj", "v_proj")):
                setattr(child, n, QKVSlice(fused, i))
            counts["qkv"] += 1
        mlp = [getattr(child, n, None) for n in ("gate_proj", "up_proj", "down_proj")]
        if all(isinstance(lin, nn.Linear) for lin in mlp) and _is_silu(getattr(child, "act_fn", None)):
            setattr(module, name, HgemmSwiGLU(*mlp, implementation=implementation))
            counts["mlp"] += 1
            continue
        sub = fuse_projections(child, implementation)
        counts["qkv"] += sub["qkv"]
        counts["mlp"] += sub["mlp"]
    return counts
