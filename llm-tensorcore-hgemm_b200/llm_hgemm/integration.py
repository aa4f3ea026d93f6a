"""Inference-only adapter routing a bias-free FP16 ``nn.Linear`` through
``hgemm`` (reference llm_hgemm/integration.py:8-46).

The weight W[N, K] is packed once as a contiguous B = W^T [K, N]; an input
[..., K] is flattened to A [M, K]. As in the reference, a non-contiguous or
empty input takes ``F.linear`` (kept so that such inputs produce exactly the
stock layer's output), training or grad mode is rejected, and a weight
changed after construction (tracked through tensor versions) is rejected.
"""

import torch
import torch.nn.functional as F
from torch import nn

from .dispatch import last_selected
from .ops import hgemm


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
