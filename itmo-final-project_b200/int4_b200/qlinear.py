"""``Int4Linear`` and ``quantize_model_linears`` -- same API and buffers as ``int4_triton.qlinear``.

Buffer names and dtypes match the reference (``qlinear.py:17-21``), so state
dicts interchange with it.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .gemm import w4a16_matmul
from .quantize import dequantize_int4, quantize_int4


class Int4Linear(nn.Module):
    """A linear layer whose weight is stored as packed 4-bit groups; activations stay 16-bit.

    ``forward`` runs the B200 W4A16 matmul on the packed weight directly (no
    dequantized copy is ever materialised).  The buffers carry the reference's
    names, shapes and dtypes so a state dict saved by one loads in the other.
    """

    def __init__(self, in_features: int, out_features: int, group_size: int = 128, bias: bool = False, device=None):
        super().__init__()
        assert in_features % group_size == 0
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        n_groups = in_features // group_size
        self.register_buffer("qweight", torch.empty((in_features // 8, out_features), dtype=torch.int32, device=device))
        self.register_buffer("scales", torch.empty((n_groups, out_features), dtype=torch.float16, device=device))
        self.register_buffer("zeros", torch.empty((n_groups, out_features), dtype=torch.float16, device=device))
        self.register_buffer("bias", torch.empty(out_features, device=device) if bias else None)

    @classmethod
    @torch.no_grad()
    def from_linear(cls, linear: nn.Linear, group_size: int = 128) -> "Int4Linear":
        w = linear.weight.data
        m = cls(linear.in_features, linear.out_features, group_size, linear.bias is not None, device=w.device)
        m.qweight, m.scales, m.zeros = quantize_int4(w.contiguous(), group_size)
        if linear.bias is not None:
            m.bias = linear.bias.data.clone()
        return m

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = w4a16_matmul(x, self.qweight, self.scales, self.zeros)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y

    def dequantize(self, dtype=torch.bfloat16) -> torch.Tensor:
        return dequantize_int4(self.qweight, self.scales, self.zeros, dtype)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, group_size={self.group_size}"


def _iter_linears(model: nn.Module, skip):
    """(parent, attribute name, layer) of each nn.Linear whose dotted path contains none of ``skip``.

    The parent is returned so that the caller can swap the layer in place.
    """
    for prefix, parent in model.named_modules():
        for attr, layer in parent.named_children():
            if not isinstance(layer, nn.Linear):
                continue
            path = attr if not prefix else prefix + "." + attr
            if all(pattern not in path for pattern in skip):
                yield parent, attr, layer


@torch.no_grad()
def quantize_model_linears(model: nn.Module, group_size: int = 128, skip=("lm_head",), fake: bool = False) -> nn.Module:
    """Swap the model's nn.Linear layers for Int4Linear, in place; returns the model.

    Layers whose dotted name contains one of the ``skip`` substrings keep full
    precision (by default the lm_head).  With ``fake=True`` nothing is swapped:
    each weight is replaced by its quantize-then-dequantize round trip, which is
    the accuracy yardstick the W4 kernels are compared with.  Same semantics as
    the reference's helper (``qlinear.py:54-68``).
    """
    for parent, child_name, child in list(_iter_linears(model, skip)):
        q = Int4Linear.from_linear(child, group_size)
        if fake:
            child.weight.data.copy_(q.dequantize(child.weight.dtype))
        else:
            setattr(parent, child_name, q)
        torch.cuda.empty_cache()
    return model
