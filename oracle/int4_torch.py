"""Torch restatement of the reference's quantize / dequantize helpers -- TEST INFRASTRUCTURE ONLY.

The checker, never the product: only ``tests/`` and ``bench.py``'s CPU-baseline
legs may import it, and ``int4_b200`` never does.

``oracle/int4_oracle.py`` restates the reference in numpy; it is pinned bit for
bit to fixtures made by running the reference's own torch code.  That numpy
form takes seconds per 10^7 weights, too slow to fake-quantize a whole
Llama-3.2-1B-shaped model (about 10^9 decoder weights) inside a test.  This
module restates the same algorithm as elementwise torch ops, the way the
reference itself writes it (``int4_triton/quantize.py:102-135`` is plain torch),
so it runs on the host cores or on a GPU tensor in well under a second:

* ``quantize_int4``   -- ``quantize_int4_ref`` (``quantize.py:102-117``): per
  group of G consecutive K-elements of a row, max(max, 0) and min(min, 0),
  scale = (max - min) / 15 (1 when exactly 0, tested before the fp16 rounding),
  scale rounded to fp16 and back, zero = clamp(floor(-min / scale + 0.5), 0, 15),
  q = clamp(floor(w / scale + 0.5) + zero, 0, 15), eight K-consecutive nibbles
  per int32 word (nibble i at bits 4i..4i+3, two's-complement wrap), outputs
  transposed to [K/8, N] and [K/G, N].
* ``dequantize_int4`` -- ``dequantize_int4_ref`` (``quantize.py:120-135``): fp32
  (q - z) * s, rounded once to the requested dtype.
* ``fake_quantize_model_`` -- the ``fake=True`` branch of
  ``quantize_model_linears`` (``int4_triton/qlinear.py:54-68``): every
  ``nn.Linear`` whose dotted name contains none of ``skip`` gets its weight
  replaced by dequantize(quantize(weight)) in the weight's dtype.

Every step is a separate elementwise torch op (IEEE division, no fused
multiply-add between the division and the +0.5), so the result does not
depend on the device for finite inputs.  ``tests/test_oracle_golden.py`` pins
this module to the numpy oracle and to the reference-generated fixtures on the
CPU; the GPU model tests check it against the numpy oracle again on the device
they run it on.
"""
from __future__ import annotations

import torch


def quantize_int4(w: torch.Tensor, group_size: int = 128):
    """``quantize_int4_ref``: (qweight int32[K/8, N], scales fp16[K/G, N], zeros fp16[K/G, N]), contiguous."""
    N, K = w.shape
    G = K if group_size == -1 else group_size
    assert K % G == 0 and K % 8 == 0, (K, G)
    wg = w.float().reshape(N, K // G, G)
    hi = torch.clamp(wg.amax(dim=-1), min=0.0)                       # quantize.py:107
    lo = torch.clamp(wg.amin(dim=-1), max=0.0)                       # quantize.py:108
    scale = (hi - lo) / 15.0                                         # quantize.py:109
    scale = torch.where(scale == 0.0, torch.ones_like(scale), scale)  # quantize.py:110, before the fp16 round
    scale = scale.to(torch.float16).float()                          # quantize.py:110
    zero = torch.clamp(torch.floor(-lo / scale + 0.5), 0.0, 15.0)    # quantize.py:111
    q = torch.floor(wg / scale.unsqueeze(-1) + 0.5) + zero.unsqueeze(-1)
    q = torch.clamp(q, 0.0, 15.0).to(torch.int64).reshape(N, K // 8, 8)  # quantize.py:112
    shifts = torch.arange(0, 32, 4, device=w.device, dtype=torch.int64)
    word = (q << shifts).sum(dim=-1)                                 # quantize.py:114-116, < 2^32
    word = torch.where(word >= 2 ** 31, word - 2 ** 32, word).to(torch.int32)  # int32 wrap-around
    return (word.t().contiguous(), scale.to(torch.float16).t().contiguous(),
            zero.to(torch.float16).t().contiguous())


def unpack_int4(qweight: torch.Tensor) -> torch.Tensor:
    """int32 [K/8, N] -> int32 [N, K] nibbles in [0, 15] (``quantize.py:120-125``)."""
    K8, N = qweight.shape
    shifts = torch.arange(0, 32, 4, device=qweight.device, dtype=torch.int32)
    return ((qweight.t().unsqueeze(-1) >> shifts) & 0xF).reshape(N, K8 * 8)


def dequantize_int4(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                    dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """``dequantize_int4_ref``: fp32 (q - z) * s rounded once to ``dtype``; [N, K]."""
    q = unpack_int4(qweight).float()
    N, K = q.shape
    G = K // scales.shape[0]
    s = scales.float().t().repeat_interleave(G, dim=1)
    z = zeros.float().t().repeat_interleave(G, dim=1)
    return ((q - z) * s).to(dtype)


@torch.no_grad()
def fake_quantize_model_(model: torch.nn.Module, group_size: int = 128, skip=("lm_head",)) -> torch.nn.Module:
    """In place: each selected nn.Linear weight becomes its INT4 round trip (``qlinear.py:54-68``, fake=True)."""
    for prefix, parent in model.named_modules():
        for attr, layer in parent.named_children():
            path = attr if not prefix else prefix + "." + attr
            if isinstance(layer, torch.nn.Linear) and all(p not in path for p in skip):
                w = layer.weight.data
                layer.weight.data.copy_(dequantize_int4(*quantize_int4(w, group_size), dtype=w.dtype))
    return model
