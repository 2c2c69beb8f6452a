"""Group-wise asymmetric INT4 quantization -- same API and storage format as ``int4_triton.quantize``.

For every group of ``group_size`` consecutive elements along K (per output row n)::

    scale = (max - min) / 15,  zero = round(-min / scale)        (min <= 0 <= max)
    q     = clamp(round(w / scale) + zero, 0, 15)
    w_hat = (q - zero) * scale

Storage (reference ``int4_triton/quantize.py:1-13``)::

    qweight : int32 [K // 8, N]   8 int4 values packed along K, nibble i = row 8*k8 + i
    scales  : fp16  [K // G, N]
    zeros   : fp16  [K // G, N]   integer-valued zero points

All work runs in the sm_100a kernels of ``libint4_b200.so``; the ``*_ref``
names of the reference are provided with identical results (the quantize
kernel is bit-exact with ``quantize_int4_ref``), computed on the GPU.
"""
from __future__ import annotations

import torch

from . import _lib


def _check_weight(w: torch.Tensor) -> None:
    if not w.is_cuda:
        raise ValueError("int4_b200 computes on the GPU only: move the tensor to a CUDA device first")


def _quantize(w: torch.Tensor, group_size: int):
    N, K = w.shape
    G = K if group_size == -1 else group_size
    assert G > 0 and K % G == 0 and G % 8 == 0, (K, group_size)
    qweight = torch.empty((K // 8, N), dtype=torch.int32, device=w.device)
    scales = torch.empty((K // G, N), dtype=torch.float16, device=w.device)
    zeros = torch.empty_like(scales)
    if N == 0 or K == 0:
        return qweight, scales, zeros
    L = _lib.lib()
    with torch.cuda.device(w.device):
        st = L.i4b_quantize_int4(w.data_ptr(), _lib.DTYPE_CODE[w.dtype], N, K, w.stride(0), w.stride(1), G,
                                 qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
                                 _lib.stream_handle(w.device))
    _lib.check(st, "quantize_int4")
    return qweight, scales, zeros


def quantize_int4(w: torch.Tensor, group_size: int = 128):
    """Quantize W[N, K] (fp16 or bf16, CUDA) -> (qweight int32 [K/8, N], scales fp16 [K/G, N], zeros fp16 [K/G, N]).

    Same preconditions as the reference (``int4_triton/quantize.py:67-75``); the
    result is bit-exact with ``quantize_int4_ref``.
    """
    assert w.dim() == 2 and w.is_cuda
    assert w.dtype in (torch.float16, torch.bfloat16)
    K = w.shape[1]
    if group_size == -1:
        group_size = K
    assert K % group_size == 0 and group_size % 8 == 0
    assert group_size & (group_size - 1) == 0, "group_size must be a power of 2"
    return _quantize(w, group_size)


def quantize_int4_ref(w: torch.Tensor, group_size: int = 128):
    """``quantize_int4_ref`` of the reference (``quantize.py:102-117``), computed on the GPU.

    Accepts fp16 / bf16 / fp32 and any group size that is a multiple of 8
    dividing K; bit-exact with the reference's torch implementation.
    """
    assert w.dim() == 2
    _check_weight(w)
    assert w.dtype in (torch.float16, torch.bfloat16, torch.float32)
    return _quantize(w, group_size)


def unpack_int4_ref(qweight: torch.Tensor) -> torch.Tensor:
    """int32 [K/8, N] -> int32 [N, K] with values in [0, 15] (``quantize.py:120-125``)."""
    K8, N = qweight.shape
    shifts = torch.arange(0, 32, 4, device=qweight.device, dtype=torch.int32)
    return ((qweight.t()[:, :, None] >> shifts) & 0xF).reshape(N, K8 * 8)


def dequantize_int4(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                    dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """W_hat[N, K] = (q - zero) * scale in fp32, rounded once to ``dtype`` (GPU kernel)."""
    _check_weight(qweight)
    K8, N = qweight.shape
    K = K8 * 8
    G = K // scales.shape[0]
    assert scales.shape == zeros.shape == (K // G, N)
    out = torch.empty((N, K), dtype=dtype, device=qweight.device)
    if N == 0 or K == 0:
        return out
    qw, s, z = qweight.contiguous(), scales.contiguous(), zeros.contiguous()
    L = _lib.lib()
    with torch.cuda.device(qweight.device):
        st = L.i4b_dequantize_int4(qw.data_ptr(), s.data_ptr(), z.data_ptr(), N, K, G, _lib.DTYPE_CODE[dtype],
                                   out.data_ptr(), _lib.stream_handle(qweight.device))
    _lib.check(st, "dequantize_int4")
    return out


def dequantize_int4_ref(qweight, scales, zeros, dtype=torch.float16) -> torch.Tensor:
    """``dequantize_int4_ref`` of the reference (``quantize.py:128-135``), computed on the GPU."""
    return dequantize_int4(qweight, scales, zeros, dtype)
