"""Y = X @ W^T with X in bf16/fp16 and W either INT4-packed (W4A16) or bf16/fp16 (W16A16).

Same public functions as ``int4_triton.gemm`` (``gemm.py:303-317``).  The
dispatch on M happens inside ``libint4_b200.so`` (``i4b_w4a16_matmul``):
M <= 8 runs the register-dequant decode GEMVs, 9 <= M <= 32 the
register-dequant kernel with its in-kernel deterministic split-K reduction, and
larger M the TMA + tcgen05/TMEM GEMM (the reference switches at M = 64; on B200
the tcgen05 GEMM wins from 33 tokens on).  ``w16a16_matmul`` switches at M = 16.  Launches are asynchronous on the current stream and
capture into CUDA graphs (no host synchronisation, no allocation outside torch).
"""
from __future__ import annotations

import torch

from . import _lib


# Above these M the C side may run the TMA + tcgen05 GEMM, whose operands need 16-byte aligned bases and
# row strides (capi.cu: w4_register_path, kSkinnyMaxM).
_W4_GEMV_M, _W16_SMALL_M = 8, 16


def _tma_ok(t: torch.Tensor) -> bool:
    return t.stride(1) == 1 and t.data_ptr() % 16 == 0 and (t.stride(0) * t.element_size()) % 16 == 0


def _unit_n_stride(t: torch.Tensor, tma: bool) -> torch.Tensor:
    ok = _tma_ok(t) if tma else (t.stride(1) == 1 and t.data_ptr() % 16 == 0)
    return t if ok else t.contiguous()


def w4a16_matmul(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor) -> torch.Tensor:
    """x[..., K] (bf16/fp16) @ W^T, W given as packed int4 (see quantize.py). Returns x.dtype [..., N]."""
    assert x.dtype in (torch.bfloat16, torch.float16)
    K = x.shape[-1]
    assert qweight.shape[0] * 8 == K, (qweight.shape, K)
    if not x.is_cuda:
        raise ValueError("int4_b200 computes on the GPU only: x must be a CUDA tensor")
    group_size = K // scales.shape[0]
    N = qweight.shape[1]
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M == 0 or N == 0:
        return y.reshape(*x.shape[:-1], N)
    tma = M > _W4_GEMV_M
    qweight = _unit_n_stride(qweight, tma)
    scales = _unit_n_stride(scales, tma)
    zeros = _unit_n_stride(zeros, tma)
    if scales.stride(0) != zeros.stride(0):
        scales, zeros = scales.contiguous(), zeros.contiguous()
    L = _lib.lib()
    dev = x.device
    stream = _lib.stream_handle(dev)
    with torch.cuda.device(dev):
        need = L.i4b_w4a16_workspace_size(M, N, K, group_size)
        ws_ptr, ws_size = _lib.workspace(dev, stream, need)
        st = L.i4b_w4a16_matmul(x2.data_ptr(), _lib.DTYPE_CODE[x.dtype], M, K, x2.stride(0), x2.stride(1),
                                qweight.data_ptr(), N, qweight.stride(0), scales.data_ptr(), zeros.data_ptr(),
                                scales.stride(0), group_size, y.data_ptr(), y.stride(0), ws_ptr, ws_size, stream)
    _lib.check(st, "w4a16_matmul")
    return y.reshape(*x.shape[:-1], N)


def w4a16_matmul_argmax(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                        logits: bool = False):
    """Greedy choice fused into the W4 matmul (an lm_head): index of the first maximum of each row of
    x[M, K] @ W^T (1 <= M <= 8), as ``(x @ W^T).argmax(-1, keepdim=True)`` on the stored logits.  Returns the
    int64 indices [M, 1], and the logits [M, N] too when ``logits`` is true.  No counterpart in ``int4_triton``."""
    assert x.dtype in (torch.bfloat16, torch.float16) and x.dim() == 2
    if not x.is_cuda:
        raise ValueError("int4_b200 computes on the GPU only: x must be a CUDA tensor")
    M, K = x.shape
    N = qweight.shape[1]
    G = K // scales.shape[0]
    if x.stride(1) != 1:
        x = x.contiguous()
    out = torch.empty((M, 1), dtype=torch.long, device=x.device)
    y = torch.empty((M, N), dtype=x.dtype, device=x.device) if logits else None
    L = _lib.lib()
    dev = x.device
    stream = _lib.stream_handle(dev)
    with torch.cuda.device(dev):
        need = L.i4b_w4a16_argmax_workspace_size(M, N, K, G)
        ws_ptr, ws_size = _lib.workspace(dev, stream, need)
        st = L.i4b_w4a16_matmul_argmax(x.data_ptr(), _lib.DTYPE_CODE[x.dtype], M, K, x.stride(0), qweight.data_ptr(), N,
                                       qweight.stride(0), scales.data_ptr(), zeros.data_ptr(), scales.stride(0), G,
                                       None if y is None else y.data_ptr(), N, out.data_ptr(), ws_ptr, ws_size,
                                       stream)
    _lib.check(st, "w4a16_matmul_argmax")
    return (out, y) if logits else out


def w16a16_matmul(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x[..., K] @ w[N, K]^T with full-precision weights: the same kernel structure as the W4 path."""
    assert x.dtype == w.dtype and x.dtype in (torch.bfloat16, torch.float16)
    if not (x.is_cuda and w.is_cuda):
        raise ValueError("int4_b200 computes on the GPU only: x and w must be CUDA tensors")
    K = x.shape[-1]
    N = w.shape[0]
    assert w.shape[1] == K, (w.shape, K)
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M == 0 or N == 0:
        return y.reshape(*x.shape[:-1], N)
    if M > _W16_SMALL_M and K % 8 == 0 and not _tma_ok(w):
        w = w.contiguous()
    L = _lib.lib()
    dev = x.device
    stream = _lib.stream_handle(dev)
    with torch.cuda.device(dev):
        need = L.i4b_w16a16_workspace_size(M, N, K)
        ws_ptr, ws_size = _lib.workspace(dev, stream, need)
        st = L.i4b_w16a16_matmul(x2.data_ptr(), _lib.DTYPE_CODE[x.dtype], M, K, x2.stride(0), x2.stride(1),
                                 w.data_ptr(), N, w.stride(0), w.stride(1), y.data_ptr(), y.stride(0),
                                 ws_ptr, ws_size, stream)
    _lib.check(st, "w16a16_matmul")
    return y.reshape(*x.shape[:-1], N)
