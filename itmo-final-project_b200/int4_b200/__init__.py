"""int4_b200 -- B200-native (sm_100a) INT4 W4A16: drop-in for ``int4_triton``.

Same seven public names as the reference package (``int4_triton/__init__.py``),
plus ``dequantize_int4`` (the GPU dequantize kernel), ``unpack_int4_ref`` and
``w4a16_matmul_argmax`` (the greedy choice fused into a W4 lm_head matmul).
"""
from .gemm import w4a16_matmul, w4a16_matmul_argmax, w16a16_matmul
from .qlinear import Int4Linear, quantize_model_linears
from .quantize import dequantize_int4, dequantize_int4_ref, quantize_int4, quantize_int4_ref, unpack_int4_ref

__all__ = [
    "quantize_int4",
    "quantize_int4_ref",
    "dequantize_int4_ref",
    "w4a16_matmul",
    "w16a16_matmul",
    "Int4Linear",
    "quantize_model_linears",
    "dequantize_int4",
    "unpack_int4_ref",
    "w4a16_matmul_argmax",
]
