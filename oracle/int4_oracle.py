"""CPU oracle for the INT4 W4A16 hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path (``int4_b200``) never
imports it and has no CPU fallback.

It restates, in numpy float32 / uint32 arithmetic, the reference project's
torch implementation of the storage format (homomorfism/itmo-final-project,
package ``int4_triton``):

* ``quantize_int4``   follows ``int4_triton/quantize.py:102-117``
  (``quantize_int4_ref``): per group of G consecutive K-elements of a row,
  ``wmax = max(max(w), 0)``, ``wmin = min(min(w), 0)``,
  ``scale = (wmax - wmin) / 15`` (1 when exactly 0, tested before the fp16
  rounding), scale rounded to fp16 and back, ``zero = clamp(floor(-wmin /
  scale + 0.5), 0, 15)``, ``q = clamp(floor(w / scale + 0.5) + zero, 0, 15)``,
  eight K-consecutive nibbles packed into one int32 word (nibble i at bits
  4i..4i+3, int32 wrap-around sum), outputs transposed to ``[K/8, N]`` and
  ``[K/G, N]``.
* ``unpack_int4``     follows ``int4_triton/quantize.py:120-125``.
* ``dequantize_int4`` follows ``int4_triton/quantize.py:128-135``: fp32
  ``(q - z) * s`` rounded once to the requested dtype.
* ``w4a16_matmul``    is the parity expression of the reference tests,
  ``x.float() @ dequantize_int4_ref(qw, s, z, torch.float32).t()``
  (``tests/test_kernels.py:54-57``).
* ``w16a16_matmul``   is ``x.float() @ w.float().t()``
  (``tests/test_kernels.py:68``).

Parity is pinned: ``tests/test_oracle_golden.py`` checks this module bit for
bit against fixtures that ``tests/golden/make_golden.py`` produced by running
the reference's own torch functions.

Non-finite behaviour.  The reference runs on x86 CPUs, where ``0/0`` yields
the negative default NaN (0xFFC00000), NaN operands propagate, and a float
-> int32 cast of NaN gives INT_MIN.  numpy on x86 uses the same SSE
instructions, so the NaN/INT_MIN bit patterns of degenerate groups (fp16
scale underflowing to 0, inf or NaN weights) match the reference exactly on
x86 hosts; the committed fixtures pin them platform-independently.
"""
from __future__ import annotations

import warnings

import numpy as np

F16, BF16, F32 = "float16", "bfloat16", "float32"


# ----------------------------------------------------------------------------- bf16 helpers


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (torch's ``.to(bfloat16)``).

    NaN keeps its sign and becomes a quiet NaN with the top payload bits, as
    torch's conversion (truncation of a quiet NaN) does.
    """
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    quiet_nan = (u >> np.uint32(16)) | np.uint32(0x0040)
    return np.where(nan, quiet_nan, rounded).astype(np.uint16)


def to_f32(values: np.ndarray, dtype: str) -> np.ndarray:
    """Interpret stored values (fp16 / fp32 arrays, or uint16 bf16 bits) as float32."""
    if dtype == BF16:
        return bf16_bits_to_f32(values)
    return np.asarray(values).astype(np.float32)


# ----------------------------------------------------------------------------- quantize


def quantize_int4(w: np.ndarray, group_size: int = 128, dtype: str = F32):
    """Restatement of ``quantize_int4_ref`` (``int4_triton/quantize.py:102-117``).

    ``w``: ``[N, K]`` weights -- float16/float32 arrays, or uint16 bf16 bit
    patterns with ``dtype="bfloat16"``.  Returns ``(qweight int32[K/8, N],
    scales float16[K/G, N], zeros float16[K/G, N])``, all C-contiguous.
    """
    wf = to_f32(w, dtype)
    N, K = wf.shape
    G = K if group_size == -1 else group_size
    assert K % G == 0 and K % 8 == 0
    one, half, fifteen, zero_f = (np.float32(v) for v in (1.0, 0.5, 15.0, 0.0))
    with warnings.catch_warnings(), np.errstate(all="ignore"):
        warnings.simplefilter("ignore", RuntimeWarning)
        wg = wf.reshape(N, K // G, G)
        wmax = np.maximum(wg.max(axis=-1), zero_f)                       # quantize.py:107
        wmin = np.minimum(wg.min(axis=-1), zero_f)                       # quantize.py:108
        scale = (wmax - wmin) / fifteen                                  # quantize.py:109
        scale = np.where(scale == zero_f, one, scale)                    # quantize.py:110 (before fp16)
        scale = scale.astype(np.float16).astype(np.float32)              # quantize.py:110 (.half().float())
        zero = np.clip(np.floor(-wmin / scale + half), zero_f, fifteen)  # quantize.py:111
        q = np.floor(wg / scale[..., None] + half) + zero[..., None]     # quantize.py:112
        q = np.clip(q, zero_f, fifteen).astype(np.int32)                 # NaN -> INT_MIN (x86 cvttps2dq)
    q = q.reshape(N, K // 8, 8).astype(np.uint32)
    shifts = (np.arange(8, dtype=np.uint32) * np.uint32(4))
    packed = np.zeros((N, K // 8), dtype=np.uint32)
    for i in range(8):                                                   # quantize.py:114-116, int32 wrap
        packed += q[..., i] << shifts[i]
    qweight = np.ascontiguousarray(packed.view(np.int32).T)
    scales = np.ascontiguousarray(scale.astype(np.float16).T)
    zeros = np.ascontiguousarray(zero.astype(np.float16).T)
    return qweight, scales, zeros


# ----------------------------------------------------------------------------- unpack / dequantize


def unpack_int4(qweight: np.ndarray) -> np.ndarray:
    """``int32[K/8, N] -> int32[N, K]`` nibbles in [0, 15] (``quantize.py:120-125``)."""
    qw = np.asarray(qweight).view(np.uint32)
    K8, N = qw.shape
    shifts = np.arange(8, dtype=np.uint32) * np.uint32(4)
    q = (qw.T[:, :, None] >> shifts) & np.uint32(0xF)
    return q.reshape(N, K8 * 8).astype(np.int32)


def dequantize_int4_f32(qweight, scales, zeros) -> np.ndarray:
    """fp32 ``W_hat[N, K] = (q - z) * s`` (``quantize.py:128-135`` before the final cast)."""
    q = unpack_int4(qweight).astype(np.float32)
    N, K = q.shape
    G = K // scales.shape[0]
    s = np.repeat(np.asarray(scales).astype(np.float32).T, G, axis=1)
    z = np.repeat(np.asarray(zeros).astype(np.float32).T, G, axis=1)
    with np.errstate(all="ignore"):
        return (q - z) * s


def dequantize_int4(qweight, scales, zeros, dtype: str = F16) -> np.ndarray:
    """``dequantize_int4_ref`` (``quantize.py:128-135``): fp32 result rounded once to ``dtype``.

    bf16 results are returned as uint16 bit patterns.
    """
    w = dequantize_int4_f32(qweight, scales, zeros)
    if dtype == F32:
        return w
    if dtype == F16:
        return w.astype(np.float16)
    if dtype == BF16:
        return f32_to_bf16_bits(w)
    raise ValueError(dtype)


# ----------------------------------------------------------------------------- matmuls


def w4a16_matmul(x: np.ndarray, qweight, scales, zeros, x_dtype: str = BF16) -> np.ndarray:
    """fp32 ``x @ W_hat^T`` -- the reference tests' oracle (``tests/test_kernels.py:54-57``)."""
    xf = to_f32(x, x_dtype)
    return xf @ dequantize_int4_f32(qweight, scales, zeros).T


def w16a16_matmul(x: np.ndarray, w: np.ndarray, dtype: str = BF16) -> np.ndarray:
    """fp32 ``x @ w^T`` (``tests/test_kernels.py:68``)."""
    return to_f32(x, dtype) @ to_f32(w, dtype).T


def rel_fro_error(out: np.ndarray, ref: np.ndarray) -> float:
    """Relative Frobenius error ``||out - ref|| / ||ref||`` in float64."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-30))


def w4a16_matmul_threaded(x: np.ndarray, qweight, scales, zeros, x_dtype: str = BF16, threads: int = 1) -> np.ndarray:
    """``w4a16_matmul`` split over output columns on ``threads`` host threads (numpy releases the GIL).

    Same arithmetic per column as ``w4a16_matmul``; used to time the
    reference's CPU path with all host cores.
    """
    import concurrent.futures as cf

    qw = np.asarray(qweight)
    N = qw.shape[1]
    if threads <= 1 or N < 2 * threads:
        return w4a16_matmul(x, qweight, scales, zeros, x_dtype)
    xf = to_f32(x, x_dtype)
    bounds = np.linspace(0, N, threads + 1).astype(int)

    def part(i):
        a, b = bounds[i], bounds[i + 1]
        return xf @ dequantize_int4_f32(qw[:, a:b], scales[:, a:b], zeros[:, a:b]).T

    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        return np.concatenate(list(ex.map(part, range(threads))), axis=1)
