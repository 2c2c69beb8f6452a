"""Seeded input recipes shared by the golden-fixture generator and the parity tests.

Every input is drawn from torch's CPU generator with a fixed seed, so the same
tensors are rebuilt on any machine; ``golden.json`` also records a sha256 of
each rebuilt input so that a change of generator is caught instead of being
reported as a kernel mismatch.

The shapes follow the reference's tests (``tests/test_kernels.py:17-110``) and
the benchmark configurations: one Llama-3.2-1B-shaped decoder block (seven
linears, ``benchmarks/bench_gemm.py:18-26``), weights N(0, 0.02) with 0.1% of
entries scaled x10 as outliers.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

LLAMA_1B_LINEARS = {
    "q_proj": (2048, 2048),
    "k_proj": (512, 2048),
    "v_proj": (512, 2048),
    "o_proj": (2048, 2048),
    "gate_proj": (8192, 2048),
    "up_proj": (8192, 2048),
    "down_proj": (2048, 8192),
}

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def sha256(t) -> str:
    """sha256 of the raw bytes of a tensor / array (made C-contiguous first)."""
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        t = t.numpy()
    return hashlib.sha256(np.ascontiguousarray(t).tobytes()).hexdigest()


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def weight(shape, dtype="bfloat16", seed=0, std=0.02, outlier_frac=0.0) -> torch.Tensor:
    """W ~ N(0, std) in ``dtype``; ``outlier_frac`` of the entries (seeded randperm) scaled x10."""
    g = gen(seed)
    w = torch.randn(shape, generator=g) * std
    if outlier_frac > 0:
        n = w.numel()
        idx = torch.randperm(n, generator=g)[: max(1, int(round(n * outlier_frac)))]
        w.view(-1)[idx] *= 10.0
    return w.to(DTYPES[dtype])


def activations(M, K, dtype="bfloat16", seed=1) -> torch.Tensor:
    return torch.randn((M, K), generator=gen(seed)).to(DTYPES[dtype])


def degenerate_weight(dtype="float32") -> torch.Tensor:
    """Eight rows of 32 (one group each at G=32) that reach every special case of the rounding:

    row 0 all zero (scale forced to 1); row 1 tiny positive (fp16 scale
    underflows to 0, zero becomes NaN); row 2 one tiny negative entry (zero
    becomes 15, 0/0 nibbles); row 3 a NaN; rows 4/5 +inf / -inf; row 6 large
    finite values; row 7 a range whose scale overflows fp16.
    """
    w = torch.zeros(8, 32, dtype=torch.float32)
    w[1] = 1e-9
    w[2, 0] = -1e-9
    w[3, 5] = float("nan")
    w[4, 3] = float("inf")
    w[5, 3] = float("-inf")
    w[6] = torch.randn(32, generator=gen(7)) * 1e4
    w[7, 0] = 65504.0 * 30.0
    w[7, 1] = -1.0
    return w.to(DTYPES[dtype])


# name -> (shape, dtype, group_size, seed, outlier_frac)
QUANT_CASES = {}
for _dt in ("float16", "bfloat16"):
    for _shape in ((512, 2048), (2048, 8192), (100, 256)):
        for _g in (32, 128, -1):
            QUANT_CASES[f"ref_{_shape[0]}x{_shape[1]}_g{_g}_{_dt}"] = (_shape, _dt, _g, 0, 0.0)
QUANT_CASES["cfg1_2048x2048_g128_bfloat16"] = ((2048, 2048), "bfloat16", 128, 0, 0.0)
for _name, (_n, _k) in LLAMA_1B_LINEARS.items():
    QUANT_CASES[f"block_{_name}_g128"] = ((_n, _k), "bfloat16", 128, 100, 1e-3)
for _name in ("gate_proj", "down_proj"):
    for _g in (32, 64):
        QUANT_CASES[f"sweep_{_name}_g{_g}"] = (LLAMA_1B_LINEARS[_name], "bfloat16", _g, 100, 1e-3)
QUANT_CASES["small_73x256_g32_bfloat16"] = ((73, 256), "bfloat16", 32, 1, 0.0)
QUANT_CASES["small_73x256_g64_bfloat16"] = ((73, 256), "bfloat16", 64, 1, 0.0)
QUANT_CASES["small_300x256_g128_float16"] = ((300, 256), "float16", 128, 0, 0.0)
QUANT_CASES["fp32_96x512_g64"] = ((96, 512), "float32", 64, 3, 0.0)

# Cases whose full arrays (inputs and outputs) are small enough to commit.
SMALL_QUANT = [k for k, v in QUANT_CASES.items() if v[0][0] * v[0][1] <= 128 * 1024]


def quant_input(name: str) -> torch.Tensor:
    shape, dt, _g, seed, frac = QUANT_CASES[name]
    return weight(shape, dt, seed=seed, outlier_frac=frac)


# GEMM parity cases with committed outputs: name -> (quant case, M, x dtype, x seed, strided x)
GEMM_CASES = {
    "gemm_300x256_m1": ("small_300x256_g128_float16", 1, "bfloat16", 11, False),
    "gemm_300x256_m7": ("small_300x256_g128_float16", 7, "bfloat16", 12, False),
    "gemm_300x256_m128": ("small_300x256_g128_float16", 128, "bfloat16", 13, False),
    "gemm_300x256_m7_fp16": ("small_300x256_g128_float16", 7, "float16", 14, False),
    "gemm_73x256_g32_m16_strided": ("small_73x256_g32_bfloat16", 16, "bfloat16", 15, True),
    "gemm_73x256_g64_m65_strided": ("small_73x256_g64_bfloat16", 65, "bfloat16", 16, True),
    "gemm_cfg1_m1": ("cfg1_2048x2048_g128_bfloat16", 1, "bfloat16", 1, False),
}


def gemm_input(name: str) -> torch.Tensor:
    """Activations ``[M, K]``; strided cases take every other column of ``[M, 2K]`` like the reference test."""
    qcase, M, dt, seed, strided = GEMM_CASES[name]
    K = QUANT_CASES[qcase][0][1]
    if strided:
        return activations(M, 2 * K, dt, seed)[:, ::2]
    return activations(M, K, dt, seed)
