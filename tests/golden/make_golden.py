"""Generate the golden fixtures by running the REFERENCE's own torch functions.

Run once in a container where the reference project is present::

    python tests/golden/make_golden.py --reference <path to homomorfism/itmo-final-project>

It imports ``int4_triton.quantize.quantize_int4_ref`` / ``dequantize_int4_ref``
(``int4_triton/quantize.py:102-135``) from that checkout, runs them on CPU on
the seeded inputs of ``cases.py`` and writes

* ``golden.json``      -- sha256 of every rebuilt input and of every output
  (qweight / scales / zeros) for all quantize cases, including the full-size
  ones (2048x8192, the seven decoder-block linears);
* ``golden_small.npz`` -- full input and output arrays of the small cases,
  the degenerate-group cases and the GEMM cases, whose outputs are the
  reference tests' expression ``x.float() @ dequantize_int4_ref(qw, s, z,
  torch.float32).t()`` (``tests/test_kernels.py:54-57``).

The fixtures are committed; nothing at test or bench time reads the reference.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout (read only)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from int4_triton.quantize import dequantize_int4_ref, quantize_int4_ref  # the reference itself

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    meta = {"torch": torch.__version__, "quant": {}, "degenerate": {}, "gemm": {}}
    arrays = {}

    for name, (shape, dt, g, seed, frac) in cases.QUANT_CASES.items():
        w = cases.quant_input(name)
        qw, s, z = quantize_int4_ref(w, g)
        meta["quant"][name] = {
            "shape": list(shape), "dtype": dt, "group_size": g, "seed": seed, "outlier_frac": frac,
            "input_sha256": cases.sha256(w),
            "qweight_sha256": cases.sha256(qw), "scales_sha256": cases.sha256(s), "zeros_sha256": cases.sha256(z),
        }
        if name in cases.SMALL_QUANT:
            arrays[f"{name}/w"] = _np(w)
            arrays[f"{name}/qweight"] = _np(qw)
            arrays[f"{name}/scales"] = _np(s)
            arrays[f"{name}/zeros"] = _np(z)
            for odt in ("float32", "float16", "bfloat16"):
                arrays[f"{name}/dequant_{odt}"] = _np(dequantize_int4_ref(qw, s, z, cases.DTYPES[odt]))
        print("quant", name, flush=True)

    for dt in ("float32", "bfloat16", "float16"):
        w = cases.degenerate_weight(dt)
        qw, s, z = quantize_int4_ref(w, 32)
        key = f"degenerate_{dt}"
        meta["degenerate"][key] = {"dtype": dt, "group_size": 32}
        arrays[f"{key}/w"] = _np(w)
        arrays[f"{key}/qweight"] = _np(qw)
        arrays[f"{key}/scales"] = _np(s)
        arrays[f"{key}/zeros"] = _np(z)

    for name, (qcase, M, dt, seed, strided) in cases.GEMM_CASES.items():
        w = cases.quant_input(qcase)
        g = cases.QUANT_CASES[qcase][2]
        qw, s, z = quantize_int4_ref(w, g)
        x = cases.gemm_input(name)
        ref = x.float() @ dequantize_int4_ref(qw, s, z, torch.float32).t()
        meta["gemm"][name] = {"quant_case": qcase, "M": M, "dtype": dt, "seed": seed, "strided": strided,
                              "x_sha256": cases.sha256(x)}
        arrays[f"{name}/x"] = _np(x)
        arrays[f"{name}/y_ref"] = _np(ref)
        print("gemm", name, flush=True)

    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "golden_small.npz"), **arrays)
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    main()
