"""Pin the CPU oracle against fixtures produced by the reference's own torch code (CPU only).

The fixtures come from ``tests/golden/make_golden.py``, which ran
``quantize_int4_ref`` / ``dequantize_int4_ref`` (``int4_triton/quantize.py:102-135``)
and the reference tests' matmul expression (``tests/test_kernels.py:54-57``).
"""
from __future__ import annotations

import numpy as np
import pytest

import cases
from oracle import int4_oracle as orc


def _stored(a, dtype):
    """Fixture arrays hold fp16 and bf16 as uint16 bit patterns; the oracle takes fp16 as float16."""
    return a.view(np.float16) if dtype == "float16" else a


def _w_numpy(name_or_tensor, dtype):
    t = name_or_tensor
    if dtype == "bfloat16":
        import torch

        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def test_rebuilt_inputs_match_recorded_hashes(golden_meta):
    """The seeded torch CPU generator still produces the inputs the fixtures were made from."""
    for name in ("ref_100x256_g32_float16", "small_73x256_g64_bfloat16", "cfg1_2048x2048_g128_bfloat16",
                 "block_k_proj_g128"):
        assert cases.sha256(cases.quant_input(name)) == golden_meta["quant"][name]["input_sha256"], name
    for name in cases.GEMM_CASES:
        assert cases.sha256(cases.gemm_input(name)) == golden_meta["gemm"][name]["x_sha256"], name


@pytest.mark.parametrize("name", cases.SMALL_QUANT)
def test_oracle_quantize_small_bit_exact(name, golden_arrays):
    shape, dt, g, _seed, _frac = cases.QUANT_CASES[name]
    w = _stored(golden_arrays[f"{name}/w"], dt)
    qw, s, z = orc.quantize_int4(w, g, dt)
    np.testing.assert_array_equal(qw, golden_arrays[f"{name}/qweight"])
    np.testing.assert_array_equal(s.view(np.uint16), golden_arrays[f"{name}/scales"])
    np.testing.assert_array_equal(z.view(np.uint16), golden_arrays[f"{name}/zeros"])
    for odt in ("float32", "float16", "bfloat16"):
        d = orc.dequantize_int4(qw, s, z, odt)
        ref = golden_arrays[f"{name}/dequant_{odt}"]
        if odt == "float16":
            d = d.view(np.uint16)
        np.testing.assert_array_equal(d, ref, err_msg=f"dequant {odt}")


@pytest.mark.parametrize("dt", ["float32", "bfloat16", "float16"])
def test_oracle_degenerate_groups_bit_exact(dt, golden_arrays):
    """All-zero, underflowing, inf and NaN groups give the reference's exact bits (x86 NaN rules)."""
    key = f"degenerate_{dt}"
    qw, s, z = orc.quantize_int4(_stored(golden_arrays[f"{key}/w"], dt), 32, dt)
    np.testing.assert_array_equal(qw, golden_arrays[f"{key}/qweight"])
    np.testing.assert_array_equal(s.view(np.uint16), golden_arrays[f"{key}/scales"])
    np.testing.assert_array_equal(z.view(np.uint16), golden_arrays[f"{key}/zeros"])


@pytest.mark.parametrize("name", ["ref_512x2048_g32_bfloat16", "ref_2048x8192_g128_float16",
                                  "ref_2048x8192_g-1_bfloat16", "cfg1_2048x2048_g128_bfloat16",
                                  "block_gate_proj_g128", "block_down_proj_g128", "sweep_down_proj_g32"])
def test_oracle_quantize_full_size_hashes(name, golden_meta):
    """Full-size cases: the oracle's outputs hash to the reference's outputs."""
    shape, dt, g, _seed, _frac = cases.QUANT_CASES[name]
    w = _w_numpy(cases.quant_input(name), dt)
    qw, s, z = orc.quantize_int4(w, g, dt)
    m = golden_meta["quant"][name]
    assert cases.sha256(qw) == m["qweight_sha256"]
    assert cases.sha256(s) == m["scales_sha256"]
    assert cases.sha256(z) == m["zeros_sha256"]


@pytest.mark.parametrize("name", list(cases.GEMM_CASES))
def test_oracle_gemm_matches_reference_expression(name, golden_arrays):
    qcase, M, dt, _seed, _strided = cases.GEMM_CASES[name]
    g = cases.QUANT_CASES[qcase][2]
    w = _w_numpy(cases.quant_input(qcase), cases.QUANT_CASES[qcase][1])
    qw, s, z = orc.quantize_int4(w, g, cases.QUANT_CASES[qcase][1])
    x = golden_arrays[f"{name}/x"]
    xin = x if dt == "bfloat16" else x.view(np.float16)
    y = orc.w4a16_matmul(xin, qw, s, z, dt)
    ref = golden_arrays[f"{name}/y_ref"]
    # Same fp32 products; only the BLAS summation order differs from torch's.
    assert orc.rel_fro_error(y, ref) < 1e-6


# ----------------------------------------------------------------------------- the torch restatement


def _as_torch(a, dt):
    import torch

    if dt == "bfloat16":
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    if dt == "float16":
        return torch.from_numpy(a.view(np.float16).copy())
    return torch.from_numpy(np.ascontiguousarray(a))


@pytest.mark.parametrize("name", cases.SMALL_QUANT)
def test_torch_oracle_small_bit_exact(name, golden_arrays):
    """oracle/int4_torch.py gives the reference-generated bits on the small fixtures."""
    import torch

    from oracle import int4_torch as ot

    shape, dt, g, _seed, _frac = cases.QUANT_CASES[name]
    w = _as_torch(golden_arrays[f"{name}/w"], dt)
    qw, s, z = ot.quantize_int4(w, g)
    np.testing.assert_array_equal(qw.numpy(), golden_arrays[f"{name}/qweight"])
    np.testing.assert_array_equal(s.view(torch.int16).numpy().view(np.uint16), golden_arrays[f"{name}/scales"])
    np.testing.assert_array_equal(z.view(torch.int16).numpy().view(np.uint16), golden_arrays[f"{name}/zeros"])
    for odt, tdt in (("float32", torch.float32), ("float16", torch.float16), ("bfloat16", torch.bfloat16)):
        d = ot.dequantize_int4(qw, s, z, tdt)
        got = d.numpy() if odt == "float32" else d.view(torch.int16).numpy().view(np.uint16)
        np.testing.assert_array_equal(got, golden_arrays[f"{name}/dequant_{odt}"], err_msg=f"dequant {odt}")


@pytest.mark.parametrize("name", ["cfg1_2048x2048_g128_bfloat16", "block_gate_proj_g128", "sweep_down_proj_g32"])
def test_torch_oracle_full_size_hashes(name, golden_meta):
    from oracle import int4_torch as ot

    shape, dt, g, _seed, _frac = cases.QUANT_CASES[name]
    qw, s, z = ot.quantize_int4(cases.quant_input(name), g)
    m = golden_meta["quant"][name]
    assert cases.sha256(qw.numpy()) == m["qweight_sha256"]
    assert cases.sha256(s.numpy()) == m["scales_sha256"]
    assert cases.sha256(z.numpy()) == m["zeros_sha256"]


def test_torch_oracle_fake_quantizes_the_selected_linears():
    """fake_quantize_model_ replaces every decoder linear's weight by its INT4 round trip and skips lm_head."""
    import torch

    from oracle import int4_torch as ot

    torch.manual_seed(0)
    model = torch.nn.ModuleDict({"mlp": torch.nn.Linear(256, 64, bias=False), "lm_head": torch.nn.Linear(256, 32)})
    model = model.to(torch.bfloat16)
    before = {k: v.weight.detach().clone() for k, v in model.items()}
    ot.fake_quantize_model_(model, 128)
    w = before["mlp"]
    qw, s, z = orc.quantize_int4(w.view(torch.int16).numpy().view(np.uint16), 128, "bfloat16")
    want = orc.dequantize_int4(qw, s, z, "bfloat16")
    np.testing.assert_array_equal(model["mlp"].weight.view(torch.int16).numpy().view(np.uint16), want)
    assert torch.equal(model["lm_head"].weight, before["lm_head"])
