"""The fused decode-step kernels against the torch expressions transformers' Llama uses.

add_rmsnorm and rope_kv_cache / silu_mul reproduce transformers' bf16 rounding
points, so they are compared with a tolerance of one bf16 ulp of the output
(the fp32 reductions differ only in summation order); decode_attention is an
fp32 softmax like scaled_dot_product_attention and is compared within 1e-2.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ulp_close(a: torch.Tensor, b: torch.Tensor, ulps: int = 1):
    """bf16 tensors equal up to ``ulps`` units in the last place (compared as ordered integers)."""
    ia = a.contiguous().view(torch.int16).int()
    ib = b.contiguous().view(torch.int16).int()
    ia = torch.where(ia < 0, -32768 - ia, ia)
    ib = torch.where(ib < 0, -32768 - ib, ib)
    diff = (ia - ib).abs().max().item()
    assert diff <= ulps, diff


@pytest.mark.parametrize("rows,H", [(1, 2048), (8, 2048), (3, 256)])
@pytest.mark.parametrize("with_delta", [False, True])
def test_add_rmsnorm_matches_llama_rmsnorm(cuda_device, rows, H, with_delta):
    from int4_b200.decode import add_rmsnorm, rms_norm

    g = torch.Generator(device="cuda").manual_seed(rows * H)
    h = torch.randn(rows, H, device="cuda", generator=g).to(torch.bfloat16) * 3
    d = torch.randn(rows, H, device="cuda", generator=g).to(torch.bfloat16) if with_delta else None
    w = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)
    ref_h = h + d if with_delta else h.clone()
    ref = rms_norm(ref_h, w, 1e-5)
    out = torch.empty_like(h)
    add_rmsnorm(h, d, w, out, 1e-5)
    assert torch.equal(h, ref_h)
    _ulp_close(out, ref)


def _rope_reference(t, cos, sin):
    x1, x2 = t.chunk(2, dim=-1)
    return t * cos + torch.cat((-x2, x1), dim=-1) * sin


@pytest.mark.parametrize("B,nq,nkv", [(1, 32, 8), (4, 4, 1)])
def test_rope_kv_cache_matches_apply_rotary_pos_emb(cuda_device, B, nq, nkv):
    from int4_b200.decode import rope_kv_cache

    hd, max_seq, p = 64, 96, 37
    g = torch.Generator(device="cuda").manual_seed(B + nq)
    qkv = torch.randn(B, (nq + 2 * nkv) * hd, device="cuda", generator=g).to(torch.bfloat16)
    ang = torch.randn(max_seq, hd // 2, device="cuda", generator=g)
    cos = torch.cat([ang.cos(), ang.cos()], -1).to(torch.bfloat16)
    sin = torch.cat([ang.sin(), ang.sin()], -1).to(torch.bfloat16)
    kc = torch.zeros(B, nkv, max_seq, hd, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = torch.empty(B, nq, hd, device="cuda", dtype=torch.bfloat16)
    pos = torch.tensor([p], device="cuda")
    rope_kv_cache(qkv, cos, sin, pos, q, kc, vc, nq, nkv)
    qr, kr, vr = qkv.split([nq * hd, nkv * hd, nkv * hd], -1)
    _ulp_close(q, _rope_reference(qr.view(B, nq, hd), cos[p], sin[p]), 0)
    _ulp_close(kc[:, :, p], _rope_reference(kr.view(B, nkv, hd), cos[p], sin[p]), 0)
    assert torch.equal(vc[:, :, p], vr.view(B, nkv, hd))
    assert kc[:, :, :p].abs().sum() == 0 and kc[:, :, p + 1:].abs().sum() == 0
    # a position outside the cache writes nothing
    before = kc.clone()
    rope_kv_cache(qkv, cos, sin, torch.tensor([max_seq], device="cuda"), q, kc, vc, nq, nkv)
    assert torch.equal(kc, before)


@pytest.mark.parametrize("B,nq,nkv,p", [(1, 32, 8, 0), (1, 32, 8, 700), (2, 4, 2, 63)])
def test_decode_attention_matches_sdpa(cuda_device, B, nq, nkv, p):
    from int4_b200.decode import decode_attention

    hd, max_seq = 64, 1024
    g = torch.Generator(device="cuda").manual_seed(p + nq)
    q = torch.randn(B, nq, hd, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, nkv, max_seq, hd, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, nkv, max_seq, hd, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(B, nq * hd, device="cuda", dtype=torch.bfloat16)
    decode_attention(q, kc, vc, torch.tensor([p], device="cuda"), out, nq, nkv, hd ** -0.5)
    ref = F.scaled_dot_product_attention(q[:, :, None].float(), kc[:, :, :p + 1].float(), vc[:, :, :p + 1].float(),
                                         enable_gqa=True)
    err = (out.float() - ref.reshape(B, nq * hd)).abs().max().item()
    assert err <= 1e-2, err


@pytest.mark.parametrize("B,I", [(1, 8192), (5, 4096), (2, 64)])
def test_silu_mul_matches_swiglu(cuda_device, B, I):
    from int4_b200.decode import silu_mul

    g = torch.Generator(device="cuda").manual_seed(B * I)
    gu = (torch.randn(B, 2 * I, device="cuda", generator=g) * 4).to(torch.bfloat16)
    out = torch.empty(B, I, device="cuda", dtype=torch.bfloat16)
    silu_mul(gu, out)
    gate, up = gu.chunk(2, -1)
    _ulp_close(out, F.silu(gate) * up, 1)


@pytest.mark.parametrize("rows,n", [(1, 128256), (3, 64128), (2, 1001)])
def test_argmax_matches_torch_including_ties(cuda_device, rows, n):
    from int4_b200.decode import argmax_last

    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.randn(rows, n, device="cuda", generator=g).to(torch.bfloat16)
    x[:, n // 3] = 50.0  # the same maximum twice: the first index wins
    x[:, 2 * n // 3] = 50.0
    assert torch.equal(argmax_last(x), x.argmax(-1, keepdim=True))
    y = torch.randn(rows, n, device="cuda", generator=g).to(torch.bfloat16)
    assert torch.equal(argmax_last(y), y.argmax(-1, keepdim=True))


@pytest.mark.parametrize("M", [1, 3, 16, 32])
def test_matmul_with_rmsnorm_prologue_matches_norm_then_matmul(cuda_device, M):
    import int4_b200
    from int4_b200.decode import PROLOGUE_RMSNORM, add_rmsnorm, w4a16_matmul_prologue

    N, K = 3072, 2048
    g = torch.Generator(device="cuda").manual_seed(M)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    q = int4_b200.quantize_int4(w, 128)
    h = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    d = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, device="cuda", generator=g)).to(torch.bfloat16)
    resid = torch.empty_like(h)
    y = w4a16_matmul_prologue(PROLOGUE_RMSNORM, h, *q, delta=d, norm_weight=nw, eps=1e-5, resid_out=resid)
    hh, x = h.clone(), torch.empty_like(h)
    add_rmsnorm(hh, d, nw, x, 1e-5)
    ref = int4_b200.w4a16_matmul(x, *q)
    assert torch.equal(resid, hh)
    err = ((y.float() - ref.float()).norm() / ref.float().norm()).item()
    assert err < 1e-3, err
    # without a delta and without a residual output
    y0 = w4a16_matmul_prologue(PROLOGUE_RMSNORM, h, *q, norm_weight=nw, eps=1e-5)
    x0 = torch.empty_like(h)
    add_rmsnorm(h.clone(), None, nw, x0, 1e-5)
    ref0 = int4_b200.w4a16_matmul(x0, *q)
    assert ((y0.float() - ref0.float()).norm() / ref0.float().norm()).item() < 1e-3


@pytest.mark.parametrize("M", [1, 5, 32])
def test_matmul_with_swiglu_prologue_matches_silu_mul_then_matmul(cuda_device, M):
    import int4_b200
    from int4_b200.decode import PROLOGUE_SWIGLU, silu_mul, w4a16_matmul_prologue

    N, K = 2048, 8192
    g = torch.Generator(device="cuda").manual_seed(100 + M)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    q = int4_b200.quantize_int4(w, 128)
    gu = (torch.randn(M, 2 * K, device="cuda", generator=g) * 2).to(torch.bfloat16)
    y = w4a16_matmul_prologue(PROLOGUE_SWIGLU, gu, *q)
    act = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
    silu_mul(gu, act)
    from int4_b200 import _lib

    L = _lib.lib()
    L.i4b_set_w4_small_m_override(32)  # the prologue entry runs the register kernels: compare with those
    try:
        same_kernel = int4_b200.w4a16_matmul(act, *q)
    finally:
        L.i4b_set_w4_small_m_override(0)
    assert torch.equal(y, same_kernel)  # same activations, same kernel: same bits
    routed = int4_b200.w4a16_matmul(act, *q)  # M = 32 on 16 Mi weights: the tcgen05 GEMM
    assert ((routed.float() - y.float()).norm() / y.float().norm()).item() < 1e-3
