"""The allocation-free W4A16 entry point gives the same results as the regular one.

``i4b_w4a16_matmul_noalloc`` serves callers that cannot allocate device
memory -- a plugin whose host program owns every cudaMalloc, or code on a path
where an allocation may not run -- so it takes no workspace and uses a scratch
array built into the library instead.  Each case calls it twice in a row
through the C ABI and compares both outputs with ``i4b_w4a16_matmul`` given a
torch-allocated workspace, within the suite's relative Frobenius bound (the two
run the same kernels, so they also agree bit for bit).  The cases cover the
plans that use scratch: split-K partials with tickets (many K splits) and the
large-M copy of a strided activation.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FRO_TOL = 1e-2
I4B_BF16 = 1
I4B_ERR_SCRATCH_LIMIT = 8


def _rel_fro(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float(torch.linalg.norm(a - b) / max(float(torch.linalg.norm(b)), 1e-30))


def _call(L, fn, x, qw, s, z, y, ws=None):
    M, K = x.shape
    N = qw.shape[1]
    G = K // s.shape[0]
    stream = torch.cuda.current_stream(x.device).cuda_stream
    args = [x.data_ptr(), I4B_BF16, M, K, x.stride(0), x.stride(1), qw.data_ptr(), N, qw.stride(0), s.data_ptr(),
            z.data_ptr(), s.stride(0), G, y.data_ptr(), y.stride(0)]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    return getattr(L, fn)(*args, stream)


# (M, N, K, G, strided x): 64 and 16 K-splits use fp32 partials + tickets; M=100 with a strided x copies it.
CASES = [(1, 64, 65536, 128, False), (16, 256, 16384, 32, False), (100, 512, 2048, 128, True), (1, 2048, 2048, 128, False)]


@pytest.mark.parametrize("M,N,K,G,strided", CASES)
def test_noalloc_matches_regular_entry_point_twice(M, N, K, G, strided):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import int4_b200
    from int4_b200 import _lib

    L = _lib.lib()
    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(M * 7 + N + K)
    w = (torch.randn(N, K, generator=gen) * 0.02).to(torch.bfloat16).to(dev)
    qw, s, z = int4_b200.quantize_int4(w, G)
    if strided:
        x = torch.randn(M, 2 * K, generator=gen).to(torch.bfloat16).to(dev)[:, ::2]
    else:
        x = torch.randn(M, K, generator=gen).to(torch.bfloat16).to(dev)

    need = L.i4b_w4a16_workspace_size(M, N, K, G)
    assert 0 < need <= 16 << 20 or (M, N, K) == (1, 2048, 2048)
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=dev)
    y_ref = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    assert _call(L, "i4b_w4a16_matmul", x, qw, s, z, y_ref, ws) == 0

    outs = []
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
        assert _call(L, "i4b_w4a16_matmul_noalloc", x, qw, s, z, y) == 0
        outs.append(y)
    torch.cuda.synchronize()
    for y in outs:
        assert torch.isfinite(y).all()
        assert _rel_fro(y, y_ref) < FRO_TOL
        assert torch.equal(y, y_ref)
    assert _lib.device_error_flags(0, clear=True) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import int4_b200
    from int4_b200 import _lib

    L = _lib.lib()
    dev = torch.device("cuda", 0)
    M, N, K = 4096, 256, 8192  # the large-M plan reserves an M x K bf16 copy: 64 MiB > 16 MiB
    assert L.i4b_w4a16_workspace_size(M, N, K, 128) > 16 << 20
    w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
    qw, s, z = int4_b200.quantize_int4(w, 128)
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    y = torch.zeros(M, N, dtype=torch.bfloat16, device=dev)
    assert _call(L, "i4b_w4a16_matmul_noalloc", x, qw, s, z, y) == I4B_ERR_SCRATCH_LIMIT
    assert L.i4b_status_string(I4B_ERR_SCRATCH_LIMIT).decode().startswith("sizes exceed")
    torch.cuda.synchronize()
    assert np.count_nonzero(y.float().cpu().numpy()) == 0  # nothing was launched


def test_noalloc_split_k_after_a_copy_plan_on_the_shared_array():
    """The strided large-M call writes its activation copy into the shared scratch; a split-K call straight after
    it on the same stream must still find its tickets cleared and match the regular entry point."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import int4_b200
    from int4_b200 import _lib

    L = _lib.lib()
    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(5)
    w1 = (torch.randn(512, 2048, generator=gen) * 0.02).to(torch.bfloat16).to(dev)
    w2 = (torch.randn(64, 65536, generator=gen) * 0.02).to(torch.bfloat16).to(dev)
    q1, q2 = int4_b200.quantize_int4(w1, 128), int4_b200.quantize_int4(w2, 128)
    x1 = torch.randn(100, 4096, generator=gen).to(torch.bfloat16).to(dev)[:, ::2]
    x2 = torch.randn(1, 65536, generator=gen).to(torch.bfloat16).to(dev)
    refs = []
    for x, q in ((x1, q1), (x2, q2)):
        need = L.i4b_w4a16_workspace_size(x.shape[0], q[0].shape[1], x.shape[1], 128)
        ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=dev)
        y = torch.empty(x.shape[0], q[0].shape[1], dtype=torch.bfloat16, device=dev)
        assert _call(L, "i4b_w4a16_matmul", x, *q, y, ws) == 0
        refs.append(y)
    for _ in range(2):
        outs = []
        for x, q in ((x1, q1), (x2, q2)):  # back to back, one stream, no synchronisation in between
            y = torch.full((x.shape[0], q[0].shape[1]), float("nan"), dtype=torch.bfloat16, device=dev)
            assert _call(L, "i4b_w4a16_matmul_noalloc", x, *q, y) == 0
            outs.append(y)
        torch.cuda.synchronize()
        for y, r in zip(outs, refs):
            assert _rel_fro(y, r) < FRO_TOL
            assert torch.equal(y, r)
    assert _lib.device_error_flags(0, clear=True) == 0


def test_noalloc_reports_a_bad_argument_before_the_scratch_limit():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from int4_b200 import _lib

    L = _lib.lib()
    stream = torch.cuda.current_stream(torch.device("cuda", 0)).cuda_stream
    M, N, K = 4096, 256, 8192  # would exceed the scratch, but the dtype code is invalid
    st = L.i4b_w4a16_matmul_noalloc(None, 7, M, K, K, 1, None, N, N, None, None, N, 128, None, N, stream)
    assert st == 1  # I4B_ERR_INVALID_ARG
