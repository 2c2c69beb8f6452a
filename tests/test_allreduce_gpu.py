"""The tensor-parallel all-reduce fused into the W4 matmul (``i4b_w4a16_matmul_allreduce``).

* Two ranks (needs two GPUs; ``tests/allreduce_worker.py`` under torchrun): row-parallel shards of the
  decoder shapes, M = 1..32, against the fp32 oracle of the full product, bit-identical across ranks,
  calls and CUDA-graph replay; the SwiGLU prologue likewise.
* One GPU: a group of one rank is exactly ``i4b_w4a16_matmul``; and the failure path -- a group whose
  other rank never publishes (its buffer is a second local buffer nothing writes flags into) -- ends the
  call after the bounded wait with bit 1 of ``i4b_device_error_flags`` set, and the context keeps working.
"""
from __future__ import annotations

import ctypes
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
PEER_TIMEOUT_BIT = 2


def _group(world: int, rank: int, capacity: int, buffers: list[int]):
    from int4_b200.peer import MAX_RANKS, PeerGroupStruct

    return PeerGroupStruct(world, rank, capacity, (ctypes.c_void_p * MAX_RANKS)(*(buffers + [None] * (MAX_RANKS - len(buffers)))))


def _alloc(L, capacity: int) -> int:
    from int4_b200 import _lib

    p = ctypes.c_void_p()
    _lib.check(L.i4b_peer_buffer_alloc(capacity, ctypes.byref(p)), "i4b_peer_buffer_alloc")
    return p.value


def _call(L, grp, x, q, s, z):
    from int4_b200 import _lib

    M, K = x.shape
    N = q.shape[1]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    st = L.i4b_w4a16_matmul_allreduce(ctypes.byref(grp), 0, x.data_ptr(), _lib.DTYPE_CODE[x.dtype], None, None, 0.0,
                                      None, M, K, x.stride(0), q.data_ptr(), N, q.stride(0), s.data_ptr(),
                                      z.data_ptr(), s.stride(0), K // s.shape[0], y.data_ptr(), y.stride(0),
                                      _lib.stream_handle(x.device))
    return st, y


def test_two_rank_fused_allreduce_matches_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(HERE, "allreduce_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.parametrize("M,N,K", [(1, 2048, 2048), (8, 2048, 8192), (32, 264, 1024)])
def test_group_of_one_is_the_plain_matmul(cuda_device, M, N, K):
    import cases
    from int4_b200 import _lib, quantize_int4, w4a16_matmul

    L = _lib.lib()
    w = cases.weight((N, K), "bfloat16", seed=N + K).to(cuda_device)
    q, s, z = quantize_int4(w, 128)
    x = cases.activations(M, K, "bfloat16", seed=M).to(cuda_device)
    buf = _alloc(L, M * N)
    try:
        st, y = _call(L, _group(1, 0, M * N, [buf]), x, q, s, z)
        assert st == 0, L.i4b_status_string(st)
        assert torch.equal(y.view(torch.int16), w4a16_matmul(x, q, s, z).view(torch.int16))
    finally:
        torch.cuda.synchronize()
        L.i4b_peer_buffer_free(buf)


def test_missing_rank_times_out_and_reports(cuda_device):
    """A rank that never publishes: the wait gives up (bounded), flags the error, and the GPU stays usable."""
    import cases
    from int4_b200 import _lib, quantize_int4, w4a16_matmul

    L = _lib.lib()
    _lib.device_error_flags(cuda_device.index, clear=True)
    N, K, M = 512, 1024, 2
    w = cases.weight((N, K), "bfloat16", seed=3).to(cuda_device)
    q, s, z = quantize_int4(w, 128)
    x = cases.activations(M, K, "bfloat16", seed=4).to(cuda_device)
    bufs = [_alloc(L, M * N), _alloc(L, M * N)]
    try:
        st, _ = _call(L, _group(2, 0, M * N, bufs), x, q, s, z)
        assert st == 0, L.i4b_status_string(st)
        flags = _lib.device_error_flags(cuda_device.index, clear=True)
        assert flags & PEER_TIMEOUT_BIT, flags
        assert _lib.device_error_flags(cuda_device.index, clear=True) == 0
        ref = x.float() @ _dequant(q, s, z).t()
        y = w4a16_matmul(x, q, s, z)
        assert ((y.float() - ref).norm() / ref.norm()).item() < 1e-2
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            L.i4b_peer_buffer_free(b)


def _dequant(q, s, z):
    from int4_b200 import dequantize_int4_ref

    return dequantize_int4_ref(q, s, z, torch.float32)


def test_argmax_exchange_of_one_rank_is_torch_argmax(cuda_device):
    import cases
    from int4_b200 import _lib
    from int4_b200.peer import argmax_allreduce

    L = _lib.lib()
    x = cases.activations(5, 128256, "bfloat16", seed=8).to(cuda_device)
    x[1, 77] = x[1, 99] = 20.0  # equal maxima: the first index
    x[2, :] = float("-inf")
    buf = _alloc(L, 64)
    try:

        class One:  # a peer group of one rank, built straight from the C ABI
            _lib = L
            struct = _group(1, 0, 64, [buf])

        for _ in range(2):
            got = argmax_allreduce(One, x, 0)
            assert torch.equal(got, x.float().argmax(-1, keepdim=True)), got.view(-1).tolist()
    finally:
        torch.cuda.synchronize()
        L.i4b_peer_buffer_free(buf)
