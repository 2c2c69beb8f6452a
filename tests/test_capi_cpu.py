"""The C-ABI library loads on a machine without a GPU and exports every symbol the header declares.

No compute call is made: only status strings, version, and argument
validation that returns before any CUDA call.
"""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "int4_b200.h")


def _declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(i4b_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    from int4_b200 import _lib

    if not os.path.exists(_lib.LIB_PATH):
        from int4_b200 import build

        build.build()
    return _lib.lib()


def test_header_declares_the_reference_surface():
    names = _declared_functions()
    for required in ("i4b_quantize_int4", "i4b_dequantize_int4", "i4b_w4a16_matmul", "i4b_w16a16_matmul",
                     "i4b_w4a16_workspace_size", "i4b_w16a16_workspace_size"):
        assert required in names


def test_library_exports_every_declared_symbol(L):
    handle = ctypes.CDLL(os.path.join(ROOT, "itmo-final-project_b200", "int4_b200", "libint4_b200.so"))
    missing = [n for n in _declared_functions() if not hasattr(handle, n)]
    assert not missing, missing


def test_version_and_status_strings(L):
    assert L.i4b_abi_version() == 1
    assert L.i4b_status_string(0) == b"ok"
    assert L.i4b_status_string(5) == b"workspace too small"
    assert L.i4b_status_string(99) == b"unknown status"


def test_argument_validation_before_any_device_call(L):
    # bad dtype, bad group, K not a multiple of 8: rejected before touching CUDA
    assert L.i4b_quantize_int4(None, 7, 4, 32, 32, 1, 32, None, None, None, None) == 1
    assert L.i4b_quantize_int4(None, 1, 4, 32, 32, 1, 12, None, None, None, None) == 3
    assert L.i4b_quantize_int4(None, 1, 4, 36, 36, 1, 36, None, None, None, None) == 2
    assert L.i4b_w4a16_matmul(None, 2, 1, 256, 256, 1, None, 8, 8, None, None, 8, 128, None, 8, None, 0, None) == 1
    assert L.i4b_w4a16_matmul(None, 1, 1, 256, 256, 1, None, 8, 8, None, None, 8, 16, None, 8, None, 0, None) == 3
    # empty problems are a no-op
    assert L.i4b_w4a16_matmul(None, 1, 0, 256, 256, 1, None, 8, 8, None, None, 8, 128, None, 8, None, 0, None) == 0
    assert L.i4b_w4a16_workspace_size(1, 8, 256, 16) == 0


def test_fused_allreduce_validation_before_any_device_call(L):
    import ctypes

    from int4_b200.peer import MAX_RANKS, PeerGroupStruct

    fake = [0x100000 * (i + 1) for i in range(2)]  # never dereferenced: every case below fails validation first

    def call(grp, prologue=0, dtype=1, M=1, N=64, K=256, G=128):
        return L.i4b_w4a16_matmul_allreduce(ctypes.byref(grp), prologue, 0x1000, dtype, None, None, 0.0, None, M, K, K,
                                            0x2000, N, N, 0x3000, 0x4000, N, G, 0x5000, N, None)

    def grp(world, rank, cap, bufs):
        return PeerGroupStruct(world, rank, cap, (ctypes.c_void_p * MAX_RANKS)(*(bufs + [None] * (MAX_RANKS - len(bufs)))))

    assert L.i4b_w4a16_matmul_allreduce(None, 0, None, 1, None, None, 0.0, None, 1, 256, 256, None, 64, 64, None,
                                        None, 64, 128, None, 64, None) == 1  # no group
    assert call(grp(9, 0, 64, fake)) == 1            # more ranks than a group holds
    assert call(grp(2, 2, 64, fake)) == 1            # rank outside the group
    assert call(grp(2, 0, 64, fake), prologue=1) == 1  # RMSNorm of a K shard is rejected
    assert call(grp(2, 0, 64, fake), dtype=0, prologue=2) == 1  # SwiGLU prologue is bf16 only
    assert call(grp(2, 0, 63, fake)) == 2            # M * N beyond the buffers' capacity
    assert call(grp(2, 0, 64, fake), M=33) == 2       # beyond the small-M kernel
    assert call(grp(2, 0, 64, fake), G=96) == 3
    assert call(grp(2, 0, 64, [fake[0]])) == 1        # a rank without a buffer
    assert call(grp(2, 0, 64, [fake[0], fake[1] + 16])) == 1  # buffers are 256-byte aligned allocations
    assert call(grp(2, 0, 64, fake), M=0) == 0        # empty: no-op
    assert L.i4b_peer_buffer_bytes(0) == 256 + 2 * 8 * 1024 * 4
    # control, reserved, then 2 slots x 8 source ranks x capacity tagged 64-bit values
    assert L.i4b_peer_buffer_bytes(1000) == 256 + 2 * 8 * 1024 * 4 + 2 * 8 * 1000 * 8
    assert L.i4b_ipc_get_handle(None, None) == 1 and L.i4b_ipc_open_handle(None, None) == 1


def test_argmax_allreduce_validation_before_any_device_call(L):
    import ctypes

    from int4_b200.peer import MAX_RANKS, PeerGroupStruct

    bufs = [0x100000, 0x200000]
    grp = PeerGroupStruct(2, 1, 16, (ctypes.c_void_p * MAX_RANKS)(*(bufs + [None] * (MAX_RANKS - 2))))
    call = L.i4b_argmax_allreduce
    assert call(None, 0x1000, 4, 100, 100, 0, 0x2000, None) == 1             # no group
    assert call(ctypes.byref(grp), 0x1000, 4, 100, 99, 0, 0x2000, None) == 2  # row stride below n
    assert call(ctypes.byref(grp), 0x1000, 9, 100, 100, 0, 0x2000, None) == 2  # 2 * rows beyond capacity
    assert call(ctypes.byref(grp), None, 4, 100, 100, 0, 0x2000, None) == 1
    assert call(ctypes.byref(grp), 0x1000, 0, 100, 100, 0, 0x2000, None) == 0   # no rows: no-op


def test_w4_workspace_query_covers_the_register_plan_and_the_tuning_hooks(L):
    """Up to M = 32 the size query covers the register-dequant plan, which the prologue and all-reduce entry
    points (sized by the same query) always run; the tuning hooks only ever move the answer between the
    two paths' needs and are restored by their reset values."""
    try:
        sizes = {}
        for small in (0, 8, 32):  # 0: default routing
            L.i4b_set_w4_small_m_override(small)
            sizes[small] = [L.i4b_w4a16_workspace_size(M, 2048, 8192, 128) for M in (1, 16, 32, 48)]
        # forcing the register path up to 32 never asks for more than the default covers at M <= 32
        assert all(d >= r for d, r in zip(sizes[0][:3], sizes[32][:3]))
        # M = 48 is always the tcgen05 GEMM
        assert sizes[0][3] == sizes[8][3] == sizes[32][3] > 0
        L.i4b_set_gemm_override(6, 2)  # tuning: a K split of the TMEM-weight tile adds fp32 partials
        split = L.i4b_w4a16_workspace_size(48, 2048, 8192, 128)
        L.i4b_set_gemm_override(0, 0)
        assert split >= 2 * 48 * 2048 * 4
        assert L.i4b_w4a16_workspace_size(48, 2048, 8192, 128) == sizes[0][3]
    finally:
        L.i4b_set_w4_small_m_override(0)
        L.i4b_set_gemm_override(0, 0)


def test_bench_stdout_is_one_json_line_per_run():
    """The driver parses bench.py's stdout: the reference arm prints exactly one JSON line there, whatever
    native libraries write to file descriptor 1."""
    import json
    import subprocess
    import sys

    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3", "--decode-steps", "0"], capture_output=True, text=True, timeout=600,
                         cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout[:2000]
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["steps"] == 1 and line["warmup"] == 1
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0
