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
