"""ctypes binding of ``libint4_b200.so`` (the C ABI declared in ``include/int4_b200.h``).

The library is built in place by ``int4_b200.build``.  There is no fallback:
if the library is missing, or the device is not a B200, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB = None
_LOCK = threading.Lock()
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libint4_b200.so")

I4B_F16, I4B_BF16, I4B_F32 = 0, 1, 2
DTYPE_CODE = {torch.float16: I4B_F16, torch.bfloat16: I4B_BF16, torch.float32: I4B_F32}

_c_i64, _c_int, _c_size, _c_vp = ctypes.c_int64, ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p

_SIGNATURES = {
    "i4b_status_string": (ctypes.c_char_p, [_c_int]),
    "i4b_abi_version": (_c_int, []),
    "i4b_last_cuda_error": (_c_int, []),
    "i4b_quantize_int4": (_c_int, [_c_vp, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_vp, _c_vp]),
    "i4b_dequantize_int4": (_c_int, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_int, _c_int, _c_vp, _c_vp]),
    "i4b_w4a16_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64, _c_int]),
    "i4b_w4a16_matmul": (_c_int, [_c_vp, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp,
                                  _c_i64, _c_int, _c_vp, _c_i64, _c_vp, _c_size, _c_vp]),
    "i4b_w4a16_matmul_noalloc": (_c_int, [_c_vp, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp,
                                          _c_vp, _c_i64, _c_int, _c_vp, _c_i64, _c_vp]),
    "i4b_w4a16_matmul_prologue": (_c_int, [_c_int, _c_vp, _c_vp, _c_vp, ctypes.c_float, _c_vp, _c_i64, _c_i64, _c_i64,
                                           _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_i64, _c_int, _c_vp, _c_i64, _c_vp,
                                           _c_size, _c_vp]),
    "i4b_w4a16_argmax_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64, _c_int]),
    "i4b_w4a16_matmul_argmax": (_c_int, [_c_vp, _c_int, _c_i64, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp,
                                         _c_i64, _c_int, _c_vp, _c_i64, _c_vp, _c_vp, _c_size, _c_vp]),
    "i4b_w16a16_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "i4b_w16a16_matmul": (_c_int, [_c_vp, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_i64,
                                   _c_vp, _c_i64, _c_vp, _c_size, _c_vp]),
    "i4b_add_rmsnorm": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, ctypes.c_float, _c_vp]),
    "i4b_rope_kv_cache": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64,
                                   _c_i64, _c_vp]),
    "i4b_decode_attention": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                      ctypes.c_float, _c_vp]),
    "i4b_silu_mul": (_c_int, [_c_vp, _c_vp, _c_i64, _c_i64, _c_vp]),
    "i4b_argmax_rows": (_c_int, [_c_vp, _c_i64, _c_i64, _c_vp, _c_vp]),
    "i4b_set_pdl": (None, [_c_int]),
    "i4b_set_w4_kernel_override": (None, [_c_int, _c_int, _c_int]),
    "i4b_set_w4_small_m_override": (None, [_c_int]),
    "i4b_set_skinny_override": (None, [_c_int, _c_int, _c_int]),
    "i4b_set_gemm_override": (None, [_c_int, _c_int]),
    "i4b_device_error_flags": (_c_int, [_c_int, _c_int]),
    "i4b_tile_w4_bytes": (_c_size, [_c_i64, _c_i64, _c_int]),
    "i4b_tile_w4": (_c_int, [_c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_i64, _c_i64, _c_int, _c_vp, _c_vp]),
    "i4b_decode_workspace_size": (_c_int, [_c_vp, ctypes.POINTER(_c_size)]),
    "i4b_decode_layers": (_c_int, [_c_vp, _c_vp, _c_size, _c_vp]),
    "i4b_set_decode_trace": (None, [_c_vp, _c_size]),
    "i4b_peer_buffer_bytes": (_c_size, [_c_i64]),
    "i4b_argmax_allreduce": (_c_int, [_c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_vp, _c_vp]),
    "i4b_decode_peer_capacity": (_c_i64, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "i4b_peer_buffer_alloc": (_c_int, [_c_i64, ctypes.POINTER(_c_vp)]),
    "i4b_peer_buffer_free": (_c_int, [_c_vp]),
    "i4b_ipc_get_handle": (_c_int, [_c_vp, _c_vp]),
    "i4b_ipc_open_handle": (_c_int, [_c_vp, ctypes.POINTER(_c_vp)]),
    "i4b_ipc_close_handle": (_c_int, [_c_vp]),
    "i4b_w4a16_matmul_allreduce": (_c_int, [_c_vp, _c_int, _c_vp, _c_int, _c_vp, _c_vp, ctypes.c_float, _c_vp, _c_i64,
                                            _c_i64, _c_i64, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_i64, _c_int, _c_vp,
                                            _c_i64, _c_vp]),
}


class DecodeModel(ctypes.Structure):
    """``i4b_decode_model`` of include/int4_b200.h."""

    _fields_ = [(n, ctypes.c_int32) for n in ("layers", "hidden", "heads", "kv_heads", "head_dim", "intermediate",
                                              "vocab", "group_size", "batch", "max_seq", "cache_batch")] + \
               [("eps", ctypes.c_float), ("attn_scale", ctypes.c_float)] + \
               [(n, ctypes.c_void_p) for n in ("tokens", "pos", "embed", "w_qkv", "w_o", "w_gu", "w_down", "ln1",
                                               "ln2", "cos_table", "sin_table", "k_cache", "v_cache", "h_out",
                                               "peers")]


class Int4B200Error(RuntimeError):
    """A C-ABI call returned a non-zero status (``status``: the ``i4b_status`` code)."""

    def __init__(self, message: str, status: int = 0):
        super().__init__(message)
        self.status = status


STATUS_SHAPE = 2  # I4B_ERR_SHAPE


def lib() -> ctypes.CDLL:
    """Load the library once (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        with _LOCK:
            if _LIB is None:
                if not os.path.exists(LIB_PATH):
                    raise Int4B200Error(
                        f"{LIB_PATH} is missing: build it with `python -m int4_b200.build` "
                        "(int4_b200 has no CPU or fallback path)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _LIB = handle
    return _LIB


def check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        msg = L.i4b_status_string(status).decode()
        if status == 6:  # I4B_ERR_CUDA
            msg += f" (cudaError {L.i4b_last_cuda_error()})"
        raise Int4B200Error(f"{what}: {msg} [status {status}]", status)


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# Per (device, stream) workspace, zero-filled once; the kernels leave their
# ticket counters at zero, so it is reused without clearing.
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


_WS_LOCK = threading.Lock()


def workspace(device: torch.device, stream: int, nbytes: int) -> tuple[int, int]:
    """(pointer, size) of a workspace of at least ``nbytes`` for this device and stream.  Growing it
    replaces the buffer: the old one returns to torch's allocator in the stream's order, so launches already
    queued on this stream still find it intact."""
    if nbytes == 0:
        return 0, 0
    key = (device.index, stream)
    with _WS_LOCK:
        ws = _WORKSPACES.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            if ws is not None:
                size = max(size, 2 * ws.numel())
            ws = torch.zeros(size, dtype=torch.uint8, device=device)
            _WORKSPACES[key] = ws
        return ws.data_ptr(), ws.numel()


def device_error_flags(device: int = 0, clear: bool = True) -> int:
    """Device-side error flags of the library's kernels (synchronises the device)."""
    return lib().i4b_device_error_flags(device, 1 if clear else 0)


def set_pdl(enable: bool) -> None:
    """Programmatic dependent launch for the small-M kernels (see include/int4_b200.h)."""
    lib().i4b_set_pdl(1 if enable else 0)


def set_skinny_override(wn: int = 0, wk: int = 0, splits: int = 0) -> None:
    lib().i4b_set_skinny_override(wn, wk, splits)
