"""Peer exchange buffers of a tensor-parallel group, for the all-reduce fused into the W4 matmul.

The reference runs on one GPU; its tensor-parallel form (o_proj / down_proj
split along K) needs the ranks' partial outputs summed after every
row-parallel projection.  ``w4a16_matmul_allreduce`` does that inside the
matmul's epilogue: every rank stores its fp32 partials straight into every
other rank's exchange buffer over NVLink, raises a flag per CTA, waits
(bounded) for the other ranks' flags and adds the partials in rank order, so
all ranks hold bit-identical outputs.

``PeerGroup`` sets the buffers up once per group: each rank allocates a
zero-filled buffer through the C ABI, the CUDA-IPC handles are exchanged with
``torch.distributed.all_gather_object``, and each rank maps the others'
buffers.  Plain peer stores and flag loads only; no multicast object.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

MAX_RANKS = 8
HANDLE_BYTES = 64


class PeerGroupStruct(ctypes.Structure):
    """``i4b_peer_group`` of include/int4_b200.h."""

    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("capacity", ctypes.c_int64),
                ("buffers", ctypes.c_void_p * MAX_RANKS)]


class PeerGroup:
    """Exchange buffers of every rank of ``group``, mapped into this process.

    ``capacity`` is the largest M * N a fused call exchanges.  Every rank must
    construct it at the same point (it runs collectives) on its own device,
    and then make the same sequence of fused calls.  ``close()`` (also
    collective) unmaps and frees the buffers.
    """

    def __init__(self, group=None, capacity: int = 1 << 16, lib=None, dist=None):
        if dist is None:
            import torch.distributed as dist
        self._dist, self.group = dist, group
        self._lib = lib if lib is not None else _lib.lib()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= MAX_RANKS:
            raise ValueError(f"a peer group holds 1..{MAX_RANKS} ranks, not {self.world}")
        self.capacity = int(capacity)
        L = self._lib
        local = ctypes.c_void_p()
        _lib.check(L.i4b_peer_buffer_alloc(self.capacity, ctypes.byref(local)), "i4b_peer_buffer_alloc")
        self._local = local.value
        handle = (ctypes.c_char * HANDLE_BYTES)()
        _lib.check(L.i4b_ipc_get_handle(self._local, handle), "i4b_ipc_get_handle")
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, (bytes(handle), self.capacity), group=group)
        # the epilogue addresses the other ranks' buffers with this rank's layout: the capacities must agree
        if any(c != self.capacity for _, c in gathered):
            _lib.check(L.i4b_peer_buffer_free(self._local), "i4b_peer_buffer_free")
            raise ValueError(f"peer group capacities differ across ranks: {[c for _, c in gathered]}")
        handles = [h for h, _ in gathered]
        self._opened: list[int] = []
        ptrs = []
        for p, h in enumerate(handles):
            if p == self.rank:
                ptrs.append(self._local)
                continue
            if not isinstance(h, (bytes, bytearray)) or len(h) != HANDLE_BYTES:
                raise RuntimeError(f"rank {p} sent a malformed IPC handle")
            out = ctypes.c_void_p()
            raw = (ctypes.c_char * HANDLE_BYTES).from_buffer_copy(h)
            _lib.check(L.i4b_ipc_open_handle(raw, ctypes.byref(out)), f"i4b_ipc_open_handle(rank {p})")
            ptrs.append(out.value)
            self._opened.append(out.value)
        self.buffers = ptrs
        self.struct = PeerGroupStruct(self.world, self.rank, self.capacity,
                                      (ctypes.c_void_p * MAX_RANKS)(*(ptrs + [None] * (MAX_RANKS - self.world))))
        dist.barrier(group=group)  # every rank has mapped every buffer before any fused call

    def close(self) -> None:
        """Unmap the other ranks' buffers and free this rank's (collective)."""
        if self.struct is None:
            return
        self._dist.barrier(group=self.group)  # no rank still stores into a buffer about to be freed
        for p in self._opened:
            _lib.check(self._lib.i4b_ipc_close_handle(p), "i4b_ipc_close_handle")
        self._opened = []
        self._dist.barrier(group=self.group)
        _lib.check(self._lib.i4b_peer_buffer_free(self._local), "i4b_peer_buffer_free")
        self.struct = None


def w4a16_matmul_allreduce(peers: PeerGroup, x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                           zeros: torch.Tensor, *, prologue: int = 0, delta=None, norm_weight=None,
                           eps: float = 1e-5, resid_out=None) -> torch.Tensor:
    """Sum over the group's ranks of ``x @ W_hat^T`` (this rank's K shard), for 1 <= M <= 32 rows.

    ``prologue`` 0 multiplies x [M, K] (bf16 or fp16); ``PROLOGUE_SWIGLU`` derives the activations from
    x = (g | u) [M, 2K] as ``decode.w4a16_matmul_prologue`` does (RMSNorm needs whole rows, so it is not
    offered for a K shard).  Bit-identical on every rank.
    """
    assert x.is_cuda and x.dim() == 2 and x.stride(-1) == 1
    M = x.shape[0]
    K = qweight.shape[0] * 8
    N = qweight.shape[1]
    G = K // scales.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    st = peers._lib.i4b_w4a16_matmul_allreduce(
        ctypes.byref(peers.struct), prologue, x.data_ptr(), _lib.DTYPE_CODE[x.dtype],
        None if delta is None else delta.data_ptr(), None if norm_weight is None else norm_weight.data_ptr(), eps,
        None if resid_out is None else resid_out.data_ptr(), M, K, x.stride(0), qweight.data_ptr(), N,
        qweight.stride(0), scales.data_ptr(), zeros.data_ptr(), scales.stride(0), G, y.data_ptr(), y.stride(0),
        _lib.stream_handle(x.device))
    _lib.check(st, "w4a16_matmul_allreduce")
    return y


def argmax_allreduce(peers: PeerGroup, x: torch.Tensor, offset: int) -> torch.Tensor:
    """Greedy token of rows split over the ranks: x [rows, n] holds columns [offset, offset + n) of each row.

    Returns int64 [rows, 1], the first index of the maximum of the whole row (torch.argmax), the same on every
    rank, without gathering the rows.
    """
    assert x.is_cuda and x.dim() == 2 and x.dtype == torch.bfloat16 and x.stride(-1) == 1
    rows, n = x.shape
    out = torch.empty((rows, 1), dtype=torch.int64, device=x.device)
    st = peers._lib.i4b_argmax_allreduce(ctypes.byref(peers.struct), x.data_ptr(), rows, n, x.stride(0), offset,
                                         out.data_ptr(), _lib.stream_handle(x.device))
    _lib.check(st, "argmax_allreduce")
    return out
