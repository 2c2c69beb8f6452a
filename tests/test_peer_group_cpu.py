"""Host logic of ``int4_b200.peer.PeerGroup`` on two ``gloo`` ranks, without a GPU.

The C library is replaced by a fake that records calls: buffer allocation,
the 64-byte CUDA-IPC handle of each rank's buffer, and the mapping of the
other ranks' handles.  Checked: every rank ends with a table in which slot p
holds rank p's buffer (its own allocation for itself, the mapping of rank p's
handle otherwise); world, rank and capacity are those of the group; ``close``
unmaps exactly what was mapped and frees the local buffer, after a barrier.
"""
from __future__ import annotations

import ctypes
import os
import socket
import struct

import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2
CAP = 4096


class FakeLib:
    """Stands in for libint4_b200.so: pointers are plain integers, handles encode (rank, pointer)."""

    def __init__(self, rank: int):
        self.rank = rank
        self.calls: list[tuple] = []

    def i4b_peer_buffer_alloc(self, capacity, out):
        self.calls.append(("alloc", capacity))
        ctypes.cast(out, ctypes.POINTER(ctypes.c_void_p))[0] = 0x10000000 * (self.rank + 1)
        return 0

    def i4b_ipc_get_handle(self, ptr, handle):
        self.calls.append(("handle", ptr))
        ctypes.memmove(handle, struct.pack("<qq", self.rank, ptr) + b"\0" * 48, 64)
        return 0

    def i4b_ipc_open_handle(self, handle, out):
        src, ptr = struct.unpack("<qq", bytes(handle)[:16])
        mapped = 0x7000000000 + ptr  # where the other rank's buffer appears in this process
        self.calls.append(("open", src))
        ctypes.cast(out, ctypes.POINTER(ctypes.c_void_p))[0] = mapped
        return 0

    def i4b_ipc_close_handle(self, ptr):
        self.calls.append(("close", ptr))
        return 0

    def i4b_peer_buffer_free(self, ptr):
        self.calls.append(("free", ptr))
        return 0


def _worker(rank: int, port: int, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    from int4_b200.peer import PeerGroup

    fake = FakeLib(rank)
    g = PeerGroup(None, capacity=CAP, lib=fake, dist=dist)
    table = [g.struct.buffers[i] for i in range(8)]
    info = (g.struct.world, g.struct.rank, g.struct.capacity)
    g.close()
    g.close()  # idempotent
    results[rank] = (table, info, fake.calls)
    dist.destroy_process_group()


def test_peer_group_maps_every_rank_buffer():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    results = mp.Manager().dict()
    mp.spawn(_worker, args=(port, results), nprocs=WORLD, join=True)
    for rank in range(WORLD):
        table, info, calls = results[rank]
        assert info == (WORLD, rank, CAP)
        for p in range(WORLD):
            own = 0x10000000 * (p + 1)
            assert table[p] == (own if p == rank else 0x7000000000 + own), (rank, p, table)
        assert all(t is None for t in table[WORLD:])
        other = 0x7000000000 + 0x10000000 * (2 - rank)
        assert calls == [("alloc", CAP), ("handle", 0x10000000 * (rank + 1)), ("open", 1 - rank),
                         ("close", other), ("free", 0x10000000 * (rank + 1))], calls
