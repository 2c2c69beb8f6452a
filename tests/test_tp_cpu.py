"""Tensor-parallel partition math of the decode path, on CPU with two ``gloo`` ranks.

The Llama model is sharded as the north star describes: q/k/v/gate/up
column-parallel (slices along N), o/down row-parallel (slices along K) with an
all-reduce.  Checked here against the oracle, without a GPU:

* quantizing a shard gives the same qweight / scales / zeros bits as slicing
  the quantized full weight (rows for column shards; k8 rows and group rows
  for row shards whose width is a multiple of G);
* the all-reduced row-parallel partial products equal the unsharded product,
  and the gathered column-parallel outputs equal it too.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
from oracle import int4_oracle as orc

WORLD = 2
G = 128


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _worker(rank: int, port: int, errors):
    from int4_b200.decode import column_shard, head_shard, row_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        N, K = 512, 1024
        w = cases.weight((N, K), "bfloat16", seed=11, outlier_frac=1e-3)
        x = cases.activations(3, K, "bfloat16", seed=12)
        qw, s, z = orc.quantize_int4(_bits(w), G, "bfloat16")
        full = orc.w4a16_matmul(_bits(x), qw, s, z)

        # column-parallel: this rank's output features
        wc = column_shard(w, rank, WORLD)
        qc = orc.quantize_int4(_bits(wc), G, "bfloat16")
        n0, n1 = rank * N // WORLD, (rank + 1) * N // WORLD
        np.testing.assert_array_equal(qc[0], qw[:, n0:n1])
        np.testing.assert_array_equal(qc[1], s[:, n0:n1])
        np.testing.assert_array_equal(qc[2], z[:, n0:n1])
        yc = torch.from_numpy(np.ascontiguousarray(orc.w4a16_matmul(_bits(x), *qc)))
        parts = [torch.empty_like(yc) for _ in range(WORLD)]
        dist.all_gather(parts, yc)
        assert orc.rel_fro_error(torch.cat(parts, 1).numpy(), full) < 1e-6

        # row-parallel: this rank's input features, then an all-reduce of the partial products
        wr = row_shard(w, rank, WORLD)
        qr = orc.quantize_int4(_bits(wr), G, "bfloat16")
        k0, k1 = rank * K // WORLD, (rank + 1) * K // WORLD
        np.testing.assert_array_equal(qr[0], qw[k0 // 8:k1 // 8])
        np.testing.assert_array_equal(qr[1], s[k0 // G:k1 // G])
        np.testing.assert_array_equal(qr[2], z[k0 // G:k1 // G])
        yr = torch.from_numpy(np.ascontiguousarray(orc.w4a16_matmul(_bits(x[:, k0:k1]), *qr)))
        dist.all_reduce(yr)
        assert orc.rel_fro_error(yr.numpy(), full) < 1e-6

        # head shards of a q projection are column shards at head granularity
        hq = head_shard(w, 8, 64, rank, WORLD)
        assert torch.equal(hq, w[rank * 256:(rank + 1) * 256])
    except Exception as e:  # reported to the parent
        errors.append(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_match_the_unsharded_oracle():
    ctx = mp.get_context("spawn")
    errors = ctx.Manager().list()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, errors)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert not list(errors), list(errors)
    assert codes == [0] * WORLD, codes


def test_row_shard_rejects_uneven_splits():
    from int4_b200.decode import column_shard, row_shard

    w = torch.zeros(6, 10)
    with pytest.raises(AssertionError):
        row_shard(w, 0, 4)
    with pytest.raises(AssertionError):
        column_shard(w, 0, 4)


def test_fused_row_parallel_sum_falls_back_to_nccl_only_on_a_refused_shape(monkeypatch):
    """``LlamaTP``'s per-launch decode sums the o / down outputs inside the matmul; when the library refuses
    the shape (its grid cannot be resident at once: I4B_ERR_SHAPE, decided on the host from the plan, the same
    on every rank) it answers None and turns the fused sums off for later steps, so every rank takes NCCL's
    all-reduce together.  Any other failure propagates.  The library call is replaced by a fake here."""
    from types import SimpleNamespace

    from int4_b200 import decode
    from int4_b200._lib import STATUS_SHAPE, Int4B200Error

    calls = []

    def fake(peers, x, qw, s, z, *, prologue=0):
        calls.append(prologue)
        if fake.mode == "ok":
            return x + 1
        raise Int4B200Error("w4a16_matmul_allreduce: refused", fake.status)

    monkeypatch.setattr(decode, "w4a16_matmul_allreduce", fake)
    helper = decode.LlamaTP._matmul_allreduce_or_none
    me = SimpleNamespace(peers=object(), matmul_allreduce=True)
    x = torch.zeros(1, 4)
    q = (None, None, None)

    fake.mode, fake.status = "ok", 0
    assert torch.equal(helper(me, x, q), x + 1) and me.matmul_allreduce
    assert torch.equal(helper(me, x, q, decode.PROLOGUE_SWIGLU), x + 1) and calls == [0, decode.PROLOGUE_SWIGLU]

    fake.mode, fake.status = "refuse", STATUS_SHAPE
    assert helper(me, x, q) is None and me.matmul_allreduce is False

    me.matmul_allreduce = True
    fake.status = 6  # a CUDA error is not a refusal
    with pytest.raises(Int4B200Error):
        helper(me, x, q)
    assert me.matmul_allreduce is True
