"""One rank of the fused tensor-parallel all-reduce check (launched by tests/test_allreduce_gpu.py via torchrun).

Every rank builds the same seeded full weight W[N, K], quantizes it on the GPU
and keeps its row-parallel shard (K / world columns of W: k8 rows of qweight,
group rows of scales / zeros).  ``w4a16_matmul_allreduce`` of the rank's slice
of x must then give, on every rank:

* the full product within 1e-2 relative Frobenius error of the fp32 oracle
  ``x.float() @ dequantize_int4_ref(qweight, scales, zeros, fp32).t()`` (the
  reference tests' expression, tests/test_kernels.py:54-57);
* the same bits on every rank, and on four calls in a row (the exchange
  slots alternate between calls);
* the same bits when replayed from a CUDA graph.

The SwiGLU prologue (down_proj of a Llama MLP, gate | up sliced per rank) is
checked the same way against torch's ``silu(g) * u``; ``argmax_allreduce`` of
rows split over the ranks against torch.argmax of the whole row (ties across
and within ranks, an all -inf row).  Exit status 0 only if
every check holds on every rank and no bounded wait expired.
"""
from __future__ import annotations

import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "itmo-final-project_b200"), HERE, os.path.join(HERE, "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402
import torch.nn.functional as F  # noqa: E402

SHAPES = [(2048, 2048, 128), (2048, 8192, 128), (264, 1024, 64), (72, 512, 32)]  # N, K, G
TOKENS = (1, 3, 8, 16, 32)


def rel_fro(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()


def same_on_all_ranks(y: torch.Tensor, world: int) -> bool:
    parts = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(parts, y.contiguous())
    ref = parts[0].view(torch.int16)
    return all(torch.equal(p.view(torch.int16), ref) for p in parts[1:])


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import cases
    from int4_b200 import _lib, dequantize_int4_ref, quantize_int4
    from int4_b200.decode import PROLOGUE_SWIGLU
    from int4_b200.peer import PeerGroup, w4a16_matmul_allreduce

    peers = PeerGroup(None, capacity=32 * 2048)
    failures = []
    worst = 0.0
    with torch.no_grad():
        for N, K, G in SHAPES:
            w = cases.weight((N, K), "bfloat16", seed=N + K, outlier_frac=1e-3).to(dev)
            qf, sf, zf = quantize_int4(w, G)
            wdq = dequantize_int4_ref(qf, sf, zf, torch.float32)  # [N, K] fp32, exact
            ks = K // world
            k0 = rank * ks
            q = qf[k0 // 8:(k0 + ks) // 8].contiguous()
            s = sf[k0 // G:(k0 + ks) // G].contiguous()
            z = zf[k0 // G:(k0 + ks) // G].contiguous()
            for M in TOKENS:
                x = cases.activations(M, K, "bfloat16", seed=M + N).to(dev)
                ref = x.float() @ wdq.t()
                ys = [w4a16_matmul_allreduce(peers, x[:, k0:k0 + ks].contiguous(), q, s, z) for _ in range(4)]
                err = rel_fro(ys[0], ref)
                worst = max(worst, err)
                if err > 1e-2:
                    failures.append(f"N={N} K={K} G={G} M={M}: rel err {err:.3e}")
                if not all(torch.equal(y.view(torch.int16), ys[0].view(torch.int16)) for y in ys[1:]):
                    failures.append(f"N={N} K={K} M={M}: repeated calls differ")
                if not same_on_all_ranks(ys[0], world):
                    failures.append(f"N={N} K={K} M={M}: ranks differ")
            # SwiGLU prologue: this rank's gate | up slices of an MLP whose down_proj is W
            for M in (1, 8):
                gu = cases.activations(M, 2 * K, "bfloat16", seed=7 + M).to(dev)
                g_full, u_full = gu[:, :K], gu[:, K:]
                act = F.silu(g_full) * u_full  # transformers' LlamaMLP in bf16
                ref = act.float() @ wdq.t()
                src = torch.cat([g_full[:, k0:k0 + ks], u_full[:, k0:k0 + ks]], dim=1).contiguous()
                y = w4a16_matmul_allreduce(peers, src, q, s, z, prologue=PROLOGUE_SWIGLU)
                err = rel_fro(y, ref)
                worst = max(worst, err)
                if err > 1e-2:
                    failures.append(f"SwiGLU N={N} K={K} M={M}: rel err {err:.3e}")
                if not same_on_all_ranks(y, world):
                    failures.append(f"SwiGLU N={N} K={K} M={M}: ranks differ")
        # CUDA-graph replay of two fused calls (o / down shapes) equals the eager result
        N, K, G = SHAPES[0]
        w = cases.weight((N, K), "bfloat16", seed=5, outlier_frac=1e-3).to(dev)
        qf, sf, zf = quantize_int4(w, G)
        ks = K // world
        k0 = rank * ks
        q, s, z = (qf[k0 // 8:(k0 + ks) // 8].contiguous(), sf[k0 // G:(k0 + ks) // G].contiguous(),
                   zf[k0 // G:(k0 + ks) // G].contiguous())
        x = cases.activations(4, ks, "bfloat16", seed=11 + rank).to(dev)
        eager = w4a16_matmul_allreduce(peers, x, q, s, z)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            a = w4a16_matmul_allreduce(peers, x, q, s, z)
            b = w4a16_matmul_allreduce(peers, x, q, s, z)
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            if not (torch.equal(a.view(torch.int16), eager.view(torch.int16))
                    and torch.equal(b.view(torch.int16), eager.view(torch.int16))):
                failures.append("graph replay differs from the eager call")
                break
        del graph
        # greedy token of rows split over the ranks (vocab-parallel lm_head), against torch.argmax of the row
        from int4_b200.peer import argmax_allreduce

        V = 1000 * world + 8 * world  # each rank holds V / world columns
        vl = V // world
        full = cases.activations(6, V, "bfloat16", seed=21).to(dev)
        full[1, :] = float("-inf")                        # nothing above -inf: index 0, as torch.argmax
        full[2, 5] = full[2, vl + 7] = 30.0               # equal maxima on two ranks: the lower index
        full[3, vl * (world - 1) + 3] = 40.0              # the maximum on the last rank
        full[4, 10] = full[4, 11] = 50.0                  # equal maxima inside one rank
        full[5, V - 1] = 60.0                             # the last column
        ref = full.float().argmax(-1, keepdim=True)
        for _ in range(2):
            got = argmax_allreduce(peers, full[:, rank * vl:(rank + 1) * vl].contiguous(), rank * vl)
            if not torch.equal(got, ref):
                failures.append(f"argmax_allreduce {got.view(-1).tolist()} != {ref.view(-1).tolist()}")
                break
    flags = _lib.device_error_flags(local)
    if flags:
        failures.append(f"device error flags {flags}")
    peers.close()
    bad = torch.tensor([float(len(failures)), worst], device=dev)
    dist.all_reduce(bad, op=dist.ReduceOp.MAX)
    torch.cuda.synchronize()
    dist.destroy_process_group()
    for f in failures:
        print(f"rank {rank}: {f}")
    if rank == 0:
        print(f"fused all-reduce, {world} ranks: worst rel Frobenius error {bad[1].item():.3e}, "
              f"{int(bad[0].item())} failing checks on the worst rank")
    return 0 if bad[0].item() == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
