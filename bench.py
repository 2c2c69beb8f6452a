"""Benchmark of the B200-native W4A16 path (one JSON line on rank 0).

Workload ``block``: the seven linears of one
Llama-3.2-1B-shaped decoder block (q/k/v/o 2048-wide, gate/up 8192, down
K=8192), weights N(0, 0.02) with 0.1% of entries x10, INT4 G=128, bf16
activations.  A step runs them as the tensor-parallel dataflow of the block,
the linears that share an input stacked into one projection (four launches):

    q|k|v = x @ [Wq;Wk;Wv]^T        (column shards, N / world)
    o = q @ Wo^T ; all-reduce(o)    (row shard, K / world; NCCL when world > 1)
    g|u = o @ [Wgate;Wup]^T         (column shards)
    d = g @ Wdown^T ; all-reduce(d) (row shard)

At M = 1 this is one decoder block's decode-step GEMV work (32.4 MB of packed
weights).  Steps are captured in one CUDA graph and cycle through enough
copies of the weights that the working set exceeds the 126 MB L2, so every
step streams its weights from HBM.  ``value`` is the block time in
microseconds (max over ranks); ``roofline`` relates the algorithmic bytes
(N*K/2 + 4*N*K/G + 2*M*K + 2*M*N per linear) to the measured HBM peak.

``--impl reference`` times the reference's CPU path (the numpy restatement
of ``x.float() @ dequantize_int4_ref(...).t()`` in ``oracle/``) on the same
configuration with all host threads, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "itmo-final-project_b200"), os.path.join(ROOT, "tests", "golden")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

BLOCK = [  # name, N, K, column-parallel?
    ("q_proj", 2048, 2048, True),
    ("k_proj", 512, 2048, True),
    ("v_proj", 512, 2048, True),
    ("o_proj", 2048, 2048, False),
    ("gate_proj", 8192, 2048, True),
    ("up_proj", 8192, 2048, True),
    ("down_proj", 2048, 8192, False),
]
GROUP = 128
L2_BYTES = 126 * 1024 * 1024


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def alg_bytes(M, N, K, G=GROUP) -> int:
    return N * K // 2 + 4 * N * K // G + 2 * M * K + 2 * M * N


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        # the first sample can take a second (nvidia-smi start-up): wait for it, then 0.2 s more
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < 3.0:
            time.sleep(0.05)
        time.sleep(0.2)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = max(smax, float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- distributed


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ----------------------------------------------------------------------------- block workload


def block_weights(rank: int, world: int, copies: int, dev):
    """Per-rank shards of the seven linears, quantized on the GPU, ``copies`` rotating copies."""
    import cases
    import int4_b200 as ib

    layers = []
    for li, (name, N, K, colpar) in enumerate(BLOCK):
        w = cases.weight((N, K), "bfloat16", seed=100 + li, outlier_frac=1e-3)
        if colpar:
            n0, n1 = rank * N // world, (rank + 1) * N // world
            w = w[n0:n1]
        else:
            k0, k1 = rank * K // world, (rank + 1) * K // world
            w = w[:, k0:k1]
        qs = [ib.quantize_int4(w.contiguous().to(dev), GROUP)]
        for _ in range(copies - 1):
            qs.append(tuple(t.clone() for t in qs[0]))
        layers.append((name, w.shape[0], w.shape[1], qs))
    # q|k|v and gate|up share their input: each group runs as one stacked projection (quantization is per
    # output column, so stacking the quantized tensors is the same bits as quantizing the stacked weight)
    def stack(ids):
        n = sum(layers[i][1] for i in ids)
        qs = [tuple(torch.cat([layers[i][3][c][t] for i in ids], dim=1) for t in range(3)) for c in range(copies)]
        return ("|".join(layers[i][0] for i in ids), n, layers[ids[0]][2], qs, [layers[i][1] for i in ids])
    return [stack([0, 1, 2]), layers[3] + ([layers[3][1]],), stack([4, 5]), layers[6] + ([layers[6][1]],)]


def block_step(x, layers, copy: int, world: int, peers=None):
    """The block's dataflow as four launches: q|k|v, o_proj, gate|up, down_proj.

    Under TP the row-parallel o / down outputs are summed over the ranks inside their matmuls when a peer
    group is given (``w4a16_matmul_allreduce``: fp32 partials through peer exchange buffers), else by an
    NCCL all-reduce after them.
    """
    import int4_b200 as ib
    from int4_b200.peer import w4a16_matmul_allreduce

    def mm(i, inp):
        qw, s, z = layers[i][3][copy]
        return ib.w4a16_matmul(inp, qw, s, z)

    def mm_sum(i, inp):
        if world == 1:
            return mm(i, inp)
        if peers is not None:
            qw, s, z = layers[i][3][copy]
            return w4a16_matmul_allreduce(peers, inp, qw, s, z)
        import torch.distributed as dist

        out = mm(i, inp)
        dist.all_reduce(out)
        return out

    qkv = mm(0, x)
    o = mm_sum(1, qkv[:, :layers[0][4][0]])
    gu = mm(2, o)
    return mm_sum(3, gu[:, :layers[2][4][0]])


def run_block(args, world, rank, local):
    import int4_b200 as ib
    from int4_b200 import _lib

    dev = torch.device("cuda", local)
    M = args.m
    shard_bytes = sum(alg_bytes(M, N, K) for (_, N, K, _) in
                      [(n, (N // world if c else N), (K if c else K // world), c) for (n, N, K, c) in BLOCK])
    copies = max(2, math.ceil(2 * L2_BYTES / max(1, shard_bytes - 2 * M * 2048)))
    copies = min(copies, 64)
    layers = block_weights(rank, world, copies, dev)
    g = torch.Generator().manual_seed(1)
    x = torch.randn((M, 2048), generator=g).to(torch.bfloat16).to(dev)
    peers = None
    if world > 1 and args.peer_allreduce != 0 and M <= 32:
        from int4_b200.peer import PeerGroup

        peers = PeerGroup(None, capacity=M * 2048)

    # One graph holds `chunk` steps (a divisor of K, at most 200); the timed
    # region replays it K / chunk times, i.e. exactly K steps.
    chunk = max(d for d in range(1, min(args.steps, 200) + 1) if args.steps % d == 0)
    reps = args.steps // chunk
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):  # warm-up (eager) on the capture stream: workspace, module load
        for i in range(args.warmup):
            block_step(x, layers, i % copies, world, peers)
    torch.cuda.synchronize()

    def capture(fn):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            for i in range(chunk):
                fn(i)
        gr.replay()  # upload / first replay, untimed
        torch.cuda.synchronize()
        return gr

    def timed(gr, clocks=None):
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        torch.cuda.nvtx.range_push("timed")  # lets a profiler select the timed launches
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        barrier(world)
        return e0.elapsed_time(e1) * 1e-3, wall

    graph = capture(lambda i: block_step(x, layers, i % copies, world, peers))
    # The timed region lasts well under a millisecond, shorter than the sampling period: the clocks are
    # sampled over ~0.3 s of the same replays (untimed, the same count on every rank) on both sides of it.
    t_est = max_over_ranks(timed(graph)[0], world)
    n_soak = max(1, min(20000, int(0.3 * reps / max(t_est, 1e-6))))

    def soak():
        for i in range(n_soak):
            graph.replay()
            if i % 64 == 63:
                torch.cuda.synchronize()
        torch.cuda.synchronize()

    with ClockSampler(local) as clk:
        soak()
        t_dev, _ = timed(graph)
        soak()
    us_per_step = max_over_ranks(t_dev, world) * 1e6 / args.steps

    # L2-hot variant (the reference's timing method: the same weights every step)
    graph_hot = capture(lambda i: block_step(x, layers, 0, world, peers))
    hot_us = max_over_ranks(timed(graph_hot)[0], world) * 1e6 / args.steps

    # End to end through the public API: pinned host x in, block output back to the host, every step.
    x_host = torch.randn((M, 2048), generator=g).to(torch.bfloat16).pin_memory()
    y_host = torch.empty((M, 2048), dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step(i):
        x_dev.copy_(x_host, non_blocking=True)
        d = block_step(x_dev, layers, i % copies, world, peers)
        y_host.copy_(d, non_blocking=True)

    graph_e2e = capture(e2e_step)
    t_dev, wall = timed(graph_e2e)
    e2e_us = max_over_ranks(max(t_dev, wall), world) * 1e6 / args.steps

    flags = _lib.device_error_flags(local)
    if peers is not None:
        del graph, graph_hot, graph_e2e
        graph = graph_hot = graph_e2e = None
        peers.close()
    # algorithmic bytes / flops of the seven linears (shard shapes), as the metric defines them
    shards = [((N // world if c else N), (K if c else K // world)) for (_, N, K, c) in BLOCK]
    total_bytes = sum(alg_bytes(M, n, k) for (n, k) in shards)
    total_flops = sum(2 * M * n * k for (n, k) in shards)
    del graph, graph_hot, graph_e2e
    return {
        "us_per_step": us_per_step, "hot_us": hot_us, "e2e_us": e2e_us, "clocks": clk.summary(),
        "bytes_per_step_rank": total_bytes, "flops_per_step_rank": total_flops, "copies": copies,
        "launches_per_step": len(layers), "device_error_flags": flags,
        "tp_sum": "none" if world == 1 else ("in the o/down matmuls (peer buffers)" if peers is not None
                                            else "NCCL all-reduce"),
        "h2d": M * 2048 * 2, "d2h": M * 2048 * 2,
    }


def cpu_block_sample(M: int, threads: int, steps: int = 1, warmup: int = 1) -> tuple[float, str]:
    """The reference's CPU path for the whole block at M tokens, seconds per block: each linear is
    ``x.float() @ dequantize_int4_ref(qweight, scales, zeros, torch.float32).t()`` (the reference tests'
    expression, ``tests/test_kernels.py:54-57``), its output rounded to bf16 for the next linear.  The helper is
    the oracle's torch restatement of ``dequantize_int4_ref`` (``int4_triton/quantize.py:120-135``); torch runs
    the matmuls on ``threads`` host threads.  Quantization (``quantize_int4_ref``) is set-up, not timed."""
    import cases
    from oracle import int4_torch as ot

    torch.set_num_threads(threads)
    qs = []
    for li, (name, N, K, _) in enumerate(BLOCK):
        qs.append(ot.quantize_int4(cases.weight((N, K), "bfloat16", seed=100 + li, outlier_frac=1e-3), GROUP))
    x = cases.activations(M, 2048, "bfloat16", seed=1)

    def lin(inp, i):
        return (inp.float() @ ot.dequantize_int4(*qs[i], dtype=torch.float32).t()).to(torch.bfloat16)

    def step():
        q = lin(x, 0)
        lin(x, 1)
        lin(x, 2)
        o = lin(q, 3)
        gg = lin(o, 4)
        lin(o, 5)
        lin(gg, 6)

    for _ in range(warmup):  # untimed
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    return dt, (f"{steps} full block step(s) at M={M} after {warmup} untimed: 7 x (dequantize_int4_ref to fp32, then "
                f"x.float() @ W^T), torch on {threads} threads")


# ----------------------------------------------------------------------------- model workload

LLAMA_1B = dict(vocab_size=128256, hidden_size=2048, intermediate_size=8192, num_hidden_layers=16,
                num_attention_heads=32, num_key_value_heads=8, head_dim=64, max_position_embeddings=131072,
                rms_norm_eps=1e-5, tie_word_embeddings=True, rope_theta=500000.0,
                rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                              "original_max_position_embeddings": 8192})


def build_llama(dev, seed: int = 0):
    """Random-init Llama-3.2-1B-shaped model (transformers' init: N(0, 0.02) weights, RMSNorm weights 1), bf16."""
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(seed)
    with torch.device(dev):
        model = LlamaForCausalLM(LlamaConfig(**LLAMA_1B))
    return model.to(torch.bfloat16).eval()


def time_decode(m, B: int, prompt: int, steps: int, warmup: int, world: int, dev, vocab: int, trace: bool = False):
    """Prefill ``prompt`` random tokens, then time ``steps`` greedy decode steps replayed from a CUDA graph."""
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, vocab, (B, prompt), generator=g).to(dev)
    m.prefill(ids)  # untimed: module loading, workspaces, library heuristics
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    logits = m.prefill(ids)
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(e0.elapsed_time(e1), world)
    from int4_b200.decode import argmax_last

    tok = argmax_last(logits[:, -1])
    first = tok.clone()
    pos = torch.tensor([prompt], device=dev)

    def step():
        tok.copy_(m.decode_greedy(tok, pos))
        pos.add_(1)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(warmup):
            step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step()

    def reset():
        m.prefill(ids)
        tok.copy_(first)
        pos.fill_(prompt)
        torch.cuda.synchronize()

    reset()
    barrier(world)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("timed")  # lets a profiler select the timed launches
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    dev_s = max_over_ranks(e0.elapsed_time(e1) * 1e-3, world)

    # end to end: every step copies the input token in from pinned host memory and the next token back out
    reset()
    tok_in = torch.empty((B, 1), dtype=torch.long).pin_memory()
    tok_in.copy_(first.cpu())
    tok_out = torch.empty((B, 1), dtype=torch.long).pin_memory()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        tok.copy_(tok_in, non_blocking=True)
        graph.replay()
        tok_out.copy_(tok, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    e2e_s = max_over_ranks(max(wall, e0.elapsed_time(e1) * 1e-3), world)
    del graph
    res = {"prefill_ms": prefill_ms, "decode_s": dev_s, "e2e_s": e2e_s, "h2d": B * 8, "d2h": B * 8}
    if trace and getattr(m, "persistent", None) is not None:
        reset()
        res["trace"] = m.persistent.trace(tok, pos)
    return res


def run_model(args, world, rank, local, B=None, steps=None, nll=False):
    """W4 (and, with --compare-bf16, bf16) decode of the Llama-3.2-1B-shaped model; optionally the config-4
    mean-NLL check afterwards on the same random-init weights."""
    from int4_b200.decode import LlamaTP

    dev = torch.device("cuda", local)
    B = args.m if B is None else B
    steps = args.steps if steps is None else steps
    prompt = args.prompt
    hf = build_llama(dev)
    res = {}
    for label, w4 in (("w4", True), ("bf16", False))[:2 if args.compare_bf16 else 1]:
        persistent = None if args.persistent < 0 else bool(args.persistent) and w4
        m = LlamaTP(hf, w4=w4, quantize_lm_head=w4 and args.lm_head_w4, rank=rank, world=world, persistent=persistent,
                    peer_allreduce=args.peer_allreduce != 0,
                    matmul_allreduce=args.peer_allreduce == 1 or (args.peer_allreduce < 0 and B <= 8),
                    max_seq=prompt + steps + args.warmup + 8, max_batch=B, device=dev)
        with ClockSampler(local) as clk:
            r = time_decode(m, B, prompt, steps, args.warmup, world, dev, LLAMA_1B["vocab_size"],
                            trace=bool(args.trace) and w4)
        r["clocks"] = clk.summary()
        r["persistent"] = m.persistent is not None
        if world == 1:
            r["tp_sum"] = "none"
        elif m.persistent is not None:
            r["tp_sum"] = "inside the persistent decode launch (peer buffers)"
        elif m.peers is not None and m.matmul_allreduce:
            r["tp_sum"] = "inside the o/down matmuls (peer buffers)"
        else:
            r["tp_sum"] = "NCCL all-reduce"
        r["greedy"] = "argmax exchange (peer buffers)" if world > 1 and m.peers is not None else \
            ("logits all-gather + argmax" if world > 1 else "argmax")
        m.close()
        # bytes one decode step must read on this rank: projection weights + the KV cache up to the mean position
        mean_pos = prompt + steps / 2
        kv = 2 * len(m.layers) * m.nkv_l * m.hd * 2 * B * mean_pos
        r["bytes_per_step_rank"] = m.weight_bytes() + kv
        res[label] = r
        del m
        torch.cuda.empty_cache()
    if nll:
        res["nll"] = model_nll(hf, world, rank, dev)
    del hf
    torch.cuda.empty_cache()
    return res


NLL_SEQS, NLL_LEN = 8, 2048


@torch.no_grad()
def model_nll(hf, world: int, rank: int, dev) -> dict:
    """BASELINE config 4's quality check: mean next-token NLL over 8 seeded random 2048-token sequences, the W4
    model's prompt pass (this library, tensor-parallel when world > 1) against the fake-quant model
    (``quantize_model_linears(fake=True)``: the same dequantized weights run by transformers with cuBLAS), as the
    reference's ``eval_ppl`` computes it (``benchmarks/eval_llama.py:77-117``).  Random tokens on a random-init
    model stand in for WikiText-2 and the checkpoint."""
    import copy

    import torch.nn.functional as F

    import int4_b200 as ib
    from int4_b200.decode import LlamaTP

    g = torch.Generator().manual_seed(2024)
    ids = torch.randint(0, LLAMA_1B["vocab_size"], (NLL_SEQS, NLL_LEN), generator=g).to(dev)
    m = LlamaTP(hf, w4=True, group_size=GROUP, rank=rank, world=world, max_seq=NLL_LEN, max_batch=1, device=dev,
                persistent=False)
    nw4 = 0.0
    for i in range(NLL_SEQS):
        lw = m.prefill(ids[i:i + 1], all_logits=True)[0, :-1].float()
        nw4 += F.cross_entropy(lw, ids[i, 1:], reduction="sum").item()
        del lw
    m.close()
    del m
    fake = copy.deepcopy(hf)
    ib.quantize_model_linears(fake, GROUP, skip=("lm_head",), fake=True)
    nref = 0.0
    for i in range(NLL_SEQS):
        lr = fake(ids[i:i + 1], use_cache=False).logits[0, :-1].float()
        nref += F.cross_entropy(lr, ids[i, 1:], reduction="sum").item()
        del lr
    del fake
    torch.cuda.empty_cache()
    tok = NLL_SEQS * (NLL_LEN - 1)
    return {"w4": nw4 / tok, "fake_quant_reference": nref / tok, "abs_diff": abs(nw4 - nref) / tok,
            "sequences": NLL_SEQS, "seq_len": NLL_LEN, "tolerance": 1e-3}


def cpu_model_sample(threads: int, B: int = 1, steps: int = 2) -> tuple[float, str]:
    """The reference's model-level CPU path: the fake-quant Llama-3.2-1B (decoder linears replaced by their
    dequantized INT4 round trip, G=128, ``quantize_model_linears(fake=True)`` semantics restated by the oracle's
    torch helpers) in transformers on the host cores; seconds per decode step after a 32-token prompt."""
    from oracle import int4_torch as ot

    torch.set_num_threads(threads)
    hf = build_llama("cpu")
    with torch.no_grad():
        ot.fake_quantize_model_(hf, GROUP, skip=("lm_head",))
        ids = torch.randint(0, LLAMA_1B["vocab_size"], (B, 32), generator=torch.Generator().manual_seed(7))
        out = hf(ids, use_cache=True)
        past = out.past_key_values
        tok = out.logits[:, -1:].argmax(-1)
        t0 = time.perf_counter()
        for _ in range(steps):
            out = hf(tok, past_key_values=past, use_cache=True)
            past = out.past_key_values
            tok = out.logits[:, -1:].argmax(-1)
        dt = (time.perf_counter() - t0) / steps
    return dt, f"{steps} greedy decode steps of the fake-quant (dequantized W4 G={GROUP}) model in transformers, " \
               f"batch {B}, after a 32-token prompt, {threads} threads"


MODEL_METRIC = "W4 decode tokens/s (Llama-3.2-1B shape)"


def model_config(args) -> dict:
    return {"workload": f"llama-3.2-1b random-init, W4 G={GROUP} decoder linears"
                        f"{' + W4 lm_head' if args.lm_head_w4 else ', bf16 lm_head'}, batch {args.m}, "
                        f"{args.prompt}-token prompt then greedy decode (CUDA graph per step)",
            "model": "Llama-3.2-1B-shaped (random-init)", "group_size": GROUP, "global_batch": args.m,
            "seq_len": args.prompt, "parallelism": f"tp{args.gpus}", "pdl": bool(args.pdl),
            "l2": "inputs larger than L2: 0.65-1 GB of weights streamed per step"}


def main_model(args, world, rank, local, threads):
    res = run_model(args, world, rank, local)
    if rank != 0:
        return
    pk = peaks()
    w4, bf = res["w4"], res.get("bf16")
    if "trace" in w4:
        print(json.dumps({"persistent_decode_trace": w4["trace"]}), file=sys.stderr, flush=True)
    tps = args.m * args.steps / w4["decode_s"]
    step_s = w4["decode_s"] / args.steps
    achieved = w4["bytes_per_step_rank"] / step_s / 1e9
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        dt, sample = cpu_model_sample(threads, args.m, 2)
        cpu = {"value": args.m / dt, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample}
    line = {
        "metric": MODEL_METRIC, "value": tps, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "w4a16-bf16", "data": "synthetic (random-init weights, random token ids)",
        "config": dict(model_config(args), decode="one launch for all layers (i4b_decode_layers)"
                       if w4["persistent"] else "one launch per projection / glue op",
                       tp_sum=w4["tp_sum"], greedy=w4["greedy"]),
        "bf16_tokens_per_s": args.m * args.steps / bf["decode_s"] if bf else None,
        "w4_over_bf16": bf["decode_s"] / w4["decode_s"] if bf else None,
        "prefill_ms": {"w4": w4["prefill_ms"], "bf16": bf["prefill_ms"] if bf else None},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"], "traffic": None,
                     "kernel": "whole decode step (projection weights + KV cache bytes / step time)",
                     "peak_source": pk["source"]},
        "cpu_baseline": cpu,
        "e2e": {"value": args.m * args.steps / w4["e2e_s"], "unit": "tokens/s", "h2d_bytes_per_step": w4["h2d"],
                "d2h_bytes_per_step": w4["d2h"]},
        "clocks": w4["clocks"],
    }
    print(json.dumps(line), flush=True)


def decode_summary(args, dec: dict, world: int) -> dict:
    """The config-4 decode numbers measured inside the block run (W4 tokens/s is BASELINE's lead metric)."""
    if "error" in dec:
        return {"metric": MODEL_METRIC, "error": dec["error"]}
    pk = peaks()
    w4, bf = dec["w4"], dec.get("bf16")
    steps = args.decode_steps
    step_s = w4["decode_s"] / steps
    achieved = w4["bytes_per_step_rank"] / step_s / 1e9
    out = {
        "metric": MODEL_METRIC, "tokens_per_s": steps / w4["decode_s"], "unit": "tokens/s", "steps": steps,
        "ms_per_token": step_s * 1e3, "batch": 1, "prompt": args.prompt,
        "bf16_tokens_per_s": steps / bf["decode_s"] if bf else None,
        "w4_over_bf16": bf["decode_s"] / w4["decode_s"] if bf else None,
        "e2e_tokens_per_s": steps / w4["e2e_s"],
        "prefill_ms": {"w4": w4["prefill_ms"], "bf16": bf["prefill_ms"] if bf else None},
        "decode": "one launch for all layers (i4b_decode_layers)" if w4["persistent"] else
                  "one launch per projection / glue op",
        "tp_sum": w4["tp_sum"], "greedy": w4["greedy"], "lm_head": "bf16 (cuBLAS)",
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"],
                     "kernel": "whole decode step: projection weights + lm_head + KV cache bytes per rank / step time"},
        "clocks": w4["clocks"],
    }
    if "nll" in dec:
        out["nll"] = dec["nll"]
    return out


COMPARE_M = (1, 8, 32, 128, 1024)


def main_compare(args, world, rank, local, threads):
    """BASELINE config 2 as the reference's benchmark tabulates it (``benchmarks/bench_gemm.py:46-60``): device
    time of the block's seven linears per M, W4 (this library) next to torch bf16 (cuBLAS) and W16 (this library's
    full-precision path), weights rotated past L2; one JSON line per M on rank 0 (one GPU: no tensor parallelism)."""
    import cases
    import int4_b200 as ib
    import torch.nn.functional as F

    dev = torch.device("cuda", local)
    lin = []
    for li, (name, N, K, _) in enumerate(BLOCK):
        w = cases.weight((N, K), "bfloat16", seed=100 + li, outlier_frac=1e-3).to(dev)
        lin.append((name, N, K, w, ib.quantize_int4(w, GROUP)))
    pk = peaks()
    for M in COMPARE_M:
        x = {K: torch.randn(M, K, device=dev).to(torch.bfloat16) for K in (2048, 8192)}
        res = {}
        for label, fn in (("w4", lambda xx, l: ib.w4a16_matmul(xx, *l[4])), ("bf16", lambda xx, l: F.linear(xx, l[3])),
                          ("w16", lambda xx, l: ib.w16a16_matmul(xx, l[3]))):
            wbytes = sum((l[1] * l[2] // 2 + 4 * l[1] * l[2] // GROUP) if label == "w4" else 2 * l[1] * l[2]
                         for l in lin)
            copies = max(1, math.ceil(2 * L2_BYTES / wbytes))
            sets = [lin] + [[(l[0], l[1], l[2], l[3].clone() if label != "w4" else l[3],
                              tuple(t.clone() for t in l[4]) if label == "w4" else l[4]) for l in lin]
                            for _ in range(copies - 1)]
            reps = 20

            def run(i):
                for l in sets[i % copies]:
                    fn(x[l[2]], l)
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for i in range(3):
                    run(i)
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=side):
                for i in range(reps):
                    run(i)
            gr.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            gr.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / reps
            flops = sum(2 * M * l[1] * l[2] for l in lin)
            res[label] = {"us": us, "GB/s": (wbytes + sum(2 * M * (l[1] + l[2]) for l in lin)) / us / 1e3,
                          "TFLOP/s": flops / us / 1e6}
            del gr, sets
            torch.cuda.empty_cache()
        if rank == 0:
            print(json.dumps({"workload": "compare (BASELINE config 2)", "M": M, "G": GROUP, "block_us": res,
                              "w4_over_bf16": res["bf16"]["us"] / res["w4"]["us"],
                              "peaks": {"hbm_gbs": pk["hbm_gbs"], "bf16_tflops": pk["bf16_tflops"]}}), flush=True)


GEMV_SHAPES = {"qkv": (3072, 2048), "o_proj": (2048, 2048), "gate_up": (16384, 2048), "down_proj": (2048, 8192),
               "lm_head": (128256, 2048), "gate_proj": (8192, 2048)}


def main_gemv(args, world, rank, local, threads):
    """A fixed number of launches of one W4 matmul (a --layer shape of the Llama-3.2-1B block, G=128, --m tokens),
    for profiler captures: --launches launches of each --kernel choice, after two warm-up launches each, plus
    the quantizer (quantize_pow2_kernel) once per weight.  Prints the device time of the last launch of each."""
    import int4_b200 as ib
    from int4_b200 import _lib

    dev = torch.device("cuda", local)
    N, K = GEMV_SHAPES[args.layer]
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    q = ib.quantize_int4(w, GROUP)
    x = torch.randn(args.m, K, generator=g).to(torch.bfloat16).to(dev)
    L = _lib.lib()
    out = {}
    for kernel in [int(k) for k in args.kernel.split(",")]:
        L.i4b_set_w4_kernel_override(kernel, 0, 0)
        for _ in range(2):
            ib.w4a16_matmul(x, *q)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(args.launches):
            e0.record()
            ib.w4a16_matmul(x, *q)
            e1.record()
        torch.cuda.synchronize()
        out[kernel] = e0.elapsed_time(e1) * 1e3
    L.i4b_set_w4_kernel_override(0, 0, 0)
    assert _lib.device_error_flags(local) == 0
    if rank == 0:
        print(json.dumps({"workload": "gemv", "layer": args.layer, "N": N, "K": K, "M": args.m,
                          "last_launch_us": out}), flush=True)


SWEEP = [("gate_proj", 8192, 2048), ("down_proj", 2048, 8192)]


def main_sweep(args, world, rank, local, threads):
    """gate_proj and down_proj, G in {32, 64, 128}, M in {1, 2, 16, 64}; device time per
    matmul and HBM GB/s of its algorithmic bytes (weights rotated past L2); one JSON line per case."""
    import cases
    import int4_b200 as ib

    dev = torch.device("cuda", local)
    pk = peaks()
    for li, (name, N, K) in enumerate(SWEEP):
        w = cases.weight((N, K), "bfloat16", seed=300 + li, outlier_frac=1e-3).to(dev)
        for G in (32, 64, 128):
            q = ib.quantize_int4(w, G)
            nb = N * K // 2 + 4 * N * K // G
            copies = max(2, math.ceil(2 * L2_BYTES / nb))
            qs = [q] + [tuple(t.clone() for t in q) for _ in range(copies - 1)]
            for M in (1, 2, 16, 64):
                x = torch.randn(M, K, device=dev).to(torch.bfloat16)
                reps = 60
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    for i in range(3):
                        ib.w4a16_matmul(x, *qs[i % copies])
                torch.cuda.synchronize()
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=side):
                    for i in range(reps):
                        ib.w4a16_matmul(x, *qs[i % copies])
                gr.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                gr.replay()
                e1.record()
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / reps
                gbs = alg_bytes(M, N, K, G) / us / 1e3
                if rank == 0:
                    print(json.dumps({"workload": "sweep (BASELINE config 3)", "layer": name, "N": N, "K": K, "G": G,
                                      "M": M, "us": us, "GB/s": gbs, "frac_of_hbm": gbs / pk["hbm_gbs"]}), flush=True)
                del gr
            del qs
            torch.cuda.empty_cache()


def _json_only_stdout() -> None:
    """Keep stdout for the JSON lines: native libraries that write to file descriptor 1 (NCCL prints its
    version line there at start-up) go to stderr, while Python's sys.stdout keeps the original stdout."""
    try:
        sys.stdout.flush()
        real = os.dup(1)
        os.dup2(2, 1)
        sys.stdout = os.fdopen(real, "w", buffering=1)
    except OSError:
        pass


def main():
    _json_only_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 20000 block steps, 256 decode steps for the model workload)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layer", choices=sorted(GEMV_SHAPES), default="gate_up", help="gemv workload: the shape")
    ap.add_argument("--kernel", default="0", help="gemv workload: comma-separated W4 kernel choices "
                    "(i4b_set_w4_kernel_override: 0 automatic, 1 register-streaming, 2 staged, 3 staged / lm_head "
                    "streaming, 6 slab-streaming)")
    ap.add_argument("--launches", type=int, default=3, help="gemv workload: launches per kernel choice")
    ap.add_argument("--workload", choices=["block", "model", "compare", "sweep", "gemv"], default="block",
                    help="block: BASELINE config 2 at --m tokens (default; the same run also times config 4's "
                         "decode and checks its NLL); model: configs 4/5 decode; compare: config 2's W4 / cuBLAS "
                         "bf16 / W16 block table over M; sweep: config 3's group-size x M table")
    ap.add_argument("--decode-steps", type=int, default=64,
                    help="block workload: greedy decode steps of the config-4 model timed in the same run "
                         "(0 skips the decode section)")
    ap.add_argument("--nll", type=int, default=1, help="block workload: config-4 mean-NLL check after the decode")
    ap.add_argument("--prompt", type=int, default=512, help="model workload: prompt tokens before decoding")
    ap.add_argument("--lm-head-w4", type=int, default=0, help="model workload: quantize the lm_head too")
    ap.add_argument("--m", type=int, default=1, help="tokens per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--trace", type=int, default=0,
                    help="model workload: after timing, trace one persistent step and print its per-stage "
                         "breakdown as a second JSON line on stderr")
    ap.add_argument("--persistent", type=int, default=-1,
                    help="model workload: 1 = all decoder layers of a step in one launch (i4b_decode_layers), "
                         "0 = one launch per projection / glue op, -1 = whichever the model qualifies for")
    ap.add_argument("--compare-bf16", type=int, default=1,
                    help="model workload: also time the same decode loop with bf16 projections")
    ap.add_argument("--peer-allreduce", type=int, default=-1,
                    help="tensor-parallel runs: 1 = sum the row-parallel outputs inside every W4 matmul through peer "
                         "exchange buffers; 0 = NCCL all-reduces only; -1 (default) = what measured fastest: the "
                         "block sums inside its o/down matmuls (4 ranks: 24.1 against 44.4 us with NCCL; 8 ranks: "
                         "28.8 against 65.0), the decode inside its persistent launch or, where that does not fit "
                         "(8 ranks), inside the per-launch o/down matmuls for batches up to 8 (whose grids are "
                         "resident at once), and the greedy token by peer exchange")
    ap.add_argument("--pdl", type=int, default=1,
                    help="programmatic dependent launch for the small-M kernels (weights fetched before the wait)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.steps is None:
        args.steps = 256 if args.workload == "model" else 20000

    config = {"workload": f"llama-3.2-1b decoder block, 7 linears, W4 G={GROUP}, M={args.m}",
              "model": "Llama-3.2-1B-shaped (random-init)", "group_size": GROUP, "tokens_per_step": args.m,
              "parallelism": f"tp{args.gpus}", "global_batch": args.m, "seq_len": 1, "pdl": bool(args.pdl),
              "l2": "inputs larger than L2: weights rotate over copies whose total exceeds 2x L2"}
    metric = "per-block W4A16 GEMM us (Llama-3.2-1B decoder block, decode step)"
    threads = os.cpu_count() or 1

    if args.impl == "reference" and args.workload == "model":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if int(os.environ.get("RANK", "0")) != 0:
            return
        ref_steps = min(args.steps, 2)
        dt, sample = cpu_model_sample(threads, args.m, ref_steps)
        v = args.m / dt
        print(json.dumps({
            "impl": "reference", "metric": MODEL_METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": ref_steps, "steps_requested": args.steps, "warmup": 0, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16 (fake-quant W4)",
            "data": "synthetic", "config": model_config(args),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        ref_steps = min(args.steps, 5)
        ref_warmup = min(args.warmup, 1)  # one untimed CPU block step (~0.15 s) keeps the arm within minutes
        dt, sample = cpu_block_sample(args.m, threads, ref_steps, ref_warmup)
        v = dt * 1e6
        dec = None
        if args.decode_steps > 0:  # config 4's decode on the host cores: the fake-quant model in transformers
            dts, dsample = cpu_model_sample(threads, 1, 2)
            dec = {"metric": MODEL_METRIC, "tokens_per_s": 1.0 / dts, "unit": "tokens/s", "ms_per_token": dts * 1e3,
                   "cores": threads, "kind": "port", "sample": dsample}
        print(json.dumps({
            "impl": "reference", "metric": metric, "value": v, "unit": "us", "n_gpus": world,
            "steps": ref_steps, "steps_requested": args.steps, "warmup": ref_warmup,
            "warmup_requested": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "w4a16-bf16", "data": "synthetic", "config": config,
            "cpu_baseline": {"value": v, "unit": "us", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "decode": dec,
        }), flush=True)
        return

    world, rank, local = dist_setup()
    if args.pdl:
        from int4_b200 import _lib

        _lib.set_pdl(True)
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if args.workload in ("model", "compare", "sweep", "gemv"):
        {"model": main_model, "compare": main_compare, "sweep": main_sweep, "gemv": main_gemv}[args.workload](
            args, world, rank, local, threads)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    r = run_block(args, world, rank, local)
    dec = None
    if args.decode_steps > 0:
        # BASELINE config 4 in the same run: W4 decode tokens/s next to bf16 in the same loop, batch 1
        try:
            dec = run_model(args, world, rank, local, B=1, steps=args.decode_steps, nll=bool(args.nll))
        except Exception as ex:  # reported in the line; the block number stands on its own
            dec = {"error": f"{type(ex).__name__}: {ex}"}
    pk = peaks()
    us = r["us_per_step"]
    achieved = r["bytes_per_step_rank"] / (us * 1e-6) / 1e9  # per rank, GB/s
    cpu = None
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        dt, sample = cpu_block_sample(args.m, threads, 1)
        cpu = {"value": dt * 1e6, "unit": "us", "cores": threads, "kind": "port", "sample": sample}
    if rank == 0:
        prof_traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            with open(tp) as f:
                prof_traffic = json.load(f).get(f"block_m{args.m}")
        line = {
            "metric": metric, "value": us, "unit": "us", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": us / 1e3, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "w4a16-bf16", "data": "synthetic (seeded N(0,0.02) weights, 0.1% x10)",
            "config": config,
            "block_gbs_per_gpu": achieved, "block_us_l2_hot": r["hot_us"],
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "traffic": prof_traffic,
                         "kernel": "the 4 decode GEMV launches of a step: w4_slab_kernel (q|k|v, o, gate|up) and "
                                   "w4_gemv_kernel (down)",
                         "peak_source": pk["source"]},
            "cpu_baseline": cpu,
            "e2e": {"value": r["e2e_us"], "unit": "us", "h2d_bytes_per_step": r["h2d"],
                    "d2h_bytes_per_step": r["d2h"]},
            "gpu_launches": r["launches_per_step"] * args.steps,
            "clocks": r["clocks"], "device_error_flags": r["device_error_flags"],
        }
        if dec is not None:
            line["decode"] = decode_summary(args, dec, world)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
