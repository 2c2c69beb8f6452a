"""Tensor-parallel Llama decoding on the W4A16 kernels: the model-level caller of the path.

The reference measures its kernels inside a Hugging Face ``LlamaForCausalLM``
whose ``nn.Linear`` layers ``quantize_model_linears`` swapped for
``Int4Linear`` (``benchmarks/eval_llama.py:121-183``, ``int4_triton/qlinear.py:54-68``),
one GPU.  ``LlamaTP`` runs the same network from the same HF weights, with
the projections laid out for the kernels and for tensor parallelism:

* q/k/v are one column-parallel projection per layer (this rank's heads of
  q, k and v stacked along N), gate/up likewise; o_proj and down_proj are
  row-parallel (this rank's slice of K) followed by an all-reduce -- in a
  W4 decode step the sum runs inside the o / down matmul itself
  (``peer.w4a16_matmul_allreduce``), elsewhere it is NCCL's;
* the lm_head is vocab-parallel followed by an all-gather of the logits;
* every INT4 weight is quantized per shard -- for column shards that is the
  same bits as slicing the fully quantized tensor, and for row shards too as
  long as the shard width is a multiple of the group size (checked);
* norms, rotary embedding, attention over a static KV cache, SwiGLU and the
  residual stream follow ``transformers``' Llama (RMSNorm in fp32, rotary
  tables rounded to bf16, scaled-dot-product attention), so a one-rank
  ``LlamaTP`` matches the HF model with the same weights.

``w4=False`` keeps every projection in bf16 (``torch.nn.functional.linear``):
the same model and decode loop, for the W4-versus-bf16 comparison.  All
steps are free of host synchronisation and of shape changes, so a decode
step can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _lib
from .gemm import w4a16_matmul, w4a16_matmul_argmax
from .peer import argmax_allreduce, w4a16_matmul_allreduce
from .quantize import quantize_int4


def column_shard(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [rank*N/world, (rank+1)*N/world) of W[N, K]: this rank's output features."""
    n = w.shape[0]
    assert n % world == 0, (n, world)
    return w[rank * n // world:(rank + 1) * n // world]


def row_shard(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Columns [rank*K/world, (rank+1)*K/world) of W[N, K]: this rank's input features."""
    k = w.shape[1]
    assert k % world == 0, (k, world)
    return w[:, rank * k // world:(rank + 1) * k // world]


def head_shard(w: torch.Tensor, heads: int, head_dim: int, rank: int, world: int) -> torch.Tensor:
    """This rank's heads (rows) of a q/k/v projection W[heads*head_dim, K]."""
    assert heads % world == 0, (heads, world)
    h = heads // world
    return w[rank * h * head_dim:(rank + 1) * h * head_dim]


class Projection:
    """One (possibly stacked) projection y = x @ W^T, INT4 (quantize_int4 layout) or bf16."""

    def __init__(self, w: torch.Tensor, w4: bool, group_size: int):
        w = w.detach().to(torch.bfloat16).contiguous()
        self.out_features, self.in_features = w.shape
        if w4:
            assert self.in_features % group_size == 0, (self.in_features, group_size)
            self.q = quantize_int4(w, group_size)
            self.w = None
        else:
            self.q = None
            self.w = w

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.q is not None:
            return w4a16_matmul(x, *self.q)
        return F.linear(x, self.w)

    def weight_bytes(self) -> int:
        if self.q is not None:
            return sum(t.numel() * t.element_size() for t in self.q)
        return self.w.numel() * self.w.element_size()


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """transformers' LlamaRMSNorm: statistics in fp32, result cast back, then scaled."""
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return weight * h.to(x.dtype)


# ---------------------------------------------------------------------- fused decode-step kernels (C ABI)


def _stream(t: torch.Tensor) -> int:
    return _lib.stream_handle(t.device)


def add_rmsnorm(h: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, out: torch.Tensor,
                eps: float) -> None:
    """h = bf16(h + delta) in place (delta may be None); out = rms_norm(h, weight, eps).  h, out: [rows, H]."""
    rows, H = h.shape
    st = _lib.lib().i4b_add_rmsnorm(h.data_ptr(), None if delta is None else delta.data_ptr(), weight.data_ptr(),
                                    out.data_ptr(), rows, H, eps, _stream(h))
    _lib.check(st, "add_rmsnorm")


def rope_kv_cache(qkv, cos, sin, pos, q_out, k_cache, v_cache, nq: int, nkv: int) -> None:
    """Rotary embedding of q and k of one token per sequence; k and v written to the caches at ``pos``."""
    B = qkv.shape[0]
    st = _lib.lib().i4b_rope_kv_cache(qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), pos.data_ptr(), q_out.data_ptr(),
                                      k_cache.data_ptr(), v_cache.data_ptr(), B, nq, nkv, 64, k_cache.shape[2],
                                      _stream(qkv))
    _lib.check(st, "rope_kv_cache")


def decode_attention(q, k_cache, v_cache, pos, out, nq: int, nkv: int, scale: float) -> None:
    """out[B, nq*64] = grouped-query attention of q[B, nq, 64] over cache positions 0..pos."""
    B = q.shape[0]
    st = _lib.lib().i4b_decode_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), pos.data_ptr(),
                                         out.data_ptr(), B, nq, nkv, 64, k_cache.shape[2], scale, _stream(q))
    _lib.check(st, "decode_attention")


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor) -> None:
    """out[B, I] = bf16(bf16(silu(g)) * u) for gate_up[B, 2I] = (g | u)."""
    B, I2 = gate_up.shape
    st = _lib.lib().i4b_silu_mul(gate_up.data_ptr(), out.data_ptr(), B, I2 // 2, _stream(gate_up))
    _lib.check(st, "silu_mul")


PROLOGUE_RMSNORM, PROLOGUE_SWIGLU = 1, 2


def w4a16_matmul_prologue(kind: int, src: torch.Tensor, qweight, scales, zeros, *, delta=None, norm_weight=None,
                          eps: float = 1e-5, resid_out=None) -> torch.Tensor:
    """W4A16 matmul of M <= 32 bf16 rows whose activations the kernel derives from ``src``.

    kind PROLOGUE_RMSNORM: x = rms_norm(src + delta, norm_weight, eps); ``resid_out`` receives src + delta.
    kind PROLOGUE_SWIGLU:  x = silu(g) * u for src = (g | u).
    """
    M = src.shape[0]
    K = qweight.shape[0] * 8
    N = qweight.shape[1]
    G = K // scales.shape[0]
    y = torch.empty((M, N), dtype=torch.bfloat16, device=src.device)
    L = _lib.lib()
    stream = _stream(src)
    need = L.i4b_w4a16_workspace_size(M, N, K, G)
    ws_ptr, ws_size = _lib.workspace(src.device, stream, need)
    st = L.i4b_w4a16_matmul_prologue(kind, src.data_ptr(), None if delta is None else delta.data_ptr(),
                                     None if norm_weight is None else norm_weight.data_ptr(), eps,
                                     None if resid_out is None else resid_out.data_ptr(), M, K, src.stride(0),
                                     qweight.data_ptr(), N, qweight.stride(0), scales.data_ptr(), zeros.data_ptr(),
                                     scales.stride(0), G, y.data_ptr(), y.stride(0), ws_ptr, ws_size, stream)
    _lib.check(st, "w4a16_matmul_prologue")
    return y


def argmax_last(x: torch.Tensor) -> torch.Tensor:
    """Index of the first maximum along the last dim of a bf16 tensor (torch.argmax(-1, keepdim=True))."""
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    out = torch.empty(x2.shape[0], dtype=torch.long, device=x.device)
    st = _lib.lib().i4b_argmax_rows(x2.data_ptr(), x2.shape[0], x2.shape[1], out.data_ptr(), _stream(x2))
    _lib.check(st, "argmax_rows")
    return out.view(*x.shape[:-1], 1)


def tile_w4(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """The quantize_int4 triple re-laid into the 16-column x 512-k pieces the persistent decode streams.

    ``out`` (uint8, 16-byte aligned, at least ``tile_w4_bytes`` long) receives the pieces when given.
    """
    K, N = qweight.shape[0] * 8, qweight.shape[1]
    G = K // scales.shape[0]
    L = _lib.lib()
    nbytes = L.i4b_tile_w4_bytes(N, K, G)
    if nbytes == 0:
        raise ValueError(f"tile_w4: N={N} must be a multiple of 16, K={K} of 512, group size {G} in (32, 64, 128)")
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device=qweight.device)
    assert out.dtype == torch.uint8 and out.numel() >= nbytes and out.is_contiguous()
    st = L.i4b_tile_w4(qweight.data_ptr(), N, qweight.stride(0), scales.data_ptr(), zeros.data_ptr(), scales.stride(0),
                       K, G, out.data_ptr(), _stream(qweight))
    _lib.check(st, "tile_w4")
    return out


def interleave_gate_up(q: tuple[torch.Tensor, torch.Tensor, torch.Tensor], inter: int):
    """Columns of a stacked (gate | up) quantize_int4 triple reordered to gate 0, up 0, gate 1, up 1, ...

    Quantization is per output column, so this is the same bits as quantizing the interleaved weight.
    """
    j = torch.arange(inter, device=q[0].device)
    perm = torch.stack([j, j + inter], dim=1).reshape(-1)
    return tuple(t[:, perm].contiguous() for t in q)


class PersistentDecoder:
    """Every decoder layer of a single-token decode step in one launch (``i4b_decode_layers``).

    Holds the tiled weights of all layers (one buffer per projection kind), the stacked norm weights,
    the residual-stream buffer and the workspace (zeroed once; every launch leaves it zero).  Under
    tensor parallelism it also holds a peer group of its own: the o_proj / down_proj epilogues store
    their partial outputs into every rank's exchange buffer, and the stages that consume the residual
    stream add them up (collective set-up; ``close`` releases it).
    """

    def __init__(self, model: "LlamaTP", layer_q: list, group_size: int):
        dev = model.device
        H, I = model.hidden, model.inter_l
        nq, nkv = model.nh_l, model.nkv_l
        Lc = len(layer_q)
        L = _lib.lib()
        shapes = {"qkv": ((nq + 2 * nkv) * 64, H), "o": (H, nq * 64), "gu": (2 * I, H), "down": (H, I)}
        self.tiles = {}
        for kind, (N, K) in shapes.items():
            per = L.i4b_tile_w4_bytes(N, K, group_size)
            buf = torch.empty(Lc * per, dtype=torch.uint8, device=dev)
            for li, qd in enumerate(layer_q):
                q = qd[kind]
                if kind == "gu":
                    q = interleave_gate_up(q, I)
                tile_w4(*q, out=buf[li * per:(li + 1) * per])
            self.tiles[kind] = buf
        self.ln1 = torch.stack([ly["ln1"] for ly in model.layers]).contiguous()
        self.ln2 = torch.stack([ly["ln2"] for ly in model.layers]).contiguous()
        self.h = torch.empty(model.max_batch, H, device=dev, dtype=torch.bfloat16)
        m = _lib.DecodeModel()
        m.layers, m.hidden, m.heads, m.kv_heads, m.head_dim = Lc, H, nq, nkv, 64
        m.intermediate, m.vocab, m.group_size = I, model.embed.shape[0], group_size
        m.batch, m.max_seq, m.cache_batch = model.max_batch, model.max_seq, model.max_batch
        m.eps, m.attn_scale = model.eps, 64 ** -0.5
        m.embed = model.embed.data_ptr()
        m.w_qkv, m.w_o = self.tiles["qkv"].data_ptr(), self.tiles["o"].data_ptr()
        m.w_gu, m.w_down = self.tiles["gu"].data_ptr(), self.tiles["down"].data_ptr()
        m.ln1, m.ln2 = self.ln1.data_ptr(), self.ln2.data_ptr()
        m.cos_table, m.sin_table = model.cos.data_ptr(), model.sin.data_ptr()
        m.k_cache, m.v_cache = model.k_cache.data_ptr(), model.v_cache.data_ptr()
        m.h_out = self.h.data_ptr()
        self.peers = None
        if model.world > 1:
            from .peer import PeerGroup

            self.peers = PeerGroup(model.group, capacity=L.i4b_decode_peer_capacity(Lc, model.world, H))
            m.peers = ctypes.addressof(self.peers.struct)
        self.m = m
        nbytes = ctypes.c_size_t(0)
        _lib.check(L.i4b_decode_workspace_size(ctypes.byref(m), ctypes.byref(nbytes)), "decode_workspace_size")
        self.ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=dev)

    STAGES = ("qkv", "attention", "o_proj", "gate_up", "down_proj")

    def trace(self, ids: torch.Tensor, pos: torch.Tensor) -> dict:
        """Run one step with the kernel's trace hook on; per-stage medians over CTAs and inner layers (µs).

        Projection stages: ``wait`` (entry to dependency met), ``stage_x`` (inputs staged), ``pieces``,
        ``epilogue``, ``publish``; warp 0's ``weight_wait`` / ``mma`` per piece; ``producer_lead`` (pieces
        the producer had issued ahead of the stage); ``first_warp_done`` / ``last_warp_done`` (from the
        start of the pieces) and ``last_warp``.  Attention: ``wait``, ``queries``, ``blocks``,
        ``fence``, ``ticket``.  ``layer_us``: median CTA's time from one qkv entry to the next.
        """
        import numpy as np

        L = self.m.layers
        grid = torch.cuda.get_device_properties(self.h.device).multi_processor_count
        buf = torch.zeros(grid * L * 5 * 16, dtype=torch.int64, device=self.h.device)
        lib = _lib.lib()
        lib.i4b_set_decode_trace(buf.data_ptr(), buf.numel() * 8)
        try:
            self.run(ids, pos)
            torch.cuda.synchronize()
        finally:
            lib.i4b_set_decode_trace(None, 0)
        t = buf.view(grid, L, 5, 16).cpu().numpy().astype(np.float64)
        valid = t[..., 7] > 0
        # SM clock from the trace itself: clock64 cycles per %globaltimer ns between stage entries of one CTA
        cta = int(np.argmax(valid[:, :, 0].sum(1)))
        ent = [(t[cta, l, 0, 0], t[cta, l, 0, 7]) for l in range(L) if valid[cta, l, 0]]
        mhz = (ent[-1][0] - ent[0][0]) / max(ent[-1][1] - ent[0][1], 1) * 1e3 if len(ent) > 1 else 1965.0
        inner = range(1, L - 1) if L > 2 else range(L)
        out = {"sm_mhz": round(mhz, 1), "stages": {}}
        names = [("wait", 0, 1), ("stage_x", 1, 2), ("pieces", 2, 3), ("epilogue", 3, 4), ("publish", 4, 6)]
        anames = [("wait", 0, 1), ("queries", 1, 2), ("blocks", 2, 3), ("fence", 3, 4), ("ticket", 4, 5)]
        for si, sname in enumerate(self.STAGES):
            rows = np.concatenate([t[valid[:, l, si], l, si] for l in inner]) if any(
                valid[:, l, si].any() for l in inner) else None
            if rows is None or len(rows) == 0:
                continue
            d = {"ctas": int(valid[:, inner[0], si].sum())}
            for nm, a, b in (anames if si == 1 else names):
                d[nm] = round(float(np.median(rows[:, b] - rows[:, a])) / mhz, 2)
            if si != 1:
                npc = np.maximum(rows[:, 10], 1)
                d["weight_wait_per_piece"] = round(float(np.median(rows[:, 8] / npc)) / mhz, 3)
                d["mma_per_piece"] = round(float(np.median(rows[:, 9] / npc)) / mhz, 3)
                d["pieces_warp0"] = float(np.median(rows[:, 10]))
                d["producer_lead"] = float(np.median(rows[:, 11]))
                d["first_warp_done"] = round(float(np.median(rows[:, 12] - rows[:, 2])) / mhz, 2)
                d["last_warp_done"] = round(float(np.median(rows[:, 13] - rows[:, 2])) / mhz, 2)
                d["last_warp"] = float(np.median(rows[:, 14]))
            out["stages"][sname] = d
        g0 = [np.median(t[valid[:, l, 0], l, 0, 7]) for l in range(L) if valid[:, l, 0].any()]
        out["layer_us"] = round(float(np.median(np.diff(g0))) / 1e3, 2) if len(g0) > 1 else None
        return out

    def close(self) -> None:
        if self.peers is not None:
            self.peers.close()
            self.peers = None
            self.m.peers = None

    def run(self, ids: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Residual stream [B, H] after the last layer for token ids[B, 1] at position pos (device int64)."""
        B = ids.shape[0]
        ids = ids.reshape(B)
        assert ids.dtype == torch.int64 and ids.is_contiguous() and pos.dtype == torch.int64
        self.m.batch = B
        self.m.tokens = ids.data_ptr()
        self.m.pos = pos.data_ptr()
        st = _lib.lib().i4b_decode_layers(ctypes.byref(self.m), self.ws.data_ptr(), self.ws.numel(), _stream(ids))
        _lib.check(st, "decode_layers")
        return self.h[:B]


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


class LlamaTP:
    """Llama decoder for one tensor-parallel rank, built from an HF ``LlamaForCausalLM``.

    ``group`` is the ``torch.distributed`` process group of the ranks (None when
    ``world == 1``).  ``max_seq`` and ``max_batch`` size the static KV cache.
    ``fused`` runs a decode step's norms, rotary embedding, attention and SwiGLU
    as the library's fused kernels; ``fused=False`` runs them as the torch ops
    transformers uses.  ``persistent`` (default: whenever the model qualifies --
    W4, fused, batch <= 8, hidden and per-rank widths of 512 * 2^k, and under
    tensor parallelism the peer all-reduce) runs all decoder layers of a decode
    step as one launch of ``i4b_decode_layers``; tensor-parallel ranks then add
    each other's o / down partials inside that launch.
    ``peer_allreduce`` (tensor parallelism) sets up the peer exchange buffers:
    the persistent decode sums the ranks' o / down partials inside its launch,
    and ``decode_greedy`` exchanges the ranks' best tokens instead of
    all-gathering the logits.  ``matmul_allreduce`` additionally sums the o /
    down outputs of the per-launch decode (<= 32 tokens) inside those matmuls
    (``i4b_w4a16_matmul_allreduce``) instead of an NCCL all-reduce: measured at
    two ranks, batch 1, 1231 against 977 tokens/s; a shape whose grid cannot be
    resident at once falls back to NCCL on every rank.  It is off by default
    (the persistent decode sums inside its own launch where it runs).
    """

    def __init__(self, hf_model, *, w4: bool = True, group_size: int = 128, quantize_lm_head: bool = False,
                 rank: int = 0, world: int = 1, group=None, max_seq: int = 2048, max_batch: int = 1,
                 device: torch.device | None = None, fused: bool = True, persistent: bool | None = None,
                 peer_allreduce: bool = True, matmul_allreduce: bool = False):
        cfg = hf_model.config
        self.fused = fused
        self.cfg = cfg
        self.rank, self.world, self.group = rank, world, group
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        H = cfg.hidden_size
        nh, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        hd = getattr(cfg, "head_dim", None) or H // nh
        inter = cfg.intermediate_size
        assert nh % world == 0 and nkv % world == 0 and inter % world == 0, "heads / MLP width must split over ranks"
        if w4:
            assert (nh // world * hd) % group_size == 0 and (inter // world) % group_size == 0, \
                "row-parallel shards must hold whole quantization groups"
        self.hd, self.nh_l, self.nkv_l = hd, nh // world, nkv // world
        self.hidden, self.inter_l = H, inter // world
        if fused:
            assert hd == 64, "the fused decode kernels are written for head_dim 64"
        self.eps = cfg.rms_norm_eps
        self.max_seq, self.max_batch = max_seq, max_batch
        self.w4 = w4

        def bf(t):
            return t.detach().to(dev, torch.bfloat16)

        self.embed = bf(hf_model.model.embed_tokens.weight)
        self.layers = []
        for layer in hf_model.model.layers:
            at, mlp = layer.self_attn, layer.mlp
            qkv = torch.cat([head_shard(bf(at.q_proj.weight), nh, hd, rank, world),
                             head_shard(bf(at.k_proj.weight), nkv, hd, rank, world),
                             head_shard(bf(at.v_proj.weight), nkv, hd, rank, world)], 0)
            gu = torch.cat([column_shard(bf(mlp.gate_proj.weight), rank, world),
                            column_shard(bf(mlp.up_proj.weight), rank, world)], 0)
            self.layers.append({
                "ln1": bf(layer.input_layernorm.weight),
                "ln2": bf(layer.post_attention_layernorm.weight),
                "qkv": Projection(qkv, w4, group_size),
                "o": Projection(row_shard(bf(at.o_proj.weight), rank, world), w4, group_size),
                "gu": Projection(gu, w4, group_size),
                "down": Projection(row_shard(bf(mlp.down_proj.weight), rank, world), w4, group_size),
            })
            del qkv, gu
        self.norm = bf(hf_model.model.norm.weight)
        vocab = hf_model.lm_head.weight.shape[0]
        assert vocab % world == 0, "vocab must split over ranks"
        self.vocab = vocab
        self.lm_head = Projection(column_shard(bf(hf_model.lm_head.weight), rank, world),
                                  w4 and quantize_lm_head, group_size)

        # rotary tables exactly as transformers computes them (fp32, then cast to the activation dtype)
        rot = hf_model.model.rotary_emb
        inv_freq = rot.inv_freq.detach().float().to(dev)
        pos = torch.arange(max_seq, device=dev, dtype=torch.float32)
        freqs = pos[:, None] * inv_freq[None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        scale = float(getattr(rot, "attention_scaling", 1.0))
        self.cos = (emb.cos() * scale).to(torch.bfloat16)
        self.sin = (emb.sin() * scale).to(torch.bfloat16)

        n_layers = len(self.layers)
        self.k_cache = torch.zeros(n_layers, max_batch, self.nkv_l, max_seq, hd, device=dev, dtype=torch.bfloat16)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.positions = torch.arange(max_seq, device=dev)

        def pow2_chunks(k: int) -> bool:  # a power-of-two number of 8-value chunks, at least one 512-k piece
            return k >= 512 and k % 8 == 0 and (k // 8) & (k // 8 - 1) == 0

        qualifies = (w4 and (world == 1 or peer_allreduce) and fused and hd == 64 and max_batch <= 8
                     and group_size in (32, 64, 128) and world <= 8
                     and pow2_chunks(H) and pow2_chunks(self.inter_l) and pow2_chunks(self.nh_l * hd)
                     and self.nh_l // self.nkv_l in (1, 2, 4, 8) and self.nh_l % self.nkv_l == 0)
        if persistent and not qualifies:
            raise ValueError("persistent decode needs W4 (G 32/64/128), fused kernels, head_dim 64, batch <= 8, "
                             "hidden and per-rank intermediate / q widths of 512 * 2^k, and under tensor "
                             "parallelism the peer all-reduce")
        self.persistent = None
        if qualifies and persistent is not False:
            self.persistent = PersistentDecoder(
                self, [{k: L[k].q for k in ("qkv", "o", "gu", "down")} for L in self.layers], group_size)
        # Under tensor parallelism the W4 decode step sums the row-parallel o / down outputs inside their
        # matmuls (peer exchange buffers over NVLink) instead of a separate NCCL all-reduce.
        self.matmul_allreduce = matmul_allreduce
        self.peers = None
        if world > 1 and w4 and fused and peer_allreduce:
            from .peer import PeerGroup

            self.peers = PeerGroup(group, capacity=max_batch * H)

    def close(self) -> None:
        """Release the peer exchange buffers (collective when tensor-parallel)."""
        if self.persistent is not None:
            self.persistent.close()
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    # ------------------------------------------------------------------ collectives

    def _all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            torch.distributed.all_reduce(x, group=self.group)
        return x

    def _matmul_allreduce_or_none(self, x: torch.Tensor, q, prologue: int = 0):
        """The row-parallel matmul with the ranks' sum inside it, or None when the library refuses the shape
        (the fused sum needs its whole grid resident at once).  The refusal comes from the host-side plan, the
        same on every rank, so all ranks then take NCCL's all-reduce together, for this and later steps."""
        from ._lib import STATUS_SHAPE, Int4B200Error

        try:
            if prologue:
                return w4a16_matmul_allreduce(self.peers, x, *q, prologue=prologue)
            return w4a16_matmul_allreduce(self.peers, x, *q)
        except Int4B200Error as e:
            if e.status != STATUS_SHAPE:
                raise
            self.matmul_allreduce = False
            return None

    def _gather_vocab(self, logits: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return logits
        parts = [torch.empty_like(logits) for _ in range(self.world)]
        torch.distributed.all_gather(parts, logits.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)

    # ------------------------------------------------------------------ forward

    def weight_bytes(self) -> int:
        """Bytes of the projection weights this rank streams per decode step (embedding excluded)."""
        b = sum(L[k].weight_bytes() for L in self.layers for k in ("qkv", "o", "gu", "down"))
        return b + self.lm_head.weight_bytes()

    def _layer(self, i: int, h: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos0, mask) -> torch.Tensor:
        L = self.layers[i]
        B, S, _ = h.shape
        hd, nq, nkv = self.hd, self.nh_l, self.nkv_l
        x = rms_norm(h, L["ln1"], self.eps)
        qkv = L["qkv"](x)
        q, k, v = qkv.split([nq * hd, nkv * hd, nkv * hd], dim=-1)
        q = q.view(B, S, nq, hd).transpose(1, 2)
        k = k.view(B, S, nkv, hd).transpose(1, 2)
        v = v.view(B, S, nkv, hd).transpose(1, 2)
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        kc, vc = self.k_cache[i, :B], self.v_cache[i, :B]
        if mask is None:  # prefill from position 0: attend causally within the prompt
            kc[:, :, :S] = k
            vc[:, :, :S] = v
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=hd ** -0.5, enable_gqa=True)
        else:  # one token at device-side position pos0: write the cache, attend to positions <= pos0
            kc.index_copy_(2, pos0, k)
            vc.index_copy_(2, pos0, v)
            a = F.scaled_dot_product_attention(q, kc, vc, attn_mask=mask, scale=hd ** -0.5, enable_gqa=True)
        a = a.transpose(1, 2).reshape(B, S, nq * hd)
        h = h + self._all_reduce(L["o"](a))
        x = rms_norm(h, L["ln2"], self.eps)
        g, u = L["gu"](x).chunk(2, dim=-1)
        h = h + self._all_reduce(L["down"](F.silu(g) * u))
        return h

    def _head(self, h: torch.Tensor) -> torch.Tensor:
        return self._gather_vocab(self.lm_head(rms_norm(h, self.norm, self.eps)))

    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, all_logits: bool = False) -> torch.Tensor:
        """Run the prompt ids[B, S] from position 0 and fill the KV cache; logits of the last (or every) token."""
        B, S = ids.shape
        assert B <= self.max_batch and S <= self.max_seq
        h = F.embedding(ids, self.embed)
        cos, sin = self.cos[:S], self.sin[:S]
        for i in range(len(self.layers)):
            h = self._layer(i, h, cos, sin, None, None)
        return self._head(h if all_logits else h[:, -1:])

    @torch.no_grad()
    def decode_step(self, ids: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """One token per sequence: ids[B, 1] at position ``pos`` (a one-element int64 device tensor); logits [B, 1, V]."""
        B = ids.shape[0]
        return self._gather_vocab(self._decode_local(ids, pos)).view(B, 1, -1)

    @torch.no_grad()
    def decode_greedy(self, ids: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """``decode_step`` followed by the greedy choice: next token ids [B, 1] (first maximum of the logits,
        as ``logits[:, -1].argmax(-1)`` in the reference's decode loop).  Under tensor parallelism with the peer
        all-reduce, each rank picks the first maximum of its vocabulary shard and the ranks exchange those
        candidates (``argmax_allreduce``) instead of all-gathering the logits."""
        if self.world == 1 and self.fused and self.lm_head.q is not None and ids.shape[0] <= 8:
            # W4 lm_head on one GPU: the greedy choice runs inside the lm_head GEMV (no logits round trip)
            return w4a16_matmul_argmax(self._decode_hidden(ids, pos), *self.lm_head.q)
        local = self._decode_local(ids, pos)
        if self.world > 1 and self.peers is not None:
            return argmax_allreduce(self.peers, local, self.rank * local.shape[-1])
        return argmax_last(self._gather_vocab(local))

    def _decode_local(self, ids: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """This rank's logits [B, V / world] of one decode step."""
        if self.persistent is not None or self.fused:
            return self.lm_head(self._decode_hidden(ids, pos))
        B = ids.shape[0]
        h = F.embedding(ids, self.embed)
        cos = self.cos.index_select(0, pos)
        sin = self.sin.index_select(0, pos)
        mask = (self.positions <= pos)[None, None, None, :]
        for i in range(len(self.layers)):
            h = self._layer(i, h, cos, sin, pos, mask)
        return self.lm_head(rms_norm(h, self.norm, self.eps)).view(B, -1)

    def _decode_hidden(self, ids: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """The final-normed hidden state [B, H] of one decode step (the lm_head's input); fused kernels only."""
        B = ids.shape[0]
        if self.persistent is not None and B <= self.max_batch:
            h = self.persistent.run(ids, pos)
            x = torch.empty_like(h)
            add_rmsnorm(h, None, self.norm, x, self.eps)
            return x
        assert self.fused, "the unfused decode step has no separate hidden-state form"
        return self._decode_step_fused(ids, pos)

    def _decode_step_fused(self, ids: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        B = ids.shape[0]
        nq, nkv, hd = self.nh_l, self.nkv_l, self.hd
        cur = F.embedding(ids.view(B), self.embed)  # [B, H], the residual stream (ping-pongs with `other`)
        other = torch.empty_like(cur)
        x = torch.empty_like(cur)
        q = torch.empty(B, nq, hd, device=cur.device, dtype=torch.bfloat16)
        att = torch.empty(B, nq * hd, device=cur.device, dtype=torch.bfloat16)
        act = torch.empty(B, self.inter_l, device=cur.device, dtype=torch.bfloat16)
        fold = self.w4 and B <= 32  # norms and SwiGLU run inside the W4 kernels' activation staging
        delta = None
        for i, L in enumerate(self.layers):
            kc, vc = self.k_cache[i, :B], self.v_cache[i, :B]
            if fold:
                if delta is None:
                    qkv = w4a16_matmul_prologue(PROLOGUE_RMSNORM, cur, *L["qkv"].q, norm_weight=L["ln1"], eps=self.eps)
                else:
                    qkv = w4a16_matmul_prologue(PROLOGUE_RMSNORM, cur, *L["qkv"].q, delta=delta, norm_weight=L["ln1"],
                                                eps=self.eps, resid_out=other)
                    cur, other = other, cur
            else:
                add_rmsnorm(cur, delta, L["ln1"], x, self.eps)
                qkv = L["qkv"](x)
            rope_kv_cache(qkv, self.cos, self.sin, pos, q, kc, vc, nq, nkv)
            decode_attention(q, kc, vc, pos, att, nq, nkv, hd ** -0.5)
            fused_ar = fold and self.peers is not None and self.matmul_allreduce
            if fused_ar:
                o = self._matmul_allreduce_or_none(att, L["o"].q)
                fused_ar = o is not None
            if not fused_ar:
                o = self._all_reduce(L["o"](att))
            if fold:
                gu = w4a16_matmul_prologue(PROLOGUE_RMSNORM, cur, *L["gu"].q, delta=o, norm_weight=L["ln2"],
                                           eps=self.eps, resid_out=other)
                cur, other = other, cur
                delta = self._matmul_allreduce_or_none(gu, L["down"].q, PROLOGUE_SWIGLU) if fused_ar else None
                if delta is None:
                    delta = self._all_reduce(w4a16_matmul_prologue(PROLOGUE_SWIGLU, gu, *L["down"].q))
            else:
                add_rmsnorm(cur, o, L["ln2"], x, self.eps)
                silu_mul(L["gu"](x), act)
                delta = self._all_reduce(L["down"](act))
        add_rmsnorm(cur, delta, self.norm, x, self.eps)
        return x
