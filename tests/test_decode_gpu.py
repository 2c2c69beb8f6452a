"""Model-level parity of the W4 decode path against the reference's own quality oracle.

The reference validates its W4 kernels at model level by comparing with the
"fake-quant" model: ``quantize_model_linears(model, fake=True)`` writes
``dequantize_int4_ref(..., bf16)`` back into every ``nn.Linear``
(``int4_triton/qlinear.py:54-68``, ``benchmarks/eval_llama.py:215-220``).  Here a
small random-init Llama (``transformers``' own implementation, llama3 rotary
scaling, GQA, tied embeddings) is that oracle; ``LlamaTP`` built from the same
weights must give logits within the north star's 2e-2 max-abs bound, for the
prompt (tcgen05 GEMM path, M > 16) and for cached decode steps (GEMV path,
M = 1), eager and replayed from a CUDA graph.
"""
from __future__ import annotations

import copy
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2  # max-abs logits bound of the north star
HERE = os.path.dirname(os.path.abspath(__file__))


def tiny_config():
    from transformers import LlamaConfig

    return LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=131072,
                       rms_norm_eps=1e-5, tie_word_embeddings=True, rope_theta=500000.0,
                       rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                                     "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})


def build_hf(seed: int = 0, config=None):
    from transformers import LlamaForCausalLM

    torch.manual_seed(seed)
    with torch.device("cuda"):
        model = LlamaForCausalLM(config if config is not None else tiny_config())
    return model.to(torch.bfloat16).eval()


@pytest.fixture(scope="module")
def models(cuda_device):
    from int4_b200 import quantize_model_linears

    hf = build_hf()
    fake = copy.deepcopy(hf)
    quantize_model_linears(fake, 128, skip=("lm_head",), fake=True)
    return hf, fake


def _ids(B, S, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 512, (B, S), generator=g).cuda()


@torch.no_grad()
def test_bf16_decoder_matches_transformers(models):
    from int4_b200.decode import LlamaTP

    hf, _ = models
    ids = _ids(1, 40, 1)
    ours = LlamaTP(hf, w4=False, max_seq=128).prefill(ids, all_logits=True).float()
    ref = hf(ids).logits.float()
    assert (ours - ref).abs().max().item() <= LOGIT_TOL


@torch.no_grad()
@pytest.mark.parametrize("S", [8, 40])
def test_w4_prefill_matches_fake_quant_reference(models, S):
    from int4_b200.decode import LlamaTP

    hf, fake = models
    ids = _ids(1, S, 2 + S)
    ours = LlamaTP(hf, w4=True, max_seq=128).prefill(ids, all_logits=True).float()
    ref = fake(ids).logits.float()
    err = (ours - ref).abs().max().item()
    assert err <= LOGIT_TOL, err


@torch.no_grad()
def test_w4_cached_decode_matches_full_recompute(models):
    from int4_b200.decode import LlamaTP

    hf, fake = models
    m = LlamaTP(hf, w4=True, max_seq=128)
    ids = _ids(1, 24, 5)
    logits = m.prefill(ids)
    seq = ids
    for step in range(6):
        nxt = logits[:, -1].argmax(-1, keepdim=True)
        seq = torch.cat([seq, nxt], 1)
        pos = torch.tensor([seq.shape[1] - 1], device="cuda")
        logits = m.decode_step(nxt, pos)
        ref = fake(seq).logits[:, -1:].float()
        err = (logits.float() - ref).abs().max().item()
        assert err <= LOGIT_TOL, (step, err)


@torch.no_grad()
def test_decode_step_replays_from_a_cuda_graph(models):
    from int4_b200.decode import LlamaTP

    hf, _ = models
    m = LlamaTP(hf, w4=True, max_seq=128)
    ids = _ids(1, 16, 7)
    first = m.prefill(ids)[:, -1].argmax(-1, keepdim=True)
    tok = first.clone()
    pos = torch.tensor([16], device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        m.decode_step(tok, pos)  # warm-up (writes position 16, rewritten below)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        out = m.decode_step(tok, pos)
    eager = []
    m.prefill(ids)
    for i in range(3):
        eager.append(m.decode_step(tok, pos).clone())
        tok.copy_(eager[-1][:, -1].argmax(-1, keepdim=True))
        pos += 1
    tok.copy_(first)
    pos.fill_(16)
    m.prefill(ids)
    for i in range(3):
        g.replay()
        torch.testing.assert_close(out, eager[i], rtol=0, atol=0)
        tok.copy_(out[:, -1].argmax(-1, keepdim=True))
        pos += 1
    torch.cuda.synchronize()


def test_two_rank_tensor_parallel_matches_one_rank():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(HERE, "tp_decode_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


@torch.no_grad()
def test_fused_decode_kernels_match_the_torch_ops(models):
    """The 9-launch fused decode step against the same step run as transformers' torch ops."""
    from int4_b200.decode import LlamaTP

    hf, _ = models
    fused = LlamaTP(hf, w4=True, max_seq=128, max_batch=2, fused=True)
    plain = LlamaTP(hf, w4=True, max_seq=128, max_batch=2, fused=False)
    ids = _ids(2, 20, 9)
    tok = fused.prefill(ids)[:, -1].argmax(-1, keepdim=True)
    plain.prefill(ids)
    for step in range(5):
        pos = torch.tensor([20 + step], device="cuda")
        a, b = fused.decode_step(tok, pos), plain.decode_step(tok, pos)
        err = (a.float() - b.float()).abs().max().item()
        assert err <= LOGIT_TOL, (step, err)
        tok = b[:, -1].argmax(-1, keepdim=True)
