"""One rank of the two-GPU tensor-parallel decode check (launched by tests/test_decode_gpu.py via torchrun).

Every rank builds the same seeded tiny Llama, runs its ``LlamaTP`` shard (NCCL
all-reduce after o/down, all-gather of the vocab-parallel logits) for a prompt
and three cached decode steps, and compares with a one-rank ``LlamaTP`` of the
same weights.  Exit status 0 only if every rank stays within 2e-2 max-abs.
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


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from int4_b200.decode import LlamaTP
    from test_decode_gpu import build_hf

    worst = 0.0
    with torch.no_grad():
        hf = build_hf(0)
        g = torch.Generator().manual_seed(3)
        ids = torch.randint(0, 512, (1, 24), generator=g).to(dev)
        for lm_w4 in (False, True):
            tp = LlamaTP(hf, w4=True, quantize_lm_head=lm_w4, rank=rank, world=world, max_seq=64, device=dev)
            one = LlamaTP(hf, w4=True, quantize_lm_head=lm_w4, rank=0, world=1, max_seq=64, device=dev)
            a, b = tp.prefill(ids, all_logits=True), one.prefill(ids, all_logits=True)
            worst = max(worst, (a.float() - b.float()).abs().max().item())
            tok = b[:, -1].argmax(-1, keepdim=True)
            for step in range(3):
                pos = torch.tensor([24 + step], device=dev)
                a, b = tp.decode_step(tok, pos), one.decode_step(tok, pos)
                worst = max(worst, (a.float() - b.float()).abs().max().item())
                tok = b[:, -1].argmax(-1, keepdim=True)
    t = torch.tensor([worst], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    torch.cuda.synchronize()
    dist.destroy_process_group()
    if rank == 0:
        print(f"max |logits(tp{world}) - logits(tp1)| = {t.item():.3e}")
    return 0 if t.item() <= 2e-2 else 1


if __name__ == "__main__":
    sys.exit(main())
