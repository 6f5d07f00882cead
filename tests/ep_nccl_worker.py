"""One rank of the two-GPU expert-parallel check (launched by
tests/test_ep.py under torch.distributed.run). Every rank loads the same
seeded experts, runs its own token batch through ExpertParallel over NCCL
(owning half of the experts) and compares with its own single-GPU
tlmg_expert_ffn_batch call bit for bit; prints EP-OK on success."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from tierlm_b200 import _lib, synth  # noqa: E402
from tierlm_b200.ep import ExpertParallel  # noqa: E402
from tierlm_b200.moe import MoeContext  # noqa: E402


def main() -> int:
    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    _lib.check(_lib.load().tlmg_init(local))
    D, de, E, k = 2048, 768, 32, 8
    rng = np.random.default_rng(99)
    experts = [synth.rand_expert(rng, D, de, (12, 12, 14)) for _ in range(E)]
    ctx = MoeContext(1, D, de, E, k, device=local)
    for e, (payload, off, dts) in enumerate(experts):
        ctx.set_expert(0, e, dts, payload, off)
    ctx.set_stream(torch.cuda.current_stream(dev))
    ep = ExpertParallel(ctx, D, E, k, device=dev)
    ok = True
    for call, n in enumerate((64, 5 if rank == 0 else 0, 17)):
        trng = np.random.default_rng(1000 * rank + call)
        x = torch.from_numpy(trng.standard_normal((n, D)).astype(np.float32)).to(dev)
        lg = torch.from_numpy(trng.standard_normal((n, E)).astype(np.float32)).to(dev)
        ffn = torch.empty((max(n, 1), D), device=dev)
        ep.ffn_batch(0, x, lg, ffn)
        ref = torch.empty((max(n, 1), D), device=dev)
        if n:
            ctx.expert_ffn_batch(0, x, lg, ref)
        ctx.check()
        a = ffn[:n].cpu().numpy().view(np.uint32)
        b = ref[:n].cpu().numpy().view(np.uint32)
        if not np.array_equal(a, b):
            print(f"rank {rank} call {call}: {int((a != b).sum())} differing values", flush=True)
            ok = False
    dist.barrier()
    ctx.close()
    dist.destroy_process_group()
    if ok:
        print(f"EP-OK rank {rank}", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
