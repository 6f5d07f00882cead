"""One rank of the multi-GPU expert-parallel check (launched by
tests/test_ep.py under torch.distributed.run). Every rank loads the same
seeded experts, runs its own token batches through ExpertParallel over NCCL
(argument "nccl") or PeerExpertParallel over peer memory (argument "peer"),
owning its share of the experts, and compares with its own single-GPU
tlmg_expert_ffn_batch call bit for bit; prints EP-OK on success.

With "peer" it then checks failure detection on the host side of a bounded
device wait: rank 0 makes one more layer call that no other rank joins, its
barrier gives up after 1 s, and the call raises TLMG_EIO; the other ranks
wait for that on the host before closing."""
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
from tierlm_b200.ep import ExpertParallel, PeerExpertParallel  # noqa: E402
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
    peer = len(sys.argv) > 1 and sys.argv[1] == "peer"
    ep = PeerExpertParallel(ctx, D, E, k, 64, device=dev) if peer else ExpertParallel(ctx, D, E, k, device=dev)
    ok = True
    sizes = (64, 5 if rank == 0 else 0, 17, 1, 33)
    outs = []
    for call, n in enumerate(sizes):
        trng = np.random.default_rng(1000 * rank + call)
        x = torch.from_numpy(trng.standard_normal((n, D)).astype(np.float32)).to(dev)
        lg = torch.from_numpy(trng.standard_normal((n, E)).astype(np.float32)).to(dev)
        ffn = torch.empty((max(n, 1), D), device=dev)
        ids = torch.empty((max(n, 1), k), dtype=torch.int32, device=dev)
        w = torch.empty((max(n, 1), k), device=dev)
        if peer:   # back-to-back calls, one check after the last
            ep.ffn_batch(0, x, lg, ffn, check=call == len(sizes) - 1, ids=ids, w=w)
        else:
            ep.ffn_batch(0, x, lg, ffn)
        outs.append((x, lg, ffn, ids, w))
    ctx.check()
    for call, (x, lg, ffn, ids, w) in enumerate(outs):
        n = x.shape[0]
        ref = torch.empty((max(n, 1), D), device=dev)
        rid = torch.empty((max(n, 1), k), dtype=torch.int32, device=dev)
        rw = torch.empty((max(n, 1), k), device=dev)
        if n:
            ctx.expert_ffn_batch(0, x, lg, ref, rid, rw)
        ctx.check()
        a = ffn[:n].cpu().numpy().view(np.uint32)
        b = ref[:n].cpu().numpy().view(np.uint32)
        if not np.array_equal(a, b):
            print(f"rank {rank} call {call}: {int((a != b).sum())} differing values", flush=True)
            ok = False
        if peer and not (torch.equal(ids[:n], rid[:n]) and torch.equal(w[:n].view(torch.int32),
                                                                         rw[:n].view(torch.int32))):
            print(f"rank {rank} call {call}: ids / weights differ", flush=True)
            ok = False
    dist.barrier()
    if peer:
        if rank == 0:
            x = torch.zeros((3, D), device=dev)
            lg = torch.zeros((3, E), device=dev)
            ffn = torch.empty((3, D), device=dev)
            try:
                ep.ffn_batch(0, x, lg, ffn)
                print("rank 0: a layer call no peer joined did not fail", flush=True)
                ok = False
            except _lib.TlmError as e:
                if e.code != _lib.TLMG_EIO:
                    print(f"rank 0: expected TLMG_EIO, got {e.code}", flush=True)
                    ok = False
        dist.barrier()   # rank 0's kernels are done before any peer unmaps its buffer
        try:
            ep.close()
        except _lib.TlmError as e:
            if not (rank == 0 and e.code == _lib.TLMG_EIO):
                raise
        dist.barrier()
    ctx.close()
    dist.destroy_process_group()
    if ok:
        print(f"EP-OK rank {rank}", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
