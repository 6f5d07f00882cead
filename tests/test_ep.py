"""Expert parallelism (tierlm_b200.ep): partition, exchange and combine.

CPU (gloo, world size 2): the exchange logic of ExpertParallel runs with a
stand-in backend whose dispatch / experts / combine are the CPU oracle
(route, the reference's per-expert SwiGLU block, the rank-ordered combine of
src/lib/tlm_model.c:1029-1036); every rank's result must equal the
single-process oracle expert FFN bit for bit, and every owner must only
see records of its own experts.

GPU: the C ABI (tlmg_ep_dispatch / tlmg_ep_experts / tlmg_ep_combine) with
N ranks emulated in one process (the exchange done by slicing) against
tlmg_expert_ffn_batch, and with two real GPUs over NCCL when present.
"""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch
from conftest import ROOT, same_bits

from tierlm_b200.ep import ExpertParallel, owned_range, owner

D, DE, E, K, DTS = 256, 256, 6, 2, (12, 12, 14)


def test_owner_partition():
    """owner() and owned_range() agree and cover every expert exactly once."""
    for n_ranks in (1, 2, 3, 4, 8):
        for n_exp in (n_ranks, 6, 16, 128, 160):
            if n_exp < n_ranks:
                continue
            seen = []
            for r in range(n_ranks):
                lo, hi = owned_range(r, n_ranks, n_exp)
                assert lo < hi
                seen += list(range(lo, hi))
                assert all(owner(e, n_ranks, n_exp) == r for e in range(lo, hi))
            assert seen == list(range(n_exp))


# ---------------------------------------------------------------------------
class OracleEpBackend:
    """CPU stand-in for MoeContext's ep_* methods on the oracle. Its record
    is { int32 expert id, 12 zero bytes, the token's f32 input row }."""

    def __init__(self, experts, router=0):
        import oracle
        self.o = oracle
        self.experts = experts
        self.router = router
        self.ep_record_bytes = 16 + 4 * D
        self.owner_seen = set()

    def ep_dispatch(self, layer, x, logits, n_ranks, send, perm, w):
        n = x.shape[0]
        dest = np.zeros(n * K, np.int64)
        for t in range(n):
            ids, ww = self.o.route(self.router, logits[t].numpy(), K)
            for r in range(K):
                p = t * K + r
                dest[p] = owner(int(ids[r]), n_ranks, E)
                w[p] = float(ww[r])
                rec = np.zeros(self.ep_record_bytes, np.uint8)
                rec[:4] = np.array([ids[r]], np.int32).view(np.uint8)
                rec[16:] = x[t].numpy().view(np.uint8)
                self._pending = getattr(self, "_pending", {})
                self._pending[p] = rec
        order = sorted(range(n * K), key=lambda p: (dest[p], p))     # grouped by owner, ascending pair
        for q, p in enumerate(order):
            perm[p] = q
            send[q] = torch.from_numpy(self._pending[p])
        self._pending = {}
        return [int((dest == d).sum()) for d in range(n_ranks)]

    def ep_experts(self, layer, lo, hi, n_rec, recv, eo):
        geom = dict(d_model=D, d_expert=DE, n_experts=1, top_k=1, router=0)
        for q in range(n_rec):
            rec = recv[q].numpy()
            e = int(rec[:4].view(np.int32)[0])
            assert lo <= e < hi, (e, lo, hi)
            self.owner_seen.add(e)
            x = rec[16:].view(np.float32)
            _, _, _, one, _ = self.o.expert_ffn(geom, [self.experts[e]], x, np.zeros(1, np.float32),
                                                want_intermediates=True)
            eo[q] = torch.from_numpy(one[0])

    def ep_combine(self, n, back, perm, w, ffn):
        b = back.numpy()
        for t in range(n):
            f = np.zeros(D, np.float32)
            for r in range(K):
                c = (np.float32(w[t * K + r].item()) * b[int(perm[t * K + r])]).astype(np.float32)
                f = (f + c).astype(np.float32)
            ffn[t] = torch.from_numpy(f)


def _experts():
    from tierlm_b200 import synth
    rng = np.random.default_rng(404)
    return [synth.rand_expert(rng, D, DE, DTS) for _ in range(E)]


def _tokens(rank, n):
    rng = np.random.default_rng(50 + rank)
    return rng.standard_normal((n, D)).astype(np.float32), rng.standard_normal((n, E)).astype(np.float32)


def _gloo_rank(rank, world, port, sizes, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        be = OracleEpBackend(_experts())
        ep = ExpertParallel(be, D, E, K)
        out = []
        for call, n in enumerate(sizes[rank]):
            x, lg = _tokens(rank + 10 * call, n)
            ffn = torch.zeros((n, D))
            counts = ep.ffn_batch(0, torch.from_numpy(x), torch.from_numpy(lg), ffn)
            out.append((x, lg, ffn.numpy(), counts))
        q.put((rank, out, sorted(be.owner_seen), (ep.lo, ep.hi)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_gloo_world2_matches_single_process(orc):
    """Two gloo ranks: per-call token counts 5/3, then 4/0 (an idle home
    still takes part in every exchange); results equal the oracle's
    single-process expert FFN bit for bit; each owner saw only its experts."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    sizes = {0: [5, 4], 1: [3, 0]}
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, sizes, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, out, seen, rng_ = q.get(timeout=240)
            res[rank] = (out, seen, rng_)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    experts = _experts()
    geom = dict(d_model=D, d_expert=DE, n_experts=E, top_k=K, router=0)
    for rank in (0, 1):
        out, seen, (lo, hi) = res[rank]
        assert (lo, hi) == owned_range(rank, 2, E)
        assert all(lo <= e < hi for e in seen)
        for x, lg, ffn, counts in out:
            assert sum(counts["sent"]) == x.shape[0] * K
            for t in range(x.shape[0]):
                ref, _, _ = orc.expert_ffn(geom, experts, x[t], lg[t])
                assert same_bits(ffn[t], ref).all(), (rank, t)
    # what rank 0 sent to rank 1 is what rank 1 received from rank 0
    for c in range(2):
        assert res[0][0][c][3]["sent"][1] == res[1][0][c][3]["received"][0]


# ---------------------------------------------------------------------------
def _gpu_ctx(experts, D_, de, E_, k):
    from tierlm_b200.moe import MoeContext
    ctx = MoeContext(1, D_, de, E_, k)
    for e, (payload, off, dts) in enumerate(experts):
        ctx.set_expert(0, e, dts, payload, off)
    ctx.set_stream(torch.cuda.current_stream())        # ordered with the torch copies of the emulated exchange
    return ctx


@pytest.mark.gpu
@pytest.mark.parametrize("n_ranks", [1, 2, 3, 4])
def test_ep_c_abi_emulated_ranks(n_ranks):
    """N homes and owners emulated on one GPU through the C ABI: dispatch with
    N ranks, hand each owner the records of every home in home order, return
    the rows, combine; each home's ffn equals tlmg_expert_ffn_batch bitwise."""
    from tierlm_b200 import synth
    dev = torch.device("cuda:0")
    D_, de, E_, k = 1024, 512, 24, 4
    rng = np.random.default_rng(31 + n_ranks)
    experts = [synth.rand_expert(rng, D_, de, (12, 12, 14)) for _ in range(E_)]
    ctx = _gpu_ctx(experts, D_, de, E_, k)
    RB = ctx.ep_record_bytes
    homes = []
    for h in range(n_ranks):
        n = 7 + 5 * h if h != 1 else 0                              # home 1 has no tokens
        x = torch.from_numpy(rng.standard_normal((n, D_)).astype(np.float32)).to(dev)
        lg = torch.from_numpy(rng.standard_normal((n, E_)).astype(np.float32)).to(dev)
        send = torch.empty((max(n * k, 1), RB), dtype=torch.uint8, device=dev)
        perm = torch.empty(max(n * k, 1), dtype=torch.int32, device=dev)
        w = torch.empty(max(n * k, 1), dtype=torch.float32, device=dev)
        counts = ctx.ep_dispatch(0, x, lg, n_ranks, send, perm, w)
        assert sum(counts) == n * k
        homes.append(dict(x=x, lg=lg, send=send, perm=perm, w=w, counts=counts,
                          starts=np.concatenate([[0], np.cumsum(counts)]).astype(int)))
    backs = [torch.empty((max(hm["x"].shape[0] * k, 1), D_), device=dev) for hm in homes]
    for o in range(n_ranks):
        lo, hi = owned_range(o, n_ranks, E_)
        parts = [hm["send"][hm["starts"][o]:hm["starts"][o + 1]] for hm in homes]
        recv = torch.cat(parts) if sum(p.shape[0] for p in parts) else torch.empty((0, RB), dtype=torch.uint8,
                                                                                  device=dev)
        ids = recv[:, :4].contiguous().view(torch.int32).flatten().cpu().numpy()
        assert ((ids >= lo) & (ids < hi)).all()
        eo = torch.empty((max(recv.shape[0], 1), D_), device=dev)
        ctx.ep_experts(0, lo, hi, recv.shape[0], recv.contiguous(), eo)
        at = 0
        for hm, back, p in zip(homes, backs, parts):
            back[hm["starts"][o]:hm["starts"][o + 1]] = eo[at:at + p.shape[0]]
            at += p.shape[0]
    for hm, back in zip(homes, backs):
        n = hm["x"].shape[0]
        ffn = torch.empty((max(n, 1), D_), device=dev)
        ctx.ep_combine(n, back, hm["perm"], hm["w"], ffn)
        ref = torch.empty((max(n, 1), D_), device=dev)
        if n:
            ctx.expert_ffn_batch(0, hm["x"], hm["lg"], ref)
        ctx.check()
        assert same_bits(ffn[:n].cpu().numpy(), ref[:n].cpu().numpy()).all()
    ctx.close()


@pytest.mark.gpu
def test_ep_dispatch_device_counts():
    """Counts written to device memory (no host wait) equal the host counts,
    and the records, permutation and weights are the same bytes."""
    from tierlm_b200 import synth
    dev = torch.device("cuda:0")
    D_, de, E_, k, n, nr = 1024, 512, 24, 4, 37, 3
    rng = np.random.default_rng(41)
    experts = [synth.rand_expert(rng, D_, de, (12, 12, 14)) for _ in range(E_)]
    ctx = _gpu_ctx(experts, D_, de, E_, k)
    RB = ctx.ep_record_bytes
    x = torch.from_numpy(rng.standard_normal((n, D_)).astype(np.float32)).to(dev)
    lg = torch.from_numpy(rng.standard_normal((n, E_)).astype(np.float32)).to(dev)
    outs = []
    for mode in ("host", "device"):
        send = torch.zeros((n * k, RB), dtype=torch.uint8, device=dev)
        perm = torch.zeros(n * k, dtype=torch.int32, device=dev)
        w = torch.zeros(n * k, dtype=torch.float32, device=dev)
        if mode == "host":
            counts = ctx.ep_dispatch(0, x, lg, nr, send, perm, w)
        else:
            cd = torch.full((nr,), -1, dtype=torch.int64, device=dev)
            ctx.ep_dispatch_async(0, x, lg, nr, send, perm, w, cd)
            ctx.check()
            counts = cd.tolist()
        outs.append((counts, send.cpu(), perm.cpu(), w.cpu()))
    assert outs[0][0] == outs[1][0] and sum(outs[0][0]) == n * k
    for a, b in zip(outs[0][1:], outs[1][1:]):
        assert torch.equal(a, b)
    empty = torch.full((nr,), -1, dtype=torch.int64, device=dev)   # no tokens: zero counts
    ctx.ep_dispatch_async(0, x[:0], lg[:0], nr, send, perm, w, empty)
    ctx.check()
    assert empty.tolist() == [0] * nr
    ctx.close()


@pytest.mark.gpu
def test_ep_foreign_record_is_loud():
    """A record naming an expert outside the owner's range gets a NaN row and
    the context reports TLMG_EINVAL at the next check."""
    from tierlm_b200 import _lib, synth
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(5)
    experts = [synth.rand_expert(rng, 512, 256, (12, 12, 14)) for _ in range(8)]
    ctx = _gpu_ctx(experts, 512, 256, 8, 2)
    RB = ctx.ep_record_bytes
    x = torch.from_numpy(rng.standard_normal((3, 512)).astype(np.float32)).to(dev)
    lg = torch.from_numpy(rng.standard_normal((3, 8)).astype(np.float32)).to(dev)
    send = torch.empty((6, RB), dtype=torch.uint8, device=dev)
    perm = torch.empty(6, dtype=torch.int32, device=dev)
    w = torch.empty(6, dtype=torch.float32, device=dev)
    ctx.ep_dispatch(0, x, lg, 1, send, perm, w)
    eo = torch.zeros((6, 512), device=dev)
    ids = send[:, :4].contiguous().view(torch.int32).flatten().cpu().numpy()
    lo = int(ids.min()) + 1                                  # the smallest expert is now foreign
    ctx.ep_experts(0, lo, 8, 6, send, eo)
    with pytest.raises(_lib.TlmError) as ei:
        ctx.check()
    assert ei.value.code == _lib.TLMG_EINVAL
    e = eo.cpu().numpy()
    assert np.isnan(e[ids < lo]).all() and not np.isnan(e[ids >= lo]).any()
    ctx.check()                                              # the error was reported once
    ctx.close()


@pytest.mark.gpu
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_ep_two_gpus(exchange):
    """Two ranks (skipped with fewer than two GPUs), the exchange over NCCL
    or over peer memory: each rank's expert-parallel result (and, over peer
    memory, its ids and weights) equals its own single-GPU batched call
    bitwise; over peer memory a layer call that no peer joins fails with
    TLMG_EIO after the bounded barrier wait."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(ROOT / "tests" / "ep_nccl_worker.py"), exchange]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert r.stdout.count("EP-OK") == 2, r.stdout[-2000:]


@pytest.mark.gpu
def test_ep_peer_one_rank():
    """PeerExpertParallel with one rank (no peers): back-to-back layer calls,
    n = 0 included, equal tlmg_expert_ffn_batch bitwise; more tokens than
    the exchange was opened for is an error."""
    from tierlm_b200 import synth
    from tierlm_b200.ep import PeerExpertParallel
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(17)
    D_, de, E_, k = 1024, 512, 24, 4
    experts = [synth.rand_expert(rng, D_, de, (12, 12, 14)) for _ in range(E_)]
    ctx = _gpu_ctx(experts, D_, de, E_, k)
    ep = PeerExpertParallel(ctx, D_, E_, k, 40, device=dev)
    runs = []
    for n in (40, 0, 3, 1, 29):
        x = torch.from_numpy(rng.standard_normal((n, D_)).astype(np.float32)).to(dev)
        lg = torch.from_numpy(rng.standard_normal((n, E_)).astype(np.float32)).to(dev)
        ffn = torch.empty((max(n, 1), D_), device=dev)
        ep.ffn_batch(0, x, lg, ffn, check=False)
        runs.append((x, lg, ffn))
    ctx.check()
    for x, lg, ffn in runs:
        n = x.shape[0]
        if not n:
            continue
        ref = torch.empty_like(ffn)
        ctx.expert_ffn_batch(0, x, lg, ref)
        ctx.check()
        assert torch.equal(ffn[:n].view(torch.int32), ref[:n].view(torch.int32))
    with pytest.raises(ValueError):
        ep.ffn_batch(0, torch.zeros((41, D_), device=dev), torch.zeros((41, E_), device=dev),
                     torch.zeros((41, D_), device=dev))
    ep.close()
    ctx.close()


@pytest.mark.gpu
def test_ep_ffn_batch_raises_device_errors():
    """ExpertParallel.ffn_batch on the CUDA path (device-side counts) raises
    the error its own kernels flagged, without an explicit ctx.check(): the
    owner range is narrowed by one expert, so records naming expert 0 are
    foreign (NaN rows, TLMG_EINVAL). The next call with the true range
    succeeds (the error is reported once)."""
    from tierlm_b200 import _lib, synth
    from tierlm_b200.ep import ExpertParallel
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(9)
    D_, de, E_, k = 512, 256, 8, 2
    experts = [synth.rand_expert(rng, D_, de, (12, 12, 14)) for _ in range(E_)]
    ctx = _gpu_ctx(experts, D_, de, E_, k)
    ep = ExpertParallel(ctx, D_, E_, k, device=dev)
    x = torch.from_numpy(rng.standard_normal((5, D_)).astype(np.float32)).to(dev)
    lg = torch.from_numpy(rng.standard_normal((5, E_)).astype(np.float32)).to(dev)
    lg[:, 0] = 10.0                                          # every token routes to expert 0
    ffn = torch.empty((5, D_), device=dev)
    ep.lo = 1
    with pytest.raises(_lib.TlmError) as ei:
        ep.ffn_batch(0, x, lg, ffn)
    assert ei.value.code == _lib.TLMG_EINVAL
    assert torch.isnan(ffn).all(dim=1).all()
    ep.lo = 0
    ep.ffn_batch(0, x, lg, ffn)
    ref = torch.empty_like(ffn)
    ctx.expert_ffn_batch(0, x, lg, ref)
    ctx.check()
    assert torch.equal(ffn.view(torch.int32), ref.view(torch.int32))
    ctx.close()
