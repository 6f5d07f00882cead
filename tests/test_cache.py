"""HBM expert-slot cache (tlmg_cache_enable / tlmg_set_expert_host): experts
in pinned host memory, a pool of HBM slots smaller than the expert count,
side-stream copies on misses. Every result must equal the HBM-resident
context bit for bit; the decisions are the reference store's policy
(src/lib/tlm_store.c, tests/test_store_policy.py replays it against the
reference): a call's hits are never evicted by its own misses, victims are
the lowest (frequency, last use), hints obey the demand reserve."""
from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import same_bits

pytestmark = pytest.mark.gpu

D, DE, E, K = 512, 256, 24, 4
DTS = (12, 12, 14)


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from tierlm_b200 import _lib
    _lib.check(_lib.load().tlmg_init(0))
    return torch.device("cuda:0")


def _experts(n_layers=1, seed=8):
    from tierlm_b200 import synth
    rng = np.random.default_rng(seed)
    return [[synth.rand_expert(rng, D, DE, DTS) for _ in range(E)] for _ in range(n_layers)]


def _contexts(experts, n_slots, n_layers=1):
    from tierlm_b200.moe import MoeContext
    res = MoeContext(n_layers, D, DE, E, K)
    cac = MoeContext(n_layers, D, DE, E, K)
    slot_bytes = max(p.nbytes for lay in experts for p, _, _ in lay) + 3 * 512
    cac.cache_enable(n_slots, slot_bytes)
    pinned = []
    for l in range(n_layers):
        for e, (payload, off, dts) in enumerate(experts[l]):
            res.set_expert(l, e, dts, payload, off)
            p = torch.from_numpy(payload).pin_memory()
            pinned.append(p)
            cac.set_expert_host(l, e, dts, p, off)
    return res, cac, pinned


def test_cache_matches_resident(dev):
    """40 tokens through a 10-slot cache of 24 experts (host and device
    buffers): identical bits, ids and weights; misses, hits and evictions."""
    experts = _experts()
    res, cac, pinned = _contexts(experts, n_slots=10)
    rng = np.random.default_rng(3)
    seen = set()
    for t in range(40):
        x = rng.standard_normal(D).astype(np.float32)
        lg = rng.standard_normal(E).astype(np.float32)
        if t % 5 == 0:
            lg[:] = lg[0]                          # all-tie row: ids 0..3
        a, b = np.zeros(D, np.float32), np.zeros(D, np.float32)
        ia, ib = np.zeros(K, np.int32), np.zeros(K, np.int32)
        wa, wb = np.zeros(K, np.float32), np.zeros(K, np.float32)
        res.expert_ffn(0, x, lg, a, ia, wa)
        if t % 2:
            cac.expert_ffn(0, x, lg, b, ib, wb)
        else:
            xd, ld, fd = (torch.from_numpy(v).to(dev) for v in (x, lg, np.zeros(D, np.float32)))
            cac.expert_ffn(0, xd, ld, fd)
            cac.check()
            b = fd.cpu().numpy()
            ib, wb = ia, wa
        assert np.array_equal(ia, ib) and same_bits(wa, wb).all(), t
        assert same_bits(a, b).all(), t
        seen.update(int(i) for i in ia)
    st = cac.cache_stats()
    assert st["misses"] >= min(len(seen), 10) and st["hits"] > 0 and st["evictions"] > 0, st
    assert st["misses"] + st["hits"] == 40 * K, st
    per_expert = 2 * DE * (D // 256 * 144) + D * (DE // 256 * 210)   # gate + up (Q4_K) + down (Q6_K) bytes
    assert st["bytes"] == st["misses"] * per_expert, st
    res.close()
    cac.close()


def test_cache_prefetch_and_policy(dev):
    """Hints follow the reference store's rules: with exactly top_k slots
    every hint is dropped (the demand reserve); with 2 top_k slots a hint of
    the next token's experts turns misses into hint hits once the
    frequencies of earlier selections have decayed (one tick per token).
    Results stay bit-identical to resident experts throughout."""
    experts = _experts(seed=9)
    for n_slots, expect_hints in ((K, False), (2 * K, True)):
        res, cac, pinned = _contexts(experts, n_slots=n_slots)
        rng = np.random.default_rng(4)
        for t in range(48):
            x = rng.standard_normal(D).astype(np.float32)
            lg = rng.standard_normal(E).astype(np.float32)
            ids = np.argsort(-lg, kind="stable")[:K].astype(np.int32)   # softmax top-k = largest logits
            cac.cache_prefetch(0, ids)
            a, b = np.zeros(D, np.float32), np.zeros(D, np.float32)
            res.expert_ffn(0, x, lg, a)
            cac.expert_ffn(0, x, lg, b)
            cac.cache_tick()
            assert same_bits(a, b).all(), (n_slots, t)
        st = cac.cache_stats()
        assert st["hits"] + st["misses"] == 48 * K, st
        if expect_hints:
            assert st["prefetched"] > 0 and st["prefetch_hits"] > 0, st
        else:
            assert st["prefetched"] == 0 and st["prefetch_hits"] == 0, st
        res.close()
        cac.close()


def test_cache_lookahead_moe_layer(dev):
    """moe_layer over 4 cached layers with the GPU router lookahead (the next
    layer's RMSNorm + router on the current residual, top-k hints after the
    current acquisition) gives the resident context's bits, and the hints
    are taken and used."""
    from tierlm_b200 import synth
    from tierlm_b200.moe import MoeContext
    NL = 4
    rng = np.random.default_rng(12)
    experts = [[synth.rand_expert(rng, D, DE, DTS) for _ in range(E)] for _ in range(NL)]
    norms = [(1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32) for _ in range(NL)]
    routers = [(0.05 * rng.standard_normal((E, D))).astype(np.float32) for _ in range(NL)]
    res, cac, pinned = _contexts(experts, n_slots=3 * K, n_layers=NL)
    for ctx in (res, cac):
        for l_ in range(NL):
            ctx.set_layer(l_, norms[l_], 0, routers[l_], D * 4)
    cac.cache_lookahead(1, 0)
    for t in range(24):
        h = rng.standard_normal(D).astype(np.float32)
        ha, hb = h.copy(), h.copy()
        for l_ in range(NL):
            ia, ib = np.zeros(K, np.int32), np.zeros(K, np.int32)
            res.moe_layer(l_, ha, ia)
            cac.moe_layer(l_, hb, ib)
            assert np.array_equal(ia, ib) and same_bits(ha, hb).all(), (t, l_)
        cac.cache_tick()
    st = cac.cache_stats()
    assert st["hits"] + st["misses"] == 24 * NL * K, st
    assert st["prefetched"] > 0 and st["prefetch_hits"] > 0, st
    res.close()
    cac.close()


def test_cache_many_and_batch(dev):
    """expert_ffn_many (layers in turn) and expert_ffn_batch on cached layers
    give the resident bits (per-token path inside)."""
    NL = 2
    experts = _experts(n_layers=NL, seed=10)
    res, cac, pinned = _contexts(experts, n_slots=6, n_layers=NL)
    rng = np.random.default_rng(5)
    T = 9
    x = rng.standard_normal((T, D)).astype(np.float32)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    a, b = np.zeros((T, D), np.float32), np.zeros((T, D), np.float32)
    res.expert_ffn_many(0, x, lg, a)
    cac.expert_ffn_many(0, x, lg, b)
    assert same_bits(a, b).all()
    a2, b2 = np.zeros((T, D), np.float32), np.zeros((T, D), np.float32)
    res.expert_ffn_batch(1, x, lg, a2)
    cac.expert_ffn_batch(1, x, lg, b2)
    assert same_bits(a2, b2).all()
    res.close()
    cac.close()


def test_cache_errors(dev):
    """Too few slots, resident and cached experts mixed in one layer, and a
    cached layer on the expert-parallel path are refused loudly."""
    from tierlm_b200 import _lib
    from tierlm_b200.moe import MoeContext
    experts = _experts(seed=11)
    ctx = MoeContext(1, D, DE, E, K)
    with pytest.raises(_lib.TlmError) as ei:
        ctx.cache_enable(K - 1, 1 << 20)
    assert ei.value.code == _lib.TLMG_EINVAL
    ctx.cache_enable(K, 1 << 20)
    payload, off, dts = experts[0][0]
    p = torch.from_numpy(payload).pin_memory()
    ctx.set_expert_host(0, 0, dts, p, off)
    with pytest.raises(_lib.TlmError) as ei:
        ctx.set_expert(0, 1, dts, payload, off)
    assert ei.value.code == _lib.TLMG_EBUSY
    x = torch.zeros((1, D), device=dev)
    lg = torch.zeros((1, E), device=dev)
    send = torch.empty((K, ctx.ep_record_bytes), dtype=torch.uint8, device=dev)
    perm = torch.empty(K, dtype=torch.int32, device=dev)
    w = torch.empty(K, device=dev)
    with pytest.raises(_lib.TlmError) as ei:
        ctx.ep_dispatch(0, x, lg, 1, send, perm, w)
    assert ei.value.code == _lib.TLMG_EUNSUP
    ctx.close()
