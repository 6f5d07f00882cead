"""The expert cache's slot policy against the reference's own store.

One scripted trace - demand acquisitions of skewed routing over the layers
of a store made by the reference's tlmc, router-lookahead hints for the next
layer (partly wrong, as a lookahead is), waits, releases and step ticks - is
replayed through the reference's tlm_store (src/lib/tlm_store.c, driven by
oracle/ref_store.c, every load completed where the trace says) and through
libtlmg's slot policy (tlmg_store_*). After every operation the two must
hold the same expert in every slot with the same references and hint flags
(and, once the loads are waited for, the same state), and report the same
hits, misses, hints issued / used / dropped and evictions.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
REFSTORE = ROOT / "oracle" / "_ref" / "libtlmstore.so"


def _ref():
    L = C.CDLL(str(REFSTORE))
    P, I = C.c_void_p, C.c_int
    for n, res, args in (("refstore_open", P, [C.c_char_p, I]), ("refstore_close", None, [P]),
                         ("refstore_acquire", I, [P, I, P, I]), ("refstore_prefetch", None, [P, I, P, I]),
                         ("refstore_quiesce", None, [P]), ("refstore_wait_release", I, [P]),
                         ("refstore_tick", None, [P]), ("refstore_n_slots", I, [P]),
                         ("refstore_slot", None, [P, I, P]), ("refstore_stats", None, [P, P])):
        f = getattr(L, n)
        f.restype, f.argtypes = res, args
    return L


def _trace(rng, n_steps, L, E, k, k_la):
    """ops: ("acq", layer, ids) / ("pf", layer, ids) / ("wait",) / ("tick",)."""
    pop = [rng.permutation(E) for _ in range(L)]
    p = 1.0 / np.arange(1, E + 1) ** 1.1
    p /= p.sum()
    ops = []
    for _ in range(n_steps):
        ids = [pop[l_][rng.choice(E, size=k, replace=False, p=p)] for l_ in range(L)]
        for l_ in range(L):
            ops.append(("acq", l_, ids[l_]))
            if l_ + 1 < L:                       # lookahead for the next layer: half right, half guessed
                guess = list(ids[l_ + 1][: k // 2]) + list(pop[l_ + 1][rng.choice(E, size=k_la, replace=False, p=p)])
                seen, la = set(), []
                for g in guess:
                    if g not in seen:
                        seen.add(g)
                        la.append(int(g))
                ops.append(("pf", l_ + 1, np.array(la[:k_la], np.int32)))
            ops.append(("wait",))
        ops.append(("tick",))
    return ops


@pytest.mark.skipif(not REFSTORE.exists(), reason="oracle/_ref not built (make -C oracle gate)")
@pytest.mark.parametrize("n_slots", [8, 24, 60])
def test_policy_replays_the_reference_store(n_slots):
    from oracle import gate
    from tierlm_b200.store import StorePolicy
    R = _ref()
    man = gate.store("config1")                   # 4 layers x 32 experts, top-4
    L, E, k = 4, 32, 4
    h = R.refstore_open(str(man).encode(), n_slots)
    assert h, "reference store did not open"
    assert R.refstore_n_slots(h) == n_slots
    pol = StorePolicy(L * E, n_slots, k)
    rng = np.random.default_rng(n_slots)
    held = []
    out = (C.c_int * 4)()
    st = (C.c_int64 * 6)()
    try:
        for i, op in enumerate(_trace(rng, 40, L, E, k, 6)):
            if op[0] == "acq":
                ids = np.ascontiguousarray(op[2], np.int32)
                rc = R.refstore_acquire(h, op[1], ids.ctypes.data, len(ids))
                slots, loads, ok = pol.acquire(op[1] * E + ids)
                assert (rc == 0) == ok, (i, rc)
                held.extend(int(s) for s in slots if s >= 0)
            elif op[0] == "pf":
                ids = np.ascontiguousarray(op[2], np.int32)
                R.refstore_prefetch(h, op[1], ids.ctypes.data, len(ids))
                pol.prefetch(op[1] * E + ids)
            elif op[0] == "wait":
                assert R.refstore_wait_release(h) == 0
                for s in range(n_slots):
                    if pol.slot(s)[0] == 1:
                        pol.load_done(s)
                for s in held:
                    pol.release(s)
                held = []
            else:
                R.refstore_tick(h)
                pol.tick()
            quiet = op[0] in ("wait", "tick")
            for s in range(n_slots):
                R.refstore_slot(h, s, out)
                a, b = tuple(out), pol.slot(s)
                if not quiet:
                    # between acquire and wait the reference's reads complete when the disk
                    # answers: LOADING and READY are the same occupied slot there (with top_k 4
                    # at most 4 demand loads are in flight, so the hint rule "more than 4"
                    # cannot depend on it)
                    a, b = (min(a[0], 1),) + a[1:], (min(b[0], 1),) + b[1:]
                assert a == b, (i, op[0], s, tuple(out), pol.slot(s))
            R.refstore_stats(h, st)
            assert list(st) == pol.stats(), (i, op[0], list(st), pol.stats())
        hits, misses, issued, used, dropped, ev = pol.stats()
        assert misses > 0 and hits > 0 and issued > 0
        if n_slots < L * E:
            assert ev > 0
    finally:
        R.refstore_wait_release(h)
        R.refstore_close(h)
        pol.close()
