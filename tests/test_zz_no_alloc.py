"""GPU: the allocation-free expert FFN (tlmg_expert_ffn_noalloc).

Some callers cannot allocate device memory on their decode path: a host
runtime that sizes every buffer once at start-up and then runs a
latency-bound token loop, where cudaMalloc / cudaFree may block or
synchronise the device. tlmg_expert_ffn_noalloc serves them with the
caller's buffers plus one fixed scratch array inside the library. This test
calls it through the C ABI twice in a row, with different inputs, and
checks every output bit against the context-based tlmg_expert_ffn on the
same experts; it also checks that free device memory does not change across
the calls. It lives in its own file so that pytest collects it last.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_noalloc_matches_context_path():
    from conftest import same_bits
    from tierlm_b200 import _lib, synth
    from tierlm_b200.moe import MoeContext
    from tierlm_b200.quant import stream_handle

    assert torch.cuda.is_available()
    lib = _lib.load()
    _lib.check(lib.tlmg_init(0))
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(2026)
    D, de, E, k = 2048, 768, 24, 8
    experts = [synth.rand_expert(rng, D, de, (12, 12, 14)) for _ in range(E)]

    ctx = MoeContext(1, D, de, E, k)
    for e, (payload, off, dts) in enumerate(experts):
        ctx.set_expert(0, e, dts, payload, off)
    # the caller's own device copies of the expert payloads
    bufs = [torch.from_numpy(p).to(dev) for p, _, _ in experts]
    table = (_lib.ExpertSlot * E)()
    for e, (payload, off, dts) in enumerate(experts):
        for m in range(3):
            table[e].m[m] = bufs[e].data_ptr() + off[m]
            table[e].dt[m] = dts[m]

    xs = torch.from_numpy(rng.standard_normal((2, D)).astype(np.float32)).to(dev)
    lgs = torch.from_numpy(rng.standard_normal((2, E)).astype(np.float32)).to(dev)
    want = torch.zeros((2, D), device=dev)
    want_ids = torch.zeros((2, k), dtype=torch.int32, device=dev)
    want_w = torch.zeros((2, k), device=dev)
    for t in range(2):
        ctx.expert_ffn(0, xs[t], lgs[t], want[t], want_ids[t], want_w[t])
    ctx.check()
    got = torch.full((2, D), float("nan"), device=dev)
    ids = torch.full((2, k), -1, dtype=torch.int32, device=dev)
    w = torch.full((2, k), float("nan"), device=dev)
    torch.cuda.synchronize()
    stream = C.c_void_p(stream_handle())
    free = []
    for t in range(2):                                  # two calls in a row
        free.append(torch.cuda.mem_get_info(dev)[0])
        rc = lib.tlmg_expert_ffn_noalloc(table, E, D, de, k, 0, 1.0, C.c_void_p(xs[t].data_ptr()),
                                         C.c_void_p(lgs[t].data_ptr()), C.c_void_p(got[t].data_ptr()),
                                         C.c_void_p(ids[t].data_ptr()), C.c_void_p(w[t].data_ptr()), stream)
        _lib.check(rc)
    torch.cuda.synchronize()
    free.append(torch.cuda.mem_get_info(dev)[0])
    assert free[1] == free[2], free                     # no device allocation by the second call
    assert np.array_equal(ids.cpu().numpy(), want_ids.cpu().numpy())
    assert same_bits(w.cpu().numpy(), want_w.cpu().numpy()).all()
    assert same_bits(got.cpu().numpy(), want.cpu().numpy()).all()
    # sizes beyond the fixed scratch are refused with a clear error
    rc = lib.tlmg_expert_ffn_noalloc(table, E, D, 256 * 200, k, 0, 1.0, C.c_void_p(xs[0].data_ptr()),
                                     C.c_void_p(lgs[0].data_ptr()), C.c_void_p(got[0].data_ptr()), None, None, stream)
    assert rc == _lib.TLMG_ERANGE and b"scratch" in lib.tlmg_errmsg()
    ctx.close()
