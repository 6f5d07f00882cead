"""CPU: pin the oracle (oracle/tlmo.c) to the reference.

- golden vectors produced by the reference's own compiled sources
  (tests/golden/make_golden.py): activation quantisation bytes, row dots of
  every integer and float dtype (random, zero, max-magnitude, quantised and
  extreme-scale rows; bell, +-1, spike and NaN activations), strided /
  unaligned / sub-range matvec, the router in all three modes with ties,
  NaNs, masks and all-masked fallbacks, and the expert FFN;
- the known-answer blocks and rules of the reference's tests/test_quant.c.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
from conftest import cases, fma32, load_npz, same_bits, split


def test_act_quant_golden(orc):
    z = load_npz("act_quant.npz")
    xs = split(z["x"], z["n"])
    outs = split(z["out"], z["out_len"])
    assert len(xs) > 60
    for x, kind, ref in zip(xs, z["kind"], outs):
        got = orc.quantize_act(int(kind), x)[:ref.size]
        assert np.array_equal(got, ref), (int(kind), x.size)


def test_dot_golden(orc):
    z = load_npz("dots.npz")
    ws = split(z["w"], z["w_len"])
    acts = split(z["a"], z["a_len"])
    n_nan = 0
    for w, a, dt, n, y in zip(ws, acts, z["dt"], z["n"], z["y"]):
        got = orc.vec_dot(int(dt), w, a, int(n))
        assert same_bits(got, y), (int(dt), int(n), got, y)
        n_nan += bool(np.isnan(y))
    assert n_nan > 0   # the NaN-activation edge really ran


def test_matvec_golden(orc):
    for c in cases("matvec.npz"):
        dt, n, rb, off, r0, r1 = (int(c[k]) for k in ("dt", "n", "rb", "off", "r0", "r1"))
        y = orc.matvec_rows(dt, c["mem"], rb, c["act"], n, r0, r1, w_offset=off)
        assert same_bits(y[r0:r1], c["y"][r0:r1]).all(), (dt, n, rb, off)


@pytest.mark.parametrize("mode", [0, 1])
def test_route_golden(orc, mode):
    """Mode 0 (libm expf, as the reference) must be bit-exact; mode 1 (the
    correctly rounded expf of the CUDA tier) must give the same ids and
    weights within 2 ulp (libm expf misrounds ~4e-5 of inputs by 1 ulp)."""
    orc.set_expf_mode(mode)
    try:
        for c in cases("route.npz"):
            ids, w = orc.route(int(c["router"]), c["logits"], int(c["k"]), float(c["scale"]),
                               mask=c.get("mask"), bias=c.get("bias"))
            if mode == 0:
                assert np.array_equal(ids, c["ids"]), c
                assert same_bits(w, c["w"]).all(), c
            else:
                assert np.array_equal(ids, c["ids"])
                np.testing.assert_allclose(w, c["w"], rtol=3e-7, atol=1e-30)
    finally:
        orc.set_expf_mode(0)


def ffn_inputs(c):
    from tests.golden.make_golden import ffn_case
    seed, D, de, E, k = (int(c[x]) for x in ("seed", "D", "de", "E", "k"))
    experts, x, logits, digest = ffn_case(seed, D, de, E, k, tuple(int(v) for v in c["dts"]))
    assert digest == str(c["digest"]), "synthetic weight generator drifted from the fixture"
    return experts, x, logits


def test_expert_ffn_golden(orc):
    for c in cases("expert_ffn.npz"):
        experts, x, logits = ffn_inputs(c)
        geom = dict(d_model=int(c["D"]), d_expert=int(c["de"]), n_experts=int(c["E"]), top_k=int(c["k"]),
                    router=int(c["router"]))
        ffn, ids, w = orc.expert_ffn(geom, experts, x, logits)
        assert np.array_equal(ids, c["ids"])
        assert same_bits(w, c["w"]).all()
        assert same_bits(ffn, c["ffn"]).all(), np.abs(ffn - c["ffn"]).max()


# ---- known answers of the reference test suite ---------------------------
def put_f16(buf, off, v):
    buf[off:off + 2] = np.array([v], np.float16).view(np.uint8)


def test_q4k_q6k_element_order(orc):
    """tests/test_quant.c:398-423: hand-built blocks, dequantised."""
    blk = np.zeros(210, np.uint8)
    put_f16(blk, 0, 1.0)
    put_f16(blk, 2, 0.0)
    blk[4 + 1] = 2
    blk[4 + 8 + 2] = 3
    blk[16 + 32 * 0 + 5] = 0x70
    blk[16 + 32 * 3 + 9] = 0x04
    y = orc.dequantize_row(12, blk, 256)
    assert np.count_nonzero(y) == 2 and y[37] == 14.0 and y[201] == 12.0
    blk = np.zeros(210, np.uint8)
    put_f16(blk, 208, 1.0)
    blk[192:208] = 1
    blk[128:192] = 0xAA
    blk[64 + 32 + 7] = 0x50
    y = orc.dequantize_row(14, blk, 256)
    assert np.count_nonzero(y) == 1 and y[231] == 5.0


def test_act_quant_rules(orc):
    """tests/test_quant.c:434-538."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal(512).astype(np.float32)
    x[3] = -100.0
    buf = orc.quantize_act(15, x)
    for b in range(2):
        blk = buf[292 * b: 292 * (b + 1)]
        d = blk[:4].view(np.float32)[0]
        q = blk[4:260].view(np.int8)
        amax = np.abs(x[256 * b: 256 * (b + 1)]).max()
        assert d == np.float32(amax) / np.float32(127.0) and d > 0
        assert q.min() >= -127 and (np.abs(q) == 127).any()
        assert np.array_equal(blk[260:292].view(np.int16), q.reshape(16, 16).astype(np.int32).sum(1))
    assert buf[4 + 3].view(np.int8) == -127
    z = np.zeros(40, np.float32)
    z[33] = 1.0
    zb = orc.quantize_act(8, z[:34])
    assert zb[:4].view(np.float32)[0] == 0.0 and zb[36:40].view(np.float32)[0] == np.float32(1 / 127)
    assert zb[36 + 4 + 1].view(np.int8) == 127
    v = ((np.arange(32) - 16) * 2.0 ** -140).astype(np.float32)
    ab = orc.quantize_act(8, v)
    q = ab[4:36].view(np.int8)
    assert q[0] == -127 and q[16] == 0 and q[24] == 64
    v = rng.standard_normal(512).astype(np.float32)
    v[10] = np.nan
    v[300] = np.inf
    kb = orc.quantize_act(15, v)
    assert np.isnan(kb[:4].view(np.float32)[0]) and kb[292:296].view(np.float32)[0] == np.inf


def test_dot_vs_double_reference(orc):
    """tests/test_quant.c:559-631: |dot - double ref| < 2e-6 * sum|w*x|."""
    from tierlm_b200 import synth
    rng = np.random.default_rng(5)
    n = 2048
    for dt in (8, 12, 13, 14, 15, 39):
        for rep in range(6):
            w = synth.rand_rows(dt, 1, n, rng).reshape(-1)
            x = rng.standard_normal(n).astype(np.float32)
            kind = orc.act_kind_for(dt)
            a = orc.quantize_act(kind, x)
            wd = orc.dequantize_row(dt, w, n).astype(np.float64)
            ad = a[: orc.qact_bytes(kind, n)]
            bs = 292 if kind == 15 else 36
            qk = 256 if kind == 15 else 32
            xd = np.concatenate([ad[bs * b: bs * b + 4].view(np.float32).astype(np.float64) *
                                 ad[bs * b + 4: bs * b + 4 + qk].view(np.int8) for b in range(n // qk)])
            ref = float((wd * xd).sum())
            sa = float(np.abs(wd * xd).sum())
            got = orc.vec_dot(dt, w, a, n)
            assert abs(got - ref) <= 2e-6 * sa + 1e-30, (dt, got, ref)


def test_block_partials_consistent(orc):
    """The exported per-block int32 partials reproduce the row dot through the
    reference's fmaf chain (tlm_quant.c:838-841, :880)."""
    from tierlm_b200 import synth
    rng = np.random.default_rng(9)
    n = 1024
    for dt in (12, 13, 14):
        w = synth.rand_rows(dt, 1, n, rng).reshape(-1)
        a = orc.quantize_act(15, rng.standard_normal(n).astype(np.float32))
        isum, msum = orc.block_partials(dt, w, a, n)
        acc = np.float32(0.0)
        bb = {12: 144, 13: 176, 14: 210}[dt]
        for b in range(n // 256):
            da = a[292 * b: 292 * b + 4].view(np.float32)[0]
            if dt == 14:
                dA = np.float32(w[bb * b + 208: bb * b + 210].view(np.float16).astype(np.float32)[0] * da)
                acc = fma32(dA, np.float32(isum[b]), acc)
            else:
                dA = np.float32(w[bb * b: bb * b + 2].view(np.float16).astype(np.float32)[0] * da)
                dM = np.float32(w[bb * b + 2: bb * b + 4].view(np.float16).astype(np.float32)[0] * da)
                acc = fma32(dA, np.float32(isum[b]), acc)
                acc = fma32(-dM, np.float32(msum[b]), acc)
        assert same_bits(acc, orc.vec_dot(dt, w, a, n))


def test_expf_cr_sample(orc):
    """The oracle twin of the device expf is correctly rounded: compare with
    exp in float64 rounded once to float32 on a dense sample of the routing
    and SiLU range (the full 2^32-input check was run once on the host)."""
    lib = orc.lib()
    rng = np.random.default_rng(1)
    xs = np.concatenate([np.linspace(-103.9, 88.7, 20001), rng.uniform(-20, 20, 20000),
                         rng.uniform(-1e-3, 1e-3, 5000)]).astype(np.float32)
    bad = 0
    for x in xs:
        ref = np.float32(np.exp(np.float64(x)))
        bad += not bool(same_bits(lib.tlmo_expf_cr(float(x)), ref))
    assert bad == 0
    assert lib.tlmo_expf_cr(89.0) == np.inf and lib.tlmo_expf_cr(-104.0) == 0.0
    assert np.isnan(lib.tlmo_expf_cr(float("nan")))
