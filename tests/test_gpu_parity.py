"""GPU parity: the sm_100a kernels, called through the C ABI, against the
reference's golden vectors and the CPU oracle on the same seeded inputs.

Bar (the reference's own numerics contract, src/lib/tlm_quant.h:113-128):
bit-exact for activation codes, integer block partials and every row dot.
Routing and SiLU use expf: the CUDA tier's expf is correctly rounded while
the reference calls libm expf, which misrounds ~4e-5 of inputs by one ulp.
So the layer-level tests are bit-exact against the oracle run with the same
correctly rounded expf (tlmo_set_expf_mode(1)), and against the reference's
golden outputs (libm expf) they require identical expert ids and
ROUTE_RTOL / FFN_RTOL relative agreement.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch
from conftest import cases, load_npz, same_bits, split

pytestmark = pytest.mark.gpu

ROUTE_RTOL = 3e-7      # weights: one-ulp expf differences through softmax / renorm
FFN_RTOL = 1e-5        # ffn: relative L2 vs the reference's libm-expf output


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from tierlm_b200 import _lib
    _lib.check(_lib.load().tlmg_init(0))
    return torch.device("cuda:0")


def to_dev(a: np.ndarray, dev, pad: int = 64) -> torch.Tensor:
    t = torch.zeros(a.nbytes + pad, dtype=torch.uint8, device=dev)
    t[: a.nbytes] = torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)).to(dev)
    return t


def test_quantize_act_golden(dev):
    from tierlm_b200 import quant
    z = load_npz("act_quant.npz")
    for x, kind, ref in zip(split(z["x"], z["n"]), z["kind"], split(z["out"], z["out_len"])):
        xt = torch.from_numpy(x).to(dev)
        out = quant.quantize_act(int(kind), xt)
        torch.cuda.synchronize()
        got = out.cpu().numpy()[: ref.size]
        assert np.array_equal(got, ref), (int(kind), x.size)


def test_dot_golden(dev):
    from tierlm_b200 import quant
    z = load_npz("dots.npz")
    for w, a, dt, n, y in zip(split(z["w"], z["w_len"]), split(z["a"], z["a_len"]), z["dt"], z["n"], z["y"]):
        W = to_dev(w, dev)
        A = to_dev(a, dev)
        out = torch.full((1,), -1.0, device=dev)
        quant.matvec_rows(int(dt), W, w.size, A, out, int(n), 0, 1)
        assert same_bits(out.cpu().numpy()[0], y), (int(dt), int(n))


def test_matvec_golden_strided_unaligned(dev):
    from tierlm_b200 import quant
    for c in cases("matvec.npz"):
        dt, n, rb, off, r0, r1 = (int(c[k]) for k in ("dt", "n", "rb", "off", "r0", "r1"))
        M = to_dev(c["mem"], dev)
        A = to_dev(c["act"], dev)
        y = torch.full((48,), -12345.0, device=dev)
        quant.matvec_rows(dt, M, rb, A, y, n, r0, r1, w_offset=off)
        got = y.cpu().numpy()
        assert same_bits(got[r0:r1], c["y"][r0:r1]).all(), (dt, n, rb, off)
        assert (got[:r0] == -12345.0).all() and (got[r1:] == -12345.0).all()


@pytest.mark.parametrize("dt", [8, 12, 13, 14, 15, 39, 0, 1, 2])
def test_matvec_random_vs_oracle(dev, orc, dt):
    """A 3000-row matrix of every dtype at a few widths, every row bit-exact."""
    from tierlm_b200 import quant, synth
    rng = np.random.default_rng(100 + dt)
    for n in (256, 2048, 768 if dt != 39 else 736, 4352 if dt != 39 else 4320):   # 4352: rows past 48 KB of staging
        rows = 3000
        if dt in (0, 1, 2):
            wf = rng.standard_normal((rows, n)).astype(np.float32)
            W = wf if dt == 0 else (wf.astype(np.float16) if dt == 1 else
                                    (wf.view(np.uint32) >> 16).astype(np.uint16))
            Wb = np.ascontiguousarray(W).view(np.uint8).reshape(rows, -1)
            x = rng.standard_normal(n).astype(np.float32)
            act = np.frombuffer(x.tobytes(), np.uint8).copy()
        else:
            Wb = synth.rand_rows(dt, rows, n, rng)
            x = rng.standard_normal(n).astype(np.float32)
            act = orc.quantize_act(orc.act_kind_for(dt), x)
        rb = Wb.shape[1]
        ref = orc.matvec_rows(dt, Wb, rb, act, n, 0, rows)
        y = torch.empty(rows, device=dev)
        quant.matvec_rows(dt, to_dev(Wb, dev), rb, to_dev(act, dev), y, n, 0, rows)
        got = y.cpu().numpy()
        bad = np.flatnonzero(~same_bits(got, ref))
        assert bad.size == 0, (dt, n, bad[:5], got[bad[:5]], ref[bad[:5]])


@pytest.mark.parametrize("dt", [12, 14])
def test_matvec_tall_vs_oracle(dev, orc, dt):
    """A tall matrix (70,000 rows of 2048: an lm_head's shape, each warp
    walking many rows through its deeper row pipeline), every row bit-exact."""
    from tierlm_b200 import quant, synth
    rng = np.random.default_rng(700 + dt)
    rows, n = 70000, 2048
    Wb = synth.rand_rows(dt, rows, n, rng)
    act = orc.quantize_act(orc.act_kind_for(dt), rng.standard_normal(n).astype(np.float32))
    ref = orc.matvec_rows(dt, Wb, Wb.shape[1], act, n, 0, rows)
    y = torch.empty(rows, device=dev)
    quant.matvec_rows(dt, to_dev(Wb, dev), Wb.shape[1], to_dev(act, dev), y, n, 0, rows)
    bad = np.flatnonzero(~same_bits(y.cpu().numpy(), ref))
    assert bad.size == 0, (dt, bad[:5])


@pytest.mark.parametrize("dt", [0, 1, 2, 8, 12, 13, 14, 15])
def test_dequantize_rows_vs_oracle(dev, orc, dt):
    """tlmg_dequantize_rows (the decoder step's embedding gather) against
    the oracle's tlm_dequantize_row restatement, bit for bit, on rows that
    start at odd byte offsets (a padded row stride)."""
    from tierlm_b200 import quant, synth
    rng = np.random.default_rng(300 + dt)
    rows, n = 37, 2048
    if dt in (0, 1, 2):
        wf = rng.standard_normal((rows, n)).astype(np.float32)
        W = wf if dt == 0 else (wf.astype(np.float16) if dt == 1 else (wf.view(np.uint32) >> 16).astype(np.uint16))
        Wb = np.ascontiguousarray(W).view(np.uint8).reshape(rows, -1)
    else:
        Wb = synth.rand_rows(dt, rows, n, rng)
    rb = Wb.shape[1] + 3                                   # odd stride: every row at a different alignment
    Wp = np.zeros((rows, rb), np.uint8)
    Wp[:, : Wb.shape[1]] = Wb
    ref = np.stack([orc.dequantize_row(dt, Wb[r], n) for r in range(rows)])
    y = quant.dequantize_rows(dt, to_dev(Wp, dev), rb, n, rows)
    assert same_bits(y.cpu().numpy(), ref).all(), dt


@pytest.mark.parametrize("dt", [8, 12, 13, 14, 15, 39])
def test_block_partials_vs_oracle(dev, orc, dt):
    """Integer block dot-product partial sums, bit-exact."""
    from tierlm_b200 import quant, synth
    rng = np.random.default_rng(7 + dt)
    n, rows = 2048, 512
    Wb = synth.rand_rows(dt, rows, n, rng)
    for r in range(0, rows, 7):                     # sprinkle the edge modes
        Wb[r] = synth.rand_rows(dt, 1, n, rng, mode=(r // 7) % 5 if (r // 7) % 5 != 3 else 0)
    act = orc.quantize_act(orc.act_kind_for(dt), rng.standard_normal(n).astype(np.float32))
    isum, msum = quant.block_partials(dt, to_dev(Wb, dev), Wb.shape[1], to_dev(act, dev), n, rows)
    isum, msum = isum.cpu().numpy(), msum.cpu().numpy()
    for r in range(rows):
        ri, rm = orc.block_partials(dt, Wb[r], act, n)
        assert np.array_equal(isum[r], ri) and np.array_equal(msum[r], rm), (dt, r)


def test_route_golden(dev, orc):
    from tierlm_b200 import quant
    orc.set_expf_mode(1)
    try:
        for c in cases("route.npz"):
            lg = torch.from_numpy(c["logits"]).to(dev)
            mask = torch.from_numpy(c["mask"]).to(dev) if "mask" in c else None
            bias = torch.from_numpy(c["bias"]).to(dev) if "bias" in c else None
            ids, w = quant.route(int(c["router"]), lg, int(c["k"]), float(c["scale"]), mask=mask, bias=bias)
            ids, w = ids.cpu().numpy(), w.cpu().numpy()
            oid, ow = orc.route(int(c["router"]), c["logits"], int(c["k"]), float(c["scale"]),
                                mask=c.get("mask"), bias=c.get("bias"))
            assert np.array_equal(ids, oid) and same_bits(w, ow).all(), c
            assert np.array_equal(ids, c["ids"])
            np.testing.assert_allclose(w, c["w"], rtol=ROUTE_RTOL, atol=1e-30)
    finally:
        orc.set_expf_mode(0)


def build_ctx(experts, D, de, E, k, router, n_layers=1, d_shared=0):
    from tierlm_b200.moe import MoeContext
    ctx = MoeContext(n_layers, D, de, E, k, router=router, d_shared=d_shared)
    for layer in range(n_layers):
        for e, (payload, off, dts) in enumerate(experts[layer] if n_layers > 1 else experts):
            ctx.set_expert(layer, e, dts, payload, off)
    return ctx


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


@pytest.mark.parametrize("fused", [True, False])
def test_expert_ffn_golden(dev, orc, fused):
    """The routed-expert FFN (incl. the Qwen3-30B-A3B layer shape) against
    the reference's output and, bit for bit, against the oracle - through
    the persistent kernel and through the multi-kernel path."""
    from tests.golden.make_golden import ffn_case
    for c in cases("expert_ffn.npz"):
        seed, D, de, E, k, router = (int(c[x]) for x in ("seed", "D", "de", "E", "k", "router"))
        dts = tuple(int(v) for v in c["dts"])
        experts, x, logits, digest = ffn_case(seed, D, de, E, k, dts)
        assert digest == str(c["digest"])
        ctx = build_ctx(experts, D, de, E, k, router)
        ctx.set_fused(fused)
        ffn = np.zeros(D, np.float32)
        ids = np.zeros(k, np.int32)
        w = np.zeros(k, np.float32)
        ctx.expert_ffn(0, x, logits, ffn, ids, w)            # host buffers
        assert np.array_equal(ids, c["ids"]), (ids, c["ids"])
        np.testing.assert_allclose(w, c["w"], rtol=ROUTE_RTOL)
        assert rel_l2(ffn, c["ffn"]) < FFN_RTOL
        orc.set_expf_mode(1)
        try:
            geom = dict(d_model=D, d_expert=de, n_experts=E, top_k=k, router=router)
            off, oid, ow = orc.expert_ffn(geom, experts, x, logits)
        finally:
            orc.set_expf_mode(0)
        assert np.array_equal(ids, oid) and same_bits(w, ow).all()
        bad = np.flatnonzero(~same_bits(ffn, off))
        assert bad.size == 0, (seed, bad[:5], ffn[bad[:5]], off[bad[:5]])
        # device buffers give the same bits
        xd, ld, fd = (torch.from_numpy(v).to(dev) for v in (x, logits, np.zeros(D, np.float32)))
        ctx.expert_ffn(0, xd, ld, fd)
        torch.cuda.synchronize()
        assert same_bits(fd.cpu().numpy(), ffn).all()
        ctx.close()


@pytest.mark.parametrize("variant", ["qwen-like", "shared-gated", "sigmoid-router"])
def test_moe_layer_vs_oracle(dev, orc, variant):
    """The whole moe() block (RMSNorm, router, route, experts, shared expert,
    h += ffn), bit-exact against the oracle with the same expf."""
    from tierlm_b200 import synth
    rng = np.random.default_rng({"qwen-like": 1, "shared-gated": 2, "sigmoid-router": 3}[variant])
    D, de, E, k = 512, 256, 16, 4
    router = 2 if variant == "sigmoid-router" else 0
    ds = 256 if variant == "shared-gated" else 0
    dts = (12, 12, 14) if variant != "sigmoid-router" else (14, 14, 8)
    experts = [synth.rand_expert(rng, D, de, dts) for _ in range(E)]
    norm = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    rw = (rng.standard_normal((E, D)) / np.sqrt(D)).astype(np.float32)
    bias = (0.05 * rng.standard_normal(E)).astype(np.float32) if router == 2 else None
    layer = dict(ffn_norm=norm, router_dt=0, router_w=rw, router_rb=4 * D, router_bias=bias)
    ctx = build_ctx(experts, D, de, E, k, router, d_shared=ds)
    ctx.set_layer(0, ffn_norm=norm, router_dt=0, router_w=rw, router_row_bytes=4 * D, router_bias=bias)
    if ds:
        sh = [synth.rand_rows(8, ds, D, rng), synth.rand_rows(8, ds, D, rng), synth.rand_rows(8, D, ds, rng)]
        gi = (rng.standard_normal(D) / np.sqrt(D)).astype(np.float32)
        ctx.set_shared(0, (8, 8, 8), sh[0], sh[1], sh[2], gi)
        layer["shared"] = ((8, 8, 8), sh)
        layer["shared_gate_inp"] = gi
    geom = dict(d_model=D, d_expert=de, n_experts=E, top_k=k, router=router, d_shared=ds, norm_eps=1e-6)
    for step in range(3):
        h = (rng.standard_normal(D) * (1 + step)).astype(np.float32)
        orc.set_expf_mode(1)
        try:
            ref_h, rid, rw_ = orc.moe_layer(geom, layer, experts, h)
        finally:
            orc.set_expf_mode(0)
        got = h.copy()
        ids = np.zeros(k, np.int32)
        w = np.zeros(k, np.float32)
        ctx.moe_layer(0, got, ids, w)
        assert np.array_equal(ids, rid), (ids, rid)
        assert same_bits(w, rw_).all()
        bad = np.flatnonzero(~same_bits(got, ref_h))
        assert bad.size == 0, (variant, step, bad[:5], got[bad[:5]], ref_h[bad[:5]])
    ctx.close()


def test_expert_ffn_many_matches_single(dev):
    """The batched host-buffer call equals per-token calls, layer by layer
    (token t uses layer (layer0 + t) % n_layers), through the persistent
    multi-token launch and through the per-token multi-kernel path."""
    from tierlm_b200 import synth
    rng = np.random.default_rng(21)
    D, de, E, k, NL = 512, 256, 16, 4, 3
    experts = [[synth.rand_expert(rng, D, de, (12, 12, 14)) for _ in range(E)] for _ in range(NL)]
    ctx = build_ctx(experts, D, de, E, k, 0, n_layers=NL)
    T = 7
    x = rng.standard_normal((T, D)).astype(np.float32)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    out = np.zeros((T, D), np.float32)
    n0 = ctx.launches
    ctx.expert_ffn_many(1, x, lg, out)
    assert ctx.launches - n0 == 1
    for fused in (True, False):
        ctx.set_fused(fused)
        for t in range(T):
            one = np.zeros(D, np.float32)
            ctx.expert_ffn((1 + t) % NL, x[t], lg[t], one)
            assert same_bits(one, out[t]).all(), (fused, t)
    ctx.set_fused(True)
    pinned_x = torch.from_numpy(x).pin_memory()
    pinned_l = torch.from_numpy(lg).pin_memory()
    pinned_o = torch.zeros((T, D)).pin_memory()
    ctx.expert_ffn_many(1, pinned_x, pinned_l, pinned_o)
    assert same_bits(pinned_o.numpy(), out).all()
    ctx.close()


def test_errors_are_loud(dev):
    """Bad arguments return the reference's error codes and NaN-fill rows
    (tlm_matvec_rows, src/lib/tlm_quant.c:1123-1127)."""
    from tierlm_b200 import TlmError, quant
    from tierlm_b200.moe import MoeContext
    W = torch.zeros(1024, dtype=torch.uint8, device=dev)
    A = torch.zeros(1024, dtype=torch.uint8, device=dev)
    y = torch.ones(4, device=dev)
    with pytest.raises(TlmError) as e:
        quant.matvec_rows(12, W, 144, A, y, 100, 1, 3)
    assert e.value.code == -3
    got = y.cpu().numpy()
    assert np.isnan(got[1]) and np.isnan(got[2]) and got[0] == 1 and got[3] == 1
    with pytest.raises(TlmError):
        MoeContext(1, 500, 256, 8, 2)                # d_model not a multiple of 256
    ctx = MoeContext(1, 256, 256, 4, 2)
    with pytest.raises(TlmError) as e:                # slots not loaded
        ctx.expert_ffn(0, np.zeros(256, np.float32), np.zeros(4, np.float32), np.zeros(256, np.float32))
    assert e.value.code == -6
    with pytest.raises(TlmError) as e:                # payload too short
        ctx.set_expert(0, 0, (12, 12, 14), np.zeros(100, np.uint8), (0, 0, 0))
    assert e.value.code == -4
    ctx.close()


def test_qmv_host_adapter(dev, orc):
    """The tier-table adapter (tlm_qmv_fn signature, host buffers)."""
    from tierlm_b200 import _lib, synth
    lib = _lib.load()
    rng = np.random.default_rng(4)
    for dt in (12, 14, 8):
        n, rows = 1024, 9
        Wb = synth.rand_rows(dt, rows, n, rng)
        act = orc.quantize_act(orc.act_kind_for(dt), rng.standard_normal(n).astype(np.float32))
        y = np.zeros(rows, np.float32)
        lib.tlmg_qmv_host(dt, Wb.ctypes.data, Wb.shape[1], act.ctypes.data, y.ctypes.data, n, rows)
        ref = orc.matvec_rows(dt, Wb, Wb.shape[1], act, n, 0, rows)
        assert same_bits(y, ref).all()
        d = lib.tlmg_qdot_host(dt, Wb[3].ctypes.data, act.ctypes.data, n, None)
        assert same_bits(np.float32(d), ref[3])
    ptr = C.c_void_p
    assert ptr is not None


FUSED_SHAPES = [
    # (D, de, E, k, dtypes, fused kernel expected)
    (2048, 768, 24, 8, (12, 12, 14), True),    # config-2 layer shape
    (2048, 768, 24, 8, (13, 13, 13), True),
    (2048, 768, 24, 8, (14, 14, 14), True),
    (512, 256, 32, 4, (14, 14, 14), True),     # config-1 shape: fewer units than lanes
    (4096, 1536, 12, 8, (12, 12, 12), True),   # 235B-A22B shape: two units per lane
    (1024, 512, 160, 6, (12, 12, 13), True),   # E > 136: one thread per router entry
    (2048, 768, 24, 8, (13, 13, 15), False),   # Q8_K down: multi-kernel path
    (1024, 512, 16, 4, (8, 8, 8), False),      # Q8_0 experts: multi-kernel path
]


@pytest.mark.parametrize("shape", FUSED_SHAPES, ids=lambda s: f"D{s[0]}-de{s[1]}-E{s[2]}-k{s[3]}-{s[4]}")
def test_fused_matches_multikernel(dev, orc, shape):
    """The persistent kernels and the multi-kernel path give identical bits
    over many consecutive tokens (the grid barrier, the stage ring and the
    double-buffered routing are reused token after token), the single-token
    kernel too over one-token launches, all equal the oracle, and the
    persistent kernel really runs as one launch for the whole token batch
    where it applies."""
    from tierlm_b200 import synth
    D, de, E, k, dts, fused_expected = shape
    rng = np.random.default_rng(D + de + E + k + sum(dts))
    experts = [synth.rand_expert(rng, D, de, dts) for _ in range(E)]
    ctx = build_ctx(experts, D, de, E, k, 0)
    T = 12
    x = rng.standard_normal((T, D)).astype(np.float32)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    lg[5] = 0.0                                   # all-tie routing row
    outs, launches = {}, {}
    for fused in ("static", False):
        ctx.set_fused(fused)
        xd, ld = torch.from_numpy(x).to(dev), torch.from_numpy(lg).to(dev)
        od = torch.zeros((T, D), device=dev)
        n0 = ctx.launches
        for rep in range(2):                      # twice: queue heads, epochs and counts reset between launches
            ctx.expert_ffn_many(0, xd, ld, od)
        try:
            ctx.check()
        except RuntimeError as ex:
            raise AssertionError(f"kernel mode {fused!r}: {ex}") from ex
        launches[fused] = (ctx.launches - n0) // 2
        outs[fused] = od.cpu().numpy()
    # a persistent kernel serves all T tokens in one launch
    assert (launches["static"] == 1) == fused_expected, launches
    assert same_bits(outs["static"], outs[False]).all()
    # one token per launch through the single-token kernel (where its
    # shared memory suffices), twice over: the same bits
    ctx.set_fused("single")
    o1 = torch.zeros((T, D), device=dev)
    for rep in range(2):
        for t in range(T):
            ctx.expert_ffn(0, xd[t], ld[t], o1[t])
    try:
        ctx.check()
    except RuntimeError as ex:
        raise AssertionError(f"kernel mode 'single': {ex}") from ex
    assert same_bits(o1.cpu().numpy(), outs[False]).all()
    outs[True] = outs["static"]
    orc.set_expf_mode(1)
    try:
        geom = dict(d_model=D, d_expert=de, n_experts=E, top_k=k, router=0)
        for t in (0, 5, T - 1):
            ref, _, _ = orc.expert_ffn(geom, experts, x[t], lg[t])
            bad = np.flatnonzero(~same_bits(outs[True][t], ref))
            assert bad.size == 0, (t, bad[:4], outs[True][t][bad[:4]], ref[bad[:4]])
    finally:
        orc.set_expf_mode(0)
    ctx.close()


BATCH_SHAPES = [
    # (D, de, E, k, dtypes, router, n_tok, batched kernels expected)
    (2048, 768, 32, 8, (12, 12, 14), 0, 64, True),    # config-2 layer shape, bs=64: 16 pairs per expert
    (2048, 768, 24, 8, (13, 13, 13), 0, 3, True),
    (512, 256, 16, 4, (14, 14, 14), 0, 5, True),      # nbd = 1: 32 down rows per warp
    (4096, 1536, 12, 8, (12, 12, 12), 0, 9, True),    # two blocks per lane, nbd = 6 (30 of 32 lanes)
    (1024, 512, 160, 6, (12, 12, 13), 0, 33, True),   # E > 128
    (1024, 512, 40, 4, (12, 12, 14), 1, 17, True),    # sigmoid router
    (1024, 512, 4, 4, (12, 12, 14), 0, 40, True),     # every expert > 16 tokens: several passes per tile
    (2048, 768, 8, 4, (12, 12, 14), 0, 100, True),    # prefill-like: 50 tokens per expert, wide passes
    (1024, 512, 6, 3, (13, 13, 13), 0, 64, True),     # wide passes, Q5_K
    (4096, 1536, 4, 2, (12, 12, 14), 0, 60, True),    # config-5 dims, 30 tokens per expert: wide passes, one CTA per SM
    (1024, 768, 8, 2, (13, 13, 15), 0, 4, False),     # Q8_K down: per-token fallback
]


def test_expert_ffn_batch_prefill_config2(dev):
    """Prefill at the config-2 layer shape with every expert present: 2048
    tokens through 128 experts (top-8, gate/up Q4_K, down Q6_K; ~128 tokens
    per expert, the tensor-core kernels' 32-token passes) in one batched
    call; sampled rows (ffn, ids, weights) equal the single-token path bit
    for bit."""
    from tierlm_b200 import synth
    D, de, E, k, T = 2048, 768, 128, 8, 2048
    rng = np.random.default_rng(2048128)
    experts = [synth.rand_expert(rng, D, de, (12, 12, 14)) for _ in range(E)]
    ctx = build_ctx(experts, D, de, E, k, 0)
    ctx.set_batch_kernels("mma")
    x = torch.from_numpy(rng.standard_normal((T, D)).astype(np.float32)).to(dev)
    lg = torch.from_numpy(rng.standard_normal((T, E)).astype(np.float32)).to(dev)
    out = torch.zeros((T, D), device=dev)
    ids = torch.zeros((T, k), dtype=torch.int32, device=dev)
    w = torch.zeros((T, k), device=dev)
    ctx.expert_ffn_batch(0, x, lg, out, ids, w)
    ctx.check()
    hits = torch.zeros(E, dtype=torch.int64, device=dev).scatter_add_(0, ids.flatten().long(),
                                                                     torch.ones(T * k, dtype=torch.int64, device=dev))
    assert int(hits.min()) >= 24                     # every expert runs the wide (prefill) passes
    out, ids, w = out.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()
    for t in list(range(0, T, 97)) + [T - 1]:
        one, i1, w1 = np.zeros(D, np.float32), np.zeros(k, np.int32), np.zeros(k, np.float32)
        ctx.expert_ffn(0, x[t].cpu().numpy(), lg[t].cpu().numpy(), one, i1, w1)
        assert np.array_equal(i1, ids[t]) and same_bits(w1, w[t]).all(), t
        bad = np.flatnonzero(~same_bits(one, out[t]))
        assert bad.size == 0, (t, bad[:4], out[t][bad[:4]], one[bad[:4]])
    ctx.close()


@pytest.mark.parametrize("shape", BATCH_SHAPES,
                         ids=lambda s: f"D{s[0]}-de{s[1]}-E{s[2]}-k{s[3]}-{s[4]}-r{s[5]}-n{s[6]}")
def test_expert_ffn_batch_matches_single(dev, orc, shape):
    """Batched decode (n tokens through one layer, each selected expert
    read once) gives the bits of n single-token calls: ffn rows, expert ids
    and weights; host and device buffers agree; the grouped kernels run as
    seven launches for the whole batch where they apply; one row equals the
    oracle."""
    from tierlm_b200 import synth
    D, de, E, k, dts, router, T, batched = shape
    rng = np.random.default_rng(7 * D + de + E + k + T)
    experts = [synth.rand_expert(rng, D, de, dts) for _ in range(E)]
    ctx = build_ctx(experts, D, de, E, k, router)
    x = rng.standard_normal((T, D)).astype(np.float32)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    lg[T // 2] = 0.0                              # all-tie routing row
    out = np.zeros((T, D), np.float32)
    ids = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    ctx.expert_ffn_batch(0, x, lg, out, ids, w)
    ctx.check()
    for t in range(T):
        one, i1, w1 = np.zeros(D, np.float32), np.zeros(k, np.int32), np.zeros(k, np.float32)
        ctx.expert_ffn(0, x[t], lg[t], one, i1, w1)
        assert np.array_equal(i1, ids[t]) and same_bits(w1, w[t]).all(), t
        bad = np.flatnonzero(~same_bits(one, out[t]))
        assert bad.size == 0, (t, bad[:4], out[t][bad[:4]], one[bad[:4]])
    xd, ld = torch.from_numpy(x).to(dev), torch.from_numpy(lg).to(dev)
    for tiled in ("warp", "tiled", "mma"):        # every batched kernel variant
        ctx.set_batch_kernels(tiled)
        od = torch.zeros((T, D), device=dev)
        n0 = ctx.launches
        ctx.expert_ffn_batch(0, xd, ld, od)
        ctx.check()
        assert ((ctx.launches - n0) == 7) == batched, ctx.launches - n0
        assert same_bits(od.cpu().numpy(), out).all(), tiled
    orc.set_expf_mode(1)
    try:
        geom = dict(d_model=D, d_expert=de, n_experts=E, top_k=k, router=router)
        ref, rid, _ = orc.expert_ffn(geom, experts, x[T - 1], lg[T - 1])
        assert np.array_equal(rid, ids[T - 1])
        assert same_bits(out[T - 1], ref).all()
    finally:
        orc.set_expf_mode(0)
    ctx.close()


@pytest.mark.parametrize("router", [1, 2])
def test_expert_ffn_batch_mask_bias(dev, router):
    """Batched decode with a pruning mask and (sigmoid router) a selection
    bias: the routing of every token excludes the masked experts and equals
    the single-token path, every mode of the batched kernels gives the same
    bits, and an empty batch is a no-op."""
    from tierlm_b200 import synth
    D, de, E, k, T = 1024, 512, 32, 4, 21
    rng = np.random.default_rng(60 + router)
    experts = [synth.rand_expert(rng, D, de, (12, 12, 14)) for _ in range(E)]
    ctx = build_ctx(experts, D, de, E, k, router)
    mask = np.zeros(E, np.uint8)
    mask[[0, 3, 7, 8, 30]] = 1
    bias = (0.5 * rng.standard_normal(E)).astype(np.float32) if router == 2 else None
    ctx.set_layer(0, mask=mask, router_bias=bias)
    x = rng.standard_normal((T, D)).astype(np.float32)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    lg[:, 3] = 10.0                                   # the largest logit belongs to a masked expert
    outs = []
    for mode in ("mma", "tiled", "warp"):
        ctx.set_batch_kernels(mode)
        out, ids, w = np.zeros((T, D), np.float32), np.zeros((T, k), np.int32), np.zeros((T, k), np.float32)
        ctx.expert_ffn_batch(0, x, lg, out, ids, w)
        assert not np.isin(ids, np.flatnonzero(mask)).any()
        outs.append((out, ids, w))
    for out, ids, w in outs[1:]:
        assert same_bits(out, outs[0][0]).all() and np.array_equal(ids, outs[0][1]) and same_bits(w, outs[0][2]).all()
    out, ids, w = outs[0]
    for t in (0, T // 2, T - 1):
        one, i1, w1 = np.zeros(D, np.float32), np.zeros(k, np.int32), np.zeros(k, np.float32)
        ctx.expert_ffn(0, x[t], lg[t], one, i1, w1)
        assert np.array_equal(i1, ids[t]) and same_bits(w1, w[t]).all() and same_bits(one, out[t]).all(), t
    n0 = ctx.launches
    ctx.expert_ffn_batch(0, x[:0], lg[:0], out[:0])   # empty batch
    assert ctx.launches == n0
    ctx.close()
