"""The whole decoder step on the GPU (tlmg_decode_step) against the same
step composed from the CPU oracle's restatements of the reference's parts
(tlm_model_step, src/lib/tlm_model.c:1058-1103): embedding row
(tlm_dequantize_row), per layer attention() (:730-763: rmsnorm, q/k/v
matvecs, qk-norm, rope(), the K/V write, attn_heads, o-proj, h += o) and
moe(), then the final rmsnorm and lm_head. Both sides use the correctly
rounded expf, so every logit of every position must be bit-identical, with
the step replayed as a captured graph (from the second position on) and
with every step eager.

The model is tiny and mixes dtypes on purpose: layer 0 has q/k/v of one
dtype (one fused matvec on the GPU) and qk-norm, layer 1 has three
different q/k/v dtypes and none; the embedding, lm_head and o-projections
use other formats again."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch
from conftest import same_bits

pytestmark = pytest.mark.gpu

EPS, THETA = 1e-6, 10000.0

# small: D 512, rows whose lengths are not 16-byte multiples (the kernels
# with a separate norm / quantisation kernel); wide: D 2048 with Q6_K q|k|v,
# Q4_K o and Q6_K lm_head rows of 16-byte multiples (the matvecs that form
# their own activations) and an f32 router on the normalised residual
SHAPES = {
    "small": dict(D=512, DE=256, E=8, K=2, H=4, KVH=2, HD=64, V=300,
                  LAYER_DTS=[(14, 14, 14, 8), (12, 8, 14, 13)], EMB_DT=14, HEAD_DT=8),
    "wide": dict(D=2048, DE=768, E=8, K=2, H=8, KVH=2, HD=128, V=512,
                 LAYER_DTS=[(14, 14, 14, 12), (12, 8, 14, 13)], EMB_DT=12, HEAD_DT=14),
}


def _model(seed, shape="small"):
    from tierlm_b200 import synth
    c = SHAPES[shape]
    D, DE, E, H, KVH, HD = c["D"], c["DE"], c["E"], c["H"], c["KVH"], c["HD"]
    rng = np.random.default_rng(seed)

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    layers = []
    for l_, dts in enumerate(c["LAYER_DTS"]):
        mats = [synth.rand_rows(dts[0], H * HD, D, rng), synth.rand_rows(dts[1], KVH * HD, D, rng),
                synth.rand_rows(dts[2], KVH * HD, D, rng), synth.rand_rows(dts[3], D, H * HD, rng)]
        layers.append(dict(dts=dts, mats=mats, attn_norm=norm(D), q_norm=norm(HD) if l_ == 0 else None,
                           k_norm=norm(HD) if l_ == 0 else None, ffn_norm=norm(D),
                           router_w=(rng.standard_normal((E, D)) / np.sqrt(D)).astype(np.float32),
                           experts=[synth.rand_expert(rng, D, DE, (12, 12, 14)) for _ in range(E)]))
    inv = np.array([np.float32(THETA ** (-2.0 * j / HD)) for j in range(HD // 2)], np.float32)
    return dict(cfg=c, layers=layers, emb=synth.rand_rows(c["EMB_DT"], c["V"], D, rng),
                head=synth.rand_rows(c["HEAD_DT"], c["V"], D, rng), out_norm=norm(D), inv=inv)


def _mv(orc, dt, W, x, rows):
    kind = orc.act_kind_for(dt)
    act = x.view(np.uint8) if kind == 0 else orc.quantize_act(kind, x)
    return orc.matvec_rows(dt, W, W.shape[1], act, x.size, 0, rows)


def _ref_steps(orc, m, tokens):
    """Logits of every position, the reference's step composed on the oracle."""
    c = m["cfg"]
    D, DE, E, K, H, KVH, HD, V = (c[x] for x in ("D", "DE", "E", "K", "H", "KVH", "HD", "V"))
    L = len(m["layers"])
    page = 16
    kp = np.zeros((L, KVH, page, HD), np.float32)
    vp = np.zeros((L, KVH, page, HD), np.float32)
    geom = dict(d_model=D, d_expert=DE, n_experts=E, top_k=K, router=0, norm_eps=EPS)
    out = []
    for pos, tok in enumerate(tokens):
        h = orc.dequantize_row(c["EMB_DT"], m["emb"][tok], D)
        cs = np.array([np.float32(math.cos(pos * float(f))) for f in m["inv"]], np.float32)
        sn = np.array([np.float32(math.sin(pos * float(f))) for f in m["inv"]], np.float32)
        for l_, A in enumerate(m["layers"]):
            xb = orc.rmsnorm(h, A["attn_norm"], EPS)
            q = _mv(orc, A["dts"][0], A["mats"][0], xb, H * HD).reshape(H, HD)
            k = _mv(orc, A["dts"][1], A["mats"][1], xb, KVH * HD).reshape(KVH, HD)
            v = _mv(orc, A["dts"][2], A["mats"][2], xb, KVH * HD).reshape(KVH, HD)
            if A["q_norm"] is not None:
                q = np.stack([orc.rmsnorm(q[i], A["q_norm"], EPS) for i in range(H)])
            if A["k_norm"] is not None:
                k = np.stack([orc.rmsnorm(k[i], A["k_norm"], EPS) for i in range(KVH)])

            def rope(x):
                a, b = x[:, : HD // 2], x[:, HD // 2:]
                return np.concatenate([a * cs - b * sn, b * cs + a * sn], axis=1).astype(np.float32)

            q, k = rope(q), rope(k)
            kp[l_, :, pos], vp[l_, :, pos] = k, v
            att = orc.decode_attention(q, kp[l_:l_ + 1], vp[l_:l_ + 1], np.zeros(1, np.int32), page, pos + 1)
            h = (h + _mv(orc, A["dts"][3], A["mats"][3], att.reshape(-1), D)).astype(np.float32)
            layer = dict(ffn_norm=A["ffn_norm"], router_dt=0, router_w=A["router_w"], router_rb=4 * D)
            h = orc.moe_layer(geom, layer, A["experts"], h)[0]
        xb = orc.rmsnorm(h, m["out_norm"], EPS)
        out.append(_mv(orc, c["HEAD_DT"], m["head"], xb, V))
    return np.stack(out)


def _gpu_ctx(m):
    from tierlm_b200.moe import MoeContext
    c = m["cfg"]
    D, DE, E, K, H, KVH, HD, V = (c[x] for x in ("D", "DE", "E", "K", "H", "KVH", "HD", "V"))
    L = len(m["layers"])
    ctx = MoeContext(L, D, DE, E, K, router=0)
    for l_, A in enumerate(m["layers"]):
        for e, (payload, off, dts) in enumerate(A["experts"]):
            ctx.set_expert(l_, e, dts, payload, off)
        ctx.set_layer(l_, ffn_norm=A["ffn_norm"], router_dt=0, router_w=A["router_w"], router_row_bytes=4 * D)
    ctx.step_open(H, KVH, HD, V, m["inv"], 1.0, max_ctx=16, kv_dtype=0, attn_mode=0)
    for l_, A in enumerate(m["layers"]):
        ctx.set_attention(l_, A["attn_norm"], A["dts"], *A["mats"], q_norm=A["q_norm"], k_norm=A["k_norm"])
    ctx.set_embedding(c["EMB_DT"], m["emb"])
    ctx.set_output(m["out_norm"], c["HEAD_DT"], m["head"])
    return ctx


@pytest.mark.parametrize("shape", list(SHAPES))
def test_decode_step_matches_composed_oracle(orc, shape):
    from tierlm_b200 import _lib
    _lib.check(_lib.load().tlmg_init(0))
    m = _model(5, shape)
    V = m["cfg"]["V"]
    tokens = [7, 299, 0, 123, 7, 42]
    orc.set_expf_mode(1)
    try:
        ref = _ref_steps(orc, m, tokens)
    finally:
        orc.set_expf_mode(0)
    ctx = _gpu_ctx(m)
    got = np.zeros((len(tokens), V), np.float32)
    for pos, tok in enumerate(tokens):
        ctx.decode_step(tok, pos, got[pos])
    # device logits (asynchronous) and a step without logits give the same state
    dl = torch.empty(V, device="cuda:0")
    for pos, tok in enumerate(tokens):
        ctx.decode_step(tok, pos, dl if pos == len(tokens) - 1 else None)
    ctx.check()
    info = ctx.step_info()
    assert not info["graphs_off"] and info["replays"] == 2 * len(tokens) - 1 and info["captures"] == 2, info
    ctx.close()
    # every step eager (no graph replay): the same bits
    ctx = _gpu_ctx(m)
    ctx.step_graphs(False)
    eager = np.zeros_like(got)
    for pos, tok in enumerate(tokens):
        ctx.decode_step(tok, pos, eager[pos])
    ctx.close()
    assert same_bits(eager, got).all()
    assert np.isfinite(ref).all()
    for pos in range(len(tokens)):
        bad = np.flatnonzero(~same_bits(got[pos], ref[pos]))
        assert bad.size == 0, (pos, bad[:5], got[pos][bad[:5]], ref[pos][bad[:5]])
    assert same_bits(dl.cpu().numpy(), ref[-1]).all()


def test_decode_step_errors(orc):
    """Out-of-range token / position and missing weights are errors."""
    from tierlm_b200 import _lib
    from tierlm_b200.moe import MoeContext
    _lib.check(_lib.load().tlmg_init(0))
    m = _model(6)
    c = m["cfg"]
    V = c["V"]
    ctx = _gpu_ctx(m)
    lg = np.zeros(V, np.float32)
    for tok, pos, code in ((V, 0, _lib.TLMG_EINVAL), (-1, 0, _lib.TLMG_EINVAL), (0, 16, _lib.TLMG_ERANGE)):
        with pytest.raises(_lib.TlmError) as ei:
            ctx.decode_step(tok, pos, lg)
        assert ei.value.code == code
    ctx.close()
    bare = MoeContext(len(m["layers"]), c["D"], c["DE"], c["E"], c["K"], router=0)
    with pytest.raises(_lib.TlmError):
        bare.decode_step(0, 0, lg)
    bare.step_open(c["H"], c["KVH"], c["HD"], V, m["inv"], 1.0, max_ctx=16)
    with pytest.raises(_lib.TlmError) as ei:
        bare.decode_step(0, 0, lg)
    assert ei.value.code == _lib.TLMG_ENOTFOUND
    bare.close()


def test_decode_step_stats(orc):
    """tlmg_step_stats counts every step; steps run while profiling add
    their attention / MoE / other device time (each phase positive, their
    sum the step's), give the same logits as graph replay, and reset zeroes
    the counters."""
    from tierlm_b200 import _lib
    _lib.check(_lib.load().tlmg_init(0))
    m = _model(8)
    V = m["cfg"]["V"]
    ctx = _gpu_ctx(m)
    plain = np.zeros((3, V), np.float32)
    for pos, tok in enumerate((3, 1, 4)):
        ctx.decode_step(tok, pos, plain[pos])
    s0 = ctx.step_stats()
    assert s0["tokens"] == 3 and s0["attn_ns"] == 0 and s0["moe_ns"] == 0
    ctx.profile(True)
    prof = np.zeros((3, V), np.float32)
    for pos, tok in enumerate((3, 1, 4)):
        ctx.decode_step(tok, pos, prof[pos])
    ctx.profile(False)
    s1 = ctx.step_stats(reset=True)
    assert s1["tokens"] == 6 and s1["attn_ns"] > 0 and s1["moe_ns"] > 0 and s1["other_ns"] > 0, s1
    assert s1["expert_wait_ns"] == 0
    assert ctx.step_stats() == dict(tokens=0, attn_ns=0, moe_ns=0, expert_wait_ns=0, other_ns=0)
    assert same_bits(prof, plain).all()
    ctx.close()
