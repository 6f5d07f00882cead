"""Decode attention over a paged KV cache (attn_heads, src/lib/tlm_model.c:683-719).

CPU: the oracle's paged restatement against golden vectors written by the
reference's own attn_heads (tests/golden/make_golden.py attention).
GPU: TLMG_ATTN_EXACT bit-identical to the oracle (correctly rounded expf),
TLMG_ATTN_SPLIT within float rounding, the bf16 page append, and the
argument checks.
"""
from __future__ import annotations

import numpy as np
import pytest
from conftest import cases, same_bits


def to_pages(k, v, page, seed=0, spare=3):
    """Contiguous [KV][T][hd] -> shuffled pages [n_pages][KV][page][hd] + table."""
    KV, T, hd = k.shape
    n_used = -(-T // page)
    n_pages = n_used + spare
    rng = np.random.default_rng(seed)
    table = rng.permutation(n_pages)[:n_used].astype(np.int32)
    kp = np.full((n_pages, KV, page, hd), np.nan, np.float32)   # unused rows poison a wrong read
    vp = np.full((n_pages, KV, page, hd), np.nan, np.float32)
    for j in range(n_used):
        rows = slice(j * page, min(T, (j + 1) * page))
        n = rows.stop - rows.start
        kp[table[j], :, :n] = k[:, rows]
        vp[table[j], :, :n] = v[:, rows]
    return kp, vp, table


def attn_case(seed, T, H, KV, hd):
    from tests.golden.make_golden import attn_case as gen
    return gen(seed, T, H, KV, hd)


@pytest.mark.parametrize("page", [1, 16, 64])
def test_attention_oracle_golden(orc, page):
    """The oracle (libm expf, paged, shuffled pages) reproduces the
    reference's attn_heads bit for bit."""
    for c in cases("attention.npz"):
        seed, T, H, KV, hd = (int(c[x]) for x in ("seed", "T", "H", "KV", "hd"))
        q, k, v = attn_case(seed, T, H, KV, hd)
        kp, vp, table = to_pages(k, v, page, seed)
        out = orc.decode_attention(q, kp, vp, table, page, T)
        assert same_bits(out, c["out"]).all(), (seed, T, page, np.abs(out - c["out"]).max())


def test_attention_oracle_cr_close(orc):
    """With the correctly rounded expf of the CUDA tier the oracle stays
    within float rounding of the reference (libm expf misrounds rarely)."""
    orc.set_expf_mode(1)
    try:
        for c in cases("attention.npz"):
            seed, T, H, KV, hd = (int(c[x]) for x in ("seed", "T", "H", "KV", "hd"))
            q, k, v = attn_case(seed, T, H, KV, hd)
            kp, vp, table = to_pages(k, v, 16, seed)
            out = orc.decode_attention(q, kp, vp, table, 16, T)
            np.testing.assert_allclose(out, c["out"], rtol=1e-5, atol=1e-6)
    finally:
        orc.set_expf_mode(0)


def test_attention_reference_pins_fixture(orc):
    """When the reference library is built here, it still writes the fixture."""
    R = orc.ref()
    if R is None:
        pytest.skip("reference library (oracle/_ref) not built")
    for c in cases("attention.npz"):
        seed, T, H, KV, hd = (int(c[x]) for x in ("seed", "T", "H", "KV", "hd"))
        q, k, v = attn_case(seed, T, H, KV, hd)
        out = np.zeros((H, hd), np.float32)
        assert R.tlmref_attn_heads(q.ctypes.data, k.ctypes.data, v.ctypes.data, T, H, KV, hd, out.ctypes.data) == 0
        assert same_bits(out, c["out"]).all()


def bf16_round(a: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 (round to nearest even) -> float32, finite inputs."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


# ---- GPU ---------------------------------------------------------------------
GPU_CASES = [   # (seed, T, H, KV, hd, page)
    (21, 1, 8, 2, 64, 16), (22, 16, 8, 2, 64, 16), (23, 17, 32, 4, 128, 16), (24, 300, 32, 4, 128, 64),
    (25, 768, 32, 4, 128, 16), (26, 1025, 16, 16, 64, 32), (27, 200, 32, 2, 256, 8), (28, 130, 4, 4, 128, 1),
]


def _gpu_inputs(seed, T, H, KV, hd, page, dtype):
    import torch
    q, k, v = attn_case(seed, T, H, KV, hd)
    kp, vp, table = to_pages(k, v, page, seed)
    dev = torch.device("cuda:0")
    tq = torch.from_numpy(q).to(dev)
    tk = torch.from_numpy(np.nan_to_num(kp, nan=0.0)).to(dev).to(dtype)
    tv = torch.from_numpy(np.nan_to_num(vp, nan=0.0)).to(dev).to(dtype)
    tt = torch.from_numpy(table).to(dev)
    return q, tq, tk, tv, tt, table


@pytest.mark.gpu
@pytest.mark.parametrize("case", GPU_CASES)
def test_attention_exact_bits(orc, case):
    """EXACT on f32 pages: the same bits as the oracle's restatement of
    attn_heads (correctly rounded expf)."""
    import torch
    from tierlm_b200 import attention as A
    seed, T, H, KV, hd, page = case
    q, tq, tk, tv, tt, table = _gpu_inputs(seed, T, H, KV, hd, page, torch.float32)
    out = A.decode_attention(tq, tk, tv, tt, T, A.EXACT).cpu().numpy()
    orc.set_expf_mode(1)
    try:
        ref = orc.decode_attention(q, tk.cpu().numpy(), tv.cpu().numpy(), table, page, T)
    finally:
        orc.set_expf_mode(0)
    assert same_bits(out, ref).all(), np.abs(out - ref).max()


@pytest.mark.gpu
def test_attention_exact_long_context(orc):
    """T above the shared-memory bound of the softmax (p kept in the work
    buffer): still bit-identical."""
    import torch
    from tierlm_b200 import attention as A
    seed, T, H, KV, hd, page = 31, 20000, 8, 2, 128, 256
    q, tq, tk, tv, tt, table = _gpu_inputs(seed, T, H, KV, hd, page, torch.float32)
    out = A.decode_attention(tq, tk, tv, tt, T, A.EXACT).cpu().numpy()
    orc.set_expf_mode(1)
    try:
        ref = orc.decode_attention(q, tk.cpu().numpy(), tv.cpu().numpy(), table, page, T)
    finally:
        orc.set_expf_mode(0)
    assert same_bits(out, ref).all()


@pytest.mark.gpu
def test_attention_exact_matches_reference_fixture():
    """EXACT against the reference's own outputs: equal within the rare
    1-ulp misrounding of the reference's libm expf."""
    import torch
    from tierlm_b200 import attention as A
    for c in cases("attention.npz"):
        seed, T, H, KV, hd = (int(c[x]) for x in ("seed", "T", "H", "KV", "hd"))
        q, tq, tk, tv, tt, _ = _gpu_inputs(seed, T, H, KV, hd, 16, torch.float32)
        out = A.decode_attention(tq, tk, tv, tt, T, A.EXACT).cpu().numpy()
        np.testing.assert_allclose(out, c["out"], rtol=1e-5, atol=1e-6)


def rel_l2(a, b) -> float:
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
@pytest.mark.parametrize("case", GPU_CASES + [(41, 9000, 32, 4, 128, 64), (42, 5000, 16, 2, 64, 128),
                                   (43, 3000, 8, 1, 256, 32)])
def test_attention_split(orc, case, dtype_name):
    """SPLIT (flash-decoding) against the oracle on the same page contents
    (bf16 pages widened exactly to f32). f32 pages (CUDA cores, f32 FMA):
    relative L2 error below 2e-6, every element within 1e-5 relative +
    1e-6 absolute. bf16 pages (tensor cores; q and p carried as bf16
    high + remainder, 16 significant bits): relative L2 below 2e-5, every
    element within 1e-4 relative + 1e-5 absolute."""
    import torch
    from tierlm_b200 import attention as A
    dtype = getattr(torch, dtype_name)
    seed, T, H, KV, hd, page = case
    q, tq, tk, tv, tt, table = _gpu_inputs(seed, T, H, KV, hd, page, dtype)
    out = A.decode_attention(tq, tk, tv, tt, T, A.SPLIT).cpu().numpy()
    ref = orc.decode_attention(q, tk.float().cpu().numpy(), tv.float().cpu().numpy(), table, page, T)
    tol = (2e-6, 1e-5, 1e-6) if dtype == torch.float32 else (2e-5, 1e-4, 1e-5)
    assert rel_l2(out, ref) < tol[0], rel_l2(out, ref)
    np.testing.assert_allclose(out, ref, rtol=tol[1], atol=tol[2])


@pytest.mark.gpu
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_kv_write_then_attend(orc, dtype_name):
    """Appending positions one by one through tlmg_kv_write builds the same
    pages as the host (bf16: round to nearest even), and attention over
    them matches the oracle."""
    import torch
    from tierlm_b200 import attention as A
    dtype = getattr(torch, dtype_name)
    T, H, KV, hd, page = 70, 8, 2, 128, 16
    q, k, v = attn_case(51, T, H, KV, hd)
    n_pages = 8
    table = np.array([5, 1, 7, 0, 3], np.int32)
    kv = A.PagedKV(n_pages, KV, page, hd, dtype=dtype)
    dev = torch.device("cuda:0")
    for t in range(T):
        kv.write(torch.from_numpy(np.ascontiguousarray(k[:, t])).to(dev),
                 torch.from_numpy(np.ascontiguousarray(v[:, t])).to(dev), int(table[t // page]), t)
    kp = kv.k.float().cpu().numpy()
    vp = kv.v.float().cpu().numpy()
    rnd = (lambda a: a) if dtype == torch.float32 else bf16_round
    for t in range(T):
        pg, r = table[t // page], t % page
        assert same_bits(kp[pg, :, r], rnd(k[:, t])).all()
        assert same_bits(vp[pg, :, r], rnd(v[:, t])).all()
    tt = torch.from_numpy(table).to(dev)
    out = kv.attend(torch.from_numpy(q).to(dev), tt, T, A.EXACT).cpu().numpy()
    orc.set_expf_mode(1)
    try:
        ref = orc.decode_attention(q, kp, vp, table, page, T)
    finally:
        orc.set_expf_mode(0)
    assert same_bits(out, ref).all()


@pytest.mark.gpu
def test_attention_bad_page_and_args():
    """An out-of-range page entry is not dereferenced (NaN result); bad
    shapes and short scratch are rejected with the reference's codes."""
    import torch
    from tierlm_b200 import TlmError
    from tierlm_b200 import attention as A
    dev = torch.device("cuda:0")
    T, H, KV, hd, page = 40, 8, 2, 64, 16
    q, tq, tk, tv, tt, table = _gpu_inputs(61, T, H, KV, hd, page, torch.float32)
    bad = tt.clone()
    bad[1] = 1 << 20
    for mode in (A.EXACT, A.SPLIT):
        out = A.decode_attention(tq, tk, tv, bad, T, mode).cpu().numpy()
        assert np.isnan(out).all()
        good = A.decode_attention(tq, tk, tv, tt, T, mode).cpu().numpy()
        assert np.isfinite(good).all()
    with pytest.raises(TlmError) as e:
        A.decode_attention(tq[:, :48].contiguous(), tk[..., :48].contiguous(), tv[..., :48].contiguous(), tt, T)
    assert e.value.code == -3
    from tierlm_b200._lib import load
    import ctypes as C
    L = load()
    w = torch.empty(16, dtype=torch.uint8, device=dev)
    out = torch.empty((H, hd), dtype=torch.float32, device=dev)
    rc = L.tlmg_decode_attention(A.EXACT, 0, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tk.shape[0], tt.data_ptr(),
                                 page, T, H, KV, hd, w.data_ptr(), 16, out.data_ptr(), C.c_void_p(1))
    assert rc == -5
    rc = L.tlmg_decode_attention(A.EXACT, 0, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tk.shape[0], tt.data_ptr(),
                                 page, 0, H, KV, hd, w.data_ptr(), 16, out.data_ptr(), C.c_void_p(1))
    assert rc == -3
    torch.cuda.synchronize()
