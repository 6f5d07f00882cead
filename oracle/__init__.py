"""CPU oracle loader - TEST INFRASTRUCTURE ONLY.

Loads oracle/liboracle.so (tlmo.c, the C restatement of the reference's
scalar algorithms) and, when it has been built, oracle/_ref/libtlmref.so
(the reference's own sources compiled in place by oracle/Makefile).
Only tests/, the package smoke check and bench.py's CPU-baseline leg may
import this module; the product path never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libtlmref.so"

_P, _I, _I64, _SZ, _F = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float


class Expert(C.Structure):
    _fields_ = [("base", _P), ("off", C.c_uint64 * 3), ("dt", C.c_int32 * 3)]


class Geom(C.Structure):
    _fields_ = [("d_model", C.c_int32), ("d_expert", C.c_int32), ("d_shared", C.c_int32),
                ("n_experts", C.c_int32), ("top_k", C.c_int32), ("router", C.c_int32),
                ("routed_scale", C.c_float), ("norm_eps", C.c_float)]


class Layer(C.Structure):
    _fields_ = [("ffn_norm", _P), ("router_dt", C.c_int32), ("router_w", _P), ("router_rb", _SZ),
                ("router_bias", _P), ("mask", _P), ("experts", C.POINTER(Expert)), ("has_shared", C.c_int32),
                ("sh_dt", C.c_int32 * 3), ("sh_w", _P * 3), ("shared_gate_inp", _P),
                ("has_dense", C.c_int32), ("d_ffn", C.c_int32), ("dn_dt", C.c_int32 * 3), ("dn_w", _P * 3)]


_SIGS = {
    "tlmo_f16_to_f32": (_F, [C.c_uint16]),
    "tlmo_f32_to_f16": (C.c_uint16, [_F]),
    "tlmo_row_bytes": (_SZ, [_I, _I64]),
    "tlmo_qact_bytes": (_SZ, [_I, _I64]),
    "tlmo_act_kind_for": (_I, [_I]),
    "tlmo_quantize_act": (None, [_I, _P, _I64, _P]),
    "tlmo_vec_dot": (_F, [_I, _P, _P, _I64]),
    "tlmo_dequantize_row": (_I, [_I, _P, _P, _I64]),
    "tlmo_matvec_rows": (None, [_I, _P, _SZ, _P, _P, _I64, _I64, _I64]),
    "tlmo_block_partials": (_I64, [_I, _P, _P, _I64, _P, _P]),
    "tlmo_set_expf_mode": (None, [_I]),
    "tlmo_get_expf_mode": (_I, []),
    "tlmo_expf": (_F, [_F]),
    "tlmo_expf_cr": (_F, [_F]),
    "tlmo_route": (None, [_I, _P, _P, _P, _I, _I, _F, _P, _P]),
    "tlmo_expert_ffn": (_I, [C.POINTER(Geom), C.POINTER(Expert), _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "tlmo_moe_layer": (_I, [C.POINTER(Geom), C.POINTER(Layer), _P, _P, _P]),
    "tlmo_moe_layer_ex": (_I, [C.POINTER(Geom), C.POINTER(Layer), _P, _P, _P, _P]),
    "tlmo_rmsnorm": (None, [_P, _P, _P, _I64, _F]),
    "tlmo_decode_attention": (None, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
}

_lib = None
_ref = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        srcs = [HERE / "tlmo.c", HERE / "tlmo.h"]
        if not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in srcs):
            build()
        L = C.CDLL(str(LIB))
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _lib = L
    return _lib


def ref() -> C.CDLL | None:
    """The reference's own library (oracle/_ref), or None when not built."""
    global _ref
    if _ref is None and REF_LIB.exists():
        R = C.CDLL(str(REF_LIB))
        R.tlm_quantize_act.argtypes = [_I, _P, _I64, _P]
        R.tlm_quantize_act.restype = None
        R.tlm_vec_dot.argtypes = [_I, _P, _P, _I64]
        R.tlm_vec_dot.restype = _F
        R.tlm_matvec_rows.argtypes = [_I, _P, _SZ, _P, _P, _I64, _I64, _I64, _P]
        R.tlm_matvec_rows.restype = None
        R.tlm_quantize_row.argtypes = [_I, _P, _P, _I64]
        R.tlm_quantize_row.restype = _I
        R.tlm_quant_tier.restype = C.c_char_p
        R.tlmref_open.argtypes = [_I]
        R.tlmref_threads.restype = _I
        R.tlmref_tier.restype = C.c_char_p
        R.tlmref_cpu_model.restype = C.c_char_p
        R.tlmref_physical_cores.restype = _I
        R.tlmref_expert_ffn.argtypes = [_I, _I, _I, _P, _P, _P, _P, _P, _P, _P]
        R.tlmref_expert_ffn.restype = _I
        R.tlmref_attn_heads.argtypes = [_P, _P, _P, _I, _I, _I, _I, _P]
        R.tlmref_attn_heads.restype = _I
        _ref = R
    return _ref


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


# ---- numpy conveniences --------------------------------------------------
def qact_bytes(kind: int, n: int) -> int:
    return lib().tlmo_qact_bytes(kind, n)


def row_bytes(dt: int, n: int) -> int:
    return lib().tlmo_row_bytes(dt, n)


def act_kind_for(dt: int) -> int:
    return lib().tlmo_act_kind_for(dt)


def quantize_act(kind: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(max(qact_bytes(kind, x.size), 4), np.uint8)
    lib().tlmo_quantize_act(kind, _p(x), x.size, _p(out))
    return out


def matvec_rows(dt: int, W: np.ndarray, rb: int, act: np.ndarray, n: int, r0: int, r1: int,
                w_offset: int = 0) -> np.ndarray:
    y = np.full(r1, np.nan, np.float32)
    lib().tlmo_matvec_rows(dt, W.ctypes.data + w_offset, rb, _p(act), _p(y), n, r0, r1)
    return y


def dequantize_row(dt: int, src: np.ndarray, n: int) -> np.ndarray:
    y = np.zeros(n, np.float32)
    assert lib().tlmo_dequantize_row(dt, _p(src), _p(y), n) == 0
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rmsnorm (src/lib/tlm_model.c:164-169): x * (1 / sqrtf(mean(x^2) + eps)) * w."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    lib().tlmo_rmsnorm(_p(out), _p(x), _p(w), x.size, eps)
    return out


def vec_dot(dt: int, wrow: np.ndarray, act: np.ndarray, n: int) -> float:
    return float(lib().tlmo_vec_dot(dt, _p(wrow), _p(act), n))


def block_partials(dt: int, wrow: np.ndarray, act: np.ndarray, n: int, w_offset: int = 0):
    nb = n // (256 if dt in (12, 13, 14, 15) else 32)
    isum = np.zeros(nb, np.int32)
    msum = np.zeros(nb, np.int32)
    rc = lib().tlmo_block_partials(dt, wrow.ctypes.data + w_offset, _p(act), n, _p(isum), _p(msum))
    assert rc == nb, rc
    return isum, msum


def set_expf_mode(mode: int) -> None:
    lib().tlmo_set_expf_mode(mode)


def decode_attention(q: np.ndarray, k_pages: np.ndarray, v_pages: np.ndarray, page_table: np.ndarray,
                     page: int, T: int) -> np.ndarray:
    """One decode position's attention over T cached positions (tlmo.c).
    q [H][hd]; k_pages / v_pages [n_pages][KV][page][hd]; page_table[i] = the
    page holding positions [i*page, (i+1)*page). Returns out [H][hd]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k_pages = np.ascontiguousarray(k_pages, dtype=np.float32)
    v_pages = np.ascontiguousarray(v_pages, dtype=np.float32)
    table = np.ascontiguousarray(page_table, dtype=np.int32)
    H, hd = q.shape
    KV = k_pages.shape[1]
    assert k_pages.shape[2] == page and k_pages.shape[3] == hd and v_pages.shape == k_pages.shape
    assert table.size * page >= T and (T == 0 or table[: (T + page - 1) // page].max() < k_pages.shape[0])
    out = np.zeros((H, hd), np.float32)
    lib().tlmo_decode_attention(_p(q), _p(k_pages), _p(v_pages), _p(table), page, T, H, KV, hd, _p(out))
    return out


def route(router: int, logits: np.ndarray, k: int, routed_scale: float = 1.0, mask=None, bias=None):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    ids = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    lib().tlmo_route(router, _p(logits), _p(mask), _p(bias), logits.size, k, routed_scale, _p(ids), _p(w))
    return ids, w


def expert_ffn(geom: dict, experts: list[tuple[np.ndarray, tuple, tuple]], x: np.ndarray, logits: np.ndarray,
               mask=None, bias=None, want_intermediates: bool = False):
    """experts: per expert (payload uint8, item_off[3], dt[3]). Returns
    (ffn, ids, w) or (ffn, ids, w, eo, h) with intermediates."""
    g = Geom(geom["d_model"], geom["d_expert"], geom.get("d_shared", 0), geom["n_experts"], geom["top_k"],
             geom.get("router", 0), geom.get("routed_scale", 1.0), geom.get("norm_eps", 1e-6))
    arr = (Expert * len(experts))()
    for i, (payload, off, dt) in enumerate(experts):
        arr[i].base = payload.ctypes.data
        arr[i].off[:] = list(off)
        arr[i].dt[:] = list(dt)
    x = np.ascontiguousarray(x, np.float32)
    logits = np.ascontiguousarray(logits, np.float32)
    D, de, k = g.d_model, g.d_expert, g.top_k
    ffn = np.zeros(D, np.float32)
    ids = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    eo = np.zeros((k, D), np.float32) if want_intermediates else None
    hb = np.zeros((k, de), np.float32) if want_intermediates else None
    rc = lib().tlmo_expert_ffn(C.byref(g), arr, _p(mask), _p(bias), _p(x), _p(logits), _p(ffn), _p(ids), _p(w),
                               _p(eo), _p(hb))
    assert rc == 0
    return (ffn, ids, w, eo, hb) if want_intermediates else (ffn, ids, w)


def moe_layer(geom: dict, layer: dict, experts, h: np.ndarray, want_onorm: bool = False):
    """The whole moe() block on a copy of h; returns (h_out, ids, w), plus
    the route hook's output norms with want_onorm. layer["dense"] = (dts,
    mats, d_ffn) makes it a dense-FFN layer."""
    g = Geom(geom["d_model"], geom["d_expert"], geom.get("d_shared", 0), geom["n_experts"], geom["top_k"],
             geom.get("router", 0), geom.get("routed_scale", 1.0), geom.get("norm_eps", 1e-6))
    arr = (Expert * max(len(experts), 1))()
    for i, (payload, off, dt) in enumerate(experts):
        arr[i].base = payload.ctypes.data
        arr[i].off[:] = list(off)
        arr[i].dt[:] = list(dt)
    L = Layer()
    keep = []
    for name in ("ffn_norm", "router_w", "router_bias", "mask", "shared_gate_inp"):
        v = layer.get(name)
        if v is not None:
            v = np.ascontiguousarray(v)
            keep.append(v)
            setattr(L, name, v.ctypes.data)
    L.router_dt = layer.get("router_dt", 0)
    L.router_rb = layer.get("router_rb", 0)
    L.experts = arr
    if layer.get("shared") is not None:
        dts, mats = layer["shared"]
        L.has_shared = 1
        L.sh_dt[:] = list(dts)
        for m in range(3):
            keep.append(mats[m])
            L.sh_w[m] = mats[m].ctypes.data
    if layer.get("dense") is not None:
        dts, mats, d_ffn = layer["dense"]
        L.has_dense = 1
        L.d_ffn = d_ffn
        L.dn_dt[:] = list(dts)
        for m in range(3):
            keep.append(mats[m])
            L.dn_w[m] = mats[m].ctypes.data
    h = np.array(h, np.float32, copy=True)
    k = max(g.top_k, 1)
    ids = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    onorm = np.zeros(k, np.float32)
    rc = lib().tlmo_moe_layer_ex(C.byref(g), C.byref(L), _p(h), _p(ids), _p(w), _p(onorm) if want_onorm else None)
    assert rc == 0
    return (h, ids, w, onorm) if want_onorm else (h, ids, w)
