"""ctypes binding of libtlmg.so (the C ABI declared in include/tlmg.h).

The library is the product: there is no CPU fallback. load() raises when
the shared object is missing or cannot be loaded, and every wrapper in this
package goes through it.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtlmg.so"

# error codes (include/tlmg.h; same numbering as the reference's TLM_E*)
TLMG_OK, TLMG_EIO, TLMG_ENOMEM, TLMG_EINVAL, TLMG_EFORMAT = 0, -1, -2, -3, -4
TLMG_ERANGE, TLMG_ENOTFOUND, TLMG_EUNSUP, TLMG_EBUSY = -5, -6, -7, -8

# dtype codes (= tlm_dtype)
F32, F16, BF16, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, MXFP4 = 0, 1, 2, 8, 12, 13, 14, 15, 39
DTYPE_NAMES = {F32: "f32", F16: "f16", BF16: "bf16", Q8_0: "q8_0", Q4_K: "q4_k", Q5_K: "q5_k",
               Q6_K: "q6_k", Q8_K: "q8_k", MXFP4: "mxfp4"}


class TlmError(RuntimeError):
    """A negative return code from libtlmg, with its thread-local message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libtlmg error {code}: {msg}")
        self.code = code


class ExpertSlot(C.Structure):
    """tlmg_expert_slot: device pointers of one expert's gate, up, down."""
    _fields_ = [("m", C.c_void_p * 3), ("dt", C.c_int32 * 3), ("pad", C.c_int32)]


class PacketInfo(C.Structure):
    """tlmg_packet_info: a parsed tlm packet header (include/tlmg.h)."""
    _fields_ = [("type", C.c_uint32), ("version", C.c_uint32), ("layer", C.c_uint32), ("n_items", C.c_uint32),
                ("id", C.c_uint32), ("dtype", C.c_uint32), ("layout", C.c_uint32), ("crc32c", C.c_uint32),
                ("payload_len", C.c_uint64), ("total_len", C.c_uint64), ("item_off", C.c_uint64 * 3),
                ("item_dt", C.c_int32 * 3), ("mixed", C.c_int32)]


class Geom(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("d_model", C.c_int32), ("d_expert", C.c_int32),
                ("d_shared", C.c_int32), ("n_experts", C.c_int32), ("top_k", C.c_int32),
                ("router", C.c_int32), ("routed_scale", C.c_float), ("norm_eps", C.c_float)]


_lib = None

_P, _I, _I64, _SZ, _F = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float
_SIGS = {
    "tlmg_errmsg": (C.c_char_p, []),
    "tlmg_tier": (C.c_char_p, []),
    "tlmg_init": (_I, [_I]),
    "tlmg_sync": (_I, [_P]),
    "tlmg_dtype_block": (_I, [_I]),
    "tlmg_dtype_block_bytes": (_SZ, [_I]),
    "tlmg_row_bytes": (_SZ, [_I, _I64]),
    "tlmg_qact_bytes": (_SZ, [_I, _I64]),
    "tlmg_act_kind_for": (_I, [_I]),
    "tlmg_quantize_act": (_I, [_I, _P, _I64, _P, _P]),
    "tlmg_matvec_rows": (_I, [_I, _P, _SZ, _P, _P, _I64, _I64, _I64, _P]),
    "tlmg_dequantize_rows": (_I, [_I, _P, _SZ, _P, _I64, _I64, _P]),
    "tlmg_block_partials": (_I, [_I, _P, _SZ, _P, _I64, _I64, _P, _P, _P]),
    "tlmg_route": (_I, [_I, _P, _P, _P, _I, _I, _F, _P, _P, _P]),
    "tlmg_attention_work_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "tlmg_decode_attention": (_I, [_I, _I, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P, _SZ, _P, _P]),
    "tlmg_kv_write": (_I, [_I, _P, _P, _P, _P, _I, C.c_int32, _I, _I, _I, _I, _P]),
    "tlmg_qmv_host": (None, [_I, _P, _SZ, _P, _P, _I64, _I64]),
    "tlmg_qdot_host": (_F, [_I, _P, _P, _I64, _P]),
    "tlmg_open": (_I, [C.POINTER(Geom), _I, C.POINTER(_P)]),
    "tlmg_close": (None, [_P]),
    "tlmg_set_expert": (_I, [_P, _I, _I, _P, _P, _SZ, _P]),
    "tlmg_set_layer": (_I, [_P, _I, _P, _I, _P, _SZ, _P, _P]),
    "tlmg_set_shared": (_I, [_P, _I, _P, _P, _P, _P, _P]),
    "tlmg_expert_ffn": (_I, [_P, _I, _P, _P, _P, _P, _P]),
    "tlmg_expert_ffn_many": (_I, [_P, _I, _I, _P, _P, _P]),
    "tlmg_expert_ffn_batch": (_I, [_P, _I, _I, _P, _P, _P, _P, _P]),
    "tlmg_ep_record_bytes": (_SZ, [_P]),
    "tlmg_ep_dispatch": (_I, [_P, _I, _I, _P, _P, _I, _P, _P, _P, _P]),
    "tlmg_ep_experts": (_I, [_P, _I, _I, _I, _I64, _P, _P]),
    "tlmg_ep_combine": (_I, [_P, _I, _P, _P, _P, _P]),
    "tlmg_step_open": (_I, [_P, _I, _I, _I, _I, _P, C.c_float, _I, _I, _I]),
    "tlmg_set_attention": (_I, [_P, _I, _P, _P, _P, _P, _P, _P]),
    "tlmg_set_embedding": (_I, [_P, _I, _P, _SZ]),
    "tlmg_set_output": (_I, [_P, _P, _I, _P, _SZ]),
    "tlmg_decode_step": (_I, [_P, _I, _I, _P]),
    "tlmg_step_graphs": (_I, [_P, _I]),
    "tlmg_step_info": (_I, [_P, _P]),
    "tlmg_step_stats": (_I, [_P, _P, _I]),
    "tlmg_ep_open": (_I, [_P, _I, _I, _I]),
    "tlmg_ep_handle_bytes": (_SZ, []),
    "tlmg_ep_handle": (_I, [_P, _P]),
    "tlmg_ep_connect": (_I, [_P, _P]),
    "tlmg_ep_layer": (_I, [_P, _I, _I, _P, _P, _P, _P, _P]),
    "tlmg_ep_close": (_I, [_P]),
    "tlmg_moe_layer": (_I, [_P, _I, _P, _P, _P]),
    "tlmg_moe_layer_ex": (_I, [_P, _I, _P, _P, _P, _P]),
    "tlmg_set_dense_ffn": (_I, [_P, _I, _I, _P, _P, _P, _P]),
    "tlmg_set_stream": (_I, [_P, _P]),
    "tlmg_set_fused": (_I, [_P, _I]),
    "tlmg_set_batch_kernels": (_I, [_P, _I]),
    "tlmg_cache_enable": (_I, [_P, _I, _SZ]),
    "tlmg_set_expert_host": (_I, [_P, _I, _I, _P, _P, _SZ, _P]),
    "tlmg_cache_prefetch": (_I, [_P, _I, _P, _I]),
    "tlmg_crc32c": (C.c_uint32, [C.c_uint32, _P, _SZ]),
    "tlmg_packet_parse": (_I, [_P, _SZ, _I, _P]),
    "tlmg_set_expert_packet": (_I, [_P, _I, _I, _P, _SZ, _I]),
    "tlmg_cache_stats": (_I, [_P, _P]),
    "tlmg_cache_tick": (_I, [_P]),
    "tlmg_cache_lookahead": (_I, [_P, _I, _I]),
    "tlmg_store_open": (_I, [_I, _I, _I, C.POINTER(_P)]),
    "tlmg_store_close": (None, [_P]),
    "tlmg_store_acquire": (_I, [_P, _P, _I, _P, _P]),
    "tlmg_store_prefetch": (_I, [_P, _P, _I, _P, _P]),
    "tlmg_store_load_done": (_I, [_P, _I]),
    "tlmg_store_release": (_I, [_P, _I]),
    "tlmg_store_tick": (_I, [_P]),
    "tlmg_store_slot": (_I, [_P, _I, _P]),
    "tlmg_store_stats": (_I, [_P, _P]),
    "tlmg_check": (_I, [_P]),
    "tlmg_trace": (_I, [_P, _I, _P, _I]),
    "tlmg_profile": (_I, [_P, _I]),
    "tlmg_profile_read": (_I, [_P, _I, C.POINTER(C.c_double), C.POINTER(_I64), C.POINTER(_I64)]),
    "tlmg_launch_count": (_I64, [_P]),
    "tlmg_expert_ffn_noalloc": (_I, [_P, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P]),
}


def load() -> C.CDLL:
    """Load libtlmg.so (building it first when a toolchain is present)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists() and os.environ.get("TLMG_NO_BUILD") != "1":
        from . import build as _build
        _build.build()
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m tierlm_b200.build`")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def declared_symbols() -> list[str]:
    return list(_SIGS)


def errmsg() -> str:
    return (load().tlmg_errmsg() or b"").decode(errors="replace")


def check(rc: int) -> int:
    if rc < 0:
        raise TlmError(rc, errmsg())
    return rc
