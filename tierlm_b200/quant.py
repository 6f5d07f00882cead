"""Kernel-level interface of the sm_100a tier, mirroring the reference's
src/lib/tlm_quant.h (tlm_quantize_act, tlm_matvec_rows, tlm_vec_dot,
tlm_row_bytes, tlm_qact_bytes, tlm_act_kind_for) on CUDA tensors.

Device buffers are torch CUDA tensors (uint8 for packed blocks, float32 for
vectors); torch is only the allocator and stream holder. Errors raise
TlmError with the library's message; as in the reference, a failed matvec
also leaves NaN in the requested output rows.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import (BF16, DTYPE_NAMES, F16, F32, MXFP4, Q4_K, Q5_K, Q6_K, Q8_0, Q8_K,  # noqa: F401
                   TlmError, check, load)


CUDA_STREAM_LEGACY = 1   # cudaStreamLegacy: the legacy default stream handle


def stream_handle(stream=None) -> int:
    """cudaStream_t of a torch stream for the C ABI. torch's default stream
    has handle 0, which the ABI reads as "the library's own stream", so it
    is passed as cudaStreamLegacy instead."""
    s = (stream or torch.cuda.current_stream()).cuda_stream
    return s if s else CUDA_STREAM_LEGACY


def _stream_ptr() -> int:
    return stream_handle()


def tier() -> str:
    return load().tlmg_tier().decode()


def dtype_block(dt: int) -> int:
    return load().tlmg_dtype_block(dt)


def dtype_block_bytes(dt: int) -> int:
    return load().tlmg_dtype_block_bytes(dt)


def row_bytes(dt: int, n: int) -> int:
    return load().tlmg_row_bytes(dt, n)


def qact_bytes(kind: int, n: int) -> int:
    return load().tlmg_qact_bytes(kind, n)


def act_kind_for(dt: int) -> int:
    return load().tlmg_act_kind_for(dt)


def _dev(t: torch.Tensor, what: str) -> int:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TlmError(-3, f"{what} must be a CUDA tensor")
    if not t.is_contiguous():
        raise TlmError(-3, f"{what} must be contiguous")
    return t.data_ptr()


def quantize_act(kind: int, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """tlm_quantize_act: f32 x[n] -> Q8_K / Q8_0 blocks (or an f32 copy)."""
    n = x.numel()
    if x.dtype != torch.float32:
        raise TlmError(-3, "quantize_act: x must be float32")
    nbytes = qact_bytes(kind, n)
    if out is None:
        out = torch.empty(max(nbytes, 4), dtype=torch.uint8, device=x.device)
    check(load().tlmg_quantize_act(kind, _dev(x, "x"), n, _dev(out, "out"), C.c_void_p(_stream_ptr())))
    return out


def matvec_rows(dt: int, W: torch.Tensor, row_bytes_: int, act: torch.Tensor, y: torch.Tensor, n: int,
                r0: int, r1: int, w_offset: int = 0) -> None:
    """tlm_matvec_rows: y[r] = dot(W[r], act) for r in [r0, r1). W is the
    uint8 weight buffer; w_offset lets rows start at any byte offset."""
    rc = load().tlmg_matvec_rows(dt, C.c_void_p(_dev(W, "W") + w_offset), row_bytes_, _dev(act, "act"),
                                 _dev(y, "y"), n, r0, r1, C.c_void_p(_stream_ptr()))
    check(rc)


def dequantize_rows(dt: int, src: torch.Tensor, row_bytes_: int, n: int, rows: int,
                    y: torch.Tensor | None = None) -> torch.Tensor:
    """tlm_dequantize_row over `rows` rows of n elements (row stride
    row_bytes_) -> f32 [rows][n]."""
    if y is None:
        y = torch.empty((rows, n), dtype=torch.float32, device=src.device)
    check(load().tlmg_dequantize_rows(dt, _dev(src, "src"), row_bytes_, _dev(y, "y"), n, rows,
                                      C.c_void_p(_stream_ptr())))
    return y


def vec_dot(dt: int, wrow: torch.Tensor, act: torch.Tensor, n: int) -> float:
    """tlm_vec_dot on one device row (synchronous)."""
    y = torch.empty(1, dtype=torch.float32, device=wrow.device)
    matvec_rows(dt, wrow, row_bytes(dt, n), act, y, n, 0, 1)
    return float(y.item())


def block_partials(dt: int, W: torch.Tensor, row_bytes_: int, act: torch.Tensor, n: int, nrows: int,
                   w_offset: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact per-block int32 partials (isum, msum) of rows [0, nrows)."""
    nb = n // dtype_block(dt)
    isum = torch.empty((nrows, nb), dtype=torch.int32, device=W.device)
    msum = torch.empty((nrows, nb), dtype=torch.int32, device=W.device)
    check(load().tlmg_block_partials(dt, C.c_void_p(_dev(W, "W") + w_offset), row_bytes_, _dev(act, "act"),
                                     n, nrows, _dev(isum, "isum"), _dev(msum, "msum"),
                                     C.c_void_p(_stream_ptr())))
    return isum, msum


def route(router: int, logits: torch.Tensor, k: int, routed_scale: float = 1.0,
          mask: torch.Tensor | None = None, bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Router top-k (reference route/topk): returns (ids int32[k], w f32[k])."""
    E = logits.numel()
    ids = torch.empty(k, dtype=torch.int32, device=logits.device)
    w = torch.empty(k, dtype=torch.float32, device=logits.device)
    check(load().tlmg_route(router, _dev(logits, "logits"), _dev(mask, "mask") if mask is not None else None,
                            _dev(bias, "bias") if bias is not None else None, E, k, routed_scale,
                            _dev(ids, "ids"), _dev(w, "w"), C.c_void_p(_stream_ptr())))
    return ids, w
