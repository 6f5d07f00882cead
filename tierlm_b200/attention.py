"""Decode attention over a paged KV cache in HBM (attn_heads,
src/lib/tlm_model.c:683-719, and the K/V write of attention(),
src/lib/tlm_model.c:730-763) on CUDA tensors.

One layer's K and V caches are page pools [n_pages][KV][page_size][hd]
(float32 or bfloat16); a sequence's page table (int32) maps position t to
page table[t // page_size], row t % page_size. EXACT reproduces the
reference's order of operations bit for bit on f32 pages; SPLIT is the
flash-decoding kernel for long contexts (equal within float rounding).
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import BF16, F32, check, load
from .quant import _dev, stream_handle

EXACT, SPLIT = 0, 1
_KV_DT = {torch.float32: F32, torch.bfloat16: BF16}


def kv_dtype_code(t: torch.Tensor) -> int:
    if t.dtype not in _KV_DT:
        raise ValueError(f"KV pages must be float32 or bfloat16, not {t.dtype}")
    return _KV_DT[t.dtype]


def work_bytes(mode: int, kv_dtype: torch.dtype, T: int, H: int, KV: int, hd: int) -> int:
    return int(load().tlmg_attention_work_bytes(mode, _KV_DT[kv_dtype], T, H, KV, hd))


class PagedKV:
    """K and V page pools of one layer plus a scratch buffer for attention."""

    def __init__(self, n_pages: int, KV: int, page_size: int, hd: int, dtype=torch.float32, device="cuda"):
        shape = (n_pages, KV, page_size, hd)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.page_size, self.KV, self.hd = page_size, KV, hd
        self._work = torch.empty(0, dtype=torch.uint8, device=device)

    def write(self, k: torch.Tensor, v: torch.Tensor, page_id: int, pos: int) -> None:
        """k, v float32 [KV][hd] -> row pos % page_size of page page_id."""
        check(load().tlmg_kv_write(kv_dtype_code(self.k), _dev(k.contiguous(), "k"), _dev(v.contiguous(), "v"),
                                   self.k.data_ptr(), self.v.data_ptr(), self.k.shape[0], page_id,
                                   self.page_size, pos, self.KV, self.hd, C.c_void_p(stream_handle())))

    def attend(self, q: torch.Tensor, page_table: torch.Tensor, T: int, mode: int = EXACT,
               out: torch.Tensor | None = None) -> torch.Tensor:
        return decode_attention(q, self.k, self.v, page_table, T, mode, out=out, work=self)


def decode_attention(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor, page_table: torch.Tensor,
                     T: int, mode: int = EXACT, out: torch.Tensor | None = None, work=None) -> torch.Tensor:
    """q float32 [H][hd] -> out float32 [H][hd] over positions [0, T)."""
    n_pages, KV, page, hd = k_pages.shape
    H = q.shape[0]
    if v_pages.shape != k_pages.shape or v_pages.dtype != k_pages.dtype:
        raise ValueError("K and V page pools differ in shape or dtype")
    if page_table.dtype != torch.int32:
        raise ValueError("page_table must be int32")
    dt = kv_dtype_code(k_pages)
    need = int(load().tlmg_attention_work_bytes(mode, dt, T, H, KV, hd))
    holder = work if isinstance(work, PagedKV) else None
    if holder is not None:
        if holder._work.numel() < need:
            holder._work = torch.empty(need, dtype=torch.uint8, device=q.device)
        wbuf = holder._work
    else:
        wbuf = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty((H, hd), dtype=torch.float32, device=q.device)
    q = q.contiguous()
    check(load().tlmg_decode_attention(mode, dt, _dev(q, "q"), _dev(k_pages, "k_pages"), _dev(v_pages, "v_pages"),
                                       n_pages, _dev(page_table, "page_table"), page, T, H, KV, hd,
                                       wbuf.data_ptr(), wbuf.numel(), _dev(out, "out"),
                                       C.c_void_p(stream_handle())))
    return out


def _main() -> None:
    """`python -m tierlm_b200.attention --ctx T --kv bf16 --mode split`: one
    layer's decode attention (32 query heads, 4 KV heads, head_dim 128,
    64-position pages, shuffled page table) on random pages, `--calls`
    times, each call timed with CUDA events."""
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--kv", choices=["bf16", "f32"], default="bf16")
    ap.add_argument("--mode", choices=["exact", "split"], default="split")
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--page", type=int, default=64)
    a = ap.parse_args()
    dev = torch.device("cuda:0")
    dtype = torch.bfloat16 if a.kv == "bf16" else torch.float32
    n_pages = -(-a.ctx // a.page)
    g = torch.Generator(device=dev).manual_seed(0)
    kv = PagedKV(n_pages, a.kv_heads, a.page, a.head_dim, dtype=dtype, device=dev)
    kv.k.copy_(torch.randn(kv.k.shape, generator=g, device=dev))
    kv.v.copy_(torch.randn(kv.v.shape, generator=g, device=dev))
    table = torch.randperm(n_pages, device=dev, generator=g).to(torch.int32)
    q = torch.randn((a.heads, a.head_dim), generator=g, device=dev)
    mode = SPLIT if a.mode == "split" else EXACT
    nbytes = 2 * a.ctx * a.kv_heads * a.head_dim * kv.k.element_size()
    for i in range(a.calls):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = kv.attend(q, table, a.ctx, mode)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3
        print(f"call {i}: {us:.1f} us (host launch included), {nbytes / us / 1e3:.1f} GB/s of K/V, "
              f"|out| = {float(out.abs().sum()):.4f}")


if __name__ == "__main__":
    _main()
