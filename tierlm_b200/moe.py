"""Layer-level interface: HBM-resident expert slots and the MoE block.

MoeContext wraps a tlmg_ctx (include/tlmg.h). It mirrors the MoE half of
the reference's tlm_model (src/lib/tlm_model.h): experts are uploaded once
from packet payload bytes (set_expert), and expert_ffn / moe_layer replace
run_batch() + combine and moe() (src/lib/tlm_model.c:900-1055).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import Geom, check, load


def _ptr(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, torch.Tensor):
        if not a.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return a.data_ptr()
    if isinstance(a, np.ndarray):
        if not a.flags["C_CONTIGUOUS"]:
            raise ValueError("array must be C-contiguous")
        return a.ctypes.data
    raise TypeError(f"unsupported buffer type {type(a)!r}")


class MoeContext:
    def __init__(self, n_layers: int, d_model: int, d_expert: int, n_experts: int, top_k: int,
                 router: int = 0, routed_scale: float = 1.0, norm_eps: float = 1e-6, d_shared: int = 0,
                 device: int = 0):
        self.geom = Geom(n_layers, d_model, d_expert, d_shared, n_experts, top_k, router, routed_scale, norm_eps)
        self._lib = load()
        h = C.c_void_p()
        check(self._lib.tlmg_open(C.byref(self.geom), device, C.byref(h)))
        self._h = h
        self.device = device

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            self._lib.tlmg_close(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    FUSED_MODES = {"default": 1, "static": 2, "single": 4}

    def set_fused(self, on) -> None:
        """Persistent kernels (True, default: the static kernel), "single"
        (one-token launches by the single-token kernel), or the multi-kernel
        path (False). Identical bits."""
        mode = self.FUSED_MODES[on] if isinstance(on, str) else (1 if on else 0)
        check(self._lib.tlmg_set_fused(self._h, mode))

    BATCH_KERNELS = {"warp": 0, "tiled": 1, "mma": 2}

    def set_batch_kernels(self, mode: str, down: str | None = None) -> None:
        """Batched expert kernels: "mma" (tcgen05 tensor cores, default),
        "tiled" (CUDA cores, CTA per row tile) or "warp"; `down` picks the
        down projection's separately. Identical bits."""
        g = self.BATCH_KERNELS[mode]
        d = g if down is None else self.BATCH_KERNELS[down]
        if g == 0 and d != 0:
            raise ValueError("gate/up 'warp' combines only with down 'warp'")
        check(self._lib.tlmg_set_batch_kernels(self._h, g if g == d else 10 * g + d))

    def check(self) -> None:
        """Wait for queued work; raise if a kernel reported an expired wait."""
        check(self._lib.tlmg_check(self._h))

    def trace(self, on: bool = True):
        """Switch the persistent kernel's phase trace on / off; returns the
        last launch's stamps as int64 [CTAs, TRACE_POINTS] (ns) or None; the
        points are listed at tlmg_trace in include/tlmg.h."""
        buf = np.zeros(4096 * self.TRACE_POINTS, np.uint64)
        n = check(self._lib.tlmg_trace(self._h, 1 if on else 0, buf.ctypes.data, buf.size))
        return buf[:n].reshape(-1, self.TRACE_POINTS).astype(np.int64) if n else None

    TRACE_POINTS = 32

    def set_stream(self, stream=None) -> None:
        """Queue work on a torch.cuda.Stream (None: the context's own stream)."""
        from .quant import stream_handle
        ptr = None if stream is None else stream_handle(stream)
        check(self._lib.tlmg_set_stream(self._h, ptr))

    KERNEL_CLASSES = ("expert_ffn_gateup_or_fused", "expert_ffn_down", "route")

    def kernel_times(self, fn) -> tuple[str, float, int, int]:
        """Run fn() with per-launch event timing; return the dominant kernel
        class as (name, total ms, launches, algorithmic bytes per launch)."""
        check(self._lib.tlmg_profile(self._h, 1))
        try:
            fn()
            best = None
            for cls, name in enumerate(self.KERNEL_CLASSES):
                ms, n, b = C.c_double(), C.c_int64(), C.c_int64()
                check(self._lib.tlmg_profile_read(self._h, cls, C.byref(ms), C.byref(n), C.byref(b)))
                if best is None or ms.value > best[1]:
                    best = (name, ms.value, n.value, b.value)
            return best
        finally:
            check(self._lib.tlmg_profile(self._h, 0))

    @property
    def launches(self) -> int:
        return int(self._lib.tlmg_launch_count(self._h))

    def set_expert(self, layer: int, expert: int, dts, payload: np.ndarray, item_off) -> None:
        dt = (C.c_int32 * 3)(*dts)
        off = (C.c_uint64 * 3)(*item_off)
        payload = np.ascontiguousarray(payload, dtype=np.uint8)
        check(self._lib.tlmg_set_expert(self._h, layer, expert, dt, payload.ctypes.data, payload.nbytes, off))

    def set_expert_packet(self, layer: int, expert: int, packet, verify_crc: bool = True, host: bool = False) -> None:
        """Load an EXPERT packet of the tlm store (header + payload, see
        tierlm_b200/packet.py) into expert (layer, expert): HBM-resident, or
        with host=True registered for the slot cache (the packet buffer is
        then borrowed like set_expert_host's payload)."""
        n = packet.nbytes if hasattr(packet, "nbytes") else packet.numel() * packet.element_size()
        flags = (1 if verify_crc else 0) | (2 if host else 0)
        check(self._lib.tlmg_set_expert_packet(self._h, layer, expert, _ptr(packet), n, flags))

    # ---- HBM expert-slot cache (experts in host memory)
    def cache_enable(self, n_slots: int, slot_bytes: int) -> None:
        check(self._lib.tlmg_cache_enable(self._h, n_slots, slot_bytes))

    def set_expert_host(self, layer: int, expert: int, dts, payload, item_off) -> None:
        """Register an expert in host memory (a pinned torch tensor or a numpy
        array that outlives the context); the cache copies it on demand."""
        dt = (C.c_int32 * 3)(*dts)
        off = (C.c_uint64 * 3)(*item_off)
        n = payload.nbytes if hasattr(payload, "nbytes") else payload.numel() * payload.element_size()
        check(self._lib.tlmg_set_expert_host(self._h, layer, expert, dt, _ptr(payload), n, off))

    def cache_prefetch(self, layer: int, ids) -> None:
        a = np.ascontiguousarray(ids, dtype=np.int32)
        check(self._lib.tlmg_cache_prefetch(self._h, layer, a.ctypes.data, a.size))

    def cache_stats(self) -> dict:
        out = (C.c_int64 * 6)()
        check(self._lib.tlmg_cache_stats(self._h, out))
        return dict(zip(("hits", "misses", "prefetched", "prefetch_hits", "evictions", "bytes"), list(out)))

    def cache_tick(self) -> None:
        """One model step has passed (the selection frequencies' decay clock)."""
        check(self._lib.tlmg_cache_tick(self._h))

    def cache_lookahead(self, depth: int = 1, k: int = 0) -> None:
        """Router lookahead of moe_layer on cached layers (depth 1 or 0 = off)."""
        check(self._lib.tlmg_cache_lookahead(self._h, depth, k))

    def set_layer(self, layer: int, ffn_norm=None, router_dt: int = 0, router_w=None, router_row_bytes: int = 0,
                  router_bias=None, mask=None) -> None:
        check(self._lib.tlmg_set_layer(self._h, layer, _ptr(ffn_norm), router_dt, _ptr(router_w), router_row_bytes,
                                       _ptr(router_bias), _ptr(mask)))

    def set_shared(self, layer: int, dts, gate, up, down, gate_inp=None) -> None:
        dt = (C.c_int32 * 3)(*dts)
        check(self._lib.tlmg_set_shared(self._h, layer, dt, _ptr(gate), _ptr(up), _ptr(down), _ptr(gate_inp)))

    def expert_ffn(self, layer: int, x, logits, ffn, ids=None, w=None) -> None:
        """Routed-expert FFN of one token; host (numpy / pinned) or CUDA buffers."""
        check(self._lib.tlmg_expert_ffn(self._h, layer, _ptr(x), _ptr(logits), _ptr(ffn), _ptr(ids), _ptr(w)))

    def expert_ffn_many(self, layer0: int, x, logits, ffn) -> None:
        n_tok = (x.shape[0] if hasattr(x, "shape") and len(x.shape) == 2 else 1)
        check(self._lib.tlmg_expert_ffn_many(self._h, layer0, n_tok, _ptr(x), _ptr(logits), _ptr(ffn)))

    def expert_ffn_batch(self, layer: int, x, logits, ffn, ids=None, w=None) -> None:
        """Batched decode: x [n][D] and logits [n][E] of n tokens through one
        layer; ffn [n][D], ids/w [n][top_k] out. Bit-identical per token to
        expert_ffn; every selected expert is read once per call."""
        n_tok = x.shape[0] if hasattr(x, "shape") and len(x.shape) == 2 else 1
        check(self._lib.tlmg_expert_ffn_batch(self._h, layer, n_tok, _ptr(x), _ptr(logits), _ptr(ffn),
                                              _ptr(ids), _ptr(w)))

    # ---- expert parallelism (device buffers; see tierlm_b200.ep)
    @property
    def ep_record_bytes(self) -> int:
        return int(self._lib.tlmg_ep_record_bytes(self._h))

    def ep_dispatch(self, layer: int, x, logits, n_ranks: int, send, perm, w) -> list[int]:
        """Route + quantise x [n][D]; pack one record per (token, rank) pair
        into send grouped by owner GPU; returns the records per owner."""
        n_tok = x.shape[0]
        counts = (C.c_int64 * n_ranks)()
        check(self._lib.tlmg_ep_dispatch(self._h, layer, n_tok, _ptr(x), _ptr(logits), n_ranks, _ptr(send),
                                         _ptr(perm), _ptr(w), counts))
        return list(counts)

    def ep_dispatch_async(self, layer: int, x, logits, n_ranks: int, send, perm, w, counts) -> None:
        """ep_dispatch with the per-owner record counts written to a device
        int64 tensor on the stream; returns without waiting."""
        if not (isinstance(counts, torch.Tensor) and counts.is_cuda and counts.dtype == torch.int64):
            raise TypeError("counts must be a CUDA int64 tensor")
        check(self._lib.tlmg_ep_dispatch(self._h, layer, x.shape[0], _ptr(x), _ptr(logits), n_ranks, _ptr(send),
                                         _ptr(perm), _ptr(w), _ptr(counts)))

    def ep_experts(self, layer: int, e_lo: int, e_hi: int, n_rec: int, recv, eo) -> None:
        """Owner side of experts [e_lo, e_hi): n_rec received records -> eo [n_rec][D]."""
        check(self._lib.tlmg_ep_experts(self._h, layer, e_lo, e_hi, n_rec, _ptr(recv) if n_rec else None,
                                        _ptr(eo) if n_rec else None))

    def ep_combine(self, n_tok: int, back, perm, w, ffn) -> None:
        """Home side: ffn[t] = sum_r w[t, r] * back[perm[t, r]] in ascending r."""
        check(self._lib.tlmg_ep_combine(self._h, n_tok, _ptr(back), _ptr(perm), _ptr(w), _ptr(ffn)))

    # ---- the whole decoder step (tlm_model_step on the GPU)
    def step_open(self, n_heads: int, n_kv_heads: int, head_dim: int, vocab: int, inv_freq,
                  attn_scale: float = 1.0, max_ctx: int = 1024, kv_dtype: int = 0, attn_mode: int = 0) -> None:
        """KV pages for max_ctx positions (kv_dtype F32 = 0 or BF16 = 2),
        attention mode 0 = exact, 1 = split; inv_freq f32[head_dim / 2]."""
        inv = np.ascontiguousarray(inv_freq, np.float32)
        check(self._lib.tlmg_step_open(self._h, n_heads, n_kv_heads, head_dim, vocab, _ptr(inv), float(attn_scale),
                                       max_ctx, kv_dtype, attn_mode))

    def set_attention(self, layer: int, attn_norm, dts, q, k, v, o, row_bytes=None, q_norm=None,
                      k_norm=None) -> None:
        """Attention weights of a layer: dts = (q, k, v, o) dtypes."""
        dt = (C.c_int32 * 4)(*dts)
        w = (C.c_void_p * 4)(*[_ptr(m) for m in (q, k, v, o)])
        rb = (C.c_size_t * 4)(*(row_bytes or (0, 0, 0, 0)))
        check(self._lib.tlmg_set_attention(self._h, layer, _ptr(attn_norm), dt, w, rb, _ptr(q_norm), _ptr(k_norm)))

    def set_embedding(self, dt: int, table, row_bytes: int = 0) -> None:
        check(self._lib.tlmg_set_embedding(self._h, dt, _ptr(table), row_bytes))

    def set_output(self, out_norm, dt: int, lm_head, row_bytes: int = 0) -> None:
        check(self._lib.tlmg_set_output(self._h, _ptr(out_norm), dt, _ptr(lm_head), row_bytes))

    def decode_step(self, token: int, pos: int, logits=None) -> None:
        """One position through every layer; logits f32[vocab] (host or
        CUDA) or None (no lm_head)."""
        check(self._lib.tlmg_decode_step(self._h, token, pos, _ptr(logits)))

    def step_graphs(self, on: bool) -> None:
        """Graph replay of the step from the second call on (default on)."""
        check(self._lib.tlmg_step_graphs(self._h, 1 if on else 0))

    def step_info(self) -> dict:
        out = (C.c_int64 * 4)()
        check(self._lib.tlmg_step_info(self._h, out))
        return {"steps": out[0], "replays": out[1], "captures": out[2], "graphs_off": bool(out[3])}

    def step_stats(self, reset: bool = False) -> dict:
        """tlm_model_stats of the step: tokens, attn_ns, moe_ns, expert_wait_ns,
        other_ns (phase times from steps run while profiling)."""
        out = (C.c_uint64 * 5)()
        check(self._lib.tlmg_step_stats(self._h, out, 1 if reset else 0))
        return dict(zip(("tokens", "attn_ns", "moe_ns", "expert_wait_ns", "other_ns"), list(out)))

    def profile(self, on: bool) -> None:
        check(self._lib.tlmg_profile(self._h, 1 if on else 0))

    def ep_open(self, rank: int, n_ranks: int, max_tok: int) -> bytes:
        """Opens this rank's peer-memory exchange; returns its handle (bytes
        to hand to every peer)."""
        check(self._lib.tlmg_ep_open(self._h, rank, n_ranks, max_tok))
        buf = C.create_string_buffer(self._lib.tlmg_ep_handle_bytes())
        check(self._lib.tlmg_ep_handle(self._h, buf))
        return buf.raw

    def ep_connect(self, handles: list[bytes]) -> None:
        """Maps every peer's exchange buffer (handles in rank order)."""
        check(self._lib.tlmg_ep_connect(self._h, b"".join(handles)))

    def ep_layer(self, layer: int, x, logits, ffn, ids=None, w=None) -> None:
        """One expert-parallel layer over peer memory (device tensors):
        ffn = the routed experts' combine of x; no host wait."""
        n = x.shape[0]
        check(self._lib.tlmg_ep_layer(self._h, layer, n, _ptr(x) if n else None, _ptr(logits) if n else None,
                                      _ptr(ffn) if n else None, _ptr(ids), _ptr(w)))

    def ep_close(self) -> None:
        check(self._lib.tlmg_ep_close(self._h))

    def moe_layer(self, layer: int, h, ids=None, w=None, onorm=None) -> None:
        """moe() of one token (h += ffn in place); onorm receives the route
        hook's per-rank output norms."""
        if onorm is None:
            check(self._lib.tlmg_moe_layer(self._h, layer, _ptr(h), _ptr(ids), _ptr(w)))
        else:
            check(self._lib.tlmg_moe_layer_ex(self._h, layer, _ptr(h), _ptr(ids), _ptr(w), _ptr(onorm)))

    def set_dense_ffn(self, layer: int, dts, gate, up, down, d_ffn: int) -> None:
        """Make `layer` a dense-FFN layer (host weight rows, packed)."""
        check(self._lib.tlmg_set_dense_ffn(self._h, layer, d_ffn, (C.c_int32 * 3)(*dts), _ptr(gate), _ptr(up),
                                           _ptr(down)))
