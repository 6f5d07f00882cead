"""Seeded synthetic weights and inputs for tests and benchmarks.

Random K-quant rows follow the generator rules of the reference's own test
suite (tests/test_quant.c:642-691, make_wrow): random code bytes with finite
random scale fields, plus the edge modes all-zero, maximum magnitude and
extreme scales. Expert payloads are packed like tlmc's build_expert
(src/bin/tlmc.c:1132-1157): gate | up | down at 64-byte aligned offsets.
Device variants build the same layouts directly in HBM with torch, for the
full-size benchmark (tens of GB of experts).
"""
from __future__ import annotations

import numpy as np

from ._lib import MXFP4, Q4_K, Q5_K, Q6_K, Q8_0, Q8_K

BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210), Q8_K: (256, 292), MXFP4: (32, 17)}


def row_bytes(dt: int, n: int) -> int:
    qk, bb = BLOCK[dt]
    assert n % qk == 0
    return n // qk * bb


def _f16b(v, shape) -> np.ndarray:
    """f16 little-endian bytes of v broadcast to `shape`: uint8 [*shape, 2]."""
    a = np.ascontiguousarray(np.broadcast_to(np.asarray(v, np.float16), shape))
    return a.view(np.uint8).reshape(*shape, 2)


def fix_scales(dt: int, blocks: np.ndarray, rng: np.random.Generator, mode: int = 0) -> None:
    """blocks: uint8 [..., bb] view of whole blocks; rewrite the scale fields
    in place the way the reference's make_wrow does."""
    nb = blocks.shape[:-1]
    if mode == 4:
        dv = np.where(rng.integers(0, 2, nb) == 1, 65504.0, 2.0 ** -24) * np.where(rng.integers(0, 2, nb) == 1, -1.0, 1.0)
    else:
        dv = rng.uniform(-0.05, 0.05, nb)
    if mode == 1:
        dv = np.zeros(nb)
    if dt == Q8_0:
        blocks[..., 0:2] = _f16b(0.01 if mode == 2 else dv, nb)
        if mode == 2:
            blocks[..., 2:34] = np.where(rng.integers(0, 2, (*nb, 32)) == 1, 0x80, 0x7F)
    elif dt in (Q4_K, Q5_K):
        dmin = dv if mode == 4 else rng.uniform(0, 0.05, nb)
        blocks[..., 0:2] = _f16b(0.01 if mode == 2 else dv, nb)
        blocks[..., 2:4] = _f16b(0.01 if mode == 2 else (0.0 if mode == 1 else dmin), nb)
        if mode == 2:
            blocks[..., 4:] = 0xFF
    elif dt == Q6_K:
        blocks[..., 208:210] = _f16b(0.01 if mode == 2 else dv, nb)
        if mode == 2:
            fill = np.where(rng.integers(0, 2, nb) == 1, 0xFF, 0x00).astype(np.uint8)
            blocks[..., 0:192] = fill[..., None]
            blocks[..., 192:208] = np.tile(np.array([0x7F, 0x80], np.uint8), 8)
    elif dt == Q8_K:
        d = np.full(nb, 1e30) if mode == 2 else (dv * 1e3 if mode == 4 else dv)
        blocks[..., 0:4] = np.ascontiguousarray(np.asarray(d, np.float32)).view(np.uint8).reshape(*nb, 4)
        if mode == 2:
            blocks[..., 4:260] = np.where(rng.integers(0, 2, (*nb, 256)) == 1, 0x80, 0x7F)
    elif dt == MXFP4:
        if mode == 2:
            blocks[..., 0] = 254
            blocks[..., 1:] = np.where(rng.integers(0, 2, nb) == 1, 0x77, 0xFF)[..., None]
        elif mode == 4:
            blocks[..., 0] = np.array([0, 1, 254, 255], np.uint8)[rng.integers(0, 4, nb)]
        elif mode != 1:
            blocks[..., 0] = (100 + rng.integers(0, 50, nb)).astype(np.uint8)


def rand_rows(dt: int, nrows: int, n: int, rng: np.random.Generator, mode: int = 0) -> np.ndarray:
    """uint8 [nrows, row_bytes] of random blocks with finite scale fields."""
    qk, bb = BLOCK[dt]
    nb = n // qk
    if mode == 1:
        w = np.zeros((nrows, nb, bb), np.uint8)
    else:
        w = rng.integers(0, 256, (nrows, nb, bb), dtype=np.uint8)
    fix_scales(dt, w, rng, mode)
    return w.reshape(nrows, nb * bb)


def pack_expert(gate: np.ndarray, up: np.ndarray, down: np.ndarray) -> tuple[np.ndarray, tuple[int, int, int]]:
    """gate | up | down at 64-byte aligned offsets (tlmc's packet payload)."""
    parts = [np.ascontiguousarray(m).reshape(-1) for m in (gate, up, down)]
    offs, cur = [], 0
    for p in parts:
        offs.append(cur)
        cur = (cur + p.nbytes + 63) & ~63
    buf = np.zeros(cur, np.uint8)
    for o, p in zip(offs, parts):
        buf[o:o + p.nbytes] = p
    return buf, tuple(offs)


def rand_expert(rng: np.random.Generator, D: int, de: int, dts) -> tuple[np.ndarray, tuple, tuple]:
    g = rand_rows(dts[0], de, D, rng)
    u = rand_rows(dts[1], de, D, rng)
    d = rand_rows(dts[2], D, de, rng)
    payload, off = pack_expert(g, u, d)
    return payload, off, tuple(dts)


# ---- device-side generation (torch) ---------------------------------------
def device_rows(dt: int, nrows: int, n: int, gen, device) -> "torch.Tensor":  # noqa: F821
    """The same distribution as rand_rows(mode 0), built on the GPU."""
    import torch
    qk, bb = BLOCK[dt]
    nb = n // qk
    w = torch.randint(0, 256, (nrows, nb, bb), dtype=torch.uint8, device=device, generator=gen)

    def f16(lo, hi):
        v = torch.rand((nrows, nb), device=device, generator=gen) * (hi - lo) + lo
        return v.to(torch.float16).contiguous().view(torch.uint8).view(nrows, nb, 2)

    if dt == Q8_0:
        w[..., 0:2] = f16(-0.05, 0.05)
    elif dt in (Q4_K, Q5_K):
        w[..., 0:2] = f16(-0.05, 0.05)
        w[..., 2:4] = f16(0.0, 0.05)
    elif dt == Q6_K:
        w[..., 208:210] = f16(-0.05, 0.05)
    elif dt == Q8_K:
        v = (torch.rand((nrows, nb), device=device, generator=gen) * 0.1 - 0.05).contiguous()
        w[..., 0:4] = v.view(torch.uint8).view(nrows, nb, 4)
    elif dt == MXFP4:
        w[..., 0] = (100 + torch.randint(0, 50, (nrows, nb), device=device, generator=gen)).to(torch.uint8)
    return w.view(nrows, nb * bb)
