"""The expert cache's slot policy on its own (tlmg_store_*, include/tlmg.h).

Mirrors the reference's store API (tlm_store_acquire / _release /
_prefetch / _tick, src/lib/tlm_store.h:41-69) for the decisions only: keys
are layer * E + expert, and the caller moves the bytes (copy the expert into
the returned slot, then load_done).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import TLMG_EBUSY, TlmError, check, errmsg, load


class StorePolicy:
    def __init__(self, n_keys: int, n_slots: int, top_k: int):
        self._lib = load()
        h = C.c_void_p()
        check(self._lib.tlmg_store_open(n_keys, n_slots, top_k, C.byref(h)))
        self._h = h
        self.n_slots = n_slots

    def close(self) -> None:
        if self._h:
            self._lib.tlmg_store_close(self._h)
            self._h = None

    def acquire(self, keys) -> tuple[np.ndarray, np.ndarray, bool]:
        """(slots, loads, ok): ok False is the reference's TLM_EBUSY."""
        keys = np.ascontiguousarray(keys, np.int32)
        slots = np.zeros(len(keys), np.int32)
        loads = np.zeros(len(keys), np.int32)
        rc = self._lib.tlmg_store_acquire(self._h, keys.ctypes.data, len(keys), slots.ctypes.data, loads.ctypes.data)
        if rc not in (0, TLMG_EBUSY):
            raise TlmError(rc, errmsg())
        return slots, loads, rc == 0

    def prefetch(self, keys) -> list[tuple[int, int]]:
        """Started hint loads as (slot, key)."""
        keys = np.ascontiguousarray(keys, np.int32)
        slots = np.zeros(max(len(keys), 1), np.int32)
        ko = np.zeros(max(len(keys), 1), np.int32)
        n = check(self._lib.tlmg_store_prefetch(self._h, keys.ctypes.data, len(keys), slots.ctypes.data,
                                                ko.ctypes.data))
        return [(int(slots[i]), int(ko[i])) for i in range(n)]

    def load_done(self, slot: int) -> None:
        check(self._lib.tlmg_store_load_done(self._h, slot))

    def release(self, slot: int) -> None:
        check(self._lib.tlmg_store_release(self._h, slot))

    def tick(self) -> None:
        check(self._lib.tlmg_store_tick(self._h))

    def slot(self, i: int) -> tuple[int, int, int, int]:
        out = (C.c_int32 * 4)()
        check(self._lib.tlmg_store_slot(self._h, i, out))
        return tuple(out)

    def stats(self) -> list[int]:
        out = (C.c_int64 * 6)()
        check(self._lib.tlmg_store_stats(self._h, out))
        return list(out)
