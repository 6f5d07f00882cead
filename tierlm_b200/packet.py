"""Expert packets of the tlm store format (reference src/lib/tlm_packet.h:39-54).

`expert_packet` lays out one EXPERT packet the way the reference writer
does (tlm_writer_add, src/lib/tlm_packet.c:378-411: 64-byte header with
n_items 1, layout 0, CRC-32C of the payload, zero padding to 4096 bytes),
with gate | up | down at 64-byte aligned payload offsets (tlmc's expert
payload). When the three matrices have different dtypes the header carries
them in its reserved bytes (reserved[0] = 'D', reserved[1..3] = dtypes);
a uniform packet leaves reserved zero and is byte-identical to what the
reference writes. `parse` and `MoeContext.set_expert_packet` go through the
C ABI (tlmg_packet_parse / tlmg_set_expert_packet).
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np

from ._lib import PacketInfo, check, load
from .synth import pack_expert

MAGIC = 0x504D4C54        # "TLMP" (src/lib/tlm_packet.h:22)
VERSION = 2               # TLM_STORE_VERSION (src/lib/tlm_packet.h:24)
PK_EXPERT = 2             # TLM_PK_EXPERT (src/lib/tlm_packet.h:30)
HDR_BYTES = 64            # PKT_HDR_BYTES (src/lib/tlm_packet.c:55)
ALIGN_IO = 4096           # TLM_ALIGN_IO (src/lib/tlm_platform.h:18)
MIXED_MARK = 0x44         # 'D'
VERIFY_CRC, HOST = 1, 2   # TLMG_PKT_* flags

_HDR = struct.Struct("<IHHHHIIIQI3I16s")
assert _HDR.size == HDR_BYTES


def crc32c(data, crc: int = 0) -> int:
    buf = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray)) else data)
    return int(load().tlmg_crc32c(crc, buf.ctypes.data, buf.nbytes))


def header(layer: int, expert: int, dts, payload_len: int, crc: int, item_off) -> bytes:
    """The 64-byte EXPERT header; per-item dtypes go into reserved only when they differ."""
    dts = tuple(int(d) for d in dts)
    rsv = bytes(16) if len(set(dts)) == 1 else bytes([MIXED_MARK, *dts]) + bytes(12)
    return _HDR.pack(MAGIC, PK_EXPERT, VERSION, layer, 1, expert, dts[0], 0, payload_len, crc, *item_off, rsv)


def expert_packet(layer: int, expert: int, gate: np.ndarray, up: np.ndarray, down: np.ndarray, dts) -> np.ndarray:
    """One EXPERT packet (header, payload, zero padding to 4096 bytes) as uint8."""
    payload, off = pack_expert(gate, up, down)
    total = (HDR_BYTES + payload.nbytes + ALIGN_IO - 1) & ~(ALIGN_IO - 1)
    pkt = np.zeros(total, np.uint8)
    pkt[:HDR_BYTES] = np.frombuffer(header(layer, expert, dts, payload.nbytes, crc32c(payload), off), np.uint8)
    pkt[HDR_BYTES:HDR_BYTES + payload.nbytes] = payload
    return pkt


def parse(packet, verify_crc: bool = True) -> PacketInfo:
    """tlmg_packet_parse on a host buffer; raises TlmError on a bad packet."""
    buf = np.ascontiguousarray(np.frombuffer(packet, np.uint8) if isinstance(packet, (bytes, bytearray)) else packet)
    info = PacketInfo()
    check(load().tlmg_packet_parse(buf.ctypes.data, buf.nbytes, VERIFY_CRC if verify_crc else 0, C.byref(info)))
    return info
