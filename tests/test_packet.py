"""Expert packets of the tlm store format through the C ABI.

CPU: tlmg_crc32c against the published CRC-32C check value and the
reference's tlm_crc32c; a uniform packet written by tierlm_b200.packet is
byte-identical to the one the reference's own writer puts on a drive
(tlm_writer_add, src/lib/tlm_packet.c:378-411); tlmg_packet_parse accepts
and rejects the same buffers as the reference's tlm_packet_verify
(src/lib/tlm_packet.c:788-815), with the same error codes, including the
per-item dtype extension (which the reference's verify accepts unchanged).
GPU: an expert loaded from a mixed-dtype packet computes the same bits as
the same payload loaded with tlmg_set_expert, resident and slot-cached.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tierlm_b200 import _lib, packet
from tierlm_b200.synth import rand_rows

Q4_K, Q6_K = _lib.Q4_K, _lib.Q6_K


class RefLoc(C.Structure):
    """tlm_packet_loc (src/lib/tlm_packet.h:69-80), natural alignment."""
    _fields_ = [("type", C.c_uint16), ("layer", C.c_uint16), ("id", C.c_uint32), ("drive", C.c_uint8),
                ("replica_drive", C.c_uint8), ("flags", C.c_uint16), ("offset", C.c_uint64),
                ("replica_offset", C.c_uint64), ("total_len", C.c_uint64), ("crc32c", C.c_uint32),
                ("heat", C.c_float)]


def _ref():
    import oracle
    R = oracle.ref()
    if R is None:
        pytest.skip("oracle/_ref (the reference's own library) is not built")
    R.tlm_crc32c.argtypes = [C.c_uint32, C.c_void_p, C.c_size_t]
    R.tlm_crc32c.restype = C.c_uint32
    R.tlm_packet_verify.argtypes = [C.POINTER(RefLoc), C.c_void_p, C.c_uint64, C.POINTER(C.c_void_p),
                                    C.POINTER(C.c_uint64)]
    R.tlm_packet_verify.restype = C.c_int
    R.tlm_writer_open.argtypes = [C.c_char_p, C.POINTER(C.c_char_p), C.c_int]
    R.tlm_writer_open.restype = C.c_void_p
    R.tlm_writer_add.argtypes = [C.c_void_p, C.c_int, C.c_uint16, C.c_uint32, C.c_uint32, C.c_void_p, C.c_uint64,
                                 C.POINTER(C.c_uint32), C.c_int, C.c_int, C.POINTER(RefLoc)]
    R.tlm_writer_add.restype = C.c_int
    R.tlm_writer_finish.argtypes = [C.c_void_p, C.c_int]
    R.tlm_writer_finish.restype = C.c_int
    R.tlm_writer_free.argtypes = [C.c_void_p]
    R.tlm_writer_free.restype = None
    return R


def _expert(rng, D, de, dts):
    return (rand_rows(dts[0], de, D, rng), rand_rows(dts[1], de, D, rng), rand_rows(dts[2], D, de, rng))


def _ref_verify(R, buf: np.ndarray, layer: int, expert: int) -> tuple[int, int]:
    """tlm_packet_verify with the manifest entry a correct store would hold."""
    crc = packet._HDR.unpack(bytes(buf[:64]))[9] if buf.nbytes >= 64 else 0
    loc = RefLoc(type=packet.PK_EXPERT, layer=layer, id=expert, drive=0, replica_drive=0xFF,
                 total_len=buf.nbytes, crc32c=crc)
    pl, n = C.c_void_p(), C.c_uint64()
    rc = R.tlm_packet_verify(C.byref(loc), buf.ctypes.data, buf.nbytes, C.byref(pl), C.byref(n))
    return rc, n.value


def _ours(buf: np.ndarray, flags: int = packet.VERIFY_CRC) -> tuple[int, _lib.PacketInfo]:
    info = _lib.PacketInfo()
    return _lib.load().tlmg_packet_parse(buf.ctypes.data, buf.nbytes, flags, C.byref(info)), info


def test_crc32c_check_value_and_reference():
    assert packet.crc32c(b"123456789") == 0xE3069283   # CRC-32C (Castagnoli) check value
    assert packet.crc32c(b"") == 0
    R = _ref()
    rng = np.random.default_rng(7)
    for n in (1, 7, 8, 9, 63, 64, 1000, 4099, 100_003):
        a = rng.integers(0, 256, n + 3, dtype=np.uint8)
        for off in (0, 1, 3):
            v = a[off:off + n]
            v = np.ascontiguousarray(v)
            assert packet.crc32c(v) == R.tlm_crc32c(0, v.ctypes.data, n)
            h = n // 3
            assert packet.crc32c(v[h:], packet.crc32c(v[:h])) == R.tlm_crc32c(0, v.ctypes.data, n)


def test_uniform_packet_bytes_match_reference_writer(tmp_path):
    R = _ref()
    rng = np.random.default_rng(11)
    D, de = 512, 256
    for layer, expert, dt in ((0, 3, Q4_K), (5, 17, Q6_K)):
        g, u, d = _expert(rng, D, de, (dt, dt, dt))
        ours = packet.expert_packet(layer, expert, g, u, d, (dt, dt, dt))
        payload = ours[64:64 + packet.parse(ours).payload_len]
        off = (C.c_uint32 * 3)(*packet.parse(ours).item_off)
        drive = str(tmp_path / f"d{layer}").encode()
        w = R.tlm_writer_open(b"store", (C.c_char_p * 1)(drive), 1)
        assert w
        loc = RefLoc()
        assert R.tlm_writer_add(w, packet.PK_EXPERT, layer, expert, dt, payload.ctypes.data, payload.nbytes, off,
                                0, -1, C.byref(loc)) == 0
        assert R.tlm_writer_finish(w, 1) == 0
        R.tlm_writer_free(w)
        raw = np.fromfile(tmp_path / f"d{layer}" / "store.tlmp", np.uint8)
        theirs = raw[loc.offset:loc.offset + loc.total_len]
        assert loc.total_len == ours.nbytes
        assert np.array_equal(theirs, ours)
        rc, info = _ours(np.ascontiguousarray(theirs))
        assert rc == 0 and info.mixed == 0 and list(info.item_dt) == [dt] * 3
        assert (info.layer, info.id, info.type, info.total_len) == (layer, expert, packet.PK_EXPERT, loc.total_len)


def test_mixed_packet_parse_and_reference_verify():
    R = _ref()
    rng = np.random.default_rng(12)
    dts = (Q4_K, Q4_K, Q6_K)
    g, u, d = _expert(rng, 512, 256, dts)
    pkt = packet.expert_packet(2, 9, g, u, d, dts)
    rc, info = _ours(pkt)
    assert rc == 0 and info.mixed == 1 and tuple(info.item_dt) == dts
    assert info.item_off[0] == 0 and info.item_off[1] == g.nbytes and info.item_off[2] == g.nbytes + u.nbytes
    assert _ref_verify(R, pkt, 2, 9) == (0, info.payload_len)


@pytest.mark.parametrize("case", ["ok", "payload_byte", "crc_field", "magic", "version", "short", "length"])
def test_parse_agrees_with_reference_verify(case):
    R = _ref()
    rng = np.random.default_rng(13)
    g, u, d = _expert(rng, 256, 256, (Q4_K, Q4_K, Q6_K))
    pkt = packet.expert_packet(1, 4, g, u, d, (Q4_K, Q4_K, Q6_K))
    n = int(packet.parse(pkt).payload_len)
    if case == "payload_byte":
        pkt[64 + n // 2] ^= 0x10
    elif case == "crc_field":
        pkt[32] ^= 1
    elif case == "magic":
        pkt[0] ^= 1
    elif case == "version":
        pkt[6] = 3
    elif case == "short":
        pkt = np.ascontiguousarray(pkt[:40])
    elif case == "length":
        pkt[24:32] = np.frombuffer(np.uint64(pkt.nbytes).tobytes(), np.uint8)
    want = {"ok": 0, "short": _lib.TLMG_EINVAL}.get(case, _lib.TLMG_EFORMAT)
    rc, _ = _ours(pkt)
    assert rc == want, _lib.errmsg()
    assert _ref_verify(R, pkt, 1, 4)[0] == want


def test_parse_flags_and_extension_errors():
    rng = np.random.default_rng(14)
    g, u, d = _expert(rng, 256, 256, (Q4_K,) * 3)
    pkt = packet.expert_packet(0, 0, g, u, d, (Q4_K,) * 3)
    pkt[64 + 5] ^= 1                                  # bad payload byte: only the CRC check sees it
    assert _ours(pkt, 0)[0] == 0
    assert _ours(pkt)[0] == _lib.TLMG_EFORMAT and "CRC" in _lib.errmsg()
    pkt[48] = 0x7F                                     # unknown header extension
    assert _ours(pkt, 0)[0] == _lib.TLMG_EFORMAT and "extension" in _lib.errmsg()
    assert _ours(pkt, 0x10)[0] == _lib.TLMG_EINVAL
    lib = _lib.load()
    assert lib.tlmg_packet_parse(None, 64, 0, None) == _lib.TLMG_EINVAL


@pytest.mark.gpu
@pytest.mark.parametrize("host", [False, True])
def test_packet_expert_matches_set_expert(host):
    import torch
    from tierlm_b200.moe import MoeContext
    rng = np.random.default_rng(15)
    D, de, E, k, dts = 512, 256, 8, 2, (Q4_K, Q4_K, Q6_K)
    experts = [_expert(rng, D, de, dts) for _ in range(E)]
    x = torch.tensor(rng.standard_normal(D), dtype=torch.float32, device="cuda")
    logits = torch.tensor(rng.standard_normal(E), dtype=torch.float32, device="cuda")
    outs = []
    keep = []
    for mode in ("payload", "packet"):
        with MoeContext(1, D, de, E, k) as ctx:
            if host:
                ctx.cache_enable(4, 1 << 20)
            for e, (g, u, d) in enumerate(experts):
                pkt = packet.expert_packet(0, e, g, u, d, dts)
                if mode == "payload":
                    info = packet.parse(pkt)
                    payload = np.ascontiguousarray(pkt[64:64 + info.payload_len])
                    if host:
                        payload = torch.from_numpy(payload).pin_memory()
                        ctx.set_expert_host(0, e, dts, payload, tuple(info.item_off))
                    else:
                        ctx.set_expert(0, e, dts, payload, tuple(info.item_off))
                    keep.append(payload)
                else:
                    if host:
                        pkt = torch.from_numpy(pkt).pin_memory()
                    ctx.set_expert_packet(0, e, pkt, host=host)
                    keep.append(pkt)
            with pytest.raises(_lib.TlmError) as ei:   # a packet of another expert is refused
                ctx.set_expert_packet(0, 1, packet.expert_packet(0, 2, *experts[2], dts))
            assert ei.value.code == _lib.TLMG_EFORMAT and "does not match" in str(ei.value)
            ffn = torch.empty(D, dtype=torch.float32, device="cuda")
            ctx.expert_ffn(0, x, logits, ffn)
            torch.cuda.synchronize()
            ctx.check()
            outs.append(ffn.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
