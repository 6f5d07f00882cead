// tlmg_packet.cu - expert packets of the tlm store format, read straight
// into the library (host code only; no kernels).
//
// A packet on a drive is a 64-byte header, the payload, and zero padding to
// a 4096-byte multiple (reference src/lib/tlm_packet.h:39-54,
// src/lib/tlm_packet.c:378-411). For an EXPERT packet the payload holds the
// gate, up and down matrices at item_off[0..2]. The reference stores one
// dtype per packet and takes each expert's dtype from the manifest's expert
// table (src/lib/tlm_model.c:880-896), so a Q4_K gate/up with a Q6_K down
// (the Q4_K_M-like mix) cannot be described by one packet. The extension
// read here uses the header's reserved bytes, which the reference writer
// zeroes (src/lib/tlm_packet.c:392) and no reference reader looks at:
//
//   reserved[0] = 'D' (0x44)   per-item dtypes present
//   reserved[1..3]             tlm_dtype of gate, up, down
//
// A packet whose reserved[0] is 0 is an ordinary reference packet and every
// item has the header's `dtype`; a mixed packet still passes the reference's
// tlm_packet_verify unchanged (the header layout, CRC and length rules are
// the reference's), so the extension is backward compatible in both
// directions for verification.

#include <cstring>

#include "tlmg_internal.h"

namespace {

constexpr uint32_t kMagic = 0x504D4C54u;   // "TLMP" (src/lib/tlm_packet.h:22)
constexpr uint32_t kVersion = 2u;          // TLM_STORE_VERSION (src/lib/tlm_packet.h:24)
constexpr uint32_t kTypeExpert = 2u;       // TLM_PK_EXPERT (src/lib/tlm_packet.h:30)
constexpr uint32_t kHdrBytes = 64u;        // PKT_HDR_BYTES (src/lib/tlm_packet.c:55)
constexpr uint64_t kAlignIO = 4096u;       // TLM_ALIGN_IO (src/lib/tlm_platform.h:18)
constexpr uint8_t kMixedMark = 0x44u;      // 'D': per-item dtypes in reserved[1..3]

// CRC-32C (Castagnoli, reflected polynomial 0x82F63B78), slicing by 8: the
// same value as the reference's tlm_crc32c (src/lib/tlm_platform.c:443-458,
// "init 0": the register starts at ~crc and the result is inverted).
struct Crc32cTables {
    uint32_t t[8][256];
    Crc32cTables() {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int b = 0; b < 8; b++) c = (c >> 1) ^ (0x82F63B78u & (0u - (c & 1u)));
            t[0][i] = c;
        }
        for (uint32_t i = 0; i < 256; i++)
            for (int s = 1; s < 8; s++) t[s][i] = (t[s - 1][i] >> 8) ^ t[0][t[s - 1][i] & 0xFFu];
    }
};
const Crc32cTables &crc_tables() {
    static const Crc32cTables tabs;   // thread-safe one-time init (C++11 statics)
    return tabs;
}

uint32_t rd32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }
uint16_t rd16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }
uint64_t rd64(const uint8_t *p) { uint64_t v; memcpy(&v, p, 8); return v; }

}  // namespace

using namespace tlmg;

extern "C" uint32_t tlmg_crc32c(uint32_t crc, const void *buf, size_t len) {
    const Crc32cTables &T = crc_tables();
    const uint8_t *p = static_cast<const uint8_t *>(buf);
    uint32_t c = ~crc;
    if (!p) return crc;
    while (len && (reinterpret_cast<uintptr_t>(p) & 7u)) {
        c = T.t[0][(c ^ *p++) & 0xFFu] ^ (c >> 8);
        len--;
    }
    while (len >= 8) {
        const uint32_t lo = rd32(p) ^ c, hi = rd32(p + 4);
        c = T.t[7][lo & 0xFFu] ^ T.t[6][(lo >> 8) & 0xFFu] ^ T.t[5][(lo >> 16) & 0xFFu] ^ T.t[4][lo >> 24] ^
            T.t[3][hi & 0xFFu] ^ T.t[2][(hi >> 8) & 0xFFu] ^ T.t[1][(hi >> 16) & 0xFFu] ^ T.t[0][hi >> 24];
        p += 8;
        len -= 8;
    }
    while (len--) c = T.t[0][(c ^ *p++) & 0xFFu] ^ (c >> 8);
    return ~c;
}

// Header checks in the order of the reference's tlm_packet_verify
// (src/lib/tlm_packet.c:788-815): buffer size (TLMG_EINVAL), magic and
// version, payload length, CRC (TLMG_EFORMAT). The manifest-side checks of
// that function (type/layer/id against the packet table, total length) are
// the caller's: tlmg_set_expert_packet checks type, layer and id.
extern "C" int tlmg_packet_parse(const void *packet, size_t len, int flags, tlmg_packet_info *out) {
    if (!packet || !out) return set_error(TLMG_EINVAL, "packet parse: NULL argument");
    if (flags & ~(TLMG_PKT_VERIFY_CRC | TLMG_PKT_HOST))
        return set_error(TLMG_EINVAL, "packet parse: unknown flags 0x%x", flags);
    if (len < kHdrBytes) return set_error(TLMG_EINVAL, "packet parse: buffer smaller than packet");
    const uint8_t *h = static_cast<const uint8_t *>(packet);
    tlmg_packet_info in;
    memset(&in, 0, sizeof in);
    const uint32_t magic = rd32(h + 0);
    in.type = rd16(h + 4);
    in.version = rd16(h + 6);
    in.layer = rd16(h + 8);
    in.n_items = rd16(h + 10);
    in.id = rd32(h + 12);
    in.dtype = rd32(h + 16);
    in.layout = rd32(h + 20);
    in.payload_len = rd64(h + 24);
    in.crc32c = rd32(h + 32);
    for (int m = 0; m < 3; m++) in.item_off[m] = rd32(h + 36 + 4 * m);
    const uint8_t *rsv = h + 48;
    if (magic != kMagic || in.version != kVersion)
        return set_error(TLMG_EFORMAT, "packet type %u layer %u id %u: bad magic/version", in.type, in.layer, in.id);
    if (in.payload_len > len - kHdrBytes)
        return set_error(TLMG_EFORMAT, "packet type %u layer %u id %u: length mismatch (payload %llu, buffer %zu)",
                         in.type, in.layer, in.id, (unsigned long long)in.payload_len, len);
    in.total_len = (kHdrBytes + in.payload_len + kAlignIO - 1) & ~(kAlignIO - 1);
    if (rsv[0] == kMixedMark) {
        in.mixed = 1;
        for (int m = 0; m < 3; m++) in.item_dt[m] = rsv[1 + m];
    } else if (rsv[0] == 0) {
        for (int m = 0; m < 3; m++) in.item_dt[m] = (int32_t)in.dtype;
    } else {
        return set_error(TLMG_EFORMAT, "packet type %u layer %u id %u: unknown header extension 0x%02x", in.type,
                         in.layer, in.id, rsv[0]);
    }
    if (flags & TLMG_PKT_VERIFY_CRC) {
        const uint32_t crc = in.payload_len ? tlmg_crc32c(0, h + kHdrBytes, (size_t)in.payload_len) : 0u;
        if (crc != in.crc32c)
            return set_error(TLMG_EFORMAT, "packet type %u layer %u id %u: CRC mismatch", in.type, in.layer, in.id);
    }
    *out = in;
    return TLMG_OK;
}

extern "C" int tlmg_set_expert_packet(tlmg_ctx *ctx, int layer, int expert, const void *packet, size_t len,
                                      int flags) {
    tlmg_packet_info in;
    int rc = tlmg_packet_parse(packet, len, flags, &in);
    if (rc) return rc;
    if (in.type != kTypeExpert || in.layer != (uint32_t)layer || in.id != (uint32_t)expert)
        return set_error(TLMG_EFORMAT,
                         "packet header (type %u layer %u id %u) does not match expert (type %u layer %d id %d)",
                         in.type, in.layer, in.id, kTypeExpert, layer, expert);
    if (in.n_items != 1) return set_error(TLMG_EUNSUP, "packet layer %d id %d: bundles are not supported", layer, expert);
    if (in.layout != 0)
        return set_error(TLMG_EUNSUP, "packet layer %d id %d: layout %u is not row-major plain", layer, expert,
                         in.layout);
    const uint8_t *payload = static_cast<const uint8_t *>(packet) + kHdrBytes;
    const uint64_t off[3] = { in.item_off[0], in.item_off[1], in.item_off[2] };
    if (flags & TLMG_PKT_HOST)
        return tlmg_set_expert_host(ctx, layer, expert, in.item_dt, payload, (size_t)in.payload_len, off);
    return tlmg_set_expert(ctx, layer, expert, in.item_dt, payload, (size_t)in.payload_len, off);
}
