// tlmg_cache.cu - HBM expert-slot cache with side-stream refill.
//
// Decisions (which expert goes into which slot, which slot is evicted, which
// router-lookahead hints are taken) are StorePolicy's, the reference store's
// rules (tlmg_store.h); this file moves the bytes. A slot's load is LOADING
// until its copy's event has completed (checked at every acquisition, as the
// reference's slot turns READY when its read completes).
//
// Ordering on the GPU: a load into a slot waits (on the copy stream) for the
// event recorded after the slot's last use on the compute stream; the
// compute stream waits for the event recorded after the load. Copies from
// pinned host memory run asynchronously to both streams.
#include <algorithm>

#include "tlmg_cache.cuh"
#include "tlmg_internal.h"
#include "tlmg_store.h"

namespace tlmg {

static size_t padded(size_t b) { return (b + 16 + 255) & ~size_t(255); }

void cache_release(ExpertCache &c) {
    if (c.copy_st) cudaStreamSynchronize(c.copy_st);
    for (cudaEvent_t e : c.loaded)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : c.used)
        if (e) cudaEventDestroy(e);
    if (c.pool) cudaFree(c.pool);
    if (c.copy_st) cudaStreamDestroy(c.copy_st);
    c = ExpertCache{};
}

int cache_init(ExpertCache &c, int n_layers, int E, int top_k, int n_slots, size_t slot_bytes) {
    cache_release(c);
    if (n_layers <= 0 || E <= 0 || n_slots <= 0 || slot_bytes == 0)
        return set_error(TLMG_EINVAL, "cache: %d layers, %d experts, %d slots of %zu bytes", n_layers, E, n_slots,
                         slot_bytes);
    c.slot_bytes = (slot_bytes + 255) & ~size_t(255);
    if (cudaMalloc(&c.pool, c.slot_bytes * (size_t)n_slots) != cudaSuccess) {
        cudaGetLastError();
        c = ExpertCache{};
        return set_error(TLMG_ENOMEM, "cache: %d slots of %zu bytes", n_slots, c.slot_bytes);
    }
    if (cudaStreamCreateWithFlags(&c.copy_st, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        cache_release(c);
        return set_error(TLMG_EIO, "cache: copy stream creation failed");
    }
    c.n_layers = n_layers;
    c.E = E;
    c.n_slots = n_slots;
    c.src.assign((size_t)n_layers * E, CacheSrc{});
    c.policy.init(n_layers * E, n_slots, top_k);
    c.held.clear();
    c.used_valid.assign(n_slots, 0);
    c.loaded.assign(n_slots, nullptr);
    c.used.assign(n_slots, nullptr);
    for (int s = 0; s < n_slots; s++)
        if (cudaEventCreateWithFlags(&c.loaded[s], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c.used[s], cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            cache_release(c);
            return set_error(TLMG_EIO, "cache: event creation failed");
        }
    c.on = true;
    return TLMG_OK;
}

int cache_register(ExpertCache &c, int layer, int e, const int32_t dt[3], const void *host, const uint64_t off[3],
                   const size_t bytes[3]) {
    if (!c.on) return set_error(TLMG_EINVAL, "cache: not enabled (tlmg_cache_enable)");
    const size_t need = padded(bytes[0]) + padded(bytes[1]) + padded(bytes[2]);
    if (need > c.slot_bytes)
        return set_error(TLMG_ERANGE, "cache: expert %d:%d needs %zu bytes, slots hold %zu", layer, e, need,
                         c.slot_bytes);
    const int key = layer * c.E + e;
    if (c.policy.where(key) >= 0)
        return set_error(TLMG_EBUSY, "cache: expert %d:%d is resident; register experts before their first use",
                         layer, e);
    CacheSrc &d = c.src[key];
    d.host = static_cast<const uint8_t *>(host);
    for (int m = 0; m < 3; m++) {
        d.off[m] = off[m];
        d.bytes[m] = bytes[m];
        d.dt[m] = dt[m];
    }
    d.ok = true;
    return TLMG_OK;
}

bool cache_has(const ExpertCache &c, int layer) {
    if (!c.on || layer < 0 || layer >= c.n_layers) return false;
    for (int e = 0; e < c.E; e++)
        if (c.src[(size_t)layer * c.E + e].ok) return true;
    return false;
}

static Slot slot_view(const ExpertCache &c, int s, const CacheSrc &d) {
    Slot v{};
    uint8_t *base = c.pool + (size_t)s * c.slot_bytes;
    size_t o = 0;
    for (int m = 0; m < 3; m++) {
        v.m[m] = base + o;
        v.dt[m] = d.dt[m];
        o += padded(d.bytes[m]);
    }
    v.ok = 1;
    return v;
}

// LOADING -> READY for every slot whose copy has completed.
static void reap(ExpertCache &c) {
    for (int s = 0; s < c.n_slots; s++) {
        if (c.policy.slot(s).state != StorePolicy::LOADING) continue;
        cudaError_t e = cudaEventQuery(c.loaded[s]);
        if (e == cudaSuccess) c.policy.load_done(s);
        else if (e != cudaErrorNotReady) cudaGetLastError();
    }
}

// Copy expert `key` into slot v on the copy stream, after the slot's last use.
static int load_slot(ExpertCache &c, int v, int key) {
    if (c.used_valid[v] && cudaStreamWaitEvent(c.copy_st, c.used[v], 0) != cudaSuccess)
        return cuda_fail(cudaGetLastError(), "cache: copy stream wait");
    const CacheSrc &d = c.src[key];
    const Slot view = slot_view(c, v, d);
    for (int m = 0; m < 3; m++) {
        cudaError_t e = cudaMemcpyAsync(const_cast<uint8_t *>(view.m[m]), d.host + d.off[m], d.bytes[m],
                                        cudaMemcpyHostToDevice, c.copy_st);
        if (e != cudaSuccess) return cuda_fail(e, "cache: expert copy");
        c.bytes_loaded += (int64_t)d.bytes[m];
    }
    if (cudaEventRecord(c.loaded[v], c.copy_st) != cudaSuccess)
        return cuda_fail(cudaGetLastError(), "cache: event record");
    return TLMG_OK;
}

int cache_acquire(ExpertCache &c, int layer, const int32_t *ids, int k, bool prefetch, cudaStream_t st, Slot *out) {
    if (!c.on) return set_error(TLMG_EINVAL, "cache: not enabled");
    if (layer < 0 || layer >= c.n_layers) return set_error(TLMG_ERANGE, "cache: layer %d", layer);
    if (k < 0 || k > 64) return set_error(TLMG_EINVAL, "cache: %d experts", k);
    int keys[64], slots[64], loads[64];
    for (int i = 0; i < k; i++) {
        if (ids[i] < 0 || ids[i] >= c.E || !c.src[(size_t)layer * c.E + ids[i]].ok)
            return set_error(TLMG_ENOTFOUND, "cache: layer %d expert %d is not registered", layer, ids[i]);
        keys[i] = layer * c.E + ids[i];
    }
    reap(c);
    if (prefetch) {
        int keys_out[64];
        const int n = c.policy.prefetch(keys, k, slots, keys_out);
        for (int i = 0; i < n; i++)
            if (int rc = load_slot(c, slots[i], keys_out[i])) return rc;
        return TLMG_OK;
    }
    const bool ok = c.policy.acquire(keys, k, slots, loads);
    for (int i = 0; i < k; i++)
        if (slots[i] >= 0) c.held.push_back(slots[i]);
    if (!ok) {
        for (int s : c.held) c.policy.release(s);
        c.held.clear();
        return set_error(TLMG_EBUSY, "cache: all %d slots are referenced or loading; it needs at least top_k slots",
                         c.n_slots);
    }
    for (int i = 0; i < k; i++)
        if (loads[i])
            if (int rc = load_slot(c, slots[i], keys[i])) return rc;
    for (int i = 0; i < k; i++) {
        if (cudaStreamWaitEvent(st, c.loaded[slots[i]], 0) != cudaSuccess)
            return cuda_fail(cudaGetLastError(), "cache: compute stream wait");
        if (out) out[i] = slot_view(c, slots[i], c.src[keys[i]]);
    }
    return TLMG_OK;
}

int cache_mark_used(ExpertCache &c, cudaStream_t st) {
    int rc = TLMG_OK;
    for (int s : c.held) {
        if (rc == TLMG_OK && cudaEventRecord(c.used[s], st) != cudaSuccess)
            rc = cuda_fail(cudaGetLastError(), "cache: event record");
        c.used_valid[s] = 1;
        c.policy.release(s);
    }
    c.held.clear();
    return rc;
}

void cache_tick(ExpertCache &c) {
    if (c.on) c.policy.tick();
}

}  // namespace tlmg

// ---------------------------------------------------------------------------
// The slot policy on its own (C ABI): for callers that manage their own slot
// memory, and for replaying a trace against the reference store.
struct tlmg_store {
    tlmg::StorePolicy p;
};

extern "C" {

int tlmg_store_open(int n_keys, int n_slots, int top_k, tlmg_store **out) {
    if (!out || n_keys <= 0 || n_slots <= 0) return tlmg::set_error(TLMG_EINVAL, "store_open: bad argument");
    tlmg_store *s = new tlmg_store();
    s->p.init(n_keys, n_slots, top_k);
    *out = s;
    return TLMG_OK;
}

void tlmg_store_close(tlmg_store *s) { delete s; }

int tlmg_store_acquire(tlmg_store *s, const int32_t *keys, int k, int32_t *slots, int32_t *loads) {
    if (!s || k < 0 || (k > 0 && (!keys || !slots || !loads)) || k > 1024)
        return tlmg::set_error(TLMG_EINVAL, "store_acquire: bad argument");
    for (int i = 0; i < k; i++)
        if (keys[i] < 0 || keys[i] >= (int)s->p.n_keys())
            return tlmg::set_error(TLMG_ENOTFOUND, "store_acquire: key %d out of range", keys[i]);
    return s->p.acquire(keys, k, slots, loads) ? TLMG_OK
                                                : tlmg::set_error(TLMG_EBUSY, "store: all %d slots are referenced, "
                                                                              "pinned or loading", s->p.n_slots());
}

int tlmg_store_prefetch(tlmg_store *s, const int32_t *keys, int k, int32_t *slots, int32_t *keys_out) {
    if (!s || k < 0 || (k > 0 && (!keys || !slots || !keys_out)) || k > 1024)
        return tlmg::set_error(TLMG_EINVAL, "store_prefetch: bad argument");
    for (int i = 0; i < k; i++)
        if (keys[i] < 0 || keys[i] >= (int)s->p.n_keys())
            return tlmg::set_error(TLMG_ENOTFOUND, "store_prefetch: key %d out of range", keys[i]);
    return s->p.prefetch(keys, k, slots, keys_out);
}

int tlmg_store_load_done(tlmg_store *s, int slot) {
    if (!s || slot < 0 || slot >= s->p.n_slots()) return tlmg::set_error(TLMG_EINVAL, "store_load_done: bad slot");
    s->p.load_done(slot);
    return TLMG_OK;
}

int tlmg_store_release(tlmg_store *s, int slot) {
    if (!s || slot >= s->p.n_slots()) return tlmg::set_error(TLMG_EINVAL, "store_release: bad slot");
    s->p.release(slot);
    return TLMG_OK;
}

int tlmg_store_tick(tlmg_store *s) {
    if (!s) return tlmg::set_error(TLMG_EINVAL, "store_tick: NULL store");
    s->p.tick();
    return TLMG_OK;
}

int tlmg_store_slot(const tlmg_store *s, int slot, int32_t out[4]) {
    if (!s || !out || slot < 0 || slot >= s->p.n_slots()) return tlmg::set_error(TLMG_EINVAL, "store_slot: bad slot");
    const tlmg::StorePolicy::SlotState &v = s->p.slot(slot);
    out[0] = v.state;
    out[1] = v.key;
    out[2] = v.refcount;
    out[3] = v.prefetched;
    return TLMG_OK;
}

int tlmg_store_stats(const tlmg_store *s, int64_t out[6]) {
    if (!s || !out) return tlmg::set_error(TLMG_EINVAL, "store_stats: bad argument");
    const tlmg::StorePolicy::Stats &st = s->p.stats();
    out[0] = st.hits;
    out[1] = st.misses;
    out[2] = st.prefetch_issued;
    out[3] = st.prefetch_used;
    out[4] = st.prefetch_dropped;
    out[5] = st.evictions;
    return TLMG_OK;
}

}  // extern "C"
