// tlmg_cache.cuh - HBM expert-slot cache (the reference's expert store,
// src/lib/tlm_store.c:586-719, with router-lookahead prefetch,
// src/lib/tlm_model.c:844-877, rebuilt for a GPU): experts live in pinned
// host memory; a fixed pool of HBM slots holds the recently used ones.
// Misses are copied host -> HBM on a side stream; the compute stream waits
// for exactly the copies it needs (events), and a slot is only reloaded
// after the compute stream has finished with it.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>
#include <cuda_runtime.h>

#include "tlmg_fused.cuh"   // Slot

namespace tlmg {

struct CacheSrc {
    const uint8_t *host = nullptr;   // packet payload (pinned for asynchronous copies)
    uint64_t off[3] = { 0, 0, 0 };   // gate / up / down inside the payload
    size_t bytes[3] = { 0, 0, 0 };
    int32_t dt[3] = { 0, 0, 0 };
    bool ok = false;
};

struct ExpertCache {
    bool on = false;
    int n_layers = 0, E = 0, n_slots = 0;
    size_t slot_bytes = 0;
    uint8_t *pool = nullptr;                // [n_slots][slot_bytes] in HBM
    cudaStream_t copy_st = nullptr;
    std::vector<CacheSrc> src;              // [layer * E + e]
    std::vector<int> where;                 // [layer * E + e] -> slot, or -1
    std::vector<int> owner;                 // [slot] -> key, or -1
    std::vector<uint64_t> stamp;            // [slot] last acquisition (LRU)
    std::vector<uint64_t> pinned;           // [slot] acquisition that may not evict it
    std::vector<char> fresh;                // [slot] loaded by a prefetch and not used since
    std::vector<cudaEvent_t> loaded;        // [slot] recorded on copy_st after its last load
    std::vector<cudaEvent_t> used;          // [slot] recorded on the compute stream after its last use
    std::vector<char> used_valid;
    uint64_t clock = 0;
    int64_t hits = 0, misses = 0, prefetched = 0, prefetch_hits = 0, evictions = 0, bytes_loaded = 0;
};

int cache_init(ExpertCache &c, int n_layers, int E, int n_slots, size_t slot_bytes);
void cache_release(ExpertCache &c);
// Records a host-resident expert (no copy).
int cache_register(ExpertCache &c, int layer, int e, const int32_t dt[3], const void *host, const uint64_t off[3],
                   const size_t bytes[3]);
bool cache_has(const ExpertCache &c, int layer);
// Makes experts ids[0..k) of `layer` resident and returns their slots'
// matrix pointers in out[0..k). prefetch = false: an acquisition for
// work queued next on `st` (st waits for the copies; the slots cannot be
// evicted by this call); prefetch = true: starts the copies only (out may
// be NULL). TLMG_EBUSY when every slot is pinned by this acquisition.
int cache_acquire(ExpertCache &c, int layer, const int32_t *ids, int k, bool prefetch, cudaStream_t st, Slot *out);
// After the launches that read the acquired slots are queued on st.
int cache_mark_used(ExpertCache &c, int layer, const int32_t *ids, int k, cudaStream_t st);

}  // namespace tlmg
