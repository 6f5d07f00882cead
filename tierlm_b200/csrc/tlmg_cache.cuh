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
#include "tlmg_store.h"

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
    StorePolicy policy;                     // which expert in which slot (the reference store's rules)
    std::vector<int> held;                  // slots referenced by the acquisition in progress
    std::vector<cudaEvent_t> loaded;        // [slot] recorded on copy_st after its last load
    std::vector<cudaEvent_t> used;          // [slot] recorded on the compute stream after its last use
    std::vector<char> used_valid;
    int64_t bytes_loaded = 0;
};

int cache_init(ExpertCache &c, int n_layers, int E, int top_k, int n_slots, size_t slot_bytes);
void cache_release(ExpertCache &c);
// Records a host-resident expert (no copy).
int cache_register(ExpertCache &c, int layer, int e, const int32_t dt[3], const void *host, const uint64_t off[3],
                   const size_t bytes[3]);
bool cache_has(const ExpertCache &c, int layer);
// Makes experts ids[0..k) of `layer` resident and returns their slots'
// matrix pointers in out[0..k). prefetch = false: an acquisition for
// work queued next on `st` (st waits for the copies; the slots stay
// referenced until cache_mark_used); prefetch = true: router-lookahead
// hints, copies started only (out may be NULL), subject to the hint rules.
// TLMG_EBUSY when no slot is free of references and loads.
int cache_acquire(ExpertCache &c, int layer, const int32_t *ids, int k, bool prefetch, cudaStream_t st, Slot *out);
// After the launches that read the acquired slots are queued on st: their
// use is recorded and the references dropped.
int cache_mark_used(ExpertCache &c, cudaStream_t st);
// One model step has passed (the frequencies' decay clock).
void cache_tick(ExpertCache &c);

}  // namespace tlmg
