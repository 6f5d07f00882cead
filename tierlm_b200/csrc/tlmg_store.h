// tlmg_store.h - the slot policy of the HBM expert cache: which expert goes
// into which slot, which slot is evicted, which hints are taken. Host code
// only (no CUDA): the cache in tlmg_cache.cu runs the copies and events,
// this decides.
//
// The rules are the reference expert store's (src/lib/tlm_store.c):
//  - slot lifecycle FREE -> LOADING -> READY (:123-190); a LOADING slot is
//    never a victim, a referenced or pinned slot neither;
//  - every selection counts: an acquisition adds 1 to each selected
//    expert's frequency, and tlmg_store_tick halves every frequency every
//    16 ticks (:34, :590-604, :738-744);
//  - victims: any FREE slot first, else the READY slot with the lowest
//    (frequency, last use) over all layers, ties to the lowest slot
//    (pick_victim, :191-216);
//  - an acquisition references all its hits before any miss picks a victim,
//    so a miss never evicts an expert the same step needs (:605-636);
//  - hints (router lookahead) take only FREE slots or READY slots whose
//    expert has frequency 0, are dropped while more than 4 demand loads are
//    in flight, are bounded in flight by min(16, slots - pinned - reserve)
//    with reserve = max(1, top_k), load with the lowest recency (last use
//    0) and count as used once a demand acquisition takes them (:694-719,
//    :229-246).
// The store has no warm pins here (tlm_store_warm is not ported): n_pinned
// stays 0.
#pragma once
#include <cstdint>
#include <vector>

namespace tlmg {

class StorePolicy {
public:
    enum State { FREE = 0, LOADING = 1, READY = 2 };
    static constexpr int DECAY_PERIOD = 16;
    static constexpr int PF_DEMAND_BACKLOG = 4;
    static constexpr int PF_MAX_INFLIGHT = 16;

    struct SlotState {
        int state = FREE;
        int key = -1;          // expert key (layer * E + id), -1 = none
        int refcount = 0;
        int pinned = 0;
        int prefetched = 0;    // loaded by a hint, not yet taken by a demand acquisition
        int demand = 0;        // an in-flight load that a demand acquisition waits for
        uint64_t last_use = 0;
    };
    struct Stats {
        int64_t hits = 0, misses = 0, prefetch_issued = 0, prefetch_used = 0, prefetch_dropped = 0, evictions = 0;
    };

    void init(int n_keys, int n_slots, int top_k) {
        slots_.assign(n_slots, SlotState{});
        where_.assign(n_keys, -1);
        freq_.assign(n_keys, 0);
        reserve_ = top_k > 0 ? (top_k > 1024 ? 1024 : top_k) : 1;
        clock_ = ticks_ = 0;
        loading_ = demand_loading_ = pf_loading_ = n_pinned_ = 0;
        st_ = Stats{};
    }
    int n_slots() const { return (int)slots_.size(); }
    size_t n_keys() const { return where_.size(); }
    int where(int key) const { return where_[key]; }
    const SlotState &slot(int s) const { return slots_[s]; }
    uint32_t freq(int key) const { return freq_[key]; }
    const Stats &stats() const { return st_; }

    // Demand acquisition of keys[0..k): out_slot[i] = the slot holding (or
    // now loading) keys[i], referenced; load[i] = 1 where this call started
    // the load (the caller copies the expert in, then calls load_done).
    // A slot of -1: no victim (every slot referenced, pinned or loading);
    // the function then returns false (the reference's TLM_EBUSY).
    bool acquire(const int *keys, int k, int *out_slot, int *load) {
        const uint64_t stamp = ++clock_;
        bool ok = true;
        for (int i = 0; i < k; i++) {
            out_slot[i] = -1;
            load[i] = 0;
            if (freq_[keys[i]] < UINT32_MAX) freq_[keys[i]]++;
        }
        for (int i = 0; i < k; i++) {   // pass 1: every hit before any miss picks a victim
            const int s = where_[keys[i]];
            if (s < 0) continue;
            take_ref(s, stamp);
            out_slot[i] = s;
            st_.hits++;
        }
        for (int i = 0; i < k; i++) {   // pass 2: misses
            if (out_slot[i] >= 0) continue;
            const int s0 = where_[keys[i]];
            if (s0 >= 0) {              // a repeated key loaded earlier in this pass
                take_ref(s0, stamp);
                out_slot[i] = s0;
                st_.hits++;
                continue;
            }
            const int v = pick_victim(false);
            if (v < 0) {
                ok = false;
                continue;
            }
            st_.misses++;
            start_load(v, keys[i], false);
            out_slot[i] = v;
            load[i] = 1;
        }
        return ok;
    }
    // Router-lookahead hints: returns how many loads were started; their
    // slots go to out_slot / out_key (the caller copies, then load_done).
    int prefetch(const int *keys, int k, int *out_slot, int *out_key) {
        int cap = n_slots() - n_pinned_ - reserve_;
        if (cap > PF_MAX_INFLIGHT) cap = PF_MAX_INFLIGHT;
        int n = 0;
        for (int i = 0; i < k; i++) {
            if (where_[keys[i]] >= 0) continue;   // resident or already loading
            if (demand_loading_ > PF_DEMAND_BACKLOG || pf_loading_ >= cap) {
                st_.prefetch_dropped++;
                continue;
            }
            const int v = pick_victim(true);
            if (v < 0) {
                st_.prefetch_dropped++;
                continue;
            }
            start_load(v, keys[i], true);
            st_.prefetch_issued++;
            out_slot[n] = v;
            out_key[n] = keys[i];
            n++;
        }
        return n;
    }
    // The load into slot s has completed (the copy is in the slot).
    void load_done(int s) {
        SlotState &sl = slots_[s];
        if (sl.state != LOADING) return;
        sl.state = READY;
        loading_--;
        if (sl.demand) demand_loading_--;
        else pf_loading_--;
    }
    void release(int s) {
        if (s >= 0 && slots_[s].refcount > 0) slots_[s].refcount--;
    }
    void tick() {
        if (++ticks_ % DECAY_PERIOD == 0)
            for (uint32_t &f : freq_) f >>= 1;
    }
    // The key slot s held before the last start_load evicted it (or -1).
    int evicted_key() const { return evicted_; }

private:
    std::vector<SlotState> slots_;
    std::vector<int> where_;
    std::vector<uint32_t> freq_;
    int reserve_ = 1, loading_ = 0, demand_loading_ = 0, pf_loading_ = 0, n_pinned_ = 0, evicted_ = -1;
    uint64_t clock_ = 0, ticks_ = 0;
    Stats st_;

    int pick_victim(bool hint) const {
        int best = -1;
        uint32_t bf = 0;
        uint64_t bl = 0;
        for (int i = 0; i < n_slots(); i++) {
            const SlotState &sl = slots_[i];
            if (sl.refcount > 0 || sl.pinned) continue;
            if (sl.state == FREE) return i;
            if (sl.state != READY) continue;
            const uint32_t f = freq_[sl.key];
            if (hint && f > 0) continue;
            if (best < 0 || f < bf || (f == bf && sl.last_use < bl)) {
                best = i;
                bf = f;
                bl = sl.last_use;
            }
        }
        return best;
    }
    void start_load(int v, int key, bool hint) {
        SlotState &sl = slots_[v];
        evicted_ = -1;
        if (sl.state == READY && sl.key >= 0) {
            where_[sl.key] = -1;
            evicted_ = sl.key;
            st_.evictions++;
        }
        loading_++;
        sl.state = LOADING;
        sl.key = key;
        where_[key] = v;
        sl.refcount = hint ? 0 : 1;
        sl.prefetched = hint;
        sl.demand = !hint;
        if (sl.demand) demand_loading_++;
        else pf_loading_++;
        sl.last_use = hint ? 0 : clock_;
    }
    void take_ref(int v, uint64_t stamp) {
        SlotState &sl = slots_[v];
        sl.refcount++;
        sl.last_use = stamp;
        if (sl.prefetched) {
            sl.prefetched = 0;
            st_.prefetch_used++;
        }
        if (sl.state == LOADING && !sl.demand) {   // a hint became demand
            sl.demand = 1;
            pf_loading_--;
            demand_loading_++;
        }
    }
};

}  // namespace tlmg
