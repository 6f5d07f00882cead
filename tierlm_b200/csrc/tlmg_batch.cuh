// tlmg_batch.cuh - batched expert FFN: n tokens through one MoE layer's
// routed experts (batched decode). Every expert selected by any token is
// read from HBM once per call and applied to all of its tokens; each
// (token, expert) pair's results are bit-identical to the single-token path.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "tlmg_fused.cuh"   // Slot

namespace tlmg {

constexpr int EP_MAX_RANKS = 64;   // expert-parallel GPUs per dispatch

// Device scratch of one batched call, for up to `cap` tokens.
struct BatchScratch {
    int cap = 0;                // tokens
    int64_t cap_pairs = 0;      // (token, expert) pairs or received records
    int cap_e = 0;              // experts
    int kmode = 2;              // gate/up kernels: 2 tensor cores, 1 tiled CUDA cores, 0 warp per row tile
                                // (each falls back to the next lower one where it does not apply)
    int kmode_dn = 2;           // the same for the down projection
    uint8_t *xq = nullptr;      // [cap] quantised inputs (swizzled Q8_K vectors)
    int32_t *ids = nullptr;     // [cap][k]
    float *w = nullptr;         // [cap][k]
    int32_t *grp = nullptr;     // expert offsets [E + 1], active experts [E], count [1], pairs [cap * k]
    float *hbuf = nullptr;      // [cap * k][de] SwiGLU rows per (token, rank) pair (tensor-core path: gate dots)
    float *ubuf = nullptr;      // [cap * k][de] up dots of the tensor-core path
    uint8_t *hq = nullptr;      // [cap * k] quantised h per pair
    float *eo = nullptr;        // [cap * k][D] expert outputs per pair
    int32_t *cnt = nullptr;     // pinned host [EP_MAX_RANKS + 2]: dispatch record counts, the count of
                                // received records naming an expert outside the owner's range, and
                                // the tensor-core kernels' error bits
};

struct BatchArgs {
    const Slot *slots;          // [E] the layer's expert slots
    const uint8_t *mask;        // [E] 1 = pruned, or NULL
    const float *bias;          // [E] router bias, or NULL
    int n, D, de, E, k, router;
    float routed_scale;
    int dt_gu, dt_dn;           // dtype of every gate/up and every down matrix of the layer
    const float *x;             // [n][D]
    const float *logits;        // [n][E]
    float *ffn;                 // [n][D] out
    int32_t *ids_out;           // [n][k] or NULL
    float *w_out;               // [n][k] or NULL
};

// True when the batched kernels serve these dtypes and shapes.
bool batch_supported(int dt_gu, int dt_dn, int D, int de, int E, int k);
int batch_reserve(BatchScratch &s, int n, int D, int de, int E, int k);
void batch_release(BatchScratch &s);
// Queues the whole batched call on `st` (no host synchronisation).
int launch_batch(BatchScratch &s, const BatchArgs &a, cudaStream_t st);

// Expert parallelism over nr GPUs: expert e is owned by GPU floor(e * nr / E).
// A dispatch record is { int32 expert id, 12 zero bytes, the token's
// quantised input (swizzled Q8_K vector) }.
size_t ep_record_bytes(int D);
// Home GPU: quantise + route a.n tokens, write one record per (token, rank)
// pair into `send` grouped by owner (ascending pair order inside an owner),
// perm[t * k + r] = the pair's record index, w[t * k + r] its weight,
// counts[d] = records for owner d (waits for the stream).
int ep_dispatch(BatchScratch &s, const BatchArgs &a, int nr, uint8_t *send, int32_t *perm, float *w, int64_t *counts,
                cudaStream_t st);
// Owner GPU of experts [lo, hi): n_rec received records -> eo [n_rec][D],
// one row per record (NaN rows for records outside [lo, hi), counted for
// batch_take_error).
int ep_experts(BatchScratch &s, const Slot *slots, int dt_gu, int dt_dn, int D, int de, int E, int lo, int hi,
               int64_t n_rec, const uint8_t *recv, float *eo, cudaStream_t st);
// TLMG_EINVAL (and a reset) once records outside an owner's range were seen;
// read after the stream has been synchronised.
int batch_take_error(BatchScratch &s);
// Home GPU: ffn[t] = sum_r w[t * k + r] * back[perm[t * k + r]] in ascending r.
int ep_combine(int n, int D, int k, const float *back, const int32_t *perm, const float *w, float *ffn,
               cudaStream_t st);

// Expert parallelism over peer memory (tlmg_ep.cu): one allocation per rank,
// mapped by every peer: record regions [nr][cap][rb], record counts
// [EPP_SLOTS], output-row regions [nr][cap][D] f32, barrier flags
// [2][EPP_SLOTS]; cap = (token, rank) pairs a home may send one owner.
constexpr int EPP_SLOTS = 8;
struct EpP2P {
    int me = 0, nr = 1, cap = 0, max_tok = 0;
    size_t rb = 0, off_rcnt = 0, off_back = 0, off_flags = 0, bytes = 0;
    uint8_t *base = nullptr;             // this rank's allocation
    uint8_t *peer[EPP_SLOTS] = {};       // every rank's allocation, mapped here (peer[me] = base)
    bool opened[EPP_SLOTS] = {};         // peer[r] is an IPC mapping to close
    int32_t *cnt = nullptr;              // [EPP_SLOTS] this call's records per owner
    int32_t *perm = nullptr;             // [max_tok * k] pair -> record index in owner order
    int32_t *slot_of = nullptr;          // [max_tok * k] pair -> its output row's index in the row regions
    float *eo = nullptr;                 // [nr * cap][D] this GPU's expert output rows
    uint32_t epoch = 0;                  // layer calls since the flags were zeroed
    uint32_t *err_host = nullptr, *err_dev = nullptr;   // a barrier that gave up
};
int epp_alloc(EpP2P &e, int me, int nr, int max_tok, int D, int k);
void epp_release(EpP2P &e);
// Launchers of tlmg_ep.cu's kernels (stream-ordered, no host wait).
void epp_send(const EpP2P &e, const int32_t *ids, int np, int k, int E, const uint8_t *xq, uint32_t qx,
              cudaStream_t st);
void epp_return(const EpP2P &e, int D, cudaStream_t st);
void epp_barrier(const EpP2P &e, int which, cudaStream_t st);
// One layer call: dispatch, barrier, expert stage, return, barrier, combine.
// Every rank of the exchange makes the same calls in the same order, n = 0
// included; a barrier that gave up shows at epp_take_error.
int epp_layer(BatchScratch &s, EpP2P &e, const BatchArgs &a, int lo, int hi, cudaStream_t st);
// TLMG_EIO once a barrier gave up (the exchange is then unusable), else the
// batched kernels' own errors; read after the stream has been synchronised.
int epp_take_error(BatchScratch &s, EpP2P &e);

}  // namespace tlmg
