// tlmg_batch.cuh - batched expert FFN: n tokens through one MoE layer's
// routed experts (batched decode). Every expert selected by any token is
// read from HBM once per call and applied to all of its tokens; each
// (token, expert) pair's results are bit-identical to the single-token path.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "tlmg_fused.cuh"   // Slot

namespace tlmg {

// Device scratch of one batched call, for up to `cap` tokens.
struct BatchScratch {
    int cap = 0;
    uint8_t *xq = nullptr;      // [cap] quantised inputs (swizzled Q8_K vectors)
    int32_t *ids = nullptr;     // [cap][k]
    float *w = nullptr;         // [cap][k]
    int32_t *grp = nullptr;     // expert offsets [E + 1], active experts [E], count [1], pairs [cap * k]
    float *hbuf = nullptr;      // [cap * k][de] SwiGLU rows per (token, rank) pair
    uint8_t *hq = nullptr;      // [cap * k] quantised h per pair
    float *eo = nullptr;        // [cap * k][D] expert outputs per pair
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

}  // namespace tlmg
