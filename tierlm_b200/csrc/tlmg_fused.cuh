// tlmg_fused.cuh - the persistent expert-FFN kernel: one launch per token and
// layer does the router top-k, the activation quantisation, gate/up +
// SwiGLU, the re-quantisation of h and down + the rank-ordered combine, with
// every selected weight row streamed HBM -> shared memory by bulk copies.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <map>

#include "../../include/tlmg.h"

namespace tlmg {

// One routed expert in HBM: device addresses of gate, up, down and their
// dtypes; ok = 1 once uploaded.
struct Slot {
    const uint8_t *m[3];
    int32_t dt[3];
    int32_t ok;
};

// One chunk of a CTA's work: contiguous rows of one selected expert's
// matrices that one shared-memory stage holds. Phase A: `nrows` (gate, up)
// row pairs of rank `rank` starting at row `row0`, two copies (gate at
// dst[0], up at dst[1]). Phase B: `nrows` rows of rank `rank`'s down matrix
// starting at row `row0`, one copy. Offsets are relative to each matrix's
// base, so one plan serves every choice of experts of the same dtypes.
struct ChunkDesc {
    uint8_t phase, rank;
    uint16_t nrows;
    uint32_t row0;
    uint32_t tx;          // bytes the chunk's copies deliver
    uint32_t lo[2];       // first copied byte (16-aligned) inside the matrix
    uint32_t size[2];     // copy sizes (multiples of 16)
    uint16_t dst[2];      // stage offset of each copy (phase B: stride between ranks)
    uint16_t roff[2];     // offset of row0's first byte inside its copy
    uint32_t pad;
};

// Host-built work plan for one dtype signature: per CTA, the number of
// phase A / phase B chunks and the chunks themselves.
constexpr int FUSED_MAXCH = 48;
struct FusedPlanKey {
    int dt_gu, dt_dn;
    bool operator<(const FusedPlanKey &o) const { return dt_gu != o.dt_gu ? dt_gu < o.dt_gu : dt_dn < o.dt_dn; }
};

// Per-context state of the persistent kernels (k_fused_ffn: a static work
// split with a grid barrier per token; k_ffn_one: one token per launch).
struct FusedScratch {
    bool enabled = false;          // usable on this device / geometry
    uint32_t *bar = nullptr;       // device: [2] sticky error, [4..11] four 64-bit barrier arrival words
    uint32_t *err_host = nullptr;  // mapped pinned word: error bits set by the kernel
    uint32_t *err_dev = nullptr;   // its device alias
    int nsm = 0;                   // CTAs = SMs (one persistent CTA per SM)
    int nsA = 0, nsB = 0;          // gate/up and down stages in shared memory
    uint64_t rounds = 0;           // grid-barrier rounds (tokens) launched since the barrier words were reset
    uint64_t launches = 0;         // launches since the barrier words were reset
    // Graph capture: every captured launch restarts the barrier words from
    // zero (a replay cannot carry host counts), and the first launch after
    // a capture or a replay restarts them too (bar_stale).
    bool graph_mode = false;
    bool bar_stale = false;
    // one-token launches by the single-token kernel (k_ffn_one,
    // tlmg_set_fused mode 4); grid words [2] count, generation
    bool single = false;
    uint32_t *obar = nullptr;
    // per-token global scratch of a launch, for up to tok_cap tokens
    int tok_cap = 0;
    uint8_t *xq = nullptr;         // [tok_cap][quantised x]
    float *hbuf = nullptr;         // [tok_cap][k * de] SwiGLU rows
    float *eo = nullptr;           // [tok_cap][k * D] expert outputs
    uint32_t *ocnt = nullptr;      // [tok_cap][D / 64] expert outputs written per 64-row group (zero between launches)
    int D = 0, de = 0, k = 0;
    size_t smem = 0;               // dynamic shared memory per CTA
    size_t smem_limit = 0;
    std::map<FusedPlanKey, void *> plans;   // device: int2 counts[nsm] | ChunkDesc [nsm][FUSED_MAXCH]
};

// Error bits the kernel reports through err_host.
enum : uint32_t { FUSED_ERR_BARRIER = 1u, FUSED_ERR_COPY = 2u, FUSED_ERR_PLAN = 4u };

// Everything one launch needs. The launch processes n_tok independent
// tokens; token t uses layer (layer0 + t) % n_layers, input x + t*D, router
// logits + t*E and writes ffn + t*D (and ids_out / w_out + t*k when given).
struct FusedArgs {
    const void *plan;              // FusedScratch::plans entry for the layers' dtypes
    const Slot *slots_all;         // [n_layers][E] slot tables, contiguous
    const uint8_t *mask_all;       // [n_layers][E] (1 = pruned) or NULL
    const float *bias_all;         // [n_layers][E] router bias or NULL
    int layer0, n_layers, n_tok;
    const float *x;                // [n_tok][D] normalised inputs
    const float *logits;           // [n_tok][E]
    float *ffn;                    // [n_tok][D] out
    float *h;                      // n_tok == 1 only: [D] in/out (h += ffn) or NULL
    const float *s_out;            // n_tok == 1 only: [D] shared-expert output or NULL
    const float *sgate;            // n_tok == 1 only: shared-expert gate (device scalar) or NULL
    int32_t *ids_out;              // [n_tok][k] or NULL
    float *w_out;                  // [n_tok][k] or NULL
    // filled by launch_fused_ffn from the FusedScratch:
    uint8_t *xq;                   // [n_tok] quantised inputs
    float *hbuf;                   // [n_tok][k * de] SwiGLU rows (cross-CTA exchange)
    float *eo;                     // [n_tok][k * D] expert outputs (cross-CTA combine)
    uint32_t *ocnt;                // [n_tok][D / 64] output group counts
    int D, de, E, k, router;
    float routed_scale;
    int dt_gu, dt_dn;              // dtype of every gate/up and every down matrix of the layers
    uint64_t *trace;               // NULL, or [gridDim][FUSED_TRACE_POINTS]
    uint64_t bar_base;             // grid-barrier rounds before this launch
    uint64_t xbar_target;          // input-quantisation count that completes this launch's
};

// Per CTA when tracing: the stamps listed at tlmg_trace (include/tlmg.h).
constexpr int FUSED_TRACE_POINTS = TLMG_TRACE_POINTS;

int fused_init(FusedScratch &f, const tlmg_geom &g);
void fused_release(FusedScratch &f);
// The work plan for a layer whose gate/up matrices are all dt_gu and down
// matrices all dt_dn, or NULL when the kernel cannot serve it.
const void *fused_plan(FusedScratch &f, const tlmg_geom &g, int dt_gu, int dt_dn);
int launch_fused_ffn(FusedScratch &f, const FusedArgs &a, cudaStream_t st);
// Error bits raised since the last call (clears them and resets the
// barrier state). Call after the stream has been synchronised.
uint32_t fused_take_error(FusedScratch &f);

}  // namespace tlmg
