// tlmg_fused.cuh - the persistent expert-FFN kernel: one launch per token and
// layer does the router top-k, the activation quantisation, gate/up +
// SwiGLU, the re-quantisation of h and down + the rank-ordered combine, with
// every selected weight row streamed HBM -> shared memory by bulk copies.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/tlmg.h"

namespace tlmg {

// One routed expert in HBM: device addresses of gate, up, down and their
// dtypes; ok = 1 once uploaded.
struct Slot {
    const uint8_t *m[3];
    int32_t dt[3];
    int32_t ok;
};

// Per-context state of the persistent kernel.
struct FusedScratch {
    bool enabled = false;          // usable on this device / geometry
    uint32_t *bar = nullptr;       // device: [0] arrivals, [1] generation
    uint32_t *err_host = nullptr;  // mapped pinned word: error bits set by the kernel
    uint32_t *err_dev = nullptr;   // its device alias
    int nsm = 0;                   // CTAs = SMs (one persistent CTA per SM)
    int slot_bytes = 0, nslot = 0; // shared-memory stage ring
    size_t smem = 0;               // dynamic shared memory per CTA
};

// Error bits the kernel reports through err_host.
enum : uint32_t { FUSED_ERR_BARRIER = 1u, FUSED_ERR_COPY = 2u, FUSED_ERR_PLAN = 4u };

// Everything one launch needs.
struct FusedArgs {
    const Slot *slots;             // [E] for the layer
    const float *logits;           // [E]
    const uint8_t *mask;           // [E] or NULL
    const float *bias;             // [E] or NULL
    const float *x;                // [D] normalised input
    float *hbuf;                   // [k * de] SwiGLU rows (cross-CTA exchange)
    float *ffn;                    // [D] out
    float *h;                      // [D] in/out (h += ffn) or NULL
    const float *s_out;            // [D] shared-expert output or NULL
    const float *sgate;            // shared-expert gate (device scalar) or NULL
    int32_t *ids_out;              // [k]
    float *w_out;                  // [k]
    int D, de, E, k, router;
    float routed_scale;
    uint32_t x_kinds;              // bit 0: Q8_K input needed, bit 1: Q8_0 input needed
    uint64_t *trace;               // NULL, or [gridDim][FUSED_TRACE_POINTS] %globaltimer stamps
};

// Phase boundaries stamped per CTA when tracing: start, routed, planned,
// phase A done, grid barrier passed, h quantised, end.
constexpr int FUSED_TRACE_POINTS = 8;

int fused_init(FusedScratch &f, const tlmg_geom &g);
void fused_release(FusedScratch &f);
// Can the kernel serve a layer whose experts use these dtypes? `dts`: the
// distinct gate/up/down dtypes present (any order), n of them.
bool fused_supports(const FusedScratch &f, const tlmg_geom &g, const int *gate_up_dts, int n_gu,
                    const int *down_dts, int n_dn);
int launch_fused_ffn(FusedScratch &f, const FusedArgs &a, cudaStream_t st);
// Error bits raised since the last call (clears them). Call after the
// stream has been synchronised.
uint32_t fused_take_error(FusedScratch &f);

}  // namespace tlmg
