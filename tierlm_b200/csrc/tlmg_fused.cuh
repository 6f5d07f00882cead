// tlmg_fused.cuh - interface of the persistent expert-FFN kernel.
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

// Device scratch owned by a context for the persistent kernel.
struct FusedScratch {
    bool enabled = false;
};

inline int fused_init(FusedScratch &, const tlmg_geom &) { return TLMG_OK; }
inline void fused_release(FusedScratch &) {}
inline bool use_fused(const FusedScratch &f, const tlmg_geom &, bool) { return f.enabled; }
inline int launch_fused_ffn(FusedScratch &, const tlmg_geom &, const Slot *, const int32_t *, const float *,
                            const float *, float *, float *, const float *, const float *, cudaStream_t) {
    return TLMG_EUNSUP;
}

}  // namespace tlmg
