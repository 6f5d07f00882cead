// tlmg_mma.cuh - grouped expert kernels on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, accumulators in TMEM) for batched decode and the
// expert-parallel owner. Exact: every K-quant sub-block's integer dot is its
// own int32 MMA accumulator, so the per-block integer sums and the fmaf
// chain are the reference's (src/lib/tlm_quant.c:253-296, :392-420).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "tlmg_fused.cuh"   // Slot

namespace tlmg {

// True when the tensor-core kernels serve a gate/up (down) matrix of this
// dtype and shape.
bool mma_gateup_supported(int dt, int D, int de);
bool mma_down_supported(int dt, int D, int de);

// grp: the expert grouping of the batched path (offsets [E + 1], active
// experts [E], count, pairs). Pair q's quantised input (swizzled Q8_K
// vector) at x + (q / xdiv) * xstride. gout[q][de] / uout[q][de] receive
// the gate / up row dots (the caller forms SiLU(gate) * up).
// err: device word; bit 0 is set when a tensor-core wait expired. The
// launchers queue one kernel each and leave launch counting to the caller.
int launch_mma_gateup(int dt, const Slot *slots, const int32_t *grp, const uint8_t *x, size_t xstride, int xdiv,
                      int D, int de, int E, int64_t max_items, bool wide, float *gout, float *uout, uint32_t *err,
                      cudaStream_t st);
// hq: quantised h per pair (swizzled Q8_K vectors of de); eo[q][D].
// wide: the experts average many tokens (prefill) - 32 tokens per pass
// instead of 8.
int launch_mma_down(int dt, const Slot *slots, const int32_t *grp, const uint8_t *hq, int D, int de, int E,
                    int64_t max_items, bool wide, float *eo, uint32_t *err, cudaStream_t st);

}  // namespace tlmg
