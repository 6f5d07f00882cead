/* tlm_kern_cuda.c - the CUDA tier of the reference's kernel table, as a
 * maintainer of the reference would add it next to tlm_kern_avx512.c
 * (fill function: src/lib/tlm_kern_avx512.c:671-689; table and function
 * types: src/lib/tlm_quant.h:146-171).
 *
 * TEST INFRASTRUCTURE ONLY here: compiled against the reference's headers
 * by oracle/Makefile into the tier check (ref_tier.c), which runs the
 * reference's own self-test and tier matrix on this table. Every entry
 * forwards to libtlmg's host adapters, which copy the operands to the GPU,
 * run the sm_100a kernel and copy the result back, so this tier is for
 * parity, not speed (the fast path is the whole MoE block on the device,
 * tlmg_moe_layer in include/tlmg.h, called in place of the reference's moe()).
 */
#define TLM_QUANT_INTERNAL 1
#include "tlm_quant.h"
#include "tlmg.h"

#define TLMG_MV(DT, NAME)                                                                         \
    static void NAME(const void *W, size_t rb, const void *a, float *y, int64_t n, int64_t rows) { \
        tlmg_qmv_host(DT, W, rb, a, y, n, rows);                                                  \
    }
#define TLMG_DOT(DT, NAME)                                                           \
    static float NAME(const void *w, const void *a, int64_t n, const float *aux) { \
        return tlmg_qdot_host(DT, w, a, n, aux);                                     \
    }
TLMG_MV(TLMG_DT_F32, mv_f32) TLMG_MV(TLMG_DT_F16, mv_f16) TLMG_MV(TLMG_DT_BF16, mv_bf16)
TLMG_MV(TLMG_DT_Q8_0, mv_q80) TLMG_MV(TLMG_DT_Q4_K, mv_q4k) TLMG_MV(TLMG_DT_Q5_K, mv_q5k)
TLMG_MV(TLMG_DT_Q6_K, mv_q6k) TLMG_MV(TLMG_DT_MXFP4, mv_mxfp4) TLMG_MV(TLMG_DT_Q8_K, mv_q8k)
TLMG_DOT(TLMG_DT_F32, dot_f32) TLMG_DOT(TLMG_DT_F16, dot_f16) TLMG_DOT(TLMG_DT_BF16, dot_bf16)
TLMG_DOT(TLMG_DT_Q8_0, dot_q80) TLMG_DOT(TLMG_DT_Q4_K, dot_q4k) TLMG_DOT(TLMG_DT_Q5_K, dot_q5k)
TLMG_DOT(TLMG_DT_Q6_K, dot_q6k) TLMG_DOT(TLMG_DT_MXFP4, dot_mxfp4) TLMG_DOT(TLMG_DT_Q8_K, dot_q8k)

/* Overwrites the entries the CUDA tier implements (every table dtype but
 * FP8E4M3_B128) and returns how many; 0 when no sm_100 device is present
 * (the tier is then absent, as an AVX-512 tier on a CPU without it). */
int tlm_kern_cuda_fill(tlm_quant_kernels *k) {
    if (tlmg_init(0) != TLMG_OK) return 0;
    k->dot[TLM_QK_F32] = dot_f32;     k->mv[TLM_QK_F32] = mv_f32;
    k->dot[TLM_QK_F16] = dot_f16;     k->mv[TLM_QK_F16] = mv_f16;
    k->dot[TLM_QK_BF16] = dot_bf16;   k->mv[TLM_QK_BF16] = mv_bf16;
    k->dot[TLM_QK_Q8_0] = dot_q80;    k->mv[TLM_QK_Q8_0] = mv_q80;
    k->dot[TLM_QK_Q4_K] = dot_q4k;    k->mv[TLM_QK_Q4_K] = mv_q4k;
    k->dot[TLM_QK_Q5_K] = dot_q5k;    k->mv[TLM_QK_Q5_K] = mv_q5k;
    k->dot[TLM_QK_Q6_K] = dot_q6k;    k->mv[TLM_QK_Q6_K] = mv_q6k;
    k->dot[TLM_QK_MXFP4] = dot_mxfp4; k->mv[TLM_QK_MXFP4] = mv_mxfp4;
    k->dot[TLM_QK_Q8_K] = dot_q8k;    k->mv[TLM_QK_Q8_K] = mv_q8k;
    return 9;
}
