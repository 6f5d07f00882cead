/* ref_moe_cpu.c - drives the REFERENCE's own CPU kernels for the expert FFN.
 *
 * TEST / BASELINE INFRASTRUCTURE ONLY. oracle/Makefile links this file with
 * the reference's unmodified sources (src/lib/tlm_quant.c, tlm_kern_avx2.c,
 * tlm_kern_avx512.c, tlm_platform.c, tlm_pool.c) into oracle/_ref/. Only
 * tests/ (golden vectors) and bench.py's CPU baseline load it.
 *
 * tlmref_expert_ffn() repeats the orchestration of the reference's
 * run_batch() + combine (src/lib/tlm_model.c:900-938, :1029-1036): the Q8_K
 * activation is quantised once, gate/up of every selected expert run as one
 * tlm_pool_for pass over output rows (grain 16, src/lib/tlm_model.c:44 and
 * :205-222), SiLU(g)*u is re-quantised per expert on the caller, down runs
 * as a second pool pass, and the outputs are combined in rank order.
 */
#define _GNU_SOURCE 1
#include "tlm_platform.h"
#include "tlm_pool.h"
#include "tlm_quant.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define REF_MAX_K 64
#define REF_ROW_GRAIN 16
#define REF_SERIAL_WORK 32768

static tlm_pool *g_pool;

int tlmref_open(int nthreads) {
    tlm_quant_init();
    if (g_pool) tlm_pool_free(g_pool);
    g_pool = tlm_pool_new(nthreads, 1);
    return g_pool ? 0 : -1;
}

int tlmref_threads(void) { return g_pool ? tlm_pool_size(g_pool) : 1; }
const char *tlmref_tier(void) { return tlm_quant_tier(); }
const char *tlmref_cpu_model(void) { return tlm_cpu()->model_name; }
int tlmref_physical_cores(void) { return tlm_cpu()->physical_cores; }

typedef struct {
    tlm_dtype      dt;
    const uint8_t *W;
    size_t         rb;
    const void    *act;
    float         *y;
    int64_t        n, rows;
} seg_t;

typedef struct {
    seg_t   seg[2 * REF_MAX_K];
    int64_t start[2 * REF_MAX_K + 1];
    int     nseg;
    int64_t work;
} job_t;

static void job_add(job_t *j, tlm_dtype dt, const uint8_t *W, int64_t rows, int64_t cols,
                    const void *act, float *y) {
    if (j->nseg == 0) j->start[0] = 0;
    seg_t *s = &j->seg[j->nseg];
    s->dt = dt;
    s->W = W;
    s->rb = tlm_row_bytes(dt, cols);
    s->act = act;
    s->y = y;
    s->n = cols;
    s->rows = rows;
    j->start[j->nseg + 1] = j->start[j->nseg] + rows;
    j->work += rows * cols;
    j->nseg++;
}

static void job_run(void *ctx, int64_t b, int64_t e, int worker) {
    (void)worker;
    const job_t *j = (const job_t *)ctx;
    for (int s = 0; s < j->nseg; s++) {
        int64_t s0 = j->start[s], s1 = j->start[s + 1];
        if (e <= s0) break;
        if (b >= s1) continue;
        int64_t r0 = (b > s0 ? b : s0) - s0, r1 = (e < s1 ? e : s1) - s0;
        const seg_t *g = &j->seg[s];
        tlm_matvec_rows(g->dt, g->W, g->rb, g->act, g->y, g->n, r0, r1, NULL);
    }
}

static void job_exec(job_t *j) {
    if (!j->nseg) return;
    tlm_pool_for(j->work < REF_SERIAL_WORK ? NULL : g_pool, j->start[j->nseg], REF_ROW_GRAIN, job_run, j);
}

/* One token through k selected experts (rank order). dt[3] = dtypes of
 * gate, up, down; gate[r]/up[r]/down[r] point at the selected experts'
 * matrices; w[r] are the routing weights. ffn[D] receives the combine. */
int tlmref_expert_ffn(int D, int de, int k, const int dt[3], const uint8_t *const *gate,
                      const uint8_t *const *up, const uint8_t *const *down, const float *x,
                      const float *w, float *ffn) {
    if (k <= 0 || k > REF_MAX_K) return -1;
    static float *eg, *eh, *eo;
    static uint8_t *ax, *ah;
    static int cap_D, cap_de, cap_k;
    if (D > cap_D || de > cap_de || k > cap_k) {
        free(eg); free(eh); free(eo); free(ax); free(ah);
        eg = malloc(sizeof(float) * (size_t)k * 2 * de);
        eh = malloc(sizeof(float) * (size_t)k * de);
        eo = malloc(sizeof(float) * (size_t)k * D);
        ax = malloc(tlm_qact_bytes(TLM_DT_Q8_K, D) + tlm_qact_bytes(TLM_DT_Q8_0, D) + 128);
        ah = malloc((tlm_qact_bytes(TLM_DT_Q8_K, de) + tlm_qact_bytes(TLM_DT_Q8_0, de) + 128) * (size_t)k);
        cap_D = D; cap_de = de; cap_k = k;
    }
    tlm_dtype gdt = (tlm_dtype)dt[0], udt = (tlm_dtype)dt[1], ddt = (tlm_dtype)dt[2];
    uint8_t *ax8k = ax, *ax80 = ax + tlm_qact_bytes(TLM_DT_Q8_K, D) + 64;
    tlm_quantize_act(TLM_DT_Q8_K, x, D, ax8k);
    tlm_quantize_act(TLM_DT_Q8_0, x, D, ax80);
    const void *ag = tlm_act_kind_for(gdt) == TLM_DT_Q8_0 ? (const void *)ax80 : (const void *)ax8k;
    const void *au = tlm_act_kind_for(udt) == TLM_DT_Q8_0 ? (const void *)ax80 : (const void *)ax8k;
    job_t j;
    j.nseg = 0;
    j.work = 0;
    for (int r = 0; r < k; r++) {
        job_add(&j, gdt, gate[r], de, D, ag, eg + (size_t)r * 2 * de);
        job_add(&j, udt, up[r], de, D, au, eg + (size_t)r * 2 * de + de);
    }
    job_exec(&j);
    j.nseg = 0;
    j.work = 0;
    size_t hstride = tlm_qact_bytes(TLM_DT_Q8_K, de) + tlm_qact_bytes(TLM_DT_Q8_0, de) + 128;
    for (int r = 0; r < k; r++) {
        float *g = eg + (size_t)r * 2 * de, *u = g + de, *hh = eh + (size_t)r * de;
        for (int i = 0; i < de; i++) hh[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
        uint8_t *a = ah + hstride * (size_t)r;
        tlm_quantize_act(tlm_act_kind_for(ddt), hh, de, a);
        job_add(&j, ddt, down[r], D, de, a, eo + (size_t)r * D);
    }
    job_exec(&j);
    for (int i = 0; i < D; i++) ffn[i] = 0.0f;
    for (int r = 0; r < k; r++)
        for (int i = 0; i < D; i++) {
            float c = w[r] * eo[(size_t)r * D + i];
            ffn[i] += c;
        }
    return 0;
}
