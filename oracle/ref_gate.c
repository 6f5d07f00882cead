/* ref_gate.c - the reference's own decoder step with its MoE blocks served
 * by libtlmg (the CUDA tier): the end-to-end gate of the quantised MoE
 * decoder step.
 *
 * TEST INFRASTRUCTURE ONLY. The reference's src/lib/tlm_model.c is compiled
 * in place through the #include below (the include path points at the
 * reference tree; nothing is copied). A store made by the reference's own
 * `tlmc synth` + `tlmc compile` is opened the way `tierlm` opens it (rt_open,
 * src/bin/tierlm.c:196-310: manifest, drives, worker pool, expert store with
 * every expert cached, model), and tokens run through one of three steps:
 *
 *   GATE_REF  the reference's tlm_model_step (src/lib/tlm_model.c:1058-1103);
 *   GATE_CPU  gate_step_impl(): tlm_model_step restated call for call with
 *             the reference's own moe() (GATE_REF == GATE_CPU bit for bit is
 *             what shows the restatement is faithful);
 *   GATE_STEP tlmg_decode_step: the whole step (embedding, attention, MoE,
 *             lm_head) on the GPU, the KV pages in HBM;
 *   GATE_GPU  gate_step_impl() with every moe() (src/lib/tlm_model.c:
 *             940-1055) replaced by tlmg_moe_layer_ex on the GPU: RMSNorm,
 *             router, experts, shared expert or the dense FFN, h += ffn.
 *             Embedding, attention and the lm_head stay on the reference's
 *             CPU code.
 *
 * Built twice (oracle/Makefile): as is, with the libm expf the reference
 * links (libtlmgate.so), and with -DGATE_CR_EXPF (libtlmgate_cr.so), where
 * every expf in tlm_model.c is bound to a correctly rounded expf - the one
 * the CUDA tier computes - so that the GPU-served step can be compared with
 * the reference bit for bit.
 */
#define _GNU_SOURCE 1
#include <math.h>
#include <stdio.h>

#ifdef GATE_CR_EXPF
/* (float)expl(x) is the correctly rounded expf on x86-64 (64-bit long double
 * mantissa; checked equal to the CUDA tier's expf on all 2^32 inputs). */
static float gate_cr_expf(float x) { return (float)expl((long double)x); }
#define expf gate_cr_expf
#endif

#include "tlm_model.c"

#include "tlm_io.h"
#include "tlm_pool.h"
#include "tlm_store.h"
#include "tlmg.h"

enum { GATE_REF = 0, GATE_CPU = 1, GATE_GPU = 2, GATE_STEP = 3 };

typedef struct {
    tlm_manifest m;
    tlm_io      *io;
    tlm_store   *st;
    tlm_pool    *pool;
    tlm_model   *M;
    tlm_kv      *kv;
    tlmg_ctx    *gpu;
    int          use_gpu;                 /* the MoE block of the current step runs on the GPU */
    /* route hook capture: per layer, the last call's ids / weights / output norms */
    int          hook_on;
    int          hook_k;
    int         *h_ids;
    float       *h_w, *h_onorm;
    int         *h_seen;
} gate;

static __thread char g_err[512];
const char *gate_errmsg(void) { return g_err; }
static int fail(int rc, const char *what) {
    snprintf(g_err, sizeof g_err, "%s: %s", what, tlm_errmsg());
    return rc ? rc : -1;
}

static void gate_hook(void *ctx, int layer, int pos, int token, const int *ids, const float *w,
                      const float *onorm, int k) {
    (void)pos; (void)token;
    gate *G = (gate *)ctx;
    if (!G->hook_on || k > G->hook_k) return;
    for (int r = 0; r < k; r++) {
        G->h_ids[layer * G->hook_k + r] = ids[r];
        G->h_w[layer * G->hook_k + r] = w[r];
        G->h_onorm[layer * G->hook_k + r] = onorm[r];
    }
    G->h_seen[layer]++;
}

void gate_close(void *p) {
    gate *G = (gate *)p;
    if (!G) return;
    if (G->gpu) tlmg_close(G->gpu);
    if (G->kv) tlm_kv_free(G->kv);
    if (G->M) tlm_model_close(G->M);
    if (G->st) tlm_store_close(G->st);
    if (G->io) tlm_io_close(G->io);
    if (G->pool) tlm_pool_free(G->pool);
    tlm_manifest_free(&G->m);
    free(G->h_ids); free(G->h_w); free(G->h_onorm); free(G->h_seen);
    free(G);
}

/* Open the store at `manifest` as tierlm does, with every expert cached,
 * `threads` pool workers (0 = all cores) and room for max_ctx positions. */
void *gate_open(const char *manifest, int threads, int max_ctx) {
    gate *G = (gate *)calloc(1, sizeof *G);
    if (!G) { snprintf(g_err, sizeof g_err, "out of memory"); return NULL; }
    if (tlm_manifest_load(&G->m, manifest)) { fail(-1, "manifest"); free(G); return NULL; }
    char paths[TLM_MAX_DRIVES][1024];
    const char *pp[TLM_MAX_DRIVES];
    for (uint32_t d = 0; d < G->m.n_drives; d++) {
        tlm_manifest_drive_path(&G->m, (int)d, paths[d], sizeof paths[d]);
        pp[d] = paths[d];
    }
    G->pool = tlm_pool_new(threads, 0);
    tlm_io_opts io;
    memset(&io, 0, sizeof io);
    io.backend = TLM_IO_PREAD;
    io.threads_per_drive = 4;
    io.queue_depth = 32;
    G->io = G->pool ? tlm_io_open(pp, (int)G->m.n_drives, &io) : NULL;
    if (!G->io) { fail(-1, "io"); gate_close(G); return NULL; }
    uint64_t total = 0, slot = 0;
    for (uint32_t i = 0; i < G->m.n_packets; i++) {
        const tlm_packet_loc *l = &G->m.packets[i];
        if (l->type != TLM_PK_EXPERT || (l->flags & 2u)) continue;
        total += l->total_len;
        if (l->total_len > slot) slot = l->total_len;
    }
    tlm_store_opts so;
    memset(&so, 0, sizeof so);
    so.budget_bytes = total + 4 * slot;     /* every expert fits: the result never depends on the cache */
    so.prefetch = 1;
    G->st = tlm_store_open(&G->m, G->io, &so);
    if (!G->st) { fail(-1, "store"); gate_close(G); return NULL; }
    tlm_model_opts mo = { 1, 0, 0.0 };
    G->M = tlm_model_open(&G->m, G->io, G->st, G->pool, &mo);
    if (!G->M) { fail(-1, "model"); gate_close(G); return NULL; }
    G->kv = tlm_kv_new(G->M, max_ctx);
    if (!G->kv) { fail(-1, "kv"); gate_close(G); return NULL; }
    const tlm_model_geom *g = &G->M->g;
    G->hook_k = g->top_k > 0 ? (int)g->top_k : 1;
    size_t n = (size_t)g->n_layers * G->hook_k;
    G->h_ids = (int *)calloc(n, sizeof(int));
    G->h_w = (float *)calloc(n, sizeof(float));
    G->h_onorm = (float *)calloc(n, sizeof(float));
    G->h_seen = (int *)calloc(g->n_layers, sizeof(int));
    if (!G->h_ids || !G->h_w || !G->h_onorm || !G->h_seen) { snprintf(g_err, sizeof g_err, "oom"); gate_close(G); return NULL; }
    tlm_model_set_route_hook(G->M, gate_hook, G);
    return G;
}

/* geometry: n_layers, d_model, vocab, n_experts, top_k, d_expert, d_shared, n_dense_layers */
int gate_geom(void *p, int *out) {
    gate *G = (gate *)p;
    const tlm_model_geom *g = &G->M->g;
    int nd = 0;
    for (uint32_t l = 0; l < g->n_layers; l++) nd += G->M->L[l].has_dense_ffn;
    out[0] = (int)g->n_layers; out[1] = (int)g->d_model; out[2] = (int)g->vocab; out[3] = (int)g->n_experts;
    out[4] = (int)g->top_k; out[5] = (int)g->d_expert; out[6] = (int)g->d_shared; out[7] = nd;
    return 0;
}

/* router mode, routed_scale, norm_eps */
int gate_geomf(void *p, float *out) {
    const tlm_model_geom *g = &((gate *)p)->M->g;
    out[0] = (float)g->router; out[1] = g->routed_scale; out[2] = g->norm_eps;
    return 0;
}

/* Upload every layer's MoE block to a tlmg context on `device`: ffn_norm,
 * router (+ bias, mask), shared expert (+ gate vector) or dense FFN, and
 * each routed expert's payload from the store (expert_mats' offsets and
 * dtype, src/lib/tlm_model.c:880-896). */
int gate_attach_gpu(void *p, int device) {
    gate *G = (gate *)p;
    tlm_model *M = G->M;
    const tlm_model_geom *g = &M->g;
    tlmg_geom tg;
    memset(&tg, 0, sizeof tg);
    tg.n_layers = (int32_t)g->n_layers;
    tg.d_model = (int32_t)g->d_model;
    tg.d_expert = (int32_t)g->d_expert;
    tg.d_shared = g->n_shared > 0 ? (int32_t)g->d_shared : 0;
    tg.n_experts = (int32_t)g->n_experts;
    tg.top_k = (int32_t)g->top_k;
    tg.router = (int32_t)g->router;
    tg.routed_scale = g->routed_scale;
    tg.norm_eps = g->norm_eps;
    int rc = tlmg_open(&tg, device, &G->gpu);
    if (rc) { snprintf(g_err, sizeof g_err, "tlmg_open: %s", tlmg_errmsg()); return rc; }
    const int E = (int)g->n_experts;
    for (int l = 0; l < (int)g->n_layers; l++) {
        layer_w *L = &M->L[l];
        if (L->has_dense_ffn) {
            int32_t dt[3] = { (int32_t)L->dg.dt, (int32_t)L->du.dt, (int32_t)L->dd.dt };
            if ((rc = tlmg_set_layer(G->gpu, l, L->ffn_norm, 0, NULL, 0, NULL, NULL)) ||
                (rc = tlmg_set_dense_ffn(G->gpu, l, (int)L->d_ffn, dt, L->dg.data, L->du.data, L->dd.data))) {
                snprintf(g_err, sizeof g_err, "layer %d dense: %s", l, tlmg_errmsg());
                return rc;
            }
            continue;
        }
        rc = tlmg_set_layer(G->gpu, l, L->ffn_norm, (int)L->router.dt, L->router.data, L->router.row_bytes,
                            L->router_bias, M->mask + (size_t)l * E);
        if (!rc && L->has_shared) {
            int32_t dt[3] = { (int32_t)L->sg.dt, (int32_t)L->su.dt, (int32_t)L->sd.dt };
            rc = tlmg_set_shared(G->gpu, l, dt, L->sg.data, L->su.data, L->sd.data, L->shared_gate_inp);
        }
        if (rc) { snprintf(g_err, sizeof g_err, "layer %d: %s", l, tlmg_errmsg()); return rc; }
        for (int e = 0; e < E; e++) {
            const expert_info *x = &M->ex[(size_t)l * E + e];
            if (!x->present) { snprintf(g_err, sizeof g_err, "layer %d expert %d has no packet", l, e); return -6; }
            tlm_expert_ref ref;
            memset(&ref, 0, sizeof ref);
            ref.slot = -1;
            int id = e;
            if ((rc = tlm_store_acquire(G->st, l, &id, 1, &ref)) == 0) rc = tlm_store_wait(G->st, &ref);
            if (rc) { tlm_store_release(G->st, &ref); return fail(rc, "store acquire"); }
            int32_t dt[3] = { (int32_t)x->dtype, (int32_t)x->dtype, (int32_t)x->dtype };
            uint64_t off[3] = { x->off[0], x->off[1], x->off[2] };
            rc = tlmg_set_expert(G->gpu, l, e, dt, ref.payload, ref.payload_len, off);
            tlm_store_release(G->st, &ref);
            if (rc) { snprintf(g_err, sizeof g_err, "layer %d expert %d: %s", l, e, tlmg_errmsg()); return rc; }
        }
    }
    /* the rest of the step: attention weights, embedding, output (KV f32,
     * exact attention: the reference's order of operations) */
    rc = tlmg_step_open(G->gpu, (int)g->n_heads, (int)g->n_kv_heads, (int)g->head_dim, (int)g->vocab, M->inv_freq,
                        M->rope_attn_scale, G->kv->max_ctx, TLMG_DT_F32, TLMG_ATTN_EXACT);
    for (int l = 0; l < (int)g->n_layers && !rc; l++) {
        layer_w *L = &M->L[l];
        const wmat *q[4] = { &L->q, &L->k, &L->v, &L->o };
        int32_t dt[4];
        const void *w[4];
        size_t rb[4];
        for (int i = 0; i < 4; i++) {
            dt[i] = (int32_t)q[i]->dt;
            w[i] = q[i]->data;
            rb[i] = q[i]->row_bytes;
        }
        rc = tlmg_set_attention(G->gpu, l, L->attn_norm, dt, w, rb, L->q_norm, L->k_norm);
    }
    if (!rc) rc = tlmg_set_embedding(G->gpu, (int)M->embd.dt, M->embd.data, M->embd.row_bytes);
    if (!rc) rc = tlmg_set_output(G->gpu, M->out_norm, (int)M->lm_head.dt, M->lm_head.data, M->lm_head.row_bytes);
    if (rc) { snprintf(g_err, sizeof g_err, "decoder step: %s", tlmg_errmsg()); return rc; }
    return 0;
}

/* moe() on the GPU, with moe()'s route-hook call (src/lib/tlm_model.c:1053). */
static int gpu_moe(gate *G, tlm_model *M, int l, int pos, int token) {
    const tlm_model_geom *g = &M->g;
    const int k = (int)g->top_k;
    int32_t ids[MAX_TOPK];
    float w[MAX_TOPK], onorm[MAX_TOPK];
    int rc = tlmg_moe_layer_ex(G->gpu, l, M->h, ids, w, M->hook ? onorm : NULL);
    if (rc) return tlm_seterr(TLM_EIO, "tlmg_moe_layer_ex: %s", tlmg_errmsg());
    if (M->hook && g->n_experts > 0 && !M->L[l].has_dense_ffn) {
        int iids[MAX_TOPK];
        for (int r = 0; r < k; r++) iids[r] = ids[r];
        M->hook(M->hook_ctx, l, pos, token, iids, w, onorm, k);
    }
    return TLM_OK;
}

/* tlm_model_step (src/lib/tlm_model.c:1058-1103) restated with the same
 * calls in the same order; only the MoE block differs when G->use_gpu. */
static int gate_step_impl(gate *G, tlm_kv *kv, int token, float *logits) {
    tlm_model *M = G->M;
    const tlm_model_geom *g = &M->g;
    if (token < 0 || (uint32_t)token >= g->vocab) return tlm_seterr(TLM_EINVAL, "token %d out of range", token);
    if (kv->len >= kv->max_ctx) return tlm_seterr(TLM_ERANGE, "context full (%d tokens)", kv->max_ctx);
    int pos = kv->len, D = (int)g->d_model, hd = (int)g->head_dim;
    const uint8_t *row = M->embd.data + (size_t)token * M->embd.row_bytes;
    if (M->embd.dt == TLM_DT_F32) memcpy(M->h, row, (size_t)D * sizeof(float));
    else if (tlm_dequantize_row(M->embd.dt, row, M->h, D) != 0)
        return tlm_seterr(TLM_EUNSUP, "cannot dequantise embedding dtype %d", (int)M->embd.dt);
    for (int j = 0; j < hd / 2; j++) {
        double a = (double)pos * (double)M->inv_freq[j];
        M->cs[j] = (float)cos(a) * M->rope_attn_scale;
        M->sn[j] = (float)sin(a) * M->rope_attn_scale;
    }
    if (!G->use_gpu && M->o.lookahead > 0) lookahead(M, 0);   /* a store hint: never changes results */
    int rc = TLM_OK;
    for (int l = 0; l < (int)g->n_layers && rc == TLM_OK; l++) {
        attention(M, kv, l, pos);
        rc = G->use_gpu ? gpu_moe(G, M, l, pos, token) : moe(M, l, pos, token);
    }
    if (rc) return rc;
    kv->len = pos + 1;
    if (logits) {
        rmsnorm(M->xb, M->h, M->out_norm, D, g->norm_eps);
        actc_set(&M->a_fin, M->xb);
        mv_job j;
        j.nseg = 0;
        j.work = 0;
        mv_add(&j, &M->lm_head, actc_get(&M->a_fin, M->lm_head.dt), logits);
        mv_exec(M, &j);
    }
    if (M->store) tlm_store_tick(M->store);
    return TLM_OK;
}

static int step_mode(gate *G, int mode, int token, float *logits) {
    if (mode == GATE_REF) return tlm_model_step(G->M, G->kv, token, logits);
    if (mode == GATE_STEP) {
        if (!G->gpu) return tlm_seterr(TLM_EINVAL, "gate: no GPU attached");
        const int pos = G->kv->len;
        if (pos >= G->kv->max_ctx) return tlm_seterr(TLM_ERANGE, "context full (%d tokens)", G->kv->max_ctx);
        if (tlmg_decode_step(G->gpu, token, pos, logits)) return tlm_seterr(TLM_EIO, "tlmg_decode_step: %s", tlmg_errmsg());
        G->kv->len = pos + 1;
        return TLM_OK;
    }
    if (mode == GATE_GPU && !G->gpu) return tlm_seterr(TLM_EINVAL, "gate: no GPU attached");
    G->use_gpu = mode == GATE_GPU;
    int rc = gate_step_impl(G, G->kv, token, logits);
    G->use_gpu = 0;
    return rc;
}

int gate_reset(void *p) { tlm_kv_reset(((gate *)p)->kv); return 0; }
int gate_hook_enable(void *p, int on) {
    gate *G = (gate *)p;
    G->hook_on = on;
    memset(G->h_seen, 0, sizeof(int) * G->M->g.n_layers);
    return 0;
}
/* ids / w / onorm of `layer` from the last hooked MoE call; returns the number of calls seen since enabling */
int gate_hook_read(void *p, int layer, int *ids, float *w, float *onorm) {
    gate *G = (gate *)p;
    for (int r = 0; r < G->hook_k; r++) {
        ids[r] = G->h_ids[layer * G->hook_k + r];
        w[r] = G->h_w[layer * G->hook_k + r];
        onorm[r] = G->h_onorm[layer * G->hook_k + r];
    }
    return G->h_seen[layer];
}

/* One position: logits f32[vocab] (may be NULL). */
int gate_step(void *p, int mode, int token, float *logits) {
    int rc = step_mode((gate *)p, mode, token, logits);
    return rc ? fail(rc, "step") : 0;
}

/* cmd_bench's flow (src/bin/tierlm.c:702-756): prefill np prompt tokens (the
 * step repeated, tlm_model_prefill), then n_gen greedy tokens (tlm_sample
 * with no sampler: argmax, ties to the lowest id) into out[]. Per position
 * the logits go to logits_all f32[(np + n_gen - 1)][vocab] when not NULL
 * (row i = the distribution after token i). */
int gate_generate(void *p, int mode, const int *prompt, int np, int n_gen, int *out, float *logits_all) {
    gate *G = (gate *)p;
    const int V = (int)G->M->g.vocab;
    float *lg = (float *)malloc(sizeof(float) * (size_t)V);
    if (!lg) return fail(TLM_ENOMEM, "generate");
    tlm_kv_reset(G->kv);
    int rc = 0, row = 0;
    for (int i = 0; i < np && !rc; i++) {
        rc = step_mode(G, mode, prompt[i], lg);
        if (!rc && logits_all) memcpy(logits_all + (size_t)row++ * V, lg, sizeof(float) * (size_t)V);
    }
    for (int t = 0; t < n_gen && !rc; t++) {
        int tok = tlm_sample(NULL, NULL, lg, V);
        out[t] = tok;
        if (t + 1 < n_gen) {
            rc = step_mode(G, mode, tok, lg);
            if (!rc && logits_all) memcpy(logits_all + (size_t)row++ * V, lg, sizeof(float) * (size_t)V);
        }
    }
    free(lg);
    return rc ? fail(rc, "generate") : 0;
}

/* Teacher-forced run (cmd_oracle, src/bin/tierlm.c:670-700): every token of
 * seq[0..n) in turn, logits of each position into logits_all f32[n][vocab]. */
int gate_teacher(void *p, int mode, const int *seq, int n, float *logits_all) {
    gate *G = (gate *)p;
    const int V = (int)G->M->g.vocab;
    tlm_kv_reset(G->kv);
    for (int i = 0; i < n; i++) {
        int rc = step_mode(G, mode, seq[i], logits_all + (size_t)i * V);
        if (rc) return fail(rc, "teacher-forced step");
    }
    return 0;
}

/* The reference's moe() alone on a given residual (the golden vectors of the
 * MoE block): h f32[D] in/out through layer `layer`; the route hook's ids,
 * weights and output norms of the call into ids / w / onorm [top_k]. mode
 * GATE_GPU runs tlmg_moe_layer_ex instead. */
int gate_moe(void *p, int mode, int layer, float *h, int *ids, float *w, float *onorm) {
    gate *G = (gate *)p;
    tlm_model *M = G->M;
    const int D = (int)M->g.d_model;
    if (layer < 0 || layer >= (int)M->g.n_layers) return fail(TLM_ERANGE, "moe layer");
    memcpy(M->h, h, sizeof(float) * (size_t)D);
    int on = G->hook_on;
    G->hook_on = 1;
    int seen = G->h_seen[layer];
    int rc = mode == GATE_GPU ? (G->gpu ? gpu_moe(G, M, layer, 0, 0) : tlm_seterr(TLM_EINVAL, "no GPU"))
                              : moe(M, layer, 0, 0);
    G->hook_on = on;
    if (rc) return fail(rc, "moe");
    memcpy(h, M->h, sizeof(float) * (size_t)D);
    if (G->h_seen[layer] != seen) gate_hook_read(G, layer, ids, w, onorm);
    return 0;
}

/* Host copies of one layer's MoE tensors for the oracle restatement: which
 * 0 ffn_norm, 1 router, 2 router_bias, 3 shared gate, 4 up, 5 down,
 * 6 shared_gate_inp, 7/8/9 dense gate/up/down. Returns the byte count (0 if
 * absent) and the dtype in *dt; copies when dst != NULL. */
int64_t gate_layer_tensor(void *p, int layer, int which, void *dst, int *dt) {
    gate *G = (gate *)p;
    tlm_model *M = G->M;
    const tlm_model_geom *g = &M->g;
    layer_w *L = &M->L[layer];
    const void *src = NULL;
    int64_t bytes = 0;
    const wmat *wm = NULL;
    *dt = TLM_DT_F32;
    switch (which) {
    case 0: src = L->ffn_norm; bytes = src ? 4 * (int64_t)g->d_model : 0; break;
    case 1: wm = &L->router; break;
    case 2: src = L->router_bias; bytes = src ? 4 * (int64_t)g->n_experts : 0; break;
    case 3: wm = L->has_shared ? &L->sg : NULL; break;
    case 4: wm = L->has_shared ? &L->su : NULL; break;
    case 5: wm = L->has_shared ? &L->sd : NULL; break;
    case 6: src = L->has_shared ? L->shared_gate_inp : NULL; bytes = src ? 4 * (int64_t)g->d_model : 0; break;
    case 7: wm = L->has_dense_ffn ? &L->dg : NULL; break;
    case 8: wm = L->has_dense_ffn ? &L->du : NULL; break;
    case 9: wm = L->has_dense_ffn ? &L->dd : NULL; break;
    default: return -1;
    }
    if (wm && wm->data) {
        src = wm->data;
        bytes = (int64_t)wm->row_bytes * wm->rows;
        *dt = (int)wm->dt;
    }
    if (dst && src && bytes) memcpy(dst, src, (size_t)bytes);
    return src ? bytes : 0;
}

/* One routed expert's payload (expert_mats' view): returns payload bytes,
 * the dtype and item offsets; copies the payload when dst != NULL. */
int64_t gate_expert(void *p, int layer, int e, void *dst, int *dt, uint32_t off[3]) {
    gate *G = (gate *)p;
    tlm_model *M = G->M;
    const expert_info *x = &M->ex[(size_t)layer * M->g.n_experts + e];
    if (!x->present) return 0;
    tlm_expert_ref ref;
    memset(&ref, 0, sizeof ref);
    ref.slot = -1;
    int id = e, rc;
    if ((rc = tlm_store_acquire(G->st, layer, &id, 1, &ref)) == 0) rc = tlm_store_wait(G->st, &ref);
    if (rc) { tlm_store_release(G->st, &ref); return fail(rc, "store acquire"); }
    *dt = (int)x->dtype;
    for (int m = 0; m < 3; m++) off[m] = x->off[m];
    int64_t n = (int64_t)x->payload_len;
    if (dst) memcpy(dst, ref.payload, (size_t)n);
    tlm_store_release(G->st, &ref);
    return n;
}
