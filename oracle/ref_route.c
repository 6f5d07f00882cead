/* ref_route.c - exposes the REFERENCE's own router for golden vectors.
 *
 * TEST INFRASTRUCTURE ONLY. The reference's src/lib/tlm_model.c is compiled
 * in place through the #include below (the include path points at the
 * reference tree; nothing is copied), so tlmref_route() runs the reference's
 * static route()/topk() (src/lib/tlm_model.c:776-839) on a minimal model
 * object holding only what route() reads: the geometry, the expert mask, the
 * probability scratch and the layer's router bias.
 */
#define _GNU_SOURCE 1
#include "tlm_model.c"

int tlmref_route(int router, const float *logits, const uint8_t *mask, const float *bias, int E, int k,
                 float routed_scale, int *ids, float *w) {
    if (E <= 0 || k <= 0 || k > E || k > MAX_TOPK) return -1;
    tlm_model M;
    layer_w L;
    memset(&M, 0, sizeof M);
    memset(&L, 0, sizeof L);
    M.g.n_layers = 1;
    M.g.n_experts = (uint32_t)E;
    M.g.top_k = (uint32_t)k;
    M.g.router = (uint32_t)router;
    M.g.routed_scale = routed_scale;
    L.router_bias = bias;
    M.L = &L;
    uint8_t *zmask = calloc((size_t)E, 1);
    float *p = malloc(sizeof(float) * (size_t)E), *lg = malloc(sizeof(float) * (size_t)E);
    if (!zmask || !p || !lg) { free(zmask); free(p); free(lg); return -2; }
    memcpy(lg, logits, sizeof(float) * (size_t)E);   /* route() overwrites its logits */
    M.mask = mask ? (uint8_t *)mask : zmask;
    M.rp = p;
    route(&M, 0, lg, k, ids, w);
    free(zmask); free(p); free(lg);
    return 0;
}

/* The reference's decode attention of one token (attn_heads,
 * src/lib/tlm_model.c:683-718) on a minimal model / KV object: q f32[H][hd]
 * (after q-norm and RoPE), k / v f32[KV][T][hd] (one layer, max_ctx = T),
 * out f32[H][hd]. Uses libm expf, as the reference does. */
int tlmref_attn_heads(const float *q, const float *k, const float *v, int T, int H, int KV, int hd, float *out) {
    if (T <= 0 || H <= 0 || KV <= 0 || H % KV || hd <= 0) return -1;
    tlm_model M;
    tlm_kv kv;
    memset(&M, 0, sizeof M);
    memset(&kv, 0, sizeof kv);
    M.g.n_layers = 1;
    M.g.n_heads = (uint32_t)H;
    M.g.n_kv_heads = (uint32_t)KV;
    M.g.head_dim = (uint32_t)hd;
    M.q = (float *)q;
    M.att = out;
    kv.mdl = &M;
    kv.max_ctx = T;
    kv.len = T;
    kv.k = (float *)k;
    kv.v = (float *)v;
    kv.scores = malloc(sizeof(float) * (size_t)H * (size_t)T);
    if (!kv.scores) return -2;
    attn_job aj = { &M, &kv, 0, T - 1 };
    attn_heads(&aj, 0, H, 0);
    free(kv.scores);
    return 0;
}
