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
