/* tlmo.h - CPU oracle for the quantised MoE decoder step.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference
 * (jbennie/tierlm) scalar algorithms for the hot path. tests/, the package's
 * smoke check and bench.py's CPU-baseline leg use it as the CHECKER; no
 * product code path may link, load or call it.
 *
 * Parity pinning: tests/test_oracle_golden.py checks this oracle against the
 * known-answer blocks of the reference's own test suite
 * (tests/test_quant.c:378-423, :434-538) and against golden vectors that
 * tests/golden/make_golden.py produced from the reference's own sources
 * (compiled by oracle/Makefile into oracle/_ref/).
 *
 * Every function cites the reference file:line it restates (paths relative
 * to the reference project root).
 */
#ifndef TLMO_H
#define TLMO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes: the numeric values of tlm_dtype (src/lib/tlm_quant.h:31-42). */
enum {
    TLMO_F32 = 0, TLMO_F16 = 1, TLMO_BF16 = 2, TLMO_Q8_0 = 8, TLMO_Q4_K = 12,
    TLMO_Q5_K = 13, TLMO_Q6_K = 14, TLMO_Q8_K = 15, TLMO_MXFP4 = 39
};

float    tlmo_f16_to_f32(uint16_t h);
uint16_t tlmo_f32_to_f16(float f);
float    tlmo_bf16_to_f32(uint16_t h);
uint16_t tlmo_f32_to_bf16(float f);

int    tlmo_dtype_block(int dt);
size_t tlmo_dtype_block_bytes(int dt);
size_t tlmo_row_bytes(int dt, int64_t n);
size_t tlmo_qact_bytes(int kind, int64_t n);
int    tlmo_act_kind_for(int wdt);

void  tlmo_quantize_act(int kind, const float *x, int64_t n, void *dst);
/* Dequantise a row of n values (src/lib/tlm_quant.c:584-665). 0 or -1. */
int   tlmo_dequantize_row(int dt, const void *src, float *y, int64_t n);
float tlmo_vec_dot(int dt, const void *wrow, const void *act, int64_t n);
void  tlmo_matvec_rows(int dt, const void *W, size_t row_bytes, const void *act, float *y,
                       int64_t n, int64_t r0, int64_t r1);
/* Exact per-block integer partial sums of one row dot (integer formats).
 * isum[b] is the block's scaled code sum, msum[b] the Q4_K/Q5_K min term
 * (0 for the other formats). Returns the number of blocks, or -1. */
int64_t tlmo_block_partials(int dt, const void *wrow, const void *act, int64_t n,
                            int32_t *isum, int32_t *msum);

/* expf used by the router softmax / sigmoid and SiLU:
 *   mode 0 = libm expf (what the reference calls),
 *   mode 1 = correctly rounded expf (the CUDA tier's device function). */
void  tlmo_set_expf_mode(int mode);
int   tlmo_get_expf_mode(void);
float tlmo_expf(float x);
float tlmo_expf_cr(float x);

/* Router (src/lib/tlm_model.c:776-839). mask/bias may be NULL. */
/* Decode attention of one token over a paged f32 KV cache (attn_heads,
 * src/lib/tlm_model.c:683-718): q [H][hd]; pages [n][KV][page][hd];
 * page_table [ceil(T / page)]; out [H][hd]. expf per tlmo_set_expf_mode. */
void tlmo_decode_attention(const float *q, const float *kp, const float *vp, const int32_t *page_table, int page,
                           int T, int H, int KV, int hd, float *out);
void tlmo_route(int router, const float *logits, const uint8_t *mask, const float *bias,
                int E, int k, float routed_scale, int *ids, float *w);

/* One routed expert in HBM-slot form: three matrices inside one payload,
 * each with its own dtype (the reference packet uses one dtype for all
 * three, src/lib/tlm_model.c:880-896; per-matrix dtypes are a superset). */
typedef struct {
    const uint8_t *base;
    uint64_t       off[3];   /* gate, up, down */
    int32_t        dt[3];
} tlmo_expert;

typedef struct {
    int32_t d_model, d_expert, d_shared, n_experts, top_k, router;
    float   routed_scale, norm_eps;
} tlmo_geom;

typedef struct {
    const float       *ffn_norm;          /* [D] */
    int32_t            router_dt;         /* normally F32 */
    const void        *router_w;          /* [E x D] */
    size_t             router_rb;
    const float       *router_bias;       /* [E] (router 2) or NULL */
    const uint8_t     *mask;              /* [E] or NULL */
    const tlmo_expert *experts;           /* [E] */
    int32_t            has_shared;
    int32_t            sh_dt[3];
    const void        *sh_w[3];           /* gate [ds x D], up [ds x D], down [D x ds] */
    const float       *shared_gate_inp;   /* [D] or NULL */
    int32_t            has_dense;         /* dense-FFN layer: no router, experts or shared expert */
    int32_t            d_ffn;
    int32_t            dn_dt[3];
    const void        *dn_w[3];           /* gate [d_ffn x D], up [d_ffn x D], down [D x d_ffn] */
} tlmo_layer;

/* Routed-expert FFN for one token (run_batch + the rank-ordered combine,
 * src/lib/tlm_model.c:900-938 and :1029-1036): x is the normalised input
 * [D], logits the router output [E]. ffn [D] receives sum_r w[r]*eo[r].
 * ids/w (top_k) may be NULL. eo_out ([k x D]) and h_out ([k x de]) may be
 * NULL; when given they receive the per-rank down outputs and SwiGLU rows. */
int tlmo_expert_ffn(const tlmo_geom *g, const tlmo_expert *experts, const uint8_t *mask,
                    const float *bias, const float *x, const float *logits, float *ffn,
                    int *ids, float *w, float *eo_out, float *h_out);

/* The whole moe() block (src/lib/tlm_model.c:940-1055) without the store:
 * RMSNorm, router matvec, route, experts, shared expert, h += ffn. */
int tlmo_moe_layer(const tlmo_geom *g, const tlmo_layer *L, float *h, int *ids, float *w);
/* The same plus the route hook's per-rank output norms onorm [top_k]
 * (src/lib/tlm_model.c:1029-1039): (float)sqrt of the double sum, in index
 * order, of c*c over c = w[r]*eo_r[i]. onorm may be NULL. A dense-FFN layer
 * (src/lib/tlm_model.c:947-964) leaves ids / w / onorm untouched. */
int tlmo_moe_layer_ex(const tlmo_geom *g, const tlmo_layer *L, float *h, int *ids, float *w, float *onorm);

/* RMSNorm (src/lib/tlm_model.c:164-169). */
void tlmo_rmsnorm(float *out, const float *x, const float *w, int64_t n, float eps);

#ifdef __cplusplus
}
#endif
#endif
