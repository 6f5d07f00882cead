/* tlmo.c - CPU oracle (test infrastructure only; see tlmo.h).
 *
 * Plain C11, compiled with -O2 -ffp-contract=off and no -ffast-math, the
 * same floating-point discipline as the reference build (Makefile:32). Each
 * routine restates the reference's scalar algorithm from its documented
 * contract; the citations name the lines it follows.
 */
#include "tlmo.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#if defined(FLT_EVAL_METHOD) && FLT_EVAL_METHOD != 0
#error "the oracle needs FLT_EVAL_METHOD == 0"
#endif

static inline uint32_t bits_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float    float_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline float    rdf32(const uint8_t *p) { float f; memcpy(&f, p, 4); return f; }

/* ---- half / bfloat conversions (src/lib/tlm_quant.c:124-172) ---------- */
float tlmo_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 31u) return float_of(s | 0x7F800000u | (m << 13) | (m ? 0x00400000u : 0u));
    if (e == 0u) return float_of(bits_of((float)m * 0x1p-24f) | s);
    return float_of(s | ((e + 112u) << 23) | (m << 13));
}

uint16_t tlmo_f32_to_f16(float f) {
    uint32_t x = bits_of(f), s = (x >> 16) & 0x8000u, a = x & 0x7FFFFFFFu;
    if (a >= 0x7F800000u)
        return (uint16_t)(a == 0x7F800000u ? (s | 0x7C00u) : (s | 0x7E00u | ((a >> 13) & 1023u)));
    if (a >= 0x477FF000u) return (uint16_t)(s | 0x7C00u);
    if (a < 0x38800000u) {
        if (a <= 0x33000000u) return (uint16_t)s;
        uint32_t sh = 126u - (a >> 23), mant = (a & 0x7FFFFFu) | 0x800000u;
        uint32_t q = mant >> sh, rem = mant & ((1u << sh) - 1u), half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(s | q);
    }
    uint32_t r = a - 0x38000000u, q = r >> 13, rem = r & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(s | q);
}

float tlmo_bf16_to_f32(uint16_t h) { return float_of((uint32_t)h << 16); }

uint16_t tlmo_f32_to_bf16(float f) {
    uint32_t x = bits_of(f);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

static inline float f16_at(const uint8_t *p) { return tlmo_f16_to_f32(rd16(p)); }

/* ---- dtype table (src/lib/tlm_quant.c:52-63) ----------------------------- */
int tlmo_dtype_block(int dt) {
    switch (dt) {
    case TLMO_F32: case TLMO_F16: case TLMO_BF16: return 1;
    case TLMO_Q8_0: case TLMO_MXFP4: return 32;
    case TLMO_Q4_K: case TLMO_Q5_K: case TLMO_Q6_K: case TLMO_Q8_K: return 256;
    default: return 0;
    }
}

size_t tlmo_dtype_block_bytes(int dt) {
    switch (dt) {
    case TLMO_F32: return 4;
    case TLMO_F16: case TLMO_BF16: return 2;
    case TLMO_Q8_0: return 34;
    case TLMO_Q4_K: return 144;
    case TLMO_Q5_K: return 176;
    case TLMO_Q6_K: return 210;
    case TLMO_Q8_K: return 292;
    case TLMO_MXFP4: return 17;
    default: return 0;
    }
}

size_t tlmo_row_bytes(int dt, int64_t n) {
    int qk = tlmo_dtype_block(dt);
    if (!qk || n < 0 || n % qk) return 0;
    return (size_t)(n / qk) * tlmo_dtype_block_bytes(dt);
}

/* src/lib/tlm_quant.c:670-678 */
size_t tlmo_qact_bytes(int kind, int64_t n) {
    if (n < 0) return 0;
    if (kind == TLMO_Q8_K) return (size_t)((n + 255) / 256) * 292u;
    if (kind == TLMO_Q8_0) return (size_t)((n + 31) / 32) * 36u;
    if (kind == TLMO_F32) return (size_t)n * 4u;
    return 0;
}

/* src/lib/tlm_quant.c:691-697 */
int tlmo_act_kind_for(int wdt) {
    switch (wdt) {
    case TLMO_Q4_K: case TLMO_Q5_K: case TLMO_Q6_K: case TLMO_Q8_K: return TLMO_Q8_K;
    case TLMO_Q8_0: case TLMO_MXFP4: return TLMO_Q8_0;
    default: return TLMO_F32;
    }
}

/* ---- activation quantiser (src/lib/tlm_quant.c:216-230, :458-512) ------ */
/* Round half to even for |v| < 2^22 by the 1.5*2^23 magic-number sum. */
static inline float rne_magic(float v) {
    volatile float t = v + 12582912.0f;   /* volatile: keep both roundings */
    return t - 12582912.0f;
}

static int q_clamp_rne(float v, int lo, int hi) {
    if (v != v) return 0;
    if (v <= (float)lo) return lo;
    if (v >= (float)hi) return hi;
    return (int)rne_magic(v);
}

/* One activation block of qk codes from nvalid inputs (rest zero). */
static void act_block(const float *x, int nvalid, int qk, float *d_out, int8_t *q) {
    float amax = 0.0f;
    int nan_seen = 0, inf_seen = 0;
    for (int i = 0; i < nvalid; i++) {
        float a = fabsf(x[i]);
        if (a != a) nan_seen = 1;
        else if (a == INFINITY) inf_seen = 1;
        else if (a > amax) amax = a;
    }
    memset(q, 0, (size_t)qk);
    if (nan_seen || inf_seen) { *d_out = nan_seen ? NAN : INFINITY; return; }
    if (!(amax > 0.0f)) { *d_out = 0.0f; return; }
    *d_out = amax / 127.0f;
    if (amax >= 0x1p-100f) {
        float inv = 127.0f / amax;
        for (int i = 0; i < nvalid; i++) q[i] = (int8_t)q_clamp_rne(x[i] * inv, -127, 127);
    } else {
        double inv = 127.0 / (double)amax;
        for (int i = 0; i < nvalid; i++) q[i] = (int8_t)q_clamp_rne((float)((double)x[i] * inv), -127, 127);
    }
}

void tlmo_quantize_act(int kind, const float *x, int64_t n, void *dst) {
    if (n <= 0) return;
    uint8_t *o = (uint8_t *)dst;
    if (kind == TLMO_Q8_K) {
        for (int64_t b = 0; b * 256 < n; b++) {
            uint8_t blk[292];
            float d;
            int8_t *q = (int8_t *)(blk + 4);
            int64_t rem = n - b * 256;
            act_block(x + b * 256, rem >= 256 ? 256 : (int)rem, 256, &d, q);
            memcpy(blk, &d, 4);
            for (int g = 0; g < 16; g++) {
                int s = 0;
                for (int i = 0; i < 16; i++) s += q[16 * g + i];
                int16_t s16 = (int16_t)s;
                memcpy(blk + 260 + 2 * g, &s16, 2);
            }
            memcpy(o + 292 * (size_t)b, blk, 292);
        }
    } else if (kind == TLMO_Q8_0) {
        for (int64_t b = 0; b * 32 < n; b++) {
            uint8_t blk[36];
            float d;
            int64_t rem = n - b * 32;
            act_block(x + b * 32, rem >= 32 ? 32 : (int)rem, 32, &d, (int8_t *)(blk + 4));
            memcpy(blk, &d, 4);
            memcpy(o + 36 * (size_t)b, blk, 36);
        }
    } else if (kind == TLMO_F32) {
        memcpy(dst, x, (size_t)n * 4u);
    }
}

/* ---- K-quant scale unpack (src/lib/tlm_quant.c:253-261) ---------------- */
/* sc[0..7] = 6-bit scales, mn[0..7] = 6-bit mins of one Q4_K/Q5_K block. */
static void kq_scales(const uint8_t *s12, int sc[8], int mn[8]) {
    for (int j = 0; j < 4; j++) {
        sc[j] = s12[j] & 63;
        mn[j] = s12[j + 4] & 63;
        sc[j + 4] = (s12[j + 8] & 15) | ((s12[j] >> 6) << 4);
        mn[j + 4] = (s12[j + 8] >> 4) | ((s12[j + 4] >> 6) << 4);
    }
}

static int k_e2m1x2_deq(int c) {
    static const int8_t t[16] = { 0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12 };
    return t[c & 15];
}

/* ---- dequantisers (src/lib/tlm_quant.c:584-665) -------------------------- */
int tlmo_dequantize_row(int dt, const void *src, float *y, int64_t n) {
    int qk = tlmo_dtype_block(dt);
    if (!qk || n < 0 || n % qk) return -1;
    const uint8_t *s = (const uint8_t *)src;
    int64_t nb = n / qk;
    for (int64_t b = 0; b < nb; b++) {
        float *o = y + b * qk;
        switch (dt) {
        case TLMO_F32: memcpy(o, s + 4 * b, 4); break;
        case TLMO_F16: o[0] = f16_at(s + 2 * b); break;
        case TLMO_BF16: o[0] = tlmo_bf16_to_f32(rd16(s + 2 * b)); break;
        case TLMO_Q8_0: {
            const uint8_t *blk = s + 34 * b;
            float d = f16_at(blk);
            for (int i = 0; i < 32; i++) o[i] = d * (float)(int8_t)blk[2 + i];
            break;
        }
        case TLMO_Q4_K: case TLMO_Q5_K: {
            int q5 = dt == TLMO_Q5_K;
            const uint8_t *blk = s + (q5 ? 176 : 144) * b;
            const uint8_t *qh = blk + 16, *qs = q5 ? blk + 48 : blk + 16;
            int sc[8], mn[8];
            kq_scales(blk + 4, sc, mn);
            float d = f16_at(blk), dmin = f16_at(blk + 2);
            for (int c = 0; c < 4; c++) {
                float d0 = d * (float)sc[2 * c], m0 = dmin * (float)mn[2 * c];
                float d1 = d * (float)sc[2 * c + 1], m1 = dmin * (float)mn[2 * c + 1];
                for (int l = 0; l < 32; l++) {
                    int lo = qs[32 * c + l] & 15, hi = qs[32 * c + l] >> 4;
                    if (q5) {
                        lo |= ((qh[l] >> (2 * c)) & 1) << 4;
                        hi |= ((qh[l] >> (2 * c + 1)) & 1) << 4;
                    }
                    o[64 * c + l] = d0 * (float)lo - m0;
                    o[64 * c + 32 + l] = d1 * (float)hi - m1;
                }
            }
            break;
        }
        case TLMO_Q6_K: {
            const uint8_t *blk = s + 210 * b, *ql = blk, *qh = blk + 128;
            const int8_t *sc = (const int8_t *)(blk + 192);
            float d = f16_at(blk + 208);
            for (int h = 0; h < 2; h++)
                for (int l = 0; l < 32; l++) {
                    int A = ql[64 * h + l], B = ql[64 * h + 32 + l], C = qh[32 * h + l];
                    int e = 128 * h + l;
                    int u[4] = { (A & 15) | ((C & 3) << 4), (B & 15) | (((C >> 2) & 3) << 4),
                                 (A >> 4) | (((C >> 4) & 3) << 4), (B >> 4) | (((C >> 6) & 3) << 4) };
                    for (int m = 0; m < 4; m++)
                        o[e + 32 * m] = d * (float)sc[(e + 32 * m) / 16] * (float)(u[m] - 32);
                }
            break;
        }
        case TLMO_Q8_K: {
            const uint8_t *blk = s + 292 * b;
            float d = rdf32(blk);
            for (int i = 0; i < 256; i++) o[i] = d * (float)(int8_t)blk[4 + i];
            break;
        }
        case TLMO_MXFP4: {
            const uint8_t *blk = s + 17 * b;
            uint8_t e = blk[0];
            float sc = e == 255 ? NAN : (e == 0 ? float_of(0x00400000u) : float_of((uint32_t)e << 23));
            for (int j = 0; j < 16; j++) {
                o[j] = 0.5f * (float)k_e2m1x2_deq(blk[1 + j] & 15) * sc;
                o[j + 16] = 0.5f * (float)k_e2m1x2_deq(blk[1 + j] >> 4) * sc;
            }
            break;
        }
        default: return -1;
        }
    }
    return 0;
}

/* ---- per-block integer partials ---------------------------------------- */
/* Q4_K / Q5_K x Q8_K (src/lib/tlm_quant.c:814-842). */
static void blk_kq(const uint8_t *blk, const uint8_t *a, int q5, int32_t *isum, int32_t *msum) {
    const uint8_t *qh = blk + 16, *qs = q5 ? blk + 48 : blk + 16;
    const int8_t *x = (const int8_t *)(a + 4);
    int sc[8], mn[8];
    kq_scales(blk + 4, sc, mn);
    int32_t is = 0, ms = 0;
    for (int c = 0; c < 4; c++) {
        int32_t lo_sum = 0, hi_sum = 0;
        for (int l = 0; l < 32; l++) {
            int lo = qs[32 * c + l] & 15, hi = qs[32 * c + l] >> 4;
            if (q5) {
                lo |= ((qh[l] >> (2 * c)) & 1) << 4;
                hi |= ((qh[l] >> (2 * c + 1)) & 1) << 4;
            }
            lo_sum += lo * x[64 * c + l];
            hi_sum += hi * x[64 * c + 32 + l];
        }
        is += sc[2 * c] * lo_sum + sc[2 * c + 1] * hi_sum;
    }
    for (int s = 0; s < 8; s++) {
        int16_t b0, b1;
        memcpy(&b0, a + 260 + 4 * s, 2);
        memcpy(&b1, a + 262 + 4 * s, 2);
        ms += mn[s] * ((int32_t)b0 + (int32_t)b1);
    }
    *isum = is;
    *msum = ms;
}

/* Q6_K x Q8_K (src/lib/tlm_quant.c:856-882): unsigned 6-bit codes, the -32
 * folded out through the activation group sums. */
static int32_t blk_q6k(const uint8_t *blk, const uint8_t *a) {
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    const int8_t *x = (const int8_t *)(a + 4);
    int32_t gsum[16] = { 0 };
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 32; l++) {
            int A = ql[64 * h + l], B = ql[64 * h + 32 + l], C = qh[32 * h + l];
            int e = 128 * h + l;
            gsum[e / 16] += ((A & 15) | ((C & 3) << 4)) * x[e];
            gsum[(e + 32) / 16] += ((B & 15) | (((C >> 2) & 3) << 4)) * x[e + 32];
            gsum[(e + 64) / 16] += ((A >> 4) | (((C >> 4) & 3) << 4)) * x[e + 64];
            gsum[(e + 96) / 16] += ((B >> 4) | (((C >> 6) & 3) << 4)) * x[e + 96];
        }
    int32_t is = 0;
    for (int g = 0; g < 16; g++) {
        int16_t bs;
        memcpy(&bs, a + 260 + 2 * g, 2);
        is += (int32_t)sc[g] * (gsum[g] - 32 * (int32_t)bs);
    }
    return is;
}

/* Q8_0 weights x Q8_0 activations (src/lib/tlm_quant.c:778-792). */
static int32_t blk_q80(const uint8_t *blk, const uint8_t *a) {
    const int8_t *q = (const int8_t *)(blk + 2), *x = (const int8_t *)(a + 4);
    int32_t s = 0;
    for (int i = 0; i < 32; i++) s += (int32_t)q[i] * x[i];
    return s;
}

/* Q8_K weights x Q8_K activations (src/lib/tlm_quant.c:886-902). */
static int32_t blk_q8k(const uint8_t *blk, const uint8_t *a) {
    const int8_t *q = (const int8_t *)(blk + 4), *x = (const int8_t *)(a + 4);
    int32_t s = 0;
    for (int i = 0; i < 256; i++) s += (int32_t)q[i] * x[i];
    return s;
}

/* MXFP4 x Q8_0 (src/lib/tlm_quant.c:794-810): doubled E2M1 codes in the
 * integer dot, the 0.5 folded into the E8M0 scale. */
static const int8_t k_e2m1x2[16] = { 0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12 };

static int32_t blk_mxfp4(const uint8_t *blk, const uint8_t *a) {
    const int8_t *x = (const int8_t *)(a + 4);
    int32_t s = 0;
    for (int j = 0; j < 16; j++) {
        s += (int32_t)k_e2m1x2[blk[1 + j] & 15] * x[j];
        s += (int32_t)k_e2m1x2[blk[1 + j] >> 4] * x[j + 16];
    }
    return s;
}

/* 2^(e-128) with NaN for 255 (src/lib/tlm_quant.c:190-197). */
static float e8m0_half(uint8_t e) {
    uint32_t b;
    if (e == 255) b = 0x7FC00000u;
    else if (e >= 2) b = (uint32_t)(e - 1) << 23;
    else b = e ? 0x00400000u : 0x00200000u;
    return float_of(b);
}

int64_t tlmo_block_partials(int dt, const void *wrow, const void *act, int64_t n,
                            int32_t *isum, int32_t *msum) {
    int qk = tlmo_dtype_block(dt);
    if (qk <= 1 || n < 0 || n % qk) return -1;
    const uint8_t *w = (const uint8_t *)wrow, *a = (const uint8_t *)act;
    int64_t nb = n / qk;
    size_t bb = tlmo_dtype_block_bytes(dt);
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = w + bb * (size_t)b;
        int32_t is = 0, ms = 0;
        switch (dt) {
        case TLMO_Q4_K: blk_kq(blk, a + 292 * (size_t)b, 0, &is, &ms); break;
        case TLMO_Q5_K: blk_kq(blk, a + 292 * (size_t)b, 1, &is, &ms); break;
        case TLMO_Q6_K: is = blk_q6k(blk, a + 292 * (size_t)b); break;
        case TLMO_Q8_K: is = blk_q8k(blk, a + 292 * (size_t)b); break;
        case TLMO_Q8_0: is = blk_q80(blk, a + 36 * (size_t)b); break;
        case TLMO_MXFP4: is = blk_mxfp4(blk, a + 36 * (size_t)b); break;
        default: return -1;
        }
        isum[b] = is;
        msum[b] = ms;
    }
    return nb;
}

/* ---- float dots: lane i mod 32, fixed tree (src/lib/tlm_quant.c:724-770) */
static float tree32(const float *r) {
    float a[16], b[8], c[4];
    for (int l = 0; l < 16; l++) a[l] = r[l] + r[l + 16];
    for (int l = 0; l < 8; l++) b[l] = a[l] + a[l + 8];
    for (int l = 0; l < 4; l++) c[l] = b[l] + b[l + 4];
    return (c[0] + c[2]) + (c[1] + c[3]);
}

static float dot_float(int dt, const uint8_t *w, const float *x, int64_t n) {
    float lanes[32] = { 0 };
    for (int64_t i = 0; i < n; i++) {
        float wi;
        if (dt == TLMO_F32) wi = rdf32(w + 4 * i);
        else if (dt == TLMO_F16) wi = f16_at(w + 2 * i);
        else wi = tlmo_bf16_to_f32(rd16(w + 2 * i));
        lanes[i & 31] = fmaf(wi, x[i], lanes[i & 31]);
    }
    return tree32(lanes);
}

/* ---- one row dot (the numerics contract, src/lib/tlm_quant.h:113-128) -- */
float tlmo_vec_dot(int dt, const void *wrow, const void *act, int64_t n) {
    int qk = tlmo_dtype_block(dt);
    if (!qk || n < 0 || n % qk) return NAN;
    const uint8_t *w = (const uint8_t *)wrow, *a = (const uint8_t *)act;
    if (qk == 1) return dot_float(dt, w, (const float *)act, n);
    int64_t nb = n / qk;
    size_t bb = tlmo_dtype_block_bytes(dt);
    float acc = 0.0f;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = w + bb * (size_t)b;
        int32_t is = 0, ms = 0;
        switch (dt) {
        case TLMO_Q4_K: case TLMO_Q5_K: {
            const uint8_t *ab = a + 292 * (size_t)b;
            blk_kq(blk, ab, dt == TLMO_Q5_K, &is, &ms);
            float da = rdf32(ab);
            float dA = f16_at(blk) * da, dM = f16_at(blk + 2) * da;
            acc = fmaf(dA, (float)is, acc);
            acc = fmaf(-dM, (float)ms, acc);
            break;
        }
        case TLMO_Q6_K: {
            const uint8_t *ab = a + 292 * (size_t)b;
            is = blk_q6k(blk, ab);
            acc = fmaf(f16_at(blk + 208) * rdf32(ab), (float)is, acc);
            break;
        }
        case TLMO_Q8_K: {
            const uint8_t *ab = a + 292 * (size_t)b;
            is = blk_q8k(blk, ab);
            acc = fmaf(rdf32(blk) * rdf32(ab), (float)is, acc);
            break;
        }
        case TLMO_Q8_0: {
            const uint8_t *ab = a + 36 * (size_t)b;
            is = blk_q80(blk, ab);
            acc = fmaf(f16_at(blk) * rdf32(ab), (float)is, acc);
            break;
        }
        case TLMO_MXFP4: {
            const uint8_t *ab = a + 36 * (size_t)b;
            is = blk_mxfp4(blk, ab);
            acc = fmaf(e8m0_half(blk[0]) * rdf32(ab), (float)is, acc);
            break;
        }
        default: return NAN;
        }
    }
    return acc;
}

/* src/lib/tlm_quant.c:1119-1143 (rows r0..r1 of a strided matrix; NaN rows
 * on a bad dtype or width). */
void tlmo_matvec_rows(int dt, const void *W, size_t row_bytes, const void *act, float *y,
                      int64_t n, int64_t r0, int64_t r1) {
    int qk = tlmo_dtype_block(dt);
    const uint8_t *base = (const uint8_t *)W;
    for (int64_t r = r0; r < r1; r++)
        y[r] = (!qk || n < 0 || n % qk) ? NAN : tlmo_vec_dot(dt, base + (size_t)r * row_bytes, act, n);
}

/* ---- expf ---------------------------------------------------------------- */
static int g_expf_mode;

void tlmo_set_expf_mode(int mode) { g_expf_mode = mode ? 1 : 0; }
int  tlmo_get_expf_mode(void) { return g_expf_mode; }

/* Correctly rounded expf: Cody-Waite reduction by ln 2 (two-part constant),
 * the degree-13 Taylor polynomial of exp(r) on |r| <= ln2/2 in double with
 * fma (truncation < 2^-57), scaling by 2^k, one rounding to float. Checked
 * exhaustively against (float)expl over all 2^32 inputs. This is the same
 * operation sequence as the CUDA tier's device function. */
float tlmo_expf_cr(float xf) {
    if (xf != xf) return xf + xf;
    if (xf > 88.72283935546875f) return INFINITY;
    if (xf < -103.97283935546875f) return 0.0f;
    double x = (double)xf;
    double k = nearbyint(x * 0x1.71547652b82fep+0);
    double r = fma(-k, 0x1.62e42feep-1, x);
    r = fma(-k, 0x1.a39ef35793c76p-33, r);
    double p = 0x1.6124613a86d09p-33;
    p = fma(p, r, 0x1.1eed8eff8d898p-29);
    p = fma(p, r, 0x1.ae64567f544e4p-26);
    p = fma(p, r, 0x1.27e4fb7789f5cp-22);
    p = fma(p, r, 0x1.71de3a556c734p-19);
    p = fma(p, r, 0x1.a01a01a01a01ap-16);
    p = fma(p, r, 0x1.a01a01a01a01ap-13);
    p = fma(p, r, 0x1.6c16c16c16c17p-10);
    p = fma(p, r, 0x1.1111111111111p-7);
    p = fma(p, r, 0x1.5555555555555p-5);
    p = fma(p, r, 0x1.5555555555555p-3);
    p = fma(p, r, 0x1p-1);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    uint64_t sb = (uint64_t)((int64_t)k + 1023) << 52;
    double s;
    memcpy(&s, &sb, 8);
    return (float)(p * s);
}

float tlmo_expf(float x) { return g_expf_mode ? tlmo_expf_cr(x) : expf(x); }

static float silu_f(float x) { return x / (1.0f + tlmo_expf(-x)); }          /* tlm_model.c:171 */
static float sigmoid_f(float x) { return 1.0f / (1.0f + tlmo_expf(-x)); }    /* tlm_model.c:172 */

/* ---- routing (src/lib/tlm_model.c:776-839) ------------------------------ */
/* Top-k by value among unmasked entries: ties -> lowest index, NaN skipped;
 * with nothing finite left, the lowest unmasked unused index. */
static void top_k(const float *v, const uint8_t *mask, int E, int k, int *ids) {
    for (int r = 0; r < k; r++) {
        int best = -1;
        for (int e = 0; e < E; e++) {
            if ((mask && mask[e]) || v[e] != v[e]) continue;
            int used = 0;
            for (int q = 0; q < r; q++) used |= ids[q] == e;
            if (used) continue;
            if (best < 0 || v[e] > v[best]) best = e;
        }
        for (int e = 0; best < 0 && e < E; e++) {
            if (mask && mask[e]) continue;
            int used = 0;
            for (int q = 0; q < r; q++) used |= ids[q] == e;
            if (!used) best = e;
        }
        ids[r] = best < 0 ? 0 : best;
    }
}

void tlmo_route(int router, const float *logits, const uint8_t *mask, const float *bias,
                int E, int k, float routed_scale, int *ids, float *w) {
    float *p = (float *)malloc((size_t)E * sizeof(float));
    float *v = (float *)malloc((size_t)E * sizeof(float));
    if (router == 2) {
        for (int e = 0; e < E; e++) {
            p[e] = sigmoid_f(logits[e]);
            v[e] = p[e] + (bias ? bias[e] : 0.0f);
        }
        top_k(v, mask, E, k, ids);
        double s = 0.0;
        for (int r = 0; r < k; r++) s += (double)p[ids[r]];
        float inv = (float)(1.0 / (s + 1e-20));
        for (int r = 0; r < k; r++) w[r] = p[ids[r]] * inv * routed_scale;
    } else {
        float mx = -INFINITY;
        for (int e = 0; e < E; e++)
            if (!(mask && mask[e]) && logits[e] > mx) mx = logits[e];
        double s = 0.0;
        for (int e = 0; e < E; e++) {
            int off = (mask && mask[e]) || logits[e] != logits[e] || mx == -INFINITY;
            p[e] = off ? 0.0f : tlmo_expf(logits[e] - mx);
            s += (double)p[e];
        }
        float inv = s > 0.0 ? (float)(1.0 / s) : 0.0f;
        for (int e = 0; e < E; e++) p[e] *= inv;
        top_k(p, mask, E, k, ids);
        for (int r = 0; r < k; r++) w[r] = p[ids[r]];
        if (router == 0) {
            double t = 0.0;
            for (int r = 0; r < k; r++) t += (double)w[r];
            if (t > 0.0) {
                float it = (float)(1.0 / t);
                for (int r = 0; r < k; r++) w[r] *= it;
            }
        }
        if (routed_scale != 1.0f)
            for (int r = 0; r < k; r++) w[r] *= routed_scale;
    }
    free(p);
    free(v);
}

/* ---- RMSNorm (src/lib/tlm_model.c:164-169) ------------------------------ */
void tlmo_rmsnorm(float *out, const float *x, const float *w, int64_t n, float eps) {
    double ss = 0.0;
    for (int64_t i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    float r = 1.0f / sqrtf((float)(ss / (double)n) + eps);
    for (int64_t i = 0; i < n; i++) out[i] = x[i] * r * w[i];
}

/* SwiGLU FFN of one expert-shaped block: gate/up [dh x D], down [D x dh]. */
static void swiglu_block(int D, int dh, const int dt[3], const uint8_t *const mats[3],
                         const float *x, float *hbuf, float *out) {
    float *g = (float *)malloc(sizeof(float) * (size_t)dh * 2);
    float *u = g + dh;
    int kx = tlmo_act_kind_for(dt[0]), ku = tlmo_act_kind_for(dt[1]), kd = tlmo_act_kind_for(dt[2]);
    void *ax = malloc(tlmo_qact_bytes(kx, D) + 64);
    void *au = malloc(tlmo_qact_bytes(ku, D) + 64);
    void *ah = malloc(tlmo_qact_bytes(kd, dh) + 64);
    tlmo_quantize_act(kx, x, D, ax);
    tlmo_quantize_act(ku, x, D, au);
    tlmo_matvec_rows(dt[0], mats[0], tlmo_row_bytes(dt[0], D), ax, g, D, 0, dh);
    tlmo_matvec_rows(dt[1], mats[1], tlmo_row_bytes(dt[1], D), au, u, D, 0, dh);
    for (int i = 0; i < dh; i++) hbuf[i] = silu_f(g[i]) * u[i];
    tlmo_quantize_act(kd, hbuf, dh, ah);
    tlmo_matvec_rows(dt[2], mats[2], tlmo_row_bytes(dt[2], dh), ah, out, dh, 0, D);
    free(g); free(ax); free(au); free(ah);
}

int tlmo_expert_ffn(const tlmo_geom *g, const tlmo_expert *experts, const uint8_t *mask,
                    const float *bias, const float *x, const float *logits, float *ffn,
                    int *ids_out, float *w_out, float *eo_out, float *h_out) {
    int D = g->d_model, de = g->d_expert, k = g->top_k, E = g->n_experts;
    if (k <= 0 || k > E || k > 64) return -1;
    int ids[64];
    float w[64];
    tlmo_route(g->router, logits, mask, bias, E, k, g->routed_scale, ids, w);
    float *eo = (float *)malloc(sizeof(float) * (size_t)D * (size_t)k);
    float *hb = (float *)malloc(sizeof(float) * (size_t)de * (size_t)k);
    for (int r = 0; r < k; r++) {
        const tlmo_expert *X = &experts[ids[r]];
        const uint8_t *mats[3] = { X->base + X->off[0], X->base + X->off[1], X->base + X->off[2] };
        swiglu_block(D, de, X->dt, mats, x, hb + (size_t)r * de, eo + (size_t)r * D);
    }
    /* combine in ascending rank order: c = w*eo rounded, then added */
    for (int i = 0; i < D; i++) ffn[i] = 0.0f;
    for (int r = 0; r < k; r++)
        for (int i = 0; i < D; i++) {
            float c = w[r] * eo[(size_t)r * D + i];
            ffn[i] += c;
        }
    if (ids_out) memcpy(ids_out, ids, sizeof(int) * (size_t)k);
    if (w_out) memcpy(w_out, w, sizeof(float) * (size_t)k);
    if (eo_out) memcpy(eo_out, eo, sizeof(float) * (size_t)D * (size_t)k);
    if (h_out) memcpy(h_out, hb, sizeof(float) * (size_t)de * (size_t)k);
    free(eo);
    free(hb);
    return 0;
}

int tlmo_moe_layer(const tlmo_geom *g, const tlmo_layer *L, float *h, int *ids, float *w) {
    return tlmo_moe_layer_ex(g, L, h, ids, w, NULL);
}

int tlmo_moe_layer_ex(const tlmo_geom *g, const tlmo_layer *L, float *h, int *ids, float *w, float *onorm) {
    int D = g->d_model, E = g->n_experts, k = g->top_k;
    float *xb = (float *)malloc(sizeof(float) * (size_t)D);
    float *ffn = (float *)malloc(sizeof(float) * (size_t)D);
    float *logits = (float *)malloc(sizeof(float) * (size_t)(E > 0 ? E : 1));
    tlmo_rmsnorm(xb, h, L->ffn_norm, D, g->norm_eps);
    if (L->has_dense) {   /* tlm_model.c:947-964: SwiGLU block, h += ffn, no router */
        float *hb = (float *)malloc(sizeof(float) * (size_t)L->d_ffn);
        const uint8_t *mats[3] = { (const uint8_t *)L->dn_w[0], (const uint8_t *)L->dn_w[1],
                                   (const uint8_t *)L->dn_w[2] };
        swiglu_block(D, L->d_ffn, L->dn_dt, mats, xb, hb, ffn);
        for (int i = 0; i < D; i++) h[i] += ffn[i];
        free(hb); free(xb); free(ffn); free(logits);
        return 0;
    }
    for (int i = 0; i < D; i++) ffn[i] = 0.0f;
    int rc = 0;
    if (E > 0) {
        int kr = tlmo_act_kind_for(L->router_dt);
        void *ar = malloc(tlmo_qact_bytes(kr, D) + 64);
        tlmo_quantize_act(kr, xb, D, ar);
        tlmo_matvec_rows(L->router_dt, L->router_w, L->router_rb, ar, logits, D, 0, E);
        free(ar);
        int rid[64];
        float rw[64];
        float *eo = onorm ? (float *)malloc(sizeof(float) * (size_t)k * D) : NULL;
        rc = tlmo_expert_ffn(g, L->experts, L->mask, L->router_bias, xb, logits, ffn, rid, rw, eo, NULL);
        if (rc == 0) {
            if (ids) memcpy(ids, rid, sizeof(int) * (size_t)k);
            if (w) memcpy(w, rw, sizeof(float) * (size_t)k);
        }
        if (rc == 0 && onorm)
            for (int r = 0; r < k; r++) {
                double nn = 0.0;
                for (int i = 0; i < D; i++) {
                    float c = rw[r] * eo[(size_t)r * D + i];
                    nn += (double)c * (double)c;
                }
                onorm[r] = (float)sqrt(nn);
            }
        free(eo);
    }
    if (rc == 0 && L->has_shared && g->d_shared > 0) {
        int ds = g->d_shared;
        float *sh = (float *)malloc(sizeof(float) * (size_t)ds);
        float *so = (float *)malloc(sizeof(float) * (size_t)D);
        const uint8_t *mats[3] = { (const uint8_t *)L->sh_w[0], (const uint8_t *)L->sh_w[1],
                                   (const uint8_t *)L->sh_w[2] };
        swiglu_block(D, ds, L->sh_dt, mats, xb, sh, so);
        float gate = 1.0f;
        if (L->shared_gate_inp) {   /* tlm_model.c:1039-1044: sequential float sum */
            float d = 0.0f;
            for (int i = 0; i < D; i++) d += L->shared_gate_inp[i] * xb[i];
            gate = sigmoid_f(d);
        }
        for (int i = 0; i < D; i++) ffn[i] += gate * so[i];
        free(sh);
        free(so);
    }
    if (rc == 0)
        for (int i = 0; i < D; i++) h[i] += ffn[i];
    free(xb);
    free(ffn);
    free(logits);
    return rc;
}

/* ---- decode attention over a paged KV cache ------------------------------
 * Restates the reference's attn_heads (src/lib/tlm_model.c:683-718) for one
 * token: for head h (kv head h / (H / KV)), scores d_t = (sum_i q_i k_ti in
 * ascending i) * (1 / sqrtf(hd)); p_t = expf(d_t - max); sum in double in
 * ascending t; inv = (float)(1 / sum); out_i = sum_t (p_t * inv) * v_ti in
 * ascending t. Positions live in pages: position t of kv head j is row
 * t % page of page page_table[t / page], pages laid out [KV][page][hd]. */
void tlmo_decode_attention(const float *q, const float *kp, const float *vp, const int32_t *page_table, int page,
                           int T, int H, int KV, int hd, float *out) {
    const int grp = H / KV;
    const float scale = 1.0f / sqrtf((float)hd);
    float *s = (float *)malloc(sizeof(float) * (size_t)T);
    for (int h = 0; h < H; h++) {
        const int kvh = h / grp;
        const float *qh = q + (size_t)h * hd;
        float mx = -INFINITY;
        for (int t = 0; t < T; t++) {
            const size_t row = (((size_t)page_table[t / page] * KV + kvh) * page + (size_t)(t % page)) * hd;
            float d = 0.0f;
            for (int i = 0; i < hd; i++) d += qh[i] * kp[row + i];
            d *= scale;
            s[t] = d;
            if (d > mx) mx = d;
        }
        double sum = 0.0;
        for (int t = 0; t < T; t++) {
            float p = tlmo_expf(s[t] - mx);
            s[t] = p;
            sum += (double)p;
        }
        const float inv = (float)(1.0 / sum);
        float *o = out + (size_t)h * hd;
        for (int i = 0; i < hd; i++) o[i] = 0.0f;
        for (int t = 0; t < T; t++) {
            const size_t row = (((size_t)page_table[t / page] * KV + kvh) * page + (size_t)(t % page)) * hd;
            const float p = s[t] * inv;
            for (int i = 0; i < hd; i++) o[i] += p * vp[row + i];
        }
    }
    free(s);
}
