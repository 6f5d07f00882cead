// tlmg_attn.cu - decode attention over a paged KV cache in HBM, and the
// paged K/V append.
//
// Reference: attn_heads (src/lib/tlm_model.c:683-719) and the K/V write of
// attention() (src/lib/tlm_model.c:730-763). The reference keeps one f32 KV
// per sequence, [layer][kv_head][max_ctx][head_dim]. Here one layer's cache
// is a pool of pages [n_pages][KV][page][hd] (f32 or bf16): position t of a
// sequence lives in page table[t / page], row t % page, so sequences grow
// page by page and share one pool.
//
// Two algorithms over the same layout:
//  exact  the reference's arithmetic order. Per head: serial f32 dot q.k
//         (each product rounded, then added), times 1/sqrtf(hd); max;
//         p = expf(s - max); serial double sum in ascending t;
//         inv = (float)(1/sum); out[i] = serial f32 sum over ascending t of
//         (p*inv)*v[t][i]. Bit-identical to the reference given the same
//         expf (correctly rounded here). Two kernels: scores (one thread per
//         position, all heads of a KV group), then one CTA per head for the
//         softmax and the output chains. Latency-bound: a serial double
//         chain and a serial float chain of T adds per head.
//  split  flash-decoding: positions are cut into spans; one CTA per
//         (span, KV head) keeps a running max / sum / output over tiles of
//         K and V staged in shared memory by cp.async (two stages), and a
//         merge kernel combines the spans. Reassociated, so equal to the
//         reference within float rounding, not bit for bit.
//
// A page-table entry outside [0, n_pages) is never dereferenced: its rows
// read as NaN (exact) or poison the head's result with NaN (split).
#include <algorithm>
#include <cmath>
#include <utility>
#include <vector>
#include <cuda_bf16.h>

#include "tlmg_dev.cuh"
#include "tlmg_internal.h"

namespace tlmg {
namespace {

constexpr int XS_ROWS = 64;          // exact scores: positions per CTA
constexpr int PSM_MAX = 16384;       // exact softmax: p kept in shared memory up to this T
constexpr int SPLIT_THREADS = 128;
constexpr int MAX_GRP = 16;          // query heads per KV head

__device__ __forceinline__ bool bad_page(int32_t e, int n_pages) { return e < 0 || e >= n_pages; }

// Four consecutive elements as floats.
__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16 *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    return make_float4(bf16_to_f32(u.x & 0xFFFFu), bf16_to_f32(u.x >> 16), bf16_to_f32(u.y & 0xFFFFu),
                       bf16_to_f32(u.y >> 16));
}
__device__ __forceinline__ float ld1(const float *p) { return *p; }
__device__ __forceinline__ float ld1(const __nv_bfloat16 *p) {
    return bf16_to_f32(*reinterpret_cast<const uint16_t *>(p));
}
__device__ __forceinline__ float2 ld2(const float *p) { return *reinterpret_cast<const float2 *>(p); }
__device__ __forceinline__ float2 ld2(const __nv_bfloat16 *p) {
    const uint32_t u = *reinterpret_cast<const uint32_t *>(p);
    return make_float2(bf16_to_f32(u & 0xFFFFu), bf16_to_f32(u >> 16));
}

__device__ __forceinline__ uint32_t saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
// 16-byte copy global -> shared; src_bytes 0 fills zeros and reads nothing.
__device__ __forceinline__ void cp16(void *dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Row offsets (elements) of positions [tb, tb + rows) of KV head kvh into
// ro[0..rows); -1 for a position at or past T_end or on a bad page.
__device__ __forceinline__ void row_offsets(const int32_t *__restrict__ table, int n_pages, int page, int KV, int kvh,
                                            int hd, int tb, int rows, int T_end, long long *ro, int *bad, int tid,
                                            int nt) {
    for (int r = tid; r < rows; r += nt) {
        const int t = tb + r;
        long long off = -1;
        if (t < T_end) {
            const int32_t e = table[t / page];
            if (bad_page(e, n_pages)) *bad = 1;
            else off = (long long)((((size_t)e * KV + kvh) * page + (size_t)(t % page)) * hd);
        }
        ro[r] = off;
    }
}

// Stages `rows` rows (row_b bytes each, at byte stride ld_b in shared
// memory) of pool; rows with offset -1 are zero-filled.
template <typename KT>
__device__ __forceinline__ void stage_rows(uint8_t *dst, int ld_b, const KT *__restrict__ pool, const long long *ro,
                                           int rows, int row_b, int tid, int nt) {
    const int c16 = row_b / 16;
    for (int idx = tid; idx < rows * c16; idx += nt) {
        const int r = idx / c16, c = idx - r * c16;
        const long long off = ro[r];
        const uint8_t *src = reinterpret_cast<const uint8_t *>(pool + (off < 0 ? 0 : off)) + 16 * c;
        cp16(dst + (size_t)r * ld_b + 16 * c, src, off < 0 ? 0 : 16);
    }
}

// ---- exact ---------------------------------------------------------------
// Scores of one KV group's heads for XS_ROWS positions: s[h][t] =
// (serial sum_i q[h][i] * k[t][i]) * scale. grid (ceil(T / XS_ROWS), KV).
template <typename KT>
__global__ void __launch_bounds__(XS_ROWS) k_attn_scores(const float *__restrict__ q, const KT *__restrict__ kpool,
                                                         const int32_t *__restrict__ table, int n_pages, int page,
                                                         int T, const int32_t *__restrict__ dT, int H, int KV,
                                                         int hd, float scale, float *__restrict__ s) {
    pdl_enter();
    if (dT) T = *dT;   // graph replay: the position count lives in device memory
    extern __shared__ float4 sm4[];
    __shared__ long long ro[XS_ROWS];
    __shared__ int bad_s;
    float *sm = reinterpret_cast<float *>(sm4);
    const int grp = H / KV, kvh = blockIdx.y, t0 = blockIdx.x * XS_ROWS, tid = threadIdx.x;
    const int row_b = hd * (int)sizeof(KT) + 16;    // padded: thread-per-row reads are conflict-free
    float *qs = sm;                                  // [grp][hd]
    uint8_t *ks = reinterpret_cast<uint8_t *>(sm + grp * hd);   // [XS_ROWS][row_b] raw K rows
    row_offsets(table, n_pages, page, KV, kvh, hd, t0, XS_ROWS, T, ro, &bad_s, tid, XS_ROWS);
    for (int i = tid; i < grp * hd; i += XS_ROWS) qs[i] = q[(size_t)kvh * grp * hd + i];
    __syncthreads();
    stage_rows(ks, row_b, kpool, ro, XS_ROWS, hd * (int)sizeof(KT), tid, XS_ROWS);
    cp_commit();
    cp_wait0();
    __syncthreads();
    const int t = t0 + tid;
    if (t >= T) return;
    if (ro[tid] < 0) {   // a bad page: the reference would read garbage; report NaN
        for (int h = 0; h < grp; h++) s[(size_t)(kvh * grp + h) * T + t] = NAN;
        return;
    }
    const KT *kr = reinterpret_cast<const KT *>(ks + (size_t)tid * row_b);
    for (int h0 = 0; h0 < grp; h0 += 4) {
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
        const float *q0 = qs + h0 * hd;
        for (int i = 0; i < hd; i += 4) {
            const float4 kv = ld4(kr + i);
#define TLMG_DOT4(D, J)                                                                                 \
    if (h0 + J < grp) {                                                                                 \
        const float4 qv = *reinterpret_cast<const float4 *>(q0 + J * hd + i);                           \
        D = __fadd_rn(D, __fmul_rn(qv.x, kv.x));                                                        \
        D = __fadd_rn(D, __fmul_rn(qv.y, kv.y));                                                        \
        D = __fadd_rn(D, __fmul_rn(qv.z, kv.z));                                                        \
        D = __fadd_rn(D, __fmul_rn(qv.w, kv.w));                                                        \
    }
            TLMG_DOT4(d0, 0)
            TLMG_DOT4(d1, 1)
            TLMG_DOT4(d2, 2)
            TLMG_DOT4(d3, 3)
#undef TLMG_DOT4
        }
        float *sr = s + (size_t)(kvh * grp + h0) * T + t;
        sr[0] = __fmul_rn(d0, scale);
        if (h0 + 1 < grp) sr[(size_t)T] = __fmul_rn(d1, scale);
        if (h0 + 2 < grp) sr[2 * (size_t)T] = __fmul_rn(d2, scale);
        if (h0 + 3 < grp) sr[3 * (size_t)T] = __fmul_rn(d3, scale);
    }
}

constexpr int XO_ROWS = 64;   // exact output: V rows per staged tile

// V-tile buffers of the exact output kernel: as many as fit beside the p
// array (up to PSM_MAX floats) in 227 KB, at most 4.
template <typename KT, int HD>
constexpr int xo_stages() {
    return (227 * 1024 - PSM_MAX * 4) / (XO_ROWS * HD * (int)sizeof(KT)) >= 4 ? 4 : 2;
}

// Softmax and output of one head (grid H, HD threads, thread i owns column
// i): the reference's max, expf, serial double sum and serial output
// chains. V is staged in 64-row tiles by cp.async, NST tiles in flight, the
// page-table entries of each tile loaded one tile earlier; the first tiles'
// copies run under the expf pass and the serial double sum, and the output
// chain reads shared memory only.
template <typename KT, int HD, int NST>
__global__ void __launch_bounds__(HD) k_attn_out_exact(const KT *__restrict__ vpool, const int32_t *__restrict__ table,
                                                       int n_pages, int page, int T, const int32_t *__restrict__ dT,
                                                       int psm_cap, int H, int KV, float *__restrict__ s,
                                                       float *__restrict__ out) {
    pdl_enter();
    if (dT) T = *dT;
    constexpr int ROW_B = HD * (int)sizeof(KT);
    constexpr int C16 = ROW_B / 16;
    extern __shared__ float4 sm4[];
    __shared__ float red[33];
    __shared__ int bad_s;
    const int h = blockIdx.x, kvh = h / (H / KV), tid = threadIdx.x;
    uint8_t *stage = reinterpret_cast<uint8_t *>(sm4);                              // [NST][XO_ROWS][ROW_B]
    float *psm = reinterpret_cast<float *>(stage + (size_t)NST * XO_ROWS * ROW_B);  // [T] when T <= psm_cap
    float *srow = s + (size_t)h * T;
    const int n_tiles = (T + XO_ROWS - 1) / XO_ROWS;
    if (tid == 0) bad_s = 0;
    __syncthreads();
    // copies: piece idx = tid + HD k is row idx / C16, column idx % C16 (a
    // warp's copies are contiguous); row offsets in ro[stage][row] are
    // written one iteration ahead from the page-table entry loaded the
    // iteration before (te, threads < XO_ROWS)
    __shared__ long long ro[NST][XO_ROWS];
    int32_t te = -1;
    auto load_te = [&](int tile) {
        const int t = tile * XO_ROWS + tid;
        te = tid < XO_ROWS && tile < n_tiles && t < T ? __ldg(table + t / page) : -1;
    };
    auto put_ro = [&](int tile) {
        if (tid < XO_ROWS) {
            const int t = tile * XO_ROWS + tid;
            long long o = -1;
            if (tile < n_tiles && t < T) {
                if (bad_page(te, n_pages)) bad_s = 1;
                else o = (long long)((((size_t)te * KV + kvh) * page + (size_t)(t % page)) * HD);
            }
            ro[tile % NST][tid] = o;
        }
    };
    auto issue = [&](int tile) {
        if (tile < n_tiles) {
            uint8_t *vd = stage + (size_t)(tile % NST) * XO_ROWS * ROW_B;
            const long long *rr = ro[tile % NST];
#pragma unroll
            for (int k = 0; k < XO_ROWS * C16 / HD; k++) {
                const int idx = tid + HD * k, r = idx / C16, c = idx - r * C16;
                const long long o = rr[r];
                const size_t oo = o < 0 ? 0 : (size_t)o;
                cp16(vd + r * ROW_B + 16 * c, reinterpret_cast<const uint8_t *>(vpool + oo) + 16 * c, o < 0 ? 0 : 16);
            }
        }
        cp_commit();
    };
#pragma unroll
    for (int k = 0; k < NST - 1; k++) {
        load_te(k);
        put_ro(k);
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NST - 1; k++) issue(k);
    load_te(NST - 1);
    // max: the first strictly greater value wins, NaN never does (as the
    // serial scan; ties between +0 and -0 give the same p)
    float mx = -INFINITY;
    for (int t = tid; t < T; t += HD) {
        const float d = srow[t];
        if (d > mx) mx = d;
    }
    for (int o = 16; o; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, mx, o);
        if (v > mx) mx = v;
    }
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = -INFINITY;
        for (int w = 0; w < HD / 32; w++)
            if (red[w] > m) m = red[w];
        red[32] = m;
    }
    __syncthreads();
    mx = red[32];
    float *pp = T <= psm_cap ? psm : srow;
    for (int t = tid; t < T; t += HD) pp[t] = cr_expf(__fsub_rn(srow[t], mx));
    __syncthreads();
    if (tid == 0) {
        double sum = 0.0;
        int t = 0;
        for (; t + 8 <= T; t += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = pp[t + j];
#pragma unroll
            for (int j = 0; j < 8; j++) sum = __dadd_rn(sum, (double)v[j]);
        }
        for (; t < T; t++) sum = __dadd_rn(sum, (double)pp[t]);
        red[0] = __double2float_rn(__ddiv_rn(1.0, sum));
    }
    __syncthreads();
    const float inv = red[0];
    float o = 0.0f;
    for (int tile = 0; tile < n_tiles; tile++) {
        put_ro(tile + NST - 1);
        load_te(tile + NST);
        asm volatile("cp.async.wait_group %0;" ::"n"(NST - 2) : "memory");
        __syncthreads();
        issue(tile + NST - 1);
        const KT *vt = reinterpret_cast<const KT *>(stage + (size_t)(tile % NST) * XO_ROWS * ROW_B) + tid;
        const float *pt = pp + tile * XO_ROWS;
        const int rows = min(XO_ROWS, T - tile * XO_ROWS);
        int r = 0;
        for (; r + 8 <= rows; r += 8) {
            float pv[8], vv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                pv[j] = __fmul_rn(pt[r + j], inv);
                vv[j] = ld1(vt + (size_t)(r + j) * HD);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) o = __fadd_rn(o, __fmul_rn(pv[j], vv[j]));
        }
        for (; r < rows; r++) o = __fadd_rn(o, __fmul_rn(__fmul_rn(pt[r], inv), ld1(vt + (size_t)r * HD)));
    }
    cp_wait0();
    __syncthreads();
    out[(size_t)h * HD + tid] = bad_s ? NAN : o;
}

// ---- split ---------------------------------------------------------------
struct SplitGeom {
    int tr;       // rows per tile
    int span;     // positions per CTA (a multiple of tr)
    int n_span;
};

// One CTA per (span, KV head). Scores in log2 units (q pre-scaled by
// scale * log2(e)); running max m, sum l and output o per head over the
// span's tiles; partials pm/pl [H][n_span], po [H][n_span][hd].
template <typename KT>
__global__ void __launch_bounds__(SPLIT_THREADS) k_attn_split(const float *__restrict__ q,
                                                              const KT *__restrict__ kpool,
                                                              const KT *__restrict__ vpool,
                                                              const int32_t *__restrict__ table, int n_pages, int page,
                                                              int T, const int32_t *__restrict__ dT, int H, int KV,
                                                              int hd, int tr, int span,
                                                              int n_span, float qscale, float *__restrict__ pm,
                                                              float *__restrict__ pl, float *__restrict__ po) {
    pdl_enter();
    extern __shared__ float4 sm4[];
    if (dT) T = *dT;
    const int grp = H / KV, kvh = blockIdx.y, sidx = blockIdx.x, tid = threadIdx.x;
    asm volatile("griddepcontrol.launch_dependents;");   // the merge grid may start and wait
    const int row_b = hd * (int)sizeof(KT) + 16;              // padded row bytes in shared memory
    const int sp_ld = grp + 1;
    float *qs = reinterpret_cast<float *>(sm4);               // [grp][hd], pre-scaled
    float *sp = qs + grp * hd;                                // [tr][grp + 1] scores -> p
    float *m_s = sp + tr * sp_ld;                             // [grp] running max
    float *l_s = m_s + MAX_GRP;                               // [grp] running sum
    float *a_s = l_s + MAX_GRP;                               // [grp] rescale of this tile
    int *bad_s = reinterpret_cast<int *>(a_s + MAX_GRP);
    uint8_t *stage = reinterpret_cast<uint8_t *>(sm4) +
                     ((size_t)(grp * hd + tr * sp_ld + 3 * MAX_GRP + 4) * 4 + 15) / 16 * 16;
    const size_t mat_b = (size_t)tr * row_b;                  // one matrix tile
    for (int i = tid; i < grp * hd; i += SPLIT_THREADS) qs[i] = q[(size_t)kvh * grp * hd + i] * qscale;
    if (tid < MAX_GRP) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.f;
    }
    if (tid == 0) *bad_s = 0;
    __syncthreads();
    const int t_lo = sidx * span, t_hi = min(T, t_lo + span);
    const int n_tiles = (t_hi - t_lo + tr - 1) / tr;
    __shared__ long long ro_s[2][64];
    auto issue = [&](int tile, int buf) {
        uint8_t *kd = stage + (size_t)buf * 2 * mat_b, *vd = kd + mat_b;
        row_offsets(table, n_pages, page, KV, kvh, hd, t_lo + tile * tr, tr, t_hi, ro_s[buf], bad_s, tid,
                    SPLIT_THREADS);
        __syncthreads();
        stage_rows(kd, row_b, kpool, ro_s[buf], tr, hd * (int)sizeof(KT), tid, SPLIT_THREADS);
        stage_rows(vd, row_b, vpool, ro_s[buf], tr, hd * (int)sizeof(KT), tid, SPLIT_THREADS);
        cp_commit();
    };
    // output ownership: column pair cp, heads hs, hs + HS2, ...
    const int np2 = hd / 2, HS2 = SPLIT_THREADS / np2, cpi = tid % np2, hs = tid / np2;
    float acc[MAX_GRP][2];
#pragma unroll
    for (int j = 0; j < MAX_GRP; j++) acc[j][0] = acc[j][1] = 0.f;
    // score ownership: row r, heads hq, hq + HSs, ...
    const int HSs = SPLIT_THREADS / tr, r_own = tid % tr, hq = tid / tr;
    const int warp = tid >> 5, lane = tid & 31;

    if (n_tiles > 0) issue(0, 0);
    for (int tile = 0; tile < n_tiles; tile++) {
        const int buf = tile & 1;
        if (tile + 1 < n_tiles) {
            issue(tile + 1, buf ^ 1);
            cp_wait1();
        } else {
            cp_wait0();
        }
        __syncthreads();
        const uint8_t *kt = stage + (size_t)buf * 2 * mat_b, *vt = kt + mat_b;
        const int tb = t_lo + tile * tr;
        // scores
        {
            const KT *kr = reinterpret_cast<const KT *>(kt + (size_t)r_own * row_b);
            float d[MAX_GRP / 2];
#pragma unroll
            for (int j = 0; j < MAX_GRP / 2; j++) d[j] = 0.f;
            for (int i = 0; i < hd; i += 4) {
                const float4 kv = ld4(kr + i);
#pragma unroll
                for (int j = 0; j < MAX_GRP / 2; j++) {
                    const int h = hq + j * HSs;
                    if (h < grp) {
                        const float4 qv = *reinterpret_cast<const float4 *>(qs + h * hd + i);
                        d[j] = __fmaf_rn(qv.x, kv.x, d[j]);
                        d[j] = __fmaf_rn(qv.y, kv.y, d[j]);
                        d[j] = __fmaf_rn(qv.z, kv.z, d[j]);
                        d[j] = __fmaf_rn(qv.w, kv.w, d[j]);
                    }
                }
            }
            const bool valid = tb + r_own < t_hi;
#pragma unroll
            for (int j = 0; j < MAX_GRP / 2; j++) {
                const int h = hq + j * HSs;
                if (h < grp) sp[r_own * sp_ld + h] = valid ? d[j] : -INFINITY;
            }
        }
        __syncthreads();
        // per head: tile max, rescale, p, tile sum (one warp per head)
        for (int h = warp; h < grp; h += SPLIT_THREADS / 32) {
            float tmax = -INFINITY;
            for (int r = lane; r < tr; r += 32) tmax = fmaxf(tmax, sp[r * sp_ld + h]);
            for (int o = 16; o; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
            const float m_old = m_s[h], m_new = fmaxf(m_old, tmax);
            const float alpha = m_new == -INFINITY ? 1.f : exp2f(m_old - m_new);
            float sum = 0.f;
            for (int r = lane; r < tr; r += 32) {
                const float p = m_new == -INFINITY ? 0.f : exp2f(sp[r * sp_ld + h] - m_new);
                sp[r * sp_ld + h] = p;
                sum += p;
            }
            for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) {
                m_s[h] = m_new;
                l_s[h] = l_s[h] * alpha + sum;
                a_s[h] = alpha;
            }
        }
        __syncthreads();
        // output
        {
#pragma unroll
            for (int j = 0; j < MAX_GRP; j++) {
                const int h = hs + j * HS2;
                if (h < grp) {
                    acc[j][0] *= a_s[h];
                    acc[j][1] *= a_s[h];
                }
            }
            // rows past the span's end hold p = 0 and zero-filled V
#pragma unroll 4
            for (int r = 0; r < tr; r++) {
                const float2 v = ld2(reinterpret_cast<const KT *>(vt + (size_t)r * row_b) + 2 * cpi);
                const float *pr = sp + r * sp_ld;
#pragma unroll
                for (int j = 0; j < MAX_GRP; j++) {
                    const int h = hs + j * HS2;
                    if (h < grp) {
                        const float p = pr[h];
                        acc[j][0] = __fmaf_rn(p, v.x, acc[j][0]);
                        acc[j][1] = __fmaf_rn(p, v.y, acc[j][1]);
                    }
                }
            }
        }
        __syncthreads();   // the next tile's copies overwrite this buffer
    }
    const bool bad = *bad_s != 0;
#pragma unroll
    for (int j = 0; j < MAX_GRP; j++) {
        const int h = hs + j * HS2;
        if (h < grp) {
            const size_t hh = (size_t)(kvh * grp + h) * n_span + sidx;
            float *o = po + hh * hd + 2 * cpi;
            o[0] = acc[j][0];
            o[1] = acc[j][1];
        }
    }
    if (tid < grp) {
        const size_t hh = (size_t)(kvh * grp + tid) * n_span + sidx;
        pm[hh] = bad ? NAN : m_s[tid];
        pl[hh] = l_s[tid];
    }
}

// ---- split on the tensor cores (bf16 pages) ---------------------------------
// mma.sync m16n8k16 (bf16 in, f32 accumulate) with the KV group's query heads
// as the M dimension. A KV group has at most 8 query heads, below the
// 64-row minimum of tcgen05.mma; the kernel is bound by HBM (two bytes of K
// or V per 8 multiply-adds), which this MMA shape clears with a wide margin.
// The 16 rows carry each head twice: rows 0..7 the bf16 high part of the
// operand (q, then p) and rows 8..15 its bf16 remainder, so q and p keep
// 16 significant bits and K / V are exact: the result stays within float
// rounding of the f32 arithmetic. One CTA (4 warps) per (span, KV head);
// K/V tiles of 64 positions are staged by cp.async in NST buffers; warp w
// owns rows 16w..16w+15 of each tile with its own running max / sum /
// output, and the four warps are merged through shared memory at the end.
constexpr int TC_ROWS = 64;

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(saddr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(saddr(p)));
}
// (hi, lo) bf16 pair words of two floats: hi = bf16(x), lo = bf16(x - hi).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

template <int HD, int NST>
__global__ void __launch_bounds__(128) k_attn_split_tc(const float *__restrict__ q,
                                                       const __nv_bfloat16 *__restrict__ kpool,
                                                       const __nv_bfloat16 *__restrict__ vpool,
                                                       const int32_t *__restrict__ table, int n_pages, int page, int lp,
                                                       int T, const int32_t *__restrict__ dT, int H, int KV, int span,
                                                       int n_span, float qscale,
                                                       float *__restrict__ pm, float *__restrict__ pl,
                                                       float *__restrict__ po) {
    pdl_enter();
    constexpr int ROW_B = HD * 2 + 16;           // padded row bytes in shared memory
    constexpr int MAT_B = TC_ROWS * ROW_B;
    constexpr int C16 = HD * 2 / 16;             // 16-byte pieces per row
    constexpr int NT = HD / 8;                   // output n-tiles
    extern __shared__ float4 sm4[];
    uint8_t *stage = reinterpret_cast<uint8_t *>(sm4);
    __shared__ int bad_s;
    if (dT) T = *dT;
    const int G = H / KV, kvh = blockIdx.y, sidx = blockIdx.x, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    asm volatile("griddepcontrol.launch_dependents;");   // the merge grid may start and wait
    if (tid == 0) bad_s = 0;
    __syncthreads();
    const int t_lo = sidx * span, t_hi = min(T, t_lo + span);
    const int n_tiles = (t_hi - t_lo + TC_ROWS - 1) / TC_ROWS;

    // Copies: piece idx = tid + 128 k is row idx / C16, 16-byte column
    // idx % C16 of the tile, so a warp's copies are contiguous. Row offsets
    // come from ro[stage][row], written one iteration ahead by thread `row`
    // from the page-table entry it loaded the iteration before (te): neither
    // the offsets nor the copies wait on the table.
    __shared__ long long ro[NST][TC_ROWS];
    int32_t te = -1;
    auto load_te = [&](int tile) {
        const int t = t_lo + tile * TC_ROWS + tid;
        te = tid < TC_ROWS && tile < n_tiles && t < t_hi ? __ldg(table + (t >> lp)) : -1;
    };
    auto put_ro = [&](int tile) {
        if (tid < TC_ROWS) {
            const int t = t_lo + tile * TC_ROWS + tid;
            long long o = -1;
            if (tile < n_tiles && t < t_hi) {
                if (bad_page(te, n_pages)) bad_s = 1;
                else o = (long long)((((size_t)te * KV + kvh) << lp) + (size_t)(t & (page - 1))) * HD;
            }
            ro[tile % NST][tid] = o;
        }
    };
    auto issue = [&](int tile) {   // after a barrier that follows put_ro(tile)
        if (tile < n_tiles) {
            uint8_t *kd = stage + (size_t)(tile % NST) * 2 * MAT_B, *vd = kd + MAT_B;
            const long long *rr = ro[tile % NST];
#pragma unroll
            for (int k = 0; k < TC_ROWS * C16 / 128; k++) {
                const int idx = tid + 128 * k, r = idx / C16, c = idx - r * C16;
                const long long o = rr[r];
                const size_t oo = o < 0 ? 0 : (size_t)o;
                const int nb = o < 0 ? 0 : 16;
                cp16(kd + r * ROW_B + 16 * c, reinterpret_cast<const uint8_t *>(kpool + oo) + 16 * c, nb);
                cp16(vd + r * ROW_B + 16 * c, reinterpret_cast<const uint8_t *>(vpool + oo) + 16 * c, nb);
            }
        }
        cp_commit();   // an empty group past the end keeps the group count uniform
    };

    float o_acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) o_acc[j][0] = o_acc[j][1] = o_acc[j][2] = o_acc[j][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

#pragma unroll
    for (int s = 0; s < NST - 1; s++) {
        load_te(s);
        put_ro(s);
    }
    __syncthreads();
#pragma unroll
    for (int s = 0; s < NST - 1; s++) issue(s);
    load_te(NST - 1);
    // query fragments (rows g: high part, g + 8: remainder) in log2 units,
    // loaded while the first tiles are in flight
    uint32_t qa[HD / 16][4];
    {
        const float *qh = q + ((size_t)kvh * G + g) * HD;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
            if (g < G) {
                const float2 u = *reinterpret_cast<const float2 *>(qh + 16 * kk + 2 * t4);
                const float2 w = *reinterpret_cast<const float2 *>(qh + 16 * kk + 8 + 2 * t4);
                x0 = u.x * qscale;
                x1 = u.y * qscale;
                x2 = w.x * qscale;
                x3 = w.y * qscale;
            }
            split2(x0, x1, qa[kk][0], qa[kk][1]);
            split2(x2, x3, qa[kk][2], qa[kk][3]);
        }
    }

    for (int tile = 0; tile < n_tiles; tile++) {
        put_ro(tile + NST - 1);
        load_te(tile + NST);
        asm volatile("cp.async.wait_group %0;" ::"n"(NST - 2) : "memory");
        __syncthreads();
        issue(tile + NST - 1);
        const uint8_t *kt = stage + (size_t)(tile % NST) * 2 * MAT_B, *vt = kt + MAT_B;
        const int rb = 16 * warp;                               // this warp's rows in the tile
        const int pos0 = t_lo + tile * TC_ROWS + rb;
        // scores: two n-tiles of 8 positions
        // (even and odd k-steps in separate accumulators: four independent chains)
        float sc[2][4], sc2[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; nt++) {
            sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
            sc2[nt][0] = sc2[nt][1] = sc2[nt][2] = sc2[nt][3] = 0.f;
        }
        // B fragments of two k-steps per ldmatrix.x4: lane l addresses row
        // (l & 7) of the n-tile, 16-byte column (l >> 3) of the 64-byte pair
#pragma unroll
        for (int kq = 0; kq < HD / 32; kq++)
#pragma unroll
            for (int nt = 0; nt < 2; nt++) {
                uint32_t b[4];
                ldsm_x4(b, kt + (rb + 8 * nt + (lane & 7)) * ROW_B + 64 * kq + 16 * (lane >> 3));
                mma16816(sc[nt], qa[2 * kq], b[0], b[1]);
                mma16816(sc2[nt], qa[2 * kq + 1], b[2], b[3]);
            }
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int j = 0; j < 4; j++) sc[nt][j] += sc2[nt][j];
        // s[nt][j] for head g at position pos0 + 8 nt + 2 t4 + j
        float sv[2][2];
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const float v = sc[nt][j] + sc[nt][2 + j];
                sv[nt][j] = pos0 + 8 * nt + 2 * t4 + j < t_hi ? v : -INFINITY;
                mx = fmaxf(mx, sv[nt][j]);
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float alpha = m_new == -INFINITY ? 1.f : exp2f(m_run - m_new);
        float p[2][2];
        float psum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int j = 0; j < 2; j++) {
                p[nt][j] = m_new == -INFINITY ? 0.f : exp2f(sv[nt][j] - m_new);
                psum += p[nt][j];
            }
        l_run = l_run * alpha + psum;
        m_run = m_new;
        if (!__all_sync(0xffffffffu, alpha == 1.f)) {
#pragma unroll
            for (int j = 0; j < NT; j++) {
                o_acc[j][0] *= alpha;
                o_acc[j][1] *= alpha;
                o_acc[j][2] *= alpha;
                o_acc[j][3] *= alpha;
            }
        }
        uint32_t pa[4];
        split2(p[0][0], p[0][1], pa[0], pa[1]);
        split2(p[1][0], p[1][1], pa[2], pa[3]);
        // P . V: V rows rb..rb+15 of the tile, two n-tiles per ldmatrix
        const uint8_t *vr = vt + (rb + (lane & 15)) * ROW_B + 16 * (lane >> 4);
#pragma unroll
        for (int j = 0; j < NT; j += 2) {
            uint32_t b[4];
            ldsm_x4_t(b, vr + 16 * j);
            mma16816(o_acc[j], pa, b[0], b[1]);
            mma16816(o_acc[j + 1], pa, b[2], b[3]);
        }
    }
    cp_wait0();
    __syncthreads();
    // merge the four warps: per head g, weights 2^(m_w - M)
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    float *wo = reinterpret_cast<float *>(stage);              // [4][8][HD]
    float *wm = wo + 4 * 8 * HD, *wl = wm + 32;                // [4][8]
    if (t4 == 0) {
        wm[warp * 8 + g] = m_run;
        wl[warp * 8 + g] = l_run;
    }
#pragma unroll
    for (int j = 0; j < NT; j++) {
        float *d = wo + (warp * 8 + g) * HD + 8 * j + 2 * t4;
        d[0] = o_acc[j][0] + o_acc[j][2];
        d[1] = o_acc[j][1] + o_acc[j][3];
    }
    __syncthreads();
    const bool bad = bad_s != 0;
    for (int idx = tid; idx < G * HD; idx += 128) {
        const int h = idx / HD, d = idx - h * HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; w++) M = fmaxf(M, wm[w * 8 + h]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const float mw = wm[w * 8 + h];
            const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
            L = __fmaf_rn(wl[w * 8 + h], f, L);
            O = __fmaf_rn(wo[(w * 8 + h) * HD + d], f, O);
        }
        const size_t hh = (size_t)(kvh * G + h) * n_span + sidx;
        po[hh * HD + d] = O;
        if (d == 0) {
            pm[hh] = bad ? NAN : M;
            pl[hh] = L;
        }
    }
}

// out[h][i] = sum_s o_s[i] 2^(m_s - M) / sum_s l_s 2^(m_s - M).
// grid (H, hd / 32), 256 threads: 32 columns x 8 span slices.
__global__ void __launch_bounds__(256) k_attn_merge(const float *__restrict__ pm, const float *__restrict__ pl,
                                                    const float *__restrict__ po, int n_span, int hd,
                                                    float *__restrict__ out) {
    __shared__ float red[2][8][33];
    __shared__ float mM;
    __shared__ int mbad;
    // launched early as a programmatic dependent of the split kernel: wait
    // until that grid has completed and its partials are visible
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int h = blockIdx.x, tid = threadIdx.x, c = tid & 31, ss = tid >> 5, col = 32 * blockIdx.y + c;
    const float *m = pm + (size_t)h * n_span, *l = pl + (size_t)h * n_span;
    float M = -INFINITY;
    int bad = 0;
    for (int s = tid; s < n_span; s += 256) {
        bad |= m[s] != m[s];
        M = fmaxf(M, m[s]);
    }
    for (int o = 16; o; o >>= 1) {
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if (c == 0) {
        red[0][ss][0] = M;
        red[1][ss][0] = (float)bad;
    }
    __syncthreads();
    if (tid == 0) {
        float mm = -INFINITY;
        int bb = 0;
        for (int w = 0; w < 8; w++) {
            mm = fmaxf(mm, red[0][w][0]);
            bb |= red[1][w][0] != 0.f;
        }
        mM = mm;
        mbad = bb;
    }
    __syncthreads();
    M = mM;
    float L = 0.f, O = 0.f;
#pragma unroll 4
    for (int s = ss; s < n_span; s += 8) {
        const float w = m[s] == -INFINITY ? 0.f : exp2f(m[s] - M);
        L = __fmaf_rn(l[s], w, L);
        O = __fmaf_rn(po[((size_t)h * n_span + s) * hd + col], w, O);
    }
    __syncthreads();
    red[0][ss][c] = L;
    red[1][ss][c] = O;
    __syncthreads();
    if (ss == 0) {
        for (int k = 1; k < 8; k++) {
            L += red[0][k][c];
            O += red[1][k][c];
        }
        out[(size_t)h * hd + col] = mbad ? NAN : __fdiv_rn(O, L);
    }
}

// ---- K/V append ------------------------------------------------------------
// Row `pos` of every KV head: k/v [KV][hd] f32 -> the pages (bf16: round to
// nearest even, NaN kept).
template <typename KT>
__global__ void k_kv_write(const float *__restrict__ k, const float *__restrict__ v, KT *__restrict__ kpool,
                           KT *__restrict__ vpool, int32_t e, int page, int pos, int KV, int hd) {
    const int n = KV * hd;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += gridDim.x * blockDim.x) {
        const int kvh = idx / hd, i = idx - kvh * hd;
        const size_t off = (((size_t)e * KV + kvh) * page + (size_t)(pos % page)) * hd + i;
        if constexpr (sizeof(KT) == 4) {
            kpool[off] = k[idx];
            vpool[off] = v[idx];
        } else {
            kpool[off] = __float2bfloat16_rn(k[idx]);
            vpool[off] = __float2bfloat16_rn(v[idx]);
        }
    }
}

int sm_count_cached() {
    static thread_local int dev = -1, n = 0;
    int d = 0;
    cudaGetDevice(&d);
    if (d != dev) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 148;
        }
        dev = d;
    }
    return n;
}

// bf16 pages with at most 8 query heads per KV head run on the tensor cores.
bool use_tc(int kv_dt, int grp) { return kv_dt == TLMG_DT_BF16 && grp <= 8; }

template <int HD>
constexpr int tc_stages() { return HD <= 128 ? 3 : 2; }

size_t tc_smem(int hd) {
    const int nst = hd <= 128 ? 3 : 2;
    const size_t st = (size_t)nst * 2 * TC_ROWS * (hd * 2 + 16);
    const size_t mg = (4 * 8 * (size_t)hd + 64) * 4;
    return std::max(st, mg);
}

SplitGeom split_geom(int T, int H, int KV, int hd, int kv_dt) {
    const int es = kv_dt == TLMG_DT_F32 ? 4 : 2;
    SplitGeom g{};
    g.tr = use_tc(kv_dt, H / KV) ? TC_ROWS : std::min(64, std::max(16, 16384 / (hd * es)));
    const int want = std::max(1, 2 * sm_count_cached() / KV);   // spans per KV head for two CTAs per SM
    int span = (T + want - 1) / want;
    span = std::max(g.tr, (span + g.tr - 1) / g.tr * g.tr);
    g.span = span;
    g.n_span = (T + span - 1) / span;
    return g;
}

size_t split_smem(const SplitGeom &g, int grp, int hd, int es) {
    const size_t head = ((size_t)(grp * hd + g.tr * (grp + 1) + 3 * MAX_GRP + 4) * 4 + 15) / 16 * 16;
    return head + 2 * 2 * (size_t)g.tr * (hd * es + 16);
}

template <typename F>
bool smem_opt_in(F fn, size_t bytes) {
    static thread_local std::vector<std::pair<const void *, size_t>> done;
    for (auto &d : done)
        if (d.first == (const void *)fn && d.second >= bytes) return true;
    if (cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
        cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    done.push_back({ (const void *)fn, bytes });
    return true;
}

// The merge kernel as a programmatic dependent launch: it is scheduled
// while the split kernel runs and waits in griddepcontrol.wait.
cudaError_t launch_merge(const float *pm, const float *pl, const float *po, int n_span, int H, int hd, float *out,
                         cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(H, hd / 32);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_attn_merge, pm, pl, po, n_span, hd, out);
}

int check_geom(const char *who, int kv_dt, int T, int H, int KV, int hd, int page, int n_pages) {
    if (kv_dt != TLMG_DT_F32 && kv_dt != TLMG_DT_BF16)
        return set_error(TLMG_EINVAL, "%s: KV dtype %d (f32 or bf16)", who, kv_dt);
    if (T <= 0 || H <= 0 || KV <= 0 || H % KV || H / KV > MAX_GRP)
        return set_error(TLMG_EINVAL, "%s: T %d, %d heads over %d KV heads (at most %d per KV head)", who, T, H, KV,
                         MAX_GRP);
    if (hd != 64 && hd != 128 && hd != 256) return set_error(TLMG_EINVAL, "%s: head_dim %d (64, 128 or 256)", who, hd);
    if (page <= 0 || page > (1 << 16) || (page & (page - 1)) || n_pages <= 0)
        return set_error(TLMG_EINVAL, "%s: page %d (a power of two up to 65536), %d pages", who, page, n_pages);
    return TLMG_OK;
}

}  // namespace

size_t attention_work_bytes(int mode, int kv_dt, int T, int H, int KV, int hd) {
    if (T <= 0 || H <= 0 || KV <= 0) return 0;
    if (mode == TLMG_ATTN_EXACT) return (size_t)H * T * 4;
    const SplitGeom g = split_geom(T, H, KV, hd, kv_dt);
    return (size_t)H * g.n_span * (2 + (size_t)hd) * 4;
}

// T = the launch's geometry (grids, spans, shared memory); with dT the
// kernels read the actual position count (<= T) from device memory.
template <typename KT>
static int launch_attention(int mode, const float *q, const KT *kp, const KT *vp, const int32_t *table, int n_pages,
                            int page, int T, const int32_t *dT, int H, int KV, int hd, float *work, float *out,
                            cudaStream_t st, int kv_dt) {
    const int grp = H / KV;
    if (mode == TLMG_ATTN_EXACT) {
        const float scale = 1.0f / sqrtf((float)hd);
        const size_t s1 = (size_t)grp * hd * 4 + (size_t)XS_ROWS * (hd * sizeof(KT) + 16);
        if (!smem_opt_in(k_attn_scores<KT>, s1)) return set_error(TLMG_EIO, "attention: shared memory opt-in failed");
        dim3 g1((T + XS_ROWS - 1) / XS_ROWS, KV);
        launch_k(k_attn_scores<KT>, g1, XS_ROWS, s1, st, q, kp, table, n_pages, page, T, dT, H, KV, hd, scale, work);
        bool ok = true;
#define TLMG_XO(HDV)                                                                                       \
    if (hd == HDV) {                                                                                       \
        constexpr int nst = xo_stages<KT, HDV>();                                                          \
        const size_t s2 = (size_t)nst * XO_ROWS * HDV * sizeof(KT) + (T <= PSM_MAX ? (size_t)T * 4 : 0);   \
        auto fn = k_attn_out_exact<KT, HDV, nst>;                                                          \
        ok = smem_opt_in(fn, s2);                                                                          \
        if (ok) launch_k(fn, H, HDV, s2, st, vp, table, n_pages, page, T, dT, T <= PSM_MAX ? T : 0, H, KV, work,   \
                         out);                                                                             \
    }
        TLMG_XO(64)
        TLMG_XO(128)
        TLMG_XO(256)
#undef TLMG_XO
        if (!ok) return set_error(TLMG_EIO, "attention: shared memory opt-in failed");
        count_launch(2);
    } else {
        const SplitGeom g = split_geom(T, H, KV, hd, kv_dt);
        float *pm = work, *pl = pm + (size_t)H * g.n_span, *po = pl + (size_t)H * g.n_span;
        const float qscale = (float)(1.4426950408889634 / std::sqrt((double)hd));
        dim3 g1(g.n_span, KV);
        if constexpr (sizeof(KT) == 2) {
            if (use_tc(kv_dt, grp)) {
                const size_t sm = tc_smem(hd);
                int lp = 0;
                while ((1 << lp) < page) lp++;
                bool ok = true;
#define TLMG_TC(HDV)                                                                                            \
    if (hd == HDV) {                                                                                            \
        auto fn = k_attn_split_tc<HDV, tc_stages<HDV>()>;                                                       \
        ok = smem_opt_in(fn, sm);                                                                               \
        if (ok) launch_k(fn, g1, 128, sm, st, q, kp, vp, table, n_pages, page, lp, T, dT, H, KV, g.span, g.n_span,    \
                         qscale, pm, pl, po);                                                                   \
    }
                TLMG_TC(64)
                TLMG_TC(128)
                TLMG_TC(256)
#undef TLMG_TC
                if (!ok) return set_error(TLMG_EIO, "attention: shared memory opt-in failed");
                cudaError_t e = launch_merge(pm, pl, po, g.n_span, H, hd, out, st);
                count_launch(2);
                if (e == cudaSuccess) e = cudaGetLastError();
                return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "attention launch");
            }
        }
        const size_t sm = split_smem(g, grp, hd, (int)sizeof(KT));
        if (!smem_opt_in(k_attn_split<KT>, sm)) return set_error(TLMG_EIO, "attention: shared memory opt-in failed");
        launch_k(k_attn_split<KT>, g1, SPLIT_THREADS, sm, st, q, kp, vp, table, n_pages, page, T, dT, H, KV, hd, g.tr, g.span,
                                                        g.n_span, qscale, pm, pl, po);
        if (launch_merge(pm, pl, po, g.n_span, H, hd, out, st) != cudaSuccess)
            return cuda_fail(cudaGetLastError(), "attention merge launch");
        count_launch(2);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "attention launch");
}

}  // namespace tlmg

using namespace tlmg;

extern "C" size_t tlmg_attention_work_bytes(int mode, int kv_dt, int T, int H, int KV, int hd) {
    return attention_work_bytes(mode, kv_dt, T, H, KV, hd);
}

namespace tlmg {

int decode_attention_impl(int mode, int kv_dt, const float *q, const void *k_pages, const void *v_pages, int n_pages,
                          const int32_t *page_table, int page_size, int T, const int32_t *dT, int H, int KV, int hd,
                          void *work, size_t work_bytes, float *out, cudaStream_t st) {
    int rc = check_geom("decode_attention", kv_dt, T, H, KV, hd, page_size, n_pages);
    if (rc) return rc;
    if (mode != TLMG_ATTN_EXACT && mode != TLMG_ATTN_SPLIT)
        return set_error(TLMG_EINVAL, "decode_attention: mode %d", mode);
    if (!q || !k_pages || !v_pages || !page_table || !work || !out)
        return set_error(TLMG_EINVAL, "decode_attention: null pointer");
    if (((uintptr_t)k_pages | (uintptr_t)v_pages | (uintptr_t)q | (uintptr_t)work) & 15u)
        return set_error(TLMG_EINVAL, "decode_attention: q, pages and work must be 16-byte aligned");
    const size_t need = attention_work_bytes(mode, kv_dt, T, H, KV, hd);
    if (work_bytes < need)
        return set_error(TLMG_ERANGE, "decode_attention: work holds %zu bytes, needs %zu", work_bytes, need);
    float *w = static_cast<float *>(work);
    if (kv_dt == TLMG_DT_F32)
        return launch_attention<float>(mode, q, (const float *)k_pages, (const float *)v_pages, page_table, n_pages,
                                       page_size, T, dT, H, KV, hd, w, out, st, kv_dt);
    return launch_attention<__nv_bfloat16>(mode, q, (const __nv_bfloat16 *)k_pages, (const __nv_bfloat16 *)v_pages,
                                           page_table, n_pages, page_size, T, dT, H, KV, hd, w, out, st, kv_dt);
}

}  // namespace tlmg

extern "C" int tlmg_decode_attention(int mode, int kv_dt, const float *q, const void *k_pages, const void *v_pages,
                                     int n_pages, const int32_t *page_table, int page_size, int T, int H, int KV,
                                     int hd, void *work, size_t work_bytes, float *out, void *stream) {
    return decode_attention_impl(mode, kv_dt, q, k_pages, v_pages, n_pages, page_table, page_size, T, nullptr, H, KV,
                                 hd, work, work_bytes, out, pick_stream(stream));
}

extern "C" int tlmg_kv_write(int kv_dt, const float *k, const float *v, void *k_pages, void *v_pages, int n_pages,
                             int32_t page_id, int page_size, int pos, int KV, int hd, void *stream) {
    int rc = check_geom("kv_write", kv_dt, 1, KV, KV, hd, page_size, n_pages);
    if (rc) return rc;
    if (page_id < 0 || page_id >= n_pages || pos < 0)
        return set_error(TLMG_ERANGE, "kv_write: page %d of %d, position %d", page_id, n_pages, pos);
    if (!k || !v || !k_pages || !v_pages) return set_error(TLMG_EINVAL, "kv_write: null pointer");
    cudaStream_t st = pick_stream(stream);
    const int n = KV * hd, blocks = (n + 255) / 256;
    if (kv_dt == TLMG_DT_F32)
        k_kv_write<float><<<blocks, 256, 0, st>>>(k, v, (float *)k_pages, (float *)v_pages, page_id, page_size, pos,
                                                  KV, hd);
    else
        k_kv_write<__nv_bfloat16><<<blocks, 256, 0, st>>>(k, v, (__nv_bfloat16 *)k_pages, (__nv_bfloat16 *)v_pages,
                                                          page_id, page_size, pos, KV, hd);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "kv_write launch");
}
