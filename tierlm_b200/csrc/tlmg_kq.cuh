// tlmg_kq.cuh - K-quant block dot products of the expert kernels (sm_100a):
// exact int32 partials of Q4_K / Q5_K / Q6_K weight blocks against Q8_K
// activation blocks in the swizzled layout, the reference's per-block fmaf
// chain step, and the warp-level Q8_K quantiser writing that layout.
// Pointers are generic: the blocks may sit in shared or global memory.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#include "tlmg_dev.cuh"

namespace tlmg {

// ---------------------------------------------------------------------------
// 16-byte loads (generic: shared or global memory)
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
// 4 / 16 bytes at a 2-byte aligned shared address
__device__ __forceinline__ uint32_t lds32_a2(const uint8_t *p) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    return (a & 2u) ? __byte_perm(w[0], w[1], 0x5432) : w[0];
}
__device__ __forceinline__ uint4 lds128_a2(const uint8_t *p) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3];
    if (!(a & 2u)) return make_uint4(w0, w1, w2, w3);
    uint32_t w4 = w[4];
    return make_uint4(__byte_perm(w0, w1, 0x5432), __byte_perm(w1, w2, 0x5432), __byte_perm(w2, w3, 0x5432),
                      __byte_perm(w3, w4, 0x5432));
}
__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(int8_t)((w >> (8 * i)) & 255u); }
// f16 bits -> f32 with the hardware conversion (exact for every finite and
// infinite value; a NaN stays a NaN).
__device__ __forceinline__ float h2f(uint32_t bits) {
    return __half2float(__ushort_as_half((unsigned short)bits));
}

// ---------------------------------------------------------------------------
// Q8_K activation blocks in shared memory, bank-swizzled: the 16-byte
// piece p (codes 16p .. 16p+15) of block beta of an NB-block vector lives at
// codes + (p * NB + beta) * 16, so lanes that read the same piece of
// consecutive blocks hit consecutive banks. bsums[16] (32 bytes, 16-aligned)
// and d per block separately.
__device__ __forceinline__ const uint8_t *swz(const uint8_t *codes, int NB, int beta, int p) {
    return codes + ((size_t)p * NB + beta) * 16;
}
struct XBlk {
    const uint8_t *codes;
    int NB, beta;
    const int16_t *bs;
    float d;
};
__device__ __forceinline__ uint4 xpiece(const XBlk &x, int p) { return lds128(swz(x.codes, x.NB, x.beta, p)); }
__device__ __forceinline__ uint32_t wsel(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
// unsigned bytes of a times signed bytes of b, plus c
__device__ __forceinline__ int dp4us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// the sum of the two signed 16-bit halves of w
__device__ __forceinline__ int hsum16(uint32_t w) { return __dp2a_lo((int)w, 0x0101, 0); }
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// Exact int32 partials (is = sum_j scale_j * dot_j, ms = sum_j min_j * bsum_j)
// and the float factors (dA = d_w * d_a, dM = dmin_w * d_a) of NM weight
// blocks of one K-quant dtype against one activation block (the reference's
// per-block integer sums, tlm_quant.c:253-296 for Q4_K / Q5_K, :392-420 for
// Q6_K). Each activation piece is loaded once for all NM weight blocks.
struct BlockSum {
    int is, ms;
    float dA, dM;
};

// Q4_K (144 B: d, dmin, scales[12], qs[128]) / Q5_K (176 B: + qh[32] before
// qs). Blocks are 16-byte aligned in the stage. Sub-block j's 6-bit scale /
// min are bytes of sc03 / mn03 (j < 4) and sc47 / mn47 (j >= 4) (reference
// tlm_quant.c:253-261). Quarter q holds sub-blocks 2q (low nibbles) and
// 2q+1 (high nibbles) of qs[32q ..].
template <int DT, int NM>
__device__ __forceinline__ void kblock_dot_k45(const uint8_t *const (&w)[NM], const XBlk &x, BlockSum (&o)[NM]) {
    constexpr int QOFF = DT == DT_Q4_K ? 16 : 48;
    uint32_t sc03[NM], sc47[NM];
    {
        const uint4 b0 = lds128(reinterpret_cast<const uint8_t *>(x.bs)),
                    b1 = lds128(reinterpret_cast<const uint8_t *>(x.bs) + 16);
        const int bs0 = hsum16(b0.x), bs1 = hsum16(b0.y), bs2 = hsum16(b0.z), bs3 = hsum16(b0.w);
        const int bs4 = hsum16(b1.x), bs5 = hsum16(b1.y), bs6 = hsum16(b1.z), bs7 = hsum16(b1.w);
#pragma unroll
        for (int m = 0; m < NM; m++) {
            const uint4 h = lds128(w[m]);
            sc03[m] = h.y & 0x3F3F3F3Fu;
            sc47[m] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
            const uint32_t mn03 = h.z & 0x3F3F3F3Fu;
            const uint32_t mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
            o[m].dA = __fmul_rn(h2f(h.x & 0xFFFFu), x.d);
            o[m].dM = __fmul_rn(h2f(h.x >> 16), x.d);
            o[m].is = 0;
            o[m].ms = (int)byte_of(mn03, 0) * bs0 + (int)byte_of(mn03, 1) * bs1 + (int)byte_of(mn03, 2) * bs2 +
                      (int)byte_of(mn03, 3) * bs3 + (int)byte_of(mn47, 0) * bs4 + (int)byte_of(mn47, 1) * bs5 +
                      (int)byte_of(mn47, 2) * bs6 + (int)byte_of(mn47, 3) * bs7;
        }
    }
#pragma unroll 1
    for (int q = 0; q < 4; q++) {
        const uint4 xl0 = xpiece(x, 4 * q), xl1 = xpiece(x, 4 * q + 1);       // sub-block 2q
        const uint4 xh0 = xpiece(x, 4 * q + 2), xh1 = xpiece(x, 4 * q + 3);   // sub-block 2q+1
#pragma unroll
        for (int m = 0; m < NM; m++) {
            const uint4 v0 = lds128(w[m] + QOFF + 32 * q), v1 = lds128(w[m] + QOFF + 32 * q + 16);
            uint4 g0 = make_uint4(0u, 0u, 0u, 0u), g1 = g0;
            if constexpr (DT == DT_Q5_K) {
                g0 = lds128(w[m] + 16);
                g1 = lds128(w[m] + 32);
            }
            int lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t qw = wsel(i < 4 ? v0 : v1, i & 3);
                const uint32_t xlw = wsel(i < 4 ? xl0 : xl1, i & 3), xhw = wsel(i < 4 ? xh0 : xh1, i & 3);
                if constexpr (DT == DT_Q4_K) {
                    lo = dp4(qw & 0x0F0F0F0Fu, xlw, lo);
                    hi = dp4us(qw & 0xF0F0F0F0u, xhw, hi);   // 16 x the high-nibble dot
                } else {
                    const uint32_t hw = wsel(i < 4 ? g0 : g1, i & 3);
                    const uint32_t l5 = (qw & 0x0F0F0F0Fu) | (((hw >> (2 * q)) & 0x01010101u) << 4);
                    const uint32_t h5 = ((qw >> 4) & 0x0F0F0F0Fu) | (((hw >> (2 * q + 1)) & 0x01010101u) << 4);
                    lo = dp4(l5, xlw, lo);
                    hi = dp4(h5, xhw, hi);
                }
            }
            if constexpr (DT == DT_Q4_K) hi >>= 4;   // exact: the sum is a multiple of 16
            const uint32_t sw = q < 2 ? sc03[m] : sc47[m];
            o[m].is += (int)((sw >> (16 * (q & 1))) & 0xFFu) * lo + (int)((sw >> (16 * (q & 1) + 8)) & 0xFFu) * hi;
        }
    }
}

// Q6_K (210 B: ql[128], qh[64], int8 scales[16], f16 d) at a 2-byte aligned
// stage address: the block's words are read 4-byte aligned and realigned
// with funnel shifts. Half h, element l + 32m (l = 0..31, m = 0..3):
// q = ((ql[64h + l + 32(m&1)] >> 4(m>>1)) & 15) | (((qh[32h + l] >> 2m) & 3) << 4),
// minus 32 (applied through the group's activation sum), in group
// 8h + 2m + l/16 with scale scales[8h + 2m + l/16] (reference
// tlm_quant.c:392-420).
template <int NM>
__device__ __forceinline__ void kblock_dot_q6(const uint8_t *const (&w)[NM], const XBlk &x, BlockSum (&o)[NM]) {
    int bsg[16];
    {
        const uint4 b0 = lds128(reinterpret_cast<const uint8_t *>(x.bs)),
                    b1 = lds128(reinterpret_cast<const uint8_t *>(x.bs) + 16);
        const uint32_t bw[8] = { b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w };
#pragma unroll
        for (int i = 0; i < 8; i++) {
            bsg[2 * i] = (int)(int16_t)(bw[i] & 0xFFFFu);
            bsg[2 * i + 1] = (int)(int16_t)(bw[i] >> 16);
        }
    }
#pragma unroll
    for (int m = 0; m < NM; m++) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(w[m]);
        const uint32_t *wp = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
        const uint32_t sh = (uint32_t)(a & 3u) * 8u;   // 0 or 16
        int is = 0;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            int dot[8];   // group 8h + 2mm + p at index 2mm + p
#pragma unroll
            for (int i = 0; i < 8; i++) dot[i] = 0;
#pragma unroll
            for (int p = 0; p < 2; p++) {   // l = 16p .. 16p+15
                uint4 xv[4];
#pragma unroll
                for (int mm = 0; mm < 4; mm++) xv[mm] = xpiece(x, 8 * h + 2 * mm + p);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int lw = 4 * p + i;
                    const int ja = 16 * h + lw, jb = 16 * h + 8 + lw, jc = 32 + 8 * h + lw;
                    const uint32_t A = __funnelshift_r(wp[ja], wp[ja + 1], sh);
                    const uint32_t B = __funnelshift_r(wp[jb], wp[jb + 1], sh);
                    const uint32_t Cq = __funnelshift_r(wp[jc], wp[jc + 1], sh);
                    const uint32_t u0 = (A & 0x0F0F0F0Fu) | ((Cq << 4) & 0x30303030u);
                    const uint32_t u1 = (B & 0x0F0F0F0Fu) | ((Cq << 2) & 0x30303030u);
                    const uint32_t u2 = ((A >> 4) & 0x0F0F0F0Fu) | (Cq & 0x30303030u);
                    const uint32_t u3 = ((B >> 4) & 0x0F0F0F0Fu) | ((Cq >> 2) & 0x30303030u);
                    dot[0 + p] = dp4(u0, wsel(xv[0], i), dot[0 + p]);
                    dot[2 + p] = dp4(u1, wsel(xv[1], i), dot[2 + p]);
                    dot[4 + p] = dp4(u2, wsel(xv[2], i), dot[4 + p]);
                    dot[6 + p] = dp4(u3, wsel(xv[3], i), dot[6 + p]);
                }
            }
            // scales 8h .. 8h+7 (bytes 192 + 8h ..)
            const uint32_t s0 = __funnelshift_r(wp[48 + 2 * h], wp[49 + 2 * h], sh);
            const uint32_t s1 = __funnelshift_r(wp[49 + 2 * h], wp[50 + 2 * h], sh);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int sc = (int)(int8_t)byte_of(i < 4 ? s0 : s1, i & 3);
                is += sc * (dot[i] - 32 * bsg[8 * h + i]);
            }
        }
        o[m].is = is;
        o[m].ms = 0;
        o[m].dA = __fmul_rn(h2f(__funnelshift_r(wp[52], wp[53], sh) & 0xFFFFu), x.d);
        o[m].dM = 0.0f;
    }
}

// The exact partials of half `half` (elements 128 half .. 128 half + 127)
// of one weight block of dtype DT against activation block x: the block's
// is / ms are the sums of its two halves' (integer addition is exact), its
// dA / dM are the same for both halves.
template <int DT>
__device__ __forceinline__ void kblock_half(const uint8_t *w, const XBlk &x, int half, BlockSum &o) {
    const uint4 bv = lds128(reinterpret_cast<const uint8_t *>(x.bs) + 16 * half);   // bsums 8 half .. 8 half + 7
    const uint32_t bw[4] = { bv.x, bv.y, bv.z, bv.w };
    if constexpr (DT == DT_Q6_K) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(w);
        const uint32_t *wp = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
        const uint32_t sh = (uint32_t)(a & 3u) * 8u;   // 0 or 16
        const int h = half;
        int dot[8];   // group 8h + 2mm + p at index 2mm + p
#pragma unroll
        for (int i = 0; i < 8; i++) dot[i] = 0;
#pragma unroll
        for (int p = 0; p < 2; p++) {
            uint4 xv[4];
#pragma unroll
            for (int mm = 0; mm < 4; mm++) xv[mm] = xpiece(x, 8 * h + 2 * mm + p);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int lw = 4 * p + i;
                const int ja = 16 * h + lw, jb = 16 * h + 8 + lw, jc = 32 + 8 * h + lw;
                const uint32_t A = __funnelshift_r(wp[ja], wp[ja + 1], sh);
                const uint32_t B = __funnelshift_r(wp[jb], wp[jb + 1], sh);
                const uint32_t Cq = __funnelshift_r(wp[jc], wp[jc + 1], sh);
                const uint32_t u0 = (A & 0x0F0F0F0Fu) | ((Cq << 4) & 0x30303030u);
                const uint32_t u1 = (B & 0x0F0F0F0Fu) | ((Cq << 2) & 0x30303030u);
                const uint32_t u2 = ((A >> 4) & 0x0F0F0F0Fu) | (Cq & 0x30303030u);
                const uint32_t u3 = ((B >> 4) & 0x0F0F0F0Fu) | ((Cq >> 2) & 0x30303030u);
                dot[0 + p] = dp4(u0, wsel(xv[0], i), dot[0 + p]);
                dot[2 + p] = dp4(u1, wsel(xv[1], i), dot[2 + p]);
                dot[4 + p] = dp4(u2, wsel(xv[2], i), dot[4 + p]);
                dot[6 + p] = dp4(u3, wsel(xv[3], i), dot[6 + p]);
            }
        }
        const uint32_t s0 = __funnelshift_r(wp[48 + 2 * h], wp[49 + 2 * h], sh);
        const uint32_t s1 = __funnelshift_r(wp[49 + 2 * h], wp[50 + 2 * h], sh);
        int is = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int sc = (int)(int8_t)byte_of(i < 4 ? s0 : s1, i & 3);
            const int bs = (int)(int16_t)((bw[i >> 1] >> (16 * (i & 1))) & 0xFFFFu);
            is += sc * (dot[i] - 32 * bs);
        }
        o.is = is;
        o.ms = 0;
        o.dA = __fmul_rn(h2f(__funnelshift_r(wp[52], wp[53], sh) & 0xFFFFu), x.d);
        o.dM = 0.0f;
    } else {
        constexpr int QOFF = DT == DT_Q4_K ? 16 : 48;
        const uint4 hd = lds128(w);
        const uint32_t sc03 = hd.y & 0x3F3F3F3Fu, mn03 = hd.z & 0x3F3F3F3Fu;
        const uint32_t sc47 = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
        const uint32_t mn47 = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
        const uint32_t sw = half ? sc47 : sc03, mw = half ? mn47 : mn03;   // sub-blocks 4 half .. 4 half + 3
        o.dA = __fmul_rn(h2f(hd.x & 0xFFFFu), x.d);
        o.dM = __fmul_rn(h2f(hd.x >> 16), x.d);
        o.ms = (int)byte_of(mw, 0) * hsum16(bw[0]) + (int)byte_of(mw, 1) * hsum16(bw[1]) +
               (int)byte_of(mw, 2) * hsum16(bw[2]) + (int)byte_of(mw, 3) * hsum16(bw[3]);
        uint4 g0 = make_uint4(0u, 0u, 0u, 0u), g1 = g0;
        if constexpr (DT == DT_Q5_K) {
            g0 = lds128(w + 16);
            g1 = lds128(w + 32);
        }
        int is = 0;
#pragma unroll
        for (int qq = 0; qq < 2; qq++) {
            const int q = 2 * half + qq;
            const uint4 xl0 = xpiece(x, 4 * q), xl1 = xpiece(x, 4 * q + 1);
            const uint4 xh0 = xpiece(x, 4 * q + 2), xh1 = xpiece(x, 4 * q + 3);
            const uint4 v0 = lds128(w + QOFF + 32 * q), v1 = lds128(w + QOFF + 32 * q + 16);
            int lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t qw = wsel(i < 4 ? v0 : v1, i & 3);
                const uint32_t xlw = wsel(i < 4 ? xl0 : xl1, i & 3), xhw = wsel(i < 4 ? xh0 : xh1, i & 3);
                if constexpr (DT == DT_Q4_K) {
                    lo = dp4(qw & 0x0F0F0F0Fu, xlw, lo);
                    hi = dp4us(qw & 0xF0F0F0F0u, xhw, hi);
                } else {
                    const uint32_t hw = wsel(i < 4 ? g0 : g1, i & 3);
                    const uint32_t l5 = (qw & 0x0F0F0F0Fu) | (((hw >> (2 * q)) & 0x01010101u) << 4);
                    const uint32_t h5 = ((qw >> 4) & 0x0F0F0F0Fu) | (((hw >> (2 * q + 1)) & 0x01010101u) << 4);
                    lo = dp4(l5, xlw, lo);
                    hi = dp4(h5, xhw, hi);
                }
            }
            if constexpr (DT == DT_Q4_K) hi >>= 4;
            is += (int)byte_of(sw, 2 * qq) * lo + (int)byte_of(sw, 2 * qq + 1) * hi;
        }
        o.is = is;
    }
}

template <int DT, int NM>
__device__ __forceinline__ void kblock_dot(const uint8_t *const (&w)[NM], const XBlk &x, BlockSum (&o)[NM]) {
    if constexpr (DT == DT_Q6_K) kblock_dot_q6<NM>(w, x, o);
    else kblock_dot_k45<DT, NM>(w, x, o);
}

// One block's step of the reference's fmaf chain.
template <int DT>
__device__ __forceinline__ float chain(float acc, float dA, int is, float dM, int ms) {
    acc = __fmaf_rn(dA, (float)is, acc);
    if constexpr (DT == DT_Q4_K || DT == DT_Q5_K) acc = __fmaf_rn(-dM, (float)ms, acc);
    return acc;
}
// The chain step of the block held by lane `src` (all lanes take part).
template <int DT>
__device__ __forceinline__ float chain_from(float acc, const BlockSum &v, int src) {
    const int is = __shfl_sync(0xFFFFFFFFu, v.is, src);
    const float dA = __shfl_sync(0xFFFFFFFFu, v.dA, src);
    int ms = 0;
    float dM = 0.0f;
    if constexpr (DT == DT_Q4_K || DT == DT_Q5_K) {
        ms = __shfl_sync(0xFFFFFFFFu, v.ms, src);
        dM = __shfl_sync(0xFFFFFFFFu, v.dM, src);
    }
    return chain<DT>(acc, dA, is, dM, ms);
}

// A full warp quantises one Q8_K block (block beta of an NB-block vector)
// into the swizzled shared layout from this lane's 8 inputs (elements
// 8*lane ..): codes, bsums[16] and d of the block.
__device__ __forceinline__ void warp_quant_swz(const float4 &a, const float4 &b, uint8_t *codes, int NB, int beta,
                                               int16_t *bs, float *d, int lane) {
    float v[8];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    int q[8];
    float dd = act_block_codes<8, 32>(v, q);
    uint32_t w0 = (q[0] & 255) | ((q[1] & 255) << 8) | ((q[2] & 255) << 16) | ((uint32_t)(q[3] & 255) << 24);
    uint32_t w1 = (q[4] & 255) | ((q[5] & 255) << 8) | ((q[6] & 255) << 16) | ((uint32_t)(q[7] & 255) << 24);
    *reinterpret_cast<uint2 *>(codes + ((size_t)(lane >> 1) * NB + beta) * 16 + 8 * (lane & 1)) = make_uint2(w0, w1);
    int s = q[0] + q[1] + q[2] + q[3] + q[4] + q[5] + q[6] + q[7];
    s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
    if ((lane & 1) == 0) bs[lane >> 1] = (int16_t)s;
    if (lane == 0) *d = dd;
}

// ---------------------------------------------------------------------------
// Quantised activation vectors (the x of a token, the h of one expert of a
// token): nb Q8_K blocks as codes[256 nb] (swizzled), bsums[16 nb], d[nb],
// each part 16-byte aligned. The layout is the same in global and in shared
// memory, so one bulk copy moves a vector.
__host__ __device__ inline uint32_t up16(uint32_t v) { return (v + 15u) & ~15u; }
__host__ __device__ inline uint32_t qv_bsums(int nb) { return 256u * (uint32_t)nb; }
__host__ __device__ inline uint32_t qv_d(int nb) { return qv_bsums(nb) + 32u * (uint32_t)nb; }
__host__ __device__ inline uint32_t qv_bytes(int nb) { return qv_d(nb) + up16(4u * (uint32_t)nb); }
struct QVec {
    uint8_t *codes;
    int16_t *bs;
    float *d;
    int nb;
};
__device__ __forceinline__ QVec qvec(uint8_t *base, int nb) {
    return QVec{ base, reinterpret_cast<int16_t *>(base + qv_bsums(nb)), reinterpret_cast<float *>(base + qv_d(nb)),
                 nb };
}
// A full warp quantises block b of a vector (this lane's 8 inputs, elements
// 8*lane ..) into q.
__device__ __forceinline__ void quant_block(const float4 &v0, const float4 &v1, const QVec &q, int b, int lane) {
    warp_quant_swz(v0, v1, q.codes, q.nb, b, q.bs + 16 * b, q.d + b, lane);
}

}  // namespace tlmg
