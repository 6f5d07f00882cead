// tlmg_dev.cuh - device building blocks of the sm_100a tier.
//
// Numerics contract (reference src/lib/tlm_quant.h:113-128): integer formats
// form an exact int32 per block; the float side is one explicit fmaf per
// block (two for Q4_K/Q5_K) in ascending block order. Everything here uses
// explicit IEEE intrinsics (__fmul_rn, __fadd_rn, __fmaf_rn, __fdiv_rn) and
// the library is built with -fmad=false, the CUDA analogue of the reference's
// -ffp-contract=off.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace tlmg {

enum : int {
    DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2, DT_Q8_0 = 8, DT_Q4_K = 12, DT_Q5_K = 13,
    DT_Q6_K = 14, DT_Q8_K = 15, DT_MXFP4 = 39
};

__host__ __device__ constexpr int dt_block(int dt) {
    switch (dt) {
    case DT_F32: case DT_F16: case DT_BF16: return 1;
    case DT_Q8_0: case DT_MXFP4: return 32;
    case DT_Q4_K: case DT_Q5_K: case DT_Q6_K: case DT_Q8_K: return 256;
    default: return 0;
    }
}

__host__ __device__ constexpr int dt_block_bytes(int dt) {
    switch (dt) {
    case DT_F32: return 4;
    case DT_F16: case DT_BF16: return 2;
    case DT_Q8_0: return 34;
    case DT_Q4_K: return 144;
    case DT_Q5_K: return 176;
    case DT_Q6_K: return 210;
    case DT_Q8_K: return 292;
    case DT_MXFP4: return 17;
    default: return 0;
    }
}

// Activation kind a weight dtype consumes (reference tlm_quant.c:691-697).
__host__ __device__ constexpr int act_kind_for(int wdt) {
    switch (wdt) {
    case DT_Q4_K: case DT_Q5_K: case DT_Q6_K: case DT_Q8_K: return DT_Q8_K;
    case DT_Q8_0: case DT_MXFP4: return DT_Q8_0;
    default: return DT_F32;
    }
}
__host__ __device__ constexpr int act_block_bytes(int kind) { return kind == DT_Q8_K ? 292 : 36; }

// ---------------------------------------------------------------------------
// scalar conversions, built from integer fields so they are exact in every
// mode (reference tlm_quant.c:124-197)
__device__ __forceinline__ float f16_to_f32(uint32_t h) {
    uint32_t s = (h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 31u) return __uint_as_float(s | 0x7F800000u | (m << 13) | (m ? 0x00400000u : 0u));
    if (e == 0u) return __uint_as_float(__float_as_uint(__fmul_rn(__uint2float_rn(m), 0x1p-24f)) | s);
    return __uint_as_float(s | ((e + 112u) << 23) | (m << 13));
}
__device__ __forceinline__ float bf16_to_f32(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ float e8m0_half(uint32_t e) {
    uint32_t b;
    if (e == 255u) b = 0x7FC00000u;
    else if (e >= 2u) b = (e - 1u) << 23;
    else b = e ? 0x00400000u : 0x00200000u;
    return __uint_as_float(b);
}

// Correctly rounded expf. Method: Cody-Waite reduction x = k ln2 + r with a
// two-part ln2, the degree-13 Taylor polynomial of exp(r) on |r| <= ln2/2
// evaluated in double with fma (truncation < 2^-57), scaling by 2^k and one
// rounding to float. Equal to (float)expl(x) for every one of the 2^32
// inputs (checked exhaustively on the host with the twin in the oracle).
__device__ __forceinline__ float cr_expf(float xf) {
    if (xf != xf) return __fadd_rn(xf, xf);
    if (xf > 88.72283935546875f) return __uint_as_float(0x7F800000u);
    if (xf < -103.97283935546875f) return 0.0f;
    double x = (double)xf;
    double k = rint(__dmul_rn(x, 0x1.71547652b82fep+0));
    double r = __fma_rn(-k, 0x1.62e42feep-1, x);
    r = __fma_rn(-k, 0x1.a39ef35793c76p-33, r);
    double p = 0x1.6124613a86d09p-33;
    p = __fma_rn(p, r, 0x1.1eed8eff8d898p-29);
    p = __fma_rn(p, r, 0x1.ae64567f544e4p-26);
    p = __fma_rn(p, r, 0x1.27e4fb7789f5cp-22);
    p = __fma_rn(p, r, 0x1.71de3a556c734p-19);
    p = __fma_rn(p, r, 0x1.a01a01a01a01ap-16);
    p = __fma_rn(p, r, 0x1.a01a01a01a01ap-13);
    p = __fma_rn(p, r, 0x1.6c16c16c16c17p-10);
    p = __fma_rn(p, r, 0x1.1111111111111p-7);
    p = __fma_rn(p, r, 0x1.5555555555555p-5);
    p = __fma_rn(p, r, 0x1.5555555555555p-3);
    p = __fma_rn(p, r, 0x1p-1);
    p = __fma_rn(p, r, 1.0);
    p = __fma_rn(p, r, 1.0);
    double s = __longlong_as_double((long long)((int)k + 1023) << 52);
    return __double2float_rn(__dmul_rn(p, s));
}
// silu(x) = x / (1 + expf(-x)) (reference tlm_model.c:171)
// Programmatic dependent launch: wait until the preceding grid of the
// stream has completed and its writes are visible (returns at once when the
// kernel was not launched as a dependent), then let the next one be
// scheduled.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
}

// 1 / sqrtf((float)(ss / n) + eps), ss = sum of x[i]^2 in double: the
// reference's RMSNorm scale (rmsnorm, src/lib/tlm_model.c:164-169), whose
// ss is a serial double sum. Every thread of the block calls this (blockDim
// a multiple of 32, at most 1024): a sum of the exact squares in any order
// gives ss within an error bound; when both ends of the bound round to the same
// float mean that is the reference's float, else thread 0 runs the serial
// sum. red: shared [32], r_sh: shared.
__device__ __forceinline__ float block_rms_inv(const float *x, int n, float eps, double *red, float *r_sh) {
    double s = 0.0;
    int i = threadIdx.x;
    const int nt = blockDim.x;
    for (; i + 7 * nt < n; i += 8 * nt) {   // eight loads in flight, then their squares
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = x[i + u * nt];
#pragma unroll
        for (int u = 0; u < 8; u++) s = __dadd_rn(s, __dmul_rn((double)v[u], (double)v[u]));
    }
    for (; i < n; i += nt) s = __dadd_rn(s, __dmul_rn((double)x[i], (double)x[i]));
    for (int o = 16; o > 0; o >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int q = 0; q < (int)(blockDim.x >> 5); q++) t = __dadd_rn(t, red[q]);
        const double bound = __dmul_rn(t, __dmul_rn(2.0 * (double)n + 8.0, 0x1p-53));
        const float flo = __double2float_rn(__ddiv_rn(__dsub_rn(t, bound), (double)n));
        const float fhi = __double2float_rn(__ddiv_rn(__dadd_rn(t, bound), (double)n));
        float f = flo;
        if (flo != fhi) {
            double q = 0.0;
            for (int i = 0; i < n; i++) q = __dadd_rn(q, __dmul_rn((double)x[i], (double)x[i]));
            f = __double2float_rn(__ddiv_rn(q, (double)n));
        }
        *r_sh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(f, eps)));
    }
    __syncthreads();
    return *r_sh;
}

__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, cr_expf(-x))); }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, cr_expf(-x))); }

// RNE then clamp to [-127, 127], NaN -> 0 (reference tlm_quant.c:216-230).
// For |v| < 2^22 the reference's 1.5*2^23 magic sum is exactly round-half-even.
__device__ __forceinline__ int q127(float v) {
    if (v != v) return 0;
    if (v <= -127.0f) return -127;
    if (v >= 127.0f) return 127;
    return __float2int_rn(v);
}

// ---------------------------------------------------------------------------
// activation quantisation of one block (reference tlm_quant.c:458-478).
// `vals` are this lane's NV consecutive inputs (already 0 beyond nvalid; a
// padded zero cannot change amax or raise a NaN/Inf flag). Lanes of the
// calling group (GROUP lanes, aligned) cover one block. Returns d; codes in q.
template <int NV, int GROUP>
__device__ __forceinline__ float act_block_codes(const float (&vals)[NV], int (&q)[NV]) {
    uint32_t amax_bits = 0u;
    int nan_seen = 0, inf_seen = 0;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        float a = fabsf(vals[i]);
        if (a != a) nan_seen = 1;
        else if (a == __uint_as_float(0x7F800000u)) inf_seen = 1;
        else amax_bits = max(amax_bits, __float_as_uint(a));
    }
    const unsigned full = 0xFFFFFFFFu;
#pragma unroll
    for (int o = GROUP / 2; o > 0; o >>= 1) {
        amax_bits = max(amax_bits, __shfl_xor_sync(full, amax_bits, o));
        nan_seen |= __shfl_xor_sync(full, nan_seen, o);
        inf_seen |= __shfl_xor_sync(full, inf_seen, o);
    }
    float amax = __uint_as_float(amax_bits);
#pragma unroll
    for (int i = 0; i < NV; i++) q[i] = 0;
    if (nan_seen || inf_seen) return nan_seen ? __uint_as_float(0x7FC00000u) : __uint_as_float(0x7F800000u);
    if (!(amax > 0.0f)) return 0.0f;
    float d = __fdiv_rn(amax, 127.0f);
    if (amax >= 0x1p-100f) {
        float inv = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < NV; i++) q[i] = q127(__fmul_rn(vals[i], inv));
    } else {
        double inv = __ddiv_rn(127.0, (double)amax);
#pragma unroll
        for (int i = 0; i < NV; i++) q[i] = q127(__double2float_rn(__dmul_rn((double)vals[i], inv)));
    }
    return d;
}

// A full warp quantises one Q8_K block (256 values, 8 per lane) into `dst`
// (292 bytes, 4-byte aligned). x: the block's inputs, nvalid of them.
__device__ __forceinline__ void warp_quant_q8k(const float *x, int nvalid, uint8_t *dst, int lane) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int e = lane * 8 + i;
        v[i] = e < nvalid ? x[e] : 0.0f;
    }
    int q[8];
    float d = act_block_codes<8, 32>(v, q);
    uint32_t w0 = (q[0] & 255) | ((q[1] & 255) << 8) | ((q[2] & 255) << 16) | ((uint32_t)(q[3] & 255) << 24);
    uint32_t w1 = (q[4] & 255) | ((q[5] & 255) << 8) | ((q[6] & 255) << 16) | ((uint32_t)(q[7] & 255) << 24);
    int s = q[0] + q[1] + q[2] + q[3] + q[4] + q[5] + q[6] + q[7];
    s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
    uint32_t *w = reinterpret_cast<uint32_t *>(dst + 4 + 8 * lane);
    w[0] = w0;
    w[1] = w1;
    if ((lane & 1) == 0) *reinterpret_cast<int16_t *>(dst + 260 + lane) = (int16_t)s;
    if (lane == 0) *reinterpret_cast<float *>(dst) = d;
}

// A full warp quantises one Q8_0 activation block (32 values, one per lane)
// into `dst` (36 bytes: f32 d, int8 q[32]).
__device__ __forceinline__ void warp_quant_q80(const float *x, int nvalid, uint8_t *dst, int lane) {
    float v[1] = { lane < nvalid ? x[lane] : 0.0f };
    int q[1];
    float d = act_block_codes<1, 32>(v, q);
    int q0 = __shfl_sync(0xFFFFFFFFu, q[0], (lane & 7) * 4 + 0);
    int q1 = __shfl_sync(0xFFFFFFFFu, q[0], (lane & 7) * 4 + 1);
    int q2 = __shfl_sync(0xFFFFFFFFu, q[0], (lane & 7) * 4 + 2);
    int q3 = __shfl_sync(0xFFFFFFFFu, q[0], (lane & 7) * 4 + 3);
    if (lane < 8)
        reinterpret_cast<uint32_t *>(dst + 4)[lane] =
            (q0 & 255) | ((q1 & 255) << 8) | ((q2 & 255) << 16) | ((uint32_t)(q3 & 255) << 24);
    if (lane == 0) *reinterpret_cast<float *>(dst) = d;
}

// ---------------------------------------------------------------------------
// weight loads at a known minimum alignment A (1, 2, 4 or 16 bytes).
template <int A> struct WLoad {
    static __device__ __forceinline__ uint32_t u32(const uint8_t *p) {
        if constexpr (A >= 4) {
            return __ldg(reinterpret_cast<const uint32_t *>(p));
        } else if constexpr (A == 2) {
            uint32_t lo = __ldg(reinterpret_cast<const uint16_t *>(p));
            uint32_t hi = __ldg(reinterpret_cast<const uint16_t *>(p + 2));
            return lo | (hi << 16);
        } else {
            return (uint32_t)__ldg(p) | ((uint32_t)__ldg(p + 1) << 8) | ((uint32_t)__ldg(p + 2) << 16) |
                   ((uint32_t)__ldg(p + 3) << 24);
        }
    }
    static __device__ __forceinline__ uint32_t u16(const uint8_t *p) {
        if constexpr (A >= 2) return __ldg(reinterpret_cast<const uint16_t *>(p));
        else return (uint32_t)__ldg(p) | ((uint32_t)__ldg(p + 1) << 8);
    }
    static __device__ __forceinline__ uint32_t u8(const uint8_t *p) { return __ldg(p); }
};

// Shared-memory weight loads at 2-byte (or better) alignment: two aligned
// words and a byte permute.
struct SLoad {
    static __device__ __forceinline__ uint32_t u32(const uint8_t *p) {
        uintptr_t a = reinterpret_cast<uintptr_t>(p);
        const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
        uint32_t o = (uint32_t)(a & 3u);
        if (o == 0u) return w[0];
        return __byte_perm(w[0], w[1], 0x3210u + 0x1111u * o);
    }
    static __device__ __forceinline__ uint32_t u16(const uint8_t *p) {
        return *reinterpret_cast<const uint16_t *>(p);
    }
    static __device__ __forceinline__ uint32_t u8(const uint8_t *p) { return *p; }
};

__device__ __forceinline__ uint32_t act32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// 6-bit scale and min k of a Q4_K/Q5_K block from the scale words
// a0 = s12[0..3], a1 = s12[4..7], a2 = s12[8..11] (reference tlm_quant.c:253-261).
__device__ __forceinline__ void kq_scale_min(uint32_t a0, uint32_t a1, uint32_t a2, int k, int &sc, int &mn) {
    if (k < 4) {
        sc = (a0 >> (8 * k)) & 63;
        mn = (a1 >> (8 * k)) & 63;
    } else {
        int i = k - 4;
        sc = ((a2 >> (8 * i)) & 15) | (((a0 >> (8 * i + 6)) & 3) << 4);
        mn = ((a2 >> (8 * i + 4)) & 15) | (((a1 >> (8 * i + 6)) & 3) << 4);
    }
}

// ---------------------------------------------------------------------------
// Lane share of one block's exact integer partials. The 8 lanes j = 0..7 of
// a group together cover the block; summing their (is, ms) over the group
// gives the reference's isum / msum exactly (integer addition is
// associative). `blk` = weight block, `act` = activation block.
template <class L>
__device__ __forceinline__ void part_q4k(const uint8_t *blk, const uint8_t *act, int j, int &is, int &ms) {
    uint32_t a0 = L::u32(blk + 4), a1 = L::u32(blk + 8), a2 = L::u32(blk + 12);
    int c = j >> 1, l0 = 16 * (j & 1);
    int sc0, mn0, sc1, mn1, scj, mnj;
    kq_scale_min(a0, a1, a2, 2 * c, sc0, mn0);
    kq_scale_min(a0, a1, a2, 2 * c + 1, sc1, mn1);
    kq_scale_min(a0, a1, a2, j, scj, mnj);
    const uint8_t *qs = blk + 16 + 16 * j;
    const uint8_t *xl = act + 4 + 64 * c + l0, *xh = xl + 32;
    int slo = 0, shi = 0;
#pragma unroll
    for (int w = 0; w < 4; w++) {
        uint32_t q = L::u32(qs + 4 * w);
        slo = dp4(q & 0x0F0F0F0Fu, act32(xl + 4 * w), slo);
        shi = dp4((q >> 4) & 0x0F0F0F0Fu, act32(xh + 4 * w), shi);
    }
    is = sc0 * slo + sc1 * shi;
    int16_t b0 = *reinterpret_cast<const int16_t *>(act + 260 + 4 * j);
    int16_t b1 = *reinterpret_cast<const int16_t *>(act + 262 + 4 * j);
    ms = mnj * ((int)b0 + (int)b1);
}

template <class L>
__device__ __forceinline__ void part_q5k(const uint8_t *blk, const uint8_t *act, int j, int &is, int &ms) {
    uint32_t a0 = L::u32(blk + 4), a1 = L::u32(blk + 8), a2 = L::u32(blk + 12);
    int c = j >> 1, l0 = 16 * (j & 1);
    int sc0, mn0, sc1, mn1, scj, mnj;
    kq_scale_min(a0, a1, a2, 2 * c, sc0, mn0);
    kq_scale_min(a0, a1, a2, 2 * c + 1, sc1, mn1);
    kq_scale_min(a0, a1, a2, j, scj, mnj);
    const uint8_t *qh = blk + 16 + l0, *qs = blk + 48 + 16 * j;
    const uint8_t *xl = act + 4 + 64 * c + l0, *xh = xl + 32;
    int slo = 0, shi = 0;
#pragma unroll
    for (int w = 0; w < 4; w++) {
        uint32_t q = L::u32(qs + 4 * w), h = L::u32(qh + 4 * w);
        uint32_t lo = (q & 0x0F0F0F0Fu) | (((h >> (2 * c)) & 0x01010101u) << 4);
        uint32_t hi = ((q >> 4) & 0x0F0F0F0Fu) | (((h >> (2 * c + 1)) & 0x01010101u) << 4);
        slo = dp4(lo, act32(xl + 4 * w), slo);
        shi = dp4(hi, act32(xh + 4 * w), shi);
    }
    is = sc0 * slo + sc1 * shi;
    int16_t b0 = *reinterpret_cast<const int16_t *>(act + 260 + 4 * j);
    int16_t b1 = *reinterpret_cast<const int16_t *>(act + 262 + 4 * j);
    ms = mnj * ((int)b0 + (int)b1);
}

// Q6_K: lane j covers half h = j/4 and l = 8*(j%4) .. +7 of that half, i.e.
// the four runs of 8 elements 128h + 32m + l (m = 0..3), each inside one
// group of 16 (reference tlm_quant.c:856-882).
template <class L>
__device__ __forceinline__ void part_q6k(const uint8_t *blk, const uint8_t *act, int j, int &is, int &ms) {
    int h = j >> 2, l0 = 8 * (j & 3);
    const uint8_t *qa = blk + 64 * h + l0, *qb = qa + 32, *qh = blk + 128 + 32 * h + l0;
    const uint8_t *x = act + 4 + 128 * h + l0;
    int s[4] = { 0, 0, 0, 0 };
#pragma unroll
    for (int w = 0; w < 2; w++) {
        uint32_t A = L::u32(qa + 4 * w), B = L::u32(qb + 4 * w), C = L::u32(qh + 4 * w);
        uint32_t u0 = (A & 0x0F0F0F0Fu) | ((C & 0x03030303u) << 4);
        uint32_t u1 = (B & 0x0F0F0F0Fu) | (((C >> 2) & 0x03030303u) << 4);
        uint32_t u2 = ((A >> 4) & 0x0F0F0F0Fu) | (((C >> 4) & 0x03030303u) << 4);
        uint32_t u3 = ((B >> 4) & 0x0F0F0F0Fu) | (((C >> 6) & 0x03030303u) << 4);
        s[0] = dp4(u0, act32(x + 4 * w), s[0]);
        s[1] = dp4(u1, act32(x + 32 + 4 * w), s[1]);
        s[2] = dp4(u2, act32(x + 64 + 4 * w), s[2]);
        s[3] = dp4(u3, act32(x + 96 + 4 * w), s[3]);
    }
    // groups of this lane's runs: g_m = 8h + 2m + (l0 >= 16)
    int gb = 8 * h + (l0 >> 4);
    uint32_t scw0 = L::u32(blk + 192 + 8 * h), scw1 = L::u32(blk + 196 + 8 * h);
    // sc[8h + t] for t = 0..7 live in bytes of scw0 (t<4) / scw1 (t>=4)
    int acc = 0;
#pragma unroll
    for (int m = 0; m < 4; m++) {
        int t = 2 * m + (l0 >> 4);
        uint32_t wsel = t < 4 ? scw0 : scw1;
        int sc = (int)(int8_t)((wsel >> (8 * (t & 3))) & 255u);
        acc += sc * s[m];
        // the -32 * bsums term of group gb+2m, counted once (by the lane
        // holding the group's first 8 elements)
        if ((l0 & 8) == 0) {
            int16_t bs = *reinterpret_cast<const int16_t *>(act + 260 + 2 * (gb + 2 * m));
            acc -= 32 * sc * (int)bs;
        }
    }
    is = acc;
    ms = 0;
}

template <class L>
__device__ __forceinline__ void part_q8k(const uint8_t *blk, const uint8_t *act, int j, int &is, int &ms) {
    const uint8_t *q = blk + 4 + 32 * j, *x = act + 4 + 32 * j;
    int s = 0;
#pragma unroll
    for (int w = 0; w < 8; w++) s = dp4(L::u32(q + 4 * w), act32(x + 4 * w), s);
    is = s;
    ms = 0;
}

template <class L>
__device__ __forceinline__ void part_q80(const uint8_t *blk, const uint8_t *act, int j, int &is, int &ms) {
    is = dp4(L::u32(blk + 2 + 4 * j), act32(act + 4 + 4 * j), 0);
    ms = 0;
}

// Doubled E2M1 value of a 4-bit code (reference k_e2m1_x2, tlm_quant.c:515):
// magnitudes 0 1 2 3 4 6 8 12 for codes 0..7, bit 3 is the sign.
__device__ __forceinline__ int e2m1x2(uint32_t c) {
    int m = (int)(c & 7u);
    int v = m < 4 ? m : (m < 6 ? 2 * m - 4 : 4 * m - 16);
    return (c & 8u) ? -v : v;
}

template <class L>
__device__ __forceinline__ void part_mxfp4(const uint8_t *blk, const uint8_t *act, int j, int &is, int &ms) {
    uint32_t b0 = L::u8(blk + 1 + 2 * j), b1 = L::u8(blk + 2 + 2 * j);
    const int8_t *x = reinterpret_cast<const int8_t *>(act + 4);
    is = e2m1x2(b0 & 15u) * x[2 * j] + e2m1x2(b1 & 15u) * x[2 * j + 1] + e2m1x2(b0 >> 4) * x[2 * j + 16] +
         e2m1x2(b1 >> 4) * x[2 * j + 17];
    ms = 0;
}

template <class L>
__device__ __forceinline__ void block_part(int dt, const uint8_t *blk, const uint8_t *act, int j, int &is, int &ms) {
    switch (dt) {
    case DT_Q4_K: part_q4k<L>(blk, act, j, is, ms); break;
    case DT_Q5_K: part_q5k<L>(blk, act, j, is, ms); break;
    case DT_Q6_K: part_q6k<L>(blk, act, j, is, ms); break;
    case DT_Q8_K: part_q8k<L>(blk, act, j, is, ms); break;
    case DT_Q8_0: part_q80<L>(blk, act, j, is, ms); break;
    case DT_MXFP4: part_mxfp4<L>(blk, act, j, is, ms); break;
    default: is = 0; ms = 0; break;
    }
}

// Float factors of one block's fmaf step(s): dA = d_w * d_a and dM =
// dmin_w * d_a (reference tlm_quant.c:838-840, :880, :790, :808, :900).
template <class L>
__device__ __forceinline__ void block_scales(int dt, const uint8_t *blk, const uint8_t *act, float &dA, float &dM) {
    float da = *reinterpret_cast<const float *>(act);
    dM = 0.0f;
    switch (dt) {
    case DT_Q4_K: case DT_Q5_K:
        dA = __fmul_rn(f16_to_f32(L::u16(blk)), da);
        dM = __fmul_rn(f16_to_f32(L::u16(blk + 2)), da);
        break;
    case DT_Q6_K: dA = __fmul_rn(f16_to_f32(L::u16(blk + 208)), da); break;
    case DT_Q8_0: dA = __fmul_rn(f16_to_f32(L::u16(blk)), da); break;
    case DT_Q8_K: dA = __fmul_rn(__uint_as_float(L::u32(blk)), da); break;
    case DT_MXFP4: dA = __fmul_rn(e8m0_half(L::u8(blk)), da); break;
    default: dA = 0.0f; break;
    }
}

// One block's step of the serial chain.
__device__ __forceinline__ float chain_step(int dt, float acc, float dA, float dM, int is, int ms) {
    acc = __fmaf_rn(dA, (float)is, acc);
    if (dt == DT_Q4_K || dt == DT_Q5_K) acc = __fmaf_rn(-dM, (float)ms, acc);
    return acc;
}

// Exact integer partials of one block plus its float factors, staged in
// shared memory between the parallel integer stage and the serial chain.
struct BlockPart {
    int is, ms;
    float dA, dM;
};
constexpr int FCHUNK = 32;   // blocks per shared-memory pass of one row

// Reduce one (is, ms) pair over the 8 lanes of a group.
__device__ __forceinline__ void group8_sum(int &is, int &ms) {
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        is += __shfl_xor_sync(0xFFFFFFFFu, is, o);
        ms += __shfl_xor_sync(0xFFFFFFFFu, ms, o);
    }
}

// The reference's fixed 32-lane float reduction tree (tlm_quant.c:724-730)
// as shuffles; the result is valid in lane 0.
__device__ __forceinline__ float tree32(float v) {
    v = __fadd_rn(v, __shfl_down_sync(0xFFFFFFFFu, v, 16));
    v = __fadd_rn(v, __shfl_down_sync(0xFFFFFFFFu, v, 8));
    v = __fadd_rn(v, __shfl_down_sync(0xFFFFFFFFu, v, 4));
    v = __fadd_rn(v, __shfl_down_sync(0xFFFFFFFFu, v, 2));
    v = __fadd_rn(v, __shfl_down_sync(0xFFFFFFFFu, v, 1));
    return v;
}

// ---------------------------------------------------------------------------
// router top-k (reference tlm_model.c:776-839), one warp. Entry e lives in
// lane e % 32, slot e / 32. The warp keeps the probabilities and the
// selection keys in shared memory (RT_SCRATCH words), not in registers, so
// a producer warp that routes stays small.
constexpr int RT_PER = 16;                  // E <= 512
constexpr int RT_SCRATCH = 2 * RT_PER * 32; // 32-bit words of router scratch

// Order-preserving map of a non-NaN float to u32 (-0 and +0 map alike, as
// they compare equal); 0 is below every key and marks "not a candidate".
__device__ __forceinline__ uint32_t fkey(float v) {
    uint32_t b = __float_as_uint(__fadd_rn(v, 0.0f));
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Top-k by key among entries with a nonzero key (unmasked, not NaN); ties ->
// lowest index; when no candidate is left, the lowest entry of `avail`
// (unmasked, unused), else 0 (reference topk, tlm_model.c:776-795). Each
// round is one warp max-reduction of the lanes' best keys and one
// min-reduction of the indices holding it; only the lane that owned the
// pick rescans its slots. Lane r returns ids[r] in id0 and ids[r + 32] in id1.
__device__ __forceinline__ void warp_topk(uint32_t *key_sm, uint32_t avail, int E, int k, int lane, int &id0,
                                          int &id1) {
    const int nper = (E + 31) >> 5;
    uint32_t bk = 0u, bi = 0xFFFFFFFFu;
    for (int s = 0; s < nper; s++) {
        const int e = lane + 32 * s;
        if (e < E) {
            const uint32_t key = key_sm[e];
            if (key > bk) { bk = key; bi = (uint32_t)e; }
        }
    }
    id0 = id1 = 0;
    for (int r = 0; r < k; r++) {
        const uint32_t m = __reduce_max_sync(0xFFFFFFFFu, bk);
        uint32_t pick;
        if (m != 0u) {
            pick = __reduce_min_sync(0xFFFFFFFFu, bk == m ? bi : 0xFFFFFFFFu);
        } else {
            const uint32_t fb = avail ? (uint32_t)(lane + 32 * (__ffs(avail) - 1)) : 0xFFFFFFFFu;
            pick = __reduce_min_sync(0xFFFFFFFFu, fb);
            if (pick == 0xFFFFFFFFu) pick = 0u;
        }
        if (lane == r) id0 = (int)pick;
        if (lane + 32 == r) id1 = (int)pick;
        if ((int)(pick & 31u) == lane && (int)pick < E) {
            avail &= ~(1u << (pick >> 5));
            key_sm[pick] = 0u;
            bk = 0u;
            bi = 0xFFFFFFFFu;
            for (int s = 0; s < nper; s++) {
                const int e = lane + 32 * s;
                if (e < E) {
                    const uint32_t key = key_sm[e];
                    if (key > bk) { bk = key; bi = (uint32_t)e; }
                }
            }
        }
    }
}

// Weight of rank r held by lane r % 32 (w0 for r < 32, w1 above).
__device__ __forceinline__ float rank_w(float w0, float w1, int r) {
    return __shfl_sync(0xFFFFFFFFu, r < 32 ? w0 : w1, r & 31);
}

// Router of one token by one full warp (lane = 0..31). scratch: RT_SCRATCH
// words of shared memory; ids_sm / w_sm: outputs (k entries), valid in all
// lanes after the call (it ends with __syncwarp). k <= 64.
static __device__ __forceinline__ void warp_route(int router, const float *__restrict__ logits,
                                                  const uint8_t *__restrict__ mask, const float *__restrict__ bias,
                                                  int E, int k, float routed_scale, uint32_t *scratch,
                                                  int32_t *ids_sm, float *w_sm, int lane) {
    float *p_sm = reinterpret_cast<float *>(scratch);
    uint32_t *key_sm = scratch + RT_PER * 32;
    const int nper = (E + 31) >> 5;
    uint32_t avail = 0u;   // bit s: entry lane + 32 s is unmasked
    for (int s = 0; s < nper; s++) {
        const int e = lane + 32 * s;
        if (e < E && !(mask && mask[e])) avail |= 1u << s;
    }
    if (router == 2) {
        for (int s = 0; s < nper; s++) {
            const int e = lane + 32 * s;
            if (e >= E) continue;
            const float p = sigmoid_f(logits[e]);
            const float v = __fadd_rn(p, bias ? bias[e] : 0.0f);
            p_sm[e] = p;
            key_sm[e] = (((avail >> s) & 1u) && v == v) ? fkey(v) : 0u;
        }
        __syncwarp();
        int id0, id1;
        warp_topk(key_sm, avail, E, k, lane, id0, id1);
        __syncwarp();
        const float p0 = lane < k ? p_sm[id0] : 0.0f, p1 = lane + 32 < k ? p_sm[id1] : 0.0f;
        double sum = 0.0;
        for (int r = 0; r < k; r++) sum = __dadd_rn(sum, (double)rank_w(p0, p1, r));
        const float inv = __double2float_rn(__ddiv_rn(1.0, __dadd_rn(sum, 1e-20)));
        if (lane < k) {
            ids_sm[lane] = id0;
            w_sm[lane] = __fmul_rn(__fmul_rn(p0, inv), routed_scale);
        }
        if (lane + 32 < k) {
            ids_sm[lane + 32] = id1;
            w_sm[lane + 32] = __fmul_rn(__fmul_rn(p1, inv), routed_scale);
        }
        __syncwarp();
        return;
    }
    // softmax over the routable entries
    float mxl = -__uint_as_float(0x7F800000u);
    for (int s = 0; s < nper; s++) {
        const int e = lane + 32 * s;
        if ((avail >> s) & 1u) {
            const float l = logits[e];
            if (l > mxl) mxl = l;
        }
    }
    const uint32_t mk = __reduce_max_sync(0xFFFFFFFFu, fkey(mxl));
    const float mx = __uint_as_float((mk & 0x80000000u) ? (mk & 0x7FFFFFFFu) : ~mk);
    const bool none = mx == -__uint_as_float(0x7F800000u);
    double part = 0.0;
    uint32_t min_bits = 0x7F800000u;   // smallest nonzero p seen
    for (int s = 0; s < nper; s++) {
        const int e = lane + 32 * s;
        if (e >= E) continue;
        const float l = logits[e];
        const float p = (!((avail >> s) & 1u) || !(l == l) || none) ? 0.0f : cr_expf(__fsub_rn(l, mx));
        p_sm[e] = p;
        part = __dadd_rn(part, (double)p);
        if (p != 0.0f) min_bits = min(min_bits, __float_as_uint(p));
    }
    // The reference sums in double, sequentially in index order. When every
    // nonzero term is >= 2^(floor(log2 E) - 29) all partial sums are exact
    // in double, so any order gives the same sum; otherwise lane 0 redoes it
    // sequentially.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part = __dadd_rn(part, __shfl_xor_sync(0xFFFFFFFFu, part, o));
    min_bits = __reduce_min_sync(0xFFFFFFFFu, min_bits);
    const int lg = 31 - __clz(E);
    const bool exact = min_bits == 0x7F800000u || __uint_as_float(min_bits) >= ldexpf(1.0f, lg - 29);
    __syncwarp();
    double sum = part;
    if (!exact) {
        if (lane == 0) {
            double q = 0.0;
            for (int e = 0; e < E; e++) q = __dadd_rn(q, (double)p_sm[e]);
            part = q;
        }
        sum = __shfl_sync(0xFFFFFFFFu, part, 0);
    }
    const float inv = sum > 0.0 ? __double2float_rn(__ddiv_rn(1.0, sum)) : 0.0f;
    for (int s = 0; s < nper; s++) {
        const int e = lane + 32 * s;
        if (e >= E) continue;
        const float p = __fmul_rn(p_sm[e], inv);
        p_sm[e] = p;
        key_sm[e] = ((avail >> s) & 1u) ? fkey(p) : 0u;   // p is never NaN here
    }
    __syncwarp();
    int id0, id1;
    warp_topk(key_sm, avail, E, k, lane, id0, id1);
    __syncwarp();
    float w0 = lane < k ? p_sm[id0] : 0.0f, w1 = lane + 32 < k ? p_sm[id1] : 0.0f;
    if (router == 0) {
        double t = 0.0;
        for (int r = 0; r < k; r++) t = __dadd_rn(t, (double)rank_w(w0, w1, r));
        if (t > 0.0) {
            const float it = __double2float_rn(__ddiv_rn(1.0, t));
            w0 = __fmul_rn(w0, it);
            w1 = __fmul_rn(w1, it);
        }
    }
    if (routed_scale != 1.0f) {
        w0 = __fmul_rn(w0, routed_scale);
        w1 = __fmul_rn(w1, routed_scale);
    }
    if (lane < k) {
        ids_sm[lane] = id0;
        w_sm[lane] = w0;
    }
    if (lane + 32 < k) {
        ids_sm[lane + 32] = id1;
        w_sm[lane + 32] = w1;
    }
    __syncwarp();
}

}  // namespace tlmg
