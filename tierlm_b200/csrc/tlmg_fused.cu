// tlmg_fused.cu - persistent expert-FFN kernel for batch-1 decode (sm_100a).
//
// One launch = one token through one MoE layer's routed experts
// (reference run_batch() + combine, src/lib/tlm_model.c:900-938, :1029-1036,
// with route(), :798-839, folded in). One CTA per SM: 16 consumer warps and
// one producer warp.
//
//   prologue   all threads: router (softmax top-k by rank, exact), x ->
//              Q8_K in shared memory, this CTA's chunk plan (host-built per
//              dtype signature: only the expert base addresses depend on
//              the routing).
//   producer   streams each chunk of selected weight rows HBM -> a ring of
//              shared-memory stages with cp.async.bulk (TMA, no multicast):
//              phase A chunks first, then phase B chunks, so the down
//              weights are on chip when h is ready.
//   phase A    gate/up + SwiGLU. A warp takes one (gate, up) row pair at a
//              time; lane l owns the 64-element quarter(s) l (+32) of the
//              row, whose activation codes stay in registers for the whole
//              launch. Exact int32 quarter sums (dp4a) are combined per
//              block with two shuffles; lanes 0 / 1 run the gate / up fmaf
//              chains over the blocks in ascending order.
//   barrier    grid-wide arrival counter (cooperative launch: all CTAs are
//              co-resident; bounded wait).
//   phase B    every CTA re-quantises h (k x de) into shared memory, then a
//              warp takes one output row: lane l owns quarters l, l+32, ...
//              of the k experts' down rows; lanes r < k run expert r's chain;
//              lane 0 combines ffn = sum_r w[r] * eo_r in ascending rank.
//
// Numerics are the reference contract (src/lib/tlm_quant.h:113-128): exact
// int32 per block, one fmaf per block (two for Q4_K/Q5_K) in block order.
// Every wait is bounded; on expiry the kernel raises an error bit the host
// reads, waits (bounded) for its own copies in flight and returns.
#include <algorithm>
#include <cstdio>
#include <vector>

#include <cuda_fp16.h>

#include "tlmg_dev.cuh"
#include "tlmg_fused.cuh"
#include "tlmg_internal.h"

namespace tlmg {

constexpr int NCW = 16;                 // consumer warps
constexpr int NTHREADS = 32 * (NCW + 1);
constexpr int MAXCH = FUSED_MAXCH;
constexpr int MAXK = 16;
constexpr int SLOT_BYTES = 24576;
constexpr uint64_t WAIT_NS = 200000000ull;       // 0.2 s: an mbarrier wait gives up
constexpr uint64_t BARRIER_NS = 500000000ull;    // 0.5 s: the grid barrier gives up

// ---------------------------------------------------------------------------
// PTX helpers: mbarrier + bulk copy (shared::cta addresses)
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// try_wait with a suspend-time hint: the warp sleeps in hardware until the
// phase completes (or the hint expires) instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Wait for the phase with `parity` to complete, for at most WAIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (now_ns() - t0 > WAIT_NS) return false;
    }
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(__cvta_generic_to_global(src)), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory"); }
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ld_acquire64(const unsigned long long *p) {
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Record error bits for the host (mapped pinned word) and make them sticky
// for later launches (device word bar[2]) until the host resets them.
__device__ __forceinline__ void raise_error(uint32_t *err, uint32_t *bar, uint32_t bits) {
    volatile uint32_t *e = err;
    *e = *e | bits;
    atomicOr(&bar[2], bits);
}

// ---------------------------------------------------------------------------
// shared-memory loads
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
// One "unit" = 64 elements of one 256-element block (quarter q = 0..3).
// The activation of a unit, in registers.
struct UAct {
    uint32_t c[16];   // 64 int8 codes in the order the weight dtype consumes them
    int bs[4];        // the activation group sums the unit's min / offset terms need
    float d;          // activation block scale
};

// Q8_K activation blocks in shared memory, bank-swizzled: the 16-byte
// piece p (codes 16p .. 16p+15) of block beta of an NB-block vector lives at
// codes + (p * NB + beta) * 16, so lanes that read the same piece of
// consecutive blocks hit consecutive banks. bsums[16] and d per block
// separately.
__device__ __forceinline__ const uint8_t *swz(const uint8_t *codes, int NB, int beta, int p) {
    return codes + ((size_t)p * NB + beta) * 16;
}
// The activation of unit (block beta, quarter q) in the order the weight
// dtype consumes it. Q4_K / Q5_K quarter q: elements 64q .. 64q+63
// (sub-blocks 2q, 2q+1). Q6_K quarter q = (h = q/2, lq = q%2): elements
// 128h + 32m + 16lq + 0..15, m = 0..3 (groups 8h + 2m + lq), matching the
// ql/qh layout (reference tlm_quant.c:406-411).
template <int DT>
__device__ __forceinline__ void load_uact(const uint8_t *codes, int NB, int beta, const int16_t *bs, float d, int q,
                                          UAct &a) {
    if constexpr (DT == DT_Q6_K) {
        const int h = q >> 1, lq = q & 1;
#pragma unroll
        for (int m = 0; m < 4; m++) {
            uint4 v = lds128(swz(codes, NB, beta, 8 * h + 2 * m + lq));
            a.c[4 * m + 0] = v.x; a.c[4 * m + 1] = v.y; a.c[4 * m + 2] = v.z; a.c[4 * m + 3] = v.w;
            a.bs[m] = bs[8 * h + 2 * m + lq];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint4 v = lds128(swz(codes, NB, beta, 4 * q + i));
            a.c[4 * i + 0] = v.x; a.c[4 * i + 1] = v.y; a.c[4 * i + 2] = v.z; a.c[4 * i + 3] = v.w;
        }
        a.bs[0] = (int)bs[4 * q] + (int)bs[4 * q + 1];
        a.bs[1] = (int)bs[4 * q + 2] + (int)bs[4 * q + 3];
        a.bs[2] = a.bs[3] = 0;
    }
    a.d = d;
}

// Exact int32 partials of one unit of a weight block in shared memory, and
// the block's float factors (used from the lane that owns quarter 0).
template <int DT>
__device__ __forceinline__ void unit_dot(const uint8_t *blk, int q, const UAct &a, int &is, int &ms, float &dA,
                                         float &dM) {
    if constexpr (DT == DT_Q4_K || DT == DT_Q5_K) {
        const uint4 hd = lds128(blk);
        uint32_t qw[8], hw[8];
        const int qoff = DT == DT_Q4_K ? 16 : 48;
        uint4 v0 = lds128(blk + qoff + 32 * q), v1 = lds128(blk + qoff + 16 + 32 * q);
        qw[0] = v0.x; qw[1] = v0.y; qw[2] = v0.z; qw[3] = v0.w;
        qw[4] = v1.x; qw[5] = v1.y; qw[6] = v1.z; qw[7] = v1.w;
        if constexpr (DT == DT_Q5_K) {
            uint4 h0 = lds128(blk + 16), h1 = lds128(blk + 32);
            hw[0] = h0.x; hw[1] = h0.y; hw[2] = h0.z; hw[3] = h0.w;
            hw[4] = h1.x; hw[5] = h1.y; hw[6] = h1.z; hw[7] = h1.w;
        }
        int lo = 0, hi = 0;
#pragma unroll
        for (int w = 0; w < 8; w++) {
            uint32_t l4 = qw[w] & 0x0F0F0F0Fu, h4 = (qw[w] >> 4) & 0x0F0F0F0Fu;
            if constexpr (DT == DT_Q5_K) {
                l4 |= ((hw[w] >> (2 * q)) & 0x01010101u) << 4;
                h4 |= ((hw[w] >> (2 * q + 1)) & 0x01010101u) << 4;
            }
            lo = dp4(l4, a.c[w], lo);
            hi = dp4(h4, a.c[8 + w], hi);
        }
        int sc0, mn0, sc1, mn1;
        kq_scale_min(hd.y, hd.z, hd.w, 2 * q, sc0, mn0);
        kq_scale_min(hd.y, hd.z, hd.w, 2 * q + 1, sc1, mn1);
        is = sc0 * lo + sc1 * hi;
        ms = mn0 * a.bs[0] + mn1 * a.bs[1];
        dA = __fmul_rn(h2f(hd.x & 0xFFFFu), a.d);
        dM = __fmul_rn(h2f(hd.x >> 16), a.d);
    } else {   // Q6_K: 2-byte aligned blocks
        const int h = q >> 1, lq = q & 1;
        const uint4 A = lds128_a2(blk + 64 * h + 16 * lq), B = lds128_a2(blk + 64 * h + 32 + 16 * lq);
        const uint4 Cq = lds128_a2(blk + 128 + 32 * h + 16 * lq);
        const uint32_t aw[4] = { A.x, A.y, A.z, A.w }, bw[4] = { B.x, B.y, B.z, B.w },
                       cw[4] = { Cq.x, Cq.y, Cq.z, Cq.w };
        int g0 = 0, g1 = 0, g2 = 0, g3 = 0;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            uint32_t u0 = (aw[w] & 0x0F0F0F0Fu) | ((cw[w] & 0x03030303u) << 4);
            uint32_t u1 = (bw[w] & 0x0F0F0F0Fu) | (((cw[w] >> 2) & 0x03030303u) << 4);
            uint32_t u2 = ((aw[w] >> 4) & 0x0F0F0F0Fu) | (((cw[w] >> 4) & 0x03030303u) << 4);
            uint32_t u3 = ((bw[w] >> 4) & 0x0F0F0F0Fu) | (((cw[w] >> 6) & 0x03030303u) << 4);
            g0 = dp4(u0, a.c[w], g0);
            g1 = dp4(u1, a.c[4 + w], g1);
            g2 = dp4(u2, a.c[8 + w], g2);
            g3 = dp4(u3, a.c[12 + w], g3);
        }
        const uint32_t s0 = lds32_a2(blk + 192 + 8 * h), s1 = lds32_a2(blk + 196 + 8 * h);
        // group 8h + 2m + lq: scale byte 2m + lq of the half's 8 scales
        is = sbyte(s0, lq) * (g0 - 32 * a.bs[0]) + sbyte(s0, 2 + lq) * (g1 - 32 * a.bs[1]) +
             sbyte(s1, lq) * (g2 - 32 * a.bs[2]) + sbyte(s1, 2 + lq) * (g3 - 32 * a.bs[3]);
        ms = 0;
        dA = __fmul_rn(h2f(*reinterpret_cast<const uint16_t *>(blk + 208)), a.d);
        dM = 0.0f;
    }
}

// Exact int32 partials of a whole block (four quarters) of a weight block in
// shared memory against activation block beta, and its float factors.
struct BlockSum {
    int is, ms;
    float dA, dM;
};
template <int DT>
__device__ __forceinline__ void block_dot(const uint8_t *blk, const uint8_t *codes, int NB, int beta,
                                          const int16_t *bs, float d, BlockSum &o) {
    o.is = o.ms = 0;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        UAct xa;
        load_uact<DT>(codes, NB, beta, bs, d, q, xa);
        int is, ms;
        unit_dot<DT>(blk, q, xa, is, ms, o.dA, o.dM);
        o.is += is;
        o.ms += ms;
    }
}
// The same for two weight blocks (gate and up) against one activation block.
template <int DT>
__device__ __forceinline__ void block_dot2(const uint8_t *g, const uint8_t *u, const uint8_t *codes, int NB, int beta,
                                           const int16_t *bs, float d, BlockSum &og, BlockSum &ou) {
    og.is = og.ms = ou.is = ou.ms = 0;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        UAct xa;
        load_uact<DT>(codes, NB, beta, bs, d, q, xa);
        int is, ms;
        unit_dot<DT>(g, q, xa, is, ms, og.dA, og.dM);
        og.is += is;
        og.ms += ms;
        unit_dot<DT>(u, q, xa, is, ms, ou.dA, ou.dM);
        ou.is += is;
        ou.ms += ms;
    }
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
// shared-memory layout
constexpr int NBUF = 4;   // routing / h buffers, by token % NBUF
struct SmemLayout {
    uint32_t stage, full, empty, xfull, xempty, idsfree, xs, xc, xd, xbs, hc, hd, hbs, p, ids, w, desc, sl, misc, total;
};
__host__ __device__ inline uint32_t up16(uint32_t v) { return (v + 15u) & ~15u; }
__host__ __device__ inline SmemLayout smem_layout(int D, int de, int k, int nslot) {
    SmemLayout L;
    uint32_t o = 0;
    const uint32_t nbx = (uint32_t)(D / 256), nbh = (uint32_t)(k * (de / 256));
    L.stage = o; o += (uint32_t)nslot * SLOT_BYTES;
    L.full = o; o += 8u * nslot;
    L.empty = o; o += 8u * nslot;
    L.xfull = o; o += 8u;
    L.xempty = o; o += 8u;
    L.idsfree = o; o += 8u * NBUF;
    L.xs = o = up16(o); o += 4u * (uint32_t)D;
    L.xc = o = up16(o); o += 256u * nbx;
    L.xd = o; o += 4u * nbx;
    L.xbs = o = up16(o); o += 32u * nbx;
    L.hc = o = up16(o); o += 256u * nbh;
    L.hd = o; o += 4u * nbh;
    L.hbs = o = up16(o); o += 32u * nbh;
    L.p = o = up16(o); o += 4u * (uint32_t)RT_SCRATCH;
    L.ids = o; o += 4u * 64 * NBUF;
    L.w = o; o += 4u * 64 * NBUF;
    L.desc = o = up16(o); o += (uint32_t)sizeof(ChunkDesc) * MAXCH;
    L.sl = o = up16(o); o += (uint32_t)sizeof(Slot) * MAXK * 2;
    L.misc = o = up16(o); o += 64;
    L.total = o;
    return L;
}

// The launch's schedule, shared by the producer and the consumers: step j
// of 2 * n_tok is phase A (gate/up) or phase B (down + combine) of a token,
// in the order A0, A1, B0, A2, B1, ..., A(n-1), B(n-2), B(n-1). Phase A of
// the next token runs while the grid barrier of the current one settles.
__device__ __forceinline__ void step_of(int j, int n, int &tok, bool &isA) {
    if (j == 0) { tok = 0; isA = true; }
    else if ((j & 1) && ((j + 1) >> 1) < n) { tok = (j + 1) >> 1; isA = true; }
    else if (j & 1) { tok = n - 1; isA = false; }
    else { tok = (j >> 1) - 1; isA = false; }
}

// Grid barriers: token number gt (counted since the host last reset the
// words; a launch's token t is gt = bar_base + t) uses the 64-bit arrival
// word gt % NBUF at bar + 4, which every CTA increments once per token, so
// barrier gt is complete at (gt / NBUF + 1) * gridDim.x arrivals. A CTA
// arrives for token gt + 1 before it waits for gt (phase A of the next
// token runs first), but it cannot arrive for gt + NBUF before every CTA
// has passed barrier gt + 2 and so arrived for gt: one word per token in
// flight keeps the counts exact.
__device__ __forceinline__ unsigned long long *barrier_word(uint32_t *bar, uint64_t gt) {
    return reinterpret_cast<unsigned long long *>(bar + 4) + (gt % NBUF);
}

// Consumer state carried from step to step.
enum : uint32_t { ST_ABORT = 1u, ST_DEAD = 2u };   // results invalid / stop waiting on copies

__device__ __forceinline__ uint64_t *trace_row(const FusedArgs &a) {
    return a.trace ? a.trace + (size_t)blockIdx.x * FUSED_TRACE_POINTS : nullptr;
}

// Phase A of token `tok`: x -> Q8_K, then gate/up + SwiGLU over this CTA's
// (rank, row) pairs (chunks cc0 .. cc0 + nA - 1 of the ring), h rows to
// hbuf[tok % NBUF], and this CTA's arrival at the token's grid barrier.
// Work item = four consecutive (gate, up) row pairs of a chunk; items go
// round-robin to the warps. Lane (g, lb) = (lane / 8, lane % 8) owns row
// pair g of the item and blocks lb, lb + 8, ... of both rows (exact int32
// block partials over the four quarters); lane 8g runs the gate chain and
// lane 8g + 1 the up chain over the blocks in ascending order, gathering
// the partials by shuffles. NB8 = blocks per lane (D <= 2048: 1, <= 4096: 2).
template <int DGU, int NB8>
__device__ __forceinline__ uint32_t consumer_a(const FusedArgs &a, uint8_t *smem, int nslot, int tok, uint32_t cc0,
                                               int nA, uint32_t *bar, uint32_t *err, uint32_t st) {
    const int D = a.D, de = a.de, k = a.k;
    const SmemLayout L = smem_layout(D, de, k, nslot);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.full);
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L.empty);
    uint8_t *xc = smem + L.xc;
    float *xd = reinterpret_cast<float *>(smem + L.xd);
    int16_t *xbs = reinterpret_cast<int16_t *>(smem + L.xbs);
    const ChunkDesc *desc = reinterpret_cast<const ChunkDesc *>(smem + L.desc);
    uint64_t *tr = trace_row(a);
    const bool tr0 = tr && tok == 0;
    const int nbx = D / 256, rbg = nbx * dt_block_bytes(DGU);
    float *hb = a.hbuf + (size_t)(tok % NBUF) * k * de;

    // x of this token (bulk-copied by the producer) -> Q8_K codes
    if (!(st & ST_DEAD) && !mbar_wait(reinterpret_cast<uint64_t *>(smem + L.xfull), (uint32_t)tok & 1u)) {
        st |= ST_DEAD | ST_ABORT;
        if (lane == 0) raise_error(err, bar, FUSED_ERR_COPY);
    }
    if (warp < nbx) {
        const float4 *x4 = reinterpret_cast<const float4 *>(smem + L.xs) + 64 * warp + 2 * lane;
        warp_quant_swz(x4[0], x4[1], xc, nbx, warp, xbs + 16 * warp, xd + warp, lane);
    }
    consumer_sync();
    if (t == 0) mbar_arrive(reinterpret_cast<uint64_t *>(smem + L.xempty));

    const int g = lane >> 3, lb = lane & 7;
    uint32_t tw = 0, t_in = tr ? (uint32_t)now_ns() : 0u;   // trace: ns waiting for chunks
    int base = 0;   // first item of chunk c
    for (int c = 0; c < nA; c++) {
        const uint32_t cc = cc0 + (uint32_t)c, s = cc % (uint32_t)nslot;
        const uint32_t tw0 = tr ? (uint32_t)now_ns() : 0u;
        if (!(st & ST_DEAD) && !mbar_wait(&full[s], (cc / (uint32_t)nslot) & 1u)) {
            st |= ST_DEAD | ST_ABORT;
            if (lane == 0) raise_error(err, bar, FUSED_ERR_COPY);
        }
        if (tr) tw += (uint32_t)now_ns() - tw0;
        const ChunkDesc d = desc[c];
        const int nit = (d.nrows + 3) >> 2;
        const uint8_t *stg = smem + L.stage + (size_t)s * SLOT_BYTES;
        if (!(st & ST_ABORT))
            for (int it = base + (warp - base % NCW + NCW) % NCW; it < base + nit; it += NCW) {
                const int row = 4 * (it - base) + g;
                const bool valid = row < d.nrows;
                const uint8_t *grow = stg + d.dst[0] + d.roff[0] + (size_t)row * rbg;
                const uint8_t *urow = stg + d.dst[1] + d.roff[1] + (size_t)row * rbg;
                BlockSum vg[NB8], vu[NB8];
#pragma unroll
                for (int i = 0; i < NB8; i++) {
                    const int b = lb + 8 * i;
                    vg[i] = BlockSum{ 0, 0, 0.f, 0.f };
                    vu[i] = vg[i];
                    if (valid && b < nbx)
                        block_dot2<DGU>(grow + b * dt_block_bytes(DGU), urow + b * dt_block_bytes(DGU), xc, nbx, b,
                                        xbs + 16 * b, xd[b], vg[i], vu[i]);
                }
                float ag = 0.0f, au = 0.0f;
#pragma unroll
                for (int i = 0; i < NB8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (8 * i + j < nbx) {
                            ag = chain_from<DGU>(ag, vg[i], (lane & ~7) | j);
                            au = chain_from<DGU>(au, vu[i], (lane & ~7) | j);
                        }
                if (lb == 0 && valid) hb[(size_t)d.rank * de + d.row0 + row] = __fmul_rn(silu_f(ag), au);
            }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        base += nit;
    }
    if (tr && lane == 0) {
        atomicAdd(reinterpret_cast<unsigned long long *>(&tr[8]), (unsigned long long)tw);
        atomicAdd(reinterpret_cast<unsigned long long *>(&tr[9]), (unsigned long long)((uint32_t)now_ns() - t_in));
    }
    // arrive at the token's grid barrier once every warp's h rows are written
    consumer_sync();
    if (t == 0) {
        if (tr0) tr[2] = now_ns();
        __threadfence();
        atomicAdd(barrier_word(bar, a.bar_base + (uint64_t)tok), 1ull);
    }
    return st;
}

// Phase B of token `tok`: wait for the token's grid barrier, re-quantise h
// (k x de, swizzled) into shared memory, then down rows + the rank-ordered
// combine over chunks cc0 .. cc0 + nB - 1. Work item = one output row of a
// chunk; items go round-robin to the warps. Lane u (+32) owns unit
// u = r * nbd + b (expert rank r, block b): the exact block partials over
// the four quarters; lane r runs expert r's chain over its blocks in
// ascending order, and lane 0 combines ffn = sum_r w[r] * eo_r in
// ascending rank. NS = unit slots per lane (k * nbd <= 32 * NS).
template <int DDN, int NS>
__device__ __forceinline__ uint32_t consumer_b(const FusedArgs &a, uint8_t *smem, int nslot, int tok, uint32_t cc0,
                                               int nA, int nB, uint32_t *bar, uint32_t *err, uint32_t st) {
    const int D = a.D, de = a.de, k = a.k;
    const SmemLayout L = smem_layout(D, de, k, nslot);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.full);
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L.empty);
    uint8_t *hc = smem + L.hc;
    float *hd = reinterpret_cast<float *>(smem + L.hd);
    int16_t *hbs = reinterpret_cast<int16_t *>(smem + L.hbs);
    const ChunkDesc *desc = reinterpret_cast<const ChunkDesc *>(smem + L.desc) + nA;
    int *misc = reinterpret_cast<int *>(smem + L.misc);
    uint64_t *tr = trace_row(a);
    const bool tr0 = tr && tok == 0;
    const int nbd = de / 256, rbd = nbd * dt_block_bytes(DDN), nbh = k * nbd;
    const float *hb = a.hbuf + (size_t)(tok % NBUF) * k * de;

    // grid barrier of this token: every CTA has written its h rows
    if (t == 0) {
        const uint64_t gt = a.bar_base + (uint64_t)tok;
        const unsigned long long *arrivals = barrier_word(bar, gt);
        const uint64_t target = (gt / NBUF + 1u) * gridDim.x;
        if (ld_acquire64(arrivals) < target) {
            const uint64_t t0 = now_ns();
            while (ld_acquire64(arrivals) < target) {
                if (now_ns() - t0 > BARRIER_NS) {
                    raise_error(err, bar, FUSED_ERR_BARRIER);
                    misc[2] = 1;
                    break;
                }
            }
        }
        __threadfence();
        if (tr0) tr[5] = now_ns();
    }
    consumer_sync();
    if (misc[2]) st |= ST_ABORT;

    // re-quantise h for all k experts (each CTA holds the full set); two
    // blocks per warp have their loads in flight together
    if (!(st & ST_ABORT)) {
        for (int b0 = warp; b0 < nbh; b0 += 2 * NCW) {
            float4 hv[2][2];
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int beta = b0 + j * NCW;
                if (beta < nbh) {
                    const float4 *h4 = reinterpret_cast<const float4 *>(hb + (size_t)(beta / nbd) * de +
                                                                        (size_t)(beta % nbd) * 256 + 8 * lane);
                    hv[j][0] = __ldcg(h4);
                    hv[j][1] = __ldcg(h4 + 1);
                }
            }
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int beta = b0 + j * NCW;
                if (beta < nbh) warp_quant_swz(hv[j][0], hv[j][1], hc, nbh, beta, hbs + 16 * beta, hd + beta, lane);
            }
        }
    }
    consumer_sync();
    if (tr0 && t == 0) tr[6] = now_ns();

    const float *wr = reinterpret_cast<const float *>(smem + L.w) + 64 * (tok % NBUF);
    uint32_t tw = 0, t_in = tr ? (uint32_t)now_ns() : 0u;
    int base = 0;
    for (int c = 0; c < nB; c++) {
        const uint32_t cc = cc0 + (uint32_t)c, s = cc % (uint32_t)nslot;
        const uint32_t tw0 = tr ? (uint32_t)now_ns() : 0u;
        if (!(st & ST_DEAD) && !mbar_wait(&full[s], (cc / (uint32_t)nslot) & 1u)) {
            st |= ST_DEAD | ST_ABORT;
            if (lane == 0) raise_error(err, bar, FUSED_ERR_COPY);
        }
        if (tr) tw += (uint32_t)now_ns() - tw0;
        const ChunkDesc d = desc[c];
        const int nit = d.nrows;
        const uint8_t *stg = smem + L.stage + (size_t)s * SLOT_BYTES;
        if (!(st & ST_ABORT))
            for (int it = base + (warp - base % NCW + NCW) % NCW; it < base + nit; it += NCW) {
                const int row = it - base;
                BlockSum v[NS];
#pragma unroll
                for (int i = 0; i < NS; i++) {
                    const int u = lane + 32 * i;
                    v[i] = BlockSum{ 0, 0, 0.f, 0.f };
                    if (u < nbh) {
                        const int r = u / nbd, b = u - r * nbd;
                        block_dot<DDN>(stg + (size_t)r * d.dst[0] + d.roff[0] + (size_t)row * rbd +
                                           b * dt_block_bytes(DDN),
                                       hc, nbh, u, hbs + 16 * u, hd[u], v[i]);
                    }
                }
                // expert lane's chain over its blocks (unit lane * nbd + b)
                float eo = 0.0f;
                for (int b = 0; b < nbd; b++) {
                    const int su = (lane < k ? lane : 0) * nbd + b;
                    if constexpr (NS == 1) {
                        eo = chain_from<DDN>(eo, v[0], su & 31);
                    } else {
                        const float e0 = chain_from<DDN>(eo, v[0], su & 31);
                        const float e1 = chain_from<DDN>(eo, v[1], su & 31);
                        eo = (su >> 5) ? e1 : e0;
                    }
                }
                float f = 0.0f;
                for (int r = 0; r < k; r++) f = __fadd_rn(f, __fmul_rn(wr[r], __shfl_sync(0xFFFFFFFFu, eo, r)));
                if (lane == 0) {
                    const int i = (int)d.row0 + row;
                    if (a.s_out) f = __fadd_rn(f, __fmul_rn(*a.sgate, a.s_out[i]));
                    a.ffn[(size_t)tok * D + i] = f;
                    if (a.h) a.h[i] = __fadd_rn(a.h[i], f);
                }
            }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        base += nit;
    }
    if (tr && lane == 0) {
        atomicAdd(reinterpret_cast<unsigned long long *>(&tr[10]), (unsigned long long)tw);
        atomicAdd(reinterpret_cast<unsigned long long *>(&tr[11]), (unsigned long long)((uint32_t)now_ns() - t_in));
    }
    consumer_sync();   // the token's routing is no longer read
    if (t == 0) {
        mbar_arrive(reinterpret_cast<uint64_t *>(smem + L.idsfree) + (tok % NBUF));
        if (tr0) tr[7] = now_ns();
    }
    return st;
}

// ---------------------------------------------------------------------------
// W: blocks per lane in phase A (D / 256 <= 8 W) and unit slots per lane in
// phase B (k * de / 256 <= 32 W).
template <int DGU, int DDN, int W>
__global__ void __launch_bounds__(NTHREADS, 1)
k_fused_ffn(const __grid_constant__ FusedArgs a, uint32_t *__restrict__ bar, uint32_t *__restrict__ err, int nslot) {
    extern __shared__ __align__(128) uint8_t smem[];
    const SmemLayout L = smem_layout(a.D, a.de, a.k, nslot);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.full);
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L.empty);
    ChunkDesc *desc = reinterpret_cast<ChunkDesc *>(smem + L.desc);
    int *misc = reinterpret_cast<int *>(smem + L.misc);   // [2] barrier abort, [3] sticky error seen

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
    uint64_t *tr = trace_row(a);
    if (tr && t == 0) {
        tr[0] = now_ns();
        tr[8] = tr[9] = tr[10] = tr[11] = 0;
    }

    // ---- prologue: the plan (same for every token; nA phase A chunks, then
    // nB phase B chunks) and the barriers
    const int2 *plan_n = reinterpret_cast<const int2 *>(a.plan);
    const ChunkDesc *plan_d = reinterpret_cast<const ChunkDesc *>(plan_n + gridDim.x) + (size_t)blockIdx.x * MAXCH;
    const int2 cnt = plan_n[blockIdx.x];
    const int nA = cnt.x, nB = cnt.y;
    const bool plan_ok = nA >= 0 && nB >= 0 && nA + nB <= MAXCH;
    constexpr int DW = (int)(sizeof(ChunkDesc) / 8);
    if (plan_ok && t < (nA + nB) * DW) reinterpret_cast<uint2 *>(desc)[t] = reinterpret_cast<const uint2 *>(plan_d)[t];
    if (t == 0) {
        for (int s = 0; s < nslot; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        mbar_init(reinterpret_cast<uint64_t *>(smem + L.xfull), 1);
        mbar_init(reinterpret_cast<uint64_t *>(smem + L.xempty), 1);
        for (int b = 0; b < NBUF; b++) mbar_init(reinterpret_cast<uint64_t *>(smem + L.idsfree) + b, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        misc[2] = 0;
        misc[3] = ld_acquire(&bar[2]) != 0;   // an earlier launch failed: do nothing until reset
    }
    __syncthreads();
    if (misc[3] || !plan_ok) {
        if (t == 0) raise_error(err, bar, misc[3] ? FUSED_ERR_BARRIER : FUSED_ERR_PLAN);
        return;   // every CTA sees the same sticky word / plan before any barrier
    }
    const int n = a.n_tok, E = a.E, k = a.k;

    if (warp == NCW) {
        // ---- producer: route each token when its phase A comes up, then
        // stream x and the chunks of each step in the consumers' order
        uint32_t *rscratch = reinterpret_cast<uint32_t *>(smem + L.p);
        uint8_t *xs = smem + L.xs;
        uint64_t *xfull = reinterpret_cast<uint64_t *>(smem + L.xfull);
        uint64_t *xempty = reinterpret_cast<uint64_t *>(smem + L.xempty);
        uint64_t *idsfree = reinterpret_cast<uint64_t *>(smem + L.idsfree);
        Slot *sl2 = reinterpret_cast<Slot *>(smem + L.sl);   // [2][MAXK] by token parity
        uint32_t cc = 0;
        int failed = 0;
        for (int j = 0; j < 2 * n && !failed; j++) {
            int tok;
            bool isA;
            step_of(j, n, tok, isA);
            const int b = tok % NBUF;
            Slot *sl = sl2 + MAXK * (tok & 1);
            if (isA) {
                if (tok >= NBUF && !mbar_wait(&idsfree[b], (uint32_t)(tok / NBUF - 1) & 1u)) failed = 1;
                if (!failed) {
                    const int layer = (a.layer0 + tok) % a.n_layers;
                    int32_t *ids = reinterpret_cast<int32_t *>(smem + L.ids) + 64 * b;
                    float *wr = reinterpret_cast<float *>(smem + L.w) + 64 * b;
                    warp_route(a.router, a.logits + (size_t)tok * E,
                               a.mask_all ? a.mask_all + (size_t)layer * E : nullptr,
                               a.bias_all ? a.bias_all + (size_t)layer * E : nullptr, E, k, a.routed_scale, rscratch,
                               ids, wr, lane);
                    if (tr && tok == 0 && lane == 0) tr[1] = now_ns();
                    if (blockIdx.x == 0 && lane < k) {
                        if (a.ids_out) a.ids_out[(size_t)tok * k + lane] = ids[lane];
                        if (a.w_out) a.w_out[(size_t)tok * k + lane] = wr[lane];
                    }
                    if (lane < k) sl[lane] = a.slots_all[(size_t)layer * E + ids[lane]];
                    __syncwarp();
                }
            }
            if (lane == 0 && !failed) {
                if (isA) {
                    if (tok >= 1 && !mbar_wait(xempty, (uint32_t)(tok - 1) & 1u)) failed = 1;
                    if (!failed) {
                        mbar_expect_tx(xfull, 4u * (uint32_t)a.D);
                        bulk_g2s(xs, a.x + (size_t)tok * a.D, 4u * (uint32_t)a.D, xfull);
                    }
                }
                const int n_c = isA ? nA : nB;
                const ChunkDesc *dd = isA ? desc : desc + nA;
                for (int c = 0; c < n_c && !failed; c++, cc++) {
                    const uint32_t s = cc % (uint32_t)nslot, u = cc / (uint32_t)nslot;
                    if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1u)) {
                        failed = 1;
                        break;
                    }
                    const ChunkDesc &d = dd[c];
                    uint8_t *stg = smem + L.stage + (size_t)s * SLOT_BYTES;
                    mbar_expect_tx(&full[s], d.tx);
                    if (isA) {
                        bulk_g2s(stg + d.dst[0], sl[d.rank].m[0] + d.lo[0], d.size[0], &full[s]);
                        bulk_g2s(stg + d.dst[1], sl[d.rank].m[1] + d.lo[1], d.size[1], &full[s]);
                    } else {
                        for (int r = 0; r < k; r++)
                            bulk_g2s(stg + (size_t)r * d.dst[0], sl[r].m[2] + d.lo[0], d.size[0], &full[s]);
                    }
                }
                if (failed) raise_error(err, bar, FUSED_ERR_COPY);
            }
            failed = __shfl_sync(0xFFFFFFFFu, failed, 0);   // consumers time out on what is missing
        }
        return;
    }

    // ---- consumers: the same schedule, A0, then (A(t+1), B(t)) pairs, then
    // B(n-1)
    uint32_t st = consumer_a<DGU, W>(a, smem, nslot, 0, 0u, nA, bar, err, 0u);
    uint32_t cc = (uint32_t)nA;
    for (int tok = 0; tok + 1 < n; tok++) {
        st = consumer_a<DGU, W>(a, smem, nslot, tok + 1, cc, nA, bar, err, st);
        cc += (uint32_t)nA;
        st = consumer_b<DDN, W>(a, smem, nslot, tok, cc, nA, nB, bar, err, st);
        cc += (uint32_t)nB;
    }
    consumer_b<DDN, W>(a, smem, nslot, n - 1, cc, nA, nB, bar, err, st);
    if (tr && t == 0) tr[12] = now_ns();
}

// ---------------------------------------------------------------------------
// host side
using KernelFn = void (*)(const FusedArgs, uint32_t *, uint32_t *, int);

// W = 1 when D <= 2048 and k * de / 256 <= 32, else 2 (D <= 4096, k * de / 256 <= 64).
static int pick_width(int D, int de, int k) {
    if (D <= 2048 && k * (de / 256) <= 32) return 1;
    if (D <= 4096 && k * (de / 256) <= 64) return 2;
    return 0;
}
static KernelFn pick_kernel(int dgu, int ddn, int D, int de, int k) {
    const int w = pick_width(D, de, k);
    if (!w) return nullptr;
#define TLMG_K(G, DN) \
    if (dgu == G && ddn == DN) return w == 1 ? k_fused_ffn<G, DN, 1> : k_fused_ffn<G, DN, 2>;
    TLMG_K(DT_Q4_K, DT_Q4_K) TLMG_K(DT_Q4_K, DT_Q5_K) TLMG_K(DT_Q4_K, DT_Q6_K)
    TLMG_K(DT_Q5_K, DT_Q4_K) TLMG_K(DT_Q5_K, DT_Q5_K) TLMG_K(DT_Q5_K, DT_Q6_K)
    TLMG_K(DT_Q6_K, DT_Q4_K) TLMG_K(DT_Q6_K, DT_Q5_K) TLMG_K(DT_Q6_K, DT_Q6_K)
#undef TLMG_K
    return nullptr;
}

int fused_init(FusedScratch &f, const tlmg_geom &g) {
    f.enabled = false;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return cuda_fail(cudaGetLastError(), "device properties");
    if (!prop.cooperativeLaunch) return TLMG_OK;
    if (g.n_experts <= 0 || g.n_experts > NTHREADS || g.n_experts > RT_PER * 32 || g.top_k > MAXK) return TLMG_OK;
    if (g.d_model % 256 || g.d_expert % 256 || g.d_model > 4096) return TLMG_OK;
    f.smem_limit = prop.sharedMemPerBlockOptin;
    int nslot = 0;
    for (int ns = 8; ns >= 2; ns--)
        if (smem_layout(g.d_model, g.d_expert, g.top_k, ns).total + 1024 <= f.smem_limit) {
            nslot = ns;
            break;
        }
    if (!nslot) return TLMG_OK;
    f.nslot = nslot;
    f.smem = smem_layout(g.d_model, g.d_expert, g.top_k, nslot).total;
    f.nsm = prop.multiProcessorCount;
    if (cudaMalloc(&f.bar, 64) != cudaSuccess) return set_error(TLMG_ENOMEM, "fused barrier allocation");
    cudaMemset(f.bar, 0, 64);
    f.rounds = 0;
    if (cudaHostAlloc(&f.err_host, 64, cudaHostAllocMapped) != cudaSuccess)
        return set_error(TLMG_ENOMEM, "fused error word allocation");
    *f.err_host = 0;
    cudaHostGetDevicePointer((void **)&f.err_dev, f.err_host, 0);
    f.enabled = true;
    return TLMG_OK;
}

void fused_release(FusedScratch &f) {
    if (f.bar) cudaFree(f.bar);
    if (f.err_host) cudaFreeHost(f.err_host);
    for (auto &kv : f.plans) cudaFree(kv.second);
    f = FusedScratch{};
}

// Split of the layer-token's work over the CTAs, in chunks that fit one
// stage: phase A = (rank, row) pairs [P*c/G, P*(c+1)/G), phase B = output
// rows [D*c/G, D*(c+1)/G).
const void *fused_plan(FusedScratch &f, const tlmg_geom &g, int dgu, int ddn) {
    if (!f.enabled || !pick_kernel(dgu, ddn, g.d_model, g.d_expert, g.top_k)) return nullptr;
    const FusedPlanKey key{ dgu, ddn };
    auto it = f.plans.find(key);
    if (it != f.plans.end()) return it->second;
    const int D = g.d_model, de = g.d_expert, k = g.top_k, G = f.nsm;
    const int rbg = D / 256 * dt_block_bytes(dgu), rbd = de / 256 * dt_block_bytes(ddn);
    if (2 * rbg + 96 > SLOT_BYTES || k * (rbd + 48) > SLOT_BYTES) return nullptr;
    if (k > 32) return nullptr;   // phase B: lane r runs expert r's chain
    if (g.n_experts > RT_PER * 32 || k > MAXK) return nullptr;
    std::vector<int2> counts(G);
    std::vector<ChunkDesc> descs((size_t)G * MAXCH);
    for (int c = 0; c < G; c++) {
        ChunkDesc *out = &descs[(size_t)c * MAXCH];
        int n = 0;
        const int64_t P = (int64_t)k * de, p0 = P * c / G, p1 = P * (c + 1) / G;
        // phase A chunks hold whole work items (4 row pairs) where a stage can
        const int fitA = (SLOT_BYTES - 96) / (2 * rbg), capA = fitA >= 4 ? fitA & ~3 : fitA;
        for (int64_t p = p0; p < p1;) {
            if (n == MAXCH) return nullptr;
            const int r = (int)(p / de), j = (int)(p % de);
            const int nr = (int)std::min<int64_t>(std::min<int64_t>(capA, p1 - p), de - j);
            ChunkDesc d{};
            d.phase = 0;
            d.rank = (uint8_t)r;
            d.nrows = (uint16_t)nr;
            d.row0 = (uint32_t)j;
            uint32_t off = 0;
            for (int m = 0; m < 2; m++) {
                const uint64_t start = (uint64_t)j * rbg, lo = start & ~15ull;
                const uint64_t hi = (start + (uint64_t)nr * rbg + 15) & ~15ull;
                d.lo[m] = (uint32_t)lo;
                d.size[m] = (uint32_t)(hi - lo);
                d.dst[m] = (uint16_t)off;
                d.roff[m] = (uint16_t)(start - lo);
                off = up16(off + d.size[m]);
            }
            if (off > (uint32_t)SLOT_BYTES) return nullptr;
            d.tx = d.size[0] + d.size[1];
            out[n++] = d;
            p += nr;
        }
        const int nA = n;
        const int i0 = (int)((int64_t)D * c / G), i1 = (int)((int64_t)D * (c + 1) / G);
        const int capB = (SLOT_BYTES - 48 * k) / (k * rbd);
        for (int i = i0; i < i1;) {
            if (n == MAXCH) return nullptr;
            const int nr = std::min(capB, i1 - i);
            ChunkDesc d{};
            d.phase = 1;
            d.nrows = (uint16_t)nr;
            d.row0 = (uint32_t)i;
            const uint64_t start = (uint64_t)i * rbd, lo = start & ~15ull;
            const uint64_t hi = (start + (uint64_t)nr * rbd + 15) & ~15ull;
            d.lo[0] = (uint32_t)lo;
            d.size[0] = (uint32_t)(hi - lo);
            d.dst[0] = (uint16_t)up16(d.size[0]);
            d.roff[0] = (uint16_t)(start - lo);
            if ((uint32_t)k * d.dst[0] > (uint32_t)SLOT_BYTES) return nullptr;
            d.tx = (uint32_t)k * d.size[0];
            out[n++] = d;
            i += nr;
        }
        counts[c] = make_int2(nA, n - nA);
    }
    KernelFn kf = pick_kernel(dgu, ddn, D, de, k);
    if (cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)f.smem) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kf, NTHREADS, f.smem) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        return nullptr;
    }
    const size_t bytes = sizeof(int2) * G + sizeof(ChunkDesc) * descs.size();
    void *dp = nullptr;
    if (cudaMalloc(&dp, bytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    cudaMemcpy(dp, counts.data(), sizeof(int2) * G, cudaMemcpyHostToDevice);
    cudaMemcpy((uint8_t *)dp + sizeof(int2) * G, descs.data(), sizeof(ChunkDesc) * descs.size(),
               cudaMemcpyHostToDevice);
    f.plans[key] = dp;
    return dp;
}

int launch_fused_ffn(FusedScratch &f, const FusedArgs &a, cudaStream_t st) {
    KernelFn kf = pick_kernel(a.dt_gu, a.dt_dn, a.D, a.de, a.k);
    if (!kf) return set_error(TLMG_EUNSUP, "fused kernel: no instance for dtypes %d/%d", a.dt_gu, a.dt_dn);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)f.nsm);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = f.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FusedArgs la = a;
    la.bar_base = f.rounds;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kf, la, f.bar, f.err_dev, f.nslot);
    count_launch();
    if (e != cudaSuccess) return cuda_fail(e, "fused expert FFN launch");
    f.rounds += (uint64_t)a.n_tok;   // every CTA arrives once per token
    return TLMG_OK;
}

uint32_t fused_take_error(FusedScratch &f) {
    if (!f.err_host) return 0;
    uint32_t e = *(volatile uint32_t *)f.err_host;
    if (e) {
        // the stream is idle (the caller synchronised): clear the sticky
        // device word and the barrier state for the next launch
        *(volatile uint32_t *)f.err_host = 0;
        cudaMemset(f.bar, 0, 64);
        f.rounds = 0;
    }
    return e;
}

}  // namespace tlmg
