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
#include "tlmg_kq.cuh"
#include "tlmg_internal.h"

namespace tlmg {

constexpr int NCW = 15;                 // consumer warps; warps NCW / NCW + 4 stream, NCW + 1 routes, NCW + 2 / NCW + 3 do duties
constexpr int NAW = 7;                  // consumer warps [0, NAW) process gate/up chunks (<= 176 units + the chains), the others down chunks
constexpr int NTHREADS = 32 * (NCW + 5);   // + gate/up stream, router, two duty warps, down stream (warp NCW + 4)
constexpr int MAXCH = FUSED_MAXCH;
constexpr int MAXK = 16;
// Stage sizes and counts (compile-time tuning; the defaults measured best):
// a gate/up stage holds the gate rows and the up rows of a chunk, half
// each (22 Q4_K rows of D = 2048); a down stage holds rows of one expert.
#ifndef TLMG_SLOT_A
#define TLMG_SLOT_A 50720
#endif
#ifndef TLMG_SLOT_B
#define TLMG_SLOT_B 24576
#endif
#ifndef TLMG_NS_A
#define TLMG_NS_A 2       // gate/up stages
#endif
#ifndef TLMG_NS_B_MAX
#define TLMG_NS_B_MAX 3   // down stages, as many as fit up to this
#endif
constexpr int SLOT_A = TLMG_SLOT_A;
constexpr int SLOT_B = TLMG_SLOT_B;
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
// Work split of one token over the CTAs, both phases per expert: expert
// rank r gets the CTAs [G r / k, G (r+1) / k), which split its rows evenly
// (qrange_lo). Phase A (gate/up): (rank, row) pairs p = r * de + j; phase B
// (down): (rank, output row) pairs q = r * D + i. A CTA's rows are then
// contiguous in one expert's matrices, so every CTA gets the same number
// of chunks (a range across an expert boundary would add a chunk, and the
// CTAs holding one set the pace of the token), and a CTA streams them
// in a few large bulk copies (copies of ~24 KB reach the HBM peak; small
// scattered ones do not).
__host__ __device__ inline int range_lo(int64_t n, int c, int G) { return (int)(n * c / G); }
// Pairs one CTA owns at most, for grids of >= 64 CTAs.
__host__ __device__ inline int range_max(int64_t n) { return (int)((n + 63) / 64 + 1); }
// Phase B split: expert rank r gets the CTAs [G r / k, G (r+1) / k) (G >= k),
// which split its D rows evenly; returns the first (rank, row) pair
// r * D + i of CTA c (c = G: k * D). Every CTA reads rows of one expert.
__host__ __device__ inline int qrange_lo(int c, int G, int k, int D) {
    if (c >= G) return k * D;
    int r = 0;
    while (r + 1 < k && (int)((int64_t)G * (r + 1) / k) <= c) r++;
    const int c0 = (int)((int64_t)G * r / k), c1 = (int)((int64_t)G * (r + 1) / k);
    return r * D + (int)((int64_t)D * (c - c0) / (c1 - c0));
}

// ---------------------------------------------------------------------------
// shared-memory layout: nsA gate/up stages of SLOT_A bytes, nsB down stages
// of SLOT_B bytes, then the small state
constexpr int NBUF = 8;   // routing / staging buffers, by token % NBUF (tokens in flight)
constexpr int NX = 3;     // quantised-x buffers, by token % NX
struct SmemLayout {
    uint32_t stageA, stageB, full, empty, seq, xs, xfull, xfree, xseq, hraw, hs, hfull, hfree, hseq, routed, idsfree,
        adone, bdone, ids, w, sl, rscr, partA, partB, desc, misc, total;
};
// Rows one gate/up stage (one down stage) holds at most, for rows of nb
// blocks of the smallest K-quant block (144 bytes).
__host__ __device__ inline int capA_rows(int nbx) { return (SLOT_A / 2 - 15) / (nbx * 144); }
__host__ __device__ inline int capB_rows(int nbd) { return (SLOT_B - 15) / (nbd * 144); }
__host__ __device__ inline SmemLayout smem_layout(int D, int de, int k, int nsA, int nsB) {
    SmemLayout L;
    uint32_t o = 0;
    const int nbx = D / 256, nbd = de / 256, ns = nsA + nsB;
    L.stageA = o; o += (uint32_t)nsA * SLOT_A;
    L.stageB = o; o += (uint32_t)nsB * SLOT_B;
    L.full = o; o += 8u * ns;
    L.empty = o; o += 8u * ns;
    L.seq = o; o += 4u * ns;
    L.xfull = o = (o + 7u) & ~7u; o += 8u * NX;
    L.xfree = o; o += 8u * NX;
    L.hfull = o; o += 16u;
    L.hfree = o; o += 16u;
    L.routed = o; o += 8u * NBUF;
    L.idsfree = o; o += 8u * NBUF;
    L.adone = o; o += 8u * NBUF;
    L.bdone = o; o += 8u * NBUF;
    L.xseq = o; o += 4u * NX;
    L.hseq = o; o += 8u;
    L.xs = o = up16(o); o += (uint32_t)NX * qv_bytes(nbx);
    L.hraw = o = up16(o); o += 2u * 4u * (uint32_t)de;        // [two experts][de] h rows of the down experts
    L.hs = o = up16(o); o += 2u * qv_bytes(nbd);              // [two experts] the same, quantised
    L.rscr = o = up16(o); o += 4u * (uint32_t)RT_SCRATCH;
    L.ids = o; o += 4u * MAXK * NBUF;
    L.w = o; o += 4u * MAXK * NBUF;
    L.sl = o = up16(o); o += (uint32_t)sizeof(Slot) * MAXK * NBUF;
    // partial sums of a chunk's units, double-buffered: gate/up [2][2 rows][nbx + 1] (block units),
    // down [2][rows][2 nbd + 1] (half-block units)
    L.partA = o = up16(o); o += 16u * 2u * 2u * (uint32_t)capA_rows(nbx) * (uint32_t)(nbx + 1);
    L.partB = o = up16(o); o += 16u * 2u * (uint32_t)capB_rows(nbd) * (uint32_t)(2 * nbd + 1);
    L.desc = o = up16(o); o += (uint32_t)sizeof(ChunkDesc) * MAXCH;
    L.misc = o = up16(o); o += 64;
    L.total = o;
    return L;
}

// Grid barriers: token number gt (counted since the host last reset the
// words; a launch's token t is gt = bar_base + t) uses the 64-bit arrival
// word gt % NBUF at bar + 8, which every CTA increments once per token when
// its gate/up rows of the token are written, so barrier gt is complete at
// (gt / NBUF + 1) * gridDim.x arrivals. A CTA arrives for token gt + NBUF
// only after its router released the routing buffer of token gt, i.e.
// after its down phase of token gt, which follows barrier gt: one word per
// token in flight keeps the counts exact. The word at bar + 4 counts the
// CTAs that quantised their share of the launch's inputs.
__device__ __forceinline__ unsigned long long *barrier_word(uint32_t *bar, uint64_t gt) {
    return reinterpret_cast<unsigned long long *>(bar + 8) + (gt % NBUF);
}
__device__ __forceinline__ unsigned long long *xbar_word(uint32_t *bar) {
    return reinterpret_cast<unsigned long long *>(bar + 4);
}
constexpr int BAR_BYTES = 32 + 8 * NBUF;   // [2] sticky error, xbar word, barrier words
// Wait until *w >= target, for at most BARRIER_NS; polls with a short sleep
// so that a waiting lane takes few issue slots from the warps computing.
__device__ __forceinline__ bool grid_wait(const unsigned long long *w, uint64_t target) {
    if (ld_acquire64(w) >= target) return true;
    const uint64_t t0 = now_ns();
    while (ld_acquire64(w) < target) {
        if (now_ns() - t0 > BARRIER_NS) return false;
        __nanosleep(128);
    }
    return true;
}
// Wait until the shared word *p equals v (the producer publishes which
// chunk / token a buffer holds before its mbarrier phase can complete), for
// at most WAIT_NS.
__device__ __forceinline__ bool seq_wait(const uint32_t *p, uint32_t v) {
    const volatile uint32_t *q = p;
    if (*q == v) return true;
    const uint64_t t0 = now_ns();
    while (*q != v) {
        if (now_ns() - t0 > WAIT_NS) return false;
        __nanosleep(64);
    }
    return true;
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Consumer state carried from item to item.
enum : uint32_t { ST_ABORT = 1u, ST_DEAD = 2u };   // results invalid / stop waiting

// The token whose phase boundaries the trace stamps: one in the middle of
// the launch (steady state).
__device__ __forceinline__ int trace_tok(const FusedArgs &a) { return a.n_tok / 2; }
__device__ __forceinline__ uint64_t *trace_row(const FusedArgs &a) {
    return a.trace ? a.trace + (size_t)blockIdx.x * FUSED_TRACE_POINTS : nullptr;
}

// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// The persistent kernel. One CTA per SM: warps 0..NCW-1 consume work items,
// warp NCW streams the tokens' x and gate/up chunks, warp NCW + 4 each
// token's down chunks and (once its grid barrier completes) its h rows,
// warp NCW + 1 routes, warps NCW + 2 / NCW + 3 do the per-token duties.
//
//   launch start  every CTA quantises its share of the launch's inputs x
//                 (n_tok x D / 256 blocks) into a.xq; one grid-wide count.
//   router        routes token t into buffer t % NBUF once the CTA is done
//                 with token t - NBUF.
//   chunks        gate/up warps [0, NAW) and down warps [NAW, NCW) process
//                 their kind of chunk in token order (the stage's sequence
//                 word names the chunk it is armed for): one (row, block)
//                 unit per thread into shared partials, a group barrier
//                 that releases the stage, then one thread per row runs the
//                 row's chains and stages the result (h row, expert output)
//                 in shared memory.
//   token A done  warp 0 writes the CTA's h rows of the token, adds them to
//                 the counts of the h blocks they belong to (the CTA
//                 completing a block quantises it into a.hq) and arrives at
//                 the token's grid barrier.
//   token B done  warp NAW writes the CTA's expert outputs, adds them to
//                 the counts of the 64-row groups they belong to (the CTA
//                 completing a group runs its rank-ordered combine) and
//                 frees the token's routing buffer.
//
// Every wait is bounded; on expiry the kernel raises an error bit the host
// reads and stops waiting (results of the launch are invalid).
template <int DGU, int DDN, int W>
__global__ void __launch_bounds__(NTHREADS, 1)
k_fused_ffn(const __grid_constant__ FusedArgs a, uint32_t *__restrict__ bar, uint32_t *__restrict__ err, int nsA,
            int nsB) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int D = a.D, de = a.de, k = a.k, E = a.E, n = a.n_tok;
    const int nbx = D / 256, nbd = de / 256;
    const SmemLayout L = smem_layout(D, de, k, nsA, nsB);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.full);
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L.empty);
    uint32_t *seq = reinterpret_cast<uint32_t *>(smem + L.seq);
    uint64_t *xfull = reinterpret_cast<uint64_t *>(smem + L.xfull);
    uint64_t *xfree = reinterpret_cast<uint64_t *>(smem + L.xfree);
    uint64_t *hfull = reinterpret_cast<uint64_t *>(smem + L.hfull);
    uint64_t *hfree = reinterpret_cast<uint64_t *>(smem + L.hfree);
    uint64_t *routed = reinterpret_cast<uint64_t *>(smem + L.routed);
    uint64_t *idsfree = reinterpret_cast<uint64_t *>(smem + L.idsfree);
    uint64_t *adone = reinterpret_cast<uint64_t *>(smem + L.adone);   // [NBUF] the CTA's gate/up results of a token staged
    uint64_t *bdone = reinterpret_cast<uint64_t *>(smem + L.bdone);   // [NBUF] the CTA's down results of a token staged
    uint32_t *xseq = reinterpret_cast<uint32_t *>(smem + L.xseq);   // [NX]: token in xs[i]
    uint32_t *hseq = reinterpret_cast<uint32_t *>(smem + L.hseq);   // [2]: token in hraw[i]
    ChunkDesc *desc = reinterpret_cast<ChunkDesc *>(smem + L.desc);
    Slot *slb = reinterpret_cast<Slot *>(smem + L.sl);     // [NBUF][MAXK] selected experts
    int *misc = reinterpret_cast<int *>(smem + L.misc);    // [3] sticky error seen
    const uint32_t qvx = qv_bytes(nbx), qvd = qv_bytes(nbd);
    const int64_t P = (int64_t)k * de, Q = (int64_t)k * D;
    const int q0 = qrange_lo(blockIdx.x, gridDim.x, k, D), q1 = qrange_lo(blockIdx.x + 1, gridDim.x, k, D);
    const int rq0 = q0 / D;   // first expert rank of the CTA's down rows

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
    uint64_t *tr = trace_row(a);
    if (tr && t == 0) {
        for (int i = 1; i < FUSED_TRACE_POINTS; i++) tr[i] = 0;
        tr[0] = now_ns();
    }

    // ---- prologue: the plan (same for every token: nA gate/up chunks, then
    // nB down chunks) and the barriers
    const int2 *plan_n = reinterpret_cast<const int2 *>(a.plan);
    const ChunkDesc *plan_d = reinterpret_cast<const ChunkDesc *>(plan_n + gridDim.x) + (size_t)blockIdx.x * MAXCH;
    const int2 cnt_pl = plan_n[blockIdx.x];
    const int nA = cnt_pl.x, nB = cnt_pl.y;
    const bool plan_ok = nA >= 0 && nB >= 0 && nA + nB <= MAXCH;
    constexpr int DW = (int)(sizeof(ChunkDesc) / 8);
    if (plan_ok && t < (nA + nB) * DW) reinterpret_cast<uint2 *>(desc)[t] = reinterpret_cast<const uint2 *>(plan_d)[t];
    const int ns = nsA + nsB;
    if (t < ns) seq[t] = 0xFFFFFFFFu;
    if (t < NX) xseq[t] = 0xFFFFFFFFu;
    if (t < 2) hseq[t] = 0xFFFFFFFFu;
    if (t == 0) {
        for (int s = 0; s < ns; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < NX; i++) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xfree[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&hfull[i], 1);
            mbar_init(&hfree[i], 1);
        }
        for (int b = 0; b < NBUF; b++) {
            mbar_init(&routed[b], 1);
            mbar_init(&idsfree[b], 1);
            mbar_init(&adone[b], 1);
            mbar_init(&bdone[b], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        misc[3] = ld_acquire(&bar[2]) != 0;   // an earlier launch failed: do nothing until reset
    }
    __syncthreads();
    if (misc[3] || !plan_ok) {
        if (t == 0) raise_error(err, bar, misc[3] ? FUSED_ERR_BARRIER : FUSED_ERR_PLAN);
        return;   // every CTA sees the same sticky word / plan before any barrier
    }

    if (warp == NCW + 1) {
        // ---- router
        uint32_t *rscratch = reinterpret_cast<uint32_t *>(smem + L.rscr);
        for (int tok = 0; tok < n; tok++) {
            const int b = tok % NBUF;
            if (tok >= NBUF && !mbar_wait(&idsfree[b], (uint32_t)(tok / NBUF - 1) & 1u)) {
                if (lane == 0) raise_error(err, bar, FUSED_ERR_COPY);
                break;   // the others time out on what is missing
            }
            const int layer = (a.layer0 + tok) % a.n_layers;
            int32_t *ids = reinterpret_cast<int32_t *>(smem + L.ids) + MAXK * b;
            float *wr = reinterpret_cast<float *>(smem + L.w) + MAXK * b;
            warp_route(a.router, a.logits + (size_t)tok * E, a.mask_all ? a.mask_all + (size_t)layer * E : nullptr,
                       a.bias_all ? a.bias_all + (size_t)layer * E : nullptr, E, k, a.routed_scale, rscratch, ids, wr,
                       lane);
            if (blockIdx.x == 0 && lane < k) {
                if (a.ids_out) a.ids_out[(size_t)tok * k + lane] = ids[lane];
                if (a.w_out) a.w_out[(size_t)tok * k + lane] = wr[lane];
            }
            if (lane < k) slb[MAXK * b + lane] = a.slots_all[(size_t)layer * E + ids[lane]];
            __syncwarp();
            if (lane == 0) {
                if (tr && tok == trace_tok(a)) tr[1] = now_ns();
                mbar_arrive(&routed[b]);
            }
        }
        return;
    }

    // ---- launch start: quantise this CTA's share of the inputs x (the
    // consumer warps), then count the CTA in
    if (warp < NCW) {
        for (int q = blockIdx.x * NCW + warp; q < n * nbx; q += gridDim.x * NCW) {
            const int tok = q / nbx, b = q - tok * nbx;
            const float4 *x4 = reinterpret_cast<const float4 *>(a.x + (size_t)tok * D + 256 * b) + 2 * lane;
            quant_block(__ldg(x4), __ldg(x4 + 1), qvec(a.xq + (size_t)tok * qvx, nbx), b, lane);
        }
        consumer_sync();
        if (t == 0) {
            __threadfence();
            atomicAdd(xbar_word(bar), 1ull);
        }
    }

    if (warp == NCW || warp == NCW + 4) {
        if (lane == 0) {
            // ---- streams, in token order, one warp each (a lane that sleeps
            // in a wait would stall a divergent lane of the same warp).
            // Warp NCW: each token's x and gate/up chunks once it is routed.
            // Warp NCW + 4: once the token is routed, the down chunks whose
            // stages earlier tokens held; once the token's grid barrier
            // completes, the raw h rows of the CTA's down experts, then the
            // token's remaining down chunks.
            const bool isA = warp == NCW;
            bool failed = isA && !grid_wait(xbar_word(bar), a.xbar_target);
            if (isA) fence_proxy_async();   // the quantised x was written by other CTAs' generic stores
            const int nc = isA ? nA : nB, nsr = isA ? nsA : nsB, s0 = isA ? 0 : nsA;
            const ChunkDesc *dd = isA ? desc : desc + nA;
            const int ne = (q1 - 1) / D - rq0 + 1;   // down experts of the CTA (1 or 2)
            for (int tok = 0; tok < n && !failed; tok++) {
                const int b = tok % NBUF;
                const Slot *sl = slb + MAXK * b;
                if (!mbar_wait(&routed[b], (uint32_t)(tok / NBUF) & 1u)) {
                    failed = true;
                    break;
                }
                if (isA) {
                    const int xb = tok % NX;
                    if (tok >= NX && !mbar_wait(&xfree[xb], (uint32_t)(tok / NX - 1) & 1u)) {
                        failed = true;
                        break;
                    }
                    mbar_expect_tx(&xfull[xb], qvx);
                    bulk_g2s(smem + L.xs + xb * qvx, a.xq + (size_t)tok * qvx, qvx, &xfull[xb]);
                    *reinterpret_cast<volatile uint32_t *>(&xseq[xb]) = (uint32_t)tok;
                    if (tr && tok == trace_tok(a)) tr[21] = now_ns();
                    if (tr && tok == trace_tok(a) + 1) tr[28] = now_ns();
                }
                // chunk c of this token into its stage (after the stage's
                // previous chunk, nsr chunks earlier, has been consumed)
                auto issue = [&](int c) -> bool {
                    const uint32_t cc = (uint32_t)(tok * nc + c), u = cc / (uint32_t)nsr;
                    const int s = s0 + (int)(cc % (uint32_t)nsr);
                    if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1u)) return false;
                    const ChunkDesc &d = dd[c];
                    uint8_t *stg = smem + (isA ? L.stageA + (size_t)s * SLOT_A : L.stageB + (size_t)(s - nsA) * SLOT_B);
                    mbar_expect_tx(&full[s], d.tx);
                    if (tr && tok == trace_tok(a) && (c == 0 || c == nc - 1))
                        tr[(isA ? 22 : 24) + (c == 0 ? 0 : 1)] = now_ns();
                    if (isA) {
                        bulk_g2s(stg + d.dst[0], sl[d.rank].m[0] + d.lo[0], d.size[0], &full[s]);
                        bulk_g2s(stg + d.dst[1], sl[d.rank].m[1] + d.lo[1], d.size[1], &full[s]);
                    } else {
                        bulk_g2s(stg, sl[d.rank].m[2] + d.lo[0], d.size[0], &full[s]);
                    }
                    *reinterpret_cast<volatile uint32_t *>(&seq[s]) = cc;
                    return true;
                };
                // Down: the chunks whose stages were held by earlier tokens
                // go out before the token's grid barrier (their weights
                // stream while the token's gate/up still runs); a chunk whose
                // stage's previous chunk belongs to this token needs this
                // token's h, so it waits until h has been issued.
                const int pre = isA ? nc : (nc < nsr ? nc : nsr);
                int c = 0;
                for (; c < pre && !failed; c++) failed = !issue(c);
                if (failed) break;
                if (!isA) {
                    const uint64_t gt = a.bar_base + (uint64_t)tok;
                    if ((tok >= 1 && !mbar_wait(&hfree[0], (uint32_t)(tok - 1) & 1u)) ||
                        !grid_wait(barrier_word(bar, gt), (gt / NBUF + 1u) * gridDim.x)) {
                        failed = true;
                        break;
                    }
                    fence_proxy_async();   // the h rows were written by other CTAs' generic stores
                    const uint32_t hb = (uint32_t)(ne * de) * 4u;   // h rows of the CTA's down experts
                    mbar_expect_tx(&hfull[0], hb);
                    bulk_g2s(smem + L.hraw, a.hbuf + (size_t)tok * P + (size_t)rq0 * de, hb, &hfull[0]);
                    *reinterpret_cast<volatile uint32_t *>(&hseq[0]) = (uint32_t)tok;
                    if (tr && tok == trace_tok(a)) tr[10] = now_ns();
                    if (tr && tok == trace_tok(a) + 1) tr[30] = now_ns();
                }
                for (; c < nc && !failed; c++) failed = !issue(c);
            }
            if (failed) raise_error(err, bar, isA ? FUSED_ERR_COPY : FUSED_ERR_BARRIER);
        }
        return;
    }

    if (warp == NCW + 2) {
        // ---- gate/up duties, token by token: once the gate/up group has
        // written all the CTA's h rows of the token (group barrier, then the
        // adone arrival), one gpu-scope fence makes them visible and the CTA
        // arrives at the token's grid barrier
        uint32_t td = 0;
        for (int tok = 0; tok < n; tok++) {
            if (!mbar_wait(&adone[tok % NBUF], (uint32_t)(tok / NBUF) & 1u)) {
                if (lane == 0) raise_error(err, bar, FUSED_ERR_BARRIER);
                break;
            }
            const uint32_t td0 = tr ? (uint32_t)now_ns() : 0u;
            if (lane == 0) {
                __threadfence();
                atomicAdd(barrier_word(bar, a.bar_base + (uint64_t)tok), 1ull);
                if (tr && tok == trace_tok(a)) tr[8] = now_ns();
                if (tr && tok == trace_tok(a) + 1) tr[29] = now_ns();
            }
            if (tr) td += (uint32_t)now_ns() - td0;
        }
        if (tr && lane == 0) atomicAdd(reinterpret_cast<unsigned long long *>(&tr[26]), (unsigned long long)td);
        return;
    }
    if (warp == NCW + 3) {
        // ---- down duties, token by token: once the down group has written
        // all the CTA's expert outputs of the token, one gpu-scope fence; the
        // counts of the 64-row output groups go out together (one lane per
        // group); the token's combine weights are copied and its routing
        // buffer freed; then the CTA completing a group combines its rows in
        // ascending rank
        uint32_t td = 0;
        // the CTA's output groups: rows [ia, ib) of expert rq0 (one expert)
        const int ia = q0 - rq0 * D, ib = q1 - rq0 * D;
        const int g0 = ia >> 6, ng = ((ib - 1) >> 6) - g0 + 1;   // <= 32 groups
        for (int tok = 0; tok < n; tok++) {
            if (!mbar_wait(&bdone[tok % NBUF], (uint32_t)(tok / NBUF) & 1u)) {
                if (lane == 0) raise_error(err, bar, FUSED_ERR_BARRIER);
                break;
            }
            const uint32_t td0 = tr ? (uint32_t)now_ns() : 0u;
            __threadfence();
            uint32_t complete = 0;
            if (lane < ng) {
                const int grp = g0 + lane;
                const int ga = ia > 64 * grp ? ia : 64 * grp, gz = ib < 64 * grp + 64 ? ib : 64 * grp + 64;
                uint32_t *gc = a.ocnt + (size_t)tok * (D / 64) + grp;
                const bool c = (int)atomicAdd(gc, (uint32_t)(gz - ga)) + (gz - ga) == 64 * k;
                if (c) *gc = 0u;   // ready for the next launch
                complete = c;
            }
            complete = __ballot_sync(0xFFFFFFFFu, complete != 0);
            const float *wr = reinterpret_cast<const float *>(smem + L.w) + MAXK * (tok % NBUF);
            float wk[MAXK];
#pragma unroll
            for (int q = 0; q < MAXK; q++) wk[q] = q < k ? wr[q] : 0.0f;
            __syncwarp();
            if (lane == 0) mbar_arrive(&idsfree[tok % NBUF]);
            if (complete) __threadfence();
            while (complete) {
                const int grp = g0 + __ffs(complete) - 1;
                complete &= complete - 1;
                // rows 64 grp + lane and + 32: every expert output loaded first
                // (independent L2 reads in flight together), then the
                // rank-ordered sums
                float e0[MAXK], e1[MAXK];
                const float *eb = a.eo + (size_t)tok * Q + 64 * grp + lane;
#pragma unroll
                for (int q = 0; q < MAXK; q++) {
                    e0[q] = q < k ? __ldcg(eb + (size_t)q * D) : 0.0f;
                    e1[q] = q < k ? __ldcg(eb + (size_t)q * D + 32) : 0.0f;
                }
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    const int i = 64 * grp + lane + 32 * hh;
                    float f = 0.0f;
#pragma unroll
                    for (int q = 0; q < MAXK; q++)
                        if (q < k) f = __fadd_rn(f, __fmul_rn(wk[q], hh ? e1[q] : e0[q]));
                    if (a.s_out) f = __fadd_rn(f, __fmul_rn(*a.sgate, a.s_out[i]));
                    a.ffn[(size_t)tok * D + i] = f;
                    if (a.h) a.h[i] = __fadd_rn(a.h[i], f);
                }
            }
            if (lane == 0) {
                if (tr && tok == trace_tok(a)) tr[15] = now_ns();
                if (tr && tok == trace_tok(a) + 1) tr[31] = now_ns();
            }
            if (tr) td += (uint32_t)now_ns() - td0;
        }
        if (tr && lane == 0) atomicAdd(reinterpret_cast<unsigned long long *>(&tr[27]), (unsigned long long)td);
        return;
    }

    // ---- consumers: warps [0, NAW) process the gate/up chunks, the others
    // the down chunks, each group chunk by chunk in token order. All
    // threads of the group split the chunk's (row, block) units, one unit
    // each, and write the units' exact partials to shared memory; after a
    // group barrier the stage is released and one thread per row (the
    // group's highest threads) runs the row's fmaf chain(s) over the blocks
    // in ascending order (the next
    // chunk's units go to the other partials buffer meanwhile). A stage is
    // thus held for one unit's work, not for a row's.
    const bool isA = warp < NAW;
    const int gth = isA ? NAW * 32 : (NCW - NAW) * 32, gt = isA ? t : t - NAW * 32;
    const int rbg = nbx * dt_block_bytes(DGU), rbd = nbd * dt_block_bytes(DDN);
    const int nc = isA ? nA : nB, nsr = isA ? nsA : nsB, s0 = isA ? 0 : nsA;
    const int nbu = isA ? nbx : 2 * nbd;         // units per row: blocks (gate/up), half blocks (down)
    const int pstr = nbu + 1;                    // partials row stride (padded: conflict-free chain reads)
    const int pcap = isA ? capA_rows(nbx) : capB_rows(nbd);
    BlockSum *part = reinterpret_cast<BlockSum *>(smem + (isA ? L.partA : L.partB));   // [2][(A: 2) pcap][pstr]
    const int pbuf = (isA ? 2 : 1) * pcap * pstr;
    auto gsync = [&]() {
        if (isA) asm volatile("bar.sync 2, %0;" ::"n"(NAW * 32) : "memory");
        else asm volatile("bar.sync 3, %0;" ::"n"((NCW - NAW) * 32) : "memory");
    };
    uint32_t st = 0;
    uint32_t tw = 0, tc = 0;   // trace (lane 0 of each warp): ns waiting for inputs / in units and chains
    int pb = 0;
    for (int tok = 0; tok < n; tok++) {
        const int xb = tok % NX;
        uint8_t *vbuf = smem + (isA ? L.xs + xb * qvx : L.hs);
        const bool trt = tr && tok == trace_tok(a) && gt == 0;
        if (!isA) {
            // the token's h rows of the CTA's down experts -> Q8_K in shared
            // memory (one block per warp of the group), then the raw buffer is free
            const uint32_t tw0 = tr ? (uint32_t)now_ns() : 0u;
            if (!(st & ST_DEAD) &&
                !(seq_wait(&hseq[0], (uint32_t)tok) && mbar_wait(&hfull[0], (uint32_t)tok & 1u))) {
                st |= ST_DEAD | ST_ABORT;
                raise_error(err, bar, FUSED_ERR_COPY);
            }
            if (tr) tw += (uint32_t)now_ns() - tw0;
            const int ne = (q1 - 1) / D - rq0 + 1;
            const float *hr = reinterpret_cast<const float *>(smem + L.hraw);
            for (int qb = warp - NAW; qb < ne * nbd && !(st & ST_ABORT); qb += NCW - NAW) {
                const int e = qb / nbd, b = qb - e * nbd;
                const float4 *h4 = reinterpret_cast<const float4 *>(hr + e * de + 256 * b) + 2 * lane;
                quant_block(h4[0], h4[1], qvec(smem + L.hs + e * qvd, nbd), b, lane);
            }
            gsync();
            if (gt == 0) mbar_arrive(&hfree[0]);
        }
        for (int c = 0; c < nc; c++) {
            const uint32_t cc = (uint32_t)(tok * nc + c);
            const int s = s0 + (int)(cc % (uint32_t)nsr);
            const ChunkDesc d = desc[(isA ? 0 : nA) + c];
            if (trt && c == 0) tr[isA ? 2 : 9] = now_ns();

            // inputs: the chunk, and (first gate/up chunk) the token's x
            const uint32_t tw0 = tr ? (uint32_t)now_ns() : 0u;
            if (!(st & ST_DEAD)) {
                bool ok = seq_wait(&seq[s], cc) && mbar_wait(&full[s], (cc / (uint32_t)nsr) & 1u);
                if (ok && c == 0 && isA)
                    ok = seq_wait(&xseq[xb], (uint32_t)tok) && mbar_wait(&xfull[xb], (uint32_t)(tok / NX) & 1u);
                if (!ok) {
                    st |= ST_DEAD | ST_ABORT;
                    raise_error(err, bar, FUSED_ERR_COPY);
                }
            }
            const uint32_t tc0 = tr ? (uint32_t)now_ns() : 0u;
            if (tr) tw += tc0 - tw0;
            if (trt && c == 0) tr[isA ? 3 : 11] = now_ns();

            // the chunk's units
            BlockSum *pp = part + pb * pbuf;
            const int units = d.nrows * nbu;
            if (!(st & ST_ABORT)) {
                if (isA) {
                    const uint8_t *stg = smem + L.stageA + (size_t)s * SLOT_A;
                    const QVec x = qvec(vbuf, nbx);
                    for (int u = gt; u < units; u += gth) {
                        const int row = u / nbx, b = u - row * nbx;
                        const uint8_t *wb[2] = { stg + d.dst[0] + d.roff[0] + (size_t)row * rbg + b * dt_block_bytes(DGU),
                                                 stg + d.dst[1] + d.roff[1] + (size_t)row * rbg + b * dt_block_bytes(DGU) };
                        BlockSum o2[2];
                        kblock_dot<DGU, 2>(wb, XBlk{ x.codes, nbx, b, x.bs + 16 * b, x.d[b] }, o2);
                        pp[row * pstr + b] = o2[0];
                        pp[(pcap + row) * pstr + b] = o2[1];
                    }
                } else {
                    const uint8_t *stg = smem + L.stageB + (size_t)(s - nsA) * SLOT_B;
                    const QVec h = qvec(vbuf + (d.rank - rq0) * qvd, nbd);
                    for (int u = gt; u < units; u += gth) {
                        const int row = u / nbu, ub = u - row * nbu, b = ub >> 1;
                        BlockSum o1;
                        kblock_half<DDN>(stg + d.roff[0] + (size_t)row * rbd + b * dt_block_bytes(DDN),
                                         XBlk{ h.codes, nbd, b, h.bs + 16 * b, h.d[b] }, ub & 1, o1);
                        pp[row * pstr + ub] = o1;
                    }
                }
            }
            gsync();   // the chunk's partials are written; the stage is no longer read
            if (gt == 0) {
                mbar_arrive(&empty[s]);
                if (c == nc - 1 && isA) mbar_arrive(&xfree[xb]);
            }

            // the rows' chains
            // the rows' chains run on the group's highest threads, which get
            // the fewest units of the next chunk (units fill threads from 0)
            if (!(st & ST_ABORT) && gth - 1 - gt < d.nrows) {
                const int row = gth - 1 - gt;
                if (isA) {
                    float ag = 0.0f, au = 0.0f;
                    for (int b = 0; b < nbx; b++) {
                        const BlockSum eg = pp[row * pstr + b], eu = pp[(pcap + row) * pstr + b];
                        ag = chain<DGU>(ag, eg.dA, eg.is, eg.dM, eg.ms);
                        au = chain<DGU>(au, eu.dA, eu.is, eu.dM, eu.ms);
                    }
                    a.hbuf[(size_t)tok * P + (size_t)d.rank * de + d.row0 + row] = __fmul_rn(silu_f(ag), au);
                } else {
                    float eo = 0.0f;
                    for (int b = 0; b < nbd; b++) {
                        const BlockSum e0 = pp[row * pstr + 2 * b], e1 = pp[row * pstr + 2 * b + 1];
                        eo = chain<DDN>(eo, e0.dA, e0.is + e1.is, e0.dM, e0.ms + e1.ms);
                    }
                    a.eo[(size_t)tok * Q + (size_t)d.rank * D + d.row0 + row] = eo;
                }
            }
            if (tr) tc += (uint32_t)now_ns() - tc0;
            pb ^= 1;
        }
        gsync();   // the token's staged rows are complete: hand them to the duty warp
        if (gt == 0) mbar_arrive(isA ? &adone[tok % NBUF] : &bdone[tok % NBUF]);
    }
    if (tr && lane == 0) {
        atomicAdd(reinterpret_cast<unsigned long long *>(&tr[isA ? 16 : 18]), (unsigned long long)tw);
        atomicAdd(reinterpret_cast<unsigned long long *>(&tr[isA ? 17 : 19]), (unsigned long long)tc);
    }
    if (tr && t == 0) tr[20] = now_ns();
}


// ---------------------------------------------------------------------------
// host side
using KernelFn = void (*)(const FusedArgs, uint32_t *, uint32_t *, int, int);

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
    if (g.n_experts <= 0 || g.n_experts > RT_PER * 32 || g.top_k > MAXK) return TLMG_OK;
    if (g.d_model % 256 || g.d_expert % 256 || g.d_model > 4096) return TLMG_OK;
    f.smem_limit = prop.sharedMemPerBlockOptin;
    // stage counts: TLMG_NS_A gate/up stages, as many down stages as fit (>= 2)
    int nsB = 0;
    for (int nb = TLMG_NS_B_MAX; nb >= 2; nb--)
        if (smem_layout(g.d_model, g.d_expert, g.top_k, TLMG_NS_A, nb).total + 1024 <= f.smem_limit) {
            nsB = nb;
            break;
        }
    if (!nsB) return TLMG_OK;
    f.nsA = TLMG_NS_A;
    f.nsB = nsB;
    f.smem = smem_layout(g.d_model, g.d_expert, g.top_k, TLMG_NS_A, nsB).total;
    f.nsm = prop.multiProcessorCount;
    f.D = g.d_model;
    f.de = g.d_expert;
    f.k = g.top_k;
    if (cudaMalloc(&f.bar, BAR_BYTES) != cudaSuccess) return set_error(TLMG_ENOMEM, "fused barrier allocation");
    cudaMemset(f.bar, 0, BAR_BYTES);
    if (cudaMalloc(&f.obar, 16) != cudaSuccess) return set_error(TLMG_ENOMEM, "single-token kernel grid words");
    cudaMemset(f.obar, 0, 16);
    f.rounds = 0;
    f.launches = 0;
    if (cudaHostAlloc(&f.err_host, 64, cudaHostAllocMapped) != cudaSuccess)
        return set_error(TLMG_ENOMEM, "fused error word allocation");
    *f.err_host = 0;
    cudaHostGetDevicePointer((void **)&f.err_dev, f.err_host, 0);
    f.enabled = true;
    return TLMG_OK;
}

static void free_tokens(FusedScratch &f) {
    for (void *p : { (void *)f.xq, (void *)f.hbuf, (void *)f.eo, (void *)f.ocnt })
        if (p) cudaFree(p);
    f.xq = nullptr;
    f.hbuf = nullptr;
    f.eo = nullptr;
    f.ocnt = nullptr;
    f.tok_cap = 0;
}

// Per-token scratch for launches of up to n_tok tokens (grows; the device
// is idle when it does, as cudaFree synchronises).
static int reserve_tokens(FusedScratch &f, int n_tok) {
    if (n_tok <= f.tok_cap) return TLMG_OK;
    free_tokens(f);
    const int cap = n_tok < 64 ? 64 : n_tok;
    const int nbx = f.D / 256;
    const size_t P = (size_t)f.k * f.de, Q = (size_t)f.k * f.D;
    if (cudaMalloc(&f.xq, (size_t)cap * qv_bytes(nbx)) != cudaSuccess ||
        cudaMalloc(&f.hbuf, (size_t)cap * P * 4) != cudaSuccess ||
        cudaMalloc(&f.eo, (size_t)cap * Q * 4) != cudaSuccess ||
        cudaMalloc(&f.ocnt, (size_t)cap * (f.D / 64) * 4) != cudaSuccess) {
        cudaGetLastError();
        free_tokens(f);
        return set_error(TLMG_ENOMEM, "fused per-token scratch for %d tokens", n_tok);
    }
    cudaMemset(f.ocnt, 0, (size_t)cap * (f.D / 64) * 4);
    f.tok_cap = cap;
    return TLMG_OK;
}

void fused_release(FusedScratch &f) {
    free_tokens(f);
    if (f.bar) cudaFree(f.bar);
    if (f.obar) cudaFree(f.obar);
    if (f.err_host) cudaFreeHost(f.err_host);
    for (auto &kv : f.plans) cudaFree(kv.second);
    f = FusedScratch{};
}

// Split of the layer-token's work over the CTAs (qrange_lo): phase A
// (rank, row) pairs, phase B (rank, output row) pairs, each cut per expert
// into balanced chunks of contiguous rows that fit one stage: a gate/up
// chunk is one copy of gate rows and one of the same up rows, a down chunk
// one copy of down rows.
const void *fused_plan(FusedScratch &f, const tlmg_geom &g, int dgu, int ddn) {
    if (!f.enabled || !pick_kernel(dgu, ddn, g.d_model, g.d_expert, g.top_k)) return nullptr;
    const FusedPlanKey key{ dgu, ddn };
    auto it = f.plans.find(key);
    if (it != f.plans.end()) return it->second;
    const int D = g.d_model, de = g.d_expert, k = g.top_k, G = f.nsm;
    const int rbg = D / 256 * dt_block_bytes(dgu), rbd = de / 256 * dt_block_bytes(ddn);
    const int capA = (SLOT_A / 2 - 15) / rbg, capB = (SLOT_B - 15) / rbd;   // <= capA_rows / capB_rows
    if (capA < 1 || capB < 1) return nullptr;
    if (de / 256 > 32) return nullptr;   // phase B: a row's blocks fit one warp
    if (G < 64) return nullptr;          // per-CTA ranges sized for >= 64 CTAs
    if (g.n_experts > RT_PER * 32 || k > MAXK) return nullptr;
    std::vector<int2> counts(G);
    std::vector<ChunkDesc> descs((size_t)G * MAXCH);
    for (int c = 0; c < G; c++) {
        ChunkDesc *out = &descs[(size_t)c * MAXCH];
        int n = 0;
        for (int ph = 0; ph < 2; ph++) {
            const int64_t len = ph == 0 ? de : D;
            const int64_t lo = qrange_lo(c, G, k, (int)len), hi = qrange_lo(c + 1, G, k, (int)len);
            const int cap = ph == 0 ? capA : capB, rbytes = ph == 0 ? rbg : rbd;
            for (int64_t p = lo; p < hi;) {
                const int r = (int)(p / len), j0 = (int)(p % len);
                const int seg = (int)std::min<int64_t>(hi - p, len - j0);   // rows of expert r
                const int nch = (seg + cap - 1) / cap, per = (seg + nch - 1) / nch;
                for (int j = j0; j < j0 + seg; j += per) {
                    if (n == MAXCH) return nullptr;
                    const int nr = std::min(per, j0 + seg - j);
                    ChunkDesc d{};
                    d.phase = (uint8_t)ph;
                    d.rank = (uint8_t)r;
                    d.nrows = (uint16_t)nr;
                    d.row0 = (uint32_t)j;
                    const uint64_t start = (uint64_t)j * rbytes, a0 = start & ~15ull;
                    const uint64_t a1 = (start + (uint64_t)nr * rbytes + 15) & ~15ull;
                    for (int m = 0; m < (ph == 0 ? 2 : 1); m++) {
                        d.lo[m] = (uint32_t)a0;
                        d.size[m] = (uint32_t)(a1 - a0);
                        d.dst[m] = (uint16_t)(m * (SLOT_A / 2));
                        d.roff[m] = (uint16_t)(start - a0);
                    }
                    if (d.size[0] > (uint32_t)(ph == 0 ? SLOT_A / 2 : SLOT_B)) return nullptr;
                    d.tx = ph == 0 ? 2 * d.size[0] : d.size[0];
                    out[n++] = d;
                }
                p += seg;
            }
            if (ph == 0) counts[c].x = n;
        }
        counts[c].y = n - counts[c].x;
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

// ---------------------------------------------------------------------------
// Single-token kernel (k_ffn_one): one token, one launch, latency first.
// Every CTA routes the token itself (the same warp_route as above), then
// one thread issues bulk copies of ALL of the CTA's weights at once: its
// share of the (rank, row) gate/up units (both matrices) and, for its
// output rows [i0, i1), the down rows of all k experts (~170 KB at the
// Qwen3-30B-A3B layer shape), while the warps quantise x into shared
// memory. Gate/up units write SiLU(g) * u to hbuf; one grid barrier (a
// self-resetting count + generation pair, so that a graph can replay the
// launch); each CTA then quantises the k h rows itself and computes its
// output rows for every expert, so the rank-ordered combine and h += ffn
// stay inside the CTA. Same operations, in the same order, as the
// multi-kernel path (k_ffn_gateup / k_quant_h / k_ffn_down): bit-identical.
namespace one {
constexpr int NT = 512;                 // 16 warps
constexpr int NW = NT / 32;
}

// Dot of one row held in shared memory against a Q8_K vector (shared or
// global), every lane returns it: the k_matvec_qs order.
template <int DT>
__device__ __forceinline__ float row_dot_s(const uint8_t *row, const uint8_t *act, int nb, BlockPart *part,
                                           int lane) {
    constexpr int BB = dt_block_bytes(DT), ABB = act_block_bytes(act_kind_for(DT));
    const int g = lane >> 3, j = lane & 7;
    float acc = 0.0f;
    for (int c0 = 0; c0 < nb; c0 += FCHUNK) {
        const int nc = min(FCHUNK, nb - c0);
        for (int p0 = 0; p0 < nc; p0 += 4) {
            const int p = p0 + g;
            const bool valid = p < nc;
            int is = 0, ms = 0;
            const uint8_t *blk = row + (size_t)(c0 + p) * BB;
            const uint8_t *ab = act + (size_t)(c0 + p) * ABB;
            if (valid) block_part<SLoad>(DT, blk, ab, j, is, ms);
            group8_sum(is, ms);
            if (valid && j == 0) {
                float dA, dM;
                block_scales<SLoad>(DT, blk, ab, dA, dM);
                part[p] = BlockPart{ is, ms, dA, dM };
            }
        }
        __syncwarp();
        if (lane == 0)
            for (int p = 0; p < nc; p++) acc = chain_step(DT, acc, part[p].dA, part[p].dM, part[p].is, part[p].ms);
        __syncwarp();
    }
    return __shfl_sync(0xFFFFFFFFu, acc, 0);
}

// The CTA's shared-memory plan, the same on host and device.
struct OneLayout {
    uint32_t gu, dn, xq, hq, hraw, eo, part, ids, w, sl, rs, bars, total;
};
__host__ __device__ inline uint32_t al16(uint32_t v) { return (v + 15u) & ~15u; }
// worst case over CTAs: U units of gate/up (at most U / de + 2 experts), R output rows
__host__ __device__ inline OneLayout one_layout(int D, int de, int k, int G, int BG, int BD) {
    OneLayout L{};
    const int64_t P = (int64_t)k * de;
    const uint32_t U = (uint32_t)((P + G - 1) / G), R = (uint32_t)((D + G - 1) / G);
    const uint32_t rbg = (uint32_t)(D / 256 * BG), rbd = (uint32_t)(de / 256 * BD);
    const uint32_t nr = U / (uint32_t)de + 2;
    uint32_t o = 0;
    L.gu = o; o += al16(2 * U * rbg + nr * 2 * 32);
    L.dn = o; o += al16((uint32_t)k * (R * rbd + 32));
    L.xq = o; o += al16((uint32_t)(D / 256) * 292);
    L.hq = o; o += al16((uint32_t)k * (de / 256) * 292);
    L.hraw = o; o += 256 * 4 * one::NW;
    L.eo = o; o += al16(R * (uint32_t)k * 4);
    L.part = o; o += al16((uint32_t)sizeof(BlockPart) * FCHUNK * one::NW);
    L.ids = o; o += 4 * MAXK;
    L.w = o; o += 4 * MAXK;
    L.sl = o; o += al16((uint32_t)sizeof(Slot) * MAXK);
    L.rs = o; o += 4 * RT_SCRATCH;
    L.bars = o = (o + 7u) & ~7u; o += 16;
    L.total = al16(o);
    return L;
}

// Grid barrier of one launch: count + generation (gb[0], gb[1]); the last
// CTA resets the count before it advances the generation. All CTAs are
// resident (cooperative launch). false: gave up after BARRIER_NS.
__device__ __forceinline__ bool one_grid_barrier(uint32_t *gb) {
    const uint32_t g0 = ld_acquire(gb + 1);
    __threadfence();
    if (atomicAdd(gb, 1u) == gridDim.x - 1) {
        atomicExch(gb, 0u);
        __threadfence();
        atomicAdd(gb + 1, 1u);
        return true;
    }
    if (ld_acquire(gb + 1) != g0) return true;
    const uint64_t t0 = now_ns();
    while (ld_acquire(gb + 1) == g0) {
        if (now_ns() - t0 > BARRIER_NS) return false;
        __nanosleep(64);
    }
    return true;
}

template <int DGU, int DDN>
__global__ void __launch_bounds__(one::NT, 1)
    k_ffn_one(const FusedArgs a, uint32_t *bar, uint32_t *err, uint32_t *gb) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int BG = dt_block_bytes(DGU), BD = dt_block_bytes(DDN);
    const int D = a.D, de = a.de, k = a.k, E = a.E, G = gridDim.x, c = blockIdx.x;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int nbx = D / 256, nbh = de / 256;
    const uint32_t rbg = (uint32_t)nbx * BG, rbd = (uint32_t)nbh * BD;
    const OneLayout L = one_layout(D, de, k, G, BG, BD);
    const int64_t P = (int64_t)k * de;
    const int u0 = range_lo(P, c, G), u1 = range_lo(P, c + 1, G);
    const int i0 = range_lo(D, c, G), i1 = range_lo(D, c + 1, G);
    uint8_t *gu_s = smem + L.gu, *dn_s = smem + L.dn, *xq_s = smem + L.xq, *hq_s = smem + L.hq;
    float *hraw = reinterpret_cast<float *>(smem + L.hraw) + 256 * warp;
    float *eo_s = reinterpret_cast<float *>(smem + L.eo);
    BlockPart *part = reinterpret_cast<BlockPart *>(smem + L.part) + FCHUNK * warp;
    int32_t *ids = reinterpret_cast<int32_t *>(smem + L.ids);
    float *wr = reinterpret_cast<float *>(smem + L.w);
    Slot *sl = reinterpret_cast<Slot *>(smem + L.sl);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);   // [0] gate/up in, [1] down in
    __shared__ int fail_s;
    const int layer = a.layer0 % a.n_layers;
    uint64_t *tr = trace_row(a);   // [0] start [1] routed [2] copies issued [3] x quantised [4] gate/up in
                                   // [5] gate/up done [6] barrier passed [7] h quantised [8] down in [9] done
    if (tr && t == 0) {
        for (int q = 1; q < FUSED_TRACE_POINTS; q++) tr[q] = 0;
        tr[0] = now_ns();
    }

    if (t == 0) {
        fail_s = ld_acquire(&bar[2]) != 0;   // an earlier launch failed: do nothing until reset
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        warp_route(a.router, a.logits, a.mask_all ? a.mask_all + (size_t)layer * E : nullptr,
                   a.bias_all ? a.bias_all + (size_t)layer * E : nullptr, E, k, a.routed_scale,
                   reinterpret_cast<uint32_t *>(smem + L.rs), ids, wr, lane);
        __syncwarp();
        if (lane < k) {
            sl[lane] = a.slots_all[(size_t)layer * E + ids[lane]];
            if (c == 0 && a.ids_out) a.ids_out[lane] = ids[lane];
            if (c == 0 && a.w_out) a.w_out[lane] = wr[lane];
        }
        if (tr && lane == 0) tr[1] = now_ns();
    }
    __syncthreads();
    if (fail_s) {
        if (t == 0) raise_error(err, bar, FUSED_ERR_BARRIER);
        return;   // every CTA reads the same sticky word before the grid barrier
    }
    // ---- every weight byte of the CTA in flight at once
    if (t == 0) {
        uint32_t off = 0, tx = 0;
        for (int pass = 0; pass < 2; pass++) {   // pass 0 counts the bytes, pass 1 issues
            if (pass == 1) mbar_expect_tx(&bars[0], tx);
            off = 0;
            for (int r = u0 / de; r * de < u1; r++) {
                const int ja = max(u0, r * de) - r * de, jb = min(u1, (r + 1) * de) - r * de;
                if (jb <= ja) continue;
                for (int m = 0; m < 2; m++) {
                    const uintptr_t src = reinterpret_cast<uintptr_t>(sl[r].m[m]) + (uintptr_t)ja * rbg;
                    const uintptr_t lo = src & ~(uintptr_t)15, hi = (src + (uintptr_t)(jb - ja) * rbg + 15) & ~(uintptr_t)15;
                    if (pass == 1) bulk_g2s(gu_s + off, reinterpret_cast<const void *>(lo), (uint32_t)(hi - lo), &bars[0]);
                    else tx += (uint32_t)(hi - lo);
                    off += (uint32_t)(hi - lo);
                }
            }
        }
        tx = 0;
        for (int pass = 0; pass < 2; pass++) {
            if (pass == 1) mbar_expect_tx(&bars[1], tx);
            off = 0;
            for (int r = 0; r < k && i1 > i0; r++) {
                const uintptr_t src = reinterpret_cast<uintptr_t>(sl[r].m[2]) + (uintptr_t)i0 * rbd;
                const uintptr_t lo = src & ~(uintptr_t)15, hi = (src + (uintptr_t)(i1 - i0) * rbd + 15) & ~(uintptr_t)15;
                if (pass == 1) bulk_g2s(dn_s + off, reinterpret_cast<const void *>(lo), (uint32_t)(hi - lo), &bars[1]);
                else tx += (uint32_t)(hi - lo);
                off += (uint32_t)(hi - lo);
            }
        }
        if (tr) tr[2] = now_ns();
    }
    // ---- x as Q8_K (k_quant_q8k's blocks)
    for (int b = warp; b < nbx; b += one::NW) warp_quant_q8k(a.x + 256 * b, 256, xq_s + 292 * b, lane);
    __syncthreads();
    if (tr && t == 0) tr[3] = now_ns();
    bool ok = mbar_wait(&bars[0], 0);
    if (tr && t == 0) tr[4] = now_ns();
    // ---- gate/up units: SiLU(gate . x) * (up . x) -> hbuf
    if (ok) {
        uint32_t base = 0;
        for (int r = u0 / de; r * de < u1; r++) {
            const int ja = max(u0, r * de) - r * de, jb = min(u1, (r + 1) * de) - r * de;
            if (jb <= ja) continue;
            uint32_t gofs[2];
            for (int m = 0; m < 2; m++) {
                const uintptr_t src = reinterpret_cast<uintptr_t>(sl[r].m[m]) + (uintptr_t)ja * rbg;
                const uintptr_t lo = src & ~(uintptr_t)15, hi = (src + (uintptr_t)(jb - ja) * rbg + 15) & ~(uintptr_t)15;
                gofs[m] = base + (uint32_t)(src - lo);
                base += (uint32_t)(hi - lo);
            }
            for (int j = ja + warp; j < jb; j += one::NW) {
                const float gv = row_dot_s<DGU>(gu_s + gofs[0] + (size_t)(j - ja) * rbg, xq_s, nbx, part, lane);
                const float uv = row_dot_s<DGU>(gu_s + gofs[1] + (size_t)(j - ja) * rbg, xq_s, nbx, part, lane);
                if (lane == 0) a.hbuf[(size_t)r * de + j] = __fmul_rn(silu_f(gv), uv);
            }
        }
    }
    __syncthreads();
    if (t == 0) {
        if (tr) tr[5] = now_ns();
        if (!ok) raise_error(err, bar, FUSED_ERR_COPY);
        if (!one_grid_barrier(gb)) {
            raise_error(err, bar, FUSED_ERR_BARRIER);
            ok = false;
        }
        fail_s = !ok;
        if (tr) tr[6] = now_ns();
    }
    __syncthreads();
    if (fail_s) {
        if (t == 0) mbar_wait(&bars[1], 0);   // no copy may land after the CTA exits
        return;
    }
    // ---- the k h rows as Q8_K (k_quant_h's blocks), read from L2
    for (int q = warp; q < k * nbh; q += one::NW) {
        const int r = q / nbh, b = q - r * nbh;
        const float *src = a.hbuf + (size_t)r * de + 256 * b;
        for (int e = lane; e < 256; e += 32) hraw[e] = __ldcg(src + e);
        __syncwarp();
        warp_quant_q8k(hraw, 256, hq_s + 292 * (size_t)q, lane);
        __syncwarp();
    }
    __syncthreads();
    if (tr && t == 0) tr[7] = now_ns();
    ok = mbar_wait(&bars[1], 0);
    if (tr && t == 0) tr[8] = now_ns();
    if (!ok) {
        if (t == 0) raise_error(err, bar, FUSED_ERR_COPY);
        return;
    }
    // ---- down rows: c_r = w_r * (down_r[i] . h_r), then the combine
    uint32_t dofs[MAXK];
    {
        uint32_t base = 0;
        for (int r = 0; r < k; r++) {
            const uintptr_t src = reinterpret_cast<uintptr_t>(sl[r].m[2]) + (uintptr_t)i0 * rbd;
            const uintptr_t lo = src & ~(uintptr_t)15, hi = (src + (uintptr_t)(i1 - i0) * rbd + 15) & ~(uintptr_t)15;
            dofs[r] = base + (uint32_t)(src - lo);
            base += (uint32_t)(hi - lo);
        }
    }
    const int nrow = i1 - i0;
    for (int q = warp; q < nrow * k; q += one::NW) {
        const int ii = q / k, r = q - ii * k;
        const float e = row_dot_s<DDN>(dn_s + dofs[r] + (size_t)ii * rbd, hq_s + 292 * (size_t)r * nbh, nbh, part, lane);
        if (lane == 0) eo_s[q] = __fmul_rn(wr[r], e);
    }
    __syncthreads();
    for (int ii = t; ii < nrow; ii += one::NT) {
        const int i = i0 + ii;
        float acc = 0.0f;
        for (int r = 0; r < k; r++) acc = __fadd_rn(acc, eo_s[ii * k + r]);
        if (a.s_out) acc = __fadd_rn(acc, __fmul_rn(*a.sgate, a.s_out[i]));
        a.ffn[i] = acc;
        if (a.h) a.h[i] = __fadd_rn(a.h[i], acc);
    }
    if (tr && t == 0) tr[9] = now_ns();
}

using OneFn = void (*)(const FusedArgs, uint32_t *, uint32_t *, uint32_t *);
static OneFn pick_one(int dgu, int ddn) {
#define TLMG_O(G, DN) \
    if (dgu == G && ddn == DN) return k_ffn_one<G, DN>;
    TLMG_O(DT_Q4_K, DT_Q4_K) TLMG_O(DT_Q4_K, DT_Q5_K) TLMG_O(DT_Q4_K, DT_Q6_K)
    TLMG_O(DT_Q5_K, DT_Q4_K) TLMG_O(DT_Q5_K, DT_Q5_K) TLMG_O(DT_Q5_K, DT_Q6_K)
    TLMG_O(DT_Q6_K, DT_Q4_K) TLMG_O(DT_Q6_K, DT_Q5_K) TLMG_O(DT_Q6_K, DT_Q6_K)
#undef TLMG_O
    return nullptr;
}

// 1: launched; 0: this launch is not the single-token kernel's (the caller
// uses another); < 0: error.
static int launch_one(FusedScratch &f, const FusedArgs &a, cudaStream_t st) {
    if (!f.single || a.n_tok != 1 || a.k > MAXK || !f.obar) return 0;
    OneFn fn = pick_one(a.dt_gu, a.dt_dn);
    if (!fn) return 0;
    const OneLayout L = one_layout(a.D, a.de, a.k, f.nsm, dt_block_bytes(a.dt_gu), dt_block_bytes(a.dt_dn));
    if ((size_t)L.total + 1024 > f.smem_limit) return 0;
    static thread_local std::vector<const void *> opted;   // instances opted in to the large shared memory
    if (std::find(opted.begin(), opted.end(), (const void *)fn) == opted.end()) {
        if (cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)f.smem_limit - 1024) !=
            cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        opted.push_back((const void *)fn);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)f.nsm);
    cfg.blockDim = dim3(one::NT);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int rc = reserve_tokens(f, 1);
    if (rc) return rc;
    FusedArgs la = a;
    la.hbuf = f.hbuf;
    cudaError_t e = cudaLaunchKernelEx(&cfg, fn, la, f.bar, f.err_dev, f.obar);
    count_launch();
    if (e != cudaSuccess) return cuda_fail(e, "single-token expert FFN launch");
    return 1;
}

int launch_fused_ffn(FusedScratch &f, const FusedArgs &a, cudaStream_t st) {
    {
        const int r1 = launch_one(f, a, st);
        if (r1 < 0) return r1;
        if (r1 == 1) return TLMG_OK;
    }
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
    int rc = reserve_tokens(f, a.n_tok);
    if (rc) return rc;
    if (f.graph_mode || f.bar_stale) {
        // the arrival words (not the sticky error words) back to zero
        cudaError_t me = cudaMemsetAsync(reinterpret_cast<uint8_t *>(f.bar) + 16, 0, BAR_BYTES - 16, st);
        if (me != cudaSuccess) return cuda_fail(me, "fused expert FFN barrier reset");
        f.rounds = 0;
        f.launches = 0;
        f.bar_stale = f.graph_mode;
    }
    FusedArgs la = a;
    la.xq = f.xq;
    la.hbuf = f.hbuf;
    la.eo = f.eo;
    la.ocnt = f.ocnt;
    la.bar_base = f.rounds;
    la.xbar_target = (f.launches + 1) * (uint64_t)f.nsm;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kf, la, f.bar, f.err_dev, f.nsA, f.nsB);
    count_launch();
    if (e != cudaSuccess) return cuda_fail(e, "fused expert FFN launch");
    f.rounds += (uint64_t)a.n_tok;   // every CTA arrives once per token
    f.launches++;                    // and once per launch after quantising its inputs
    return TLMG_OK;
}

uint32_t fused_take_error(FusedScratch &f) {
    if (!f.err_host) return 0;
    uint32_t e = *(volatile uint32_t *)f.err_host;
    if (e) {
        // the stream is idle (the caller synchronised): clear the sticky
        // device word and the barrier state for the next launch
        *(volatile uint32_t *)f.err_host = 0;
        cudaMemset(f.bar, 0, BAR_BYTES);
        if (f.obar) cudaMemset(f.obar, 0, 16);
        if (f.ocnt) cudaMemset(f.ocnt, 0, (size_t)f.tok_cap * (f.D / 64) * 4);
        f.rounds = 0;
        f.launches = 0;
    }
    return e;
}

}  // namespace tlmg
