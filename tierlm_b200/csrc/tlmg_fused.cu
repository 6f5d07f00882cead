// tlmg_fused.cu - persistent expert-FFN kernel for batch-1 decode (sm_100a).
//
// One launch = one token through one MoE layer's routed experts
// (reference run_batch() + combine, src/lib/tlm_model.c:900-938, :1029-1036,
// with route(), :798-839, folded in). One CTA per SM, 16 consumer warps and
// one producer warp:
//
//   prologue   warp 0 routes (softmax top-k, exact), warps 1.. quantise x
//              to Q8_K / Q8_0 in shared memory, then every CTA plans the
//              same deterministic split of the work:
//              phase A = (rank, row) pairs of gate/up, contiguous per CTA;
//              phase B = output rows of down, contiguous per CTA.
//   producer   streams each chunk of selected weight rows HBM -> a ring of
//              shared-memory stages with cp.async.bulk (TMA, no multicast),
//              phase A chunks first, then phase B chunks, so the down
//              weights are already on chip when h is ready.
//   phase A    each warp takes rows of a chunk: exact int32 block partials
//              (dp4a), the serial fmaf chain, SiLU(g)*u -> hbuf (global).
//   barrier    grid-wide arrival counter (bounded spin, error word on
//              timeout); the grid is launched cooperatively, so all CTAs are
//              co-resident.
//   phase B    every CTA re-quantises h for all k experts into shared memory
//              (identical in every CTA), then each warp takes output rows:
//              k experts x blocks of down, per-expert fmaf chain, combine
//              ffn = sum_r w[r] * eo_r in ascending rank order.
//
// Every wait (mbarrier, grid barrier) has an iteration limit; on expiry the
// kernel raises an error bit the host reads, waits (bounded) for its own
// copies in flight and returns.
#include <algorithm>
#include <cstdio>

#include "tlmg_dev.cuh"
#include "tlmg_fused.cuh"
#include "tlmg_internal.h"

namespace tlmg {

constexpr int NCW = 16;                 // consumer warps
constexpr int NTHREADS = 32 * (NCW + 1);
constexpr int MAXCH = 128;              // chunks per CTA
constexpr int MAXPIECE = 16;            // pieces per chunk (phase B: one per rank)
constexpr int MAXK = 16;
constexpr int SLOT_BYTES = 24576;
constexpr uint64_t WAIT_NS = 200000000ull;       // 0.2 s: an mbarrier wait gives up
constexpr uint64_t BARRIER_NS = 500000000ull;    // 0.5 s: the grid barrier gives up

struct ChunkDesc {
    uint8_t phase, rank, npiece, pad;
    uint16_t nrows, pad2;
    uint32_t row0;
    uint32_t tx;
};

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
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
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
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (now_ns() - t0 > WAIT_NS) return false;
    }
}
// Record error bits for the host (mapped pinned word) and make them sticky
// for later launches (device word bar[2]) until the host resets them.
__device__ __forceinline__ void raise_error(uint32_t *err, uint32_t *bar, uint32_t bits) {
    volatile uint32_t *e = err;
    *e = *e | bits;
    atomicOr(&bar[2], bits);
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
__device__ __forceinline__ void st_release(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int rb_of(int dt, int n) { return n / dt_block(dt) * dt_block_bytes(dt); }

// A full warp quantises one Q8_K / Q8_0 block of h read through L2 (other
// CTAs wrote it) into shared memory.
__device__ __forceinline__ void warp_quant_h(const float *src, int nvalid, int kind, uint8_t *dst, int lane) {
    if (kind == DT_Q8_K) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int e = lane * 8 + i;
            v[i] = e < nvalid ? __ldcg(src + e) : 0.0f;
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
    } else {
        float v[1] = { lane < nvalid ? __ldcg(src + lane) : 0.0f };
        int q[1];
        float d = act_block_codes<1, 32>(v, q);
        int base = (lane & 7) * 4;
        int q0 = __shfl_sync(0xFFFFFFFFu, q[0], base + 0), q1 = __shfl_sync(0xFFFFFFFFu, q[0], base + 1);
        int q2 = __shfl_sync(0xFFFFFFFFu, q[0], base + 2), q3 = __shfl_sync(0xFFFFFFFFu, q[0], base + 3);
        if (lane < 8)
            reinterpret_cast<uint32_t *>(dst + 4)[lane] =
                (q0 & 255) | ((q1 & 255) << 8) | ((q2 & 255) << 16) | ((uint32_t)(q3 & 255) << 24);
        if (lane == 0) *reinterpret_cast<float *>(dst) = d;
    }
}

// Row dot over a shared-memory row by one warp (result in lane 0).
__device__ __forceinline__ float smem_row_dot(int dt, const uint8_t *row, const uint8_t *act, int nb,
                                              BlockPart *part, int lane) {
    const int g = lane >> 3, j = lane & 7, bb = dt_block_bytes(dt), abb = act_block_bytes(act_kind_for(dt));
    float acc = 0.0f;
    for (int c0 = 0; c0 < nb; c0 += FCHUNK) {
        int nc = min(FCHUNK, nb - c0);
        for (int p0 = 0; p0 < nc; p0 += 4) {
            int p = p0 + g;
            bool valid = p < nc;
            int is = 0, ms = 0;
            const uint8_t *blk = row + (size_t)(c0 + p) * bb;
            const uint8_t *ab = act + (size_t)(c0 + p) * abb;
            if (valid) block_part<SLoad>(dt, blk, ab, j, is, ms);
            group8_sum(is, ms);
            if (valid && j == 0) {
                float dA, dM;
                block_scales<SLoad>(dt, blk, ab, dA, dM);
                part[p] = BlockPart{ is, ms, dA, dM };
            }
        }
        __syncwarp();
        if (lane == 0)
            for (int p = 0; p < nc; p++) acc = chain_step(dt, acc, part[p].dA, part[p].dM, part[p].is, part[p].ms);
        __syncwarp();
    }
    return acc;
}

struct SmemLayout {
    uint32_t stage, full, empty, xq8k, xq80, hq, p_sm, ids, w, part, desc, poff, misc, total;
};

__host__ __device__ inline uint32_t up16(uint32_t v) { return (v + 15u) & ~15u; }

__host__ __device__ inline SmemLayout smem_layout(int D, int de, int k, int nslot) {
    SmemLayout L;
    uint32_t o = 0;
    L.stage = o; o += (uint32_t)nslot * SLOT_BYTES;
    L.full = o; o += 8u * nslot;
    L.empty = o; o += 8u * nslot;
    L.xq8k = o = up16(o); o += (uint32_t)(D / 256) * 292u;
    L.xq80 = o = up16(o); o += (uint32_t)(D / 32) * 36u;
    uint32_t hs = up16((uint32_t)std::max((de + 255) / 256 * 292, (de + 31) / 32 * 36));
    L.hq = o = up16(o); o += (uint32_t)k * hs;
    L.p_sm = o = up16(o); o += 4u * RT_PER * 32;
    L.ids = o; o += 4u * 64;
    L.w = o; o += 4u * 64;
    L.part = o = up16(o); o += (uint32_t)sizeof(BlockPart) * FCHUNK * NCW;
    L.desc = o = up16(o); o += (uint32_t)sizeof(ChunkDesc) * MAXCH;
    L.poff = o; o += 2u * MAXPIECE * MAXCH;
    L.misc = o = up16(o); o += 64;
    L.total = o;
    return L;
}

__host__ __device__ inline uint32_t hq_stride(int de) {
    return up16((uint32_t)std::max((de + 255) / 256 * 292, (de + 31) / 32 * 36));
}

// Plan this CTA's chunks (both phases) into shared memory. Run by one
// thread per phase. Returns the number of chunks written from `first`.
__device__ int plan_phase_a(const FusedArgs &a, const Slot *sl, ChunkDesc *desc, uint16_t *poff, int first) {
    const int64_t P = (int64_t)a.k * a.de;
    const int64_t p0 = P * blockIdx.x / gridDim.x, p1 = P * (blockIdx.x + 1) / gridDim.x;
    int n = first;
    for (int64_t p = p0; p < p1 && n < MAXCH;) {
        int r = (int)(p / a.de), j = (int)(p % a.de);
        const Slot &s = sl[r];
        int rbg = rb_of(s.dt[0], a.D), rbu = rb_of(s.dt[1], a.D);
        int cap = (SLOT_BYTES - 96) / (rbg + rbu);
        int64_t nr64 = p1 - p;
        if (nr64 > cap) nr64 = cap;
        if (nr64 > a.de - j) nr64 = a.de - j;
        int nr = (int)nr64;
        uint32_t off = 0, tx = 0;
        for (int m = 0; m < 2; m++) {
            uintptr_t src = (uintptr_t)(s.m[m] + (size_t)j * (m ? rbu : rbg));
            uintptr_t lo = src & ~(uintptr_t)15, hi = (src + (size_t)nr * (m ? rbu : rbg) + 15) & ~(uintptr_t)15;
            poff[n * MAXPIECE + m] = (uint16_t)(off + (src - lo));
            tx += (uint32_t)(hi - lo);
            off = up16(off + (uint32_t)(hi - lo));
        }
        desc[n] = ChunkDesc{ 0, (uint8_t)r, 2, 0, (uint16_t)nr, 0, (uint32_t)j, tx };
        n++;
        p += nr;
        if (p < p1 && n == MAXCH) return -1;   // plan does not fit: refuse rather than drop rows
    }
    return n - first;
}

__device__ int plan_phase_b(const FusedArgs &a, const Slot *sl, ChunkDesc *desc, uint16_t *poff, int first) {
    const int i0 = (int)((int64_t)a.D * blockIdx.x / gridDim.x), i1 = (int)((int64_t)a.D * (blockIdx.x + 1) / gridDim.x);
    int sum = 0;
    for (int r = 0; r < a.k; r++) sum += rb_of(sl[r].dt[2], a.de);
    int cap = (SLOT_BYTES - 48 * a.k) / sum;   // each piece may add 45 bytes of alignment
    int n = first;
    for (int i = i0; i < i1 && n < MAXCH;) {
        int nr = min(cap, i1 - i);
        uint32_t off = 0, tx = 0;
        for (int r = 0; r < a.k; r++) {
            int rbd = rb_of(sl[r].dt[2], a.de);
            uintptr_t src = (uintptr_t)(sl[r].m[2] + (size_t)i * rbd);
            uintptr_t lo = src & ~(uintptr_t)15, hi = (src + (size_t)nr * rbd + 15) & ~(uintptr_t)15;
            poff[n * MAXPIECE + r] = (uint16_t)(off + (src - lo));
            tx += (uint32_t)(hi - lo);
            off = up16(off + (uint32_t)(hi - lo));
        }
        desc[n] = ChunkDesc{ 1, 0, (uint8_t)a.k, 0, (uint16_t)nr, 0, (uint32_t)i, tx };
        n++;
        i += nr;
        if (i < i1 && n == MAXCH) return -1;
    }
    return n - first;
}

// Producer: issue chunk c's bulk copies into its stage.
__device__ void issue_chunk(const FusedArgs &a, const Slot *sl, const ChunkDesc &d, uint8_t *stage,
                            uint64_t *full) {
    mbar_expect_tx(full, d.tx);
    uint32_t off = 0;
    for (int q = 0; q < d.npiece; q++) {
        const Slot &s = d.phase == 0 ? sl[d.rank] : sl[q];
        int m = d.phase == 0 ? q : 2;
        int rb = d.phase == 0 ? rb_of(s.dt[m], a.D) : rb_of(s.dt[2], a.de);
        uintptr_t src = (uintptr_t)(s.m[m] + (size_t)d.row0 * rb);
        uintptr_t lo = src & ~(uintptr_t)15, hi = (src + (size_t)d.nrows * rb + 15) & ~(uintptr_t)15;
        bulk_g2s(stage + off, (const void *)lo, (uint32_t)(hi - lo), full);
        off = up16(off + (uint32_t)(hi - lo));
    }
}

__global__ void __launch_bounds__(NTHREADS, 1)
k_fused_ffn(const FusedArgs a, uint32_t *__restrict__ bar, uint32_t *__restrict__ err, int nslot) {
    extern __shared__ __align__(128) uint8_t smem[];
    const SmemLayout L = smem_layout(a.D, a.de, a.k, nslot);
    uint8_t *stage = smem + L.stage;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.full);
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L.empty);
    uint8_t *xq8k = smem + L.xq8k, *xq80 = smem + L.xq80, *hq = smem + L.hq;
    float *p_sm = reinterpret_cast<float *>(smem + L.p_sm);
    int32_t *ids = reinterpret_cast<int32_t *>(smem + L.ids);
    float *wr = reinterpret_cast<float *>(smem + L.w);
    BlockPart *parts = reinterpret_cast<BlockPart *>(smem + L.part);
    ChunkDesc *desc = reinterpret_cast<ChunkDesc *>(smem + L.desc);
    uint16_t *poff = reinterpret_cast<uint16_t *>(smem + L.poff);
    int *misc = reinterpret_cast<int *>(smem + L.misc);   // [0] nA, [1] nB, [2] abort
    __shared__ Slot sl[MAXK];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t hs = hq_stride(a.de);
    uint64_t *tr = a.trace ? a.trace + (size_t)blockIdx.x * FUSED_TRACE_POINTS : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = now_ns();

    // ---- prologue
    if (threadIdx.x == 0) {
        for (int s = 0; s < nslot; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        misc[2] = 0;
        misc[3] = ld_acquire(&bar[2]) != 0;   // an earlier launch failed: do nothing until reset
    }
    if (warp == 0) {
        warp_route(a.router, a.logits, a.mask, a.bias, a.E, a.k, a.routed_scale, p_sm, ids, wr, lane);
        if (lane < a.k) sl[lane] = a.slots[ids[lane]];
        if (tr && lane == 0) tr[1] = now_ns();
    } else if (warp <= NCW) {
        // x -> Q8_K and/or Q8_0 blocks, one warp per block
        const int nb8k = (a.x_kinds & 1u) ? a.D / 256 : 0, nb80 = (a.x_kinds & 2u) ? a.D / 32 : 0;
        for (int b = warp - 1; b < nb8k + nb80; b += NCW) {
            if (b < nb8k) warp_quant_q8k(a.x + 256 * b, 256, xq8k + 292 * b, lane);
            else warp_quant_q80(a.x + 32 * (b - nb8k), 32, xq80 + 36 * (b - nb8k), lane);
        }
    }
    __syncthreads();
    if (misc[3]) {
        if (threadIdx.x == 0) raise_error(err, bar, FUSED_ERR_BARRIER);
        return;
    }
    if (threadIdx.x == 32) misc[0] = plan_phase_a(a, sl, desc, poff, 0);
    __syncthreads();
    if (threadIdx.x == 32) misc[1] = misc[0] < 0 ? 0 : plan_phase_b(a, sl, desc, poff, misc[0]);
    if (blockIdx.x == 0 && threadIdx.x < a.k) {
        a.ids_out[threadIdx.x] = ids[threadIdx.x];
        a.w_out[threadIdx.x] = wr[threadIdx.x];
    }
    __syncthreads();
    if (misc[0] < 0 || misc[1] < 0) {
        // the plan did not fit in MAXCH chunks: nothing was issued; every CTA
        // takes this path before the grid barrier, so none waits there
        if (threadIdx.x == 0) raise_error(err, bar, FUSED_ERR_PLAN);
        return;
    }
    const int nA = misc[0], nCh = misc[0] + misc[1];
    if (tr && threadIdx.x == 0) tr[2] = now_ns();

    if (warp == NCW) {
        // ---- producer
        if (lane == 0) {
            for (int c = 0; c < nCh; c++) {
                int s = c % nslot, u = c / nslot;
                if (u > 0 && !mbar_wait(&empty[s], (uint32_t)(u - 1) & 1u)) {
                    raise_error(err, bar, FUSED_ERR_COPY);
                    break;
                }
                issue_chunk(a, sl, desc[c], stage + (size_t)s * SLOT_BYTES, &full[s]);
            }
        }
        return;
    }

    // ---- phase A: gate/up + SwiGLU
    BlockPart *part = parts + warp * FCHUNK;
    bool abort = false;      // skip the arithmetic (results of this launch are invalid)
    bool dead = false;       // a copy wait expired: stop waiting on copies
    for (int c = 0; c < nA; c++) {
        int s = c % nslot;
        if (!dead && !mbar_wait(&full[s], (uint32_t)(c / nslot) & 1u)) {
            dead = abort = true;
            if (lane == 0) raise_error(err, bar, FUSED_ERR_COPY);
        }
        const ChunkDesc d = desc[c];
        const uint8_t *base = stage + (size_t)s * SLOT_BYTES;
        const Slot &e = sl[d.rank];
        const int dg = e.dt[0], du = e.dt[1];
        const int rbg = rb_of(dg, a.D), rbu = rb_of(du, a.D);
        const uint8_t *ag = act_kind_for(dg) == DT_Q8_0 ? xq80 : xq8k;
        const uint8_t *au = act_kind_for(du) == DT_Q8_0 ? xq80 : xq8k;
        if (!abort)
            for (int t = warp; t < d.nrows; t += NCW) {
                float g = smem_row_dot(dg, base + poff[c * MAXPIECE + 0] + (size_t)t * rbg, ag, a.D / dt_block(dg),
                                       part, lane);
                float u = smem_row_dot(du, base + poff[c * MAXPIECE + 1] + (size_t)t * rbu, au, a.D / dt_block(du),
                                       part, lane);
                if (lane == 0) a.hbuf[(size_t)d.rank * a.de + d.row0 + t] = __fmul_rn(silu_f(g), u);
            }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- grid barrier: every CTA's hbuf rows are written
    consumer_sync();
    if (tr && threadIdx.x == 0) tr[3] = now_ns();
    if (threadIdx.x == 0) {
        uint32_t gen = ld_acquire(&bar[1]);
        __threadfence();
        uint32_t arrived = atomicAdd(&bar[0], 1u);
        if (arrived == gridDim.x - 1) {
            atomicExch(&bar[0], 0u);
            __threadfence();
            st_release(&bar[1], gen + 1u);
        } else {
            const uint64_t t0 = now_ns();
            while (ld_acquire(&bar[1]) == gen) {
                if (now_ns() - t0 > BARRIER_NS) {
                    raise_error(err, bar, FUSED_ERR_BARRIER);
                    misc[2] = 1;
                    break;
                }
                __nanosleep(32);
            }
        }
        __threadfence();
    }
    consumer_sync();
    abort = abort || misc[2] != 0;
    if (tr && threadIdx.x == 0) tr[4] = now_ns();

    // ---- re-quantise h for all k experts (each CTA holds the full set)
    if (!abort) {
        for (int r = 0; r < a.k; r++) {
            const int kind = act_kind_for(sl[r].dt[2]);
            const int qk = kind == DT_Q8_K ? 256 : 32, ab = kind == DT_Q8_K ? 292 : 36;
            const int nb = (a.de + qk - 1) / qk;
            for (int b = warp; b < nb; b += NCW)
                warp_quant_h(a.hbuf + (size_t)r * a.de + (size_t)b * qk, min(qk, a.de - b * qk), kind,
                             hq + (size_t)r * hs + (size_t)b * ab, lane);
        }
    }
    consumer_sync();
    if (tr && threadIdx.x == 0) tr[5] = now_ns();

    // ---- phase B: down rows of all k experts + rank-ordered combine
    for (int c = nA; c < nCh; c++) {
        int s = c % nslot;
        if (!dead && !mbar_wait(&full[s], (uint32_t)(c / nslot) & 1u)) {
            dead = abort = true;
            if (lane == 0) raise_error(err, bar, FUSED_ERR_COPY);
        }
        const ChunkDesc d = desc[c];
        const uint8_t *base = stage + (size_t)s * SLOT_BYTES;
        if (!abort)
            for (int t = warp; t < d.nrows; t += NCW) {
                float ffn = 0.0f;
                for (int r = 0; r < a.k; r++) {
                    const int dt = sl[r].dt[2];
                    const int rbd = rb_of(dt, a.de);
                    float eo = smem_row_dot(dt, base + poff[c * MAXPIECE + r] + (size_t)t * rbd, hq + (size_t)r * hs,
                                            a.de / dt_block(dt), part, lane);
                    ffn = __fadd_rn(ffn, __fmul_rn(wr[r], eo));
                }
                if (lane == 0) {
                    const int i = (int)d.row0 + t;
                    if (a.s_out) ffn = __fadd_rn(ffn, __fmul_rn(*a.sgate, a.s_out[i]));
                    a.ffn[i] = ffn;
                    if (a.h) a.h[i] = __fadd_rn(a.h[i], ffn);
                }
            }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (tr) {
        consumer_sync();
        if (threadIdx.x == 0) tr[6] = now_ns();
    }
}

// ---------------------------------------------------------------------------
// host side
int fused_init(FusedScratch &f, const tlmg_geom &g) {
    f.enabled = false;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return cuda_fail(cudaGetLastError(), "device properties");
    if (!prop.cooperativeLaunch) return TLMG_OK;
    if (g.n_experts <= 0 || g.top_k > MAXK || g.n_experts > RT_PER * 32) return TLMG_OK;
    const size_t limit = prop.sharedMemPerBlockOptin;
    int nslot = 0;
    for (int ns = 8; ns >= 2; ns--)
        if (smem_layout(g.d_model, g.d_expert, g.top_k, ns).total + 1024 <= limit) {
            nslot = ns;
            break;
        }
    if (!nslot) return TLMG_OK;
    f.nslot = nslot;
    f.slot_bytes = SLOT_BYTES;
    f.smem = smem_layout(g.d_model, g.d_expert, g.top_k, nslot).total;
    if (cudaFuncSetAttribute(k_fused_ffn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)f.smem) != cudaSuccess) {
        cudaGetLastError();
        return TLMG_OK;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_fused_ffn, NTHREADS, f.smem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        return TLMG_OK;
    }
    f.nsm = prop.multiProcessorCount;
    if (cudaMalloc(&f.bar, 64) != cudaSuccess) return set_error(TLMG_ENOMEM, "fused barrier allocation");
    cudaMemset(f.bar, 0, 64);
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
    f = FusedScratch{};
}

bool fused_supports(const FusedScratch &f, const tlmg_geom &g, const int *gu, int n_gu, const int *dn, int n_dn) {
    if (!f.enabled) return false;
    auto ok_dt = [](int dt) {
        return dt == DT_Q4_K || dt == DT_Q5_K || dt == DT_Q6_K || dt == DT_Q8_K || dt == DT_Q8_0;
    };
    int max_gu = 0, max_dn = 0;
    for (int i = 0; i < n_gu; i++) {
        if (!ok_dt(gu[i]) || g.d_model % dt_block(gu[i])) return false;
        max_gu = std::max(max_gu, g.d_model / dt_block(gu[i]) * dt_block_bytes(gu[i]));
    }
    for (int i = 0; i < n_dn; i++) {
        if (!ok_dt(dn[i]) || g.d_expert % dt_block(dn[i])) return false;
        max_dn = std::max(max_dn, g.d_expert / dt_block(dn[i]) * dt_block_bytes(dn[i]));
    }
    if (2 * max_gu + 96 > SLOT_BYTES) return false;
    if (g.top_k * (max_dn + 48) > SLOT_BYTES) return false;
    // chunk budget: phase A chunks + expert splits, phase B chunks
    const int G = f.nsm;
    int64_t pairs = ((int64_t)g.top_k * g.d_expert + G - 1) / G;
    int64_t ca = pairs / std::max(1, (SLOT_BYTES - 96) / (2 * max_gu)) + g.top_k + 2;
    int64_t rows = (g.d_model + G - 1) / G;
    int64_t cb = rows / std::max(1, (SLOT_BYTES - 48 * g.top_k) / (g.top_k * max_dn)) + 2;
    return ca + cb <= MAXCH;
}

int launch_fused_ffn(FusedScratch &f, const FusedArgs &a, cudaStream_t st) {
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
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_fused_ffn, a, f.bar, f.err_dev, f.nslot);
    count_launch();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "fused expert FFN launch");
}

uint32_t fused_take_error(FusedScratch &f) {
    if (!f.err_host) return 0;
    uint32_t e = *(volatile uint32_t *)f.err_host;
    if (e) {
        // the stream is idle (the caller synchronised): clear the sticky
        // device word and the barrier state for the next launch
        *(volatile uint32_t *)f.err_host = 0;
        cudaMemset(f.bar, 0, 64);
    }
    return e;
}

}  // namespace tlmg
