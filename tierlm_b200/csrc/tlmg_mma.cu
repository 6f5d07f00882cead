// tlmg_mma.cu - grouped expert GEMM on tcgen05 (sm_100a), exact.
//
// Work item = (active expert, tile of 128 weight rows[, matrix]); one CTA of
// threads (gate/up: one per weight row; down: two per row, each half of the
// sub-blocks), thread r <-> weight row r <-> TMEM lane r. For each pass of
// up to TN tokens of the expert (8 for gate/up, 16 for down) and each
// K-quant block b in ascending order:
//
//   1. the tile's raw block column is staged with cp.async (16-byte pieces);
//   2. thread r unpacks its row into int8 codes in the canonical K-major
//      no-swizzle UMMA layout (core matrix = 8 rows x 16 bytes) - Q4_K / Q5_K
//      codes 0..31, Q6_K codes minus 32 - and keeps the block's scales;
//   3. one thread issues one tcgen05.mma kind::i8 (M = 128, N = TN, K = 32)
//      per sub-block: A = the sub-block's codes, B = the tokens' Q8_K codes of
//      the same elements, D = that sub-block's own int32 accumulator in TMEM
//      (a Q4_K / Q5_K sub-block is 32 elements; a Q6_K group is 16 elements,
//      its second K half reads a zero chunk of B). Each accumulator is the
//      exact integer dot of one sub-block;
//   4. thread r reads its row's accumulators (tcgen05.ld) and forms the
//      reference's per-block sums is = sum_s scale_s * dot_s (and the min
//      sum ms from the activation block sums), then the fmaf chain step of
//      block b for every token (acc = fmaf(d_w d_a, is, acc), Q4_K / Q5_K also
//      fmaf(-dmin_w d_a, ms, acc)).
//
// Integer addition is exact, so is / ms equal the reference's per-block
// integer sums, and the chain runs in block order: results are bit-identical
// to the single-token kernels (reference dot_kq_affine_ref / dot_q6_k_ref,
// src/lib/tlm_quant.c:814-882).
//
// Waits on the MMA completion barrier are bounded; on expiry the kernel sets
// bit 0 of *err, waits (bounded) once more, frees its TMEM and returns.
#include <algorithm>
#include <vector>

#include "tlmg_dev.cuh"
#include "tlmg_internal.h"
#include "tlmg_kq.cuh"
#include "tlmg_mma.cuh"

namespace tlmg {

namespace {

constexpr int MR = 128;   // rows per tile = TMEM lanes = MMA M = threads
constexpr int MAXNB = 16; // K blocks per row (K <= 4096)

template <int DT> struct KQ;
template <> struct KQ<DT_Q4_K> { static constexpr int BB = 144, SUB = 8; };
template <> struct KQ<DT_Q5_K> { static constexpr int BB = 176, SUB = 8; };
template <> struct KQ<DT_Q6_K> { static constexpr int BB = 210, SUB = 16; };

__host__ __device__ constexpr uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }
__host__ __device__ inline uint32_t qvec_bytes(int nb) { return 288u * nb + align_up(4u * nb, 16u); }

// ---------------------------------------------------------------------------
// PTX wrappers
__device__ __forceinline__ uint32_t saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// generic-proxy shared writes -> visible to the tensor cores' async proxy
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor, K-major, no swizzle: start, leading byte
// offset (between the two 16-byte K halves), stride byte offset (between
// 8-row core-matrix groups), version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc(uint32_t start, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((start >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc) {
    // D = A * B (enable-input-d false: every accumulator starts from zero)
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(z), "r"(z)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(mbar))
                 : "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t *mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(mbar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");   // visible to the tensor cores' arrive
}
// Waits for phase `parity` of the barrier to complete; false after `limit` polls.
__device__ __forceinline__ bool mbar_wait(uint64_t *mbar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; i++) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done)
            : "r"(saddr(mbar)), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(dst)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// 64 consecutive 32-bit columns of this thread's TMEM lane. The load and
// its wait are one asm statement: the registers are only valid after
// tcgen05.wait::ld, and the compiler must not schedule their uses earlier.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, int (&v)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]), "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]), "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]), "=r"(v[48]), "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]), "=r"(v[56]), "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])
        : "r"(taddr)
        : "memory");
}

constexpr uint32_t WAIT_LIMIT = 1u << 20;   // polls of a completion barrier before giving up

// 32 consecutive columns (load and wait in one statement, as tmem_ld64)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

// ---------------------------------------------------------------------------
// Row unpack: one weight block of this thread's row -> 16 chunks of 16 int8
// codes (chunk c = elements 16c .. 16c + 15) at A + c * 128 + (row % 8) * 16
// within the row's 8-row group; the block's scale factors are returned.
// half = 0 / 1 unpacks only the first / second half of the sub-blocks.
struct RowBlk {
    uint32_t s[4];   // Q4_K/Q5_K: sc03, sc47, mn03, mn47 (6-bit bytes); Q6_K: int8 scales 0..15
    float d, dmin;
};

__device__ __forceinline__ void st16(uint8_t *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    *reinterpret_cast<uint4 *>(p) = make_uint4(a, b, c, d);
}

template <int DT>
__device__ __forceinline__ RowBlk unpack_row(const uint8_t *blk, uint8_t *A, int half = -1) {
    RowBlk rb;
    if constexpr (DT == DT_Q4_K || DT == DT_Q5_K) {
        constexpr int QOFF = DT == DT_Q4_K ? 16 : 48;
        const uint4 h = lds128(blk);
        rb.d = h2f(h.x & 0xFFFFu);
        rb.dmin = h2f(h.x >> 16);
        rb.s[0] = h.y & 0x3F3F3F3Fu;
        rb.s[1] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
        rb.s[2] = h.z & 0x3F3F3F3Fu;
        rb.s[3] = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
        uint4 g[2] = { make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u) };
        if constexpr (DT == DT_Q5_K) {
            g[0] = lds128(blk + 16);
            g[1] = lds128(blk + 32);
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {   // qs piece j: chunk c = j / 2, bytes 16 (j % 2) ..
            if (half >= 0 && (j >> 2) != half) continue;   // half h: sub-blocks 4h .. 4h + 3
            const int c = j >> 1, hh = j & 1;
            const uint4 v = lds128(blk + QOFF + 16 * j);
            uint4 lo = make_uint4(v.x & 0x0F0F0F0Fu, v.y & 0x0F0F0F0Fu, v.z & 0x0F0F0F0Fu, v.w & 0x0F0F0F0Fu);
            uint4 hi = make_uint4((v.x >> 4) & 0x0F0F0F0Fu, (v.y >> 4) & 0x0F0F0F0Fu, (v.z >> 4) & 0x0F0F0F0Fu,
                                  (v.w >> 4) & 0x0F0F0F0Fu);
            if constexpr (DT == DT_Q5_K) {   // 5th bit: qh[l] bit 2c (low) / 2c + 1 (high), l = 16 hh + i
                const uint4 q = g[hh];
                lo.x |= ((q.x >> (2 * c)) & 0x01010101u) << 4;
                lo.y |= ((q.y >> (2 * c)) & 0x01010101u) << 4;
                lo.z |= ((q.z >> (2 * c)) & 0x01010101u) << 4;
                lo.w |= ((q.w >> (2 * c)) & 0x01010101u) << 4;
                hi.x |= ((q.x >> (2 * c + 1)) & 0x01010101u) << 4;
                hi.y |= ((q.y >> (2 * c + 1)) & 0x01010101u) << 4;
                hi.z |= ((q.z >> (2 * c + 1)) & 0x01010101u) << 4;
                hi.w |= ((q.w >> (2 * c + 1)) & 0x01010101u) << 4;
            }
            st16(A + (4 * c + hh) * 128, lo.x, lo.y, lo.z, lo.w);       // elements 64c + 16hh ..
            st16(A + (4 * c + 2 + hh) * 128, hi.x, hi.y, hi.z, hi.w);   // elements 64c + 32 + 16hh ..
        }
    } else {
        // Q6_K at a 2-byte aligned address: 4-byte aligned words + funnel shifts
        const uintptr_t a = reinterpret_cast<uintptr_t>(blk);
        const uint32_t *wp = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
        const uint32_t sh = (uint32_t)(a & 3u) * 8u;
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int p = 0; p < 2; p++) {
                if (half >= 0 && h != half) continue;   // half h: groups 8h .. 8h + 7
                uint32_t u[4][4];   // [mm][i]: chunk 8h + 2mm + p, word i
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int lw = 4 * p + i;
                    const int ja = 16 * h + lw, jb = 16 * h + 8 + lw, jc = 32 + 8 * h + lw;
                    const uint32_t Aw = __funnelshift_r(wp[ja], wp[ja + 1], sh);
                    const uint32_t Bw = __funnelshift_r(wp[jb], wp[jb + 1], sh);
                    const uint32_t Cw = __funnelshift_r(wp[jc], wp[jc + 1], sh);
                    u[0][i] = __vsub4((Aw & 0x0F0F0F0Fu) | ((Cw << 4) & 0x30303030u), 0x20202020u);
                    u[1][i] = __vsub4((Bw & 0x0F0F0F0Fu) | ((Cw << 2) & 0x30303030u), 0x20202020u);
                    u[2][i] = __vsub4(((Aw >> 4) & 0x0F0F0F0Fu) | (Cw & 0x30303030u), 0x20202020u);
                    u[3][i] = __vsub4(((Bw >> 4) & 0x0F0F0F0Fu) | ((Cw >> 2) & 0x30303030u), 0x20202020u);
                }
#pragma unroll
                for (int mm = 0; mm < 4; mm++) st16(A + (8 * h + 2 * mm + p) * 128, u[mm][0], u[mm][1], u[mm][2], u[mm][3]);
            }
        rb.s[0] = __funnelshift_r(wp[48], wp[49], sh);
        rb.s[1] = __funnelshift_r(wp[49], wp[50], sh);
        rb.s[2] = __funnelshift_r(wp[50], wp[51], sh);
        rb.s[3] = __funnelshift_r(wp[51], wp[52], sh);
        rb.d = h2f(__funnelshift_r(wp[52], wp[53], sh) & 0xFFFFu);
        rb.dmin = 0.0f;
    }
    return rb;
}

// ---------------------------------------------------------------------------
// Shared-memory plan of one CTA (same on host and device); TN = tokens per
// pass (MMA N, 8 or 16).
struct MPlan {
    uint32_t raw, raw_bytes;   // raw weight stages
    uint32_t A;                // unpacked int8 tiles [nmat][16 groups][16 chunks][8 rows][16 B]
    uint32_t X, xsbo;          // token codes [TN / 8 groups][KC + 1 chunks][8 tokens][16 B] (chunk KC zero)
    uint32_t dx, bs;           // f32 [TN][nb] block scales, int32 [TN][nb][8] sub-block bsums
    uint32_t xch;              // 32-bit [MR][TN]: the second thread of a row hands its results over (or none)
    uint32_t bar, total;       // mbarrier (8 B) + TMEM address (4 B)
};
template <int TN>
__host__ __device__ inline MPlan mplan(int nmat, uint32_t raw_bytes, int nb, bool xch) {
    MPlan p{};
    p.raw = 0;
    p.raw_bytes = raw_bytes;
    p.A = align_up(raw_bytes, 1024u);
    p.X = p.A + (uint32_t)nmat * MR * 256u;
    p.xsbo = (uint32_t)(16 * nb + 1) * 128u;
    p.dx = p.X + (uint32_t)(TN / 8) * p.xsbo;
    p.bs = p.dx + align_up((uint32_t)TN * nb * 4u, 16u);
    p.xch = p.bs + (uint32_t)TN * nb * 8u * 4u;
    p.bar = p.xch + (xch ? (uint32_t)MR * TN * 4u : 0u);
    p.total = p.bar + 16u;
    return p;
}

// Stages the pass's tokens: codes into the canonical B layout (cp.async),
// block scales and sub-block sums into dx / bs. Zeroes the chunk KC of each
// token group once per CTA (first == true).
template <int DT, int TN>
__device__ __forceinline__ void stage_tokens(uint8_t *sm, const MPlan &P, const uint8_t *x, size_t xstride, int xdiv,
                                             const int32_t *pairs, int nt, int nb, bool first) {
    const int KC = 16 * nb;
    uint8_t *X = sm + P.X;
    if (first)
        for (int i = threadIdx.x; i < TN; i += blockDim.x)
            *reinterpret_cast<uint4 *>(X + (i >> 3) * P.xsbo + KC * 128 + (i & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
    for (int i = threadIdx.x; i < nt * KC; i += blockDim.x) {
        const int t = i / KC, kc = i - t * KC;
        const uint8_t *v = x + (size_t)(pairs[t] / xdiv) * xstride;
        // swizzled Q8_K vector: piece p of block b at (p * nb + b) * 16
        cp16(X + (t >> 3) * P.xsbo + kc * 128 + (t & 7) * 16, v + ((size_t)(kc & 15) * nb + (kc >> 4)) * 16);
    }
    float *dx = reinterpret_cast<float *>(sm + P.dx);
    int *bs = reinterpret_cast<int *>(sm + P.bs);
    for (int i = threadIdx.x; i < nt * nb; i += blockDim.x) {
        const int t = i / nb, b = i - t * nb;
        const uint8_t *v = x + (size_t)(pairs[t] / xdiv) * xstride;
        dx[i] = reinterpret_cast<const float *>(v + 288 * nb)[b];
        if constexpr (DT != DT_Q6_K) {
            const int16_t *s16 = reinterpret_cast<const int16_t *>(v + 256 * nb) + 16 * b;
#pragma unroll
            for (int s = 0; s < 8; s++) bs[i * 8 + s] = (int)s16[2 * s] + (int)s16[2 * s + 1];
        }
    }
}

// Instruction descriptor: D s32 (c_format 2), A and B signed 8-bit, both
// K-major, N = TN, M = 128.
template <int TN>
constexpr uint32_t idesc() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(MR >> 4) << 24);
}

// Thread 0 issues the MMAs of block b for matrices m0 .. m0 + NMAT - 1 of
// the A tiles (every sub-block into its own accumulator, columns
// (m * SUB + s) * TN) and commits them to the barrier.
template <int DT, int NMAT, int TN>
__device__ __forceinline__ void issue_block(uint8_t *sm, const MPlan &P, uint32_t tmem, int b) {
    constexpr int SUB = KQ<DT>::SUB;
    const uint32_t Xs = saddr(sm + P.X), As = saddr(sm + P.A);
    const int KC = (int)(P.xsbo / 128u) - 1;
    tc_fence_after();
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int s = 0; s < SUB; s++) {
            uint64_t ad, bd;
            if constexpr (DT == DT_Q6_K) {
                // group s = chunk s; B's second K half is the zero chunk KC
                const int kc = 16 * b + s;
                ad = umma_desc(As + m * MR * 256u + s * 128u, 128u, 2048u);
                bd = umma_desc(Xs + kc * 128u, (uint32_t)(KC - kc) * 128u, P.xsbo);
            } else {
                const int kc = 16 * b + 2 * s;
                ad = umma_desc(As + m * MR * 256u + 2 * s * 128u, 128u, 2048u);
                bd = umma_desc(Xs + kc * 128u, 128u, P.xsbo);
            }
            umma_i8(tmem + (uint32_t)((m * SUB + s) * TN), ad, bd, idesc<TN>());
        }
    umma_commit(reinterpret_cast<uint64_t *>(sm + P.bar));
}

// is[t] += scale_s * dot_s[t] over sub-blocks s0 .. s0 + ns - 1 of one
// matrix whose sub-block s accumulator starts at column col0 + s * TN
// (ns * TN a multiple of 32).
template <int DT, int TN>
__device__ __forceinline__ int scale_of(const RowBlk &rb, int s) {
    if constexpr (DT == DT_Q6_K) return (int)(int8_t)byte_of(rb.s[s >> 2], s & 3);
    else return (int)byte_of(rb.s[s >> 2], s & 3);
}
template <int DT, int TN>
__device__ __forceinline__ void add_scaled(uint32_t lane_base, uint32_t col0, int s0, int ns, const RowBlk &rb,
                                           int (&is)[TN]) {
    if (ns * TN == 32) {
        constexpr int SPL = 32 / TN;
        int v[32];
        tmem_ld32(lane_base + col0 + (uint32_t)(s0 * TN), v);
#pragma unroll
        for (int j = 0; j < SPL; j++) {
            const int sc = scale_of<DT, TN>(rb, s0 + j);
#pragma unroll
            for (int t = 0; t < TN; t++) is[t] += sc * v[TN * j + t];
        }
        return;
    }
    constexpr int SPL = 64 / TN;   // sub-blocks per 64-column load
#pragma unroll 1
    for (int g = 0; g < ns; g += SPL) {
        int v[64];
        tmem_ld64(lane_base + col0 + (uint32_t)((s0 + g) * TN), v);
#pragma unroll
        for (int j = 0; j < SPL; j++) {
            const int sc = scale_of<DT, TN>(rb, s0 + g + j);
#pragma unroll
            for (int t = 0; t < TN; t++) is[t] += sc * v[TN * j + t];
        }
    }
}

// The chain step of block b for tokens t0 .. t0 + NTOK - 1 of the pass
// (acc[i] belongs to token t0 + i): acc = fmaf(d_w d_a, is, acc) and, for
// Q4_K / Q5_K, fmaf(-dmin_w d_a, ms, acc).
template <int DT, int NTOK>
__device__ __forceinline__ void chain_range(const uint8_t *sm, const MPlan &P, int b, int nb, const RowBlk &rb,
                                            const int (&is)[NTOK], float (&acc)[NTOK], int t0, int nt) {
    const float *dx = reinterpret_cast<const float *>(sm + P.dx);
    const int *bs = reinterpret_cast<const int *>(sm + P.bs);
#pragma unroll
    for (int i = 0; i < NTOK; i++) {
        const int t = t0 + i;
        if (t < nt) {
            const float d = dx[t * nb + b];
            int ms = 0;
            if constexpr (DT != DT_Q6_K) {
                const int4 b0 = *reinterpret_cast<const int4 *>(bs + (t * nb + b) * 8);
                const int4 b1 = *reinterpret_cast<const int4 *>(bs + (t * nb + b) * 8 + 4);
                ms = (int)byte_of(rb.s[2], 0) * b0.x + (int)byte_of(rb.s[2], 1) * b0.y +
                     (int)byte_of(rb.s[2], 2) * b0.z + (int)byte_of(rb.s[2], 3) * b0.w +
                     (int)byte_of(rb.s[3], 0) * b1.x + (int)byte_of(rb.s[3], 1) * b1.y +
                     (int)byte_of(rb.s[3], 2) * b1.z + (int)byte_of(rb.s[3], 3) * b1.w;
            }
            acc[i] = chain<DT>(acc[i], __fmul_rn(rb.d, d), is[i], __fmul_rn(rb.dmin, d), ms);
        }
    }
}

// The block's chain step for every token of the pass.
template <int DT, int TN>
__device__ __forceinline__ void chain_tokens(const uint8_t *sm, const MPlan &P, int b, int nb, const RowBlk &rb,
                                             const int (&is)[TN], float (&acc)[TN], int nt) {
    chain_range<DT, TN>(sm, P, b, nb, rb, is, acc, 0, nt);
}

__device__ __forceinline__ void report(uint32_t *err, bool ok) {
    if (!ok && threadIdx.x == 0) atomicOr(err, 1u);
}

// gate or up: K = D. Work item = (active expert, 128-row tile, matrix);
// two threads per weight row (warps 0-3 and 4-7; TMEM lane = row): each
// unpacks and sums half of the block's sub-blocks, they swap the partial
// integer sums of each other's tokens and each runs the chains of half of
// the pass's tokens. Raw stages hold one block column [NS][MR][BB] of the
// tile. out[m][pair][row] = the row's dot (m = 0 gate, 1 up). Small enough
// for two CTAs per SM at 8 tokens per pass.
constexpr int GU_THREADS = 2 * MR;
#ifndef TLMG_MGU_MINB
#define TLMG_MGU_MINB 2   // CTAs per SM the 8-token gate/up kernel is compiled for
#endif
#ifndef TLMG_MGU_NS8
#define TLMG_MGU_NS8 3    // raw stages of the 8-token gate/up kernel (D <= 2048)
#endif
// Work items per (expert, tile, matrix) with wide passes: 2 splits the
// token passes in halves, so that 2048-token prefill's 1,536 gate/up items
// (5.2 per CTA of 296) become 3,072 with a shorter last wave: 21.9k tok/s
// against 21.6k with 1 (B200, 48 layers).
#ifndef TLMG_GU_WIDE_PARTS
#define TLMG_GU_WIDE_PARTS 2
#endif
template <int DT, int NS, int TN>
__global__ void __launch_bounds__(GU_THREADS, TN <= 8 ? TLMG_MGU_MINB : TN <= 16 ? 2 : 1)
    k_mgu(const Slot *__restrict__ slots, const int32_t *__restrict__ grp, const uint8_t *__restrict__ x,
          size_t xstride, int xdiv, int D, int de, int E, float *__restrict__ gout, float *__restrict__ uout,
          uint32_t *err) {
    constexpr int TH = TN / 2;   // tokens per thread
    extern __shared__ __align__(1024) uint8_t sm[];
    constexpr int BB = KQ<DT>::BB, CPB = BB / 16;
    static_assert(BB % 16 == 0, "gate/up blocks must be 16-byte multiples");
    const int nb = D / 256;
    const MPlan P = mplan<TN>(1, (uint32_t)NS * MR * BB, nb, true);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + P.bar + 8);
    const int tid = threadIdx.x, warp = tid >> 5, half = tid / MR, r = tid & (MR - 1);
    pdl_enter();
    if (tid == 0) mbar_init(reinterpret_cast<uint64_t *>(sm + P.bar), 1);
    if (warp == 0) tmem_alloc(tmem_slot, 8 * TN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    uint32_t phase = 0;
    bool ok = true;
    const int tiles = de / MR, na = grp[2 * E + 1];
    const size_t rb = (size_t)nb * BB;
    const int32_t *pairs = grp + 2 * E + 2;
    int *xmine = reinterpret_cast<int *>(sm + P.xch) + (half * MR + r) * TH;         // written by this thread
    const int *xother = reinterpret_cast<const int *>(sm + P.xch) + ((1 - half) * MR + r) * TH;
    const int t0 = half * TH;   // this thread's tokens t0 .. t0 + TH - 1
    bool first = true;
    uint8_t *Arow = sm + P.A + (r >> 3) * 2048 + (r & 7) * 16;
    // wide passes: each (expert, tile, matrix) is split into PARTS items by
    // its token passes, so that the last wave of items is shorter
    constexpr int PARTS = TN > 8 ? TLMG_GU_WIDE_PARTS : 1;
    for (int item = blockIdx.x; item < na * tiles * 2 * PARTS && ok; item += gridDim.x) {
        const int part = item % PARTS, mi = item / PARTS;
        const int m = mi & 1, it = mi >> 1, ae = it / tiles, tile = it - ae * tiles, e = grp[E + 1 + ae];
        const uint8_t *w = slots[e].m[m] + (size_t)tile * MR * rb;
        float *out = m ? uout : gout;
        auto issue = [&](int b) {
            if (b < nb) {
                uint8_t *st = sm + P.raw + (b % NS) * MR * BB;
                for (int i = tid; i < MR * CPB; i += GU_THREADS) {
                    const int rr = i / CPB, c = i - rr * CPB;
                    cp16(st + rr * BB + 16 * c, w + rr * rb + (size_t)b * BB + 16 * c);
                }
            }
            cp_commit();
        };
        const int passes = (grp[e + 1] - grp[e] + TN - 1) / TN;
        const int c_lo = grp[e] + TN * (passes * part / PARTS);
        const int c_hi = min(grp[e + 1], grp[e] + TN * (passes * (part + 1) / PARTS));
        for (int c0 = c_lo; c0 < c_hi && ok; c0 += TN) {
            const int nt = min(TN, c_hi - c0);
            stage_tokens<DT, TN>(sm, P, x, xstride, xdiv, pairs + c0, nt, nb, first);
            first = false;
#pragma unroll
            for (int b = 0; b < NS - 1; b++) issue(b);
            float acc[TH];
#pragma unroll
            for (int i = 0; i < TH; i++) acc[i] = 0.0f;
            for (int b = 0; b < nb; b++) {
                cp_wait<NS - 2>();
                __syncthreads();   // block b staged; the previous block's tile, accumulators and swaps are consumed
                issue(b + NS - 1);
                const RowBlk rk = unpack_row<DT>(sm + P.raw + (b % NS) * MR * BB + r * BB, Arow, half);
                fence_async_smem();
                __syncthreads();
                if (tid == 0) issue_block<DT, 1, TN>(sm, P, tmem, b);
                const bool got = mbar_wait(reinterpret_cast<uint64_t *>(sm + P.bar), phase, WAIT_LIMIT);
                phase ^= 1u;
                tc_fence_after();
                int is[TN];
#pragma unroll
                for (int t = 0; t < TN; t++) is[t] = 0;
                add_scaled<DT, TN>(lane_base, 0u, 4 * half, 4, rk, is);   // sub-blocks 4 half .. 4 half + 3
#pragma unroll
                for (int i = 0; i < TH; i++) xmine[i] = half ? is[i] : is[TH + i];   // the other thread's tokens
                tc_fence_before();
                if (__syncthreads_or(!got)) ok = false;   // uniform across the CTA; publishes the swaps
                if (!ok) break;
                int own[TH];
#pragma unroll
                for (int i = 0; i < TH; i++) own[i] = (half ? is[TH + i] : is[i]) + xother[i];   // exact: both halves' sums
                chain_range<DT, TH>(sm, P, b, nb, rk, own, acc, t0, nt);
            }
            cp_wait<0>();
#pragma unroll
            for (int i = 0; i < TH; i++)
                if (t0 + i < nt) out[(size_t)pairs[c0 + t0 + i] * de + tile * MR + r] = acc[i];
            __syncthreads();   // staged tokens are rewritten next
        }
    }
    if (!ok) {   // an MMA may still be in flight: one more bounded wait before the TMEM goes
        mbar_wait(reinterpret_cast<uint64_t *>(sm + P.bar), phase ^ 1u, WAIT_LIMIT);   // the phase that expired
        report(err, false);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_free(tmem, 8 * TN);
}

// down: K = de. Work item = (active expert, 128-row tile); thread = weight
// row = TMEM lane. The tile's rows x all blocks (contiguous in HBM) are
// staged whole; each block is unpacked and multiplied in two halves through
// a half-block A tile (8 chunks), so that the CTA fits twice on an SM and
// the two CTAs overlap each other's copies, unpacking and epilogues.
constexpr int DN_THREADS = MR;
template <int DT, int TN>
__global__ void __launch_bounds__(DN_THREADS, TN <= 8 ? 2 : 1)
    k_mdown(const Slot *__restrict__ slots, const int32_t *__restrict__ grp, const uint8_t *__restrict__ hq, int D,
            int de, int E, float *__restrict__ eo, uint32_t *err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    constexpr int BB = KQ<DT>::BB, SUB = KQ<DT>::SUB;
    constexpr uint32_t NCOL = SUB * TN <= 64 ? 64 : SUB * TN <= 128 ? 128 : SUB * TN <= 256 ? 256 : 512;
    const int nb = de / 256;
    const uint32_t tile_bytes = (uint32_t)MR * nb * BB;   // a multiple of 16
    const MPlan P = mplan<TN>(0, align_up(tile_bytes, 1024u) + MR * 128u, nb, false);   // raw tile + half A tile
    const uint32_t Ahalf = align_up(tile_bytes, 1024u);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + P.bar + 8);
    const int r = threadIdx.x, warp = r >> 5;
    pdl_enter();
    if (r == 0) mbar_init(reinterpret_cast<uint64_t *>(sm + P.bar), 1);
    if (warp == 0) tmem_alloc(tmem_slot, NCOL);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
    uint32_t phase = 0;
    bool ok = true;
    const int tiles = D / MR, na = grp[2 * E + 1], n_items = na * tiles;
    const size_t rbd = (size_t)nb * BB;
    const int32_t *pairs = grp + 2 * E + 2;
    const uint32_t qh = qvec_bytes(nb);
    uint8_t *Arow = sm + Ahalf + (r >> 3) * 1024 + (r & 7) * 16;   // [16 groups][8 chunks][8 rows][16 B]
    const uint32_t As = saddr(sm + Ahalf), Xs = saddr(sm + P.X);
    const int KC = 16 * nb;
    auto issue_tile = [&](int item) {
        if (item < n_items) {
            const int ae = item / tiles, tile = item - ae * tiles, e = grp[E + 1 + ae];
            const uint8_t *src = slots[e].m[2] + (size_t)tile * MR * rbd;
            for (uint32_t i = r; i < tile_bytes / 16; i += DN_THREADS) cp16(sm + 16 * i, src + 16 * i);
        }
    };
    bool first = true;
    issue_tile(blockIdx.x);
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const int ae = item / tiles, tile = item - ae * tiles, e = grp[E + 1 + ae];
        const uint8_t *wt = sm + (size_t)r * rbd;
        for (int c0 = grp[e]; c0 < grp[e + 1] && ok; c0 += TN) {
            const int nt = min(TN, grp[e + 1] - c0);
            const bool last_pass = c0 + TN >= grp[e + 1];
            stage_tokens<DT, TN>(sm, P, hq, qh, 1, pairs + c0, nt, nb, first);
            cp_commit();
            cp_wait<0>();          // this item's tile and the pass's tokens
            first = false;
            __syncthreads();
            float acc[TN];
#pragma unroll
            for (int t = 0; t < TN; t++) acc[t] = 0.0f;
            for (int b = 0; b < nb && ok; b++) {
                RowBlk rk;
#pragma unroll 1
                for (int h = 0; h < 2; h++) {
                    // the half tile is free: every thread waited for the previous MMAs
                    rk = unpack_row<DT>(wt + b * BB, Arow - 8 * h * 128, h);
                    fence_async_smem();
                    __syncthreads();
                    if (last_pass && b == nb - 1 && h == 1) issue_tile(item + gridDim.x);   // raw tile consumed
                    if (r == 0) {
                        tc_fence_after();
                        if constexpr (DT == DT_Q6_K) {
#pragma unroll
                            for (int g = 0; g < 8; g++) {   // group 8h + g = chunk g of the half; B's second half: zero chunk
                                const int kc = 16 * b + 8 * h + g;
                                umma_i8(tmem + (uint32_t)((8 * h + g) * TN), umma_desc(As + g * 128u, 128u, 1024u),
                                        umma_desc(Xs + kc * 128u, (uint32_t)(KC - kc) * 128u, P.xsbo), idesc<TN>());
                            }
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; q++) {   // sub-block 4h + q = chunks 2q, 2q + 1 of the half
                                const int kc = 16 * b + 8 * h + 2 * q;
                                umma_i8(tmem + (uint32_t)((4 * h + q) * TN), umma_desc(As + 2 * q * 128u, 128u, 1024u),
                                        umma_desc(Xs + kc * 128u, 128u, P.xsbo), idesc<TN>());
                            }
                        }
                        umma_commit(reinterpret_cast<uint64_t *>(sm + P.bar));
                    }
                    const bool got = mbar_wait(reinterpret_cast<uint64_t *>(sm + P.bar), phase, WAIT_LIMIT);
                    phase ^= 1u;
                    if (__syncthreads_or(!got)) ok = false;   // uniform across the CTA
                    if (!ok) break;
                }
                if (!ok) break;
                tc_fence_after();
                int is[TN];
#pragma unroll
                for (int t = 0; t < TN; t++) is[t] = 0;
                add_scaled<DT, TN>(lane_base, 0u, 0, SUB, rk, is);
                chain_tokens<DT, TN>(sm, P, b, nb, rk, is, acc, nt);
                tc_fence_before();
            }
#pragma unroll
            for (int t = 0; t < TN; t++)
                if (t < nt) eo[(size_t)pairs[c0 + t] * D + tile * MR + r] = acc[t];
            __syncthreads();   // staged tokens are rewritten next
        }
    }
    cp_wait_all();   // a prefetched tile may still be in flight
    if (!ok) {
        mbar_wait(reinterpret_cast<uint64_t *>(sm + P.bar), phase ^ 1u, WAIT_LIMIT);   // the phase that expired
        report(err, false);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_free(tmem, NCOL);
}

}  // namespace

// ---------------------------------------------------------------------------
// Tokens per pass: NARROW_TN for decode-sized groups (small tiles, two CTAs
// per SM); when the experts average many tokens (prefill) the wider passes
// below, so that the unpack and the per-pass overheads are shared by more
// tokens.
constexpr int NARROW_TN = 8;
// Tokens per gate/up pass when the experts average many tokens (16 or 32).
// At 32 one CTA fits on an SM (177 registers, 180 KB of shared memory); at
// 16 the kernel takes two raw stages and two CTAs share an SM (113
// registers, 115 KB each). 2048-token prefill of 48 layers (B200, 16-token
// down passes): 18.6k tok/s with 32, 21.6k with 16.
#ifndef TLMG_GU_WIDE_TN
#define TLMG_GU_WIDE_TN 16
#endif
static_assert(TLMG_GU_WIDE_TN == 16 || TLMG_GU_WIDE_TN == 32, "gate/up pass width: 16 or 32 tokens");
static int gateup_stages(int D, int tn) { return tn <= 8 ? TLMG_MGU_NS8 : tn <= 16 ? 2 : D <= 2048 ? 3 : 2; }

static uint32_t gateup_smem(int dt, int D, int tn) {
    const uint32_t raw = (uint32_t)gateup_stages(D, tn) * MR * dt_block_bytes(dt);
    return tn <= 8    ? mplan<8>(1, raw, D / 256, true).total
           : tn <= 16 ? mplan<16>(1, raw, D / 256, true).total
                      : mplan<32>(1, raw, D / 256, true).total;
}
// Tokens per down pass when the experts average many tokens. 32 keeps one
// CTA per SM for Q6_K (16 groups x 32 TMEM columns, 127 KB of shared
// memory); 16 halves the TMEM columns and the staged token codes, so that
// two CTAs share an SM (110 KB each), at the price of twice the passes (each
// unpacks the tile again). 2048-token prefill of 48 layers (B200): 17.7k
// tok/s with 32, 18.7k with 16.
#ifndef TLMG_DN_WIDE_TN
#define TLMG_DN_WIDE_TN 16
#endif
static_assert(TLMG_DN_WIDE_TN == 16 || TLMG_DN_WIDE_TN == 32, "down pass width: 16 or 32 tokens");
static uint32_t down_smem(int dt, int de, int tn) {
    const uint32_t tile = align_up((uint32_t)MR * (de / 256) * dt_block_bytes(dt), 1024u) + MR * 128u;
    return tn <= 8    ? mplan<8>(0, tile, de / 256, false).total
           : tn <= 16 ? mplan<16>(0, tile, de / 256, false).total
                      : mplan<32>(0, tile, de / 256, false).total;
}
constexpr uint32_t SMEM_LIMIT = 227 * 1024;

bool mma_gateup_supported(int dt, int D, int de) {
    return (dt == DT_Q4_K || dt == DT_Q5_K) && D % 256 == 0 && D / 256 <= MAXNB && de % MR == 0 &&
           gateup_smem(dt, D, 8) <= SMEM_LIMIT;
}
bool mma_down_supported(int dt, int D, int de) {
    return (dt == DT_Q4_K || dt == DT_Q5_K || dt == DT_Q6_K) && de % 256 == 0 && de / 256 <= MAXNB && D % MR == 0 &&
           down_smem(dt, de, 8) <= SMEM_LIMIT;
}

template <typename F>
static int opt_in(F fn, uint32_t bytes) {
    static thread_local std::vector<std::pair<const void *, uint32_t>> done;
    for (auto &d : done)
        if (d.first == (const void *)fn && d.second >= bytes) return TLMG_OK;
    cudaError_t e = cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return cuda_fail(e, "tensor-core kernel shared memory");
    done.push_back({ (const void *)fn, bytes });
    return TLMG_OK;
}

static int grid_for(int64_t max_items, int per_sm) {
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    return (int)std::max<int64_t>(1, std::min<int64_t>(max_items, (int64_t)per_sm * nsm));
}

int launch_mma_gateup(int dt, const Slot *slots, const int32_t *grp, const uint8_t *x, size_t xstride, int xdiv,
                      int D, int de, int E, int64_t max_items, bool wide, float *gout, float *uout, uint32_t *err,
                      cudaStream_t st) {
    if (!mma_gateup_supported(dt, D, de)) return set_error(TLMG_EUNSUP, "tensor-core gate/up: dtype %d D %d", dt, D);
    int tn = wide ? TLMG_GU_WIDE_TN : NARROW_TN;
    if (gateup_smem(dt, D, tn) > SMEM_LIMIT) tn = 8;
    const uint32_t smem = gateup_smem(dt, D, tn);
    // CTAs per SM: as many as the kernel is compiled for and 228 KB of shared memory per SM hold
    const int per_sm = std::max(1, std::min<int>(tn <= 8 ? TLMG_MGU_MINB : 2, (int)(233472u / (smem + 1024u))));
    const int grid = grid_for(2 * max_items * (tn > NARROW_TN ? TLMG_GU_WIDE_PARTS : 1), per_sm);
    const bool three = gateup_stages(D, tn) == 3;
    using Fn = void (*)(const Slot *, const int32_t *, const uint8_t *, size_t, int, int, int, int, float *, float *,
                        uint32_t *);
    Fn fn;
    if (tn == 8)
        fn = dt == DT_Q4_K ? (three ? k_mgu<DT_Q4_K, 3, 8> : k_mgu<DT_Q4_K, 2, 8>)
                           : (three ? k_mgu<DT_Q5_K, 3, 8> : k_mgu<DT_Q5_K, 2, 8>);
    else
        fn = dt == DT_Q4_K ? (three ? k_mgu<DT_Q4_K, 3, TLMG_GU_WIDE_TN> : k_mgu<DT_Q4_K, 2, TLMG_GU_WIDE_TN>)
                           : (three ? k_mgu<DT_Q5_K, 3, TLMG_GU_WIDE_TN> : k_mgu<DT_Q5_K, 2, TLMG_GU_WIDE_TN>);
    int rc = opt_in(fn, smem);
    if (rc) return rc;
    cudaError_t e = launch_k(fn, grid, GU_THREADS, smem, st, slots, grp, x, xstride, xdiv, D, de, E, gout, uout, err);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "tensor-core gate/up launch");
}

int launch_mma_down(int dt, const Slot *slots, const int32_t *grp, const uint8_t *hq, int D, int de, int E,
                    int64_t max_items, bool wide, float *eo, uint32_t *err, cudaStream_t st) {
    if (!mma_down_supported(dt, D, de)) return set_error(TLMG_EUNSUP, "tensor-core down: dtype %d de %d", dt, de);
    int tn = wide ? TLMG_DN_WIDE_TN : NARROW_TN;
    if (down_smem(dt, de, tn) > SMEM_LIMIT) tn = 8;
    const uint32_t smem = down_smem(dt, de, tn);
    const int grid = grid_for(max_items, smem <= 113 * 1024 ? 2 : 1);
    using Fn = void (*)(const Slot *, const int32_t *, const uint8_t *, int, int, int, float *, uint32_t *);
    Fn fn;
    if (tn == 8)
        fn = dt == DT_Q4_K ? k_mdown<DT_Q4_K, 8> : dt == DT_Q5_K ? k_mdown<DT_Q5_K, 8> : k_mdown<DT_Q6_K, 8>;
    else
        fn = dt == DT_Q4_K ? k_mdown<DT_Q4_K, TLMG_DN_WIDE_TN>
             : dt == DT_Q5_K ? k_mdown<DT_Q5_K, TLMG_DN_WIDE_TN>
                             : k_mdown<DT_Q6_K, TLMG_DN_WIDE_TN>;
    int rc = opt_in(fn, smem);
    if (rc) return rc;
    cudaError_t e = launch_k(fn, grid, DN_THREADS, smem, st, slots, grp, hq, D, de, E, eo, err);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "tensor-core down launch");
}

}  // namespace tlmg
