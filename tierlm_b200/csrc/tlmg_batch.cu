// tlmg_batch.cu - batched expert FFN for n tokens of one MoE layer (batched
// decode, reference run_batch over several sequences, src/lib/tlm_model.c:
// 900-938 with the combine of :1029-1036 per token).
//
//   k_bquant    inputs x -> swizzled Q8_K vectors (one warp per block)
//   k_broute    router top-k per token (one warp per token, warp_route)
//   k_bgroup    (token, rank) pairs grouped by expert: offsets, the active
//               experts, the pair list (one CTA)
//   k_bgateup   per active expert and tile of 4 rows: every pair of the
//               expert, gate/up partials + chains + SwiGLU -> hbuf[pair]
//               (the expert's rows come from HBM once and from L1 for the
//               expert's other tokens)
//   k_bquant    h rows -> Q8_K per pair
//   k_bdown     per active expert and tile of 32 / nbd rows: every pair,
//               down partials + chain -> eo[pair]
//   k_bcombine  ffn[t] = sum_r w[t][r] * eo[t, r] in ascending rank
//
// Per pair the arithmetic is the single-token path's (exact int32 block
// partials, one fmaf per block (two for Q4_K/Q5_K) in block order, SiLU
// with the correctly rounded expf), so results are bit-identical to
// tlmg_expert_ffn on each token.
#include <algorithm>
#include <utility>
#include <vector>

#include "tlmg_batch.cuh"
#include "tlmg_dev.cuh"
#include "tlmg_internal.h"
#include "tlmg_kq.cuh"
#include "tlmg_mma.cuh"

namespace tlmg {

namespace {

constexpr int BMAXK = 16;
__host__ __device__ inline uint32_t up16b(uint32_t v) { return (v + 15u) & ~15u; }
__host__ __device__ inline uint32_t qvb(int nb) { return 256u * nb + 32u * nb + up16b(4u * nb); }

// rows x len floats -> rows quantised vectors of len / 256 blocks
__global__ void k_bquant(const float *__restrict__ in, int rows, int len, uint8_t *__restrict__ out) {
    pdl_enter();
    const int lane = threadIdx.x & 31, nb = len / 256;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
    const uint32_t qb = qvb(nb);
    for (int q = gw; q < rows * nb; q += nw) {
        const int r = q / nb, b = q - r * nb;
        const float4 *v = reinterpret_cast<const float4 *>(in + (size_t)r * len + 256 * b) + 2 * lane;
        uint8_t *base = out + (size_t)r * qb;
        warp_quant_swz(__ldg(v), __ldg(v + 1), base, nb, b, reinterpret_cast<int16_t *>(base + 256 * nb) + 16 * b,
                       reinterpret_cast<float *>(base + 288 * nb) + b, lane);
    }
}

// k_bquant of h = SiLU(g) * u formed on the fly (the tensor-core gate/up
// kernel leaves the gate and up dots in two arrays)
__global__ void k_bquant_swiglu(const float *__restrict__ g, const float *__restrict__ u, int rows, int len,
                                uint8_t *__restrict__ out) {
    pdl_enter();
    const int lane = threadIdx.x & 31, nb = len / 256;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
    const uint32_t qb = qvb(nb);
    for (int q = gw; q < rows * nb; q += nw) {
        const int r = q / nb, b = q - r * nb;
        const size_t off = (size_t)r * len + 256 * b + 8 * lane;
        const float4 g0 = __ldg(reinterpret_cast<const float4 *>(g + off)),
                     g1 = __ldg(reinterpret_cast<const float4 *>(g + off) + 1);
        const float4 u0 = __ldg(reinterpret_cast<const float4 *>(u + off)),
                     u1 = __ldg(reinterpret_cast<const float4 *>(u + off) + 1);
        const float4 h0 = make_float4(__fmul_rn(silu_f(g0.x), u0.x), __fmul_rn(silu_f(g0.y), u0.y),
                                      __fmul_rn(silu_f(g0.z), u0.z), __fmul_rn(silu_f(g0.w), u0.w));
        const float4 h1 = make_float4(__fmul_rn(silu_f(g1.x), u1.x), __fmul_rn(silu_f(g1.y), u1.y),
                                      __fmul_rn(silu_f(g1.z), u1.z), __fmul_rn(silu_f(g1.w), u1.w));
        uint8_t *base = out + (size_t)r * qb;
        warp_quant_swz(h0, h1, base, nb, b, reinterpret_cast<int16_t *>(base + 256 * nb) + 16 * b,
                       reinterpret_cast<float *>(base + 288 * nb) + b, lane);
    }
}

// one warp per token
constexpr int RW = 2;   // warps per CTA
__global__ void __launch_bounds__(32 * RW) k_broute(BatchArgs a, int32_t *__restrict__ ids, float *__restrict__ w) {
    pdl_enter();
    __shared__ uint32_t scr[RW][RT_SCRATCH];
    __shared__ int32_t sid[RW][64];
    __shared__ float sw[RW][64];
    const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * RW + wi;
    if (t >= a.n) return;
    warp_route(a.router, a.logits + (size_t)t * a.E, a.mask, a.bias, a.E, a.k, a.routed_scale, scr[wi], sid[wi],
               sw[wi], lane);
    if (lane < a.k) {
        ids[(size_t)t * a.k + lane] = sid[wi][lane];
        w[(size_t)t * a.k + lane] = sw[wi][lane];
        if (a.ids_out) a.ids_out[(size_t)t * a.k + lane] = sid[wi][lane];
        if (a.w_out) a.w_out[(size_t)t * a.k + lane] = sw[wi][lane];
    }
}

// grp: [0, E] expert offsets into the pair list, [E + 1, 2E] active experts
// in ascending id, [2E + 1] their count, [2E + 2, ..) the pairs t * k + r
// grouped by expert (in no particular order inside an expert: every pair's
// results are independent of the others)
// With rcnt, the records sit in regions of cap slots and record p exists
// only when p % cap < rcnt[p / cap]; the others are skipped.
__global__ void __launch_bounds__(1024) k_bgroup(const int32_t *__restrict__ ids, int istride, int np, int E,
                                                  int lo, int hi, int32_t *grp, float *eo, int D, int32_t *bad,
                                                  const int32_t *__restrict__ rcnt, int cap) {
    pdl_enter();
    __shared__ int cnt[RT_PER * 32], off[RT_PER * 32 + 1], fill[RT_PER * 32];
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        cnt[e] = 0;
        fill[e] = 0;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < np; p += blockDim.x) {
        if (rcnt && p % cap >= rcnt[p / cap]) continue;
        const int e = ids[(size_t)p * istride];
        if (e >= lo && e < hi) {
            atomicAdd(&cnt[e], 1);
        } else {
            // an expert outside [lo, hi): no weights here; the pair's output
            // row becomes NaN and the host is told
            atomicAdd(bad, 1);
            for (int i = 0; i < D; i++) eo[(size_t)p * D + i] = __int_as_float(0x7fc00000);
        }
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        // warp 0: lane l owns experts [l * per, (l + 1) * per); exclusive
        // scans of the pair counts and of the active-expert counts give the
        // offsets and the ascending active list
        const int lane = threadIdx.x, per = (E + 31) / 32, e0 = lane * per, e1 = min(E, e0 + per);
        int sum = 0, act = 0;
        for (int e = e0; e < e1; e++) {
            sum += cnt[e];
            act += cnt[e] != 0;
        }
        int xs = sum, xa = act;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int ys = __shfl_up_sync(0xffffffffu, xs, d), ya = __shfl_up_sync(0xffffffffu, xa, d);
            if (lane >= d) {
                xs += ys;
                xa += ya;
            }
        }
        int s = xs - sum, na = xa - act;
        for (int e = e0; e < e1; e++) {
            off[e] = s;
            s += cnt[e];
            if (cnt[e]) grp[E + 1 + na++] = e;
        }
        if (lane == 31) {
            off[E] = xs;
            grp[2 * E + 1] = xa;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e <= E; e += blockDim.x) grp[e] = off[e];
    for (int p = threadIdx.x; p < np; p += blockDim.x) {
        if (rcnt && p % cap >= rcnt[p / cap]) continue;
        const int e = ids[(size_t)p * istride];
        if (e >= lo && e < hi) grp[2 * E + 2 + off[e] + atomicAdd(&fill[e], 1)] = p;
    }
}

// Work item = (active expert, tile of 4 gate/up rows); one warp per item.
// Lane (p, j) = (lane / 8, lane % 8) owns row p of the tile and blocks
// j, j + 8, ... of the gate and up rows; for each pair of the expert it
// computes their exact partials against the pair's token, the chains run in
// block order (the holder of block b applies it, the accumulators are
// broadcast to the row's lanes by shuffle) and lane (p, 0) writes
// silu(gate) * up.
template <int DGU, int BPL>
__global__ void __launch_bounds__(256) k_bgateup(const Slot *__restrict__ slots, const int32_t *__restrict__ grp,
                                                 const uint8_t *__restrict__ xq, size_t xstride, int xdiv, int D,
                                                 int de, int E, float *__restrict__ hbuf) {
    const int lane = threadIdx.x & 31, p = lane >> 3, j = lane & 7;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
    const int nbx = D / 256, tiles = (de + 3) / 4, na = grp[2 * E + 1];
    const int rb = nbx * dt_block_bytes(DGU);
    for (int item = gw; item < na * tiles; item += nw) {
        const int ae = item / tiles, tile = item - ae * tiles, e = grp[E + 1 + ae];
        const int row = 4 * tile + p;
        const bool valid = row < de;
        const uint8_t *grow = slots[e].m[0] + (size_t)row * rb, *urow = slots[e].m[1] + (size_t)row * rb;
        for (int q = grp[e]; q < grp[e + 1]; q++) {
            const int pair = grp[2 * E + 2 + q];
            const uint8_t *xb = xq + (size_t)(pair / xdiv) * xstride;
            const int16_t *xbs = reinterpret_cast<const int16_t *>(xb + 256 * nbx);
            const float *xd = reinterpret_cast<const float *>(xb + 288 * nbx);
            BlockSum vg[BPL], vu[BPL];
#pragma unroll
            for (int i = 0; i < BPL; i++) {
                const int b = j + 8 * i;
                vg[i] = BlockSum{ 0, 0, 0.f, 0.f };
                vu[i] = vg[i];
                if (valid && b < nbx) {
                    const uint8_t *wb[2] = { grow + b * dt_block_bytes(DGU), urow + b * dt_block_bytes(DGU) };
                    BlockSum o2[2];
                    kblock_dot<DGU, 2>(wb, XBlk{ xb, nbx, b, xbs + 16 * b, xd[b] }, o2);
                    vg[i] = o2[0];
                    vu[i] = o2[1];
                }
            }
            float ag = 0.0f, au = 0.0f;
            const int base = lane & ~7;
#pragma unroll
            for (int i = 0; i < BPL; i++)
#pragma unroll
                for (int h = 0; h < 8; h++) {
                    if (h + 8 * i >= nbx) break;
                    if (j == h) {
                        ag = chain<DGU>(ag, vg[i].dA, vg[i].is, vg[i].dM, vg[i].ms);
                        au = chain<DGU>(au, vu[i].dA, vu[i].is, vu[i].dM, vu[i].ms);
                    }
                    ag = __shfl_sync(0xFFFFFFFFu, ag, base | h);
                    au = __shfl_sync(0xFFFFFFFFu, au, base | h);
                }
            if (j == 0 && valid) hbuf[(size_t)pair * de + row] = __fmul_rn(silu_f(ag), au);
        }
    }
}

// Work item = (active expert, tile of 32 / nbd down rows); one warp per
// item. Lane (g, b) = (lane / nbd, lane % nbd) owns block b of row g; per
// pair of the expert: exact partials against the pair's quantised h, then
// the row's chain in block order, lane (g, 0) writes eo[pair][row].
template <int DDN>
__global__ void __launch_bounds__(256) k_bdown(const Slot *__restrict__ slots, const int32_t *__restrict__ grp,
                                               const uint8_t *__restrict__ hq, int D, int de, int E,
                                               float *__restrict__ eo) {
    const int lane = threadIdx.x & 31, nbd = de / 256, rpt = 32 / nbd;
    const int g = lane / nbd, b = lane - g * nbd;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
    const int tiles = (D + rpt - 1) / rpt, na = grp[2 * E + 1];
    const uint32_t qh = qvb(nbd);
    const int rb = nbd * dt_block_bytes(DDN);
    const int gb = g < rpt ? g * nbd : 0;
    for (int item = gw; item < na * tiles; item += nw) {
        const int ae = item / tiles, tile = item - ae * tiles, e = grp[E + 1 + ae];
        const int row = rpt * tile + g;
        const bool valid = g < rpt && row < D;
        const uint8_t *wrow = slots[e].m[2] + (size_t)row * rb;
        for (int q = grp[e]; q < grp[e + 1]; q++) {
            const int pair = grp[2 * E + 2 + q];
            const uint8_t *hb = hq + (size_t)pair * qh;
            BlockSum v = BlockSum{ 0, 0, 0.f, 0.f };
            if (valid) {
                const uint8_t *wb[1] = { wrow + b * dt_block_bytes(DDN) };
                BlockSum o1[1];
                kblock_dot<DDN, 1>(wb,
                                   XBlk{ hb, nbd, b, reinterpret_cast<const int16_t *>(hb + 256 * nbd) + 16 * b,
                                         reinterpret_cast<const float *>(hb + 288 * nbd)[b] },
                                   o1);
                v = o1[0];
            }
            float acc = 0.0f;
            for (int h = 0; h < nbd; h++) {
                if (b == h) acc = chain<DDN>(acc, v.dA, v.is, v.dM, v.ms);
                acc = __shfl_sync(0xFFFFFFFFu, acc, gb + h);
            }
            if (b == 0 && valid) eo[(size_t)pair * D + row] = acc;
        }
    }
}

// ffn[t][i] = sum_r w[t][r] * eo[row(t, r)][i] in ascending r, row(t, r) =
// perm[t * k + r] when perm is given, else t * k + r
__global__ void k_bcombine(const float *__restrict__ eo, const int32_t *__restrict__ perm, const float *__restrict__ w,
                           int n, int D, int k, float *__restrict__ ffn) {
    pdl_enter();
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n * D; idx += gridDim.x * blockDim.x) {
        const int t = idx / D, i = idx - t * D;
        float f = 0.0f;
        // ranks in groups of 8: the group's loads are issued together, then
        // the products are added in ascending rank as before
        for (int r0 = 0; r0 < k; r0 += 8) {
            float wv[8], ev[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int r = r0 + j;
                if (r < k) {
                    const int row = perm ? perm[t * k + r] : t * k + r;
                    wv[j] = w[(size_t)t * k + r];
                    ev[j] = eo[(size_t)row * D + i];
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (r0 + j < k) f = __fadd_rn(f, __fmul_rn(wv[j], ev[j]));
        }
        ffn[idx] = f;
    }
}

// Expert-parallel dispatch layout. Pair p = t * k + r goes to the GPU owning
// expert ids[p], owner(e) = floor(e * nr / E); records are grouped by owner,
// inside an owner in ascending pair order. perm[p] = the pair's record index,
// cnt[d] = records for owner d.
// counts (int32, the dispatch's pinned words) -> int64 device counts
__global__ void k_epcount64(const int32_t *__restrict__ cnt, int nr, int64_t *__restrict__ out) {
    for (int d = threadIdx.x; d < nr; d += blockDim.x) out[d] = cnt[d];
}

__global__ void __launch_bounds__(1024) k_epcount(const int32_t *__restrict__ ids, int np, int E, int nr,
                                                   int32_t *__restrict__ perm, int32_t *__restrict__ cnt) {
    __shared__ int tot[EP_MAX_RANKS], base[EP_MAX_RANKS], wsum[32];
    const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    for (int d = threadIdx.x; d < nr; d += blockDim.x) tot[d] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < np; p += blockDim.x) atomicAdd(&tot[(int)((int64_t)ids[p] * nr / E)], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0;
        for (int d = 0; d < nr; d++) {
            base[d] = s;
            cnt[d] = tot[d];
            s += tot[d];
        }
    }
    __syncthreads();
    for (int c0 = 0; c0 < np; c0 += blockDim.x) {
        const int p = c0 + threadIdx.x;
        const int me = p < np ? (int)((int64_t)ids[p] * nr / E) : -1;
        for (int d = 0; d < nr; d++) {
            const unsigned m = __ballot_sync(0xFFFFFFFFu, me == d);
            if (lane == 0) wsum[wi] = __popc(m);
            __syncthreads();
            if (me == d) {
                int before = 0;
                for (int v = 0; v < wi; v++) before += wsum[v];
                perm[p] = base[d] + before + __popc(m & ((1u << lane) - 1u));
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                int s = 0;
                for (int v = 0; v < nwarp; v++) s += wsum[v];
                base[d] += s;
            }
            __syncthreads();
        }
    }
}

// One warp per pair: record perm[p] = { int32 expert id, 12 zero bytes,
// the token's quantised vector (qx bytes) }.
__global__ void k_eppack(const int32_t *__restrict__ ids, const int32_t *__restrict__ perm, int np, int k,
                         const uint8_t *__restrict__ xq, uint32_t qx, uint8_t *__restrict__ send, size_t rec) {
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
    for (int p = gw; p < np; p += nw) {
        uint8_t *dst = send + (size_t)perm[p] * rec;
        const uint4 *src = reinterpret_cast<const uint4 *>(xq + (size_t)(p / k) * qx);
        if (lane == 0) *reinterpret_cast<uint4 *>(dst) = make_uint4((uint32_t)ids[p], 0u, 0u, 0u);
        for (uint32_t i = lane; i < qx / 16; i += 32) reinterpret_cast<uint4 *>(dst + 16)[i] = __ldg(src + i);
    }
}

// ---------------------------------------------------------------------------
// Tiled expert kernels: one CTA works on a tile of TR rows of one expert for
// all of the expert's tokens (up to TC per pass). Thread (row, tq) owns one
// weight row and the tokens tq, tq + TQ, ...; it walks the row's blocks in
// ascending order, so every (row, token) chain stays in one thread (no
// shuffles) and each weight byte is read from HBM once per pass. Weights are
// staged with cp.async into shared memory; the tokens' quantised inputs are
// staged once per pass and read by all rows as broadcasts.

constexpr int TR = 64;              // rows per tile
constexpr int TQ = 4;               // token lanes per row: 256 threads
constexpr int TC = 16;              // tokens per pass
constexpr int TPT = TC / TQ;        // tokens per thread per pass
constexpr int NSG = 4;              // gate/up block-column stages

template <int DT> constexpr int bbytes() { return DT == DT_Q4_K ? 144 : DT == DT_Q5_K ? 176 : 210; }

__device__ __forceinline__ void cp16(void *dst, const void *src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// copy n16 16-byte pieces src -> dst with all threads of the CTA
__device__ __forceinline__ void cp_span(uint8_t *dst, const uint8_t *src, int n16) {
    for (int i = threadIdx.x; i < n16; i += blockDim.x) cp16(dst + 16 * i, src + 16 * i);
}

__device__ __forceinline__ XBlk xblk_at(const uint8_t *v, int nb, int b) {
    return XBlk{ v, nb, b, reinterpret_cast<const int16_t *>(v + 256 * nb) + 16 * b,
                 reinterpret_cast<const float *>(v + 288 * nb)[b] };
}

// gate/up of Q4_K / Q5_K (16-byte aligned blocks): block column b of the
// tile's gate and up rows is staged as [2][TR][BB] (row stride BB = 9 or 11
// 16-byte units, odd, so the rows' 16-byte loads are free of bank conflicts).
template <int DGU>
__global__ void __launch_bounds__(TR * TQ, 2)
    k_tgateup(const Slot *__restrict__ slots, const int32_t *__restrict__ grp, const uint8_t *__restrict__ x,
              size_t xstride, int xdiv, int D, int de, int E, float *__restrict__ hbuf) {
    extern __shared__ __align__(128) uint8_t sm[];
    constexpr int BB = bbytes<DGU>(), CPB = BB / 16;
    const int nbx = D / 256;
    const uint32_t qx = qvb(nbx);
    uint8_t *sw = sm, *sx = sm + NSG * 2 * TR * BB;
    const int tid = threadIdx.x, row = tid % TR, tq = tid / TR;
    const int tiles = de / TR, na = grp[2 * E + 1];
    const size_t rb = (size_t)nbx * BB;
    const int32_t *pairs = grp + 2 * E + 2;
    for (int item = blockIdx.x; item < na * tiles; item += gridDim.x) {
        const int ae = item / tiles, tile = item - ae * tiles, e = grp[E + 1 + ae];
        const uint8_t *wsg = slots[e].m[0] + (size_t)tile * TR * rb, *wsu = slots[e].m[1] + (size_t)tile * TR * rb;
        auto issue = [&](int b) {
            if (b < nbx) {
                uint8_t *st = sw + (b % NSG) * 2 * TR * BB;
                for (int i = tid; i < 2 * TR * CPB; i += TR * TQ) {
                    const int m = i / (TR * CPB), r = (i / CPB) % TR, c = i % CPB;
                    cp16(st + (m * TR + r) * BB + 16 * c, (m ? wsu : wsg) + r * rb + (size_t)b * BB + 16 * c);
                }
            }
            cp_commit();
        };
        for (int c0 = grp[e]; c0 < grp[e + 1]; c0 += TC) {
            const int nt = min(TC, grp[e + 1] - c0);
            for (int t = 0; t < nt; t++) cp_span(sx + t * qx, x + (size_t)(pairs[c0 + t] / xdiv) * xstride, qx / 16);
#pragma unroll
            for (int b = 0; b < NSG - 1; b++) issue(b);
            float ag[TPT], au[TPT];
#pragma unroll
            for (int i = 0; i < TPT; i++) ag[i] = au[i] = 0.0f;
            for (int b = 0; b < nbx; b++) {
                cp_wait<NSG - 2>();
                __syncthreads();
                issue(b + NSG - 1);
                const uint8_t *st = sw + (b % NSG) * 2 * TR * BB;
                const uint8_t *w2[2] = { st + row * BB, st + (TR + row) * BB };
#pragma unroll
                for (int i = 0; i < TPT; i++) {
                    const int t = tq + TQ * i;
                    if (t < nt) {
                        BlockSum o[2];
                        kblock_dot<DGU, 2>(w2, xblk_at(sx + t * qx, nbx, b), o);
                        ag[i] = chain<DGU>(ag[i], o[0].dA, o[0].is, o[0].dM, o[0].ms);
                        au[i] = chain<DGU>(au[i], o[1].dA, o[1].is, o[1].dM, o[1].ms);
                    }
                }
            }
            cp_wait<0>();
            __syncthreads();   // stages and staged inputs are rewritten next
#pragma unroll
            for (int i = 0; i < TPT; i++) {
                const int t = tq + TQ * i;
                if (t < nt) hbuf[(size_t)pairs[c0 + t] * de + tile * TR + row] = __fmul_rn(silu_f(ag[i]), au[i]);
            }
        }
    }
}

// down: the tile's TR rows (all nbd blocks, contiguous in HBM) are staged
// once per tile; the expert's quantised h rows are staged per pass of TC.
template <int DDN>
__global__ void __launch_bounds__(TR * TQ, 2)
    k_tdown(const Slot *__restrict__ slots, const int32_t *__restrict__ grp, const uint8_t *__restrict__ hq, int D,
            int de, int E, float *__restrict__ eo) {
    extern __shared__ __align__(128) uint8_t sm[];
    constexpr int BB = bbytes<DDN>();
    const int nbd = de / 256;
    const uint32_t qh = qvb(nbd);
    const int rbd = nbd * BB;
    const int wtile = up16b((uint32_t)(TR * rbd));
    uint8_t *sw = sm, *sx = sm + wtile;
    const int tid = threadIdx.x, row = tid % TR, tq = tid / TR;
    const int tiles = D / TR, na = grp[2 * E + 1];
    const int32_t *pairs = grp + 2 * E + 2;
    for (int item = blockIdx.x; item < na * tiles; item += gridDim.x) {
        const int ae = item / tiles, tile = item - ae * tiles, e = grp[E + 1 + ae];
        cp_span(sw, slots[e].m[2] + (size_t)tile * TR * rbd, TR * rbd / 16);
        for (int c0 = grp[e]; c0 < grp[e + 1]; c0 += TC) {
            const int nt = min(TC, grp[e + 1] - c0);
            for (int t = 0; t < nt; t++) cp_span(sx + t * qh, hq + (size_t)pairs[c0 + t] * qh, qh / 16);
            cp_commit();
            cp_wait<0>();
            __syncthreads();
            const uint8_t *w1[1] = { sw + row * rbd };
            float acc[TPT];
#pragma unroll
            for (int i = 0; i < TPT; i++) acc[i] = 0.0f;
            for (int b = 0; b < nbd; b++) {
                const uint8_t *wb[1] = { w1[0] + b * BB };
#pragma unroll
                for (int i = 0; i < TPT; i++) {
                    const int t = tq + TQ * i;
                    if (t < nt) {
                        BlockSum o[1];
                        kblock_dot<DDN, 1>(wb, xblk_at(sx + t * qh, nbd, b), o);
                        acc[i] = chain<DDN>(acc[i], o[0].dA, o[0].is, o[0].dM, o[0].ms);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < TPT; i++) {
                const int t = tq + TQ * i;
                if (t < nt) eo[(size_t)pairs[c0 + t] * D + tile * TR + row] = acc[i];
            }
            __syncthreads();   // staged h rows (and, after the last pass, the tile) are rewritten next
        }
    }
}

}  // namespace

using GateUpFn = void (*)(const Slot *, const int32_t *, const uint8_t *, size_t, int, int, int, int, float *);
using DownFn = void (*)(const Slot *, const int32_t *, const uint8_t *, int, int, int, float *);

static GateUpFn pick_gateup(int dt, int D) {
    const bool two = D > 2048;
    switch (dt) {
    case DT_Q4_K: return two ? k_bgateup<DT_Q4_K, 2> : k_bgateup<DT_Q4_K, 1>;
    case DT_Q5_K: return two ? k_bgateup<DT_Q5_K, 2> : k_bgateup<DT_Q5_K, 1>;
    case DT_Q6_K: return two ? k_bgateup<DT_Q6_K, 2> : k_bgateup<DT_Q6_K, 1>;
    default: return nullptr;
    }
}
static DownFn pick_down(int dt) {
    switch (dt) {
    case DT_Q4_K: return k_bdown<DT_Q4_K>;
    case DT_Q5_K: return k_bdown<DT_Q5_K>;
    case DT_Q6_K: return k_bdown<DT_Q6_K>;
    default: return nullptr;
    }
}

bool batch_supported(int dt_gu, int dt_dn, int D, int de, int E, int k) {
    return pick_gateup(dt_gu, D) && pick_down(dt_dn) && D % 256 == 0 && de % 256 == 0 && D <= 4096 &&
           de / 256 <= 32 && E > 0 && E <= RT_PER * 32 && k > 0 && k <= BMAXK && k <= E;
}

size_t ep_record_bytes(int D) { return 16 + qvb(D / 256); }

void batch_release(BatchScratch &s) {
    const int kmode = s.kmode, kmode_dn = s.kmode_dn;
    for (void *p : { (void *)s.xq, (void *)s.ids, (void *)s.w, (void *)s.grp, (void *)s.hbuf, (void *)s.ubuf,
                     (void *)s.hq, (void *)s.eo })
        if (p) cudaFree(p);
    if (s.cnt) cudaFreeHost(s.cnt);
    s = BatchScratch{};
    s.kmode = kmode;
    s.kmode_dn = kmode_dn;
}

// Grows the scratch to hold n_tok tokens and n_pairs (token, expert) pairs.
static int reserve(BatchScratch &s, int n_tok, int64_t n_pairs, int D, int de, int E) {
    if (n_tok <= s.cap && n_pairs <= s.cap_pairs && E <= s.cap_e) return TLMG_OK;
    const int cap = std::max({ n_tok, s.cap, 16 });
    const int64_t np = std::max<int64_t>({ n_pairs, s.cap_pairs, 64 });
    const int ce = std::max(E, s.cap_e);
    batch_release(s);
    if (cudaMalloc(&s.xq, (size_t)cap * qvb(D / 256)) != cudaSuccess || cudaMalloc(&s.ids, 4 * np) != cudaSuccess ||
        cudaMalloc(&s.w, 4 * np) != cudaSuccess || cudaMalloc(&s.grp, 4 * (2 * (size_t)ce + 2 + np)) != cudaSuccess ||
        cudaMalloc(&s.hbuf, 4 * np * de) != cudaSuccess || cudaMalloc(&s.ubuf, 4 * np * de) != cudaSuccess ||
        cudaMalloc(&s.hq, np * qvb(de / 256)) != cudaSuccess ||
        cudaMalloc(&s.eo, 4 * np * D) != cudaSuccess || cudaMallocHost(&s.cnt, 4 * (EP_MAX_RANKS + 2)) != cudaSuccess) {
        cudaGetLastError();
        batch_release(s);
        return set_error(TLMG_ENOMEM, "batched expert FFN scratch for %d tokens / %lld pairs", n_tok,
                         (long long)n_pairs);
    }
    s.cnt[EP_MAX_RANKS] = 0;
    s.cnt[EP_MAX_RANKS + 1] = 0;
    s.cap = cap;
    s.cap_pairs = np;
    s.cap_e = ce;
    return TLMG_OK;
}

int batch_reserve(BatchScratch &s, int n, int D, int de, int E, int k) {
    return reserve(s, n, (int64_t)n * k, D, de, E);
}

static int sm_count() {
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    return nsm;
}

static unsigned warp_blocks(int64_t warps, int nsm) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, 8 * (int64_t)nsm));
}

// The expert stage shared by batched decode and the expert-parallel owner:
// np pairs, pair q's expert id at ids[q * istride] and its quantised input at
// x + (q / xdiv) * xstride -> eo[q] (f32 [D]).
using TGateUpFn = void (*)(const Slot *, const int32_t *, const uint8_t *, size_t, int, int, int, int, float *);
using TDownFn = void (*)(const Slot *, const int32_t *, const uint8_t *, int, int, int, float *);

static TGateUpFn pick_tgateup(int dt) {
    return dt == DT_Q4_K ? k_tgateup<DT_Q4_K> : dt == DT_Q5_K ? k_tgateup<DT_Q5_K> : nullptr;
}
static TDownFn pick_tdown(int dt) {
    return dt == DT_Q4_K ? k_tdown<DT_Q4_K> : dt == DT_Q5_K ? k_tdown<DT_Q5_K> : dt == DT_Q6_K ? k_tdown<DT_Q6_K>
                                                                                            : nullptr;
}
static size_t tgateup_smem(int dt, int D) {
    return (size_t)NSG * 2 * TR * dt_block_bytes(dt) + (size_t)TC * qvb(D / 256);
}
static size_t tdown_smem(int dt, int de) {
    return up16b((uint32_t)(TR * (de / 256) * dt_block_bytes(dt))) + (size_t)TC * qvb(de / 256);
}
constexpr size_t SMEM_MAX = 227 * 1024;

// Opts a kernel into `bytes` of dynamic shared memory (once per size).
template <typename F>
static bool smem_opt_in(F fn, size_t bytes) {
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

// The expert stage shared by batched decode and the expert-parallel owner:
// np pairs, pair q's expert id at ids[q * istride] and its quantised input at
// x + (q / xdiv) * xstride -> eo[q] (f32 [D]).
static int expert_stage(BatchScratch &s, const Slot *slots, int dt_gu, int dt_dn, int D, int de, int E, int lo,
                         int hi, const int32_t *ids, int istride, int64_t np, const uint8_t *x, size_t xstride,
                         int xdiv, float *eo, cudaStream_t st, const int32_t *rcnt = nullptr, int cap = 0) {
    const int nsm = sm_count();
    launch_k(k_bgroup, 1, 1024, 0, st, ids, istride, (int)np, E, lo, hi, s.grp, eo, D, s.cnt + EP_MAX_RANKS, rcnt, cap);
    // at most min(np, E) experts are active
    const int64_t na_max = std::min<int64_t>(np, E);
    const size_t sgu = tgateup_smem(dt_gu, D), sdn = tdown_smem(dt_dn, de);
    uint32_t *err = reinterpret_cast<uint32_t *>(s.cnt + EP_MAX_RANKS + 1);
    TGateUpFn tgu = s.kmode >= 1 ? pick_tgateup(dt_gu) : nullptr;
    const bool mma_gu = s.kmode >= 2 && mma_gateup_supported(dt_gu, D, de);
    const bool wide = np >= 24 * na_max;   // >= 24 tokens per expert on average
    if (mma_gu) {
        int rc = launch_mma_gateup(dt_gu, slots, s.grp, x, xstride, xdiv, D, de, E, na_max * (de / 128), wide,
                                   s.hbuf, s.ubuf, err, st);
        if (rc) return rc;
    } else if (tgu && sgu <= SMEM_MAX && smem_opt_in(tgu, sgu)) {
        const int64_t items = na_max * (de / TR);
        tgu<<<(unsigned)std::min<int64_t>(items, 2 * (int64_t)nsm), TR * TQ, sgu, st>>>(slots, s.grp, x, xstride,
                                                                                         xdiv, D, de, E, s.hbuf);
    } else {
        // one warp per (expert, tile of 4 rows)
        pick_gateup(dt_gu, D)<<<warp_blocks(na_max * ((de + 3) / 4), nsm), 256, 0, st>>>(slots, s.grp, x, xstride,
                                                                                        xdiv, D, de, E, s.hbuf);
    }
    if (mma_gu)
        launch_k(k_bquant_swiglu, warp_blocks(np * (de / 256), nsm), 256, 0, st, (const float *)s.hbuf,
                 (const float *)s.ubuf, (int)np, de, s.hq);
    else
        launch_k(k_bquant, warp_blocks(np * (de / 256), nsm), 256, 0, st, (const float *)s.hbuf, (int)np, de, s.hq);
    TDownFn tdn = s.kmode_dn >= 1 ? pick_tdown(dt_dn) : nullptr;
    if (s.kmode_dn >= 2 && mma_down_supported(dt_dn, D, de)) {
        int rc = launch_mma_down(dt_dn, slots, s.grp, s.hq, D, de, E, na_max * (D / 128), wide, eo, err, st);
        if (rc) return rc;
    } else if (tdn && sdn <= SMEM_MAX && smem_opt_in(tdn, sdn)) {
        const int64_t items = na_max * (D / TR);
        tdn<<<(unsigned)std::min<int64_t>(items, 3 * (int64_t)nsm), TR * TQ, sdn, st>>>(slots, s.grp, s.hq, D, de, E,
                                                                                        eo);
    } else {
        const int rpt = 32 / (de / 256);
        pick_down(dt_dn)<<<warp_blocks(na_max * ((D + rpt - 1) / rpt), nsm), 256, 0, st>>>(slots, s.grp, s.hq, D, de,
                                                                                          E, eo);
    }
    count_launch(4);
    return TLMG_OK;
}

static unsigned combine_blocks(int n, int D) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(((int64_t)n * D + 255) / 256, 4 * (int64_t)sm_count()));
}

int launch_batch(BatchScratch &s, const BatchArgs &a, cudaStream_t st) {
    if (!batch_supported(a.dt_gu, a.dt_dn, a.D, a.de, a.E, a.k))
        return set_error(TLMG_EUNSUP, "batched expert FFN: dtypes %d/%d or shape unsupported", a.dt_gu, a.dt_dn);
    if (a.n <= 0) return TLMG_OK;
    int rc = batch_reserve(s, a.n, a.D, a.de, a.E, a.k);
    if (rc) return rc;
    const int np = a.n * a.k, nsm = sm_count();
    // the seven kernels of the call as programmatic dependents of each other
    // (each waits in griddepcontrol.wait before it reads its inputs)
    struct PdlScope {
        bool prev = pdl_on();
        PdlScope() { set_pdl(true); }
        ~PdlScope() { set_pdl(prev); }
    } pdl_scope;
    launch_k(k_bquant, warp_blocks((int64_t)a.n * (a.D / 256), nsm), 256, 0, st, a.x, a.n, a.D, s.xq);
    launch_k(k_broute, (a.n + RW - 1) / RW, 32 * RW, 0, st, a, s.ids, s.w);
    count_launch(2);
    if ((rc = expert_stage(s, a.slots, a.dt_gu, a.dt_dn, a.D, a.de, a.E, 0, a.E, s.ids, 1, np, s.xq, qvb(a.D / 256),
                           a.k, s.eo, st)))
        return rc;
    launch_k(k_bcombine, combine_blocks(a.n, a.D), 256, 0, st, (const float *)s.eo, (const int32_t *)nullptr,
             (const float *)s.w, a.n, a.D, a.k, a.ffn);
    count_launch(1);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "batched expert FFN launch");
}

int ep_dispatch(BatchScratch &s, const BatchArgs &a, int nr, uint8_t *send, int32_t *perm, float *w, int64_t *counts,
                cudaStream_t st) {
    if (!batch_supported(a.dt_gu, a.dt_dn, a.D, a.de, a.E, a.k))
        return set_error(TLMG_EUNSUP, "expert-parallel dispatch: dtypes %d/%d or shape unsupported", a.dt_gu, a.dt_dn);
    if (nr < 1 || nr > EP_MAX_RANKS || nr > a.E)
        return set_error(TLMG_EINVAL, "expert-parallel dispatch: %d ranks (1..%d, at most E)", nr, EP_MAX_RANKS);
    const bool dev_counts = is_device_ptr(counts);
    if (a.n <= 0) {
        if (dev_counts) {
            cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(int64_t) * (size_t)nr, st);
            if (e != cudaSuccess) return cuda_fail(e, "expert-parallel dispatch");
        } else {
            for (int d = 0; d < nr; d++) counts[d] = 0;
        }
        return TLMG_OK;
    }
    int rc = batch_reserve(s, a.n, a.D, a.de, a.E, a.k);
    if (rc) return rc;
    const int np = a.n * a.k, nsm = sm_count();
    const uint32_t qx = qvb(a.D / 256);
    BatchArgs r = a;
    r.w_out = w;
    k_bquant<<<warp_blocks((int64_t)a.n * (a.D / 256), nsm), 256, 0, st>>>(a.x, a.n, a.D, s.xq);
    k_broute<<<(a.n + RW - 1) / RW, 32 * RW, 0, st>>>(r, s.ids, s.w);
    k_epcount<<<1, 1024, 0, st>>>(s.ids, np, a.E, nr, perm, s.cnt);
    k_eppack<<<warp_blocks(np, nsm), 256, 0, st>>>(s.ids, perm, np, a.k, s.xq, qx, send, ep_record_bytes(a.D));
    count_launch(4);
    if (dev_counts) {
        // device counts: written on the stream, no wait (the caller's
        // exchange of the counts is ordered after them on the same stream)
        k_epcount64<<<1, 32, 0, st>>>(s.cnt, nr, counts);
        count_launch(1);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "expert-parallel dispatch");
        return TLMG_OK;
    }
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);    // the record counts size the exchange
    if (e != cudaSuccess) return cuda_fail(e, "expert-parallel dispatch");
    for (int d = 0; d < nr; d++) counts[d] = s.cnt[d];
    return batch_take_error(s);
}

int ep_experts(BatchScratch &s, const Slot *slots, int dt_gu, int dt_dn, int D, int de, int E, int lo, int hi,
               int64_t n_rec, const uint8_t *recv, float *eo, cudaStream_t st) {
    if (!batch_supported(dt_gu, dt_dn, D, de, E, 1))
        return set_error(TLMG_EUNSUP, "expert-parallel experts: dtypes %d/%d or shape unsupported", dt_gu, dt_dn);
    if (n_rec <= 0) return TLMG_OK;
    if (n_rec > INT32_MAX / 2) return set_error(TLMG_EINVAL, "expert-parallel experts: %lld records", (long long)n_rec);
    int rc = reserve(s, 1, n_rec, D, de, E);
    if (rc) return rc;
    const size_t rec = ep_record_bytes(D);
    if ((rc = expert_stage(s, slots, dt_gu, dt_dn, D, de, E, lo, hi, reinterpret_cast<const int32_t *>(recv),
                           (int)(rec / 4), n_rec, recv + 16, rec, 1, eo, st)))
        return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "expert-parallel expert launch");
}

int batch_take_error(BatchScratch &s) {
    if (!s.cnt) return TLMG_OK;
    if (s.cnt[EP_MAX_RANKS + 1]) {
        s.cnt[EP_MAX_RANKS + 1] = 0;
        return set_error(TLMG_EIO, "batched expert kernel gave up waiting for its tensor-core MMAs; results of this "
                                   "call are invalid");
    }
    if (s.cnt[EP_MAX_RANKS] == 0) return TLMG_OK;
    const int n = s.cnt[EP_MAX_RANKS];
    s.cnt[EP_MAX_RANKS] = 0;
    return set_error(TLMG_EINVAL, "expert parallel: %d received records named experts this GPU does not own "
                                  "(their output rows are NaN)", n);
}

int ep_combine(int n, int D, int k, const float *back, const int32_t *perm, const float *w, float *ffn,
               cudaStream_t st) {
    if (n <= 0) return TLMG_OK;
    k_bcombine<<<combine_blocks(n, D), 256, 0, st>>>(back, perm, w, n, D, k, ffn);
    count_launch(1);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "expert-parallel combine launch");
}

int epp_layer(BatchScratch &s, EpP2P &e, const BatchArgs &a, int lo, int hi, cudaStream_t st) {
    if (!batch_supported(a.dt_gu, a.dt_dn, a.D, a.de, a.E, a.k))
        return set_error(TLMG_EUNSUP, "expert-parallel layer: dtypes %d/%d or shape unsupported", a.dt_gu, a.dt_dn);
    if (!e.base || e.nr > a.E) return set_error(TLMG_EINVAL, "expert-parallel layer: exchange not open");
    for (int r = 0; r < e.nr; r++)
        if (!e.peer[r]) return set_error(TLMG_EINVAL, "expert-parallel layer: rank %d not connected", r);
    if (a.n < 0 || a.n > e.max_tok || (int64_t)a.n * a.k > e.cap || ep_record_bytes(a.D) != e.rb)
        return set_error(TLMG_EINVAL, "expert-parallel layer: %d tokens (exchange sized for %d)", a.n, e.max_tok);
    int rc = reserve(s, std::max(a.n, 1), (int64_t)e.nr * e.cap, a.D, a.de, a.E);
    if (rc) return rc;
    const int np = a.n * a.k, nsm = sm_count();
    const uint32_t qx = qvb(a.D / 256);
    e.epoch++;
    if (a.n > 0) {
        k_bquant<<<warp_blocks((int64_t)a.n * (a.D / 256), nsm), 256, 0, st>>>(a.x, a.n, a.D, s.xq);
        k_broute<<<(a.n + RW - 1) / RW, 32 * RW, 0, st>>>(a, s.ids, s.w);
        count_launch(2);
    }
    k_epcount<<<1, 1024, 0, st>>>(s.ids, np, a.E, e.nr, e.perm, e.cnt);
    epp_send(e, s.ids, np, a.k, a.E, s.xq, qx, st);
    epp_barrier(e, 0, st);
    count_launch(3);
    const int32_t *rcnt = reinterpret_cast<const int32_t *>(e.base + e.off_rcnt);
    if ((rc = expert_stage(s, a.slots, a.dt_gu, a.dt_dn, a.D, a.de, a.E, lo, hi, reinterpret_cast<const int32_t *>(e.base),
                           (int)(e.rb / 4), (int64_t)e.nr * e.cap, e.base + 16, e.rb, 1, e.eo, st, rcnt, e.cap)))
        return rc;
    epp_return(e, a.D, st);
    epp_barrier(e, 1, st);
    count_launch(2);
    if (a.n > 0) {
        const float *back = reinterpret_cast<const float *>(e.base + e.off_back);
        k_bcombine<<<combine_blocks(a.n, a.D), 256, 0, st>>>(back, e.slot_of, s.w, a.n, a.D, a.k, a.ffn);
        count_launch(1);
    }
    cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? TLMG_OK : cuda_fail(err, "expert-parallel layer launch");
}

int epp_take_error(BatchScratch &s, EpP2P &e) {
    if (e.err_host && *reinterpret_cast<volatile uint32_t *>(e.err_host))
        return set_error(TLMG_EIO, "expert parallel: a peer barrier gave up after 1 s (a rank stopped or fell "
                                   "behind); the exchange must be reopened");
    return batch_take_error(s);
}

}  // namespace tlmg
