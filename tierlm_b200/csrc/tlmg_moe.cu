// tlmg_moe.cu - layer level of the sm_100a tier: HBM-resident expert slots,
// the routed-expert FFN (gate/up + SwiGLU, re-quantisation, down + the
// rank-ordered weighted combine) and the whole moe() block.
//
// Reference: moe() / run_batch() / expert_mats(), src/lib/tlm_model.c:880-1055.
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "tlmg_dev.cuh"
#include "tlmg_batch.cuh"
#include "tlmg_cache.cuh"
#include "tlmg_fused.cuh"
#include "tlmg_internal.h"
#include "tlmg_step.cuh"

namespace tlmg {

// Bump allocator for expert slots: large cudaMalloc chunks, 256-byte
// aligned sub-allocations, freed together with the context.
struct Arena {
    std::vector<void *> chunks;
    uint8_t *cur = nullptr;
    size_t left = 0;
    static constexpr size_t kChunk = size_t(256) << 20;
    void *get(size_t bytes) {
        bytes = (bytes + 255) & ~size_t(255);
        if (bytes > left) {
            size_t sz = bytes > kChunk ? bytes : kChunk;
            void *p = nullptr;
            if (cudaMalloc(&p, sz) != cudaSuccess) {
                cudaGetLastError();
                return nullptr;
            }
            chunks.push_back(p);
            cur = (uint8_t *)p;
            left = sz;
        }
        void *r = cur;
        cur += bytes;
        left -= bytes;
        return r;
    }
    void release() {
        for (void *p : chunks) cudaFree(p);
        chunks.clear();
        cur = nullptr;
        left = 0;
    }
};

struct Layer {
    Slot *d_slots = nullptr;       // [E] on the device
    std::vector<Slot> h_slots;     // host mirror
    bool slots_dirty = false;
    bool ready = false;                 // every expert loaded (or registered with the cache); set by sync_slots
    float *ffn_norm = nullptr;
    int router_dt = -1;
    void *router_w = nullptr;
    size_t router_rb = 0;
    float *router_bias = nullptr;
    uint8_t *mask = nullptr;
    const void *fused_plan = nullptr;   // the persistent kernel's plan when it can serve this layer
    int dt_gu = -1, dt_dn = -1;         // uniform gate/up and down dtypes of the layer (or -1)
    bool has_shared = false;
    bool cached = false;                // experts registered in host memory, served by the HBM slot cache
    int live = 1 << 30;                 // unmasked (routable) experts
    int sh_dt[3] = { 0, 0, 0 };
    void *sh_w[3] = { nullptr, nullptr, nullptr };
    float *sh_gate_inp = nullptr;
    // dense-FFN layer (no router, no experts): gate/up [d_ffn x D], down [D x d_ffn]
    bool has_dense = false;
    int d_ffn = 0;
    int dn_dt[3] = { 0, 0, 0 };
    void *dn_w[3] = { nullptr, nullptr, nullptr };
    float *dn_gu = nullptr, *dn_h = nullptr, *dn_out = nullptr;   // [2 d_ffn], [d_ffn], [D]
    uint8_t *dn_hq = nullptr;
};

}  // namespace tlmg

using namespace tlmg;

struct tlmg_ctx {
    tlmg_geom g;
    int device = 0;
    cudaStream_t st = nullptr;       // where work is queued (own_st or the caller's)
    cudaStream_t own_st = nullptr;
    std::vector<Layer> L;
    Arena arena;
    std::vector<void *> owned;     // other device allocations
    // device scratch for one token
    float *x = nullptr, *logits = nullptr, *ffn = nullptr, *h = nullptr, *hbuf = nullptr;
    uint8_t *xq8k = nullptr, *xq80 = nullptr, *hq = nullptr;
    int32_t *ids = nullptr;
    float *w = nullptr;
    size_t hq_stride = 0;
    float *sg = nullptr, *sh = nullptr, *s_out = nullptr, *sgate = nullptr;
    uint8_t *shq = nullptr;
    float *cw = nullptr;           // [top_k][D] weighted expert outputs w[r] * eo_r (output norms)
    float *onorm = nullptr;        // [64] per-rank output norms
    // many-token scratch
    float *mx = nullptr, *mlog = nullptr, *mffn = nullptr;
    int m_cap = 0;
    // batched-decode staging on the device (host-pointer calls)
    float *bx = nullptr, *blog = nullptr, *bffn = nullptr, *bw = nullptr;
    int32_t *bids = nullptr;
    int b_cap = 0;
    // pinned staging
    uint8_t *pin = nullptr;
    size_t pin_cap = 0;
    int64_t launch0 = 0;
    FusedScratch fused;
    BatchScratch batch;            // batched-decode scratch (tlmg_expert_ffn_batch)
    EpP2P epp;                     // peer-memory expert parallelism (tlmg_ep_open)
    StepModel *step = nullptr;     // the whole decoder step (tlmg_step_open)
    uint64_t wgen = 1;             // bumped by every call that changes weights, layers or launch set-up
    ExpertCache cache;             // HBM expert-slot cache (tlmg_cache_enable)
    Slot *pin_slots = nullptr;     // pinned [n_layers][E] slot-table mirror of cached layers
    int32_t *pin_ids = nullptr;    // pinned [64] routed ids of a cached layer
    // router lookahead of cached layers (tlmg_cache_lookahead)
    int la_depth = 0, la_k = 0, la_k_now = 0;
    int la_layer = -1;             // layer whose predicted ids are in pin_la, -1 = none
    float *la_x = nullptr, *la_logits = nullptr, *la_w = nullptr;
    uint8_t *la_q = nullptr;
    int32_t *la_ids = nullptr, *pin_la = nullptr;
    bool fused_on = true;
    uint64_t *trace = nullptr;     // device [nsm][FUSED_TRACE_POINTS] when tracing
    Slot *slots_all = nullptr;     // device [n_layers][E]: every layer's slot table, contiguous
    uint8_t *mask_all = nullptr;   // device [n_layers][E] (zero-filled) once any layer has a mask
    float *bias_all = nullptr;     // device [n_layers][E] (zero-filled) once any layer has a router bias
    // per-launch event timing (tlmg_profile)
    bool prof = false;
    std::vector<cudaEvent_t> ev_pool;
    struct Mark { int cls; cudaEvent_t a, b; int64_t bytes; };
    std::vector<Mark> marks;
    int64_t prof_bytes[3] = { 0, 0, 0 };
};

namespace tlmg {

static void *dalloc(tlmg_ctx *c, size_t bytes) {
    void *p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    c->owned.push_back(p);
    return p;
}

static int ensure_pin(tlmg_ctx *c, size_t bytes) {
    if (bytes <= c->pin_cap) return TLMG_OK;
    if (c->pin) cudaFreeHost(c->pin);
    c->pin = nullptr;
    c->pin_cap = 0;
    if (cudaMallocHost(&c->pin, bytes) != cudaSuccess) {
        cudaGetLastError();
        return set_error(TLMG_ENOMEM, "pinned staging of %zu bytes failed", bytes);
    }
    c->pin_cap = bytes;
    return TLMG_OK;
}

static int check_layer(tlmg_ctx *c, int layer) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    if (layer < 0 || layer >= c->g.n_layers)
        return set_error(TLMG_ERANGE, "layer %d out of range [0, %d)", layer, c->g.n_layers);
    return TLMG_OK;
}

static int sync_slots(tlmg_ctx *c, Layer &Ly) {
    if (!Ly.slots_dirty) return TLMG_OK;
    cudaError_t e = cudaMemcpy(Ly.d_slots, Ly.h_slots.data(), sizeof(Slot) * Ly.h_slots.size(),
                               cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "slot table upload");
    Ly.slots_dirty = false;
    // the persistent and batched kernels serve layers whose (loaded) experts
    // all share one gate/up dtype and one down dtype; calls that need every
    // expert check layer_ready() as well
    int dgu = -1, ddn = -1;
    bool uniform = true;
    for (const Slot &sl : Ly.h_slots) {
        if (!sl.ok) continue;
        if (dgu < 0) { dgu = sl.dt[0]; ddn = sl.dt[2]; }
        if (sl.dt[0] != dgu || sl.dt[1] != dgu || sl.dt[2] != ddn) uniform = false;
    }
    uniform = uniform && dgu >= 0;
    if (Ly.cached) {
        const int l = (int)(&Ly - c->L.data());
        Ly.ready = true;
        for (int e2 = 0; e2 < c->g.n_experts && Ly.ready; e2++)
            Ly.ready = c->cache.src[(size_t)l * c->g.n_experts + e2].ok;
    } else {
        Ly.ready = !Ly.h_slots.empty();
        for (const Slot &sl : Ly.h_slots) Ly.ready = Ly.ready && sl.ok;
    }
    Ly.dt_gu = uniform ? dgu : -1;
    Ly.dt_dn = uniform ? ddn : -1;
    Ly.fused_plan = uniform && !Ly.cached ? fused_plan(c->fused, c->g, dgu, ddn) : nullptr;
    return TLMG_OK;
}

// ---------------------------------------------------------------------------
// kernels

// Dot of one weight row with an activation, by one warp, result in lane 0.
template <class LD>
__device__ __forceinline__ float warp_row_dot_t(int dt, const uint8_t *wr, const uint8_t *act, int nb,
                                                BlockPart *part, int lane) {
    const int g = lane >> 3, j = lane & 7, bb = dt_block_bytes(dt), abb = act_block_bytes(act_kind_for(dt));
    float acc = 0.0f;
    for (int c0 = 0; c0 < nb; c0 += FCHUNK) {
        int nc = min(FCHUNK, nb - c0);
        for (int p0 = 0; p0 < nc; p0 += 4) {
            int p = p0 + g;
            bool valid = p < nc;
            int is = 0, ms = 0;
            const uint8_t *blk = wr + (size_t)(c0 + p) * bb;
            const uint8_t *ab = act + (size_t)(c0 + p) * abb;
            if (valid) block_part<LD>(dt, blk, ab, j, is, ms);
            group8_sum(is, ms);
            if (valid && j == 0) {
                float dA, dM;
                block_scales<LD>(dt, blk, ab, dA, dM);
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

// Slot matrices start 256-byte aligned, so a block's alignment follows from
// its dtype's block size.
__device__ __forceinline__ float warp_row_dot(int dt, const uint8_t *wr, const uint8_t *act, int nb,
                                              BlockPart *part, int lane) {
    switch (dt) {
    case DT_Q4_K: case DT_Q5_K: return warp_row_dot_t<WLoad<16>>(dt, wr, act, nb, part, lane);
    case DT_Q8_K: return warp_row_dot_t<WLoad<4>>(dt, wr, act, nb, part, lane);
    case DT_Q6_K: case DT_Q8_0: return warp_row_dot_t<WLoad<2>>(dt, wr, act, nb, part, lane);
    default: return warp_row_dot_t<WLoad<1>>(dt, wr, act, nb, part, lane);
    }
}

constexpr int FFN_WARPS = 8;

// gate/up rows of the k selected experts + SwiGLU: one warp per (rank, row).
__global__ void __launch_bounds__(FFN_WARPS * 32)
k_ffn_gateup(const Slot *__restrict__ slots, const int32_t *__restrict__ ids, int k, int D, int de,
             const uint8_t *__restrict__ xq8k, const uint8_t *__restrict__ xq80, float *__restrict__ hbuf) {
    __shared__ BlockPart part[FFN_WARPS][FCHUNK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t p = (int64_t)blockIdx.x * FFN_WARPS + warp; p < (int64_t)k * de; p += (int64_t)gridDim.x * FFN_WARPS) {
        int r = (int)(p / de), j = (int)(p % de);
        Slot s = slots[ids[r]];
        float gu[2];
#pragma unroll
        for (int m = 0; m < 2; m++) {
            int dt = s.dt[m];
            const uint8_t *act = act_kind_for(dt) == DT_Q8_0 ? xq80 : xq8k;
            size_t rb = (size_t)(D / dt_block(dt)) * dt_block_bytes(dt);
            gu[m] = warp_row_dot(dt, s.m[m] + (size_t)j * rb, act, D / dt_block(dt), part[warp], lane);
        }
        if (lane == 0) hbuf[p] = __fmul_rn(silu_f(gu[0]), gu[1]);
    }
}

// Re-quantise SwiGLU rows per rank with the activation kind of that
// expert's down matrix: one warp per activation block.
__global__ void k_quant_h(const Slot *__restrict__ slots, const int32_t *__restrict__ ids, int k, int de,
                          const float *__restrict__ hbuf, uint8_t *__restrict__ hq, size_t hq_stride) {
    const int lane = threadIdx.x & 31;
    int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int nb8k = (de + 255) / 256, nb80 = (de + 31) / 32;
    int per = nb80 > nb8k ? nb80 : nb8k;
    int r = (int)(wid / per), b = (int)(wid % per);
    if (r >= k) return;
    int kind = act_kind_for(slots[ids[r]].dt[2]);
    const float *h = hbuf + (size_t)r * de;
    uint8_t *dst = hq + hq_stride * r;
    if (kind == DT_Q8_K) {
        if (b < nb8k) warp_quant_q8k(h + 256 * b, min(256, de - 256 * b), dst + 292 * b, lane);
    } else {
        if (b < nb80) warp_quant_q80(h + 32 * b, min(32, de - 32 * b), dst + 36 * b, lane);
    }
}

// down rows of all k experts + rank-ordered combine: one warp per output
// row i. ffn[i] = sum_r w[r]*eo_r[i] (product rounded, then added; ascending
// r). With s_out: ffn[i] += sgate * s_out[i]. With h: h[i] += ffn[i].
__global__ void __launch_bounds__(FFN_WARPS * 32)
k_ffn_down(const Slot *__restrict__ slots, const int32_t *__restrict__ ids, const float *__restrict__ w, int k,
           int D, int de, const uint8_t *__restrict__ hq, size_t hq_stride, const float *__restrict__ s_out,
           const float *__restrict__ sgate, float *__restrict__ ffn, float *__restrict__ h, float *__restrict__ cw = nullptr) {
    __shared__ BlockPart part[FFN_WARPS][FCHUNK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = blockIdx.x * FFN_WARPS + warp; i < D; i += gridDim.x * FFN_WARPS) {
        float acc = 0.0f;
        for (int r = 0; r < k; r++) {
            Slot s = slots[ids[r]];
            int dt = s.dt[2];
            size_t rb = (size_t)(de / dt_block(dt)) * dt_block_bytes(dt);
            float eo = warp_row_dot(dt, s.m[2] + (size_t)i * rb, hq + hq_stride * r, de / dt_block(dt), part[warp], lane);
            const float c = __fmul_rn(w[r], eo);
            if (cw && lane == 0) cw[(size_t)r * D + i] = c;
            acc = __fadd_rn(acc, c);
        }
        if (lane == 0) {
            if (s_out) acc = __fadd_rn(acc, __fmul_rn(*sgate, s_out[i]));
            ffn[i] = acc;
            if (h) h[i] = __fadd_rn(h[i], acc);
        }
    }
}

// RMSNorm (reference tlm_model.c:164-169): the sum of squares is a double
// sum in index order. A fixed tree gives the same float after the division
// unless the value lies within the two sums' combined error bound of a float
// rounding boundary; then thread 0 redoes the sequential sum.
#ifndef TLMG_NORM_THREADS
#define TLMG_NORM_THREADS 512
#endif
constexpr int NORM_THREADS = TLMG_NORM_THREADS;   // threads of the one-CTA RMSNorm kernel
__global__ void k_rmsnorm(const float *__restrict__ x, const float *__restrict__ wn, int n, float eps,
                          float *__restrict__ out, uint8_t *__restrict__ q8k) {
    pdl_enter();
    __shared__ double red[32];
    __shared__ float r_sh;
    const float r = block_rms_inv(x, n, eps, red, &r_sh);
    const int nt = blockDim.x;
    int i = threadIdx.x;
    for (; i + 3 * nt < n; i += 4 * nt) {   // loads of four elements in flight together
        float xv[4], wv[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            xv[u] = x[i + u * nt];
            wv[u] = wn[i + u * nt];
        }
#pragma unroll
        for (int u = 0; u < 4; u++) out[i + u * nt] = __fmul_rn(__fmul_rn(xv[u], r), wv[u]);
    }
    for (; i < n; i += nt) out[i] = __fmul_rn(__fmul_rn(x[i], r), wn[i]);
    if (!q8k) return;
    // and out as Q8_K (tlm_quantize_act), one warp per 256-value block
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nb = (n + 255) / 256;
    for (int b = warp; b < nb; b += nt >> 5) warp_quant_q8k(out + 256 * b, min(256, n - 256 * b), q8k + 292 * b, lane);
}

__global__ void k_set_f32(float *p, float v) { *p = v; }

// silu(g)*u over a shared-expert row pair buffer [g | u].
__global__ void k_swiglu(const float *__restrict__ gu, int n, float *__restrict__ h) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) h[i] = __fmul_rn(silu_f(gu[i]), gu[n + i]);
}

// sgate = sigmoid(sum_i g[i]*x[i]) as a sequential float sum (reference
// tlm_model.c:1039-1044).
__global__ void k_shared_gate(const float *__restrict__ g, const float *__restrict__ x, int n, float *out) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    float d = 0.0f;
    for (int i = 0; i < n; i++) d = __fadd_rn(d, __fmul_rn(g[i], x[i]));
    *out = sigmoid_f(d);
}

// onorm[r] = (float)sqrt(sum_i (double)c[i] * c[i]) over c = cw[r][0..D) (the
// per-rank output norm moe() hands to the route hook, reference
// tlm_model.c:1029-1039), one warp per rank. The reference sums in index
// order; every term is exact in double and nonnegative, so a tree sum is
// within (2D + 8) * 2^-53 of it (relative), and when both ends of that
// interval give the same float the result is the reference's; otherwise
// lane 0 redoes the sequential sum.
__global__ void k_onorm(const float *__restrict__ cw, int D, float *__restrict__ onorm) {
    const int r = blockIdx.x, lane = threadIdx.x;
    const float *c = cw + (size_t)r * D;
    double s = 0.0;
    for (int i = lane; i < D; i += 32) s = __dadd_rn(s, __dmul_rn((double)c[i], (double)c[i]));
    for (int o = 16; o > 0; o >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, o));
    if (lane != 0) return;
    const double bound = __dmul_rn(s, __dmul_rn(2.0 * (double)D + 8.0, 0x1p-53));
    const float lo = __double2float_rn(__dsqrt_rn(fmax(__dsub_rn(s, bound), 0.0)));
    const float hi = __double2float_rn(__dsqrt_rn(__dadd_rn(s, bound)));
    if (lo == hi) {
        onorm[r] = lo;
        return;
    }
    double q = 0.0;
    for (int i = 0; i < D; i++) q = __dadd_rn(q, __dmul_rn((double)c[i], (double)c[i]));
    onorm[r] = __double2float_rn(__dsqrt_rn(q));
}

// h[i] += y[i] (the residual update of moe(), reference tlm_model.c:963, :1049).
__global__ void k_add(float *__restrict__ h, const float *__restrict__ y, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) h[i] = __fadd_rn(h[i], y[i]);
}

static int launched(const char *what) {
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, what);
}

// The persistent kernel runs when enabled, when it has a plan for the
// layer's dtypes and when x is 16-byte aligned (it reads x as float4).
static bool use_fused_path(const tlmg_ctx *c, const Layer &Ly, const float *x) {
    return c->fused_on && Ly.fused_plan && !Ly.cached && x && ((uintptr_t)x & 15u) == 0;
}

static cudaEvent_t prof_event(tlmg_ctx *c) {
    cudaEvent_t e = nullptr;
    if (!c->ev_pool.empty()) {
        e = c->ev_pool.back();
        c->ev_pool.pop_back();
    } else if (cudaEventCreate(&e) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return e;
}

// Bracket one launch of kernel class `cls` that serves n_tok tokens: call
// with begin = true before the launch and false after it.
static void prof_mark(tlmg_ctx *c, int cls, bool begin, int n_tok = 1) {
    if (!c->prof) return;
    if (begin) {
        cudaEvent_t a = prof_event(c);
        if (!a) return;
        cudaEventRecord(a, c->st);
        c->marks.push_back({ cls, a, nullptr, c->prof_bytes[cls] * n_tok });
    } else if (!c->marks.empty() && c->marks.back().b == nullptr && c->marks.back().cls == cls) {
        cudaEvent_t b = prof_event(c);
        if (!b) return;
        cudaEventRecord(b, c->st);
        c->marks.back().b = b;
    }
}

// Algorithmic weight bytes of one launch per class, from slot 0's dtypes.
static void prof_bytes(tlmg_ctx *c, const Layer &Ly) {
    if (!c->prof || Ly.h_slots.empty()) return;
    const Slot &s = Ly.h_slots[0];
    const int64_t D = c->g.d_model, de = c->g.d_expert, k = c->g.top_k;
    int64_t gu = k * de * (int64_t)(tlmg_row_bytes(s.dt[0], D) + tlmg_row_bytes(s.dt[1], D));
    int64_t dn = k * D * (int64_t)tlmg_row_bytes(s.dt[2], de);
    bool fused = c->fused_on && Ly.fused_plan;
    c->prof_bytes[0] = fused ? gu + dn : gu;
    c->prof_bytes[1] = dn;
    c->prof_bytes[2] = 4 * (int64_t)c->g.n_experts;
}

// x (device f32[D], normalised) -> the activation kinds the layer needs.
static int quant_inputs(tlmg_ctx *c, const float *x) {
    int rc = launch_quant_act(DT_Q8_K, x, c->g.d_model, c->xq8k, c->st);
    if (rc == TLMG_OK && c->g.d_model % 32 == 0) rc = launch_quant_act(DT_Q8_0, x, c->g.d_model, c->xq80, c->st);
    return rc;
}

// Arguments of a persistent-kernel launch of n_tok tokens from `layer`.
static FusedArgs fused_args(tlmg_ctx *c, const Layer &Ly, int layer, int n_tok) {
    const tlmg_geom &g = c->g;
    FusedArgs a{};
    a.plan = Ly.fused_plan;
    a.slots_all = c->slots_all;
    a.mask_all = c->mask_all;
    a.bias_all = c->bias_all;
    a.layer0 = layer;
    a.n_layers = g.n_layers;
    a.n_tok = n_tok;
    a.D = g.d_model;
    a.de = g.d_expert;
    a.E = g.n_experts;
    a.k = g.top_k;
    a.router = g.router;
    a.routed_scale = g.routed_scale;
    a.dt_gu = Ly.dt_gu;
    a.dt_dn = Ly.dt_dn;
    a.trace = c->trace;
    return a;
}

// Cached layer: the routed ids come to the host (one stream synchronisation),
// the cache makes those experts resident (side-stream copies that the
// compute stream waits for) and the layer's slot table is refreshed on the
// compute stream from a pinned mirror.
static int cache_route_acquire(tlmg_ctx *c, int layer) {
    const int k = c->g.top_k, E = c->g.n_experts;
    Layer &Ly = c->L[layer];
    if (!c->pin_ids && cudaMallocHost(&c->pin_ids, 4 * 64) != cudaSuccess) {
        cudaGetLastError();
        return set_error(TLMG_ENOMEM, "cache: pinned id buffer");
    }
    if (!c->pin_slots) {
        if (cudaMallocHost(&c->pin_slots, sizeof(Slot) * (size_t)c->g.n_layers * E) != cudaSuccess) {
            cudaGetLastError();
            c->pin_slots = nullptr;
            return set_error(TLMG_ENOMEM, "cache: pinned slot table");
        }
        memset(c->pin_slots, 0, sizeof(Slot) * (size_t)c->g.n_layers * E);
    }
    cudaError_t e = cudaMemcpyAsync(c->pin_ids, c->ids, 4 * (size_t)k, cudaMemcpyDeviceToHost, c->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->st);   // also ends the previous table upload
    if (e != cudaSuccess) return cuda_fail(e, "cache: routed ids");
    Slot got[64];
    int rc = cache_acquire(c->cache, layer, c->pin_ids, k, false, c->st, got);
    if (rc) return rc;
    // the lookahead hints for the next layer go out only now that this
    // layer's experts are referenced, so a hint never takes their slots
    // (reference moe(), src/lib/tlm_model.c:1014-1018)
    if (c->la_layer >= 0) {
        const int la = c->la_layer;
        c->la_layer = -1;
        if ((rc = cache_acquire(c->cache, la, c->pin_la, c->la_k_now, true, c->st, nullptr))) return rc;
    }
    Slot *tab = c->pin_slots + (size_t)layer * E;
    for (int r = 0; r < k; r++) {
        Ly.h_slots[c->pin_ids[r]] = got[r];
        tab[c->pin_ids[r]] = got[r];
    }
    e = cudaMemcpyAsync(Ly.d_slots, tab, sizeof(Slot) * (size_t)E, cudaMemcpyHostToDevice, c->st);
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "cache: slot table upload");
}

// Routed experts for one token on the device: logits -> ids/w -> ffn (and
// h += ffn when h != NULL). Inputs already quantised in xq8k / xq80.
static int run_experts(tlmg_ctx *c, int layer, const float *logits, float *ffn, float *h, const float *s_out,
                       const float *sgate, const float *x, float *cw = nullptr) {
    const tlmg_geom &g = c->g;
    Layer &Ly = c->L[layer];
    prof_bytes(c, Ly);
    if (!cw && use_fused_path(c, Ly, x)) {
        FusedArgs a = fused_args(c, Ly, layer, 1);
        a.x = x;
        a.logits = logits;
        a.ffn = ffn;
        a.h = h;
        a.s_out = s_out;
        a.sgate = sgate;
        a.ids_out = c->ids;
        a.w_out = c->w;
        prof_mark(c, 0, true);
        int rc = launch_fused_ffn(c->fused, a, c->st);
        prof_mark(c, 0, false);
        return rc;
    }
    prof_mark(c, 2, true);
    int rc = launch_route(g.router, logits, Ly.mask, Ly.router_bias, g.n_experts, g.top_k, g.routed_scale, c->ids,
                          c->w, c->st);
    prof_mark(c, 2, false);
    if (rc) return rc;
    if (Ly.cached && (rc = cache_route_acquire(c, layer))) return rc;
    (void)x;
    int k = g.top_k, D = g.d_model, de = g.d_expert;
    unsigned grid = (unsigned)std::min<int64_t>(((int64_t)k * de + FFN_WARPS - 1) / FFN_WARPS, 148 * 8);
    prof_mark(c, 0, true);
    k_ffn_gateup<<<grid, FFN_WARPS * 32, 0, c->st>>>(Ly.d_slots, c->ids, k, D, de, c->xq8k, c->xq80, c->hbuf);
    prof_mark(c, 0, false);
    if ((rc = launched("ffn gate/up"))) return rc;
    int per = std::max((de + 255) / 256, (de + 31) / 32);
    int64_t nw = (int64_t)k * per;
    k_quant_h<<<(unsigned)((nw + 7) / 8), 256, 0, c->st>>>(Ly.d_slots, c->ids, k, de, c->hbuf, c->hq, c->hq_stride);
    if ((rc = launched("ffn requant"))) return rc;
    prof_mark(c, 1, true);
    k_ffn_down<<<(unsigned)std::min(148 * 8, (D + FFN_WARPS - 1) / FFN_WARPS), FFN_WARPS * 32, 0, c->st>>>(
        Ly.d_slots, c->ids, c->w, k, D, de, c->hq, c->hq_stride, s_out, sgate, ffn, h, cw);
    prof_mark(c, 1, false);
    if ((rc = launched("ffn down"))) return rc;
    return Ly.cached ? cache_mark_used(c->cache, c->st) : TLMG_OK;
}

// Every expert of the layer is loaded (or registered with the slot cache);
// valid after sync_slots().
static bool layer_ready(tlmg_ctx *, Layer &Ly) { return Ly.ready; }

// Device-pointer core of tlmg_expert_ffn.
static int expert_ffn_dev(tlmg_ctx *c, int layer, const float *x, const float *logits, float *ffn) {
    Layer &Ly = c->L[layer];
    int rc = sync_slots(c, Ly);
    if (rc) return rc;
    if (!layer_ready(c, Ly)) return set_error(TLMG_ENOTFOUND, "layer %d: not every expert slot is loaded", layer);
    if (!use_fused_path(c, Ly, x) && (rc = quant_inputs(c, x))) return rc;
    return run_experts(c, layer, logits, ffn, nullptr, nullptr, nullptr, x);
}

enum PtrKind { PK_DEVICE, PK_PINNED, PK_PAGEABLE };
static PtrKind ptr_kind(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return PK_PAGEABLE;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return PK_DEVICE;
    if (a.type == cudaMemoryTypeHost) return PK_PINNED;
    return PK_PAGEABLE;
}

// host -> device copy of `bytes` from src into dst (device), through the
// pinned staging area at `stage_off` when src is pageable.
static int h2d(tlmg_ctx *c, void *dst, const void *src, size_t bytes, PtrKind k, size_t stage_off) {
    const void *from = src;
    if (k == PK_PAGEABLE) {
        memcpy(c->pin + stage_off, src, bytes);
        from = c->pin + stage_off;
    }
    cudaError_t e = cudaMemcpyAsync(dst, from, bytes, cudaMemcpyHostToDevice, c->st);
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "host to device copy");
}

static int d2h(tlmg_ctx *c, void *dst, const void *src, size_t bytes, PtrKind k, size_t stage_off) {
    void *to = k == PK_PAGEABLE ? (void *)(c->pin + stage_off) : dst;
    cudaError_t e = cudaMemcpyAsync(to, src, bytes, cudaMemcpyDeviceToHost, c->st);
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "device to host copy");
}

static int finish_d2h(tlmg_ctx *c, void *dst, size_t bytes, PtrKind k, size_t stage_off) {
    if (k == PK_PAGEABLE) memcpy(dst, c->pin + stage_off, bytes);
    return TLMG_OK;
}

static int stream_sync(tlmg_ctx *c) {
    cudaError_t e = cudaStreamSynchronize(c->st);
    if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
    if (int be = epp_take_error(c->batch, c->epp)) return be;
    uint32_t fe = fused_take_error(c->fused);
    if (fe)
        return set_error(TLMG_EIO, "expert FFN kernel gave up waiting (%s%s%s); results of this call are invalid",
                         fe & FUSED_ERR_BARRIER ? "grid barrier " : "", fe & FUSED_ERR_COPY ? "weight copies " : "",
                         fe & FUSED_ERR_PLAN ? "work plan" : "");
    return TLMG_OK;
}



}  // namespace tlmg

// ---------------------------------------------------------------------------
// C ABI (layer level)
extern "C" {

int tlmg_open(const tlmg_geom *g, int device, tlmg_ctx **out) {
    if (!g || !out) return set_error(TLMG_EINVAL, "tlmg_open: NULL argument");
    *out = nullptr;
    if (g->n_layers <= 0 || g->d_model <= 0 || g->n_experts < 0 || g->top_k < 0 || g->d_expert < 0 ||
        g->d_shared < 0 || (g->n_experts > 0 && (g->top_k == 0 || g->top_k > g->n_experts || g->top_k > 64)) ||
        g->n_experts > 512 || g->router < 0 || g->router > 2)
        return set_error(TLMG_EINVAL, "tlmg_open: bad geometry (layers %d, D %d, E %d, k %d, de %d, router %d)",
                         g->n_layers, g->d_model, g->n_experts, g->top_k, g->d_expert, g->router);
    if (g->d_model % 256 || g->d_expert % 256 || g->d_shared % 256)
        return set_error(TLMG_EINVAL, "tlmg_open: d_model, d_expert, d_shared must be multiples of 256");
    int rc = tlmg_init(device);
    if (rc) return rc;
    tlmg_ctx *c = new tlmg_ctx();
    c->g = *g;
    c->device = device;
    if (cudaStreamCreateWithFlags(&c->own_st, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return set_error(TLMG_EIO, "stream creation failed");
    }
    c->st = c->own_st;
    int D = g->d_model, de = g->d_expert > 0 ? g->d_expert : 256, E = g->n_experts > 0 ? g->n_experts : 1;
    int k = g->top_k > 0 ? g->top_k : 1, ds = g->d_shared > 0 ? g->d_shared : 256;
    c->hq_stride = (std::max(tlmg_qact_bytes(DT_Q8_K, de), tlmg_qact_bytes(DT_Q8_0, de)) + 255) & ~size_t(255);
    size_t xq = std::max(tlmg_qact_bytes(DT_Q8_K, D), tlmg_qact_bytes(DT_Q8_0, D)) + 256;
    bool ok = (c->x = (float *)dalloc(c, 4 * (size_t)D)) && (c->logits = (float *)dalloc(c, 4 * (size_t)E)) &&
              (c->ffn = (float *)dalloc(c, 4 * (size_t)D)) && (c->h = (float *)dalloc(c, 4 * (size_t)D)) &&
              (c->hbuf = (float *)dalloc(c, 4 * 4 * (size_t)k * de)) && (c->xq8k = (uint8_t *)dalloc(c, xq)) &&
              (c->xq80 = (uint8_t *)dalloc(c, xq)) && (c->hq = (uint8_t *)dalloc(c, c->hq_stride * k)) &&
              (c->ids = (int32_t *)dalloc(c, 4 * 64)) && (c->w = (float *)dalloc(c, 4 * 64)) &&
              (c->sg = (float *)dalloc(c, 8 * (size_t)ds)) && (c->sh = (float *)dalloc(c, 4 * (size_t)ds)) &&
              (c->s_out = (float *)dalloc(c, 4 * (size_t)D)) && (c->sgate = (float *)dalloc(c, 16)) &&
              (c->shq = (uint8_t *)dalloc(c, std::max(tlmg_qact_bytes(DT_Q8_K, ds), tlmg_qact_bytes(DT_Q8_0, ds)) + 256)) &&
              (c->cw = (float *)dalloc(c, 4 * (size_t)k * D)) && (c->onorm = (float *)dalloc(c, 4 * 64));
    if (ok) ok = ensure_pin(c, 4 * (size_t)(2 * D + E + 2 * 64) + 1024) == TLMG_OK;
    if (ok) ok = fused_init(c->fused, *g) == TLMG_OK;
    if (!ok) {
        tlmg_close(c);
        return set_error(TLMG_ENOMEM, "tlmg_open: device scratch allocation failed");
    }
    c->L.resize(g->n_layers);
    c->slots_all = (Slot *)dalloc(c, sizeof(Slot) * (size_t)E * g->n_layers);
    if (!c->slots_all) {
        tlmg_close(c);
        return set_error(TLMG_ENOMEM, "tlmg_open: slot table allocation failed");
    }
    for (int l = 0; l < g->n_layers; l++) {
        Layer &Ly = c->L[l];
        Ly.h_slots.assign(E, Slot{ { nullptr, nullptr, nullptr }, { 0, 0, 0 }, 0 });
        Ly.d_slots = c->slots_all + (size_t)l * E;
        Ly.slots_dirty = true;
    }
    c->launch0 = launches_total();
    *out = c;
    return TLMG_OK;
}

void tlmg_close(tlmg_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->st) cudaStreamSynchronize(c->st);
    if (c->own_st) cudaStreamSynchronize(c->own_st);
    fused_release(c->fused);
    batch_release(c->batch);
    epp_release(c->epp);
    if (c->step) step_graphs_release(*c->step);
    delete c->step;   // its device buffers are in c->owned
    cache_release(c->cache);
    if (c->pin_slots) cudaFreeHost(c->pin_slots);
    if (c->pin_ids) cudaFreeHost(c->pin_ids);
    if (c->pin_la) cudaFreeHost(c->pin_la);
    c->arena.release();
    for (void *p : c->owned) cudaFree(p);
    if (c->pin) cudaFreeHost(c->pin);
    if (c->own_st) cudaStreamDestroy(c->own_st);
    for (auto &m : c->marks) {
        cudaEventDestroy(m.a);
        if (m.b) cudaEventDestroy(m.b);
    }
    for (cudaEvent_t e : c->ev_pool) cudaEventDestroy(e);
    delete c;
}

int tlmg_profile(tlmg_ctx *c, int on) {
    if (c) c->wgen++;
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    cudaSetDevice(c->device);
    if (on) {
        cudaStreamSynchronize(c->st);
        for (auto &m : c->marks) {
            c->ev_pool.push_back(m.a);
            if (m.b) c->ev_pool.push_back(m.b);
        }
        c->marks.clear();
    }
    c->prof = on != 0;
    return TLMG_OK;
}

int tlmg_profile_read(tlmg_ctx *c, int cls, double *ms, int64_t *launches, int64_t *bytes_per_launch) {
    if (!c || cls < 0 || cls > 2) return set_error(TLMG_EINVAL, "profile_read: bad arguments");
    cudaSetDevice(c->device);
    cudaError_t e = cudaStreamSynchronize(c->st);
    if (e != cudaSuccess) return cuda_fail(e, "profile_read synchronize");
    double tot = 0.0;
    int64_t n = 0, bytes = 0;
    for (auto &m : c->marks) {
        if (m.cls != cls || !m.b) continue;
        float t = 0.0f;
        if (cudaEventElapsedTime(&t, m.a, m.b) == cudaSuccess) {
            tot += t;
            n++;
            bytes += m.bytes;
        }
    }
    if (ms) *ms = tot;
    if (launches) *launches = n;
    if (bytes_per_launch) *bytes_per_launch = n ? bytes / n : 0;
    return TLMG_OK;
}

int tlmg_set_fused(tlmg_ctx *c, int on) {
    if (c) c->wgen++;
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    if (on < 0 || on > 4 || on == 3) return set_error(TLMG_EINVAL, "set_fused: mode %d", on);
    c->fused_on = on != 0;
    c->fused.single = on == 4;
    return c->fused.enabled ? TLMG_OK : (on ? set_error(TLMG_EUNSUP, "persistent kernel unavailable on this device") : TLMG_OK);
}

int tlmg_set_batch_kernels(tlmg_ctx *c, int mode) {
    if (c) c->wgen++;
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    // 0..2: both projections; 10 * g + d: gate/up mode g, down mode d
    const int g = mode >= 10 ? mode / 10 : mode, d = mode >= 10 ? mode % 10 : mode;
    if (mode < 0 || g > 2 || d > 2) return set_error(TLMG_EINVAL, "batch kernel mode %d", mode);
    c->batch.kmode = g;
    c->batch.kmode_dn = d;
    return TLMG_OK;
}

int tlmg_trace(tlmg_ctx *c, int on, uint64_t *out, int cap) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    cudaSetDevice(c->device);
    const int n = c->fused.nsm * FUSED_TRACE_POINTS;
    if (on && !c->trace) {
        if (!(c->trace = (uint64_t *)dalloc(c, 8 * (size_t)n))) return set_error(TLMG_ENOMEM, "trace buffer");
        cudaMemset(c->trace, 0, 8 * (size_t)n);
    }
    int rc = stream_sync(c);
    if (rc) return rc;
    int got = 0;
    if (out && c->trace && cap > 0) {
        got = cap < n ? cap : n;
        cudaMemcpy(out, c->trace, 8 * (size_t)got, cudaMemcpyDeviceToHost);
    }
    if (!on) c->trace = nullptr;   // the buffer stays owned by the context
    return got;
}

int tlmg_check(tlmg_ctx *c) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    cudaSetDevice(c->device);
    return stream_sync(c);
}

int tlmg_set_stream(tlmg_ctx *c, void *stream) {
    if (c) c->wgen++;
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    cudaSetDevice(c->device);
    cudaStream_t next = stream ? (cudaStream_t)stream : c->own_st;
    if (next != c->st) {
        // order: work already queued on the old stream happens before new work
        cudaEvent_t ev;
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return set_error(TLMG_EIO, "event");
        cudaEventRecord(ev, c->st);
        cudaStreamWaitEvent(next, ev, 0);
        cudaEventDestroy(ev);
        c->st = next;
    }
    return TLMG_OK;
}

int64_t tlmg_launch_count(const tlmg_ctx *c) { return c ? launches_total() - c->launch0 : 0; }

int tlmg_set_expert(tlmg_ctx *c, int layer, int expert, const int32_t dt[3], const void *payload,
                    size_t payload_len, const uint64_t item_off[3]) {
    if (c) c->wgen++;
    int rc = check_layer(c, layer);
    if (rc) return rc;
    cudaSetDevice(c->device);
    if (expert < 0 || expert >= c->g.n_experts)
        return set_error(TLMG_ERANGE, "expert %d out of range [0, %d)", expert, c->g.n_experts);
    if (!dt || !payload || !item_off) return set_error(TLMG_EINVAL, "set_expert: NULL argument");
    const int D = c->g.d_model, de = c->g.d_expert;
    size_t bytes[3];
    for (int m = 0; m < 3; m++) {
        int q = dt_block(dt[m]);
        if (q <= 1 || (m < 2 ? D : de) % q)
            return set_error(TLMG_EUNSUP, "set_expert %d:%d: matrix %d dtype %d is not a block-quantised type", layer,
                             expert, m, dt[m]);
        bytes[m] = m < 2 ? (size_t)de * tlmg_row_bytes(dt[m], D) : (size_t)D * tlmg_row_bytes(dt[m], de);
        if (item_off[m] > payload_len || bytes[m] > payload_len - item_off[m])
            return set_error(TLMG_EFORMAT, "set_expert %d:%d: matrix %d [%llu, +%zu) exceeds payload %zu", layer,
                             expert, m, (unsigned long long)item_off[m], bytes[m], payload_len);
    }
    Layer &Ly = c->L[layer];
    if (Ly.cached) return set_error(TLMG_EBUSY, "layer %d is served by the slot cache (tlmg_set_expert_host)", layer);
    Slot &s = Ly.h_slots[expert];
    size_t pad[3];
    for (int m = 0; m < 3; m++) pad[m] = (bytes[m] + 16 + 255) & ~size_t(255);
    uint8_t *base = nullptr;
    bool reuse = s.ok && s.dt[0] == dt[0] && s.dt[1] == dt[1] && s.dt[2] == dt[2];
    if (reuse) {
        base = (uint8_t *)s.m[0];
    } else {
        base = (uint8_t *)c->arena.get(pad[0] + pad[1] + pad[2]);
        if (!base) return set_error(TLMG_ENOMEM, "set_expert %d:%d: HBM slot allocation failed", layer, expert);
    }
    const uint8_t *src = (const uint8_t *)payload;
    size_t off = 0;
    for (int m = 0; m < 3; m++) {
        cudaError_t e = cudaMemcpy(base + off, src + item_off[m], bytes[m], cudaMemcpyDefault);
        if (e != cudaSuccess) return cuda_fail(e, "expert upload");
        s.m[m] = base + off;
        s.dt[m] = dt[m];
        off += pad[m];
    }
    s.ok = 1;
    Ly.slots_dirty = true;
    return TLMG_OK;
}

int tlmg_cache_enable(tlmg_ctx *c, int n_slots, size_t slot_bytes) {
    if (c) c->wgen++;
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    if (c->g.n_experts <= 0) return set_error(TLMG_EINVAL, "cache: geometry has no routed experts");
    if (n_slots < c->g.top_k)
        return set_error(TLMG_EINVAL, "cache: %d slots cannot hold one token's %d experts", n_slots, c->g.top_k);
    cudaSetDevice(c->device);
    if (c->st) cudaStreamSynchronize(c->st);
    for (Layer &Ly : c->L)
        if (Ly.cached) return set_error(TLMG_EBUSY, "cache: already holds registered experts");
    return cache_init(c->cache, c->g.n_layers, c->g.n_experts, c->g.top_k, n_slots, slot_bytes);
}

int tlmg_set_expert_host(tlmg_ctx *c, int layer, int expert, const int32_t dt[3], const void *payload,
                         size_t payload_len, const uint64_t item_off[3]) {
    if (c) c->wgen++;
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (expert < 0 || expert >= c->g.n_experts)
        return set_error(TLMG_ERANGE, "expert %d out of range [0, %d)", expert, c->g.n_experts);
    if (!dt || !payload || !item_off) return set_error(TLMG_EINVAL, "set_expert_host: NULL argument");
    if (!c->cache.on) return set_error(TLMG_EINVAL, "set_expert_host: call tlmg_cache_enable first");
    cudaSetDevice(c->device);
    const int D = c->g.d_model, de = c->g.d_expert;
    size_t bytes[3];
    for (int m = 0; m < 3; m++) {
        int q = dt_block(dt[m]);
        if (q <= 1 || (m < 2 ? D : de) % q)
            return set_error(TLMG_EUNSUP, "set_expert_host %d:%d: matrix %d dtype %d is not a block-quantised type",
                             layer, expert, m, dt[m]);
        bytes[m] = m < 2 ? (size_t)de * tlmg_row_bytes(dt[m], D) : (size_t)D * tlmg_row_bytes(dt[m], de);
        if (item_off[m] > payload_len || bytes[m] > payload_len - item_off[m])
            return set_error(TLMG_EFORMAT, "set_expert_host %d:%d: matrix %d [%llu, +%zu) exceeds payload %zu", layer,
                             expert, m, (unsigned long long)item_off[m], bytes[m], payload_len);
    }
    Layer &Ly = c->L[layer];
    if (!Ly.cached)
        for (const Slot &sl : Ly.h_slots)
            if (sl.ok) return set_error(TLMG_EBUSY, "layer %d already has HBM-resident experts", layer);
    if (c->st) cudaStreamSynchronize(c->st);   // no launch may still read a slot this re-registration drops
    if ((rc = cache_register(c->cache, layer, expert, dt, payload, item_off, bytes))) return rc;
    Ly.cached = true;
    Ly.h_slots[expert] = Slot{ { nullptr, nullptr, nullptr }, { dt[0], dt[1], dt[2] }, 0 };
    Ly.slots_dirty = true;
    return TLMG_OK;
}

int tlmg_cache_prefetch(tlmg_ctx *c, int layer, const int32_t *ids, int k) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (!c->L[layer].cached) return TLMG_OK;   // resident layer: nothing to do
    if (k < 0 || (k > 0 && !ids)) return set_error(TLMG_EINVAL, "cache_prefetch: bad argument");
    cudaSetDevice(c->device);
    return cache_acquire(c->cache, layer, ids, k, true, c->st, nullptr);
}

int tlmg_cache_stats(tlmg_ctx *c, int64_t out[6]) {
    if (!c || !out) return set_error(TLMG_EINVAL, "cache_stats: NULL argument");
    const StorePolicy::Stats &k = c->cache.policy.stats();
    out[0] = k.hits;
    out[1] = k.misses;
    out[2] = k.prefetch_issued;
    out[3] = k.prefetch_used;
    out[4] = k.evictions;
    out[5] = c->cache.bytes_loaded;
    return TLMG_OK;
}

int tlmg_cache_tick(tlmg_ctx *c) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    cache_tick(c->cache);
    return TLMG_OK;
}

int tlmg_cache_lookahead(tlmg_ctx *c, int depth, int k) {
    if (c) c->wgen++;
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    if (depth < 0 || depth > 1 || k < 0 || k > 64 || k > c->g.n_experts)
        return set_error(TLMG_EINVAL, "cache_lookahead: depth %d (0 or 1), k %d (0 .. min(64, E))", depth, k);
    cudaSetDevice(c->device);
    if (depth && !c->la_x) {
        const int D = c->g.d_model, E = c->g.n_experts;
        const size_t xq = std::max(tlmg_qact_bytes(DT_Q8_K, D), tlmg_qact_bytes(DT_Q8_0, D)) + 256;
        if (!(c->la_x = (float *)dalloc(c, 4 * (size_t)D)) || !(c->la_logits = (float *)dalloc(c, 4 * (size_t)E)) ||
            !(c->la_q = (uint8_t *)dalloc(c, xq)) || !(c->la_ids = (int32_t *)dalloc(c, 4 * 64)) ||
            !(c->la_w = (float *)dalloc(c, 4 * 64)))
            return set_error(TLMG_ENOMEM, "cache_lookahead: scratch");
        if (!c->pin_la && cudaMallocHost(&c->pin_la, 4 * 64) != cudaSuccess) {
            cudaGetLastError();
            c->pin_la = nullptr;
            return set_error(TLMG_ENOMEM, "cache_lookahead: pinned ids");
        }
    }
    c->la_depth = depth;
    c->la_k = k ? k : c->g.top_k;
    return TLMG_OK;
}

int tlmg_set_layer(tlmg_ctx *c, int layer, const float *ffn_norm, int router_dt, const void *router_w,
                   size_t router_rb, const float *router_bias, const uint8_t *mask) {
    if (c) c->wgen++;
    int rc = check_layer(c, layer);
    if (rc) return rc;
    cudaSetDevice(c->device);
    Layer &Ly = c->L[layer];
    const int D = c->g.d_model, E = c->g.n_experts;
    auto up = [&](void **dst, const void *src, size_t bytes) -> bool {
        if (!src) return true;
        if (!*dst && !(*dst = dalloc(c, bytes + 16))) return false;
        return cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
    };
    if (ffn_norm && !up((void **)&Ly.ffn_norm, ffn_norm, 4 * (size_t)D)) return set_error(TLMG_EIO, "set_layer: norm upload");
    if (router_w) {
        int q = dt_block(router_dt);
        if (!q || D % q || router_rb < tlmg_row_bytes(router_dt, D))
            return set_error(TLMG_EINVAL, "set_layer: bad router dtype %d / row bytes %zu", router_dt, router_rb);
        if (Ly.router_w && (Ly.router_dt != router_dt || Ly.router_rb != router_rb)) Ly.router_w = nullptr;
        if (!up(&Ly.router_w, router_w, router_rb * (size_t)E)) return set_error(TLMG_EIO, "set_layer: router upload");
        Ly.router_dt = router_dt;
        Ly.router_rb = router_rb;
    }
    // router bias and expert mask live in [n_layers][E] arrays, zero-filled
    // for layers that have none (bias 0 and mask 0 leave routing unchanged),
    // so one launch can serve tokens of different layers
    const int NL = c->g.n_layers;
    if (router_bias) {
        if (!c->bias_all) {
            if (!(c->bias_all = (float *)dalloc(c, 4 * (size_t)E * NL))) return set_error(TLMG_ENOMEM, "bias table");
            cudaMemset(c->bias_all, 0, 4 * (size_t)E * NL);
            for (int l = 0; l < NL; l++) c->L[l].router_bias = c->bias_all + (size_t)l * E;
        }
        if (cudaMemcpy(Ly.router_bias, router_bias, 4 * (size_t)E, cudaMemcpyHostToDevice) != cudaSuccess)
            return set_error(TLMG_EIO, "set_layer: bias upload");
    }
    if (mask) {
        if (!c->mask_all) {
            if (!(c->mask_all = (uint8_t *)dalloc(c, (size_t)E * NL))) return set_error(TLMG_ENOMEM, "mask table");
            cudaMemset(c->mask_all, 0, (size_t)E * NL);
            for (int l = 0; l < NL; l++) c->L[l].mask = c->mask_all + (size_t)l * E;
        }
        if (cudaMemcpy(Ly.mask, mask, (size_t)E, cudaMemcpyHostToDevice) != cudaSuccess)
            return set_error(TLMG_EIO, "set_layer: mask upload");
        Ly.live = 0;
        for (int e = 0; e < E; e++) Ly.live += !mask[e];
    }
    return TLMG_OK;
}

int tlmg_set_shared(tlmg_ctx *c, int layer, const int32_t dt[3], const void *gate, const void *up_w,
                    const void *down, const float *gate_inp) {
    if (c) c->wgen++;
    int rc = check_layer(c, layer);
    if (rc) return rc;
    cudaSetDevice(c->device);
    const int D = c->g.d_model, ds = c->g.d_shared;
    if (ds <= 0) return set_error(TLMG_EINVAL, "set_shared: geometry has d_shared = 0");
    Layer &Ly = c->L[layer];
    const void *src[3] = { gate, up_w, down };
    for (int m = 0; m < 3; m++) {
        int q = dt_block(dt[m]);
        if (!q || (m < 2 ? D : ds) % q) return set_error(TLMG_EUNSUP, "set_shared: bad dtype %d", dt[m]);
        size_t bytes = m < 2 ? (size_t)ds * tlmg_row_bytes(dt[m], D) : (size_t)D * tlmg_row_bytes(dt[m], ds);
        void *p = dalloc(c, bytes + 256);
        if (!p || cudaMemcpy(p, src[m], bytes, cudaMemcpyHostToDevice) != cudaSuccess)
            return set_error(TLMG_EIO, "set_shared: upload failed");
        Ly.sh_w[m] = p;
        Ly.sh_dt[m] = dt[m];
    }
    if (gate_inp) {
        void *p = dalloc(c, 4 * (size_t)D);
        if (!p || cudaMemcpy(p, gate_inp, 4 * (size_t)D, cudaMemcpyHostToDevice) != cudaSuccess)
            return set_error(TLMG_EIO, "set_shared: gate upload failed");
        Ly.sh_gate_inp = (float *)p;
    } else {
        Ly.sh_gate_inp = nullptr;
    }
    Ly.has_shared = true;
    return TLMG_OK;
}

int tlmg_set_dense_ffn(tlmg_ctx *c, int layer, int d_ffn, const int32_t dt[3], const void *gate, const void *up_w,
                       const void *down) {
    if (c) c->wgen++;
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (!dt || !gate || !up_w || !down || d_ffn <= 0) return set_error(TLMG_EINVAL, "set_dense_ffn: bad argument");
    cudaSetDevice(c->device);
    const int D = c->g.d_model;
    Layer &Ly = c->L[layer];
    if (Ly.has_dense) return set_error(TLMG_EBUSY, "set_dense_ffn: layer %d already has a dense FFN", layer);
    const void *src[3] = { gate, up_w, down };
    for (int m = 0; m < 3; m++) {
        int q = dt_block(dt[m]);
        if (!q || (m < 2 ? D : d_ffn) % q) return set_error(TLMG_EUNSUP, "set_dense_ffn: bad dtype %d", dt[m]);
    }
    for (int m = 0; m < 3; m++) {
        size_t bytes = m < 2 ? (size_t)d_ffn * tlmg_row_bytes(dt[m], D) : (size_t)D * tlmg_row_bytes(dt[m], d_ffn);
        void *p = dalloc(c, bytes + 256);
        if (!p || cudaMemcpy(p, src[m], bytes, cudaMemcpyHostToDevice) != cudaSuccess)
            return set_error(TLMG_EIO, "set_dense_ffn: upload failed");
        Ly.dn_w[m] = p;
        Ly.dn_dt[m] = dt[m];
    }
    const size_t hq = std::max(tlmg_qact_bytes(DT_Q8_K, d_ffn), tlmg_qact_bytes(DT_Q8_0, d_ffn)) + 256;
    if (!(Ly.dn_gu = (float *)dalloc(c, 8 * (size_t)d_ffn)) || !(Ly.dn_h = (float *)dalloc(c, 4 * (size_t)d_ffn)) ||
        !(Ly.dn_out = (float *)dalloc(c, 4 * (size_t)D)) || !(Ly.dn_hq = (uint8_t *)dalloc(c, hq)))
        return set_error(TLMG_ENOMEM, "set_dense_ffn: scratch");
    Ly.d_ffn = d_ffn;
    Ly.has_dense = true;
    return TLMG_OK;
}

int tlmg_expert_ffn(tlmg_ctx *c, int layer, const float *x, const float *logits, float *ffn, int32_t *ids,
                    float *w) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (!x || !logits || !ffn) return set_error(TLMG_EINVAL, "expert_ffn: NULL argument");
    if (c->g.n_experts <= 0) return set_error(TLMG_EINVAL, "expert_ffn: geometry has no routed experts");
    cudaSetDevice(c->device);
    const int D = c->g.d_model, E = c->g.n_experts, k = c->g.top_k;
    PtrKind kx = ptr_kind(x);
    if (kx == PK_DEVICE) {
        if ((rc = expert_ffn_dev(c, layer, x, logits, ffn))) return rc;
        if (ids && cudaMemcpyAsync(ids, c->ids, 4 * (size_t)k, cudaMemcpyDeviceToDevice, c->st) != cudaSuccess)
            return set_error(TLMG_EIO, "ids copy");
        if (w && cudaMemcpyAsync(w, c->w, 4 * (size_t)k, cudaMemcpyDeviceToDevice, c->st) != cudaSuccess)
            return set_error(TLMG_EIO, "w copy");
        return TLMG_OK;
    }
    // host buffers: copies in and out are part of the call
    PtrKind kl = ptr_kind(logits), kf = ptr_kind(ffn);
    size_t o_x = 0, o_l = 4 * (size_t)D, o_f = o_l + 4 * (size_t)E, o_i = o_f + 4 * (size_t)D, o_w = o_i + 256;
    if ((rc = h2d(c, c->x, x, 4 * (size_t)D, kx, o_x))) return rc;
    if ((rc = h2d(c, c->logits, logits, 4 * (size_t)E, kl, o_l))) return rc;
    if ((rc = expert_ffn_dev(c, layer, c->x, c->logits, c->ffn))) return rc;
    if ((rc = d2h(c, ffn, c->ffn, 4 * (size_t)D, kf, o_f))) return rc;
    if (ids && (rc = d2h(c, c->pin + o_i, c->ids, 4 * (size_t)k, PK_PINNED, 0))) return rc;
    if (w && (rc = d2h(c, c->pin + o_w, c->w, 4 * (size_t)k, PK_PINNED, 0))) return rc;
    if ((rc = stream_sync(c))) return rc;
    finish_d2h(c, ffn, 4 * (size_t)D, kf, o_f);
    if (ids) memcpy(ids, c->pin + o_i, 4 * (size_t)k);
    if (w) memcpy(w, c->pin + o_w, 4 * (size_t)k);
    return TLMG_OK;
}

int tlmg_expert_ffn_many(tlmg_ctx *c, int layer0, int n_tok, const float *x, const float *logits, float *ffn) {
    int rc = check_layer(c, layer0);
    if (rc) return rc;
    if (n_tok <= 0) return TLMG_OK;
    if (!x || !logits || !ffn) return set_error(TLMG_EINVAL, "expert_ffn_many: NULL argument");
    cudaSetDevice(c->device);
    const int D = c->g.d_model, E = c->g.n_experts, NL = c->g.n_layers;
    PtrKind kx = ptr_kind(x);
    const float *dx = x, *dl = logits;
    float *df = ffn;
    PtrKind kl = PK_DEVICE, kf = PK_DEVICE;
    if (kx != PK_DEVICE) {
        if (n_tok > c->m_cap) {
            void *a = dalloc(c, 4 * (size_t)n_tok * D), *b = dalloc(c, 4 * (size_t)n_tok * E),
                 *f = dalloc(c, 4 * (size_t)n_tok * D);
            if (!a || !b || !f) return set_error(TLMG_ENOMEM, "expert_ffn_many: scratch allocation");
            c->mx = (float *)a;
            c->mlog = (float *)b;
            c->mffn = (float *)f;
            c->m_cap = n_tok;
        }
        kl = ptr_kind(logits);
        kf = ptr_kind(ffn);
        size_t need = 4 * (size_t)n_tok * (2 * D + E) + 64;
        if ((kx == PK_PAGEABLE || kl == PK_PAGEABLE || kf == PK_PAGEABLE) && (rc = ensure_pin(c, need))) return rc;
        if ((rc = h2d(c, c->mx, x, 4 * (size_t)n_tok * D, kx, 0))) return rc;
        if ((rc = h2d(c, c->mlog, logits, 4 * (size_t)n_tok * E, kl, 4 * (size_t)n_tok * D))) return rc;
        dx = c->mx;
        dl = c->mlog;
        df = c->mffn;
    }
    // one persistent launch for all tokens when every layer involved has the
    // same kernel plan; otherwise one call per token
    bool one = c->fused_on && ((uintptr_t)dx & 15u) == 0;
    const void *plan = nullptr;
    for (int t = 0; t < n_tok && one; t++) {
        Layer &Ly = c->L[(layer0 + t) % NL];
        if ((rc = sync_slots(c, Ly))) return rc;
        if (!layer_ready(c, Ly)) return set_error(TLMG_ENOTFOUND, "layer %d: not every expert slot is loaded",
                                                  (layer0 + t) % NL);
        if (!Ly.fused_plan || (plan && Ly.fused_plan != plan)) one = false;
        plan = Ly.fused_plan;
    }
    if (one && n_tok > 1) {
        Layer &L0 = c->L[layer0];
        prof_bytes(c, L0);
        FusedArgs a = fused_args(c, L0, layer0, n_tok);
        a.x = dx;
        a.logits = dl;
        a.ffn = df;
        prof_mark(c, 0, true, n_tok);
        rc = launch_fused_ffn(c->fused, a, c->st);
        prof_mark(c, 0, false);
        if (rc) return rc;
    } else {
        for (int t = 0; t < n_tok; t++) {
            int layer = (layer0 + t) % NL;
            if ((rc = expert_ffn_dev(c, layer, dx + (size_t)t * D, dl + (size_t)t * E, df + (size_t)t * D)))
                return rc;
        }
    }
    if (kx != PK_DEVICE) {
        size_t off = 4 * (size_t)n_tok * (D + E);
        if ((rc = d2h(c, ffn, c->mffn, 4 * (size_t)n_tok * D, kf, off))) return rc;
        if ((rc = stream_sync(c))) return rc;
        finish_d2h(c, ffn, 4 * (size_t)n_tok * D, kf, off);
    }
    return TLMG_OK;
}

int tlmg_expert_ffn_batch(tlmg_ctx *c, int layer, int n_tok, const float *x, const float *logits, float *ffn,
                          int32_t *ids, float *w) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (n_tok < 0) return set_error(TLMG_EINVAL, "expert_ffn_batch: n_tok %d", n_tok);
    if (n_tok == 0) return TLMG_OK;
    if (!x || !logits || !ffn) return set_error(TLMG_EINVAL, "expert_ffn_batch: NULL argument");
    if (c->g.n_experts <= 0) return set_error(TLMG_EINVAL, "expert_ffn_batch: geometry has no routed experts");
    cudaSetDevice(c->device);
    const int D = c->g.d_model, E = c->g.n_experts, k = c->g.top_k;
    Layer &Ly = c->L[layer];
    if ((rc = sync_slots(c, Ly))) return rc;
    if (!layer_ready(c, Ly)) return set_error(TLMG_ENOTFOUND, "layer %d: not every expert slot is loaded", layer);
    PtrKind kx = ptr_kind(x);
    const float *dx = x, *dl = logits;
    float *df = ffn;
    int32_t *di = ids;
    float *dw = w;
    PtrKind kl = PK_DEVICE, kf = PK_DEVICE;
    const size_t bx = 4 * (size_t)n_tok * D, bl = 4 * (size_t)n_tok * E, bk = 4 * (size_t)n_tok * k;
    if (kx != PK_DEVICE) {
        if (n_tok > c->b_cap) {
            void *a = dalloc(c, bx), *b = dalloc(c, bl), *f = dalloc(c, bx), *i = dalloc(c, bk), *ww = dalloc(c, bk);
            if (!a || !b || !f || !i || !ww) return set_error(TLMG_ENOMEM, "expert_ffn_batch: scratch allocation");
            c->bx = (float *)a;
            c->blog = (float *)b;
            c->bffn = (float *)f;
            c->bids = (int32_t *)i;
            c->bw = (float *)ww;
            c->b_cap = n_tok;
        }
        kl = ptr_kind(logits);
        kf = ptr_kind(ffn);
        // staging: x | logits | ffn | ids | w
        if ((rc = ensure_pin(c, 2 * bx + bl + 2 * bk + 64))) return rc;
        if ((rc = h2d(c, c->bx, x, bx, kx, 0))) return rc;
        if ((rc = h2d(c, c->blog, logits, bl, kl, bx))) return rc;
        dx = c->bx;
        dl = c->blog;
        df = c->bffn;
        di = ids ? c->bids : nullptr;
        dw = w ? c->bw : nullptr;
    }
    if (c->fused_on && !Ly.cached && Ly.dt_gu >= 0 && Ly.dt_dn >= 0 && ((uintptr_t)dx & 15u) == 0 &&
        batch_supported(Ly.dt_gu, Ly.dt_dn, D, c->g.d_expert, E, k)) {
        BatchArgs a{};
        a.slots = Ly.d_slots;
        a.mask = Ly.mask;
        a.bias = Ly.router_bias;
        a.n = n_tok;
        a.D = D;
        a.de = c->g.d_expert;
        a.E = E;
        a.k = k;
        a.router = c->g.router;
        a.routed_scale = c->g.routed_scale;
        a.dt_gu = Ly.dt_gu;
        a.dt_dn = Ly.dt_dn;
        a.x = dx;
        a.logits = dl;
        a.ffn = df;
        a.ids_out = di;
        a.w_out = dw;
        if ((rc = launch_batch(c->batch, a, c->st))) return rc;
    } else {
        // dtypes or shapes the batched kernels do not serve: one call per token
        for (int t = 0; t < n_tok; t++) {
            if ((rc = expert_ffn_dev(c, layer, dx + (size_t)t * D, dl + (size_t)t * E, df + (size_t)t * D)))
                return rc;
            if (di && cudaMemcpyAsync(di + (size_t)t * k, c->ids, 4 * (size_t)k, cudaMemcpyDeviceToDevice, c->st))
                return set_error(TLMG_EIO, "ids copy");
            if (dw && cudaMemcpyAsync(dw + (size_t)t * k, c->w, 4 * (size_t)k, cudaMemcpyDeviceToDevice, c->st))
                return set_error(TLMG_EIO, "w copy");
        }
    }
    if (kx != PK_DEVICE) {
        const size_t o_f = bx + bl, o_i = o_f + bx, o_w = o_i + bk;
        if ((rc = d2h(c, ffn, c->bffn, bx, kf, o_f))) return rc;
        if (ids && (rc = d2h(c, c->pin + o_i, c->bids, bk, PK_PINNED, 0))) return rc;
        if (w && (rc = d2h(c, c->pin + o_w, c->bw, bk, PK_PINNED, 0))) return rc;
        if ((rc = stream_sync(c))) return rc;
        finish_d2h(c, ffn, bx, kf, o_f);
        if (ids) memcpy(ids, c->pin + o_i, bk);
        if (w) memcpy(w, c->pin + o_w, bk);
    }
    return TLMG_OK;
}

// ---------------------------------------------------------------------------
// Expert parallelism: dispatch / owner experts / combine (device pointers)

static int ep_layer(tlmg_ctx *c, int layer, Layer **out) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (c->g.n_experts <= 0) return set_error(TLMG_EINVAL, "expert parallel: geometry has no routed experts");
    cudaSetDevice(c->device);
    Layer &Ly = c->L[layer];
    if ((rc = sync_slots(c, Ly))) return rc;
    if (Ly.cached) return set_error(TLMG_EUNSUP, "expert parallel: layer %d is served by the slot cache", layer);
    if (Ly.dt_gu < 0 || Ly.dt_dn < 0 ||
        !batch_supported(Ly.dt_gu, Ly.dt_dn, c->g.d_model, c->g.d_expert, c->g.n_experts, c->g.top_k))
        return set_error(TLMG_EUNSUP, "expert parallel: layer %d needs uniform K-quant gate/up and down dtypes", layer);
    *out = &Ly;
    return TLMG_OK;
}

size_t tlmg_ep_record_bytes(const tlmg_ctx *c) { return c ? ep_record_bytes(c->g.d_model) : 0; }

int tlmg_ep_dispatch(tlmg_ctx *c, int layer, int n_tok, const float *x, const float *logits, int n_ranks, void *send,
                     int32_t *perm, float *w, int64_t *counts) {
    Layer *Ly = nullptr;
    int rc = ep_layer(c, layer, &Ly);
    if (rc) return rc;
    if (n_tok < 0 || !counts || (n_tok > 0 && (!x || !logits || !send || !perm || !w)))
        return set_error(TLMG_EINVAL, "ep_dispatch: bad argument");
    if (n_tok > 0 && (ptr_kind(x) != PK_DEVICE || ptr_kind(send) != PK_DEVICE || ((uintptr_t)x & 15u) ||
                      ((uintptr_t)send & 15u)))
        return set_error(TLMG_EINVAL, "ep_dispatch: x and send must be 16-byte aligned device memory");
    BatchArgs a{};
    a.slots = Ly->d_slots;
    a.mask = Ly->mask;
    a.bias = Ly->router_bias;
    a.n = n_tok;
    a.D = c->g.d_model;
    a.de = c->g.d_expert;
    a.E = c->g.n_experts;
    a.k = c->g.top_k;
    a.router = c->g.router;
    a.routed_scale = c->g.routed_scale;
    a.dt_gu = Ly->dt_gu;
    a.dt_dn = Ly->dt_dn;
    a.x = x;
    a.logits = logits;
    return ep_dispatch(c->batch, a, n_ranks, (uint8_t *)send, perm, w, counts, c->st);
}

int tlmg_ep_experts(tlmg_ctx *c, int layer, int e_lo, int e_hi, int64_t n_rec, const void *recv, float *eo) {
    Layer *Ly = nullptr;
    int rc = ep_layer(c, layer, &Ly);
    if (rc) return rc;
    if (n_rec < 0 || (n_rec > 0 && (!recv || !eo)) || e_lo < 0 || e_hi > c->g.n_experts || e_lo > e_hi)
        return set_error(TLMG_EINVAL, "ep_experts: bad argument");
    if (n_rec > 0 && (ptr_kind(recv) != PK_DEVICE || ((uintptr_t)recv & 15u)))
        return set_error(TLMG_EINVAL, "ep_experts: recv must be 16-byte aligned device memory");
    for (int e = e_lo; e < e_hi; e++)
        if (!Ly->h_slots[e].ok)
            return set_error(TLMG_ENOTFOUND, "layer %d: owned expert %d is not loaded", layer, e);
    return ep_experts(c->batch, Ly->d_slots, Ly->dt_gu, Ly->dt_dn, c->g.d_model, c->g.d_expert, c->g.n_experts, e_lo,
                      e_hi, n_rec, (const uint8_t *)recv, eo, c->st);
}

int tlmg_ep_combine(tlmg_ctx *c, int n_tok, const float *back, const int32_t *perm, const float *w, float *ffn) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    if (n_tok < 0 || (n_tok > 0 && (!back || !perm || !w || !ffn)))
        return set_error(TLMG_EINVAL, "ep_combine: bad argument");
    cudaSetDevice(c->device);
    return ep_combine(n_tok, c->g.d_model, c->g.top_k, back, perm, w, ffn, c->st);
}

// ---------------------------------------------------------------------------
// Expert parallelism over peer memory

int tlmg_ep_open(tlmg_ctx *c, int rank, int n_ranks, int max_tok) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    if (c->g.n_experts <= 0 || n_ranks > c->g.n_experts)
        return set_error(TLMG_EINVAL, "ep_open: %d ranks for %d experts", n_ranks, c->g.n_experts);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->st);
    return epp_alloc(c->epp, rank, n_ranks, max_tok, c->g.d_model, c->g.top_k);
}

size_t tlmg_ep_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int tlmg_ep_handle(tlmg_ctx *c, void *handle) {
    if (!c || !handle) return set_error(TLMG_EINVAL, "ep_handle: NULL argument");
    if (!c->epp.base) return set_error(TLMG_EINVAL, "ep_handle: exchange not open");
    cudaSetDevice(c->device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, c->epp.base);
    if (e != cudaSuccess) return cuda_fail(e, "ep_handle");
    memcpy(handle, &h, sizeof h);
    return TLMG_OK;
}

int tlmg_ep_connect(tlmg_ctx *c, const void *handles) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    EpP2P &e = c->epp;
    if (!e.base) return set_error(TLMG_EINVAL, "ep_connect: exchange not open");
    if (e.nr > 1 && !handles) return set_error(TLMG_EINVAL, "ep_connect: NULL handles");
    cudaSetDevice(c->device);
    for (int r = 0; r < e.nr; r++) {
        if (r == e.me || e.peer[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t *)handles + r * sizeof h, sizeof h);
        void *p = nullptr;
        cudaError_t err = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (err != cudaSuccess) return cuda_fail(err, "ep_connect: mapping a peer's exchange buffer");
        e.peer[r] = (uint8_t *)p;
        e.opened[r] = true;
    }
    return TLMG_OK;
}

int tlmg_ep_layer(tlmg_ctx *c, int layer, int n_tok, const float *x, const float *logits, float *ffn, int32_t *ids,
                  float *w) {
    Layer *Ly = nullptr;
    int rc = ep_layer(c, layer, &Ly);
    if (rc) return rc;
    if (n_tok < 0 || (n_tok > 0 && (!x || !logits || !ffn)))
        return set_error(TLMG_EINVAL, "ep_layer: bad argument");
    if (n_tok > 0 && (ptr_kind(x) != PK_DEVICE || ptr_kind(logits) != PK_DEVICE || ptr_kind(ffn) != PK_DEVICE ||
                      (ids && ptr_kind(ids) != PK_DEVICE) || (w && ptr_kind(w) != PK_DEVICE) || ((uintptr_t)x & 15u)))
        return set_error(TLMG_EINVAL, "ep_layer: x, logits, ffn, ids and w must be device memory, x 16-byte aligned");
    const int E = c->g.n_experts, nr = c->epp.nr, me = c->epp.me;
    const int lo = (int)(((int64_t)me * E + nr - 1) / nr), hi = (int)(((int64_t)(me + 1) * E + nr - 1) / nr);
    for (int e = lo; e < hi; e++)
        if (!Ly->h_slots[e].ok) return set_error(TLMG_ENOTFOUND, "layer %d: owned expert %d is not loaded", layer, e);
    BatchArgs a{};
    a.slots = Ly->d_slots;
    a.mask = Ly->mask;
    a.bias = Ly->router_bias;
    a.n = n_tok;
    a.D = c->g.d_model;
    a.de = c->g.d_expert;
    a.E = E;
    a.k = c->g.top_k;
    a.router = c->g.router;
    a.routed_scale = c->g.routed_scale;
    a.dt_gu = Ly->dt_gu;
    a.dt_dn = Ly->dt_dn;
    a.x = x;
    a.logits = logits;
    a.ffn = ffn;
    a.ids_out = ids;
    a.w_out = w;
    return epp_layer(c->batch, c->epp, a, lo, hi, c->st);
}

int tlmg_ep_close(tlmg_ctx *c) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    cudaSetDevice(c->device);
    int rc = stream_sync(c);
    epp_release(c->epp);
    return rc;
}

}  // extern "C"

namespace tlmg {

// The dense-FFN branch of moe() (reference tlm_model.c:947-964) on the
// normalised input in c->x (already quantised): gate/up, SiLU(g) * u,
// re-quantise, down, h += ffn.
static int dense_ffn(tlmg_ctx *c, Layer &Ly, float *dh) {
    const int D = c->g.d_model, F = Ly.d_ffn;
    int rc;
    for (int m = 0; m < 2; m++) {
        int dt = Ly.dn_dt[m];
        const void *act = act_kind_for(dt) == DT_Q8_0 ? (const void *)c->xq80
                        : act_kind_for(dt) == DT_F32 ? (const void *)c->x : (const void *)c->xq8k;
        if ((rc = launch_matvec(dt, Ly.dn_w[m], tlmg_row_bytes(dt, D), act, Ly.dn_gu + (size_t)m * F, D, 0, F, c->st)))
            return rc;
    }
    k_swiglu<<<(F + 255) / 256, 256, 0, c->st>>>(Ly.dn_gu, F, Ly.dn_h);
    if ((rc = launched("dense swiglu"))) return rc;
    const int dd = Ly.dn_dt[2], kd = act_kind_for(dd);
    if ((rc = launch_quant_act(kd, Ly.dn_h, F, Ly.dn_hq, c->st))) return rc;
    if ((rc = launch_matvec(dd, Ly.dn_w[2], tlmg_row_bytes(dd, F), kd == DT_F32 ? (const void *)Ly.dn_h : Ly.dn_hq,
                            Ly.dn_out, F, 0, D, c->st)))
        return rc;
    k_add<<<(D + 255) / 256, 256, 0, c->st>>>(dh, Ly.dn_out, D);
    return launched("dense residual");
}

// Router lookahead (reference lookahead(), src/lib/tlm_model.c:844-877): the
// next layer's RMSNorm and router on the current residual h (before this
// layer's h += ffn), top lookahead-k ids to pinned host memory; the copy
// completes with the synchronisation that brings this layer's routed ids to
// the host, and cache_route_acquire turns them into hints after this layer's
// acquisition. Only for a cached next layer with a router (a dense-FFN layer
// has none).
static int launch_lookahead(tlmg_ctx *c, int layer, const float *dh) {
    const int l2 = layer + 1;
    if (!c->la_depth || l2 >= c->g.n_layers) return TLMG_OK;
    Layer &N = c->L[l2];
    if (!N.cached || N.has_dense || !N.router_w || !N.ffn_norm) return TLMG_OK;
    const int D = c->g.d_model, E = c->g.n_experts;
    int k = std::min(c->la_k, N.live);   // never more hints than routable experts
    if (k <= 0) return TLMG_OK;
    int rc;
    k_rmsnorm<<<1, NORM_THREADS, 0, c->st>>>(dh, N.ffn_norm, D, c->g.norm_eps, c->la_x, nullptr);
    if ((rc = launched("lookahead rmsnorm"))) return rc;
    const int kr = act_kind_for(N.router_dt);
    if (kr != DT_F32 && (rc = launch_quant_act(kr, c->la_x, D, c->la_q, c->st))) return rc;
    if ((rc = launch_matvec(N.router_dt, N.router_w, N.router_rb, kr == DT_F32 ? (const void *)c->la_x : c->la_q,
                            c->la_logits, D, 0, E, c->st)))
        return rc;
    if ((rc = launch_route(c->g.router, c->la_logits, N.mask, N.router_bias, E, k, c->g.routed_scale, c->la_ids,
                           c->la_w, c->st)))
        return rc;
    cudaError_t e = cudaMemcpyAsync(c->pin_la, c->la_ids, 4 * (size_t)k, cudaMemcpyDeviceToHost, c->st);
    if (e != cudaSuccess) return cuda_fail(e, "lookahead ids");
    c->la_layer = l2;
    c->la_k_now = k;
    return TLMG_OK;
}

static int moe_layer_impl(tlmg_ctx *c, int layer, float *h, int32_t *ids, float *w, float *onorm) {
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (!h) return set_error(TLMG_EINVAL, "moe_layer: NULL h");
    cudaSetDevice(c->device);
    Layer &Ly = c->L[layer];
    const tlmg_geom &g = c->g;
    const int D = g.d_model, E = Ly.has_dense ? 0 : g.n_experts, k = g.top_k;
    if (!Ly.ffn_norm) return set_error(TLMG_ENOTFOUND, "moe_layer: layer %d has no ffn_norm", layer);
    if (E > 0 && !Ly.router_w) return set_error(TLMG_ENOTFOUND, "moe_layer: layer %d has no router", layer);
    PtrKind kh = ptr_kind(h);
    float *dh = h;
    if (kh != PK_DEVICE) {
        if ((rc = h2d(c, c->h, h, 4 * (size_t)D, kh, 0))) return rc;
        dh = c->h;
    }
    // xb = rmsnorm(h); activations of xb
    launch_k(k_rmsnorm, 1, NORM_THREADS, 0, c->st, dh, Ly.ffn_norm, D, g.norm_eps, c->x, (uint8_t *)nullptr);
    if ((rc = launched("rmsnorm"))) return rc;
    // the persistent kernel quantises its input itself: the activations of
    // xb are only formed for the parts that read them
    const bool fused_only = E > 0 && !Ly.has_dense && !(Ly.has_shared && g.d_shared > 0) && !onorm &&
                            act_kind_for(Ly.router_dt) == DT_F32 && use_fused_path(c, Ly, c->x);
    if (!fused_only && (rc = quant_inputs(c, c->x))) return rc;
    if (Ly.has_dense) {
        // no router, no experts, no shared expert, no route hook (moe() returns early)
        if ((rc = dense_ffn(c, Ly, dh))) return rc;
        if (kh != PK_DEVICE) {
            if ((rc = d2h(c, h, dh, 4 * (size_t)D, kh, 0)) || (rc = stream_sync(c))) return rc;
            finish_d2h(c, h, 4 * (size_t)D, kh, 0);
        }
        return TLMG_OK;
    }
    const float *s_out = nullptr, *sgate = nullptr;
    if (Ly.has_shared && g.d_shared > 0) {
        const int ds = g.d_shared;
        for (int m = 0; m < 2; m++) {
            int dt = Ly.sh_dt[m];
            const void *act = act_kind_for(dt) == DT_Q8_0 ? (const void *)c->xq80 : (const void *)c->xq8k;
            if ((rc = launch_matvec(dt, Ly.sh_w[m], tlmg_row_bytes(dt, D), act, c->sg + (size_t)m * ds, D, 0, ds, c->st)))
                return rc;
        }
        k_swiglu<<<(ds + 255) / 256, 256, 0, c->st>>>(c->sg, ds, c->sh);
        if ((rc = launched("shared swiglu"))) return rc;
        int kd = act_kind_for(Ly.sh_dt[2]);
        if ((rc = launch_quant_act(kd, c->sh, ds, c->shq, c->st))) return rc;
        if ((rc = launch_matvec(Ly.sh_dt[2], Ly.sh_w[2], tlmg_row_bytes(Ly.sh_dt[2], ds), c->shq, c->s_out, ds, 0, D,
                                c->st)))
            return rc;
        if (Ly.sh_gate_inp) k_shared_gate<<<1, 32, 0, c->st>>>(Ly.sh_gate_inp, c->x, D, c->sgate);
        else k_set_f32<<<1, 1, 0, c->st>>>(c->sgate, 1.0f);   // no gate: the shared expert's weight is 1
        if ((rc = launched("shared gate"))) return rc;
        s_out = c->s_out;
        sgate = c->sgate;
    }
    if (E > 0) {
        if ((rc = sync_slots(c, Ly))) return rc;
        if (!layer_ready(c, Ly)) return set_error(TLMG_ENOTFOUND, "layer %d: not every expert slot is loaded", layer);
        int kr = act_kind_for(Ly.router_dt);
        const void *ract = kr == DT_F32 ? (const void *)c->x : kr == DT_Q8_0 ? (const void *)c->xq80 : (const void *)c->xq8k;
        if ((rc = launch_matvec(Ly.router_dt, Ly.router_w, Ly.router_rb, ract, c->logits, D, 0, E, c->st))) return rc;
        if (Ly.cached && (rc = launch_lookahead(c, layer, dh))) return rc;
        if ((rc = run_experts(c, layer, c->logits, c->ffn, dh, s_out, sgate, c->x, onorm ? c->cw : nullptr))) return rc;
        if (onorm) {
            k_onorm<<<k, 32, 0, c->st>>>(c->cw, D, c->onorm);
            if ((rc = launched("output norms"))) return rc;
        }
    } else if (s_out) {
        // no routed experts: ffn = sgate * s_out, h += ffn
        k_ffn_down<<<(unsigned)((D + FFN_WARPS - 1) / FFN_WARPS), FFN_WARPS * 32, 0, c->st>>>(
            Ly.d_slots, c->ids, c->w, 0, D, g.d_expert, c->hq, c->hq_stride, s_out, sgate, c->ffn, dh, nullptr);
        if ((rc = launched("shared combine"))) return rc;
    }
    if (kh != PK_DEVICE) {
        if ((rc = d2h(c, h, dh, 4 * (size_t)D, kh, 0))) return rc;
    }
    const size_t o_ids = 4 * (size_t)D + 256, o_w = o_ids + 256;   // inside the staging area (>= 4D + 1024)
    if (ids && E > 0) {
        if (is_device_ptr(ids)) cudaMemcpyAsync(ids, c->ids, 4 * (size_t)k, cudaMemcpyDeviceToDevice, c->st);
        else cudaMemcpyAsync(c->pin + o_ids, c->ids, 4 * (size_t)k, cudaMemcpyDeviceToHost, c->st);
    }
    if (w && E > 0) {
        if (is_device_ptr(w)) cudaMemcpyAsync(w, c->w, 4 * (size_t)k, cudaMemcpyDeviceToDevice, c->st);
        else cudaMemcpyAsync(c->pin + o_w, c->w, 4 * (size_t)k, cudaMemcpyDeviceToHost, c->st);
    }
    const float *d_onorm = c->onorm;
    const size_t o_on = o_w + 256;
    if (onorm && E > 0) {
        if (is_device_ptr(onorm)) cudaMemcpyAsync(onorm, d_onorm, 4 * (size_t)k, cudaMemcpyDeviceToDevice, c->st);
        else cudaMemcpyAsync(c->pin + o_on, d_onorm, 4 * (size_t)k, cudaMemcpyDeviceToHost, c->st);
    }
    if (kh != PK_DEVICE || (ids && !is_device_ptr(ids)) || (w && !is_device_ptr(w)) ||
        (onorm && !is_device_ptr(onorm))) {
        if ((rc = stream_sync(c))) return rc;
        if (kh != PK_DEVICE) finish_d2h(c, h, 4 * (size_t)D, kh, 0);
        if (ids && E > 0 && !is_device_ptr(ids)) memcpy(ids, c->pin + o_ids, 4 * (size_t)k);
        if (w && E > 0 && !is_device_ptr(w)) memcpy(w, c->pin + o_w, 4 * (size_t)k);
        if (onorm && E > 0 && !is_device_ptr(onorm)) memcpy(onorm, c->pin + o_on, 4 * (size_t)k);
    }
    return TLMG_OK;
}

}  // namespace tlmg

extern "C" {

int tlmg_moe_layer(tlmg_ctx *c, int layer, float *h, int32_t *ids, float *w) {
    return moe_layer_impl(c, layer, h, ids, w, nullptr);
}

int tlmg_moe_layer_ex(tlmg_ctx *c, int layer, float *h, int32_t *ids, float *w, float *onorm) {
    return moe_layer_impl(c, layer, h, ids, w, onorm);
}

// ---------------------------------------------------------------------------
// The whole decoder step

int tlmg_step_open(tlmg_ctx *c, int n_heads, int n_kv_heads, int head_dim, int vocab, const float *inv_freq,
                   float attn_scale, int max_ctx, int kv_dt, int attn_mode) {
    if (!c || !inv_freq) return set_error(TLMG_EINVAL, "step_open: NULL argument");
    if (c->step) return set_error(TLMG_EBUSY, "step_open: already open");
    const int H = n_heads, KV = n_kv_heads, hd = head_dim, L = c->g.n_layers;
    if (H <= 0 || KV <= 0 || H % KV || H / KV > 16 || (hd != 64 && hd != 128 && hd != 256) || vocab <= 0 ||
        max_ctx <= 0 || max_ctx > 65536 || (kv_dt != DT_F32 && kv_dt != DT_BF16) ||
        (attn_mode != TLMG_ATTN_EXACT && attn_mode != TLMG_ATTN_SPLIT))
        return set_error(TLMG_EINVAL, "step_open: heads %d/%d x %d, vocab %d, max_ctx %d, kv dtype %d, mode %d", H, KV,
                         hd, vocab, max_ctx, kv_dt, attn_mode);
    cudaSetDevice(c->device);
    StepModel *m = new StepModel();
    m->H = H;
    m->KV = KV;
    m->hd = hd;
    m->vocab = vocab;
    m->max_ctx = max_ctx;
    m->page = 1;
    while (m->page < max_ctx) m->page <<= 1;
    m->kv_dt = kv_dt;
    m->attn_mode = attn_mode;
    m->attn_scale = attn_scale;
    m->inv_freq.assign(inv_freq, inv_freq + hd / 2);
    m->A.resize(L);
    const int D = c->g.d_model, nq = (H + 2 * KV) * hd;
    const size_t es = kv_dt == DT_F32 ? 4 : 2, pool = (size_t)L * KV * m->page * hd * es;
    size_t work = 0;
    for (int T = 1; T <= max_ctx; T++) work = std::max(work, attention_work_bytes(attn_mode, kv_dt, T, H, KV, hd));
    m->awork_bytes = work;
    const size_t aq = std::max(tlmg_qact_bytes(DT_Q8_K, H * hd), tlmg_qact_bytes(DT_Q8_0, H * hd)) + 4 * (size_t)H * hd;
    const size_t xq = tlmg_qact_bytes(DT_Q8_K, D) + tlmg_qact_bytes(DT_Q8_0, D) + 64;
    if (!(m->kpool = dalloc(c, pool)) || !(m->vpool = dalloc(c, pool)) || !(m->table = (int32_t *)dalloc(c, 4 * L)) ||
        !(m->awork = (float *)dalloc(c, work)) || !(m->qkv = (float *)dalloc(c, 4 * (size_t)nq)) ||
        !(m->att = (float *)dalloc(c, 4 * (size_t)H * hd)) || !(m->aq = (uint8_t *)dalloc(c, aq)) ||
        !(m->xb = (float *)dalloc(c, 4 * (size_t)D)) || !(m->xq = (uint8_t *)dalloc(c, xq)) ||
        !(m->rope = (float *)dalloc(c, 4 * (size_t)max_ctx * hd)) || !(m->logits = (float *)dalloc(c, 4 * (size_t)vocab)) ||
        !(m->dargs = (int32_t *)dalloc(c, 16))) {
        delete m;
        return set_error(TLMG_ENOMEM, "step_open: KV pages and scratch (%zu bytes of pages)", 2 * pool);
    }
    // RoPE cos / sin of every position, as tlm_model_step forms them
    // (src/lib/tlm_model.c:1066-1070): double angle, double cos / sin,
    // rounded to float, times the attention scale; row pos = cs | sn
    std::vector<float> rope((size_t)max_ctx * hd);
    std::vector<int32_t> tab(L);
    for (int pos = 0; pos < max_ctx; pos++)
        for (int j = 0; j < hd / 2; j++) {
            const double a = (double)pos * (double)m->inv_freq[j];
            rope[(size_t)pos * hd + j] = (float)std::cos(a) * attn_scale;
            rope[(size_t)pos * hd + hd / 2 + j] = (float)std::sin(a) * attn_scale;
        }
    for (int l = 0; l < L; l++) tab[l] = l;
    if (cudaMemcpy(m->rope, rope.data(), 4 * rope.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->table, tab.data(), 4 * (size_t)L, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(m->kpool, 0, pool) != cudaSuccess || cudaMemset(m->vpool, 0, pool) != cudaSuccess) {
        delete m;
        return set_error(TLMG_EIO, "step_open: table upload");
    }
    c->step = m;
    return TLMG_OK;
}

// Copies host or device memory into a new device buffer of the context.
static int upload(tlmg_ctx *c, void **dst, const void *src, size_t bytes, const char *what) {
    if (!(*dst = dalloc(c, bytes + 16))) return set_error(TLMG_ENOMEM, "%s: %zu bytes", what, bytes);
    if (cudaMemcpy(*dst, src, bytes, cudaMemcpyDefault) != cudaSuccess) {
        cudaGetLastError();
        return set_error(TLMG_EIO, "%s: copy", what);
    }
    return TLMG_OK;
}

int tlmg_set_attention(tlmg_ctx *c, int layer, const float *attn_norm, const int32_t *dt, const void *const *w,
                       const size_t *rb, const float *q_norm, const float *k_norm) {
    if (c) c->wgen++;
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (!c->step) return set_error(TLMG_EINVAL, "set_attention: tlmg_step_open first");
    if (!attn_norm || !dt || !w || !w[0] || !w[1] || !w[2] || !w[3])
        return set_error(TLMG_EINVAL, "set_attention: NULL argument");
    cudaSetDevice(c->device);
    StepModel &m = *c->step;
    StepLayer &A = m.A[layer];
    const int D = c->g.d_model, hd = m.hd;
    const int rows[4] = { m.H * hd, m.KV * hd, m.KV * hd, D }, cols[4] = { D, D, D, m.H * hd };
    size_t r[4];
    for (int i = 0; i < 4; i++) {
        const int q = dt_block(dt[i]);
        r[i] = rb && rb[i] ? rb[i] : tlmg_row_bytes(dt[i], cols[i]);
        if (!q || cols[i] % q || dt[i] == DT_MXFP4 || r[i] < tlmg_row_bytes(dt[i], cols[i]) ||
            (q > 1 && act_kind_for(dt[i]) == DT_Q8_K && cols[i] % 256))
            return set_error(TLMG_EINVAL, "set_attention: matrix %d dtype %d / row bytes %zu", i, dt[i], r[i]);
    }
    A = StepLayer{};
    if ((rc = upload(c, (void **)&A.attn_norm, attn_norm, 4 * (size_t)D, "attn_norm")) ||
        (q_norm && (rc = upload(c, (void **)&A.q_norm, q_norm, 4 * (size_t)hd, "q_norm"))) ||
        (k_norm && (rc = upload(c, (void **)&A.k_norm, k_norm, 4 * (size_t)hd, "k_norm"))))
        return rc;
    A.fused_qkv = dt[0] == dt[1] && dt[1] == dt[2] && r[0] == r[1] && r[1] == r[2];
    if (A.fused_qkv) {   // q | k | v rows back to back: one matvec for all three
        uint8_t *qkv = (uint8_t *)dalloc(c, r[0] * (size_t)(rows[0] + rows[1] + rows[2]) + 16);
        if (!qkv) return set_error(TLMG_ENOMEM, "set_attention: q|k|v");
        size_t off = 0;
        for (int i = 0; i < 3; i++) {
            if (cudaMemcpy(qkv + off, w[i], r[i] * (size_t)rows[i], cudaMemcpyDefault) != cudaSuccess)
                return set_error(TLMG_EIO, "set_attention: copy");
            A.w[i] = qkv + off;
            off += r[i] * (size_t)rows[i];
        }
    } else {
        for (int i = 0; i < 3; i++)
            if ((rc = upload(c, (void **)&A.w[i], w[i], r[i] * (size_t)rows[i], "set_attention"))) return rc;
    }
    if ((rc = upload(c, (void **)&A.w[3], w[3], r[3] * (size_t)rows[3], "set_attention"))) return rc;
    for (int i = 0; i < 4; i++) {
        A.dt[i] = dt[i];
        A.rb[i] = r[i];
    }
    A.set = true;
    return TLMG_OK;
}

int tlmg_set_embedding(tlmg_ctx *c, int dt, const void *tok_embd, size_t row_bytes) {
    if (c) c->wgen++;
    if (!c || !tok_embd) return set_error(TLMG_EINVAL, "set_embedding: NULL argument");
    if (!c->step) return set_error(TLMG_EINVAL, "set_embedding: tlmg_step_open first");
    const int D = c->g.d_model, q = dt_block(dt);
    const size_t rb = row_bytes ? row_bytes : tlmg_row_bytes(dt, D);
    if (!q || D % q || dt == DT_MXFP4 || rb < tlmg_row_bytes(dt, D))
        return set_error(TLMG_EINVAL, "set_embedding: dtype %d / row bytes %zu", dt, rb);
    cudaSetDevice(c->device);
    StepModel &m = *c->step;
    int rc = upload(c, (void **)&m.embd, tok_embd, rb * (size_t)m.vocab, "set_embedding");
    if (rc) return rc;
    m.embd_dt = dt;
    m.embd_rb = rb;
    return TLMG_OK;
}

int tlmg_set_output(tlmg_ctx *c, const float *out_norm, int dt, const void *lm_head, size_t row_bytes) {
    if (c) c->wgen++;
    if (!c || !out_norm || !lm_head) return set_error(TLMG_EINVAL, "set_output: NULL argument");
    if (!c->step) return set_error(TLMG_EINVAL, "set_output: tlmg_step_open first");
    const int D = c->g.d_model, q = dt_block(dt);
    const size_t rb = row_bytes ? row_bytes : tlmg_row_bytes(dt, D);
    if (!q || D % q || dt == DT_MXFP4 || rb < tlmg_row_bytes(dt, D))
        return set_error(TLMG_EINVAL, "set_output: dtype %d / row bytes %zu", dt, rb);
    cudaSetDevice(c->device);
    StepModel &m = *c->step;
    int rc = upload(c, (void **)&m.out_norm, out_norm, 4 * (size_t)D, "set_output");
    if (!rc) rc = upload(c, (void **)&m.head, lm_head, rb * (size_t)m.vocab, "set_output");
    if (rc) return rc;
    m.head_dt = dt;
    m.head_rb = rb;
    return TLMG_OK;
}

// Activations of x for weights of dtype dt: the reference's actc_get
// (src/lib/tlm_model.c:150-161), quantised at most once per kind per x.
struct ActCache {
    const float *x;
    int n;
    uint8_t *q8k, *q80;
    bool have8k = false, have80 = false;
    int get(int dt, cudaStream_t st, const void **out) {
        const int kind = act_kind_for(dt);
        if (kind == DT_F32) {
            *out = x;
            return TLMG_OK;
        }
        bool &have = kind == DT_Q8_K ? have8k : have80;
        uint8_t *buf = kind == DT_Q8_K ? q8k : q80;
        if (!have) {
            int rc = launch_quant_act(kind, x, n, buf, st);
            if (rc) return rc;
            have = true;
        }
        *out = buf;
        return TLMG_OK;
    }
};

// The step's device work on the context's stream: embedding, every layer's
// attention() and moe(), and (head) the final norm and lm_head into
// m.logits. With dargs the token and position are read from device memory
// (the body is then position-independent and can be captured); attention
// launches are then shaped for max_ctx positions.
static int step_body(tlmg_ctx *c, int token, int pos, bool head, const int32_t *dargs,
                     const cudaEvent_t *tev = nullptr) {
    StepModel &m = *c->step;
    const tlmg_geom &g = c->g;
    const int D = g.d_model, L = g.n_layers, H = m.H, KV = m.KV, hd = m.hd;
    cudaStream_t st = c->st;
    float *dh = c->h;
    const size_t off80 = (tlmg_qact_bytes(DT_Q8_K, D) + 15) & ~size_t(15);
    const size_t aoff80 = (tlmg_qact_bytes(DT_Q8_K, H * hd) + 15) & ~size_t(15);
    if (tev) cudaEventRecord(tev[0], st);
    int rc = step_embed(m.embd_dt, m.embd, m.embd_rb, token, dargs, D, dh, st);
    if (rc) return rc;
    const int rows[3] = { H * hd, KV * hd, KV * hd };
    for (int l = 0; l < L; l++) {
        const StepLayer &A = m.A[l];
        if (tev) cudaEventRecord(tev[1 + 2 * l], st);
        // attention() (src/lib/tlm_model.c:730-763)
        const bool xq_now = act_kind_for(A.dt[0]) == DT_Q8_K;   // xb as Q8_K from the norm kernel itself
        launch_k(k_rmsnorm, 1, NORM_THREADS, 0, st, dh, A.attn_norm, D, g.norm_eps, m.xb, xq_now ? m.xq : nullptr);
        if ((rc = launched("attention rmsnorm"))) return rc;
        ActCache ax{ m.xb, D, m.xq, m.xq + off80 };
        ax.have8k = xq_now;
        const void *act;
        if (A.fused_qkv) {
            if ((rc = ax.get(A.dt[0], st, &act)) ||
                (rc = launch_matvec(A.dt[0], A.w[0], A.rb[0], act, m.qkv, D, 0, rows[0] + rows[1] + rows[2], st)))
                return rc;
        } else {
            int at = 0;
            for (int i = 0; i < 3; i++) {
                if ((rc = ax.get(A.dt[i], st, &act)) ||
                    (rc = launch_matvec(A.dt[i], A.w[i], A.rb[i], act, m.qkv + at, D, 0, rows[i], st)))
                    return rc;
                at += rows[i];
            }
        }
        if ((rc = step_heads(m, l, pos, dargs, g.norm_eps, st))) return rc;
        if ((rc = decode_attention_impl(m.attn_mode, m.kv_dt, m.qkv, m.kpool, m.vpool, L, m.table + l, m.page,
                                        dargs ? m.max_ctx : pos + 1, dargs ? dargs + 2 : nullptr, H, KV, hd, m.awork,
                                        m.awork_bytes, m.att, st)))
            return rc;
        ActCache aa{ m.att, H * hd, m.aq, m.aq + aoff80 };
        if ((rc = aa.get(A.dt[3], st, &act)) ||
            (rc = launch_matvec(A.dt[3], A.w[3], A.rb[3], act, dh, H * hd, 0, D, st, dh)))   // h += o . att
            return rc;
        // moe() (src/lib/tlm_model.c:940-1055)
        if (tev) cudaEventRecord(tev[2 + 2 * l], st);
        if ((rc = moe_layer_impl(c, l, dh, nullptr, nullptr, nullptr))) return rc;
    }
    if (tev) cudaEventRecord(tev[2 * L + 1], st);
    if (!head) {
        if (tev) cudaEventRecord(tev[2 * L + 2], st);
        return TLMG_OK;
    }
    const bool xq_now = act_kind_for(m.head_dt) == DT_Q8_K;
    launch_k(k_rmsnorm, 1, NORM_THREADS, 0, st, dh, m.out_norm, D, g.norm_eps, m.xb, xq_now ? m.xq : nullptr);
    if ((rc = launched("output rmsnorm"))) return rc;
    ActCache af{ m.xb, D, m.xq, m.xq + off80 };
    af.have8k = xq_now;
    const void *act;
    if ((rc = af.get(m.head_dt, st, &act))) return rc;
    rc = launch_matvec(m.head_dt, m.head, m.head_rb, act, m.logits, D, 0, m.vocab, st);
    if (tev) cudaEventRecord(tev[2 * L + 2], st);
    return rc;
}

// Graph replay is used from a context's second step on when nothing in the
// step depends on host decisions made per call: every MoE layer resident
// (no slot cache; the persistent kernels' barrier words are restarted per
// captured launch or reset themselves).
static bool step_graph_allowed(const tlmg_ctx *c) {
    const StepModel &m = *c->step;
    if (m.graph_off || !m.use_graphs || m.calls == 0 || c->prof) return false;
    for (const Layer &Ly : c->L)
        if (Ly.cached) return false;
    return true;
}

// Captures step_body(head) with device-side token / position. A capture
// that fails turns graphs off for the context (the step stays eager).
static int capture_step(tlmg_ctx *c, int head) {
    StepModel &m = *c->step;
    cudaStream_t st = c->st;
    int rc;
    for (Layer &Ly : c->L)
        if ((rc = sync_slots(c, Ly))) return rc;   // uploads happen before the capture
    if (m.graph[head]) {
        cudaGraphExecDestroy(m.graph[head]);
        m.graph[head] = nullptr;
    }
    cudaGraph_t gr = nullptr;
    const int64_t n0 = launches_total();
    if ((!m.cap_st && cudaStreamCreateWithFlags(&m.cap_st, cudaStreamNonBlocking) != cudaSuccess) ||
        cudaStreamBeginCapture(m.cap_st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        m.graph_off = true;
        return TLMG_OK;
    }
    c->st = m.cap_st;   // nothing runs while capturing: the graph is launched on the caller's stream
    c->fused.graph_mode = true;
    set_pdl(true);
    rc = step_body(c, 0, 0, head != 0, m.dargs);
    set_pdl(false);
    c->fused.graph_mode = false;
    c->fused.bar_stale = true;
    c->st = st;
    cudaError_t e = cudaStreamEndCapture(m.cap_st, &gr);
    cudaGraphExec_t ex = nullptr;
    if (!rc && e == cudaSuccess && gr) e = cudaGraphInstantiate(&ex, gr, 0);
    if (gr) cudaGraphDestroy(gr);
    if (rc || e != cudaSuccess || !ex) {
        cudaGetLastError();
        m.graph_off = true;   // run eagerly from now on
        return TLMG_OK;
    }
    m.graph[head] = ex;
    m.graph_gen[head] = c->wgen;
    m.graph_launches[head] = launches_total() - n0;
    m.captures++;
    return TLMG_OK;
}

static int decode_step(tlmg_ctx *c, int token, int pos, float *logits) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    StepModel *mp = c->step;
    if (!mp) return set_error(TLMG_EINVAL, "decode_step: tlmg_step_open first");
    StepModel &m = *mp;
    const int L = c->g.n_layers;
    if (token < 0 || token >= m.vocab) return set_error(TLMG_EINVAL, "decode_step: token %d out of range", token);
    if (pos < 0 || pos >= m.max_ctx) return set_error(TLMG_ERANGE, "decode_step: position %d (context %d)", pos, m.max_ctx);
    if (!m.embd) return set_error(TLMG_ENOTFOUND, "decode_step: no embedding (tlmg_set_embedding)");
    if (logits && !m.head) return set_error(TLMG_ENOTFOUND, "decode_step: no lm_head (tlmg_set_output)");
    for (int l = 0; l < L; l++)
        if (!m.A[l].set) return set_error(TLMG_ENOTFOUND, "decode_step: layer %d has no attention weights", l);
    cudaSetDevice(c->device);
    cudaStream_t st = c->st;
    const int head = logits != nullptr;
    int rc;
    bool replayed = false;
    if (step_graph_allowed(c)) {
        if (!m.graph[head] || m.graph_gen[head] != c->wgen)
            if ((rc = capture_step(c, head))) return rc;
        if (m.graph[head] && !m.graph_off) {
            if ((rc = step_set_args(m.dargs, token, pos, st))) return rc;
            cudaError_t e = cudaGraphLaunch(m.graph[head], st);
            if (e != cudaSuccess) return cuda_fail(e, "decode_step: graph launch");
            count_launch((int)m.graph_launches[head]);
            c->fused.bar_stale = true;
            replayed = true;
            m.replays++;
        }
    }
    if (!replayed) {
        // while profiling (graphs are then off) the phases are timed with events
        const cudaEvent_t *tev = nullptr;
        if (c->prof) {
            if (m.tev.empty()) {
                m.tev.resize(2 * (size_t)L + 3, nullptr);
                for (cudaEvent_t &e : m.tev)
                    if (cudaEventCreate(&e) != cudaSuccess) return cuda_fail(cudaGetLastError(), "step events");
            }
            tev = m.tev.data();
        }
        set_pdl(true);
        rc = step_body(c, token, pos, head != 0, nullptr, tev);
        set_pdl(false);
        if (rc) return rc;
        if (tev) {
            cudaError_t e = cudaEventSynchronize(tev[2 * L + 2]);
            if (e != cudaSuccess) return cuda_fail(e, "step events");
            auto ms = [&](int a, int b) {
                float t = 0.0f;
                return cudaEventElapsedTime(&t, tev[a], tev[b]) == cudaSuccess ? (double)t : 0.0;
            };
            double attn = 0.0, moe = 0.0;
            for (int l = 0; l < L; l++) {
                attn += ms(1 + 2 * l, 2 + 2 * l);
                moe += ms(2 + 2 * l, 3 + 2 * l);   // to the next layer's start, or after the last layer
            }
            const double total = ms(0, 2 * L + 2);
            m.st_attn_ns += (uint64_t)(attn * 1e6);
            m.st_moe_ns += (uint64_t)(moe * 1e6);
            m.st_other_ns += (uint64_t)std::max(0.0, (total - attn - moe) * 1e6);
        }
    }
    m.calls++;
    m.st_tokens++;
    if (!logits) return TLMG_OK;
    const size_t bytes = 4 * (size_t)m.vocab;
    if (is_device_ptr(logits)) {
        cudaError_t e = cudaMemcpyAsync(logits, m.logits, bytes, cudaMemcpyDeviceToDevice, st);
        return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "decode_step: logits copy");
    }
    cudaError_t e = cudaMemcpyAsync(logits, m.logits, bytes, cudaMemcpyDefault, st);
    if (e != cudaSuccess) return cuda_fail(e, "decode_step: logits copy");
    return stream_sync(c);
}

int tlmg_step_info(const tlmg_ctx *c, int64_t *out) {
    if (!c || !out) return set_error(TLMG_EINVAL, "step_info: NULL argument");
    if (!c->step) return set_error(TLMG_EINVAL, "step_info: tlmg_step_open first");
    const StepModel &m = *c->step;
    out[0] = m.calls;
    out[1] = m.replays;
    out[2] = m.captures;
    out[3] = m.graph_off ? 1 : 0;
    return TLMG_OK;
}

int tlmg_step_stats(tlmg_ctx *c, uint64_t *out, int reset) {
    if (!c || !out) return set_error(TLMG_EINVAL, "step_stats: NULL argument");
    if (!c->step) return set_error(TLMG_EINVAL, "step_stats: tlmg_step_open first");
    StepModel &m = *c->step;
    out[0] = m.st_tokens;
    out[1] = m.st_attn_ns;
    out[2] = m.st_moe_ns;
    out[3] = 0;   // expert_wait_ns: not measured (resident experts never wait)
    out[4] = m.st_other_ns;
    if (reset) m.st_tokens = m.st_attn_ns = m.st_moe_ns = m.st_other_ns = 0;
    return TLMG_OK;
}

int tlmg_step_graphs(tlmg_ctx *c, int on) {
    if (!c) return set_error(TLMG_EINVAL, "NULL context");
    if (!c->step) return set_error(TLMG_EINVAL, "step_graphs: tlmg_step_open first");
    c->step->use_graphs = on != 0;
    if (on) c->step->graph_off = false;
    return TLMG_OK;
}

int tlmg_decode_step(tlmg_ctx *c, int token, int pos, float *logits) { return decode_step(c, token, pos, logits); }

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free expert FFN.
//
// For callers that must not allocate device memory on their decode path: a
// host runtime that sizes every buffer once at start-up (as the reference
// sizes its slot arena and scratch in tlm_model_open) and then runs a
// latency-bound per-token loop, where cudaMalloc / cudaFree could block on
// the allocator or synchronise the device behind other streams' work. This
// entry point takes the caller's device buffers and uses, as its only
// scratch, the fixed array below, which lives in every GPU that loads the
// library until the process exits.
namespace tlmg {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(1) << 20;   // 1 MiB per device
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mu;
static uint8_t *g_noalloc_addr[64];   // device address of the array, per device ordinal

// Set-up, once per device with that device current: the array's name is
// only a host-side stand-in, so its device address must be looked up.
static int noalloc_scratch(uint8_t **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "expert_ffn_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) return set_error(TLMG_EUNSUP, "expert_ffn_noalloc: device ordinal %d >= 64", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "expert_ffn_noalloc: cudaGetSymbolAddress");
        g_noalloc_addr[dev] = (uint8_t *)p;
    }
    *out = g_noalloc_addr[dev];
    return TLMG_OK;
}

}  // namespace tlmg

extern "C" int tlmg_expert_ffn_noalloc(const tlmg_expert_slot *experts, int E, int D, int de, int k, int router,
                                       float routed_scale, const float *x, const float *logits, float *ffn,
                                       int32_t *ids, float *w, void *stream) {
    if (!experts || !x || !logits || !ffn) return set_error(TLMG_EINVAL, "expert_ffn_noalloc: NULL argument");
    if (E <= 0 || E > RT_PER * 32 || k <= 0 || k > E || k > 64 || router < 0 || router > 2)
        return set_error(TLMG_EINVAL, "expert_ffn_noalloc: E=%d k=%d router=%d unsupported", E, k, router);
    if (D <= 0 || de <= 0 || D % 256 || de % 256)
        return set_error(TLMG_EINVAL, "expert_ffn_noalloc: D=%d de=%d must be positive multiples of 256", D, de);
    for (int e = 0; e < E; e++)
        for (int m = 0; m < 3; m++) {
            int q = dt_block(experts[e].dt[m]);
            if (q <= 1 || !experts[e].m[m])
                return set_error(TLMG_EINVAL, "expert_ffn_noalloc: expert %d matrix %d: dtype %d / pointer", e, m,
                                 experts[e].dt[m]);
        }
    // scratch layout: slot table | x as Q8_K | x as Q8_0 | ids | w | SwiGLU rows | re-quantised rows
    const size_t hq_stride = (std::max(tlmg_qact_bytes(DT_Q8_K, de), tlmg_qact_bytes(DT_Q8_0, de)) + 255) & ~size_t(255);
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t o_slots = 0, o_xk = up(o_slots + sizeof(Slot) * (size_t)E);
    const size_t o_x0 = up(o_xk + tlmg_qact_bytes(DT_Q8_K, D)), o_ids = up(o_x0 + tlmg_qact_bytes(DT_Q8_0, D));
    const size_t o_w = up(o_ids + 4 * 64), o_h = up(o_w + 4 * 64), o_hq = up(o_h + 4 * (size_t)k * de);
    const size_t need = o_hq + hq_stride * (size_t)k;
    if (need > NOALLOC_SCRATCH_BYTES)
        return set_error(TLMG_ERANGE, "expert_ffn_noalloc: needs %zu bytes of scratch, the fixed array has %zu", need,
                         NOALLOC_SCRATCH_BYTES);
    uint8_t *sc = nullptr;
    int rc = noalloc_scratch(&sc);
    if (rc) return rc;
    cudaStream_t st = pick_stream(stream);
    Slot slots[RT_PER * 32];
    for (int e = 0; e < E; e++) {
        for (int m = 0; m < 3; m++) {
            slots[e].m[m] = (const uint8_t *)experts[e].m[m];
            slots[e].dt[m] = experts[e].dt[m];
        }
        slots[e].ok = 1;
    }
    Slot *d_slots = (Slot *)(sc + o_slots);
    uint8_t *xk = sc + o_xk, *x0 = sc + o_x0, *hq = sc + o_hq;
    int32_t *d_ids = (int32_t *)(sc + o_ids);
    float *d_w = (float *)(sc + o_w), *hbuf = (float *)(sc + o_h);
    // the slot table is copied from this stack frame; a copy from pageable
    // memory has consumed its source when cudaMemcpyAsync returns
    cudaError_t e = cudaMemcpyAsync(d_slots, slots, sizeof(Slot) * (size_t)E, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "expert_ffn_noalloc: slot table copy");
    if ((rc = launch_quant_act(DT_Q8_K, x, D, xk, st))) return rc;
    if ((rc = launch_quant_act(DT_Q8_0, x, D, x0, st))) return rc;
    if ((rc = launch_route(router, logits, nullptr, nullptr, E, k, routed_scale, d_ids, d_w, st))) return rc;
    unsigned grid = (unsigned)std::min<int64_t>(((int64_t)k * de + FFN_WARPS - 1) / FFN_WARPS, 148 * 8);
    k_ffn_gateup<<<grid, FFN_WARPS * 32, 0, st>>>(d_slots, d_ids, k, D, de, xk, x0, hbuf);
    if ((rc = launched("noalloc gate/up"))) return rc;
    int per = std::max((de + 255) / 256, (de + 31) / 32);
    int64_t nw = (int64_t)k * per;
    k_quant_h<<<(unsigned)((nw + 7) / 8), 256, 0, st>>>(d_slots, d_ids, k, de, hbuf, hq, hq_stride);
    if ((rc = launched("noalloc requant"))) return rc;
    k_ffn_down<<<(unsigned)std::min(148 * 8, (D + FFN_WARPS - 1) / FFN_WARPS), FFN_WARPS * 32, 0, st>>>(
        d_slots, d_ids, d_w, k, D, de, hq, hq_stride, nullptr, nullptr, ffn, nullptr);
    if ((rc = launched("noalloc down"))) return rc;
    if (ids && (e = cudaMemcpyAsync(ids, d_ids, 4 * (size_t)k, cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
        return cuda_fail(e, "expert_ffn_noalloc: ids copy");
    if (w && (e = cudaMemcpyAsync(w, d_w, 4 * (size_t)k, cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
        return cuda_fail(e, "expert_ffn_noalloc: w copy");
    return TLMG_OK;
}
