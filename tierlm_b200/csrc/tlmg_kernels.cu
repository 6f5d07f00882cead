// tlmg_kernels.cu - kernel-level ops of the sm_100a tier: activation
// quantisation, the generic row-matvec (drop-in for tlm_matvec_rows), exact
// per-block partials, the router top-k, error handling and the host-buffer
// adapters with the reference's tier-table signatures.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <vector>

#include "tlmg_dev.cuh"
#include "tlmg_internal.h"

namespace tlmg {

// ---------------------------------------------------------------------------
// errors (reference convention: src/lib/tlm_platform.h:23-41)
static thread_local char t_errmsg[512];

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_errmsg, sizeof t_errmsg, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return set_error(TLMG_EIO, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

static std::atomic<int64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
static thread_local bool t_pdl = false;
void set_pdl(bool on) { t_pdl = on; }
bool pdl_on() { return t_pdl; }
int64_t launches_total() { return g_launches.load(std::memory_order_relaxed); }

static thread_local cudaStream_t t_stream = nullptr;
static thread_local int t_stream_dev = -1;

cudaStream_t pick_stream(void *user) {
    if (user) return (cudaStream_t)user;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!t_stream || t_stream_dev != dev) {
        cudaStreamCreateWithFlags(&t_stream, cudaStreamNonBlocking);
        t_stream_dev = dev;
    }
    return t_stream;
}

bool is_device_ptr(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// ---------------------------------------------------------------------------
// activation quantisation: one warp per block
__global__ void k_quant_q8k(const float *__restrict__ x, int64_t n, uint8_t *__restrict__ dst) {
    pdl_enter();
    int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (b * 256 >= n) return;
    int64_t rem = n - b * 256;
    warp_quant_q8k(x + b * 256, rem >= 256 ? 256 : (int)rem, dst + 292 * b, lane);
}

__global__ void k_quant_q80(const float *__restrict__ x, int64_t n, uint8_t *__restrict__ dst) {
    pdl_enter();
    int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (b * 32 >= n) return;
    int64_t rem = n - b * 32;
    warp_quant_q80(x + b * 32, rem >= 32 ? 32 : (int)rem, dst + 36 * b, lane);
}

int launch_quant_act(int kind, const float *x, int64_t n, void *dst, cudaStream_t st) {
    if (n <= 0) return TLMG_OK;
    if (kind == DT_F32) {
        cudaError_t e = cudaMemcpyAsync(dst, x, (size_t)n * 4, cudaMemcpyDeviceToDevice, st);
        return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "quantize_act copy");
    }
    if (kind != DT_Q8_K && kind != DT_Q8_0)
        return set_error(TLMG_EINVAL, "quantize_act: unsupported activation kind %d", kind);
    int64_t nb = kind == DT_Q8_K ? (n + 255) / 256 : (n + 31) / 32;
    const int wpb = 8;
    unsigned grid = (unsigned)((nb + wpb - 1) / wpb);
    if (kind == DT_Q8_K) launch_k(k_quant_q8k, grid, 32 * wpb, 0, st, x, n, (uint8_t *)dst);
    else launch_k(k_quant_q80, grid, 32 * wpb, 0, st, x, n, (uint8_t *)dst);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "quantize_act launch");
}

// ---------------------------------------------------------------------------
// generic row matvec. One warp per row; the 8-lane groups of the warp take
// four blocks per pass, reduce each block's exact integer partials, and the
// group leader stores (isum, msum, dA, dM) in shared memory; lane 0 then runs
// the reference's serial fmaf chain over the blocks in ascending order.
constexpr int MV_WARPS = 8;
constexpr int MV_CHUNK = FCHUNK;

template <int A>
__global__ void __launch_bounds__(MV_WARPS * 32)
k_matvec_q(int dt, const uint8_t *__restrict__ W, size_t rb, const uint8_t *__restrict__ act,
           float *y, int64_t n, int64_t r0, int64_t r1, const float *res) {
    pdl_enter();
    __shared__ BlockPart part[MV_WARPS][MV_CHUNK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 3, j = lane & 7;
    const int qk = dt_block(dt), bb = dt_block_bytes(dt), abb = act_block_bytes(act_kind_for(dt));
    const int nb = (int)(n / qk);
    for (int64_t row = r0 + (int64_t)blockIdx.x * MV_WARPS + warp; row < r1;
         row += (int64_t)gridDim.x * MV_WARPS) {
        const uint8_t *wr = W + (size_t)row * rb;
        float acc = 0.0f;
        for (int c0 = 0; c0 < nb; c0 += MV_CHUNK) {
            int nc = min(MV_CHUNK, nb - c0);
            for (int p0 = 0; p0 < nc; p0 += 4) {
                int p = p0 + g;
                bool valid = p < nc;
                int is = 0, ms = 0;
                const uint8_t *blk = wr + (size_t)(c0 + p) * bb;
                const uint8_t *ab = act + (size_t)(c0 + p) * abb;
                if (valid) block_part<WLoad<A>>(dt, blk, ab, j, is, ms);
                group8_sum(is, ms);
                if (valid && j == 0) {
                    float dA, dM;
                    block_scales<WLoad<A>>(dt, blk, ab, dA, dM);
                    part[warp][p] = BlockPart{ is, ms, dA, dM };
                }
            }
            __syncwarp();
            if (lane == 0)
                for (int p = 0; p < nc; p++) {
                    BlockPart q = part[warp][p];
                    acc = chain_step(dt, acc, q.dA, q.dM, q.is, q.ms);
                }
            __syncwarp();
        }
        if (lane == 0) y[row] = res ? __fadd_rn(res[row], acc) : acc;
    }
}

// The same per-row computation for 16-byte aligned rows of one integer
// dtype (a template parameter, so the block code is specialised): each warp
// owns rows r, r + stride, ... and double-buffers them in shared memory,
// copying row r + stride (cp.async, 16-byte pieces) while it computes row
// r from the other buffer. Block reads then come from shared memory at any
// block alignment (Q6_K's 210-byte and Q8_0's 34-byte blocks), every row is
// read from HBM once by full-width coalesced copies, and the grid is sized
// to the resident warps so that each keeps two rows in flight.
__device__ __forceinline__ void mv_cp16(void *dst, const void *src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

// NPF row buffers per warp: rows r + stride ... r + (NPF - 1) stride are
// in flight while row r is computed (NPF = 2 by default; TLMG_MV_TALL_NPF
// for tall matrices such as an lm_head, whose warps walk many rows).
#ifndef TLMG_MV_MINB
#define TLMG_MV_MINB 4   // CTAs per SM the staged matvec is compiled for (64 registers)
#endif
template <int DT, int NPF>
__global__ void __launch_bounds__(MV_WARPS * 32, TLMG_MV_MINB)
k_matvec_qs(const uint8_t *__restrict__ W, size_t rb, const uint8_t *__restrict__ act, float *y, int nb, int64_t r0,
            int64_t r1, const float *res) {
    pdl_enter();
    extern __shared__ uint4 mv_rows[];
    __shared__ BlockPart part[MV_WARPS][MV_CHUNK];
    constexpr int BB = dt_block_bytes(DT), ABB = act_block_bytes(act_kind_for(DT));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 3, j = lane & 7;
    const int nw = blockDim.x >> 5, n16 = nb * BB / 16;
    uint4 *buf = mv_rows + (size_t)warp * NPF * n16;
    const int64_t stride = (int64_t)gridDim.x * nw;
    // one cp.async group per row slot, an empty one past the last row, so
    // that "all but the newest NPF - 1 groups complete" means "row ready"
    auto issue = [&](int64_t r, uint4 *dst) {
        if (r < r1) {
            const uint4 *src = reinterpret_cast<const uint4 *>(W + (size_t)r * rb);
            for (int i = lane; i < n16; i += 32) mv_cp16(dst + i, src + i);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    int64_t row = r0 + (int64_t)blockIdx.x * nw + warp;
#pragma unroll
    for (int q = 0; q < NPF - 1; q++) issue(row + (int64_t)q * stride, buf + q * n16);
    for (int it = 0; row < r1; row += stride, it++) {
        const uint8_t *row_s = reinterpret_cast<const uint8_t *>(buf + (it % NPF) * n16);
        issue(row + (int64_t)(NPF - 1) * stride, buf + ((it + NPF - 1) % NPF) * n16);
        asm volatile("cp.async.wait_group %0;" ::"n"(NPF - 1) : "memory");
        __syncwarp();
        float acc = 0.0f;
        for (int c0 = 0; c0 < nb; c0 += MV_CHUNK) {
            const int nc = min(MV_CHUNK, nb - c0);
            for (int p0 = 0; p0 < nc; p0 += 4) {
                const int p = p0 + g;
                const bool valid = p < nc;
                int is = 0, ms = 0;
                const uint8_t *blk = row_s + (size_t)(c0 + p) * BB;
                const uint8_t *ab = act + (size_t)(c0 + p) * ABB;
                if (valid) block_part<SLoad>(DT, blk, ab, j, is, ms);
                group8_sum(is, ms);
                if (valid && j == 0) {
                    float dA, dM;
                    block_scales<SLoad>(DT, blk, ab, dA, dM);
                    part[warp][p] = BlockPart{ is, ms, dA, dM };
                }
            }
            __syncwarp();
            if (lane == 0)
                for (int p = 0; p < nc; p++) {
                    BlockPart q = part[warp][p];
                    acc = chain_step(DT, acc, q.dA, q.dM, q.is, q.ms);
                }
            __syncwarp();
        }
        if (lane == 0) y[row] = res ? __fadd_rn(res[row], acc) : acc;
    }
}

using MvFn = void (*)(const uint8_t *, size_t, const uint8_t *, float *, int, int64_t, int64_t, const float *);
template <int NPF>
static MvFn pick_mv(int dt) {
    switch (dt) {
    case DT_Q4_K: return k_matvec_qs<DT_Q4_K, NPF>;
    case DT_Q5_K: return k_matvec_qs<DT_Q5_K, NPF>;
    case DT_Q6_K: return k_matvec_qs<DT_Q6_K, NPF>;
    case DT_Q8_0: return k_matvec_qs<DT_Q8_0, NPF>;
    case DT_Q8_K: return k_matvec_qs<DT_Q8_K, NPF>;
    default: return nullptr;
    }
}

#ifndef TLMG_MVF_U
#define TLMG_MVF_U 32
#endif
constexpr int MVF_U = TLMG_MVF_U;   // loads in flight per lane in the float matvec

// Float weights: element i into lane i mod 32 with fmaf, then the fixed
// tree (reference tlm_quant.c:724-770).
template <int A>
__global__ void __launch_bounds__(MV_WARPS * 32)
k_matvec_f(int dt, const uint8_t *__restrict__ W, size_t rb, const float *__restrict__ x,
           float *y, int64_t n, int64_t r0, int64_t r1, const float *res) {
    pdl_enter();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int64_t row = r0 + (int64_t)blockIdx.x * nw + warp; row < r1; row += (int64_t)gridDim.x * nw) {
        const uint8_t *wr = W + (size_t)row * rb;
        float acc = 0.0f;
        auto wload = [&](int64_t i) -> float {
            if (dt == DT_F32) return __uint_as_float(WLoad<A>::u32(wr + 4 * i));
            if (dt == DT_F16) return f16_to_f32(WLoad<(A < 2 ? A : 2)>::u16(wr + 2 * i));
            return bf16_to_f32(WLoad<(A < 2 ? A : 2)>::u16(wr + 2 * i));
        };
        int64_t i = lane;
        // MVF_U elements' loads issued together, then their fmaf chain in order
        for (; i + (MVF_U - 1) * 32 < n; i += MVF_U * 32) {
            float wv[MVF_U], xv[MVF_U];
#pragma unroll
            for (int u = 0; u < MVF_U; u++) {
                wv[u] = wload(i + 32 * u);
                xv[u] = __ldg(x + i + 32 * u);
            }
#pragma unroll
            for (int u = 0; u < MVF_U; u++) acc = __fmaf_rn(wv[u], xv[u], acc);
        }
        for (; i < n; i += 32) acc = __fmaf_rn(wload(i), __ldg(x + i), acc);
        acc = tree32(acc);
        if (lane == 0) y[row] = res ? __fadd_rn(res[row], acc) : acc;
    }
}

static int align_of(uintptr_t a) {
    if ((a & 15u) == 0) return 16;
    if ((a & 3u) == 0) return 4;
    if ((a & 1u) == 0) return 2;
    return 1;
}

static unsigned mv_grid(int64_t rows) {
    int64_t g = (rows + MV_WARPS - 1) / MV_WARPS;
    if (g > 148 * 16) g = 148 * 16;
    return (unsigned)(g < 1 ? 1 : g);
}

__global__ void k_fill_nan(float *y, int64_t r0, int64_t r1) {
    int64_t r = r0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r < r1) y[r] = __uint_as_float(0x7FC00000u);
}

int launch_matvec(int dt, const void *Wv, size_t rb, const void *act, float *y, int64_t n, int64_t r0,
                  int64_t r1, cudaStream_t st, const float *res) {
    int qk = dt_block(dt);
    if (qk == 0 || n < 0 || n % qk) {
        if (r1 > r0) {
            k_fill_nan<<<(unsigned)((r1 - r0 + 255) / 256), 256, 0, st>>>(y, r0, r1);
            count_launch();
        }
        return set_error(TLMG_EINVAL, "matvec_rows: bad dtype %d or n=%lld", dt, (long long)n);
    }
    if (r1 <= r0) return TLMG_OK;
    const uint8_t *W = (const uint8_t *)Wv;
    int A = align_of((uintptr_t)W | (uintptr_t)rb | (uintptr_t)(qk > 1 ? dt_block_bytes(dt) : 16));
    unsigned grid = mv_grid(r1 - r0);
    const unsigned thr = MV_WARPS * 32;
    // fewer warps per CTA when there are few rows, so that they spread over the SMs
    const int64_t rows = r1 - r0;
    const int nw = (int)std::max<int64_t>(1, std::min<int64_t>(MV_WARPS, rows / 148));
    const unsigned grid_nw = (unsigned)std::max<int64_t>(1, std::min<int64_t>((rows + nw - 1) / nw, 148 * 32));
    const size_t row_used = (size_t)(n / qk) * dt_block_bytes(dt);
    // tall matrices: more row buffers a warp (each warp walks many rows); an
    // lm_head of 151,936 Q6_K rows measured 129.6 us with 2, 123.1 with 3
    // and 124.9 with 4 (graph-timed, B200): the kernel is issue-bound
#ifndef TLMG_MV_TALL_NPF
#define TLMG_MV_TALL_NPF 3
#endif
    const int npf = rows >= 65536 && row_used <= 4096 ? TLMG_MV_TALL_NPF : 2;
    MvFn mv = npf == 4 ? pick_mv<4>(dt) : npf == 3 ? pick_mv<3>(dt) : pick_mv<2>(dt);
    if (mv && ((uintptr_t)W & 15u) == 0 && rb % 16 == 0 && row_used % 16 == 0 && row_used <= 8192) {
        // MV_WARPS warps a CTA, npf row buffers a warp; as many CTAs as are resident.
        // Each instance is opted in once to 160 KB of dynamic shared memory
        // (its static `part` array comes on top of the dynamic bytes).
        const size_t sm = (size_t)npf * row_used * MV_WARPS;
        static thread_local std::vector<const void *> opted;
        bool ok = std::find(opted.begin(), opted.end(), (const void *)mv) != opted.end();
        if (!ok) {
            ok = cudaFuncSetAttribute((const void *)mv, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024) ==
                 cudaSuccess;
            if (ok) opted.push_back((const void *)mv);
            else cudaGetLastError();
        }
        if (ok && sm <= 160 * 1024) {
            int per_sm = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, (const void *)mv, MV_WARPS * 32, sm) !=
                    cudaSuccess ||
                per_sm < 1) {
                cudaGetLastError();
                per_sm = 1;
            }
            const int nsm = 148;
            const int64_t need = (rows + MV_WARPS - 1) / MV_WARPS;
            const unsigned gq = (unsigned)std::max<int64_t>(1, std::min<int64_t>(need, (int64_t)per_sm * nsm));
            cudaError_t e = launch_k(mv, gq, MV_WARPS * 32, sm, st, W, rb, (const uint8_t *)act, y, (int)(n / qk), r0,
                                     r1, res);
            count_launch();
            if (e == cudaSuccess) e = cudaGetLastError();
            return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "matvec_rows launch");
        }
    }
    if (qk == 1) {
        const float *x = (const float *)act;
        grid = grid_nw;
        const unsigned thr_f = 32 * nw;
        switch (A) {
        case 16: case 4: launch_k(k_matvec_f<4>, grid, thr_f, 0, st, dt, W, rb, x, y, n, r0, r1, res); break;
        case 2: launch_k(k_matvec_f<2>, grid, thr_f, 0, st, dt, W, rb, x, y, n, r0, r1, res); break;
        default: launch_k(k_matvec_f<1>, grid, thr_f, 0, st, dt, W, rb, x, y, n, r0, r1, res); break;
        }
    } else {
        const uint8_t *a = (const uint8_t *)act;
        switch (A) {
        case 16: launch_k(k_matvec_q<16>, grid, thr, 0, st, dt, W, rb, a, y, n, r0, r1, res); break;
        case 4: launch_k(k_matvec_q<4>, grid, thr, 0, st, dt, W, rb, a, y, n, r0, r1, res); break;
        case 2: launch_k(k_matvec_q<2>, grid, thr, 0, st, dt, W, rb, a, y, n, r0, r1, res); break;
        default: launch_k(k_matvec_q<1>, grid, thr, 0, st, dt, W, rb, a, y, n, r0, r1, res); break;
        }
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "matvec_rows launch");
}

// ---------------------------------------------------------------------------
// exact per-block integer partials of rows [0, nrows)
template <int A>
__global__ void __launch_bounds__(MV_WARPS * 32)
k_partials(int dt, const uint8_t *__restrict__ W, size_t rb, const uint8_t *__restrict__ act, int64_t n,
           int64_t nrows, int32_t *__restrict__ isum, int32_t *__restrict__ msum) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 3, j = lane & 7;
    const int qk = dt_block(dt), bb = dt_block_bytes(dt), abb = act_block_bytes(act_kind_for(dt));
    const int nb = (int)(n / qk);
    for (int64_t row = (int64_t)blockIdx.x * MV_WARPS + warp; row < nrows; row += (int64_t)gridDim.x * MV_WARPS) {
        const uint8_t *wr = W + (size_t)row * rb;
        for (int p0 = 0; p0 < nb; p0 += 4) {
            int p = p0 + g;
            bool valid = p < nb;
            int is = 0, ms = 0;
            if (valid) block_part<WLoad<A>>(dt, wr + (size_t)p * bb, act + (size_t)p * abb, j, is, ms);
            group8_sum(is, ms);
            if (valid && j == 0) {
                isum[row * nb + p] = is;
                msum[row * nb + p] = ms;
            }
        }
    }
}

// ---------------------------------------------------------------------------
__global__ void k_route(int router, const float *__restrict__ logits, const uint8_t *__restrict__ mask,
                        const float *__restrict__ bias, int E, int k, float routed_scale, int32_t *ids, float *w) {
    __shared__ uint32_t scratch[RT_SCRATCH];
    __shared__ int32_t ids_sm[64];
    __shared__ float w_sm[64];
    warp_route(router, logits, mask, bias, E, k, routed_scale, scratch, ids_sm, w_sm, threadIdx.x & 31);
    if (threadIdx.x < k) {
        ids[threadIdx.x] = ids_sm[threadIdx.x];
        w[threadIdx.x] = w_sm[threadIdx.x];
    }
}

int launch_route(int router, const float *logits, const uint8_t *mask, const float *bias, int E, int k,
                 float routed_scale, int32_t *ids, float *w, cudaStream_t st) {
    if (E <= 0 || E > RT_PER * 32 || k <= 0 || k > E || k > 64 || router < 0 || router > 2)
        return set_error(TLMG_EINVAL, "route: unsupported E=%d k=%d router=%d (E <= %d, k <= 64)", E, k,
                         router, RT_PER * 32);
    k_route<<<1, 32, 0, st>>>(router, logits, mask, bias, E, k, routed_scale, ids, w);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "route launch");
}

}  // namespace tlmg

using namespace tlmg;

// ---------------------------------------------------------------------------
// C ABI (kernel level)
extern "C" {

const char *tlmg_errmsg(void) { return t_errmsg; }
const char *tlmg_tier(void) { return "cuda-sm100a"; }

int tlmg_init(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return set_error(TLMG_EUNSUP, "no CUDA device (%s)", cudaGetErrorString(e));
    if (device < 0 || device >= n) return set_error(TLMG_EINVAL, "device %d out of range (have %d)", device, n);
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, device);
    if (prop.major != 10) return set_error(TLMG_EUNSUP, "device %d is sm_%d%d; this library is built for sm_100a",
                                           device, prop.major, prop.minor);
    pick_stream(nullptr);
    return TLMG_OK;
}

int tlmg_sync(void *stream) {
    cudaError_t e = cudaStreamSynchronize(pick_stream(stream));
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "stream synchronize");
}

int tlmg_dtype_block(int dt) { return dt_block(dt); }
size_t tlmg_dtype_block_bytes(int dt) { return (size_t)dt_block_bytes(dt); }
size_t tlmg_row_bytes(int dt, int64_t n) {
    int qk = dt_block(dt);
    if (!qk || n < 0 || n % qk) return 0;
    return (size_t)(n / qk) * (size_t)dt_block_bytes(dt);
}
size_t tlmg_qact_bytes(int kind, int64_t n) {
    if (n < 0) return 0;
    if (kind == DT_Q8_K) return (size_t)((n + 255) / 256) * 292u;
    if (kind == DT_Q8_0) return (size_t)((n + 31) / 32) * 36u;
    if (kind == DT_F32) return (size_t)n * 4u;
    return 0;
}
int tlmg_act_kind_for(int wdt) { return act_kind_for(wdt); }

int tlmg_quantize_act(int kind, const float *x, int64_t n, void *dst, void *stream) {
    return launch_quant_act(kind, x, n, dst, pick_stream(stream));
}

int tlmg_matvec_rows(int dt, const void *W, size_t row_bytes, const void *act, float *y, int64_t n, int64_t r0,
                     int64_t r1, void *stream) {
    return launch_matvec(dt, W, row_bytes, act, y, n, r0, r1, pick_stream(stream));
}

int tlmg_block_partials(int dt, const void *W, size_t row_bytes, const void *act, int64_t n, int64_t nrows,
                        int32_t *isum, int32_t *msum, void *stream) {
    int qk = dt_block(dt);
    if (qk <= 1 || n < 0 || n % qk) return set_error(TLMG_EINVAL, "block_partials: bad dtype %d or n=%lld", dt, (long long)n);
    if (nrows <= 0) return TLMG_OK;
    cudaStream_t st = pick_stream(stream);
    const uint8_t *Wb = (const uint8_t *)W;
    const uint8_t *a = (const uint8_t *)act;
    int A = align_of((uintptr_t)Wb | (uintptr_t)row_bytes | (uintptr_t)dt_block_bytes(dt));
    unsigned grid = mv_grid(nrows);
    const unsigned thr = MV_WARPS * 32;
    switch (A) {
    case 16: k_partials<16><<<grid, thr, 0, st>>>(dt, Wb, row_bytes, a, n, nrows, isum, msum); break;
    case 4: k_partials<4><<<grid, thr, 0, st>>>(dt, Wb, row_bytes, a, n, nrows, isum, msum); break;
    case 2: k_partials<2><<<grid, thr, 0, st>>>(dt, Wb, row_bytes, a, n, nrows, isum, msum); break;
    default: k_partials<1><<<grid, thr, 0, st>>>(dt, Wb, row_bytes, a, n, nrows, isum, msum); break;
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "block_partials launch");
}

int tlmg_route(int router, const float *logits, const uint8_t *mask, const float *bias, int E, int k,
               float routed_scale, int32_t *ids, float *w, void *stream) {
    return launch_route(router, logits, mask, bias, E, k, routed_scale, ids, w, pick_stream(stream));
}

// Host-buffer adapters for the reference's tier table (tlm_qmv_fn /
// tlm_qdot_fn). Synchronous; NaN on any failure.
void tlmg_qmv_host(int dt, const void *W, size_t row_bytes, const void *act, float *y, int64_t n, int64_t nrows) {
    if (nrows <= 0) return;
    auto fail = [&](int code, const char *what) {
        set_error(code, "qmv_host: %s", what);
        for (int64_t r = 0; r < nrows; r++) y[r] = NAN;
    };
    int qk = dt_block(dt);
    if (!qk || n < 0 || n % qk) return fail(TLMG_EINVAL, "bad dtype or width");
    size_t wbytes = (size_t)(nrows - 1) * row_bytes + tlmg_row_bytes(dt, n);
    size_t abytes = qk == 1 ? (size_t)n * 4 : tlmg_qact_bytes(act_kind_for(dt), n);
    size_t woff = (uintptr_t)W & 15u;   // keep the caller's byte alignment
    cudaStream_t st = pick_stream(nullptr);
    uint8_t *dW = nullptr, *dA = nullptr;
    float *dy = nullptr;
    if (cudaMalloc(&dW, wbytes + woff + 16) != cudaSuccess || cudaMalloc(&dA, abytes + 16) != cudaSuccess ||
        cudaMalloc(&dy, (size_t)nrows * 4) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(dW); cudaFree(dA); cudaFree(dy);
        return fail(TLMG_ENOMEM, "device allocation failed");
    }
    bool ok = cudaMemcpyAsync(dW + woff, W, wbytes, cudaMemcpyHostToDevice, st) == cudaSuccess &&
              cudaMemcpyAsync(dA, act, abytes, cudaMemcpyHostToDevice, st) == cudaSuccess;
    if (ok) ok = launch_matvec(dt, dW + woff, row_bytes, dA, dy, n, 0, nrows, st) == TLMG_OK;
    if (ok) ok = cudaMemcpyAsync(y, dy, (size_t)nrows * 4, cudaMemcpyDeviceToHost, st) == cudaSuccess;
    if (ok) ok = cudaStreamSynchronize(st) == cudaSuccess;
    cudaFree(dW); cudaFree(dA); cudaFree(dy);
    if (!ok) fail(TLMG_EIO, "device copy or launch failed");
}

float tlmg_qdot_host(int dt, const void *wrow, const void *act, int64_t n, const float *aux) {
    (void)aux;   // per-128-column FP8 scales in the reference; no dtype of this tier reads it
    float y = NAN;
    tlmg_qmv_host(dt, wrow, tlmg_row_bytes(dt, n), act, &y, n, 1);
    return y;
}

}  // extern "C"
