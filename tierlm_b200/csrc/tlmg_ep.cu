// tlmg_ep.cu - expert parallelism over peer memory (one process per GPU).
//
// The reference computes every routed expert of a token in one process
// (run_batch + the rank-ordered combine, src/lib/tlm_model.c:900-938,
// :1029-1036). Here expert e of every layer is owned by GPU
// floor(e * N / E) and one layer call runs, with no host synchronisation and
// no collective library in the data path:
//
//   home     quantise x, route, group the (token, rank) pairs by owner
//            (k_epcount) and write each pair's record straight into the
//            owner's receive buffer, region [home][pair slot], and the
//            region's record count into the owner's count array (k_ep_send)
//   barrier  every GPU tells every peer it is done (a flag in the peer's
//            memory) and waits, bounded, for all peers' flags (k_ep_barrier)
//   owner    the expert FFN of every received record (the grouped
//            tensor-core kernels of the batched path, over the N regions),
//            then each output row written straight into its home's row
//            buffer, region [owner][pair slot] (k_ep_return)
//   barrier  as above
//   home     ffn[t] = sum_r w[t, r] * row(t, r) in ascending r (k_bcombine)
//
// Every row is computed exactly as on one GPU and the combine keeps rank
// order, so the result is bit-identical for any N. Peer buffers are CUDA IPC
// mappings of each rank's one allocation (plain loads and stores over
// NVLink; no multicast, no TMA). Every wait is bounded: an expired barrier
// raises an error bit that the host reads at the next check.
#include <algorithm>
#include <cstring>
#include <vector>

#include "tlmg_batch.cuh"
#include "tlmg_dev.cuh"
#include "tlmg_internal.h"

namespace tlmg {

constexpr int EPP_MAX = EPP_SLOTS;               // ranks of one exchange
constexpr uint64_t EPP_WAIT_NS = 1000000000ull;  // 1 s: a barrier gives up

struct PeerPtrs {
    uint8_t *recv[EPP_MAX];      // each rank's record regions [N][cap][RB]
    int32_t *rcnt[EPP_MAX];      // each rank's record counts [N]
    float *back[EPP_MAX];        // each rank's output-row regions [N][cap][D]
    uint32_t *flags[EPP_MAX];    // each rank's barrier flags [2][N]
};

__device__ __forceinline__ uint64_t ep_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One warp per pair: the pair's record { int32 expert id, 12 zero bytes, the
// token's quantised vector } into region [me][slot] of its owner's receive
// buffer, slot = perm[p] - the owner's first record index; thread 0 of block
// 0 writes the record counts into every owner's count array.
__global__ void k_ep_send(const int32_t *__restrict__ ids, const int32_t *__restrict__ perm,
                          const int32_t *__restrict__ cnt, int np, int k, int E, int nr, int me, int cap,
                          const uint8_t *__restrict__ xq, uint32_t qx, size_t rec, PeerPtrs pp,
                          int32_t *__restrict__ slot_of) {
    __shared__ int first[EPP_MAX];
    if (threadIdx.x == 0) {
        int s = 0;
        for (int d = 0; d < nr; d++) {
            first[d] = s;
            s += cnt[d];
        }
    }
    __syncthreads();
    if (blockIdx.x == 0 && (int)threadIdx.x < nr) pp.rcnt[threadIdx.x][me] = cnt[threadIdx.x];
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
    for (int p = gw; p < np; p += nw) {
        const int d = (int)((int64_t)ids[p] * nr / E);
        const int slot = perm[p] - first[d];
        uint8_t *dst = pp.recv[d] + ((size_t)me * cap + slot) * rec;
        const uint4 *src = reinterpret_cast<const uint4 *>(xq + (size_t)(p / k) * qx);
        if (lane == 0) {
            *reinterpret_cast<uint4 *>(dst) = make_uint4((uint32_t)ids[p], 0u, 0u, 0u);
            slot_of[p] = d * cap + slot;   // where the pair's output row comes back
        }
        for (uint32_t i = lane; i < qx / 16; i += 32) reinterpret_cast<uint4 *>(dst + 16)[i] = __ldg(src + i);
    }
    __threadfence_system();   // the peer writes are performed before the barrier's flags
}

// Every received record's output row (eo, local, [N][cap][D]) into region
// [me][slot] of its home's row buffer: one block per (home, slot) row.
__global__ void k_ep_return(const float *__restrict__ eo, const int32_t *__restrict__ rcnt, int nr, int me, int cap,
                            int D, PeerPtrs pp) {
    for (int q = blockIdx.x; q < nr * cap; q += gridDim.x) {
        const int s = q / cap, j = q - s * cap;
        if (j >= rcnt[s]) continue;
        const float4 *src = reinterpret_cast<const float4 *>(eo + (size_t)q * D);
        float4 *dst = reinterpret_cast<float4 *>(pp.back[s] + ((size_t)me * cap + j) * D);
        for (int i = threadIdx.x; i < D / 4; i += blockDim.x) dst[i] = src[i];
    }
    __threadfence_system();
}

// Barrier `which` (0 or 1) of call `epoch`: thread d raises this rank's flag
// in rank d's memory, then waits (bounded) for rank d's flag in its own.
__global__ void k_ep_barrier(PeerPtrs pp, int nr, int me, int which, uint32_t epoch, uint32_t *err) {
    const int d = threadIdx.x;
    if (d >= nr) return;
    __threadfence_system();
    st_release_sys(pp.flags[d] + which * EPP_MAX + me, epoch);
    const uint32_t *mine = pp.flags[me] + which * EPP_MAX + d;
    if (ld_acquire_sys(mine) == epoch) return;
    const uint64_t t0 = ep_now();
    while (ld_acquire_sys(mine) != epoch) {
        if (ep_now() - t0 > EPP_WAIT_NS) {
            *reinterpret_cast<volatile uint32_t *>(err) = 1u;   // the host reports TLMG_EIO at its next check
            return;
        }
        __nanosleep(256);
    }
}

static PeerPtrs peer_ptrs(const EpP2P &e) {
    PeerPtrs pp{};
    for (int r = 0; r < e.nr; r++) {
        pp.recv[r] = e.peer[r];
        pp.rcnt[r] = reinterpret_cast<int32_t *>(e.peer[r] + e.off_rcnt);
        pp.back[r] = reinterpret_cast<float *>(e.peer[r] + e.off_back);
        pp.flags[r] = reinterpret_cast<uint32_t *>(e.peer[r] + e.off_flags);
    }
    return pp;
}

static size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

int epp_alloc(EpP2P &e, int me, int nr, int max_tok, int D, int k) {
    epp_release(e);
    if (nr < 1 || nr > EPP_MAX || me < 0 || me >= nr || max_tok < 1 || D % 256)
        return set_error(TLMG_EINVAL, "ep: rank %d of %d (at most %d), %d tokens", me, nr, EPP_MAX, max_tok);
    e.me = me;
    e.nr = nr;
    e.max_tok = max_tok;
    e.cap = max_tok * k;
    e.rb = ep_record_bytes(D);
    const size_t recv = up256((size_t)nr * e.cap * e.rb);
    e.off_rcnt = recv;
    e.off_back = e.off_rcnt + 256;
    e.off_flags = e.off_back + up256((size_t)nr * e.cap * D * 4);
    e.bytes = e.off_flags + 256;
    const size_t np = (size_t)e.cap;
    if (cudaMalloc(&e.base, e.bytes) != cudaSuccess || cudaMalloc(&e.cnt, 4 * EPP_MAX) != cudaSuccess ||
        cudaMalloc(&e.perm, 4 * np) != cudaSuccess || cudaMalloc(&e.slot_of, 4 * np) != cudaSuccess ||
        cudaMalloc(&e.eo, (size_t)nr * e.cap * D * 4) != cudaSuccess ||
        cudaHostAlloc(&e.err_host, 64, cudaHostAllocMapped) != cudaSuccess) {
        cudaGetLastError();
        epp_release(e);
        return set_error(TLMG_ENOMEM, "ep: buffers for %d ranks x %d tokens", nr, max_tok);
    }
    *e.err_host = 0;
    cudaHostGetDevicePointer((void **)&e.err_dev, e.err_host, 0);
    cudaMemset(e.base + e.off_rcnt, 0, 256);
    cudaMemset(e.base + e.off_flags, 0, 256);
    cudaDeviceSynchronize();   // zeroed before any peer maps the allocation
    for (int r = 0; r < EPP_MAX; r++) e.peer[r] = nullptr;
    e.peer[me] = e.base;
    e.epoch = 0;
    return TLMG_OK;
}

void epp_release(EpP2P &e) {
    for (int r = 0; r < EPP_MAX; r++)
        if (e.opened[r] && e.peer[r]) cudaIpcCloseMemHandle(e.peer[r]);
    for (void *p : { (void *)e.base, (void *)e.cnt, (void *)e.perm, (void *)e.slot_of, (void *)e.eo })
        if (p) cudaFree(p);
    if (e.err_host) cudaFreeHost(e.err_host);
    e = EpP2P{};
}

void epp_send(const EpP2P &e, const int32_t *ids, int np, int k, int E, const uint8_t *xq, uint32_t qx,
              cudaStream_t st) {
    const unsigned blocks = (unsigned)std::max(1, std::min((np + 7) / 8, 1184));
    k_ep_send<<<blocks, 256, 0, st>>>(ids, e.perm, e.cnt, np, k, E, e.nr, e.me, e.cap, xq, qx, e.rb, peer_ptrs(e),
                                      e.slot_of);
}

void epp_return(const EpP2P &e, int D, cudaStream_t st) {
    const int32_t *rcnt = reinterpret_cast<const int32_t *>(e.base + e.off_rcnt);
    k_ep_return<<<(unsigned)std::min(e.nr * e.cap, 1184), 128, 0, st>>>(e.eo, rcnt, e.nr, e.me, e.cap, D,
                                                                         peer_ptrs(e));
}

void epp_barrier(const EpP2P &e, int which, cudaStream_t st) {
    k_ep_barrier<<<1, 32, 0, st>>>(peer_ptrs(e), e.nr, e.me, which, e.epoch, e.err_dev);
}

}  // namespace tlmg
