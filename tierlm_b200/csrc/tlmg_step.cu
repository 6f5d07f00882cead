// tlmg_step.cu - kernels of the GPU decoder step that the MoE block does
// not already have: the embedding row (tlm_dequantize_row,
// src/lib/tlm_quant.c:629-675) and the per-head part of attention()
// (src/lib/tlm_model.c:730-763: qk-norm, NeoX RoPE, the K/V write).
// Every value is formed with the reference's float operations in its order
// (the library is built without FMA contraction), so both are bit-exact.
#include <algorithm>
#include <cuda_bf16.h>

#include "tlmg_dev.cuh"
#include "tlmg_internal.h"
#include "tlmg_step.cuh"

namespace tlmg {

__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
__device__ __forceinline__ float ld_f16b(const uint8_t *p) { return f16_to_f32(ld_u16(p)); }

// Element i of a row of dtype dt (row at any byte alignment).
__device__ float dequant_at(int dt, const uint8_t *row, int i) {
    switch (dt) {
    case DT_F32: {
        const uint32_t u = ld_u16(row + 4 * i) | (ld_u16(row + 4 * i + 2) << 16);
        return __uint_as_float(u);
    }
    case DT_F16: return ld_f16b(row + 2 * i);
    case DT_BF16: return bf16_to_f32(ld_u16(row + 2 * i));
    case DT_Q8_0: {
        const uint8_t *b = row + 34 * (i / 32);
        return __fmul_rn(ld_f16b(b), (float)(int8_t)b[2 + i % 32]);
    }
    case DT_Q8_K: {
        const uint8_t *b = row + 292 * (i / 256);
        const uint32_t u = ld_u16(b) | (ld_u16(b + 2) << 16);
        return __fmul_rn(__uint_as_float(u), (float)(int8_t)b[4 + i % 256]);
    }
    case DT_Q4_K:
    case DT_Q5_K: {
        // deq_kq_affine: sub-block 2c + hi of 32 values, y = d*sc * q - dmin*mn
        const bool q5 = dt == DT_Q5_K;
        const uint8_t *b = row + (q5 ? 176 : 144) * (i / 256);
        const int e = i % 256, c = e / 64, hi = (e % 64) / 32, l = e % 32, sb = 2 * c + hi;
        const uint32_t a0 = ld_u16(b + 4) | (ld_u16(b + 6) << 16), a1 = ld_u16(b + 8) | (ld_u16(b + 10) << 16),
                       a2 = ld_u16(b + 12) | (ld_u16(b + 14) << 16);
        int sc, mn;
        kq_scale_min(a0, a1, a2, sb, sc, mn);
        const uint8_t qb = b[(q5 ? 48 : 16) + 32 * c + l];
        int q = hi ? qb >> 4 : qb & 15;
        if (q5) q |= ((b[16 + l] >> sb) & 1) << 4;
        const float d0 = __fmul_rn(ld_f16b(b), (float)sc), m0 = __fmul_rn(ld_f16b(b + 2), (float)mn);
        return __fsub_rn(__fmul_rn(d0, (float)q), m0);
    }
    case DT_Q6_K: {
        // deq_q6_k: element e = 128 h + 32 k + l takes its low nibble from
        // ql[64 h + 32 (k & 1) + l] (k < 2: low half of the byte, else high)
        // and bits 2k..2k+1 of qh[32 h + l]
        const uint8_t *b = row + 210 * (i / 256);
        const int e = i % 256, h = e / 128, kq = (e % 128) / 32, l = e % 32;
        const uint8_t ql = b[64 * h + 32 * (kq & 1) + l], qh = b[128 + 32 * h + l];
        const int u = ((kq < 2 ? ql & 15 : ql >> 4) | (((qh >> (2 * kq)) & 3) << 4)) - 32;
        return __fmul_rn(__fmul_rn(ld_f16b(b + 208), (float)(int8_t)b[192 + e / 16]), (float)u);
    }
    default: return __uint_as_float(0x7FC00000u);
    }
}

__global__ void k_embed_row(int dt, const uint8_t *__restrict__ base, size_t rb, int token,
                            const int32_t *__restrict__ dargs, int n, float *__restrict__ out) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (dargs) token = dargs[0];
    if (i < n) out[i] = dequant_at(dt, base + (size_t)token * rb, i);
}

__global__ void k_step_args(int32_t *dargs, int token, int pos) {
    pdl_enter();
    dargs[0] = token;
    dargs[1] = pos;
    dargs[2] = pos + 1;
}

int step_set_args(int32_t *dargs, int token, int pos, cudaStream_t st) {
    k_step_args<<<1, 1, 0, st>>>(dargs, token, pos);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "step arguments launch");
}

int step_embed(int dt, const uint8_t *base, size_t rb, int token, const int32_t *dargs, int D, float *h,
               cudaStream_t st) {
    const int qk = dt_block(dt);
    if (qk == 0 || D % qk || dt == DT_MXFP4) return set_error(TLMG_EUNSUP, "embedding dtype %d", dt);
    cudaError_t e = launch_k(k_embed_row, (D + 255) / 256, 256, 0, st, dt, base, rb, token, dargs, D, h);
    count_launch();
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "embedding launch");
}

__device__ __forceinline__ void kv_store(float *p, float v) { *p = v; }
__device__ __forceinline__ void kv_store(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

// One block per head (H q heads, then KV k heads), hd threads: the head's
// RMSNorm with the layer's q_norm / k_norm weights when present (rmsnorm in
// place, src/lib/tlm_model.c:744-747), then rope() (:720-727): pairs (j,
// j + hd/2), a' = a cs - b sn, b' = b cs + a sn. k-head blocks then store
// k and v of position pos into the layer's page (pages [KV][page][hd]).
template <typename KT>
__global__ void k_heads(float *__restrict__ qkv, int H, int KV, int hd, const float *__restrict__ q_norm,
                        const float *__restrict__ k_norm, float eps, const float *__restrict__ rope_all,
                        KT *__restrict__ kpage, KT *__restrict__ vpage, int page, int pos,
                        const int32_t *__restrict__ dargs) {
    pdl_enter();
    __shared__ double red[32];
    __shared__ float r_sh;
    __shared__ float v[256];
    if (dargs) pos = dargs[1];
    const float *rope = rope_all + (size_t)pos * hd;
    const int b = blockIdx.x, i = threadIdx.x, half = hd / 2;
    const bool is_q = b < H;
    float *x = qkv + (size_t)b * hd;   // q heads [H][hd] then k heads [KV][hd]
    const float *nw = is_q ? q_norm : k_norm;
    float xi = x[i];
    if (nw) {
        const float r = block_rms_inv(x, hd, eps, red, &r_sh);
        xi = __fmul_rn(__fmul_rn(xi, r), nw[i]);
    }
    v[i] = xi;
    __syncthreads();
    const float *cs = rope, *sn = rope + half;
    const int j = i < half ? i : i - half;
    const float o = i < half ? __fsub_rn(__fmul_rn(v[i], cs[j]), __fmul_rn(v[i + half], sn[j]))
                             : __fadd_rn(__fmul_rn(v[i], cs[j]), __fmul_rn(v[j], sn[j]));
    x[i] = o;
    if (!is_q) {
        const int h = b - H;
        const size_t off = ((size_t)h * page + pos) * hd + i;
        kv_store(kpage + off, o);
        kv_store(vpage + off, qkv[(size_t)(H + KV + h) * hd + i]);
    }
}

int step_heads(const StepModel &m, int l, int pos, const int32_t *dargs, float eps, cudaStream_t st) {
    const StepLayer &A = m.A[l];
    const float *rope = m.rope;
    const size_t per = (size_t)m.KV * m.page * m.hd;   // one layer's page
    if (m.kv_dt == DT_F32) {
        float *kp = static_cast<float *>(m.kpool) + (size_t)l * per, *vp = static_cast<float *>(m.vpool) + (size_t)l * per;
        launch_k(k_heads<float>, m.H + m.KV, m.hd, 0, st, m.qkv, m.H, m.KV, m.hd, A.q_norm, A.k_norm, eps, rope, kp,
                 vp, m.page, pos, dargs);
    } else {
        __nv_bfloat16 *kp = static_cast<__nv_bfloat16 *>(m.kpool) + (size_t)l * per,
                      *vp = static_cast<__nv_bfloat16 *>(m.vpool) + (size_t)l * per;
        launch_k(k_heads<__nv_bfloat16>, m.H + m.KV, m.hd, 0, st, m.qkv, m.H, m.KV, m.hd, A.q_norm, A.k_norm, eps,
                 rope, kp, vp, m.page, pos, dargs);
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "attention heads launch");
}

}  // namespace tlmg

using namespace tlmg;

// rows rows of n elements, row stride rb bytes -> y [rows][n]
__global__ void k_dequant_rows(int dt, const uint8_t *__restrict__ src, size_t rb, int64_t n, int64_t rows,
                               float *__restrict__ y) {
    const int64_t total = n * rows;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / n, i = idx - r * n;
        y[idx] = dequant_at(dt, src + (size_t)r * rb, (int)i);
    }
}

extern "C" int tlmg_dequantize_rows(int dt, const void *src, size_t row_bytes, float *y, int64_t n, int64_t rows,
                                    void *stream) {
    const int qk = dt_block(dt);
    if (!src || !y || rows < 0 || n <= 0 || n > INT32_MAX || qk == 0 || n % qk || dt == DT_MXFP4 ||
        row_bytes < tlmg_row_bytes(dt, n))
        return set_error(TLMG_EINVAL, "dequantize_rows: dtype %d, n %lld, row bytes %zu", dt, (long long)n, row_bytes);
    if (rows == 0) return TLMG_OK;
    const int64_t blocks = std::min<int64_t>((n * rows + 255) / 256, 148 * 32);
    k_dequant_rows<<<(unsigned)blocks, 256, 0, pick_stream(stream)>>>(dt, (const uint8_t *)src, row_bytes, n, rows, y);
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TLMG_OK : cuda_fail(e, "dequantize_rows launch");
}
