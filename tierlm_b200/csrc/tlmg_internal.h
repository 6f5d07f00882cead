// tlmg_internal.h - host-side helpers shared by the library's .cu files.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/tlmg.h"

namespace tlmg {

// printf-style; stores the thread-local message and returns `code`.
int set_error(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
// CUDA error -> TLMG_EIO with a message naming the failing step.
int cuda_fail(cudaError_t e, const char *what);

// The calling thread's library stream on the current device (created by
// tlmg_init); `user` overrides it when non-NULL.
cudaStream_t pick_stream(void *user);

// Kernel launches issued through the library (host-side counter).
void count_launch(int n = 1);
int64_t launches_total();

// Programmatic dependent launch of the decoder step's kernels: while a
// thread has it on, the launchers below start their kernels with
// programmatic stream serialisation (the kernel may be scheduled while its
// predecessor finishes; every such kernel waits in griddepcontrol.wait
// before it reads anything its predecessor wrote).
void set_pdl(bool on);
bool pdl_on();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_on() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, static_cast<KArgs>(args)...);
}

// Launchers of the kernel-level ops (also used by the layer code).
int launch_quant_act(int kind, const float *x, int64_t n, void *dst, cudaStream_t st);
// With res: y[r] = res[r] + dot (res may be y itself).
int launch_matvec(int dt, const void *W, size_t rb, const void *act, float *y, int64_t n, int64_t r0,
                  int64_t r1, cudaStream_t st, const float *res = nullptr);
int launch_route(int router, const float *logits, const uint8_t *mask, const float *bias, int E, int k,
                 float routed_scale, int32_t *ids, float *w, cudaStream_t st);

bool is_device_ptr(const void *p);

// Device scratch of tlmg_decode_attention (tlmg_attn.cu).
size_t attention_work_bytes(int mode, int kv_dt, int T, int H, int KV, int hd);
// tlmg_decode_attention with launch geometry for T positions; with dT the
// kernels read the actual count (1..T) from device memory (graph replay).
int decode_attention_impl(int mode, int kv_dt, const float *q, const void *k_pages, const void *v_pages, int n_pages,
                          const int32_t *page_table, int page_size, int T, const int32_t *dT, int H, int KV, int hd,
                          void *work, size_t work_bytes, float *out, cudaStream_t st);

}  // namespace tlmg
