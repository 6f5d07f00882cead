// tlmg_step.cuh - the whole decoder step on the GPU: embedding row,
// attention block, the MoE block of every layer, final norm and lm_head
// (tlm_model_step, src/lib/tlm_model.c:1058-1103).
#pragma once
#include <cstdint>
#include <vector>
#include <cuda_runtime.h>

namespace tlmg {

// Attention weights of one layer, copied into device memory. When q, k and
// v share a dtype their rows sit back to back in `qkv` ([H*hd | KV*hd |
// KV*hd] rows of D columns) and one matvec computes all three.
struct StepLayer {
    bool set = false;
    float *attn_norm = nullptr;        // [D]
    float *q_norm = nullptr, *k_norm = nullptr;   // [hd] or null
    int dt[4] = { -1, -1, -1, -1 };    // q, k, v, o
    uint8_t *w[4] = {};
    size_t rb[4] = {};
    bool fused_qkv = false;            // w[0] points at the q|k|v block
};

struct StepModel {
    int H = 0, KV = 0, hd = 0, vocab = 0, max_ctx = 0, page = 0;
    int kv_dt = 0, attn_mode = 0;
    float attn_scale = 1.0f;
    std::vector<float> inv_freq;        // [hd / 2]
    std::vector<StepLayer> A;
    int embd_dt = -1;
    uint8_t *embd = nullptr;            // [vocab][embd_rb]
    size_t embd_rb = 0;
    float *out_norm = nullptr;          // [D]
    int head_dt = -1;
    uint8_t *head = nullptr;            // [vocab][head_rb]
    size_t head_rb = 0;
    // KV pages: one page of `page` positions per layer, [L][KV][page][hd]
    void *kpool = nullptr, *vpool = nullptr;
    int32_t *table = nullptr;           // [L]: table[l] = l
    float *awork = nullptr;
    size_t awork_bytes = 0;
    // per-step scratch
    float *qkv = nullptr;               // [(H + 2 KV) * hd]
    float *att = nullptr;               // [H * hd]
    uint8_t *aq = nullptr;              // quantised att (Q8_K or Q8_0)
    float *xb = nullptr;                // [D] normalised h
    uint8_t *xq = nullptr;              // quantised xb
    float *rope = nullptr;              // [max_ctx][hd]: cs | sn of every position
    float *logits = nullptr;            // [vocab]
    int32_t *dargs = nullptr;           // [3] token, position, position + 1 (graph replay)
    // captured steps: [0] without lm_head, [1] with; valid while wgen matches
    cudaGraphExec_t graph[2] = {};
    uint64_t graph_gen[2] = {};
    int64_t graph_launches[2] = {};     // kernels in each graph
    bool use_graphs = true;             // tlmg_step_graphs
    bool graph_off = false;             // capture failed once: eager from then on
    int64_t calls = 0;                  // steps run (the first is always eager)
    int64_t replays = 0, captures = 0;
    // tlm_model_stats counters (tlmg_step_stats): steps, and the device time
    // of the phases of steps run while profiling (events at the boundaries:
    // [0] start, [1 + 2 l] layer l's attention, [2 + 2 l] its MoE block,
    // [2 L + 1] after the layers, [2 L + 2] end)
    uint64_t st_tokens = 0, st_attn_ns = 0, st_moe_ns = 0, st_other_ns = 0;
    std::vector<cudaEvent_t> tev;
    cudaStream_t cap_st = nullptr;      // private stream graphs are captured on (the caller's may be the
                                        // legacy default stream, which cannot be captured)
};

inline void step_graphs_release(StepModel &m) {
    for (cudaEvent_t e : m.tev) cudaEventDestroy(e);
    m.tev.clear();
    for (int h = 0; h < 2; h++)
        if (m.graph[h]) {
            cudaGraphExecDestroy(m.graph[h]);
            m.graph[h] = nullptr;
        }
    if (m.cap_st) cudaStreamDestroy(m.cap_st);
    m.cap_st = nullptr;
}

// Launchers (tlmg_step.cu); all asynchronous on `st`. With dargs (device
// int32 [3]: token, position, position + 1, written by step_set_args) the
// kernels read the token and position from device memory, so that one
// captured graph serves every position; else they take token / pos.
int step_set_args(int32_t *dargs, int token, int pos, cudaStream_t st);
// h = row `token` of the embedding table (rows of rb bytes from base).
int step_embed(int dt, const uint8_t *base, size_t rb, int token, const int32_t *dargs, int D, float *h,
               cudaStream_t st);
// qk-norm (when given), RoPE of the q and k heads in qkv, then k and v of
// the position into layer l's page (device buffers of m; the position's
// RoPE row of m.rope).
int step_heads(const StepModel &m, int l, int pos, const int32_t *dargs, float eps, cudaStream_t st);

}  // namespace tlmg
