/* tlmg.h - C ABI of libtlmg, the B200 (sm_100a) tier of tierlm's quantised
 * MoE decoder step.
 *
 * Plain C: pointers, sizes and integer codes only; no CUDA or torch types
 * in the signatures (a CUDA stream travels as `void *`; NULL = the
 * library's own non-blocking stream, so pass cudaStreamLegacy (0x1) to
 * order work with the legacy default stream). All fallible functions return 0 (TLMG_OK) or a
 * negative code with the same numbering as the reference's TLM_E* codes
 * (src/lib/tlm_platform.h:26-36), and leave a thread-local message for
 * tlmg_errmsg(). Numerics follow the reference contract
 * (src/lib/tlm_quant.h:113-128): exact int32 sums inside a block, then per
 * block acc = fmaf(d_w*d_a, (float)isum, acc) (and the min term for
 * Q4_K/Q5_K) in ascending block order; every result below is bit-identical
 * to the reference scalar kernels given the same inputs.
 *
 * Pointer rules. "device" pointers must be CUDA device (or managed)
 * memory. Entry points marked "host or device" accept either: host
 * buffers are staged through pinned memory by the library and the call
 * returns after the result is back on the host. Activation buffers must be
 * 4-byte aligned (src/lib/tlm_quant.h:105-106); weight rows may start at
 * any byte offset.
 */
#ifndef TLMG_H
#define TLMG_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    TLMG_OK = 0, TLMG_EIO = -1, TLMG_ENOMEM = -2, TLMG_EINVAL = -3, TLMG_EFORMAT = -4,
    TLMG_ERANGE = -5, TLMG_ENOTFOUND = -6, TLMG_EUNSUP = -7, TLMG_EBUSY = -8
};

/* dtype codes = tlm_dtype values (src/lib/tlm_quant.h:31-42). */
enum {
    TLMG_DT_F32 = 0, TLMG_DT_F16 = 1, TLMG_DT_BF16 = 2, TLMG_DT_Q8_0 = 8, TLMG_DT_Q4_K = 12,
    TLMG_DT_Q5_K = 13, TLMG_DT_Q6_K = 14, TLMG_DT_Q8_K = 15, TLMG_DT_MXFP4 = 39
};

/* ---- library --------------------------------------------------------- */
/* Thread-local message of the last failure (replaces tlm_errmsg,
 * src/lib/tlm_platform.h:37). */
const char *tlmg_errmsg(void);
/* Tier name, "cuda-sm100a" (mirrors tlm_quant_tier, src/lib/tlm_quant.h:83). */
const char *tlmg_tier(void);
/* Select the CUDA device for the calling thread and create the library's
 * stream on it (idempotent). */
int tlmg_init(int device);
/* Wait for all work the library queued on `stream` (NULL = its own). */
int tlmg_sync(void *stream);

/* ---- formats (src/lib/tlm_quant.h:45-50, :66) ------------------------ */
int    tlmg_dtype_block(int dt);
size_t tlmg_dtype_block_bytes(int dt);
size_t tlmg_row_bytes(int dt, int64_t n);
size_t tlmg_qact_bytes(int kind, int64_t n);
int    tlmg_act_kind_for(int weight_dt);

/* ---- kernel level (device pointers, asynchronous on `stream`) -------- */
/* Activation quantisation, replaces tlm_quantize_act
 * (src/lib/tlm_quant.h:69, src/lib/tlm_quant.c:458-512). kind = Q8_K,
 * Q8_0 or F32. x: device f32[n]; dst: device, tlmg_qact_bytes(kind, n). */
int tlmg_quantize_act(int kind, const float *x, int64_t n, void *dst, void *stream);

/* y[r] = dot(W[r], act) for r in [r0, r1); replaces tlm_matvec_rows
 * (src/lib/tlm_quant.h:77-79, src/lib/tlm_quant.c:1119-1143). W: device,
 * row_bytes stride, any byte offset; act: device output of
 * tlmg_quantize_act (or f32 for float weights); y: device f32 indexed by
 * absolute row. Bad dtype / width: TLMG_EINVAL and NaN in y[r0..r1). */
int tlmg_matvec_rows(int dt, const void *W, size_t row_bytes, const void *act, float *y,
                     int64_t n, int64_t r0, int64_t r1, void *stream);

/* Dequantisation of `rows` rows of n elements (row stride row_bytes),
 * replaces tlm_dequantize_row (src/lib/tlm_quant.h, src/lib/tlm_quant.c:
 * 629-675) for every dtype but MXFP4 / FP8: src device, y device f32
 * [rows][n], bit-identical to the reference. */
int tlmg_dequantize_rows(int dt, const void *src, size_t row_bytes, float *y, int64_t n, int64_t rows,
                         void *stream);

/* Per-block exact integer partials of rows [0, nrows) (integer formats):
 * isum/msum: device int32[nrows * n/block]. These are the int32 sums the
 * reference's scalar dots form before their fmaf chain
 * (dot_kq_affine_ref / dot_q6_k_ref / dot_q8_0_ref / dot_q8_k_ref /
 * dot_mxfp4_ref, src/lib/tlm_quant.c:778-902); msum is 0 except for
 * Q4_K/Q5_K. For parity checks of the integer stage. */
int tlmg_block_partials(int dt, const void *W, size_t row_bytes, const void *act, int64_t n,
                        int64_t nrows, int32_t *isum, int32_t *msum, void *stream);

/* Router top-k over device logits[E] (route/topk, src/lib/tlm_model.c:
 * 776-839): router 0 = softmax, top-k, renormalise; 1 = softmax, top-k;
 * 2 = sigmoid + bias selection, renormalise. mask (u8[E], 1 = pruned)
 * and bias (f32[E]) may be NULL. ids/w: device int32[k], f32[k]. */
int tlmg_route(int router, const float *logits, const uint8_t *mask, const float *bias, int E,
               int k, float routed_scale, int32_t *ids, float *w, void *stream);

/* ---- host-buffer adapters with the tier-table signature -------------- */
/* Same contract as tlm_qmv_fn (src/lib/tlm_quant.h:160-163): W, act, y are
 * HOST pointers; the call copies in, runs, copies out and returns. For the
 * reference's bit-exact tier self-test harness (selftest_tier,
 * src/lib/tlm_quant.c:1014-1056). Errors leave NaN in y. */
void tlmg_qmv_host(int dt, const void *W, size_t row_bytes, const void *act, float *y, int64_t n,
                   int64_t nrows);
/* Same contract as tlm_qdot_fn (src/lib/tlm_quant.h:157-158): one HOST row.
 * aux is the reference's per-128-column scale vector of FP8 rows; every
 * dtype this tier serves ignores it, as the reference's kernels for those
 * dtypes do. */
float tlmg_qdot_host(int dt, const void *wrow, const void *act, int64_t n, const float *aux);

/* ---- layer level: the MoE expert FFN with HBM-resident expert slots --- */
typedef struct tlmg_ctx tlmg_ctx;

/* Geometry of the MoE block (subset of tlm_model_geom,
 * src/lib/tlm_packet.h:84-95). */
typedef struct {
    int32_t n_layers, d_model, d_expert, d_shared, n_experts, top_k;
    int32_t router;          /* 0, 1, 2 as in tlm_model_geom.router */
    float   routed_scale, norm_eps;
} tlmg_geom;

/* Create a context on `device` (replaces the MoE half of tlm_model_open,
 * src/lib/tlm_model.h:36). Expert slots are allocated lazily per layer. */
int  tlmg_open(const tlmg_geom *g, int device, tlmg_ctx **out);
void tlmg_close(tlmg_ctx *ctx);

/* Upload one routed expert into its HBM slot: the packet payload bytes
 * (host or device pointer) with gate/up/down at item_off[0..2] (tlm_packet_hdr,
 * src/lib/tlm_packet.h:40-55; expert_mats, src/lib/tlm_model.c:880-896).
 * dt[3] are the dtypes of gate, up, down (the reference packet has one
 * dtype for all three; pass it three times). Synchronous. */
int tlmg_set_expert(tlmg_ctx *ctx, int layer, int expert, const int32_t dt[3],
                    const void *payload, size_t payload_len, const uint64_t item_off[3]);

/* ---- HBM expert-slot cache (reference expert store + lookahead,
 * src/lib/tlm_store.c:586-719, src/lib/tlm_model.c:844-877). For models
 * whose experts do not all fit in HBM: experts stay in (pinned) host
 * memory and a pool of n_slots HBM slots of slot_bytes each holds the
 * recently used ones. A layer whose experts are registered with
 * tlmg_set_expert_host is served through the cache: each call routes on
 * the GPU, brings the routed ids to the host (one stream synchronisation),
 * copies the missing experts host -> HBM on a side stream and runs the
 * expert kernels after exactly those copies; results are bit-identical to
 * HBM-resident experts. Slot decisions follow the reference store (the
 * tlmg_store policy below: frequency with decay, then recency; hits before
 * misses; hint rules). Call tlmg_cache_enable once, before registering
 * experts. */
int tlmg_cache_enable(tlmg_ctx *ctx, int n_slots, size_t slot_bytes);
/* Register one routed expert of `layer` in host memory (no copy now). The
 * payload must stay valid (and, for asynchronous copies, pinned) while the
 * context lives. Same arguments and checks as tlmg_set_expert. A layer is
 * either fully HBM-resident (tlmg_set_expert) or cached. */
int tlmg_set_expert_host(tlmg_ctx *ctx, int layer, int expert, const int32_t dt[3],
                         const void *payload, size_t payload_len, const uint64_t item_off[3]);
/* Hints for the listed experts of `layer` (host ids): copies into the slots
 * the hint rules allow, without waiting (tlm_store_prefetch). Call after
 * the current step's launches are queued. No-op for resident layers. */
int tlmg_cache_prefetch(tlmg_ctx *ctx, int layer, const int32_t *ids, int k);
/* out[6] = hits, misses, hints issued, hints used, evictions, bytes copied. */
int tlmg_cache_stats(tlmg_ctx *ctx, int64_t out[6]);
/* One model step has passed: every 16 ticks the experts' selection
 * frequencies halve (tlm_store_tick, called by tlm_model_step,
 * src/lib/tlm_model.c:1097). */
int tlmg_cache_tick(tlmg_ctx *ctx);
/* Router lookahead of tlmg_moe_layer on cached layers (reference
 * lookahead(), src/lib/tlm_model.c:844-877; depth 1 = the next layer, 0 =
 * off): with the current layer's routing, the GPU also runs the next
 * layer's RMSNorm and router on the current residual and takes its top k
 * (0 = top_k, capped at the routable experts); after the current layer's
 * experts are acquired those ids go to the cache as hints. */
int tlmg_cache_lookahead(tlmg_ctx *ctx, int depth, int k);

/* ---- the slot policy of the expert cache, on its own (host only) ---------
 * The reference store's rules (src/lib/tlm_store.c): FREE -> LOADING ->
 * READY slots; every selection adds 1 to the expert's frequency and
 * tlmg_store_tick halves all frequencies every 16 ticks; victims are a FREE
 * slot first, else the unreferenced READY slot with the lowest (frequency,
 * last use); an acquisition references its hits before any miss picks a
 * victim; hints take only FREE slots or READY slots of frequency-0 experts,
 * are dropped while more than 4 demand loads are in flight and are bounded
 * in flight by min(16, slots - max(1, top_k)). Keys are layer * E + expert.
 * No memory is moved: the caller copies an expert into a slot the policy
 * returned and then calls tlmg_store_load_done. The HBM expert cache above
 * decides with this policy; a caller managing its own slot memory can use it
 * directly. Replaces the policy half of tlm_store_acquire / _release /
 * _prefetch / _tick (src/lib/tlm_store.h:41-69). */
typedef struct tlmg_store tlmg_store;
int  tlmg_store_open(int n_keys, int n_slots, int top_k, tlmg_store **out);
void tlmg_store_close(tlmg_store *s);
/* Demand acquisition of keys[0..k): slots[i] = the referenced slot holding
 * or now loading keys[i]; loads[i] = 1 where the caller must copy the expert
 * in. TLMG_EBUSY (slots[i] = -1) when every slot is referenced or loading. */
int  tlmg_store_acquire(tlmg_store *s, const int32_t *keys, int k, int32_t *slots, int32_t *loads);
/* Router-lookahead hints: returns how many loads it started (their slots and
 * keys in slots[] / keys_out[]), or a negative code. */
int  tlmg_store_prefetch(tlmg_store *s, const int32_t *keys, int k, int32_t *slots, int32_t *keys_out);
/* The copy into `slot` has completed (LOADING -> READY). */
int  tlmg_store_load_done(tlmg_store *s, int slot);
/* Drops one reference of an acquired slot (tlm_store_release). */
int  tlmg_store_release(tlmg_store *s, int slot);
/* One model step has passed (tlm_store_tick). */
int  tlmg_store_tick(tlmg_store *s);
/* out = state (0 FREE, 1 LOADING, 2 READY), key (-1 none), references, hint
 * not yet used. */
int  tlmg_store_slot(const tlmg_store *s, int slot, int32_t out[4]);
/* out = hits, misses, hints issued, hints used, hints dropped, evictions. */
int  tlmg_store_stats(const tlmg_store *s, int64_t out[6]);

/* ---- expert packets of the tlm store (src/lib/tlm_packet.h:39-54) ------
 * A packet is the 64-byte header, the payload and zero padding to 4096
 * bytes. Extension: the reference writer zeroes the header's reserved[16]
 * (src/lib/tlm_packet.c:392); reserved[0] = 'D' (0x44) marks per-item
 * dtypes in reserved[1..3] (gate, up, down), so one EXPERT packet can hold
 * a Q4_K gate/up with a Q6_K down. reserved[0] = 0: every item has the
 * header's dtype (every packet the reference writes). Any other value of
 * reserved[0]: TLMG_EFORMAT. */
enum { TLMG_PKT_VERIFY_CRC = 1, TLMG_PKT_HOST = 2 };
typedef struct {
    uint32_t type, version, layer, n_items, id, dtype, layout;
    uint32_t crc32c;
    uint64_t payload_len;
    uint64_t total_len;      /* header + payload rounded up to 4096 */
    uint64_t item_off[3];    /* from the start of the payload */
    int32_t  item_dt[3];     /* per-item dtypes (extension) or dtype x 3 */
    int32_t  mixed;          /* 1 when the header carries per-item dtypes */
} tlmg_packet_info;
/* CRC-32C of buf[0..len) continuing `crc` (0 to start); same value as
 * tlm_crc32c (src/lib/tlm_platform.h:135). Host only. */
uint32_t tlmg_crc32c(uint32_t crc, const void *buf, size_t len);
/* Parse and check a packet in host memory (replaces the header half of
 * tlm_packet_verify, src/lib/tlm_packet.c:788-815, same order and codes):
 * len < 64 -> TLMG_EINVAL; bad magic/version or payload_len > len - 64 ->
 * TLMG_EFORMAT; with TLMG_PKT_VERIFY_CRC a payload CRC mismatch ->
 * TLMG_EFORMAT. Host only: needs no GPU. */
int tlmg_packet_parse(const void *packet, size_t len, int flags, tlmg_packet_info *out);
/* tlmg_packet_parse, then the header must name (EXPERT, layer, expert)
 * (TLMG_EFORMAT "does not match" otherwise, as tlm_packet_verify), one
 * item, layout 0; then tlmg_set_expert with the payload and the per-item
 * dtypes, or tlmg_set_expert_host with TLMG_PKT_HOST (the packet buffer
 * is then borrowed for the context's life, pinned for asynchronous
 * copies). */
int tlmg_set_expert_packet(tlmg_ctx *ctx, int layer, int expert, const void *packet, size_t len, int flags);

/* Resident per-layer tensors of the MoE block (DENSE packet,
 * src/lib/tlm_model.c:940-1055): ffn_norm f32[D]; router [E x D] of
 * router_dt (tlmc keeps it f32); router_bias f32[E] or NULL; mask u8[E]
 * or NULL. HOST pointers, copied. */
int tlmg_set_layer(tlmg_ctx *ctx, int layer, const float *ffn_norm, int router_dt,
                   const void *router_w, size_t router_row_bytes, const float *router_bias,
                   const uint8_t *mask);

/* Shared expert of a layer: gate/up [ds x D], down [D x ds] with dtypes
 * dt[3], plus the optional sigmoid gate vector f32[D]. HOST pointers. */
int tlmg_set_shared(tlmg_ctx *ctx, int layer, const int32_t dt[3], const void *gate,
                    const void *up, const void *down, const float *gate_inp);

/* Dense-FFN layer (the has_dense_ffn branch of moe(), src/lib/tlm_model.c:
 * 947-964: first_k_dense_replace / mlp_only layers): gate/up [d_ffn x D]
 * and down [D x d_ffn] with dtypes dt[3], HOST pointers, rows packed
 * (tlmg_row_bytes). tlmg_moe_layer on such a layer runs RMSNorm, the SwiGLU
 * FFN and h += ffn, with no router, experts or shared expert (and reports
 * no ids / weights). The layer still needs its ffn_norm (tlmg_set_layer). */
int tlmg_set_dense_ffn(tlmg_ctx *ctx, int layer, int d_ffn, const int32_t dt[3], const void *gate,
                       const void *up, const void *down);

/* Routed-expert FFN of one token (run_batch + rank-ordered combine,
 * src/lib/tlm_model.c:900-938, :1029-1036): x = normalised input f32[D],
 * logits f32[E]; ffn f32[D] receives sum_r w[r] * down_r(SiLU(gate_r x) *
 * up_r x). ids/w (top_k, may be NULL) receive the routing. Pointers: host
 * or device (all of one kind). */
int tlmg_expert_ffn(tlmg_ctx *ctx, int layer, const float *x, const float *logits, float *ffn,
                    int32_t *ids, float *w);

/* The same for n_tok independent (x, logits) pairs, pair t using layer
 * (layer0 + t) % n_layers: x f32[n_tok][D], logits f32[n_tok][E], ffn
 * f32[n_tok][D]. One host->device copy in, one device->host copy out when
 * the pointers are host memory. */
int tlmg_expert_ffn_many(tlmg_ctx *ctx, int layer0, int n_tok, const float *x,
                         const float *logits, float *ffn);

/* Batched decode: n_tok tokens through the SAME layer (the reference's
 * per-token run_batch, src/lib/tlm_model.c:900-938, applied to every
 * sequence of a decode batch). Each expert selected by any token is read
 * from HBM once per call. x f32[n_tok][D], logits f32[n_tok][E], ffn
 * f32[n_tok][D]; ids i32[n_tok][top_k] and w f32[n_tok][top_k] (may be
 * NULL) receive the routing. Results are bit-identical to n_tok calls of
 * tlmg_expert_ffn. Pointers: host or device (all of one kind). */
int tlmg_expert_ffn_batch(tlmg_ctx *ctx, int layer, int n_tok, const float *x,
                          const float *logits, float *ffn, int32_t *ids, float *w);

/* ---- Expert parallelism over n_ranks GPUs (one process per GPU).
 * The reference runs every expert in one process; these three calls split
 * its per-token run_batch + rank-ordered combine (src/lib/tlm_model.c:
 * 900-938, :1029-1036) at the (token, expert) pair, so a caller can move
 * the pairs between GPUs with an all-to-all. Expert e of a layer is owned
 * by GPU floor(e * n_ranks / n_experts). Results are bit-identical to
 * tlmg_expert_ffn_batch for any n_ranks. All buffers are DEVICE memory,
 * 16-byte aligned, except counts (host). Layers need uniform K-quant
 * gate/up and down dtypes (TLMG_EUNSUP otherwise). */

/* Bytes of one dispatch record: int32 expert id, 12 zero bytes, the
 * token's quantised input. */
size_t tlmg_ep_record_bytes(const tlmg_ctx *ctx);

/* Home GPU: route n_tok tokens (x f32[n_tok][D], logits f32[n_tok][E]) and
 * write one record per (token, rank) pair into send (room for n_tok * top_k
 * records), grouped by owner GPU, ascending pair order inside an owner.
 * perm i32[n_tok * top_k] receives each pair's record index, w f32[n_tok *
 * top_k] its routing weight, counts[n_ranks] the records per owner. With
 * host counts the call waits for the stream (the counts size the
 * exchange). counts may instead be a device pointer: they are then written
 * on the stream and the call returns without waiting (one host read of
 * the exchanged counts can then serve both directions); a foreign record
 * of an earlier call is then reported by a later host-count call or by
 * tlmg_check. */
int tlmg_ep_dispatch(tlmg_ctx *ctx, int layer, int n_tok, const float *x, const float *logits,
                     int n_ranks, void *send, int32_t *perm, float *w, int64_t *counts);

/* Owner GPU of experts [e_lo, e_hi) (only those need to be loaded): n_rec
 * received records of `layer` -> eo f32[n_rec][D], one expert output row
 * per record, in record order. A record naming an expert outside the range
 * gets a NaN row, and the next tlmg_ep_dispatch or tlmg_check returns
 * TLMG_EINVAL. */
int tlmg_ep_experts(tlmg_ctx *ctx, int layer, int e_lo, int e_hi, int64_t n_rec,
                    const void *recv, float *eo);

/* Home GPU: ffn[t] = sum_r w[t * k + r] * back[perm[t * k + r]] in
 * ascending r (back = the expert output rows returned in record order). */
int tlmg_ep_combine(tlmg_ctx *ctx, int n_tok, const float *back, const int32_t *perm,
                    const float *w, float *ffn);

/* ---- The whole decoder step on the GPU (tlm_model_step,
 * src/lib/tlm_model.c:1058-1103): embedding row, per layer attention()
 * (:730-763: RMSNorm, q/k/v, qk-norm, NeoX RoPE, the K/V write, decode
 * attention, o-proj, h += o) and moe() (the MoE block above), then the
 * final RMSNorm and lm_head. Every value is formed in the reference's
 * order of operations; with TLMG_ATTN_EXACT and F32 KV pages the logits
 * are bit-identical to the reference's when its expf is correctly
 * rounded (the GPU's is). The MoE layers are set as for tlmg_moe_layer. */

/* Opens the step: heads, KV heads and head_dim of attention, the vocab,
 * the RoPE inverse frequencies inv_freq[head_dim / 2] and attention scale
 * exactly as the reference's model holds them (tlm_model_open, plain or
 * YaRN-transformed), KV pages for max_ctx positions per layer (kv_dt F32
 * or BF16) and the attention mode (TLMG_ATTN_EXACT or _SPLIT). */
int tlmg_step_open(tlmg_ctx *ctx, int n_heads, int n_kv_heads, int head_dim, int vocab,
                   const float *inv_freq, float attn_scale, int max_ctx, int kv_dt, int attn_mode);
/* Attention weights of one layer (host or device memory, copied):
 * attn_norm f32[D]; dt[4] / w[4] / rb[4] = q [H*hd][D], k and v
 * [KV*hd][D], o [D][H*hd] (rb 0 = packed rows); q_norm / k_norm
 * f32[head_dim] or NULL. */
int tlmg_set_attention(tlmg_ctx *ctx, int layer, const float *attn_norm, const int32_t *dt,
                       const void *const *w, const size_t *rb, const float *q_norm, const float *k_norm);
/* Token embedding [vocab][D] of dtype dt (row_bytes 0 = packed). */
int tlmg_set_embedding(tlmg_ctx *ctx, int dt, const void *tok_embd, size_t row_bytes);
/* output_norm f32[D] and lm_head [vocab][D] of dtype dt. */
int tlmg_set_output(tlmg_ctx *ctx, const float *out_norm, int dt, const void *lm_head, size_t row_bytes);
/* One position: token at position pos (0 <= pos < max_ctx; positions
 * 0..pos-1 must have been stepped before, pos = 0 starts a new sequence)
 * -> logits f32[vocab] (host or device; NULL: no lm_head, as the
 * reference's prefill steps). Device logits: asynchronous on the
 * context's stream; host logits: the call waits. */
int tlmg_decode_step(tlmg_ctx *ctx, int token, int pos, float *logits);
/* From a context's second step on, the step runs as a captured CUDA graph
 * (one launch; the token and position are read from device memory) when
 * every MoE layer is resident and the static persistent kernel serves the
 * experts; on = 0 keeps every step eager. Results are the same either way
 * (TLMG_ATTN_SPLIT may differ in float rounding, its spans being shaped for
 * max_ctx in a graph). */
int tlmg_step_graphs(tlmg_ctx *ctx, int on);
/* out[4]: steps run, steps replayed from a graph, captures, 1 when a
 * capture failed and graphs were turned off. */
int tlmg_step_info(const tlmg_ctx *ctx, int64_t *out);
/* The step's counters in tlm_model_stats order (tlm_model_get_stats /
 * tlm_model_reset_stats, src/lib/tlm_model.h:87-96): out[5] = tokens,
 * attn_ns, moe_ns, expert_wait_ns, other_ns. tokens counts every
 * tlmg_decode_step; the phase times are device time between CUDA events
 * recorded at the phase boundaries of the steps run while tlmg_profile(ctx,
 * 1) is on (those steps run eagerly and each waits for its end; other steps
 * add no time). expert_wait_ns is always 0 here. reset != 0 zeroes them
 * after reading. */
int tlmg_step_stats(tlmg_ctx *ctx, uint64_t *out, int reset);

/* ---- Expert parallelism over peer memory (one process per GPU, all GPUs
 * of one node). The same split as above, with the exchange done by the
 * library: each rank opens one buffer, publishes its CUDA IPC handle,
 * maps every peer's, and then one tlmg_ep_layer call per layer does
 * dispatch, the owner's experts, the return of the output rows and the
 * combine, all queued on the context's stream with no host wait and no
 * collective library; two bounded barriers over peer flags order the
 * steps (a barrier that waits more than 1 s makes the next tlmg_check
 * return TLMG_EIO). Results are bit-identical to tlmg_expert_ffn_batch.
 * Every rank calls tlmg_ep_layer for the same layers in the same order,
 * with n_tok = 0 where it has no tokens. */

/* Allocates this rank's exchange buffer for up to max_tok tokens per call
 * (rank in [0, n_ranks), n_ranks <= 8). */
int tlmg_ep_open(tlmg_ctx *ctx, int rank, int n_ranks, int max_tok);
/* Size of one rank's handle (a cudaIpcMemHandle_t). */
size_t tlmg_ep_handle_bytes(void);
/* This rank's handle -> handle (tlmg_ep_handle_bytes() bytes). */
int tlmg_ep_handle(tlmg_ctx *ctx, void *handle);
/* Maps every peer's buffer: handles = the n_ranks handles in rank order
 * (this rank's own entry is ignored; NULL allowed when n_ranks == 1). */
int tlmg_ep_connect(tlmg_ctx *ctx, const void *handles);
/* One layer: x f32[n_tok][D], logits f32[n_tok][E] -> ffn f32[n_tok][D]
 * (the routed experts' combine; ids / w [n_tok][top_k] may be NULL). DEVICE
 * pointers, x 16-byte aligned. The rank's experts floor(e * n_ranks / E)
 * == rank must be loaded. */
int tlmg_ep_layer(tlmg_ctx *ctx, int layer, int n_tok, const float *x, const float *logits,
                  float *ffn, int32_t *ids, float *w);
/* Waits for the stream, then frees the buffer and unmaps the peers'
 * (every rank closes after its last layer call). */
int tlmg_ep_close(tlmg_ctx *ctx);

/* The whole moe() block for one token (src/lib/tlm_model.c:940-1055):
 * RMSNorm, router matvec, route, experts, shared expert, h += ffn.
 * h: f32[D] in/out; ids/w may be NULL. Host or device pointers. */
int tlmg_moe_layer(tlmg_ctx *ctx, int layer, float *h, int32_t *ids, float *w);

/* tlmg_moe_layer that also returns onorm f32[top_k] (may be NULL): per rank
 * r, (float)sqrt(sum_i (double)c * c) over c = w[r] * eo_r[i], the output
 * norms moe() hands to the route hook (src/lib/tlm_model.c:1029-1039,
 * :1053; tlm_route_hook, src/lib/tlm_model.h:62-70). Asking for onorm runs
 * this call on the multi-kernel expert path (the same bits). ids, w and
 * onorm are left untouched on a dense-FFN layer. */
int tlmg_moe_layer_ex(tlmg_ctx *ctx, int layer, float *h, int32_t *ids, float *w, float *onorm);

/* Run the context's work on `stream` (a cudaStream_t passed as void *) from
 * now on; NULL returns to the context's own stream. Lets a caller order the
 * MoE block with its other work and time it with events on that stream. */
int tlmg_set_stream(tlmg_ctx *ctx, void *stream);

/* Choose the expert-FFN kernels: on = 1 (default) or 2 the static
 * persistent kernel wherever it can serve the layer, 4 the same with
 * one-token launches served by the single-token kernel (every CTA fetches
 * all of its weights at once), 0 the multi-kernel path (router, gate/up,
 * re-quantise, down launches); 3 is not a mode (TLMG_EINVAL). All give
 * identical bits. TLMG_EUNSUP when on != 0 and the device cannot run the
 * persistent kernels (the multi-kernel path stays in use). */
int tlmg_set_fused(tlmg_ctx *ctx, int on);
/* Expert kernels of tlmg_expert_ffn_batch and the expert-parallel owner:
 * mode 2 (default) the tensor-core kernels (tcgen05.mma kind::i8, one int32
 * TMEM accumulator per K-quant sub-block), 1 the tiled CUDA-core kernels (a
 * CTA per 64-row tile of an expert, one thread per row and token), 0 the
 * warp-per-row-tile kernels; 10 * g + d selects gate/up mode g and down
 * mode d separately. Each falls back to the next lower mode for dtypes or
 * shapes it does not serve. Identical bits in every mode. */
int tlmg_set_batch_kernels(tlmg_ctx *ctx, int mode);
/* Wait for the context's queued work and report a failure the kernels
 * raised since the last check (a bounded wait that expired: TLMG_EIO). */
int tlmg_check(tlmg_ctx *ctx);

/* Phase trace of the persistent kernel (the reference's per-step stats,
 * src/lib/tlm_model.h:263-266, at kernel granularity): with on = 1 every
 * launch records per CTA TLMG_TRACE_POINTS u64 values, %globaltimer ns
 * unless noted, for the launch's token n_tok / 2:
 *   [0] launch start            [1] token routed
 *   [2] gate/up phase entered   [3] x arrived     [4] x quantised
 *   [5] first gate/up chunk in  [6] last gate/up chunk in
 *   [7] gate/up rows done       [8] barrier arrival
 *   [9] down phase entered      [10] barrier passed [11] h quantised
 *   [12] first down chunk in    [13] last down chunk in
 *   [14] down rows done         [15] combined
 *   [16..19] consumer warps' summed ns over all tokens: waiting for gate/up
 *            chunks, in the gate/up chunk loop, waiting for down chunks, in
 *            the down chunk loop
 *   [20] launch end
 *   [21] x copy issued  [22] / [23] first / last gate/up chunk issued
 *   [24] / [25] first / last down chunk issued
 *   [26] / [27] gate/up / down warps' summed ns in token duties
 *   [28] x copy issued, [29] barrier arrival, [30] h fetch issued and
 *        [31] down done for token n_tok / 2 + 1
 * Copies up to `cap` values of the last launch ([CTA][TLMG_TRACE_POINTS]) to
 * `out` (host) and returns how many; on = 0 stops tracing. */
#define TLMG_TRACE_POINTS 32
int tlmg_trace(tlmg_ctx *ctx, int on, uint64_t *out, int cap);

/* Per-launch timing of the expert-FFN kernels with CUDA events recorded on
 * the launch stream around each launch (off by default; on = 1 clears the
 * totals). Kernel classes: 0 = gate/up + SwiGLU (or the fused expert-FFN
 * kernel), 1 = down + combine, 2 = router top-k. */
int tlmg_profile(tlmg_ctx *ctx, int on);
/* Totals since profiling was switched on (synchronises the stream): device
 * milliseconds, launches, and the average algorithmic weight bytes one
 * launch of that class reads (from the layers' expert dtypes and the tokens
 * each launch served). */
int tlmg_profile_read(tlmg_ctx *ctx, int kclass, double *ms, int64_t *launches,
                      int64_t *bytes_per_launch);

/* ---- allocation-free expert FFN --------------------------------------- */
/* One routed expert given by device pointers to its gate [de x D], up
 * [de x D] and down [D x de] matrices and their dtypes. */
typedef struct {
    const void *m[3];
    int32_t     dt[3];
    int32_t     pad;
} tlmg_expert_slot;

/* No counterpart in the reference: this is an addition of this library.
 * The routed-expert FFN of one token, like tlmg_expert_ffn, for callers
 * that cannot allocate device memory on their decode path (a runtime that
 * sizes every buffer once at start-up and then runs a latency-bound token
 * loop, where cudaMalloc/cudaFree may block or synchronise the device).
 * No context, no allocation: experts (HOST array of E entries, device
 * pointers inside) and x f32[D], logits f32[E], ffn f32[D], ids int32[k],
 * w f32[k] (DEVICE pointers; ids/w may be NULL) are the caller's; the only
 * scratch is a fixed 1 MiB array in device memory that every GPU loading
 * the library holds until the process exits. Sizes needing more scratch
 * (about k*de*4 + k*(de+34) + 2.3*D + 40*E bytes) return TLMG_ERANGE.
 * The first call on each device looks up the array's device address (with
 * that device current): make that first call before any stream capture.
 * All calls share the array: calls that overlap on the GPU (different
 * streams or threads without ordering) race and give wrong results. Same
 * bits as tlmg_expert_ffn for the same experts and inputs. */
int tlmg_expert_ffn_noalloc(const tlmg_expert_slot *experts, int E, int D, int de, int k, int router,
                            float routed_scale, const float *x, const float *logits, float *ffn,
                            int32_t *ids, float *w, void *stream);

/* Kernel launches issued by the library since the context was opened
 * (counted on the host at each launch). */
int64_t tlmg_launch_count(const tlmg_ctx *ctx);

/* ---- decode attention over a paged KV cache ------------------------------
 * Replaces attn_heads (src/lib/tlm_model.c:683-719) and the K/V write of
 * attention() (src/lib/tlm_model.c:730-763). The reference holds one f32
 * KV per sequence, [layer][kv_head][max_ctx][head_dim]; here one layer's
 * K (and V) cache is a pool of pages [n_pages][KV][page_size][hd] of kv_dt
 * (TLMG_DT_F32 or TLMG_DT_BF16), and position t of a sequence is row
 * t % page_size of page page_table[t / page_size]; page_size is a power of
 * two (1 .. 65536). hd is 64, 128 or 256;
 * H is a multiple of KV with at most 16 query heads per KV head.
 *
 * TLMG_ATTN_EXACT: the reference's order of operations (serial f32 dot,
 *   times 1/sqrtf(hd), max, expf, serial double sum, serial f32 output
 *   sums, ascending t): bit-identical to attn_heads for f32 KV given a
 *   correctly rounded expf. Latency-bound (two serial chains of T per head).
 * TLMG_ATTN_SPLIT: flash-decoding over spans of positions with a merge;
 *   equal to the reference within float rounding. The long-context path. */
enum { TLMG_ATTN_EXACT = 0, TLMG_ATTN_SPLIT = 1 };

/* Device scratch (bytes) tlmg_decode_attention needs for this shape. */
size_t tlmg_attention_work_bytes(int mode, int kv_dt, int T, int H, int KV, int hd);

/* One decode position's attention over positions [0, T). DEVICE pointers:
 * q f32 [H][hd]; k_pages / v_pages (16-byte aligned) n_pages pages each;
 * page_table int32 [ceil(T / page_size)]; work (16-byte aligned,
 * work_bytes >= tlmg_attention_work_bytes); out f32 [H][hd]. A page-table
 * entry outside [0, n_pages) is not dereferenced: the heads that read it
 * get NaN. Asynchronous on `stream`. */
int tlmg_decode_attention(int mode, int kv_dt, const float *q, const void *k_pages, const void *v_pages,
                          int n_pages, const int32_t *page_table, int page_size, int T, int H, int KV, int hd,
                          void *work, size_t work_bytes, float *out, void *stream);

/* Appends position `pos` (row pos % page_size of page page_id) of every KV
 * head: k / v DEVICE f32 [KV][hd] -> the pages (bf16: round to nearest
 * even). Asynchronous on `stream`. */
int tlmg_kv_write(int kv_dt, const float *k, const float *v, void *k_pages, void *v_pages, int n_pages,
                  int32_t page_id, int page_size, int pos, int KV, int hd, void *stream);

#ifdef __cplusplus
}
#endif
#endif
