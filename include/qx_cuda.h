/*
 * qx_cuda.h - C ABI of the B200 decode engine for qx-mini-c's Qwen3-30B-A3B
 * forward pass.
 *
 * The reference has no CUDA seam yet: its state loop rejects every
 * `--cuda-policy` other than "none" (src/qx_format.c:6004-6005, CLI
 * src/qx_qxf_main.c:443,512-514) and reserves a `cuda_profile` JSON block
 * (src/qx_format.c:6683).  This header is the seam: a patched state loop calls
 * these functions when cuda_policy == "b200".  Each entry point below names
 * the reference function whose work it replaces.
 *
 * Conventions (same as the reference's public API, include/qx_format.h):
 *   - every function returns 1 on success, 0 on failure, and then writes a
 *     NUL-terminated message into err[err_len] (qx_set_err,
 *     src/qx_format.c:186-194);
 *   - outputs are written only on success (fail-closed);
 *   - no function exits or aborts; CUDA errors become messages;
 *   - plain pointers and sizes only; host pointers unless a name says _dev.
 *
 * Threading: an engine is used by one host thread at a time and owns one
 * CUDA stream (or the caller's, qx_cuda_options.stream).
 */
#ifndef QX_CUDA_H
#define QX_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QX_CUDA_ABI_VERSION 1u

typedef struct qx_cuda_engine qx_cuda_engine;

/* One QXF1 tensor as the caller holds it (a qx_tensor_dir_entry plus the
 * bytes it covers, e.g. from qx_acquire_span over an mmap'd file). */
typedef struct qx_cuda_tensor {
    const char *name;          /* GGUF name, e.g. "blk.0.ffn_gate_exps.weight" */
    uint32_t ggml_type;        /* qx_tensor_dir_entry.flags */
    uint32_t rank;
    uint64_t dims[4];          /* GGUF order: dims[0] = contiguous input length */
    uint64_t byte_size;
    uint64_t checksum;         /* qx_tensor_dir_entry.checksum (QXF1 FNV); checked with QX_CUDA_VERIFY_CHECKSUMS */
    const void *data;          /* host bytes, native GGUF block layout */
} qx_cuda_tensor;

/* The qx_model_manifest fields the engine uses (include/qx_format.h:41-55). */
typedef struct qx_cuda_model {
    uint32_t layers, hidden, q_heads, kv_heads, head_dim, vocab, experts, experts_per_token, moe_intermediate;
} qx_cuda_model;

#define QX_CUDA_VERIFY_CHECKSUMS 0x1u   /* verify FNV checksums of every tensor once, at create */
#define QX_CUDA_NO_GRAPH         0x2u   /* launch kernels one by one instead of replaying a CUDA graph */
#define QX_CUDA_PER_STAGE        0x4u   /* decode with one kernel per stage instead of the one-launch step kernel */
/* The reference's --activation q8_k_compat (src/qx_format.c:3869-4205):
 * activations of the attention projections, experts and head quantized to
 * Q8_K, exact int32 block sums, float epilogues in the reference's order.
 * Runs on the per-stage kernels; not with expert parallelism. */
#define QX_CUDA_Q8K_COMPAT       0x8u

typedef struct qx_cuda_options {
    int32_t device;            /* CUDA ordinal; -1 = current device */
    uint32_t ctx_tokens;       /* persistent INT8 KV capacity, 1..65536 (reference caps at 4096) */
    uint32_t flags;            /* QX_CUDA_* */
    uint32_t ep_rank;          /* expert-parallel rank (0 when ep_world <= 1) */
    uint32_t ep_world;         /* expert-parallel world size, 1..8; 0 or 1 = single GPU */
    uint32_t reserved;
    void *stream;              /* cudaStream_t to run on; NULL = engine-owned stream */
    void *nccl_comm;           /* reserved (must be NULL): ranks exchange through mapped peer memory */
} qx_cuda_options;

/* Counters for the reference's `cuda_profile` block (src/qx_format.c:6683). */
typedef struct qx_cuda_profile {
    char backend[32];          /* "b200-sm100a" */
    uint64_t device_bytes;     /* HBM held by the engine */
    uint64_t host_to_device_bytes;
    uint64_t device_to_host_bytes;
    uint64_t kernel_launches;
    uint64_t graph_replays;
    uint64_t decode_steps;
} qx_cuda_profile;

/* ---- lifetime --------------------------------------------------------- */

/* Upload every tensor once into HBM in its native block layout and build the
 * per-token CUDA graph.  Replaces the per-step span reads of the state loop
 * (qx_acquire_span / qx_read_raw_span, src/qx_format.c:858, :1757) and the
 * persistent KV allocation (:6138-6162).  The caller's buffers may be freed
 * after return. */
int qx_cuda_engine_create(const qx_cuda_model *model, const qx_cuda_tensor *tensors, uint32_t tensor_count,
                          const qx_cuda_options *options, qx_cuda_engine **out, char *err, uint64_t err_len);

/* Same, reading a QXF1 container: from a file (validated fail-closed like
 * qx_open_file, src/qx_format.c:712-841, then mmap'd) or from a caller image. */
int qx_cuda_engine_create_from_qxf(const char *path, const qx_cuda_options *options, qx_cuda_engine **out,
                                   char *err, uint64_t err_len);
int qx_cuda_engine_create_from_image(const void *image, uint64_t size, const qx_cuda_options *options,
                                     qx_cuda_engine **out, char *err, uint64_t err_len);

void qx_cuda_engine_destroy(qx_cuda_engine *engine);

/* Zero the persistent KV cache and scales (the calloc at src/qx_format.c:6155-6160). */
int qx_cuda_reset(qx_cuda_engine *engine, char *err, uint64_t err_len);

/* ---- decode ------------------------------------------------------------ */

/* One greedy step at `position`: embed `token`, run every layer (appending K/V
 * at `position`), final RMSNorm, Q6_K head, argmax.  Replaces one iteration of
 * the state loop's token loop (src/qx_format.c:6250-6627) with
 * temperature 0 (qx_sample_from_top, :3049-3057).  Optional outputs (NULL to
 * skip): logits[vocab], final_residual[hidden], experts[layers*8] (top-8 in
 * rank order per layer), routing[layers*8] (renormalised weights). */
int qx_cuda_decode_step(qx_cuda_engine *engine, uint32_t token, uint32_t position, uint32_t *next_token,
                        float *logits, float *final_residual, uint32_t *experts, float *routing,
                        char *err, uint64_t err_len);

/* `steps` greedy steps starting at (token, position) with the argmax fed back
 * on the device (no host round trip per token); tokens_out[steps] receives the
 * selected tokens.  The state loop's generation phase (:6250-6627) for any
 * number of steps up to the KV capacity. */
int qx_cuda_generate(qx_cuda_engine *engine, uint32_t token, uint32_t position, uint32_t steps,
                     uint32_t *tokens_out, char *err, uint64_t err_len);

/* ---- stage entry points (the reference's parity seams) ----------------- */

/* Final RMSNorm + full-vocabulary Q6_K head: qx_compute_real_final_head
 * (src/qx_format.c:3554-3738).  normalized[hidden], logits[vocab] may be NULL;
 * top_tokens/top_logits[top_n] (top_n 1..32) in descending order, ties to the
 * lower index. */
int qx_cuda_final_head(qx_cuda_engine *engine, const float *residual, float *normalized, float *logits,
                       uint32_t top_n, uint32_t *top_tokens, float *top_logits, char *err, uint64_t err_len);

/* One MoE FFN layer on a post-attention residual: qx_apply_real_moe_layer
 * (src/qx_format.c:5198-5317).  layer_output = residual + moe_output. */
int qx_cuda_moe_layer(qx_cuda_engine *engine, uint32_t layer, const float *residual_after_attention,
                      float *layer_output, float *moe_output, uint32_t selected[8], float weights[8],
                      char *err, uint64_t err_len);

/* One MoE FFN layer for `tokens` independent tokens at once - the batched /
 * prefill counterpart of qx_cuda_moe_layer.  The reference has no batched
 * path: its prompt prefill and decode call qx_apply_real_moe_layer
 * (src/qx_format.c:5198-5317) once per token (the prefill loop
 * :6250-6547).  Per token t: layer_output[t] = residual[t] + moe_output[t]
 * with the reference's router, top-8 and rank-order sum; the expert
 * projections run as grouped GEMMs over the tokens routed to each expert on
 * the tcgen05 tensor cores (exact integer contraction).  residual / outputs
 * are [tokens][hidden] host floats; selected / weights are [tokens][8]
 * (either may be NULL, moe_output too).  tokens <= QX_CUDA_MAX_BATCH.  Needs
 * the benchmark quant mix (IQ2_XS gate/up, IQ3_XXS down) in the one-launch
 * step kernel's layouts. */
#define QX_CUDA_MAX_BATCH 4096u
int qx_cuda_moe_batch(qx_cuda_engine *engine, uint32_t layer, uint32_t tokens, const float *residual,
                      float *layer_output, float *moe_output, uint32_t *selected, float *weights, char *err,
                      uint64_t err_len);

/* Prompt prefill: `tokens` prompt tokens at positions position ..
 * position + tokens - 1 through every layer at once, layer by layer, and the
 * greedy token after the last one.  The reference's prompt loop
 * (qx_dump_prompt_state_loop_probe_summary, src/qx_format.c:5970; its layer
 * loop :6250-6547) runs the prompt one token at a time and skips the head for
 * all but the last prompt position (:6533-6547); here the projections of all
 * tokens run as GEMMs on the tcgen05 tensor cores (exact integer
 * contraction), the per-token attention reads the cache the batch has just
 * appended, and the MoE is qx_cuda_moe_batch's.  The INT8 KV cache holds the
 * prompt afterwards, so qx_cuda_generate / qx_cuda_decode_step continue at
 * position + tokens.  final_residual[hidden] (may be NULL) is the last
 * token's.  tokens <= QX_CUDA_MAX_BATCH; same quant-mix requirement as
 * qx_cuda_moe_batch plus IQ4_XS attention. */
int qx_cuda_prefill(qx_cuda_engine *engine, const uint32_t *tokens, uint32_t tokens_count, uint32_t position,
                    uint32_t *next_token, float *final_residual, char *err, uint64_t err_len);

/* One greedy decode step for `count` independent sequences at once (batched
 * decode).  Sequence i occupies KV slot slots[i] (< QX_CUDA_MAX_SLOTS, each
 * slot its own INT8 cache of ctx_tokens positions, allocated on the first
 * call: slots x layers x ctx x (2 x kv + 8) bytes), feeds tokens[i] at
 * positions[i] and gets next_tokens[i].  Per sequence this is the reference's
 * state-loop step (src/qx_format.c:6250-6627), which has no batched form; the
 * projections, experts and head run as GEMMs over the batch on the tcgen05
 * tensor cores.  A slot's positions must be fed in order from 0 (positions
 * beyond the current one are never read).  Slots are separate from the
 * engine's single-sequence cache. */
#define QX_CUDA_MAX_SLOTS 64u
int qx_cuda_decode_batch(qx_cuda_engine *engine, uint32_t count, const uint32_t *slots, const uint32_t *tokens,
                         const uint32_t *positions, uint32_t *next_tokens, char *err, uint64_t err_len);

/* The attention half of one layer at `position`, state-loop order
 * (src/qx_format.c:6283-6423 with qx_rope_gqa_attention_partial, :5051-5196):
 * attn RMSNorm, K/V projection, K head norm + RoPE, INT8 append at
 * [layer][position], Q projection + norm + RoPE, causal GQA softmax over
 * positions 0..position, O projection.  residual[hidden] is updated in place;
 * attn_out[hidden] and context[q_heads*head_dim] may be NULL. */
int qx_cuda_attention_layer(qx_cuda_engine *engine, uint32_t layer, uint32_t position, float *residual,
                            float *attn_out, float *context, char *err, uint64_t err_len);

/* Token embedding row (Q4_K gather), qx_fill_residual_vector_from_embedding
 * without norm (src/qx_format.c:3759-3819, full-MoE mode :6261). */
int qx_cuda_embed(qx_cuda_engine *engine, uint32_t token, float *out, char *err, uint64_t err_len);

/* Final RMSNorm + Q6_K head + argmax that allocates no device memory.  No
 * counterpart in the reference (it has no device code).  For callers that
 * cannot call cudaMalloc themselves or have it called for them - a plugin
 * inside a host that owns every allocation, or code that must not allocate
 * between stream-ordered steps.  All pointers are device pointers the caller
 * owns: residual[hidden], norm_weight[hidden] (output_norm.weight, F32),
 * head (output.weight bytes, Q6_K, vocab rows; 16-byte aligned),
 * logits[vocab] (may be NULL), argmax (one uint32; 0xFFFFFFFF if a logit is
 * not finite; the call still returns 1).  Misaligned pointers are refused
 * before anything is queued.  The work is
 * queued on `stream` (cudaStream_t, NULL = default) and the call returns
 * without waiting.  Its scratch (per-CTA partial maxima and a counter) is a
 * fixed array inside this library, held by every GPU that loads it until the
 * process exits, so: hidden must be a multiple of 256 and at most 2048, vocab
 * a positive multiple of 32, and calls that overlap on the GPU (unordered
 * streams) race on that array.  The first call on each device looks up the
 * array's address; make it before any stream capture. */
int qx_cuda_final_head_noalloc(const float *residual_dev, const float *norm_weight_dev, const void *head_q6k_dev,
                               uint32_t hidden, uint32_t vocab, float *logits_dev, uint32_t *argmax_dev, void *stream,
                               char *err, uint64_t err_len);

/* ---- persistent KV ---------------------------------------------------- */

/* Write / read `count` positions of layer `layer` starting at `first`:
 * k,v int8[count*kv_heads*head_dim], scales float[count] (one scale per
 * (layer, token) shared by all KV heads, src/qx_format.c:6343-6362).  Used to
 * pre-fill history and to move KV between the CPU path and the engine (the
 * QXKVSNP1 payload, src/qx_format.c:5860-5913). */
int qx_cuda_kv_write(qx_cuda_engine *engine, uint32_t layer, uint32_t first, uint32_t count, const int8_t *k,
                     const int8_t *v, const float *k_scales, const float *v_scales, char *err, uint64_t err_len);
int qx_cuda_kv_read(qx_cuda_engine *engine, uint32_t layer, uint32_t first, uint32_t count, int8_t *k, int8_t *v,
                    float *k_scales, float *v_scales, char *err, uint64_t err_len);

/* ---- KV snapshots (QXKVSNP1) -------------------------------------------
 *
 * The reference's accumulated-KV snapshot (--kv-snapshot-out / --kv-snapshot-in,
 * qx_write_accumulated_kv_snapshot / qx_read_accumulated_kv_snapshot,
 * src/qx_format.c:5860-5969): version 2, INT8 format, the K row, V row and two
 * scales of positions 0..positions-1 of every layer, SHA-256 trailer.  The
 * bytes are the reference's, so the CPU path and this engine can continue
 * from each other's KV; ctx_tokens and seed must match on both sides (they are
 * part of the header).  Import checks the header, every scale and the digest
 * with the reference's messages ("accumulated KV snapshot header mismatch",
 * "accumulated KV snapshot payload mismatch") and leaves the device KV as it
 * was on failure; on success it replaces the whole cache (positions beyond
 * the snapshot read as zero) and returns the positions and next token. */
int qx_cuda_kv_export(qx_cuda_engine *engine, const char *path, uint32_t positions, uint32_t next_token,
                      uint32_t seed, char *err, uint64_t err_len);
int qx_cuda_kv_import(qx_cuda_engine *engine, const char *path, uint32_t seed, uint32_t *positions,
                      uint32_t *next_token, char *err, uint64_t err_len);

/* ---- introspection ----------------------------------------------------- */

int qx_cuda_profile_get(const qx_cuda_engine *engine, qx_cuda_profile *out);

/* Per-kernel device time of the last `qx_cuda_time_kernels` run.  names is a
 * ';'-separated list written into names[names_len]; ms_avg[i] / launches[i]
 * for each (up to max_kernels). */
int qx_cuda_time_kernels(qx_cuda_engine *engine, uint32_t token, uint32_t position, uint32_t steps,
                         char *names, uint64_t names_len, float *ms_avg, uint32_t *launches,
                         uint32_t max_kernels, uint32_t *kernel_count, char *err, uint64_t err_len);

/* One decode step of the persistent step kernel with device timestamps (ns,
 * %globaltimer).  With n = 3 + 6 * layers and G the kernel's CTA count, the
 * full record has n * (9 + G) stamps (fewer are written if max_stamps is
 * smaller; *count says how many):
 *   [0, n)       stamps[0] = start, then CTA 0's exit from each grid barrier:
 *                embedding+QKV, attention, O projection, router, gate/up,
 *                down per layer, then the head (last slot unused);
 *   [n, 9n)      eight in-phase markers of CTA 0 per barrier epoch e at
 *                n + 8e + k (0 where the phase sets no marker k);
 *   [9n, 9n+nG)  each CTA's arrival at barrier e at 9n + e*G + cta.
 * A profiling aid (it allocates a buffer); not part of the reference API. */
int qx_cuda_phase_trace(qx_cuda_engine *engine, uint32_t token, uint32_t position, uint64_t *stamps_ns,
                        uint32_t max_stamps, uint32_t *count, char *err, uint64_t err_len);

/* ---- expert parallelism (one process per GPU, ranks on one node) ---------
 *
 * The reference decodes on one CPU thread; this is the B200 engine's own
 * partitioning of qx_apply_real_moe_layer (src/qx_format.c:5198-5310) and of
 * the head (:3554-3738) over ep_world GPUs, created with options.ep_world > 1
 * and options.ep_rank.  Every rank holds the whole model and runs attention
 * and the router itself (identical results on every rank); rank r computes
 * the top-8 slots whose expert lies in its share (qx_cuda_ep_partition) and
 * stores their weighted outputs into every rank's exchange buffer over NVLink
 * (plain peer stores + release flags, no collective library on the data
 * path); every rank then adds the 8 slots in rank order, exactly as one GPU
 * does.  The head is split by vocabulary rows; ranks exchange (max logit,
 * index) and take the lowest index among equal maxima.  Tokens, experts and
 * the final residual equal the single-GPU engine's; decode_step's logits hold
 * only this rank's vocabulary rows.
 *
 * Set-up: every rank calls qx_cuda_ep_handle, the caller gathers the handles
 * of all ranks in rank order (any host transport), and every rank calls
 * qx_cuda_ep_connect once.  Until then decode calls fail.  All ranks must run
 * the same decode calls in the same order (their steps wait on each other, with
 * a bounded wait that fails the step with "device grid barrier timed out"). */

/* The split (host-only, no device needed): rank `rank` of `world` computes
 * experts [out[0], out[1]) and head rows [out[2], out[3]) (vocab a multiple of
 * 32).  Returns 0 on invalid arguments. */
int qx_cuda_ep_partition(uint32_t experts, uint32_t vocab, uint32_t world, uint32_t rank, uint32_t out[4]);

/* Write this rank's exchange-buffer handle (a cudaIpcMemHandle_t, 64 bytes)
 * into handle[handle_size] (handle_size >= 64). */
int qx_cuda_ep_handle(qx_cuda_engine *engine, void *handle, uint64_t handle_size, char *err, uint64_t err_len);

/* Map the peers: handles holds `world` handles of handle_size bytes each,
 * in rank order (this rank's own entry is ignored). */
int qx_cuda_ep_connect(qx_cuda_engine *engine, const void *handles, uint64_t handle_size, uint32_t world,
                       char *err, uint64_t err_len);

/* The engine's CUDA stream (cudaStream_t) for callers that time with events. */
void *qx_cuda_stream(const qx_cuda_engine *engine);

#ifdef __cplusplus
}
#endif
#endif
