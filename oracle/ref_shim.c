/*
 * TEST INFRASTRUCTURE ONLY - the reference itself, compiled as a checker.
 *
 * This translation unit #includes the reference's own src/qx_format.c (found
 * through -I at build time; see oracle/Makefile) so that its static forward
 * functions become callable, and exports thin entry points over them.  Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU legs may load the
 * resulting oracle/_ref/libqxref.so.  No product code links it.
 *
 * Every entry point calls the reference functions in the order the state loop
 * does (src/qx_format.c:6274-6432) with the same arguments; the glue here only
 * supplies buffers.  Nothing of the reference's arithmetic is restated.
 */
#include "qx_format.c"

#include <stdint.h>

#define QXREF_API __attribute__((visibility("default")))

/* Activation format of every projection / expert / head call below:
 * "f32" (default) or "q8_k_compat" (src/qx_format.c:3869-4205). */
static const char *g_activation = "f32";
QXREF_API void qxref_set_activation(int q8_k_compat) { g_activation = q8_k_compat ? "q8_k_compat" : "f32"; }

typedef struct qxref_model {
    qx_file file;
    int in_memory;
} qxref_model;

/* Open a QXF1 file through the reference's own validating loader
 * (qx_open_file, src/qx_format.c:712) with the mmap backend. */
QXREF_API int qxref_open_path(const char *path, int use_mmap, qxref_model **out, char *err, uint64_t err_len) {
    if (!out) { qx_set_err(err, err_len, "invalid argument"); return 0; }
    *out = NULL;
    if (!qx_set_io_backend(use_mmap ? "mmap" : "buffered", err, err_len)) return 0;
    qxref_model *m = (qxref_model *)calloc(1, sizeof(*m));
    if (!m) { qx_set_err(err, err_len, "out of memory"); return 0; }
    if (!qx_open_file(path, &m->file, err, err_len)) { free(m); return 0; }
    *out = m;
    return 1;
}

/* Wrap an in-memory QXF1 image (as produced by the synthetic generator) in a
 * qx_file that uses the reference's mmap code path (qx_acquire_span,
 * src/qx_format.c:858-872).  The header and directory are taken verbatim from
 * the image; the caller keeps the image alive until qxref_close. */
QXREF_API int qxref_open_image(const unsigned char *image, uint64_t size, qxref_model **out, char *err, uint64_t err_len) {
    if (!image || !out || size < sizeof(qx_header)) { qx_set_err(err, err_len, "invalid argument"); return 0; }
    *out = NULL;
    qxref_model *m = (qxref_model *)calloc(1, sizeof(*m));
    if (!m) { qx_set_err(err, err_len, "out of memory"); return 0; }
    memcpy(&m->file.header, image, sizeof(qx_header));
    if (memcmp(m->file.header.magic, QX_MAGIC, 4) != 0 || m->file.header.file_size != size ||
        m->file.header.dir_offset + (uint64_t)m->file.header.tensor_count * sizeof(qx_tensor_dir_entry) > size) {
        free(m); qx_set_err(err, err_len, "invalid QXF image"); return 0;
    }
    m->file.directory = (qx_tensor_dir_entry *)calloc(m->file.header.tensor_count, sizeof(qx_tensor_dir_entry));
    if (!m->file.directory) { free(m); qx_set_err(err, err_len, "out of memory"); return 0; }
    memcpy(m->file.directory, image + m->file.header.dir_offset,
           (size_t)m->file.header.tensor_count * sizeof(qx_tensor_dir_entry));
    m->file.fp = fopen("/dev/null", "rb");
    if (!m->file.fp) { free(m->file.directory); free(m); qx_set_err(err, err_len, "cannot open /dev/null"); return 0; }
    m->file.io_backend = QX_IO_MMAP;
    m->file.mapped_view = image;
    m->in_memory = 1;
    *out = m;
    return 1;
}

QXREF_API void qxref_close(qxref_model *m) {
    if (!m) return;
    if (m->in_memory) {
        if (m->file.fp) fclose(m->file.fp);
        free(m->file.directory);
    } else {
        qx_close_file(&m->file);
    }
    free(m);
}

QXREF_API uint32_t qxref_manifest(const qxref_model *m, uint32_t field) {
    const qx_model_manifest *mf = &m->file.header.manifest;
    switch (field) {
        case 0: return mf->layers;
        case 1: return mf->hidden;
        case 2: return mf->q_heads;
        case 3: return mf->kv_heads;
        case 4: return mf->head_dim;
        case 5: return mf->vocab;
        case 6: return mf->experts;
        case 7: return mf->moe_intermediate;
        default: return 0;
    }
}

/* Embedding gather, no norm (full-MoE mode, src/qx_format.c:6261). */
QXREF_API int qxref_embed(qxref_model *m, uint32_t token, float *out, char *err, uint64_t err_len) {
    return qx_fill_residual_vector_from_embedding(&m->file, token, NULL, out, m->file.header.manifest.hidden,
                                                  NULL, NULL, err, err_len);
}

/* Final RMSNorm + full-vocabulary Q6_K head (src/qx_format.c:3554). */
QXREF_API int qxref_final_head(qxref_model *m, const float *residual, float *normalized, float *logits,
                               uint32_t top_n, uint32_t *top_tokens, double *top_logits, char *err, uint64_t err_len) {
    qx_real_head_result result;
    uint32_t hidden = m->file.header.manifest.hidden;
    if (!qx_compute_real_final_head(&m->file, residual, normalized, hidden, top_n, g_activation, "baseline", "serial", 1u,
                                    "scalar", logits, m->file.header.manifest.vocab, &result, err, err_len)) return 0;
    for (uint32_t i = 0; i < result.top_n && top_tokens; ++i) {
        top_tokens[i] = result.top[i].token;
        if (top_logits) top_logits[i] = result.top[i].logit;
    }
    return 1;
}

/* One MoE FFN layer on the post-attention residual (src/qx_format.c:5198). */
QXREF_API int qxref_moe_layer(qxref_model *m, uint32_t layer, const float *residual_after_attention,
                              float *layer_output, float *moe_output, uint32_t selected[8], double weights[8],
                              char *err, uint64_t err_len) {
    uint32_t g = 0, u = 0, d = 0;
    double l2 = 0.0;
    return qx_apply_real_moe_layer(&m->file, layer, residual_after_attention, m->file.header.manifest.hidden,
                                   layer_output, moe_output, selected, weights, &g, &u, &d, g_activation, NULL, &l2,
                                   err, err_len);
}

/* Router-only view of the same layer: logits/probabilities are not exposed by
 * the reference, so tests read selection and weights from qxref_moe_layer. */

/* Quantize one K/V vector exactly as the state loop does (src/qx_format.c:4449). */
QXREF_API float qxref_quantize_int8(const float *src, int8_t *dst, uint32_t n) {
    return qx_quantize_int8_vector(src, (unsigned char *)dst, n);
}

QXREF_API void qxref_rope(float *vec, uint32_t heads, uint32_t head_dim, uint32_t position) {
    qx_apply_rope(vec, heads, head_dim, position, 1000000.0);
}

/* The attention half of one layer at position `step`, in state-loop order
 * (src/qx_format.c:6283-6423): attn RMSNorm, K/V projections, K head norm,
 * K RoPE, INT8 quantization and cache append at [layer][step], then
 * qx_rope_gqa_attention_partial (Q, q-norm, RoPE, softmax, O projection),
 * then residual += attention output.  The caches are [layers][ctx][kv_values]
 * int8 and the scales [layers][ctx], as allocated at src/qx_format.c:6153-6160.
 * residual is updated in place; attn_out receives the O projection output and
 * context (may be NULL) the 4096-wide pre-projection context. */
QXREF_API int qxref_attention_layer(qxref_model *m, uint32_t layer, uint32_t step, uint32_t ctx,
                                    int8_t *kcache, int8_t *vcache, float *kscales, float *vscales,
                                    float *residual, float *attn_out, float *context,
                                    float *k_out, float *v_out, char *err, uint64_t err_len) {
    qx_file *file = &m->file;
    const qx_model_manifest *mf = &file->header.manifest;
    uint32_t hidden = mf->hidden, q_heads = mf->q_heads, kv_heads = mf->kv_heads, head_dim = mf->head_dim;
    uint32_t kv_values = kv_heads * head_dim;
    char name[QX_NAME_MAX];
    float *normed = (float *)malloc((size_t)hidden * sizeof(float));
    float *kfloat = (float *)malloc((size_t)kv_values * sizeof(float));
    float *vfloat = (float *)malloc((size_t)kv_values * sizeof(float));
    unsigned char *kbuf = (unsigned char *)malloc(kv_values);
    unsigned char *vbuf = (unsigned char *)malloc(kv_values);
    int ok = normed && kfloat && vfloat && kbuf && vbuf;
    if (!ok) qx_set_err(err, err_len, "out of memory");
    snprintf(name, sizeof(name), "blk.%u.attn_norm.weight", layer);
    const qx_tensor_dir_entry *an = qx_find_tensor(file, name);
    snprintf(name, sizeof(name), "blk.%u.attn_k.weight", layer);
    const qx_tensor_dir_entry *kt = qx_find_tensor(file, name);
    snprintf(name, sizeof(name), "blk.%u.attn_v.weight", layer);
    const qx_tensor_dir_entry *vt = qx_find_tensor(file, name);
    snprintf(name, sizeof(name), "blk.%u.attn_k_norm.weight", layer);
    const qx_tensor_dir_entry *kn = qx_find_tensor(file, name);
    if (ok && (!an || !kt || !vt || !kn)) { qx_set_err(err, err_len, "attention tensor not found"); ok = 0; }
    qx_projection_workspace pw;
    memset(&pw, 0, sizeof(pw));
    double probe = 0.0;
    uint64_t vals = 0;
    if (ok) ok = qx_apply_f32_rmsnorm(file, an, residual, normed, hidden, NULL, err, err_len);
    if (ok) ok = qx_projection_matvec_fill_mode(file, kt, kbuf, kfloat, kv_values, hidden, normed, hidden, 0u, layer,
                                                1u + step * 17u, g_activation, &pw, &probe, &vals, err, err_len);
    if (ok) ok = qx_projection_matvec_fill_mode(file, vt, vbuf, vfloat, kv_values, hidden, normed, hidden, 0u, layer,
                                                (1u ^ 0x9e3779b9u) + step * 17u, g_activation, &pw, &probe, &vals, err, err_len);
    if (ok) ok = qx_apply_f32_head_rmsnorm(file, kn, kfloat, kv_heads, head_dim, err, err_len);
    if (ok) {
        qx_apply_rope(kfloat, kv_heads, head_dim, step, 1000000.0);
        if (k_out) memcpy(k_out, kfloat, (size_t)kv_values * sizeof(float));
        if (v_out) memcpy(v_out, vfloat, (size_t)kv_values * sizeof(float));
        uint64_t si = (uint64_t)layer * ctx + step;
        kscales[si] = qx_quantize_int8_vector(kfloat, kbuf, kv_values);
        vscales[si] = qx_quantize_int8_vector(vfloat, vbuf, kv_values);
        memcpy((unsigned char *)kcache + si * kv_values, kbuf, kv_values);
        memcpy((unsigned char *)vcache + si * kv_values, vbuf, kv_values);
    }
    float *out_vec = (float *)malloc((size_t)hidden * sizeof(float));
    float *ctx_capture = (float *)malloc((size_t)q_heads * head_dim * sizeof(float));
    if (ok && (!out_vec || !ctx_capture)) { qx_set_err(err, err_len, "out of memory"); ok = 0; }
    if (ok) {
        double s = 0, smin = 0, smax = 0;
        uint32_t qrun = 0;
        uint64_t qv = 0;
        const char *qn = NULL, *on = NULL;
        ok = qx_rope_gqa_attention_partial(file, layer, step, ctx, kv_values, (const unsigned char *)kcache,
                                           (const unsigned char *)vcache, kv_values, 1u, kscales, vscales, normed,
                                           hidden, q_heads, kv_heads, head_dim, 0u, 1u, out_vec, ctx_capture,
                                           q_heads * head_dim, &s, &smin, &smax, &qrun, &qv, &qn, &on, g_activation, &pw,
                                           NULL, err, err_len);
    }
    if (ok) {
        for (uint32_t i = 0; i < hidden; ++i) residual[i] += out_vec[i];
        if (attn_out) memcpy(attn_out, out_vec, (size_t)hidden * sizeof(float));
        if (context) memcpy(context, ctx_capture, (size_t)q_heads * head_dim * sizeof(float));
    }
    free(normed); free(kfloat); free(vfloat); free(kbuf); free(vbuf); free(out_vec); free(ctx_capture);
    return ok;
}

/* One full greedy decode step (src/qx_format.c:6250-6627): embed `token`,
 * run every layer at position `step`, then the final head; returns the
 * argmax token.  experts_out (may be NULL) receives layers*8 selections,
 * residual_out (may be NULL) the final residual, logits (may be NULL) the
 * vocabulary logits. */
QXREF_API int qxref_decode_step(qxref_model *m, uint32_t token, uint32_t step, uint32_t ctx,
                                int8_t *kcache, int8_t *vcache, float *kscales, float *vscales,
                                uint32_t *experts_out, double *routing_out, float *residual_out, float *logits,
                                uint32_t *next_token, double *top2_logits, char *err, uint64_t err_len) {
    const qx_model_manifest *mf = &m->file.header.manifest;
    uint32_t hidden = mf->hidden;
    float *res = (float *)malloc((size_t)hidden * sizeof(float));
    float *normed = (float *)malloc((size_t)hidden * sizeof(float));
    if (!res || !normed) { free(res); free(normed); qx_set_err(err, err_len, "out of memory"); return 0; }
    int ok = qxref_embed(m, token, res, err, err_len);
    for (uint32_t layer = 0; ok && layer < mf->layers; ++layer) {
        ok = qxref_attention_layer(m, layer, step, ctx, kcache, vcache, kscales, vscales, res, NULL, NULL, NULL, NULL,
                                   err, err_len);
        uint32_t sel[8];
        double w[8];
        if (ok) ok = qxref_moe_layer(m, layer, res, res, NULL, sel, w, err, err_len);
        if (ok && experts_out) memcpy(experts_out + (size_t)layer * 8u, sel, sizeof(sel));
        if (ok && routing_out) memcpy(routing_out + (size_t)layer * 8u, w, sizeof(w));
    }
    uint32_t top[2] = {0, 0};
    double topl[2] = {0, 0};
    if (ok) ok = qxref_final_head(m, res, normed, logits, 2u, top, topl, err, err_len);
    if (ok) {
        if (residual_out) memcpy(residual_out, res, (size_t)hidden * sizeof(float));
        if (next_token) *next_token = top[0];
        if (top2_logits) { top2_logits[0] = topl[0]; top2_logits[1] = topl[1]; }
    }
    free(res); free(normed);
    return ok;
}

/* The reference's own CLI state loop (src/qx_format.c:6721), JSON to a file. */
QXREF_API int qxref_state_loop_json(const char *qxf_path, uint32_t prompt_token, uint32_t steps, uint32_t ctx,
                                    const char *json_path, const char *dump_dir, char *err, uint64_t err_len) {
    FILE *out = fopen(json_path, "w");
    if (!out) { qx_set_err(err, err_len, "cannot open json output"); return 0; }
    if (!qx_set_io_backend("mmap", err, err_len)) { fclose(out); return 0; }
    int ok = qx_dump_state_loop_probe_summary(qxf_path, NULL, prompt_token, steps, 48u, ctx, "int8", "f32",
                                              1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 2048u, NULL, 5u, 64u, 5u, 0.0, 1u,
                                              dump_dir, 0u, NULL, NULL, NULL, out, err, err_len);
    fclose(out);
    return ok;
}

/* The reference's rope/GQA known-answer probe (src/qx_format.c:4643). */
QXREF_API int qxref_rope_gqa_golden_json(uint32_t tokens, uint32_t q_heads_run, const char *json_path, char *err,
                                         uint64_t err_len) {
    FILE *out = fopen(json_path, "w");
    if (!out) { qx_set_err(err, err_len, "cannot open json output"); return 0; }
    int ok = qx_dump_rope_gqa_golden_probe_summary(tokens, q_heads_run, 1u, out, err, err_len);
    fclose(out);
    return ok;
}

/* Block decoders, for decoder known-answer tests (src/qx_format.c:2207). */
QXREF_API int qxref_decode_block(uint32_t ggml_type, const unsigned char *block, float out[256]) {
    return qx_decode_supported_block(ggml_type, block, out);
}

QXREF_API float qxref_fp16_to_f32(uint16_t h) { return qx_fp16_to_f32(h); }

QXREF_API uint64_t qxref_fnv1a64(const void *data, uint64_t len) { return qx_fnv1a64(data, len); }

/* The lattice tables compiled into the reference (src/qx_iq2xs_tables.inc). */
QXREF_API const void *qxref_table(uint32_t which) {
    switch (which) {
        case 0: return qx_iq2xs_grid;
        case 1: return qx_iq3xxs_grid;
        case 2: return qx_iq2s_grid;
        case 3: return qx_iq3s_grid;
        case 4: return qx_ksigns_iq2xs;
        default: return NULL;
    }
}

QXREF_API uint32_t qxref_sizeof(uint32_t which) {
    return which == 0 ? (uint32_t)sizeof(qx_header) : which == 1 ? (uint32_t)sizeof(qx_tensor_dir_entry) : 0u;
}

/* The reference's accumulated-KV snapshot writer and reader (INT8 format). */
QXREF_API int qxref_kv_snapshot_write(const char *path, uint32_t layers, uint32_t positions, uint32_t ctx,
                                      uint32_t kv_heads, uint32_t head_dim, uint32_t next_token, uint32_t seed,
                                      const unsigned char *k, const unsigned char *v, const float *ks, const float *vs,
                                      char *err, uint64_t err_len) {
    return qx_write_accumulated_kv_snapshot(path, layers, positions, ctx, kv_heads, head_dim, "int8",
                                            (uint64_t)kv_heads * head_dim, next_token, seed, k, v, ks, vs, err, err_len);
}

QXREF_API int qxref_kv_snapshot_read(const char *path, uint32_t layers, uint32_t ctx, uint32_t kv_heads,
                                     uint32_t head_dim, uint32_t seed, unsigned char *k, unsigned char *v, float *ks,
                                     float *vs, uint32_t *positions, uint32_t *next_token, char *err, uint64_t err_len) {
    return qx_read_accumulated_kv_snapshot(path, layers, ctx, kv_heads, head_dim, "int8", (uint64_t)kv_heads * head_dim,
                                           seed, k, v, ks, vs, positions, next_token, err, err_len);
}
