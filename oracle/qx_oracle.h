/*
 * TEST INFRASTRUCTURE ONLY - CPU restatement of the reference's decode path.
 *
 * qx_oracle.c restates, in this repository's own code, the F32 forward path
 * of qx-mini-c's state loop (src/qx_format.c, cited per function) so that
 * the CUDA engine can be checked without the reference tree.  It is pinned
 * against the reference itself (oracle/_ref/libqxref.so, built from the
 * reference sources by oracle/Makefile): tests/test_oracle_pin.py requires
 * bit-identical outputs on the same inputs.  Only tests/, smoke() and
 * bench.py's CPU legs may load it; the engine never does.
 *
 * The entry points mirror ref_shim.c one for one (prefix qxo_ instead of
 * qxref_).  Rows of every matvec are split across threads (qxo_set_threads);
 * each row is still summed in the reference's order, so results do not depend
 * on the thread count.
 */
#ifndef QX_ORACLE_H
#define QX_ORACLE_H
#include <stdint.h>

typedef struct qxo_model qxo_model;

int qxo_open_path(const char *path, int use_mmap, qxo_model **out, char *err, uint64_t err_len);
int qxo_open_image(const unsigned char *image, uint64_t size, qxo_model **out, char *err, uint64_t err_len);
void qxo_close(qxo_model *m);
void qxo_set_threads(uint32_t n);
int qxo_embed(qxo_model *m, uint32_t token, float *out, char *err, uint64_t err_len);
int qxo_final_head(qxo_model *m, const float *residual, float *normalized, float *logits, uint32_t top_n,
                   uint32_t *top_tokens, double *top_logits, char *err, uint64_t err_len);
int qxo_moe_layer(qxo_model *m, uint32_t layer, const float *residual_after_attention, float *layer_output,
                  float *moe_output, uint32_t selected[8], double weights[8], char *err, uint64_t err_len);
int qxo_attention_layer(qxo_model *m, uint32_t layer, uint32_t step, uint32_t ctx, int8_t *kcache, int8_t *vcache,
                        float *kscales, float *vscales, float *residual, float *attn_out, float *context,
                        float *k_out, float *v_out, char *err, uint64_t err_len);
int qxo_decode_step(qxo_model *m, uint32_t token, uint32_t step, uint32_t ctx, int8_t *kcache, int8_t *vcache,
                    float *kscales, float *vscales, uint32_t *experts_out, double *routing_out, float *residual_out,
                    float *logits, uint32_t *next_token, double *top2_logits, char *err, uint64_t err_len);
float qxo_quantize_int8(const float *src, int8_t *dst, uint32_t n);
void qxo_rope(float *vec, uint32_t heads, uint32_t head_dim, uint32_t position);
int qxo_decode_block(uint32_t ggml_type, const unsigned char *block, float out[256]);
float qxo_fp16_to_f32(uint16_t h);
uint64_t qxo_fnv1a64(const void *data, uint64_t len);

#endif
