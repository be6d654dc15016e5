/*
 * Host-side plumbing of the B200 decode engine: the QXF1 container (own
 * reader/validator), FNV-1a, fp16 conversions, the IQ lattice tables, and the
 * seeded synthetic-model generator that stands in for the real GGUF weights.
 *
 * QXF1 on-disk structures must be byte-identical to the reference's
 * (include/qx_format.h:56-82 in the reference): the file format is the
 * drop-in contract, so the field order and sizes here match it exactly
 * (header 272 bytes, directory entry 208 bytes; checked by static asserts).
 */
#ifndef QX_HOST_H
#define QX_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QXH_NAME_MAX 96u
#define QXH_ALIGN 4096ull

/* ggml type ids as stored in qx_tensor_dir_entry.flags */
enum {
    QXH_F32 = 0, QXH_F16 = 1, QXH_Q4_K = 12, QXH_Q5_K = 13, QXH_Q6_K = 14,
    QXH_IQ2_XS = 17, QXH_IQ3_XXS = 18, QXH_IQ3_S = 21, QXH_IQ2_S = 22, QXH_IQ4_XS = 23
};

typedef struct qxh_manifest {          /* qx_model_manifest, include/qx_format.h:41-55 */
    uint32_t model_type, quant_type, layers, hidden, intermediate, q_heads, kv_heads, head_dim, vocab, max_ctx,
        experts, experts_per_token, moe_intermediate;
} qxh_manifest;

typedef struct qxh_header {            /* qx_header, include/qx_format.h:56-68 */
    char magic[4];
    uint32_t version, header_size, dir_entry_size, tensor_count;
    uint64_t dir_offset, data_offset, file_size, manifest_checksum;
    qxh_manifest manifest;
    uint8_t reserved[160];
} qxh_header;

typedef struct qxh_dir_entry {         /* qx_tensor_dir_entry, include/qx_format.h:70-82 */
    char name[QXH_NAME_MAX];
    uint32_t dtype, quant, rank;
    uint64_t dims[4];
    uint64_t offset, byte_size;
    uint32_t group_size, flags;
    uint64_t checksum;
    uint8_t reserved[32];
} qxh_dir_entry;

/* An opened container: either a read-only mmap of a file or a caller image. */
typedef struct qxh_file {
    qxh_header header;
    const qxh_dir_entry *dir;          /* points into the mapping / image */
    const unsigned char *base;         /* byte 0 of the container */
    uint64_t size;
    int mapped;                        /* 1 if base is our own mmap */
} qxh_file;

void qxh_set_err(char *err, uint64_t err_len, const char *msg);
uint64_t qxh_fnv1a64(const void *data, uint64_t len);
float qxh_fp16_to_f32(uint16_t h);       /* exp==31 -> +-65504, as src/qx_format.c:1868 */
uint16_t qxh_f32_to_fp16(float f);       /* round-to-nearest-even */

/* Block geometry for a ggml type: returns 0 if unsupported. */
int qxh_block_info(uint32_t ggml_type, uint32_t *block_values, uint32_t *block_bytes);

/* Open + validate, fail-closed in the order and with the messages of
 * qx_open_file (src/qx_format.c:712-841). */
int qxh_open_path(const char *path, qxh_file *out, char *err, uint64_t err_len);
int qxh_open_image(const void *image, uint64_t size, qxh_file *out, char *err, uint64_t err_len);
void qxh_close(qxh_file *f);
const qxh_dir_entry *qxh_find(const qxh_file *f, const char *name);
int qxh_verify_checksum(const qxh_file *f, const qxh_dir_entry *t, char *err, uint64_t err_len);

/* Expanded IQ lattice tables (bytes), built once from qx_iq_grids.h. */
typedef struct qxh_iq_tables {
    uint8_t iq2xs[512][8];
    uint8_t iq2s[1024][8];
    uint8_t iq3xxs[256][4];
    uint8_t iq3s[512][4];
    uint8_t ksigns[128];
} qxh_iq_tables;
const qxh_iq_tables *qxh_tables(void);

/* ---- seeded synthetic Qwen3-MoE model --------------------------------- */
typedef struct qxh_synth_config {
    uint32_t layers, hidden, q_heads, kv_heads, head_dim, vocab, experts, experts_per_token, moe_intermediate;
    uint32_t attn_type, gate_type, up_type, down_type, embd_type, head_type;   /* ggml types */
    uint64_t seed;
    uint32_t threads;                  /* 0 = all online CPUs */
} qxh_synth_config;

/* Qwen3-30B-A3B geometry with the BASELINE quant mix (IQ4_XS attention,
 * IQ2_XS gate/up, IQ3_XXS down, Q4_K embedding, Q6_K head). */
void qxh_synth_default(qxh_synth_config *cfg, uint64_t seed);
int qxh_synth_image_size(const qxh_synth_config *cfg, uint64_t *size, char *err, uint64_t err_len);
/* Fill `image` (size bytes, from qxh_synth_image_size) with a complete,
 * checksummed QXF1 container. */
int qxh_synth_build(const qxh_synth_config *cfg, void *image, uint64_t size, char *err, uint64_t err_len);
/* Deterministic N(0,1) vector for test inputs (seeded, host only). */
void qxh_normal_vector(uint64_t seed, float *out, uint64_t n);

/* SHA-256 (FIPS 180-4), for the KV snapshot trailer. */
typedef struct qxh_sha256 {
    uint32_t h[8];
    uint64_t bytes;
    unsigned char buf[64];
    uint32_t fill;
} qxh_sha256;
void qxh_sha256_init(qxh_sha256 *s);
void qxh_sha256_update(qxh_sha256 *s, const void *data, uint64_t len);
void qxh_sha256_final(qxh_sha256 *s, unsigned char out[32]);

/* QXKVSNP1 version-2 accumulated-KV snapshot with INT8 KV, the reference's
 * file format and checks (src/qx_format.c:5860-5969): 48-byte header
 * ("QXKVSNP1", version, layers, positions, ctx, kv_heads, head_dim, format 1,
 * bytes per K or V row, next token, seed), then per layer and position the K
 * row, the V row and the two F32 scales, then the SHA-256 of everything
 * before.  Buffers are [layers][ctx][kv_heads*head_dim] and [layers][ctx]. */
int qxh_kv_snapshot_write(const char *path, uint32_t layers, uint32_t positions, uint32_t ctx, uint32_t kv_heads,
                          uint32_t head_dim, uint32_t next_token, uint32_t seed, const int8_t *k, const int8_t *v,
                          const float *kscale, const float *vscale, char *err, uint64_t err_len);
int qxh_kv_snapshot_read(const char *path, uint32_t layers, uint32_t ctx, uint32_t kv_heads, uint32_t head_dim,
                         uint32_t seed, int8_t *k, int8_t *v, float *kscale, float *vscale, uint32_t *positions_out,
                         uint32_t *next_token_out, char *err, uint64_t err_len);

#ifdef __cplusplus
}
#endif
#endif
