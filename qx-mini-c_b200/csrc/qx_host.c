/*
 * Host plumbing: QXF1 reader/validator, FNV-1a, fp16, IQ tables, and the
 * seeded synthetic-model generator.  See qx_host.h.
 */
#define _GNU_SOURCE
#include "qx_host.h"
#include "qx_iq_grids.h"

#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

_Static_assert(sizeof(qxh_header) == 272, "QXF1 header must be 272 bytes");
_Static_assert(sizeof(qxh_dir_entry) == 208, "QXF1 directory entry must be 208 bytes");
_Static_assert(sizeof(qxh_manifest) == 52, "QXF1 manifest must be 52 bytes");

void qxh_set_err(char *err, uint64_t err_len, const char *msg) {
    if (err && err_len) snprintf(err, (size_t)err_len, "%s", msg);
}

/* The QXF1 checksum (qx_fnv1a64, src/qx_format.c:219-227): FNV-1a with
 * prime 1099511628211 but offset basis 1469598103934665603, one decimal
 * digit shorter than the published FNV-1a 64 basis.  Files carry checksums
 * made with this basis, so it is kept exactly. */
uint64_t qxh_fnv1a64(const void *data, uint64_t len) {
    const unsigned char *p = (const unsigned char *)data;
    uint64_t h = 1469598103934665603ull;
    for (uint64_t i = 0; i < len; ++i) { h ^= p[i]; h *= 1099511628211ull; }
    return h;
}

/* IEEE binary16 -> binary32, except that the Inf/NaN exponent maps to the
 * largest finite half (sign | 65504), which is what the reference decoders
 * see (src/qx_format.c:1854-1876). */
float qxh_fp16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
    if (e == 31u) bits = sign | 0x477fe000u;
    else if (e) bits = sign | ((e + 112u) << 23) | (m << 13);
    else if (!m) bits = sign;
    else {
        int shift = 0;
        while (!(m & 0x400u)) { m <<= 1; ++shift; }
        bits = sign | ((uint32_t)(113 - shift) << 23) | ((m & 0x3ffu) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t qxh_f32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    int32_t e = (int32_t)((x >> 23) & 0xffu);
    uint32_t m = x & 0x7fffffu;
    if (e == 0xff) return (uint16_t)(sign | (m ? 0x7e00u : 0x7c00u));
    int32_t he = e - 112;                      /* rebias 127 -> 15 */
    if (he >= 31) return (uint16_t)(sign | 0x7c00u);
    if (he <= 0) {                             /* subnormal half */
        if (he < -10) return sign;
        uint32_t full = m | 0x800000u;
        uint32_t shift = (uint32_t)(14 - he);
        uint32_t q = full >> shift, rem = full & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t q = m >> 13, rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) {
        if (++q == 0x400u) { q = 0; if (++he >= 31) return (uint16_t)(sign | 0x7c00u); }
    }
    return (uint16_t)(sign | ((uint32_t)he << 10) | q);
}

int qxh_block_info(uint32_t t, uint32_t *values, uint32_t *bytes) {
    uint32_t v = 256, b;
    switch (t) {
        case QXH_F32: v = 1; b = 4; break;
        case QXH_F16: v = 1; b = 2; break;
        case QXH_Q4_K: b = 144; break;
        case QXH_Q5_K: b = 176; break;
        case QXH_Q6_K: b = 210; break;
        case QXH_IQ2_XS: b = 74; break;
        case QXH_IQ3_XXS: b = 98; break;
        case QXH_IQ3_S: b = 110; break;
        case QXH_IQ2_S: b = 82; break;
        case QXH_IQ4_XS: b = 136; break;
        default: return 0;
    }
    if (values) *values = v;
    if (bytes) *bytes = b;
    return 1;
}

/* ---- IQ tables --------------------------------------------------------- */
static qxh_iq_tables g_tables;
static pthread_once_t g_tables_once = PTHREAD_ONCE_INIT;

static void build_tables(void) {
    static const uint8_t iq2_mag[3] = {8, 25, 43};
    static const uint8_t iq3xxs_mag[8] = {4, 12, 20, 28, 36, 44, 52, 62};
    for (int i = 0; i < 512; ++i) {
        unsigned c = qx_iq2xs_codes[i];
        for (int j = 0; j < 8; ++j) { g_tables.iq2xs[i][j] = iq2_mag[c % 3u]; c /= 3u; }
    }
    for (int i = 0; i < 1024; ++i) {
        unsigned c = qx_iq2s_codes[i];
        for (int j = 0; j < 8; ++j) { g_tables.iq2s[i][j] = iq2_mag[c % 3u]; c /= 3u; }
    }
    for (int i = 0; i < 256; ++i)
        for (int j = 0; j < 4; ++j) g_tables.iq3xxs[i][j] = iq3xxs_mag[(qx_iq3xxs_codes[i] >> (3 * j)) & 7u];
    for (int i = 0; i < 512; ++i)
        for (int j = 0; j < 4; ++j) g_tables.iq3s[i][j] = (uint8_t)(2u * ((qx_iq3s_codes[i] >> (3 * j)) & 7u) + 1u);
    /* ksigns: the 7 stored sign bits plus an 8th that makes the count even. */
    for (int i = 0; i < 128; ++i) g_tables.ksigns[i] = (uint8_t)(i | ((__builtin_popcount((unsigned)i) & 1) << 7));
}

const qxh_iq_tables *qxh_tables(void) {
    pthread_once(&g_tables_once, build_tables);
    return &g_tables;
}

/* ---- QXF1 open / validate ------------------------------------------------ */
static int traits_ok(const qxh_dir_entry *t) {
    /* ggml type -> (qx dtype, group size) pairs accepted by
     * qx_validate_tensor_traits (src/qx_format.c:693-709). */
    switch (t->flags) {
        case 0: return t->dtype == 2 && t->group_size == 0;
        case 1: return t->dtype == 1 && t->group_size == 0;
        case 8: return t->dtype == 6 && t->group_size == 0;
        case 10: case 17: case 22: return t->dtype == 5 && t->group_size == 64;
        case 11: case 18: case 21: return t->dtype == 4 && t->group_size == 64;
        case 12: case 13: case 14: return t->dtype == 3 && t->group_size == 64;
        case 23: return (t->dtype == 3 && t->group_size == 64) || (t->dtype == 6 && t->group_size == 0);
        default: return 0;
    }
}

static int expected_bytes(const qxh_dir_entry *t, uint64_t elements, uint64_t *out) {
    uint32_t bv, bb;
    if (t->flags == 8) { bv = 32; bb = 34; }
    else if (t->flags == 10) { bv = 256; bb = 84; }
    else if (t->flags == 11) { bv = 256; bb = 110; }
    else if (!qxh_block_info(t->flags, &bv, &bb)) return 0;
    if (t->dims[0] % bv || elements % bv) return 0;
    uint64_t blocks = elements / bv;
    if (blocks > UINT64_MAX / bb) return 0;
    *out = blocks * bb;
    return *out > 0;
}

static int cmp_u64pair(const void *a, const void *b) {
    const uint64_t *x = (const uint64_t *)a, *y = (const uint64_t *)b;
    return x[0] < y[0] ? -1 : x[0] > y[0];
}

static int cmp_name(const void *a, const void *b) {
    return strcmp(*(const char *const *)a, *(const char *const *)b);
}

static int validate(qxh_file *f, char *err, uint64_t err_len) {
    const qxh_header *h = &f->header;
    if (f->size < sizeof(qxh_header)) { qxh_set_err(err, err_len, "short read header"); return 0; }
    if (memcmp(h->magic, "QXF1", 4) != 0) { qxh_set_err(err, err_len, "bad QXF magic"); return 0; }
    if (h->version != 1u) { qxh_set_err(err, err_len, "unsupported QXF version"); return 0; }
    if (h->header_size != sizeof(qxh_header) || h->dir_entry_size != sizeof(qxh_dir_entry)) {
        qxh_set_err(err, err_len, "QXF struct size mismatch"); return 0;
    }
    if (qxh_fnv1a64(&h->manifest, sizeof(h->manifest)) != h->manifest_checksum) {
        qxh_set_err(err, err_len, "manifest checksum mismatch"); return 0;
    }
    const qxh_manifest *m = &h->manifest;
    if ((m->model_type != 1u && m->model_type != 2u) || m->quant_type < 1u || m->quant_type > 5u || !m->layers ||
        !m->hidden || !m->intermediate || !m->q_heads || !m->kv_heads || m->kv_heads > m->q_heads || !m->head_dim ||
        !m->vocab || !m->max_ctx ||
        (m->model_type == 2u && (!m->experts || !m->experts_per_token || m->experts_per_token > m->experts ||
                                 !m->moe_intermediate))) {
        qxh_set_err(err, err_len, "invalid QXF manifest"); return 0;
    }
    if (!h->tensor_count) { qxh_set_err(err, err_len, "empty tensor directory"); return 0; }
    if (h->file_size != f->size) { qxh_set_err(err, err_len, "declared QXF file size does not match file"); return 0; }
    uint64_t dir_bytes = (uint64_t)h->tensor_count * sizeof(qxh_dir_entry);
    if (h->dir_offset < h->header_size || h->dir_offset % QXH_ALIGN || h->data_offset % QXH_ALIGN ||
        h->dir_offset > h->file_size || dir_bytes > h->file_size - h->dir_offset ||
        h->data_offset < h->dir_offset + dir_bytes || h->data_offset > h->file_size) {
        qxh_set_err(err, err_len, "invalid QXF layout"); return 0;
    }
    f->dir = (const qxh_dir_entry *)(f->base + h->dir_offset);
    int meta_only = h->file_size == h->data_offset;
    const char **names = (const char **)malloc(h->tensor_count * sizeof(*names));
    uint64_t *spans = (uint64_t *)malloc(h->tensor_count * 2u * sizeof(uint64_t));
    if (!names || !spans) { free(names); free(spans); qxh_set_err(err, err_len, "out of memory"); return 0; }
    const char *fail = NULL;
    for (uint32_t i = 0; i < h->tensor_count && !fail; ++i) {
        const qxh_dir_entry *t = &f->dir[i];
        if (!memchr(t->name, 0, QXH_NAME_MAX) || !t->name[0]) { fail = "unterminated or empty tensor name"; break; }
        names[i] = t->name;
        if (t->dtype < 1u || t->dtype > 6u || t->quant < 1u || t->quant > 5u || (!meta_only && !traits_ok(t))) {
            fail = "invalid tensor metadata"; break;
        }
        uint64_t elements = 1;
        int dims_ok = t->rank >= 1u && t->rank <= 4u;
        for (uint32_t d = 0; d < 4u && dims_ok; ++d) {
            if (d < t->rank) {
                if (!t->dims[d] || elements > UINT64_MAX / t->dims[d]) dims_ok = 0;
                else elements *= t->dims[d];
            } else if (t->dims[d]) dims_ok = 0;
        }
        if (!dims_ok) { fail = "invalid tensor dimensions"; break; }
        if (meta_only) {
            if (t->offset || t->byte_size) fail = "invalid tensor placement";
            continue;
        }
        if (t->offset < h->data_offset || t->offset % QXH_ALIGN || !t->byte_size || t->offset > h->file_size ||
            t->byte_size > h->file_size - t->offset) { fail = "invalid tensor placement"; break; }
        uint64_t want = 0;
        if (!expected_bytes(t, elements, &want) || want != t->byte_size) {
            fail = "tensor byte size inconsistent with dimensions"; break;
        }
        spans[2 * i] = t->offset;
        spans[2 * i + 1] = t->offset + t->byte_size;
    }
    if (!fail) {
        qsort(names, h->tensor_count, sizeof(*names), cmp_name);
        for (uint32_t i = 1; i < h->tensor_count; ++i)
            if (!strcmp(names[i - 1], names[i])) { fail = "duplicate tensor name"; break; }
    }
    if (!fail && !meta_only) {
        qsort(spans, h->tensor_count, 2u * sizeof(uint64_t), cmp_u64pair);
        uint64_t end = h->data_offset;
        for (uint32_t i = 0; i < h->tensor_count; ++i) {
            if (spans[2 * i] < end) { fail = "overlapping tensor ranges"; break; }
            end = spans[2 * i + 1];
        }
    }
    free(names);
    free(spans);
    if (fail) { qxh_set_err(err, err_len, fail); return 0; }
    return 1;
}

int qxh_open_image(const void *image, uint64_t size, qxh_file *out, char *err, uint64_t err_len) {
    if (!image || !out) { qxh_set_err(err, err_len, "invalid argument"); return 0; }
    memset(out, 0, sizeof(*out));
    out->base = (const unsigned char *)image;
    out->size = size;
    if (size >= sizeof(qxh_header)) memcpy(&out->header, image, sizeof(qxh_header));
    if (!validate(out, err, err_len)) { memset(out, 0, sizeof(*out)); return 0; }
    return 1;
}

int qxh_open_path(const char *path, qxh_file *out, char *err, uint64_t err_len) {
    if (!path || !out) { qxh_set_err(err, err_len, "invalid argument"); return 0; }
    memset(out, 0, sizeof(*out));
    int fd = open(path, O_RDONLY);
    if (fd < 0) { qxh_set_err(err, err_len, strerror(errno)); return 0; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < (off_t)sizeof(qxh_header)) {
        close(fd); qxh_set_err(err, err_len, "short read header"); return 0;
    }
    void *view = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (view == MAP_FAILED) { qxh_set_err(err, err_len, "QXF file mapping failed"); return 0; }
    if (!qxh_open_image(view, (uint64_t)st.st_size, out, err, err_len)) {
        munmap(view, (size_t)st.st_size); return 0;
    }
    out->mapped = 1;
    return 1;
}

void qxh_close(qxh_file *f) {
    if (!f) return;
    if (f->mapped && f->base) munmap((void *)f->base, (size_t)f->size);
    memset(f, 0, sizeof(*f));
}

const qxh_dir_entry *qxh_find(const qxh_file *f, const char *name) {
    if (!f || !f->dir || !name) return NULL;
    for (uint32_t i = 0; i < f->header.tensor_count; ++i)
        if (!strcmp(f->dir[i].name, name)) return &f->dir[i];
    return NULL;
}

int qxh_verify_checksum(const qxh_file *f, const qxh_dir_entry *t, char *err, uint64_t err_len) {
    if (!f || !t) { qxh_set_err(err, err_len, "invalid argument"); return 0; }
    if (t->offset > f->size || t->byte_size > f->size - t->offset) {
        qxh_set_err(err, err_len, "tensor range outside file"); return 0;
    }
    if (qxh_fnv1a64(f->base + t->offset, t->byte_size) != t->checksum) {
        qxh_set_err(err, err_len, "tensor checksum mismatch"); return 0;
    }
    return 1;
}

/* ---- synthetic model ------------------------------------------------------ */
static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

typedef struct rng { uint64_t s; } rng;
static inline uint64_t rnext(rng *r) { return mix64(r->s += 0x9E3779B97F4A7C15ull); }
static inline double runif(rng *r) { return (double)((rnext(r) >> 11) + 1u) * (1.0 / 9007199254740992.0); }
static inline double rnormal(rng *r) {
    double u1 = runif(r), u2 = runif(r);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}
static inline rng rng_for(uint64_t seed, uint64_t tensor, uint64_t block) {
    rng r;
    r.s = mix64(seed * 0x9E3779B97F4A7C15ull ^ mix64(tensor + 0x1234567ull) ^ mix64(block * 0xD1B54A32D192ED03ull + 7u));
    return r;
}

void qxh_normal_vector(uint64_t seed, float *out, uint64_t n) {
    rng r = rng_for(seed, 0xFFFFFFFFull, 0);
    for (uint64_t i = 0; i < n; ++i) out[i] = (float)rnormal(&r);
}

void qxh_synth_default(qxh_synth_config *c, uint64_t seed) {
    memset(c, 0, sizeof(*c));
    c->layers = 48; c->hidden = 2048; c->q_heads = 32; c->kv_heads = 4; c->head_dim = 128; c->vocab = 151936;
    c->experts = 128; c->experts_per_token = 8; c->moe_intermediate = 768;
    c->attn_type = QXH_IQ4_XS; c->gate_type = QXH_IQ2_XS; c->up_type = QXH_IQ2_XS; c->down_type = QXH_IQ3_XXS;
    c->embd_type = QXH_Q4_K; c->head_type = QXH_Q6_K;
    c->seed = seed;
}

enum { K_NORM_ONE, K_ROUTER, K_QUANT };

typedef struct synth_tensor {
    char name[QXH_NAME_MAX];
    uint32_t type, rank, kind;
    uint64_t dims[4];
    uint64_t offset, bytes, blocks;    /* blocks of 256 values (or of 256 floats for F32) */
    uint32_t block_bytes;
    double dscale;                     /* c in d = fp16(|N(0,1)| * c) */
    double dmin_scale;                 /* Q4_K only */
} synth_tensor;

typedef struct synth_plan {
    synth_tensor *t;
    uint32_t count;
    uint64_t data_offset, file_size, dir_offset;
} synth_plan;

/* Second moments of the decoded magnitudes, used to pick block scales so a
 * projection of a unit-RMS input has roughly unit RMS output. */
static double grid_msq(uint32_t type) {
    const qxh_iq_tables *T = qxh_tables();
    double s = 0.0;
    if (type == QXH_IQ2_XS) { for (int i = 0; i < 512; ++i) for (int j = 0; j < 8; ++j) s += T->iq2xs[i][j] * (double)T->iq2xs[i][j]; return s / 4096.0; }
    if (type == QXH_IQ3_XXS) { for (int i = 0; i < 256; ++i) for (int j = 0; j < 4; ++j) s += T->iq3xxs[i][j] * (double)T->iq3xxs[i][j]; return s / 1024.0; }
    if (type == QXH_IQ2_S) { for (int i = 0; i < 1024; ++i) for (int j = 0; j < 8; ++j) s += T->iq2s[i][j] * (double)T->iq2s[i][j]; return s / 8192.0; }
    if (type == QXH_IQ3_S) { for (int i = 0; i < 512; ++i) for (int j = 0; j < 4; ++j) s += T->iq3s[i][j] * (double)T->iq3s[i][j]; return s / 2048.0; }
    return 1.0;
}

static double unit_gain_scale(uint32_t type, uint64_t fan_in) {
    double per = 1.0;                  /* E[(w/d)^2] for uniformly random block bytes */
    switch (type) {
        case QXH_IQ4_XS: per = 341.5 * 4548.0; break;                   /* (ls-32)^2 * kvalues^2 */
        case QXH_IQ2_XS: per = (85.25 / 16.0) * grid_msq(type); break;  /* ((0.5+s)/4)^2 * g^2 */
        case QXH_IQ3_XXS: per = (85.25 / 4.0) * grid_msq(type); break;  /* ((0.5+s)/2)^2 * g^2 */
        case QXH_IQ2_S: per = (85.25 / 16.0) * grid_msq(type); break;   /* ((0.5+s)/4)^2 * g^2 */
        case QXH_IQ3_S: per = 341.0 * grid_msq(type); break;             /* (1+2s)^2 * g^2 */
        case QXH_Q5_K: per = 1312.5 * 325.5; break;                      /* sc^2 * q^2 */
        case QXH_Q6_K: per = 1365.0 * 341.5; break;
        case QXH_Q4_K: per = 1312.5 * 77.5; break;
        default: break;
    }
    return 1.0 / sqrt((double)fan_in * per);
}

static int add_tensor(synth_plan *p, uint32_t cap, const char *name, uint32_t type, uint32_t kind, uint32_t rank,
                      uint64_t d0, uint64_t d1, uint64_t d2) {
    if (p->count >= cap) return 0;
    synth_tensor *t = &p->t[p->count++];
    memset(t, 0, sizeof(*t));
    snprintf(t->name, sizeof(t->name), "%s", name);
    t->type = type; t->kind = kind; t->rank = rank;
    t->dims[0] = d0; t->dims[1] = rank > 1 ? d1 : 0; t->dims[2] = rank > 2 ? d2 : 0;
    uint64_t elems = d0 * (rank > 1 ? d1 : 1) * (rank > 2 ? d2 : 1);
    uint32_t bv = 1, bb = 4;
    if (!qxh_block_info(type, &bv, &bb)) return 0;
    t->bytes = elems / bv * bb;
    t->block_bytes = bb;
    t->blocks = type == QXH_F32 ? (elems + 255u) / 256u : elems / bv;
    if (kind == K_QUANT) t->dscale = unit_gain_scale(type, d0);
    if (type == QXH_Q4_K) t->dmin_scale = 4.0 * t->dscale;
    if (type == QXH_Q5_K) t->dmin_scale = 15.5 * t->dscale;   /* E[sc*q] = 15.5 E[m]: zero-mean weights */
    return 1;
}

static int make_plan(const qxh_synth_config *c, synth_plan *p, char *err, uint64_t err_len) {
    if (!c->layers || !c->hidden || c->hidden % 256u || !c->q_heads || !c->kv_heads || c->q_heads % c->kv_heads ||
        !c->head_dim || (c->q_heads * c->head_dim) % 256u || !c->vocab || c->experts < c->experts_per_token ||
        !c->experts_per_token || !c->moe_intermediate || c->moe_intermediate % 256u) {
        qxh_set_err(err, err_len, "unsupported synthetic model geometry"); return 0;
    }
    uint32_t cap = 3u + c->layers * 12u;
    p->t = (synth_tensor *)calloc(cap, sizeof(synth_tensor));
    p->count = 0;
    if (!p->t) { qxh_set_err(err, err_len, "out of memory"); return 0; }
    uint64_t H = c->hidden, QD = (uint64_t)c->q_heads * c->head_dim, KD = (uint64_t)c->kv_heads * c->head_dim;
    int ok = add_tensor(p, cap, "token_embd.weight", c->embd_type, K_QUANT, 2, H, c->vocab, 0);
    char n[QXH_NAME_MAX];
    for (uint32_t l = 0; l < c->layers && ok; ++l) {
#define L(suffix) (snprintf(n, sizeof(n), "blk.%u." suffix, l), n)
        ok = ok && add_tensor(p, cap, L("attn_norm.weight"), QXH_F32, K_NORM_ONE, 1, H, 0, 0);
        ok = ok && add_tensor(p, cap, L("attn_q.weight"), c->attn_type, K_QUANT, 2, H, QD, 0);
        ok = ok && add_tensor(p, cap, L("attn_k.weight"), c->attn_type, K_QUANT, 2, H, KD, 0);
        ok = ok && add_tensor(p, cap, L("attn_v.weight"), c->attn_type, K_QUANT, 2, H, KD, 0);
        ok = ok && add_tensor(p, cap, L("attn_output.weight"), c->attn_type, K_QUANT, 2, QD, H, 0);
        ok = ok && add_tensor(p, cap, L("attn_q_norm.weight"), QXH_F32, K_NORM_ONE, 1, c->head_dim, 0, 0);
        ok = ok && add_tensor(p, cap, L("attn_k_norm.weight"), QXH_F32, K_NORM_ONE, 1, c->head_dim, 0, 0);
        ok = ok && add_tensor(p, cap, L("ffn_norm.weight"), QXH_F32, K_NORM_ONE, 1, H, 0, 0);
        ok = ok && add_tensor(p, cap, L("ffn_gate_inp.weight"), QXH_F32, K_ROUTER, 2, H, c->experts, 0);
        ok = ok && add_tensor(p, cap, L("ffn_gate_exps.weight"), c->gate_type, K_QUANT, 3, H, c->moe_intermediate, c->experts);
        ok = ok && add_tensor(p, cap, L("ffn_up_exps.weight"), c->up_type, K_QUANT, 3, H, c->moe_intermediate, c->experts);
        ok = ok && add_tensor(p, cap, L("ffn_down_exps.weight"), c->down_type, K_QUANT, 3, c->moe_intermediate, H, c->experts);
#undef L
    }
    ok = ok && add_tensor(p, cap, "output_norm.weight", QXH_F32, K_NORM_ONE, 1, H, 0, 0);
    ok = ok && add_tensor(p, cap, "output.weight", c->head_type, K_QUANT, 2, H, c->vocab, 0);
    if (!ok) { free(p->t); p->t = NULL; qxh_set_err(err, err_len, "unsupported synthetic tensor type"); return 0; }
    /* The BASELINE head distribution: d = fp16(|N(0,1)| * 1e-3). */
    p->t[p->count - 1].dscale = 1.0e-3;
    p->dir_offset = QXH_ALIGN;     /* header (272 B) padded to 4096 */
    uint64_t cur = (p->dir_offset + (uint64_t)p->count * sizeof(qxh_dir_entry) + QXH_ALIGN - 1) / QXH_ALIGN * QXH_ALIGN;
    p->data_offset = cur;
    for (uint32_t i = 0; i < p->count; ++i) {
        p->t[i].offset = cur;
        cur = (cur + p->t[i].bytes + QXH_ALIGN - 1) / QXH_ALIGN * QXH_ALIGN;
    }
    p->file_size = cur;
    return 1;
}

int qxh_synth_image_size(const qxh_synth_config *c, uint64_t *size, char *err, uint64_t err_len) {
    synth_plan p;
    if (!c || !size) { qxh_set_err(err, err_len, "invalid argument"); return 0; }
    if (!make_plan(c, &p, err, err_len)) return 0;
    *size = p.file_size;
    free(p.t);
    return 1;
}

static inline uint16_t half_abs_normal(rng *r, double scale) {
    return qxh_f32_to_fp16((float)(fabs(rnormal(r)) * scale));
}

static inline void put16(unsigned char *p, uint16_t v) { p[0] = (unsigned char)v; p[1] = (unsigned char)(v >> 8); }

static void fill_bytes(rng *r, unsigned char *p, uint32_t n) {
    while (n >= 8) { uint64_t v = rnext(r); memcpy(p, &v, 8); p += 8; n -= 8; }
    if (n) { uint64_t v = rnext(r); memcpy(p, &v, n); }
}

/* One 256-value block (or 256 floats) of tensor t. */
static void gen_block(const synth_tensor *t, uint64_t seed, uint32_t tindex, uint64_t b, unsigned char *dst) {
    rng r = rng_for(seed, tindex, b);
    if (t->type == QXH_F32) {
        uint64_t elems = t->bytes / 4u, first = b * 256u, n = elems - first < 256u ? elems - first : 256u;
        float *f = (float *)(void *)dst;
        for (uint64_t i = 0; i < n; ++i) f[i] = t->kind == K_ROUTER ? (float)(0.02 * rnormal(&r)) : 1.0f;
        return;
    }
    switch (t->type) {
        case QXH_Q6_K:         /* ql[128] qh[64] uniform bits; int8 scales U[-64,63]; d @208 */
            fill_bytes(&r, dst, 192);
            for (int i = 0; i < 16; ++i) dst[192 + i] = (unsigned char)(int8_t)((int)(rnext(&r) & 127u) - 64);
            put16(dst + 208, half_abs_normal(&r, t->dscale));
            break;
        case QXH_Q4_K:         /* d, dmin, scales[12], qs[128] */
        case QXH_Q5_K:         /* d, dmin, scales[12], qh[32], qs[128] */
            put16(dst, half_abs_normal(&r, t->dscale));
            put16(dst + 2, half_abs_normal(&r, t->dmin_scale));
            fill_bytes(&r, dst + 4, t->block_bytes - 4u);
            break;
        default:               /* IQ2_XS/IQ3_XXS/IQ4_XS/...: d @0 then uniform payload */
            put16(dst, half_abs_normal(&r, t->dscale));
            fill_bytes(&r, dst + 2, t->block_bytes - 2u);
            break;
    }
}

typedef struct synth_job {
    const synth_plan *p;
    const qxh_synth_config *c;
    unsigned char *image;
    uint32_t nthreads, tid;
    uint64_t total_blocks;
    uint64_t *prefix;        /* cumulative blocks per tensor */
    int phase;               /* 0 = fill, 1 = checksum */
    uint32_t *order;         /* tensor order for checksums (largest first) */
    volatile uint32_t *next; /* shared cursor for checksum phase */
} synth_job;

static void *synth_worker(void *arg) {
    synth_job *j = (synth_job *)arg;
    const synth_plan *p = j->p;
    if (j->phase == 0) {
        uint64_t per = (j->total_blocks + j->nthreads - 1) / j->nthreads;
        uint64_t lo = per * j->tid, hi = lo + per > j->total_blocks ? j->total_blocks : lo + per;
        uint32_t ti = 0;
        for (uint64_t g = lo; g < hi; ++g) {
            while (j->prefix[ti + 1] <= g) ++ti;
            const synth_tensor *t = &p->t[ti];
            uint64_t b = g - j->prefix[ti];
            unsigned char *dst = j->image + t->offset + (t->type == QXH_F32 ? b * 1024u : b * t->block_bytes);
            gen_block(t, j->c->seed, ti, b, dst);
        }
    } else {
        qxh_dir_entry *dir = (qxh_dir_entry *)(void *)(j->image + p->dir_offset);
        for (;;) {
            uint32_t k = __atomic_fetch_add(j->next, 1u, __ATOMIC_RELAXED);
            if (k >= p->count) break;
            uint32_t i = j->order[k];
            dir[i].checksum = qxh_fnv1a64(j->image + p->t[i].offset, p->t[i].bytes);
        }
    }
    return NULL;
}

static int cmp_size_desc(const void *a, const void *b, void *ctx) {
    const synth_plan *p = (const synth_plan *)ctx;
    uint64_t x = p->t[*(const uint32_t *)a].bytes, y = p->t[*(const uint32_t *)b].bytes;
    return x < y ? 1 : x > y ? -1 : 0;
}

static uint32_t dtype_for(uint32_t type) {
    switch (type) {
        case QXH_F32: return 2;
        case QXH_F16: return 1;
        case QXH_Q4_K: case QXH_Q5_K: case QXH_Q6_K: case QXH_IQ4_XS: return 3;
        case QXH_IQ3_XXS: case QXH_IQ3_S: return 4;
        case QXH_IQ2_XS: case QXH_IQ2_S: return 5;
        default: return 6;
    }
}

static int run_threads(synth_job *tmpl, uint32_t n) {
    pthread_t *th = (pthread_t *)calloc(n, sizeof(pthread_t));
    synth_job *jobs = (synth_job *)calloc(n, sizeof(synth_job));
    if (!th || !jobs) { free(th); free(jobs); return 0; }
    for (uint32_t i = 0; i < n; ++i) {
        jobs[i] = *tmpl;
        jobs[i].tid = i;
        if (pthread_create(&th[i], NULL, synth_worker, &jobs[i]) != 0) {
            for (uint32_t k = 0; k < i; ++k) pthread_join(th[k], NULL);
            free(th); free(jobs); return 0;
        }
    }
    for (uint32_t i = 0; i < n; ++i) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
    return 1;
}

int qxh_synth_build(const qxh_synth_config *c, void *image_v, uint64_t size, char *err, uint64_t err_len) {
    unsigned char *image = (unsigned char *)image_v;
    synth_plan p;
    if (!c || !image) { qxh_set_err(err, err_len, "invalid argument"); return 0; }
    if (!make_plan(c, &p, err, err_len)) return 0;
    if (size != p.file_size) { free(p.t); qxh_set_err(err, err_len, "synthetic image size mismatch"); return 0; }
    memset(image, 0, p.data_offset);
    /* zero the alignment padding between tensors */
    for (uint32_t i = 0; i < p.count; ++i) {
        uint64_t end = p.t[i].offset + p.t[i].bytes;
        uint64_t next = i + 1 < p.count ? p.t[i + 1].offset : p.file_size;
        memset(image + end, 0, next - end);
    }
    qxh_header *h = (qxh_header *)(void *)image;
    memcpy(h->magic, "QXF1", 4);
    h->version = 1; h->header_size = sizeof(qxh_header); h->dir_entry_size = sizeof(qxh_dir_entry);
    h->tensor_count = p.count; h->dir_offset = p.dir_offset; h->data_offset = p.data_offset; h->file_size = p.file_size;
    qxh_manifest *m = &h->manifest;
    m->model_type = 2; m->quant_type = 5; m->layers = c->layers; m->hidden = c->hidden; m->intermediate = 6144;
    m->q_heads = c->q_heads; m->kv_heads = c->kv_heads; m->head_dim = c->head_dim; m->vocab = c->vocab;
    m->max_ctx = 40960; m->experts = c->experts; m->experts_per_token = c->experts_per_token;
    m->moe_intermediate = c->moe_intermediate;
    h->manifest_checksum = qxh_fnv1a64(m, sizeof(*m));
    qxh_dir_entry *dir = (qxh_dir_entry *)(void *)(image + p.dir_offset);
    for (uint32_t i = 0; i < p.count; ++i) {
        const synth_tensor *t = &p.t[i];
        qxh_dir_entry *e = &dir[i];
        memcpy(e->name, t->name, QXH_NAME_MAX);
        e->dtype = dtype_for(t->type);
        e->quant = 5;
        e->rank = t->rank;
        for (int d = 0; d < 4; ++d) e->dims[d] = t->dims[d];
        e->offset = t->offset;
        e->byte_size = t->bytes;
        e->group_size = t->type == QXH_F32 || t->type == QXH_F16 ? 0u : 64u;
        e->flags = t->type;
    }
    uint64_t *prefix = (uint64_t *)calloc(p.count + 1u, sizeof(uint64_t));
    uint32_t *order = (uint32_t *)calloc(p.count, sizeof(uint32_t));
    if (!prefix || !order) { free(prefix); free(order); free(p.t); qxh_set_err(err, err_len, "out of memory"); return 0; }
    for (uint32_t i = 0; i < p.count; ++i) { prefix[i + 1] = prefix[i] + p.t[i].blocks; order[i] = i; }
    uint32_t n = c->threads;
    if (!n) { long on = sysconf(_SC_NPROCESSORS_ONLN); n = on > 0 ? (uint32_t)on : 1u; }
    if (n > 256u) n = 256u;
    volatile uint32_t next = 0;
    synth_job tmpl;
    memset(&tmpl, 0, sizeof(tmpl));
    tmpl.p = &p; tmpl.c = c; tmpl.image = image; tmpl.nthreads = n; tmpl.total_blocks = prefix[p.count];
    tmpl.prefix = prefix; tmpl.order = order; tmpl.next = &next;
    int ok = run_threads(&tmpl, n);
    if (ok) {
        qsort_r(order, p.count, sizeof(uint32_t), cmp_size_desc, &p);
        tmpl.phase = 1;
        ok = run_threads(&tmpl, n);
    }
    free(prefix);
    free(order);
    free(p.t);
    if (!ok) { qxh_set_err(err, err_len, "thread start failed"); return 0; }
    return 1;
}

/* ---- SHA-256 (FIPS 180-4) ------------------------------------------------ */

static const uint32_t qxh_sha_k[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

#define QXH_ROR(x, n) (((x) >> (n)) | ((x) << (32 - (n))))

static void qxh_sha256_block(qxh_sha256 *s, const unsigned char *p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
        w[i] = ((uint32_t)p[4 * i] << 24) | ((uint32_t)p[4 * i + 1] << 16) | ((uint32_t)p[4 * i + 2] << 8) | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
        const uint32_t a = w[i - 15], b = w[i - 2];
        w[i] = w[i - 16] + (QXH_ROR(a, 7) ^ QXH_ROR(a, 18) ^ (a >> 3)) + w[i - 7] + (QXH_ROR(b, 17) ^ QXH_ROR(b, 19) ^ (b >> 10));
    }
    uint32_t v[8];
    memcpy(v, s->h, sizeof v);
    for (int i = 0; i < 64; ++i) {
        const uint32_t e = v[4], a = v[0];
        const uint32_t t1 = v[7] + (QXH_ROR(e, 6) ^ QXH_ROR(e, 11) ^ QXH_ROR(e, 25)) + ((e & v[5]) ^ (~e & v[6])) +
                            qxh_sha_k[i] + w[i];
        const uint32_t t2 = (QXH_ROR(a, 2) ^ QXH_ROR(a, 13) ^ QXH_ROR(a, 22)) + ((a & v[1]) ^ (a & v[2]) ^ (v[1] & v[2]));
        memmove(v + 1, v, 7 * sizeof(uint32_t));
        v[4] += t1;
        v[0] = t1 + t2;
    }
    for (int i = 0; i < 8; ++i) s->h[i] += v[i];
}

void qxh_sha256_init(qxh_sha256 *s) {
    static const uint32_t h0[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    memcpy(s->h, h0, sizeof h0);
    s->bytes = 0;
    s->fill = 0;
}

void qxh_sha256_update(qxh_sha256 *s, const void *data, uint64_t len) {
    const unsigned char *p = (const unsigned char *)data;
    s->bytes += len;
    while (len) {
        uint32_t take = 64u - s->fill;
        if (take > len) take = (uint32_t)len;
        memcpy(s->buf + s->fill, p, take);
        s->fill += take;
        p += take;
        len -= take;
        if (s->fill == 64u) {
            qxh_sha256_block(s, s->buf);
            s->fill = 0;
        }
    }
}

void qxh_sha256_final(qxh_sha256 *s, unsigned char out[32]) {
    const uint64_t bits = s->bytes * 8u;
    const unsigned char one = 0x80u, zero = 0u;
    qxh_sha256_update(s, &one, 1);
    while (s->fill != 56u) qxh_sha256_update(s, &zero, 1);
    unsigned char len[8];
    for (int i = 0; i < 8; ++i) len[i] = (unsigned char)(bits >> (56 - 8 * i));
    qxh_sha256_update(s, len, 8);
    for (int i = 0; i < 8; ++i) {
        out[4 * i] = (unsigned char)(s->h[i] >> 24);
        out[4 * i + 1] = (unsigned char)(s->h[i] >> 16);
        out[4 * i + 2] = (unsigned char)(s->h[i] >> 8);
        out[4 * i + 3] = (unsigned char)s->h[i];
    }
}

/* ---- QXKVSNP1 accumulated-KV snapshot (INT8 KV) ---------------------------- */

static void qxh_le32(unsigned char *p, uint32_t v) {
    p[0] = (unsigned char)v; p[1] = (unsigned char)(v >> 8); p[2] = (unsigned char)(v >> 16); p[3] = (unsigned char)(v >> 24);
}
static uint32_t qxh_rd32(const unsigned char *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

int qxh_kv_snapshot_write(const char *path, uint32_t layers, uint32_t positions, uint32_t ctx, uint32_t kv_heads,
                          uint32_t head_dim, uint32_t next_token, uint32_t seed, const int8_t *k, const int8_t *v,
                          const float *kscale, const float *vscale, char *err, uint64_t err_len) {
    const uint64_t row = (uint64_t)kv_heads * head_dim;
    if (!path || !*path || !k || !v || !kscale || !vscale || positions == 0u || positions > ctx || row > UINT32_MAX) {
        qxh_set_err(err, err_len, "invalid accumulated KV snapshot output");
        return 0;
    }
    FILE *fp = fopen(path, "wb");
    if (!fp) { qxh_set_err(err, err_len, "cannot open accumulated KV snapshot output"); return 0; }
    unsigned char hdr[48] = {0};
    memcpy(hdr, "QXKVSNP1", 8);
    const uint32_t fields[10] = {2u, layers, positions, ctx, kv_heads, head_dim, 1u /* int8 */, (uint32_t)row,
                                 next_token, seed};
    for (int i = 0; i < 10; ++i) qxh_le32(hdr + 8 + 4 * i, fields[i]);
    qxh_sha256 h;
    qxh_sha256_init(&h);
    qxh_sha256_update(&h, hdr, sizeof hdr);
    int ok = fwrite(hdr, 1, sizeof hdr, fp) == sizeof hdr;
    for (uint32_t l = 0; l < layers && ok; ++l)
        for (uint32_t p = 0; p < positions && ok; ++p) {
            const uint64_t slot = (uint64_t)l * ctx + p;
            unsigned char sc[8];
            uint32_t bits;
            memcpy(&bits, &kscale[slot], 4); qxh_le32(sc, bits);
            memcpy(&bits, &vscale[slot], 4); qxh_le32(sc + 4, bits);
            qxh_sha256_update(&h, k + slot * row, row);
            qxh_sha256_update(&h, v + slot * row, row);
            qxh_sha256_update(&h, sc, 8);
            ok = fwrite(k + slot * row, 1, (size_t)row, fp) == row && fwrite(v + slot * row, 1, (size_t)row, fp) == row &&
                 fwrite(sc, 1, 8, fp) == 8;
        }
    unsigned char digest[32];
    qxh_sha256_final(&h, digest);
    if (ok) ok = fwrite(digest, 1, 32, fp) == 32;
    if (fclose(fp) != 0) ok = 0;
    if (!ok) qxh_set_err(err, err_len, "cannot write complete accumulated KV snapshot");
    return ok;
}

int qxh_kv_snapshot_read(const char *path, uint32_t layers, uint32_t ctx, uint32_t kv_heads, uint32_t head_dim,
                         uint32_t seed, int8_t *k, int8_t *v, float *kscale, float *vscale, uint32_t *positions_out,
                         uint32_t *next_token_out, char *err, uint64_t err_len) {
    const uint64_t row = (uint64_t)kv_heads * head_dim;
    FILE *fp = path ? fopen(path, "rb") : NULL;
    if (!fp) { qxh_set_err(err, err_len, "cannot open accumulated KV snapshot input"); return 0; }
    unsigned char hdr[48];
    int ok = fread(hdr, 1, sizeof hdr, fp) == sizeof hdr;
    const uint32_t positions = ok ? qxh_rd32(hdr + 16) : 0u;
    if (!ok || memcmp(hdr, "QXKVSNP1", 8) != 0 || qxh_rd32(hdr + 8) != 2u || qxh_rd32(hdr + 12) != layers ||
        positions == 0u || positions > ctx || qxh_rd32(hdr + 20) != ctx || qxh_rd32(hdr + 24) != kv_heads ||
        qxh_rd32(hdr + 28) != head_dim || qxh_rd32(hdr + 32) != 1u || qxh_rd32(hdr + 36) != row ||
        qxh_rd32(hdr + 44) != seed) {
        fclose(fp);
        qxh_set_err(err, err_len, "accumulated KV snapshot header mismatch");
        return 0;
    }
    qxh_sha256 h;
    qxh_sha256_init(&h);
    qxh_sha256_update(&h, hdr, sizeof hdr);
    for (uint32_t l = 0; l < layers && ok; ++l)
        for (uint32_t p = 0; p < positions && ok; ++p) {
            const uint64_t slot = (uint64_t)l * ctx + p;
            unsigned char sc[8];
            ok = fread(k + slot * row, 1, (size_t)row, fp) == row && fread(v + slot * row, 1, (size_t)row, fp) == row &&
                 fread(sc, 1, 8, fp) == 8;
            if (!ok) break;
            qxh_sha256_update(&h, k + slot * row, row);
            qxh_sha256_update(&h, v + slot * row, row);
            qxh_sha256_update(&h, sc, 8);
            uint32_t kb = qxh_rd32(sc), vb = qxh_rd32(sc + 4);
            memcpy(&kscale[slot], &kb, 4);
            memcpy(&vscale[slot], &vb, 4);
            if (!isfinite(kscale[slot]) || !isfinite(vscale[slot])) ok = 0;
        }
    unsigned char want[32], got[32];
    if (ok) ok = fread(want, 1, 32, fp) == 32;
    if (ok) {
        qxh_sha256_final(&h, got);
        ok = memcmp(want, got, 32) == 0;
    }
    if (ok && fgetc(fp) != EOF) ok = 0;
    if (fclose(fp) != 0) ok = 0;
    if (!ok) { qxh_set_err(err, err_len, "accumulated KV snapshot payload mismatch"); return 0; }
    *positions_out = positions;
    *next_token_out = qxh_rd32(hdr + 40);
    return 1;
}
