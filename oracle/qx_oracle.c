/*
 * TEST INFRASTRUCTURE ONLY - CPU restatement of the reference decode path.
 * See qx_oracle.h.  Citations are to the reference's src/qx_format.c.
 *
 * Numerics follow the reference operation by operation:
 *   - weights are decoded to float exactly as the block decoders do, and
 *     every dot product is accumulated in double in input order
 *     (qx_projection_matvec_fill_mode :4266-4280, packed experts :4774-4783,
 *     head :3683-3711);
 *   - norms, softmaxes, RoPE and SwiGLU are computed in double and rounded to
 *     float where the reference stores floats.
 */
#define _GNU_SOURCE
#include "qx_oracle.h"
#include "qx_host.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define QXO_API __attribute__((visibility("default")))

struct qxo_model {
    qxh_file f;
    unsigned char *owned;              /* image copy for qxo_open_path (read from mmap) */
};

static uint32_t g_threads = 1;
QXO_API void qxo_set_threads(uint32_t n) { g_threads = n ? n : 1; }

QXO_API float qxo_fp16_to_f32(uint16_t h) { return qxh_fp16_to_f32(h); }
QXO_API uint64_t qxo_fnv1a64(const void *d, uint64_t n) { return qxh_fnv1a64(d, n); }

static inline uint16_t rd16(const unsigned char *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const unsigned char *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline float rdf32(const unsigned char *p) { uint32_t b = rd32(p); float f; memcpy(&f, &b, 4); return f; }

/* ---- block decoders (weights as the reference's float values) ---------- */

/* IQ2_XS, src/qx_format.c:1914-1933: 8 groups of 32; each u16 holds a 9-bit
 * lattice index and a 7-bit sign index; two 4-bit scales per group. */
static void dec_iq2_xs(const unsigned char *b, float *out) {
    const qxh_iq_tables *T = qxh_tables();
    float d = qxh_fp16_to_f32(rd16(b));
    for (int g = 0; g < 8; ++g) {
        unsigned char sc = b[66 + g];
        float lo = d * (0.5f + (float)(sc & 15)) * 0.25f;
        float hi = d * (0.5f + (float)(sc >> 4)) * 0.25f;
        for (int l = 0; l < 4; ++l) {
            uint16_t q = rd16(b + 2 + 2 * (4 * g + l));
            const uint8_t *grid = T->iq2xs[q & 511u];
            uint8_t s = T->ksigns[q >> 9];
            float db = l < 2 ? lo : hi;
            for (int j = 0; j < 8; ++j) out[32 * g + 8 * l + j] = db * (float)grid[j] * ((s >> j) & 1 ? -1.0f : 1.0f);
        }
    }
}

/* IQ3_XXS, :1935-1959: per group of 32 a u32 carries four 7-bit sign indices
 * and a 4-bit scale; qs holds 8-bit lattice indices of 4 values each. */
static void dec_iq3_xxs(const unsigned char *b, float *out) {
    const qxh_iq_tables *T = qxh_tables();
    float d = qxh_fp16_to_f32(rd16(b));
    for (int g = 0; g < 8; ++g) {
        uint32_t aux = rd32(b + 66 + 4 * g);
        float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
        for (int l = 0; l < 4; ++l) {
            uint8_t s = T->ksigns[(aux >> (7 * l)) & 127u];
            const uint8_t *g1 = T->iq3xxs[b[2 + 8 * g + 2 * l]];
            const uint8_t *g2 = T->iq3xxs[b[2 + 8 * g + 2 * l + 1]];
            for (int j = 0; j < 4; ++j) {
                out[32 * g + 8 * l + j] = db * (float)g1[j] * ((s >> j) & 1 ? -1.0f : 1.0f);
                out[32 * g + 8 * l + 4 + j] = db * (float)g2[j] * ((s >> (j + 4)) & 1 ? -1.0f : 1.0f);
            }
        }
    }
}

static const signed char kv_iq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

/* IQ4_XS, :2036-2053: 6-bit sub-block scales (4 low bits in scales_l, 2 high
 * in scales_h), non-linear 4-bit codebook. */
static void dec_iq4_xs(const unsigned char *b, float *out) {
    float d = qxh_fp16_to_f32(rd16(b));
    uint16_t sh = rd16(b + 2);
    for (int g = 0; g < 8; ++g) {
        int ls = ((b[4 + g / 2] >> (4 * (g % 2))) & 15) | (((sh >> (2 * g)) & 3) << 4);
        float dl = d * (float)(ls - 32);
        const unsigned char *qs = b + 8 + 16 * g;
        for (int j = 0; j < 16; ++j) {
            out[32 * g + j] = dl * (float)kv_iq4nl[qs[j] & 15];
            out[32 * g + 16 + j] = dl * (float)kv_iq4nl[qs[j] >> 4];
        }
    }
}

/* K-quant 6-bit scale/min unpacking, :2079-2087. */
static void scale_min_k4(int j, const unsigned char *q, unsigned *sc, unsigned *mn) {
    if (j < 4) { *sc = q[j] & 63u; *mn = q[j + 4] & 63u; }
    else { *sc = (q[j + 4] & 15u) | ((q[j - 4] >> 6) << 4); *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
}

/* Q4_K, :2089-2110. */
static void dec_q4_k(const unsigned char *b, float *out) {
    float d = qxh_fp16_to_f32(rd16(b)), dmin = qxh_fp16_to_f32(rd16(b + 2));
    const unsigned char *q = b + 16;
    for (int c = 0; c < 4; ++c) {
        unsigned s1, m1, s2, m2;
        scale_min_k4(2 * c, b + 4, &s1, &m1);
        scale_min_k4(2 * c + 1, b + 4, &s2, &m2);
        float d1 = d * (float)s1, n1 = dmin * (float)m1, d2 = d * (float)s2, n2 = dmin * (float)m2;
        for (int l = 0; l < 32; ++l) out[64 * c + l] = d1 * (float)(q[l] & 15) - n1;
        for (int l = 0; l < 32; ++l) out[64 * c + 32 + l] = d2 * (float)(q[l] >> 4) - n2;
        q += 32;
    }
}

/* Q6_K, :2147-2169: low 4 bits in ql, high 2 in qh, int8 scales per 16. */
static void dec_q6_k(const unsigned char *b, float *out) {
    float d = qxh_fp16_to_f32(rd16(b + 208));
    for (int h = 0; h < 2; ++h) {
        const unsigned char *ql = b + 64 * h, *qh = b + 128 + 32 * h;
        const signed char *sc = (const signed char *)(b + 192 + 8 * h);
        for (int l = 0; l < 32; ++l) {
            int is = l / 16;
            int q1 = (int)((ql[l] & 15) | ((qh[l] & 3) << 4)) - 32;
            int q2 = (int)((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            out[128 * h + l] = d * (float)sc[is] * (float)q1;
            out[128 * h + l + 32] = d * (float)sc[is + 2] * (float)q2;
            out[128 * h + l + 64] = d * (float)sc[is + 4] * (float)q3;
            out[128 * h + l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
    }
}

QXO_API int qxo_decode_block(uint32_t type, const unsigned char *b, float out[256]) {
    switch (type) {
        case QXH_IQ2_XS: dec_iq2_xs(b, out); return 1;
        case QXH_IQ3_XXS: dec_iq3_xxs(b, out); return 1;
        case QXH_IQ4_XS: dec_iq4_xs(b, out); return 1;
        case QXH_Q4_K: dec_q4_k(b, out); return 1;
        case QXH_Q6_K: dec_q6_k(b, out); return 1;
        default: return 0;
    }
}

/* ---- threaded row-parallel matvec ----------------------------------------- */
typedef struct mv_job {
    const unsigned char *rows;        /* first row */
    uint64_t row_bytes;
    uint32_t type, blocks, r0, r1;
    const float *x;
    double *out;
} mv_job;

static void *mv_worker(void *a) {
    mv_job *j = (mv_job *)a;
    uint32_t bb = 0;
    qxh_block_info(j->type, NULL, &bb);
    float w[256];
    for (uint32_t r = j->r0; r < j->r1; ++r) {
        const unsigned char *row = j->rows + (uint64_t)r * j->row_bytes;
        double dot = 0.0;
        if (j->type == QXH_F32) {
            for (uint32_t i = 0; i < j->blocks * 256u; ++i) dot += (double)rdf32(row + 4u * i) * (double)j->x[i];
        } else {
            for (uint32_t b = 0; b < j->blocks; ++b) {
                qxo_decode_block(j->type, row + (uint64_t)b * bb, w);
                for (int i = 0; i < 256; ++i) dot += (double)w[i] * (double)j->x[256u * b + i];
            }
        }
        j->out[r] = dot;
    }
    return NULL;
}

/* out[r] = sum_i W[r][i] * x[i] in double, one row per call of the reference's
 * inner loop; rows split over g_threads threads. */
static void matvec(const unsigned char *rows, uint32_t type, uint32_t nrows, uint32_t in_dims, const float *x,
                   double *out) {
    uint32_t bb = 4, blocks = in_dims / 256u;
    qxh_block_info(type, NULL, &bb);
    uint64_t row_bytes = type == QXH_F32 ? 4ull * in_dims : (uint64_t)blocks * bb;
    uint32_t n = g_threads > nrows ? nrows : g_threads;
    if (n <= 1) {
        mv_job j = {rows, row_bytes, type, blocks, 0, nrows, x, out};
        mv_worker(&j);
        return;
    }
    pthread_t th[256];
    mv_job jobs[256];
    int joined[256];
    if (n > 256) n = 256;
    uint32_t per = (nrows + n - 1) / n;
    for (uint32_t t = 0; t < n; ++t) {
        uint32_t r0 = t * per, r1 = r0 + per > nrows ? nrows : r0 + per;
        jobs[t] = (mv_job){rows, row_bytes, type, blocks, r0 < nrows ? r0 : nrows, r1, x, out};
        joined[t] = 0;
        if (jobs[t].r0 >= jobs[t].r1) continue;
        if (pthread_create(&th[t], NULL, mv_worker, &jobs[t]) == 0) joined[t] = 1;
        else mv_worker(&jobs[t]);
    }
    for (uint32_t t = 0; t < n; ++t)
        if (joined[t]) pthread_join(th[t], NULL);
}

/* ---- model access ----------------------------------------------------------- */
QXO_API int qxo_open_image(const unsigned char *image, uint64_t size, qxo_model **out, char *err, uint64_t err_len) {
    if (!out) { qxh_set_err(err, err_len, "invalid argument"); return 0; }
    qxo_model *m = (qxo_model *)calloc(1, sizeof(*m));
    if (!m) { qxh_set_err(err, err_len, "out of memory"); return 0; }
    if (!qxh_open_image(image, size, &m->f, err, err_len)) { free(m); return 0; }
    *out = m;
    return 1;
}

QXO_API int qxo_open_path(const char *path, int use_mmap, qxo_model **out, char *err, uint64_t err_len) {
    (void)use_mmap;
    if (!out) { qxh_set_err(err, err_len, "invalid argument"); return 0; }
    qxo_model *m = (qxo_model *)calloc(1, sizeof(*m));
    if (!m) { qxh_set_err(err, err_len, "out of memory"); return 0; }
    if (!qxh_open_path(path, &m->f, err, err_len)) { free(m); return 0; }
    *out = m;
    return 1;
}

QXO_API void qxo_close(qxo_model *m) {
    if (!m) return;
    qxh_close(&m->f);
    free(m->owned);
    free(m);
}

static const qxh_dir_entry *need(qxo_model *m, const char *name, char *err, uint64_t err_len) {
    const qxh_dir_entry *t = qxh_find(&m->f, name);
    if (!t) qxh_set_err(err, err_len, "tensor not found");
    return t;
}

static const qxh_dir_entry *needl(qxo_model *m, uint32_t layer, const char *suffix, char *err, uint64_t err_len) {
    char name[QXH_NAME_MAX];
    snprintf(name, sizeof(name), "blk.%u.%s", layer, suffix);
    return need(m, name, err, err_len);
}

static const unsigned char *data(qxo_model *m, const qxh_dir_entry *t) { return m->f.base + t->offset; }

/* RMSNorm, :3358-3371: rms = sqrt(sum x^2 / n + 1e-6) in double; each value
 * is (float)(x / rms) then multiplied by the float weight in float. */
static void rmsnorm(const float *x, const unsigned char *w, float *dst, uint32_t n) {
    double ss = 0.0;
    for (uint32_t i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    double rms = sqrt(ss / (double)n + 1.0e-6);
    for (uint32_t i = 0; i < n; ++i) dst[i] = (float)((double)x[i] / rms) * rdf32(w + 4u * i);
}

/* Per-head RMSNorm, :3740-3757: multiplies by 1/rms (double) and the weight in double. */
static void head_rmsnorm(float *v, const unsigned char *w, uint32_t heads, uint32_t hd) {
    for (uint32_t h = 0; h < heads; ++h) {
        float *x = v + (uint64_t)h * hd;
        double ss = 0.0;
        for (uint32_t i = 0; i < hd; ++i) ss += (double)x[i] * (double)x[i];
        double inv = 1.0 / sqrt(ss / (double)hd + 1.0e-6);
        for (uint32_t i = 0; i < hd; ++i) x[i] = (float)((double)x[i] * inv * (double)rdf32(w + 4u * i));
    }
}

/* Split-half RoPE with theta 1e6, :4625-4641. */
QXO_API void qxo_rope(float *vec, uint32_t heads, uint32_t hd, uint32_t pos) {
    uint32_t half = hd / 2u;
    for (uint32_t h = 0; h < heads; ++h) {
        float *x = vec + (uint64_t)h * hd;
        for (uint32_t i = 0; i < half; ++i) {
            double f = pow(1000000.0, -(2.0 * (double)i) / (double)hd);
            double a = (double)pos * f, c = cos(a), s = sin(a);
            float x0 = x[i], x1 = x[i + half];
            x[i] = (float)((double)x0 * c - (double)x1 * s);
            x[i + half] = (float)((double)x0 * s + (double)x1 * c);
        }
    }
}

/* Dynamic INT8, :4449-4463: one scale (absmax/127, or 1) for the whole vector. */
QXO_API float qxo_quantize_int8(const float *src, int8_t *dst, uint32_t n) {
    float amax = 0.0f;
    for (uint32_t i = 0; i < n; ++i) {
        float a = isfinite(src[i]) ? fabsf(src[i]) : 0.0f;
        if (a > amax) amax = a;
    }
    float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
    for (uint32_t i = 0; i < n; ++i) {
        int q = isfinite(src[i]) ? (int)lrintf(src[i] / scale) : 0;
        dst[i] = (int8_t)(q < -127 ? -127 : q > 127 ? 127 : q);
    }
    return scale;
}

/* Projection rows stored as float, non-finite dots forced to 0 (:4284-4285). */
static void project(const unsigned char *rows, uint32_t type, uint32_t nrows, uint32_t in_dims, const float *x,
                    float *out, double *tmp) {
    matvec(rows, type, nrows, in_dims, x, tmp);
    for (uint32_t r = 0; r < nrows; ++r) out[r] = isfinite(tmp[r]) ? (float)tmp[r] : 0.0f;
}

QXO_API int qxo_embed(qxo_model *m, uint32_t token, float *out, char *err, uint64_t err_len) {
    const qxh_dir_entry *e = need(m, "token_embd.weight", err, err_len);
    if (!e) return 0;
    uint32_t hidden = m->f.header.manifest.hidden, vocab = m->f.header.manifest.vocab;
    if (token >= vocab) { qxh_set_err(err, err_len, "token id out of range"); return 0; }
    uint32_t bb = 0;
    qxh_block_info(e->flags, NULL, &bb);
    uint64_t row = e->byte_size / vocab;       /* :1659-1668 */
    const unsigned char *p = data(m, e) + (uint64_t)token * row;
    for (uint32_t b = 0; b < hidden / 256u; ++b) qxo_decode_block(e->flags, p + (uint64_t)b * bb, out + 256u * b);
    return 1;
}

/* Final head, :3554-3738 (kernel policy "baseline", F32). */
QXO_API int qxo_final_head(qxo_model *m, const float *residual, float *normalized, float *logits, uint32_t top_n,
                           uint32_t *top_tokens, double *top_logits, char *err, uint64_t err_len) {
    const qxh_dir_entry *nw = need(m, "output_norm.weight", err, err_len), *lm = need(m, "output.weight", err, err_len);
    if (!nw || !lm) return 0;
    uint32_t hidden = m->f.header.manifest.hidden, vocab = m->f.header.manifest.vocab;
    if (lm->flags != QXH_Q6_K) { qxh_set_err(err, err_len, "final head requires Q6_K output.weight"); return 0; }
    if (top_n == 0) top_n = 1;
    if (top_n > 32) top_n = 32;
    rmsnorm(residual, data(m, nw), normalized, hidden);
    double *dots = (double *)malloc((size_t)vocab * sizeof(double));
    if (!dots) { qxh_set_err(err, err_len, "out of memory"); return 0; }
    matvec(data(m, lm), QXH_Q6_K, vocab, hidden, normalized, dots);
    uint32_t tt[32];
    double tl[32];
    for (uint32_t i = 0; i < top_n; ++i) { tt[i] = 0; tl[i] = -1.0e300; }
    for (uint32_t r = 0; r < vocab; ++r) {
        double lg = dots[r];
        if (!isfinite(lg)) { free(dots); qxh_set_err(err, err_len, "non-finite final logit"); return 0; }
        if (logits) logits[r] = (float)lg;
        for (uint32_t k = 0; k < top_n; ++k) {           /* strict > keeps the lowest index on ties */
            if (lg > tl[k]) {
                for (uint32_t s = top_n - 1; s > k; --s) { tt[s] = tt[s - 1]; tl[s] = tl[s - 1]; }
                tt[k] = r; tl[k] = lg;
                break;
            }
        }
    }
    free(dots);
    for (uint32_t i = 0; i < top_n; ++i) {
        if (top_tokens) top_tokens[i] = tt[i];
        if (top_logits) top_logits[i] = tl[i];
    }
    return 1;
}

/* MoE layer, :5198-5317. */
QXO_API int qxo_moe_layer(qxo_model *m, uint32_t layer, const float *x, float *layer_output, float *moe_output,
                          uint32_t selected[8], double weights[8], char *err, uint64_t err_len) {
    const qxh_dir_entry *nw = needl(m, layer, "ffn_norm.weight", err, err_len);
    const qxh_dir_entry *rt = needl(m, layer, "ffn_gate_inp.weight", err, err_len);
    const qxh_dir_entry *gt = needl(m, layer, "ffn_gate_exps.weight", err, err_len);
    const qxh_dir_entry *ut = needl(m, layer, "ffn_up_exps.weight", err, err_len);
    const qxh_dir_entry *dt = needl(m, layer, "ffn_down_exps.weight", err, err_len);
    if (!nw || !rt || !gt || !ut || !dt) return 0;
    uint32_t H = m->f.header.manifest.hidden, E = (uint32_t)rt->dims[1], I = (uint32_t)gt->dims[1];
    if (E < 8 || E > 128) { qxh_set_err(err, err_len, "unsupported real MoE tensor layout"); return 0; }
    float *xin = (float *)calloc((size_t)(3u * H + 3u * I), sizeof(float));
    double *tmp = (double *)malloc((size_t)(H > I ? H : I) * sizeof(double));
    if (!xin || !tmp) { free(xin); free(tmp); qxh_set_err(err, err_len, "out of memory"); return 0; }
    float *moe = xin + H, *y = moe + H, *gv = y + H, *uv = gv + I, *hv = uv + I;
    rmsnorm(x, data(m, nw), xin, H);
    double logit[128], prob[128], mx = -1.0e300;
    matvec(data(m, rt), QXH_F32, E, H, xin, logit);        /* router in double, :5257-5263 */
    for (uint32_t e = 0; e < E; ++e) if (logit[e] > mx) mx = logit[e];
    double den = 0.0;
    for (uint32_t e = 0; e < E; ++e) { prob[e] = exp(logit[e] - mx); den += prob[e]; }
    for (uint32_t e = 0; e < E; ++e) prob[e] /= den;
    unsigned char taken[128] = {0};
    double wsum = 0.0;
    for (uint32_t k = 0; k < 8; ++k) {                     /* repeated strict-> argmax, :5273-5283 */
        uint32_t best = 0;
        double bp = -1.0;
        for (uint32_t e = 0; e < E; ++e) if (!taken[e] && prob[e] > bp) { best = e; bp = prob[e]; }
        taken[best] = 1;
        selected[k] = best;
        weights[k] = bp;
        wsum += bp;
    }
    for (uint32_t k = 0; k < 8; ++k) weights[k] /= wsum;
    uint32_t gbb, ubb, dbb;
    qxh_block_info(gt->flags, NULL, &gbb);
    qxh_block_info(ut->flags, NULL, &ubb);
    qxh_block_info(dt->flags, NULL, &dbb);
    for (uint32_t k = 0; k < 8; ++k) {
        uint32_t e = selected[k];
        uint64_t gsl = (uint64_t)I * (H / 256u) * gbb, usl = (uint64_t)I * (H / 256u) * ubb,
                 dsl = (uint64_t)H * (I / 256u) * dbb;       /* expert slice, :4749-4763 */
        matvec(data(m, gt) + e * gsl, gt->flags, I, H, xin, tmp);
        for (uint32_t i = 0; i < I; ++i) gv[i] = isfinite(tmp[i]) ? (float)tmp[i] : 0.0f;
        matvec(data(m, ut) + e * usl, ut->flags, I, H, xin, tmp);
        for (uint32_t i = 0; i < I; ++i) uv[i] = isfinite(tmp[i]) ? (float)tmp[i] : 0.0f;
        for (uint32_t i = 0; i < I; ++i) {                 /* SwiGLU in double, :5297 / :2511 */
            double g = (double)gv[i];
            hv[i] = (float)(g / (1.0 + exp(-g)) * (double)uv[i]);
        }
        matvec(data(m, dt) + e * dsl, dt->flags, H, I, hv, tmp);
        for (uint32_t i = 0; i < H; ++i) y[i] = isfinite(tmp[i]) ? (float)tmp[i] : 0.0f;
        for (uint32_t i = 0; i < H; ++i) moe[i] += (float)(weights[k] * (double)y[i]);   /* :5303 */
    }
    for (uint32_t i = 0; i < H; ++i) layer_output[i] = x[i] + moe[i];                     /* :5306-5309 */
    if (moe_output) memcpy(moe_output, moe, (size_t)H * sizeof(float));
    free(xin);
    free(tmp);
    return 1;
}

/* Attention half of a layer in state-loop order (:6283-6423) with the GQA
 * core of qx_rope_gqa_attention_partial (:5051-5196). */
QXO_API int qxo_attention_layer(qxo_model *m, uint32_t layer, uint32_t step, uint32_t ctx, int8_t *kcache,
                                int8_t *vcache, float *kscales, float *vscales, float *residual, float *attn_out,
                                float *context, float *k_out, float *v_out, char *err, uint64_t err_len) {
    const qxh_manifest *mf = &m->f.header.manifest;
    uint32_t H = mf->hidden, QH = mf->q_heads, KH = mf->kv_heads, D = mf->head_dim, KV = KH * D, Q = QH * D;
    const qxh_dir_entry *an = needl(m, layer, "attn_norm.weight", err, err_len);
    const qxh_dir_entry *qt = needl(m, layer, "attn_q.weight", err, err_len);
    const qxh_dir_entry *kt = needl(m, layer, "attn_k.weight", err, err_len);
    const qxh_dir_entry *vt = needl(m, layer, "attn_v.weight", err, err_len);
    const qxh_dir_entry *ot = needl(m, layer, "attn_output.weight", err, err_len);
    const qxh_dir_entry *qn = needl(m, layer, "attn_q_norm.weight", err, err_len);
    const qxh_dir_entry *kn = needl(m, layer, "attn_k_norm.weight", err, err_len);
    if (!an || !qt || !kt || !vt || !ot || !qn || !kn) return 0;
    if (step >= ctx) { qxh_set_err(err, err_len, "steps exceed ctx"); return 0; }
    uint32_t T = step + 1u;
    float *xn = (float *)malloc((size_t)(H + 2u * KV + 2u * Q + H) * sizeof(float));
    double *tmp = (double *)malloc((size_t)(Q > H ? Q : H) * sizeof(double));
    double *sc = (double *)malloc((size_t)T * sizeof(double)), *wt = (double *)malloc((size_t)T * sizeof(double));
    if (!xn || !tmp || !sc || !wt) { free(xn); free(tmp); free(sc); free(wt); qxh_set_err(err, err_len, "out of memory"); return 0; }
    float *k = xn + H, *v = k + KV, *q = v + KV, *cx = q + Q, *o = cx + Q;
    rmsnorm(residual, data(m, an), xn, H);
    project(data(m, kt), kt->flags, KV, H, xn, k, tmp);
    project(data(m, vt), vt->flags, KV, H, xn, v, tmp);
    head_rmsnorm(k, data(m, kn), KH, D);
    qxo_rope(k, KH, D, step);
    if (k_out) memcpy(k_out, k, (size_t)KV * sizeof(float));
    if (v_out) memcpy(v_out, v, (size_t)KV * sizeof(float));
    uint64_t slot = (uint64_t)layer * ctx + step;
    kscales[slot] = qxo_quantize_int8(k, kcache + slot * KV, KV);
    vscales[slot] = qxo_quantize_int8(v, vcache + slot * KV, KV);
    project(data(m, qt), qt->flags, Q, H, xn, q, tmp);
    head_rmsnorm(q, data(m, qn), QH, D);
    qxo_rope(q, QH, D, step);
    memset(cx, 0, (size_t)Q * sizeof(float));
    uint32_t group = QH / KH;
    for (uint32_t h = 0; h < QH; ++h) {
        uint32_t kvh = h / group;
        double mx = -1.0e300;
        for (uint32_t t = 0; t < T; ++t) {
            uint64_t st = (uint64_t)layer * ctx + t;
            const int8_t *kp = kcache + st * KV + (uint64_t)kvh * D;
            float ks = kscales[st];
            double s = 0.0;
            for (uint32_t d = 0; d < D; ++d) s += (double)q[h * D + d] * (double)((float)kp[d] * ks);
            s /= sqrt((double)D);
            if (!isfinite(s)) s = 0.0;
            sc[t] = s;
            if (s > mx) mx = s;
        }
        double den = 0.0;
        for (uint32_t t = 0; t < T; ++t) { wt[t] = exp(sc[t] - mx); den += wt[t]; }
        if (!isfinite(den) || den <= 0.0) den = 1.0;
        for (uint32_t t = 0; t < T; ++t) {
            double w = wt[t] / den;
            uint64_t st = (uint64_t)layer * ctx + t;
            const int8_t *vp = vcache + st * KV + (uint64_t)kvh * D;
            float vs = vscales[st];
            for (uint32_t d = 0; d < D; ++d) cx[h * D + d] += (float)(w * (double)((float)vp[d] * vs));
        }
    }
    if (context) memcpy(context, cx, (size_t)Q * sizeof(float));
    project(data(m, ot), ot->flags, H, Q, cx, o, tmp);
    for (uint32_t i = 0; i < H; ++i) residual[i] += o[i];
    if (attn_out) memcpy(attn_out, o, (size_t)H * sizeof(float));
    free(xn); free(tmp); free(sc); free(wt);
    return 1;
}

QXO_API int qxo_decode_step(qxo_model *m, uint32_t token, uint32_t step, uint32_t ctx, int8_t *kcache,
                            int8_t *vcache, float *kscales, float *vscales, uint32_t *experts_out,
                            double *routing_out, float *residual_out, float *logits, uint32_t *next_token,
                            double *top2_logits, char *err, uint64_t err_len) {
    const qxh_manifest *mf = &m->f.header.manifest;
    uint32_t H = mf->hidden;
    float *res = (float *)malloc((size_t)H * sizeof(float)), *nrm = (float *)malloc((size_t)H * sizeof(float));
    if (!res || !nrm) { free(res); free(nrm); qxh_set_err(err, err_len, "out of memory"); return 0; }
    int ok = qxo_embed(m, token, res, err, err_len);
    for (uint32_t l = 0; ok && l < mf->layers; ++l) {
        ok = qxo_attention_layer(m, l, step, ctx, kcache, vcache, kscales, vscales, res, NULL, NULL, NULL, NULL, err,
                                 err_len);
        uint32_t sel[8];
        double w[8];
        if (ok) ok = qxo_moe_layer(m, l, res, res, NULL, sel, w, err, err_len);
        if (ok && experts_out) memcpy(experts_out + 8u * l, sel, sizeof(sel));
        if (ok && routing_out) memcpy(routing_out + 8u * l, w, sizeof(w));
    }
    uint32_t tt[2];
    double tl[2];
    if (ok) ok = qxo_final_head(m, res, nrm, logits, 2, tt, tl, err, err_len);
    if (ok) {
        if (residual_out) memcpy(residual_out, res, (size_t)H * sizeof(float));
        if (next_token) *next_token = tt[0];
        if (top2_logits) { top2_logits[0] = tl[0]; top2_logits[1] = tl[1]; }
    }
    free(res); free(nrm);
    return ok;
}
