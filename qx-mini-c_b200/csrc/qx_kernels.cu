// sm_100a kernels of one greedy decode step.
//
// Matvecs: weight row tiles (16 rows, native GGUF blocks) are streamed into
// shared memory with cp.async, issued before the prologue so the DRAM latency
// overlaps the activation preparation; each warp reduces a 16-row tile over a
// range of blocks with exact integer tensor-core dots (qx_imma.cuh), partial
// sums are combined in a fixed order, so every output is the correctly
// rounded float of a double-accurate dot product, as in the reference's
// double accumulation (src/qx_format.c:4266-4280, :4774-4783, :3683-3711).
// Norms, RoPE, router softmax, SwiGLU and the attention softmax use double,
// and the attention context is accumulated in float in position order, the
// way qx_rope_gqa_attention_partial does it (src/qx_format.c:5127-5172).
#include <cfloat>

#include "qx_common.cuh"

namespace qx {

// ---------------------------------------------------------------------------
// embedding: Q4_K row gather (src/qx_format.c:2089-2110, :3759-3819)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_embed(Dev d) {
    const int tok = *d.token;
    if (tok < 0 || tok >= d.dm.vocab) {
        if (threadIdx.x == 0) atomicOr(d.err, kErrToken);
        return;
    }
    const int nblk = d.dm.hidden / 256;
    const uint8_t* row = d.tok_embd + (size_t)tok * (size_t)(nblk * 144);
    const int t = threadIdx.x;
    const int c = t >> 6, l = t & 63;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 144;
        const float dd = h2f(ld16(blk)), dmin = h2f(ld16(blk + 2));
        const uint8_t* s = blk + 4;
        const int j = 2 * c + (l >= 32);
        uint32_t sc, mn;
        if (j < 4) { sc = s[j] & 63u; mn = s[j + 4] & 63u; }
        else { sc = (s[j + 4] & 15u) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
        const uint8_t qb = blk[16 + 32 * c + (l & 31)];
        const uint32_t q = l < 32 ? (qb & 15u) : (qb >> 4);
        // d*sc*q - dmin*m with each product rounded to float, no contraction
        d.x[b * 256 + t] = __fsub_rn(__fmul_rn(__fmul_rn(dd, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
    }
}

// ---------------------------------------------------------------------------
// Q/K/V projections with the attention RMSNorm in the prologue
// (qx_projection_matvec_fill_mode, src/qx_format.c:4207-4297; :6283-6290).
// 2 tiles per CTA, 4 block-parts per tile.
// ---------------------------------------------------------------------------
// Bytes of one 256-value block of a ggml type on the decode path.
constexpr uint32_t block_bytes(int fmt) {
    return fmt == 17 ? 74u : fmt == 22 ? 82u : fmt == 18 ? 98u : fmt == 21 ? 110u : fmt == 23 ? 136u : fmt == 14 ? 210u
                                                                                                           : 176u;
}

constexpr int kQkvTiles = 2;

__global__ void __launch_bounds__(kThreads) k_qkv(Dev d, LayerW w) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kWarps];
    const int H = d.dm.hidden, Q = d.dm.q_dim(), KV = d.dm.kv_dim();
    const int nblk = H / 256;
    const uint32_t rb = (uint32_t)nblk * 136u, tb = (uint32_t)kTileRows * rb;
    Carve cv(smem);
    uint8_t* tiles = cv.take<uint8_t>(kQkvTiles * tb);
    float* xs = cv.take<float>(H);
    uint32_t* xb = cv.take<uint32_t>(xq_words(H));
    int* sb = cv.take<int>(H / 256);
    double* part = cv.take<double>(kWarps * kTileRows);
    const int ntiles = (Q + 2 * KV) / kTileRows;
    for (int k = 0; k < kQkvTiles; ++k) {
        const int t = blockIdx.x * kQkvTiles + k;
        if (t >= ntiles) break;
        const int r0 = t * kTileRows;
        const uint8_t* src = r0 < Q ? w.wq + (size_t)r0 * rb
                             : r0 < Q + KV ? w.wk + (size_t)(r0 - Q) * rb
                                           : w.wv + (size_t)(r0 - Q - KV) * rb;
        stage_copy(tiles + k * tb, src, tb);
    }
    cp_async_commit();
    uint32_t K4[4];
    load_kv_regs(d.tables, K4);
    rmsnorm_to_smem(d.x, w.attn_norm, xs, H, scratch);
    build_xq(xs, H, xb, sb);
    cp_async_wait<0>();
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int parts = kWarps / kQkvTiles, tile = warp / parts, p = warp % parts;
    const int t = blockIdx.x * kQkvTiles + tile;
    if (t < ntiles) {
        const uint8_t* base = tiles + tile * tb;
        Acc acc{};
        const int g = lane >> 2;
        dot_iq4_xs_mma(base + g * rb, base + (g + 8) * rb, p * nblk / parts, (p + 1) * nblk / parts, XQ{xb, sb}, K4,
                       lane, acc);
        store_tile_rows(part, warp, acc);
    }
    __syncthreads();
    if (threadIdx.x < kQkvTiles * kTileRows) {
        const int tl = threadIdx.x / kTileRows, r = threadIdx.x % kTileRows;
        const int tt = blockIdx.x * kQkvTiles + tl;
        if (tt < ntiles) d.qkv[tt * kTileRows + r] = finite_or_zero_d(sum_parts(part, tl, parts, r));
    }
}

// ---------------------------------------------------------------------------
// Attention for one query head per CTA (128 threads = head dims), exact
// reference order: per-head Q/K RMSNorm (:3740-3757), split-half RoPE
// (:4625-4641), INT8 quantize-and-append of the current K/V (:4449-4463,
// :6343-6400), scores and softmax in double, context accumulated in float over
// positions 0..pos in order (:5127-5172).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) k_attn(Dev d, LayerW w, int layer) {
    const int D = 128, KVH = d.dm.kv_heads, QH = d.dm.q_heads, group = QH / KVH;
    const int Q = d.dm.q_dim(), KV = d.dm.kv_dim(), ctx = d.dm.ctx;
    const int h = blockIdx.x, g = h / group, i = threadIdx.x;
    const int pos = *d.pos;
    if (pos < 0 || pos >= ctx) {
        if (i == 0 && h == 0) atomicOr(d.err, kErrPosition);
        return;
    }
    __shared__ double scratch_d[4];
    __shared__ float scratch_f[4];
    __shared__ float qv[128];
    __shared__ double qd[128];
    __shared__ float kcur[1024];
    __shared__ float vcur[1024];
    __shared__ __align__(16) int8_t k8[1024];
    __shared__ __align__(16) int8_t v8[1024];
    const double* rope = d.rope + (size_t)pos * 128;
    for (int j = i; j < KV; j += 128) {
        kcur[j] = d.qkv[Q + j];
        vcur[j] = d.qkv[Q + KV + j];
    }
    qv[i] = d.qkv[h * D + i];
    __syncthreads();
    for (int hh = i >> 5; hh <= KVH; hh += 4) {
        if (hh < KVH) warp_norm_rope(kcur + hh * D, w.k_norm, rope, i & 31);
        else warp_norm_rope(qv, w.q_norm, rope, i & 31);
    }
    __syncthreads();
    // one INT8 scale over all KV values of the token (K and V separately)
    float ka = 0.f, va = 0.f;
    for (int j = i; j < KV; j += 128) {
        ka = fmaxf(ka, isfinite(kcur[j]) ? fabsf(kcur[j]) : 0.f);
        va = fmaxf(va, isfinite(vcur[j]) ? fabsf(vcur[j]) : 0.f);
    }
    ka = block_max_f(ka, scratch_f);
    va = block_max_f(va, scratch_f);
    const float ksc = ka > 0.f ? ka / 127.0f : 1.0f, vsc = va > 0.f ? va / 127.0f : 1.0f;
    for (int j = i; j < KV; j += 128) {
        const int qk = isfinite(kcur[j]) ? (int)lrintf(kcur[j] / ksc) : 0;
        const int qq = isfinite(vcur[j]) ? (int)lrintf(vcur[j] / vsc) : 0;
        k8[j] = (int8_t)max(-127, min(127, qk));
        v8[j] = (int8_t)max(-127, min(127, qq));
    }
    __syncthreads();
    const size_t slot = (size_t)layer * ctx + pos;
    if (h == 0) {
        for (int j = i; j < KV; j += 128) {
            d.kcache[slot * KV + j] = k8[j];
            d.vcache[slot * KV + j] = v8[j];
        }
        if (i == 0) { d.kscale[slot] = ksc; d.vscale[slot] = vsc; }
    }
    qd[i] = (double)qv[i];
    __syncthreads();
    // scores: thread i takes positions i, i+128, ...; dot over d in order, double
    double* sc = d.attn_scores + (size_t)h * ctx;
    const int T = pos + 1;
    const double sqrt_d = sqrt((double)D);
    double mloc = -1.0e300;
    for (int t = i; t < T; t += 128) {
        const size_t st = (size_t)layer * ctx + t;
        const int8_t* kp = t == pos ? k8 + g * D : d.kcache + st * KV + g * D;
        const float ks = t == pos ? ksc : d.kscale[st];
        const double s = score_row(qd, kp, ks, sqrt_d);
        sc[t] = s;
        mloc = fmax(mloc, s);
    }
    const double mx = block_max_d(mloc, scratch_d);
    for (int t = i; t < T; t += 128) sc[t] = exp(sc[t] - mx);
    double den = fixed_order_sum(sc, T, scratch_d);
    if (!isfinite(den) || den <= 0.0) den = 1.0;
    for (int t = i; t < T; t += 128) sc[t] = sc[t] / den;
    __syncthreads();
    // context[d] += (float)(w_t * (double)vval_t) for t = 0..pos in order
    float acc = 0.0f;
    const int8_t* vbase = d.vcache + (size_t)layer * ctx * KV + g * D + i;
    const float* vsb = d.vscale + (size_t)layer * ctx;
    for (int t = 0; t < T; ++t) {
        const float vv = t == pos ? i8_to_f32(v8[g * D + i]) * vsc : i8_to_f32(vbase[(size_t)t * KV]) * vsb[t];
        acc += (float)(sc[t] * (double)vv);
    }
    d.ctxv[h * D + i] = acc;
}

// ---------------------------------------------------------------------------
// O projection + residual add (:5183, :6420-6423).  One tile per CTA, 8 parts.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_oproj(Dev d, LayerW w) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int Q = d.dm.q_dim();
    const int nblk = Q / 256;
    const uint32_t rb = (uint32_t)nblk * 136u, tb = (uint32_t)kTileRows * rb;
    Carve cv(smem);
    uint8_t* tile = cv.take<uint8_t>(tb);
    float* xs = cv.take<float>(Q);
    uint32_t* xb = cv.take<uint32_t>(xq_words(Q));
    int* sb = cv.take<int>(Q / 256);
    double* part = cv.take<double>(kWarps * kTileRows);
    stage_copy(tile, w.wo + (size_t)blockIdx.x * tb, tb);
    cp_async_commit();
    uint32_t K4[4];
    load_kv_regs(d.tables, K4);
    copy_to_smem(d.ctxv, xs, Q);
    build_xq(xs, Q, xb, sb);
    cp_async_wait<0>();
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
    Acc acc{};
    dot_iq4_xs_mma(tile + g * rb, tile + (g + 8) * rb, warp * nblk / kWarps, (warp + 1) * nblk / kWarps, XQ{xb, sb},
                   K4, lane, acc);
    store_tile_rows(part, warp, acc);
    __syncthreads();
    if (threadIdx.x < kTileRows) {
        const int r = blockIdx.x * kTileRows + threadIdx.x;
        const float o = finite_or_zero_d(sum_parts(part, 0, kWarps, threadIdx.x));
        d.attn_out[r] = o;
        d.x[r] = d.x[r] + o;
    }
}

// ---------------------------------------------------------------------------
// Projections of other quant types (per-stage path for mixes other than the
// benchmark one).  k_proj: IQ4_XS (23) or Q6_K (14) rows of W [rows][K], two
// 16-row tiles per CTA, exact integer tensor-core dots; input `in` is RMS-
// normed with norm_w when given; residual != 0: the O projection epilogue
// (attn_out = o, x += o), else out[row] = o.  k_proj_q5k: Q5_K rows, one warp
// per row, weights decoded to the reference's floats, double FMA.
// ---------------------------------------------------------------------------
template <int FMT>
__global__ void __launch_bounds__(kThreads) k_proj(Dev d, const float* in, const float* norm_w, const uint8_t* W,
                                                   int rows, int K, float* out, int residual) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kWarps];
    const int nblk = K / 256;
    const uint32_t rb = (uint32_t)nblk * block_bytes(FMT), tb = (uint32_t)kTileRows * rb;
    Carve cv(smem);
    uint8_t* tiles = cv.take<uint8_t>(2 * tb);
    float* xs = cv.take<float>(K);
    uint32_t* xb = cv.take<uint32_t>(xq_words(K));
    int* sb = cv.take<int>(K / 256);
    double* part = cv.take<double>(kWarps * kTileRows);
    const int ntiles = rows / kTileRows;
    for (int k = 0; k < 2; ++k) {
        const int t = blockIdx.x * 2 + k;
        if (t < ntiles) stage_copy(tiles + k * tb, W + (size_t)t * tb, tb);
    }
    cp_async_commit();
    uint32_t K4[4];
    if (FMT == 23) load_kv_regs(d.tables, K4);
    if (norm_w) rmsnorm_to_smem(in, norm_w, xs, K, scratch);
    else copy_to_smem(in, xs, K);
    build_xq(xs, K, xb, sb);
    cp_async_wait<0>();
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
    const int parts = kWarps / 2, tile = warp / parts, p = warp % parts, t = blockIdx.x * 2 + tile;
    if (t < ntiles) {
        const uint8_t* base = tiles + tile * tb;
        Acc acc{};
        if (FMT == 23)
            dot_iq4_xs_mma(base + g * rb, base + (g + 8) * rb, p * nblk / parts, (p + 1) * nblk / parts, XQ{xb, sb}, K4,
                           lane, acc);
        else
            dot_q6_k_mma(base + g * rb, base + (g + 8) * rb, p * nblk / parts, (p + 1) * nblk / parts, XQ{xb, sb}, lane,
                         acc);
        store_tile_rows(part, warp, acc);
    }
    __syncthreads();
    if (threadIdx.x < 2 * kTileRows) {
        const int tl = threadIdx.x / kTileRows, r = threadIdx.x % kTileRows, tt = blockIdx.x * 2 + tl;
        if (tt < ntiles) {
            const int row = tt * kTileRows + r;
            const float o = finite_or_zero_d(sum_parts(part, tl, parts, r));
            if (residual) {
                d.attn_out[row] = o;
                d.x[row] = d.x[row] + o;
            } else {
                out[row] = o;
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads) k_proj_q5k(Dev d, const float* in, const float* norm_w, const uint8_t* W,
                                                       int rows, int K, float* out, int residual) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kWarps];
    float* xs = reinterpret_cast<float*>(smem);
    if (norm_w) rmsnorm_to_smem(in, norm_w, xs, K, scratch);
    else copy_to_smem(in, xs, K);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, row = blockIdx.x * kWarps + warp;
    if (row >= rows) return;
    const double v = dot_q5_k_row(W + (size_t)row * (K / 256) * 176, K / 256, xs, lane);
    if (lane == 0) {
        const float o = finite_or_zero_d(v);
        if (residual) {
            d.attn_out[row] = o;
            d.x[row] = d.x[row] + o;
        } else {
            out[row] = o;
        }
    }
}

// ---------------------------------------------------------------------------
// Router: FFN RMSNorm + F32 router matvec in double, softmax, top-8 by
// repeated strict-> argmax (lowest index on ties), renormalisation
// (qx_apply_real_moe_layer, src/qx_format.c:5250-5285).
// ---------------------------------------------------------------------------
constexpr int kRouterRowsPerCta = 8;

__global__ void __launch_bounds__(kThreads) k_router(Dev d, LayerW w, int layer) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kWarps];
    __shared__ double probs[256];
    __shared__ double wsel[8];
    __shared__ int isel[8];
    const int H = d.dm.hidden, E = d.dm.experts;
    float* xs = reinterpret_cast<float*>(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * kRouterRowsPerCta + warp;
    const float* row = w.router + (size_t)(e < E ? e : 0) * H;
    // prefetch this warp's router row into registers while the norm runs
    float4 wv[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int i = (k * 32 + lane) * 4;
        wv[k] = i < H ? *reinterpret_cast<const float4*>(row + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    rmsnorm_to_smem(d.x, w.ffn_norm, xs, H, scratch);
    if (blockIdx.x == 0)
        for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4)
            *reinterpret_cast<float4*>(d.xn + i) = *reinterpret_cast<const float4*>(xs + i);
    if (e < E) {
        double acc = 0.0;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int i = (k * 32 + lane) * 4;
            if (i < H) {
                acc += (double)wv[k].x * (double)xs[i] + (double)wv[k].y * (double)xs[i + 1];
                acc += (double)wv[k].z * (double)xs[i + 2] + (double)wv[k].w * (double)xs[i + 3];
            }
        }
        for (int i = (16 * 32 + lane) * 4; i < H; i += 128) {
            const float4 v = *reinterpret_cast<const float4*>(row + i);
            acc += (double)v.x * (double)xs[i] + (double)v.y * (double)xs[i + 1];
            acc += (double)v.z * (double)xs[i + 2] + (double)v.w * (double)xs[i + 3];
        }
        acc = warp_sum_d(acc);
        if (lane == 0) d.router_logits[e] = acc;
    }
    if (!last_cta(d.counters + kCntRouter, gridDim.x)) return;
    const int t = threadIdx.x;
    const double lg = t < E ? d.router_logits[t] : -1.0e300;
    double m = lg;
    for (int o = 16; o; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncthreads();
    if (lane == 0) scratch[warp] = m;
    __syncthreads();
    m = scratch[0];
    for (int i = 1; i < kWarps; ++i) m = fmax(m, scratch[i]);
    const double ex = t < E ? exp(lg - m) : 0.0;
    const double den = block_sum_d(ex, scratch);
    if (t < 256) probs[t] = t < E ? ex / den : -1.0;
    __syncthreads();
    if (warp == 0) {
        for (int k = 0; k < 8; ++k) {
            double bv = -2.0;
            int bi = 0x7fffffff;
            for (int i = lane; i < E; i += 32) {
                const double p = probs[i];
                if (p > bv || (p == bv && i < bi)) { bv = p; bi = i; }
            }
            for (int o = 16; o; o >>= 1) {
                const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (lane == 0) { isel[k] = bi; wsel[k] = bv; probs[bi] = -1.0; }
            __syncwarp();
        }
        if (lane == 0) {
            double sum = 0.0;
            for (int k = 0; k < 8; ++k) sum += wsel[k];
            if (!(sum > 0.0) || !isfinite(sum)) atomicOr(d.err, kErrRouter);
            for (int k = 0; k < 8; ++k) {
                const double wk = wsel[k] / sum;
                d.sel[layer * 8 + k] = isel[k];
                d.selw[layer * 8 + k] = (float)wk;
                d.selw_d[k] = wk;
            }
            d.counters[kCntRouter] = 0u;
        }
    }
}

// ---------------------------------------------------------------------------
// Fused gate/up IQ2_XS matvecs of the 8 selected experts with SwiGLU
// (qx_packed_expert_matvec_mode :4739-4787, :5291-5297, qx_silu :2511).
// CTA = (expert rank, 16-row tile): tile 0 = gate rows, tile 1 = up rows;
// 4 block-parts each.
// ---------------------------------------------------------------------------
template <int FMT>   // IQ2_XS (17) or IQ2_S (22)
__global__ void __launch_bounds__(kThreads) k_gateup(Dev d, LayerW w, int layer) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int H = d.dm.hidden, I = d.dm.moe_inter;
    const int nblk = H / 256;
    const uint32_t rb = (uint32_t)nblk * block_bytes(FMT), tb = (uint32_t)kTileRows * rb;
    Carve cv(smem);
    uint8_t* tiles = cv.take<uint8_t>(2 * tb);
    IqTab* T = cv.take<IqTab>(1);
    float* xs = cv.take<float>(H);
    uint32_t* xb = cv.take<uint32_t>(xq_words(H));
    int* sb = cv.take<int>(H / 256);
    double* part = cv.take<double>(kWarps * kTileRows);
    const int tiles_per_expert = I / kTileRows;
    const int k = blockIdx.x / tiles_per_expert, i0 = (blockIdx.x % tiles_per_expert) * kTileRows;
    const size_t off = (size_t)d.sel[layer * 8 + k] * ((size_t)I * rb) + (size_t)i0 * rb;
    stage_copy(tiles, w.gate + off, tb);
    stage_copy(tiles + tb, w.up + off, tb);
    cp_async_commit();
    if (FMT == 17) load_iq_tables(T, d.tables, true, false);
    copy_to_smem(d.xn, xs, H);
    build_xq(xs, H, xb, sb);
    cp_async_wait<0>();
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
    const int parts = kWarps / 2, tile = warp / parts, p = warp % parts;
    const uint8_t* base = tiles + tile * tb;
    Acc acc{};
    if (FMT == 17)
        dot_iq2_xs_mma(base + g * rb, base + (g + 8) * rb, p * nblk / parts, (p + 1) * nblk / parts, XQ{xb, sb}, *T,
                       lane, acc);
    else
        dot_iq2_s_mma(base + g * rb, base + (g + 8) * rb, p * nblk / parts, (p + 1) * nblk / parts, XQ{xb, sb},
                      d.tables->iq2s, lane, acc);
    store_tile_rows(part, warp, acc);
    __syncthreads();
    if (threadIdx.x < kTileRows) {
        const float gv = finite_or_zero_d(sum_parts(part, 0, parts, threadIdx.x));
        const float uv = finite_or_zero_d(sum_parts(part, 1, parts, threadIdx.x));
        const double gd = (double)gv;
        d.hbuf[k * I + i0 + threadIdx.x] = (float)(gd / (1.0 + exp(-gd)) * (double)uv);
    }
}

// ---------------------------------------------------------------------------
// IQ3_XXS down projections of the 8 experts with the rank-ordered weighted sum
// and the residual add fused (:5298-5309).  CTA = rows [16c, 16c+16) of all 8
// experts; warp k computes expert k on its own input h[k].
// ---------------------------------------------------------------------------
template <int FMT>   // IQ3_XXS (18), IQ3_S (21) or IQ4_XS (23)
__global__ void __launch_bounds__(kThreads) k_down(Dev d, LayerW w, int layer) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int H = d.dm.hidden, I = d.dm.moe_inter;
    const int nblk = I / 256;
    const uint32_t rb = (uint32_t)nblk * block_bytes(FMT), tb = (uint32_t)kTileRows * rb;
    Carve cv(smem);
    uint8_t* tiles = cv.take<uint8_t>(8 * tb);
    IqTab* T = cv.take<IqTab>(1);
    float* hs = cv.take<float>(8 * I);
    uint32_t* xb = cv.take<uint32_t>(xq_words(8 * I));
    int* sb = cv.take<int>(8 * (I / 256));
    double* part = cv.take<double>(kWarps * kTileRows);
    const size_t slice = (size_t)H * rb;
    for (int k = 0; k < 8; ++k)
        stage_copy(tiles + k * tb, w.down + (size_t)d.sel[layer * 8 + k] * slice + (size_t)blockIdx.x * tb, tb);
    cp_async_commit();
    uint32_t K4[4];
    if (FMT == 18) load_iq_tables(T, d.tables, false, true);
    if (FMT == 23) load_kv_regs(d.tables, K4);
    copy_to_smem(d.hbuf, hs, 8 * I);
    build_xq(hs, 8 * I, xb, sb);   // expert k's groups start at k * I / 16 (I % 256 == 0)
    cp_async_wait<0>();
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
    const uint8_t* base = tiles + warp * tb;
    Acc acc{};
    const XQ xw{xb + warp * xq_words(I), sb + warp * (I / 256)};
    if (FMT == 18) dot_iq3_xxs_mma(base + g * rb, base + (g + 8) * rb, 0, nblk, xw, *T, lane, acc);
    if (FMT == 21) dot_iq3_s_mma(base + g * rb, base + (g + 8) * rb, 0, nblk, xw, d.tables->iq3s, lane, acc);
    if (FMT == 23) dot_iq4_xs_mma(base + g * rb, base + (g + 8) * rb, 0, nblk, xw, K4, lane, acc);
    store_tile_rows(part, warp, acc);
    __syncthreads();
    if (threadIdx.x < kTileRows) {
        const int r = blockIdx.x * kTileRows + threadIdx.x;
        float moe = 0.0f;
        for (int k = 0; k < 8; ++k)
            moe += (float)(d.selw_d[k] * (double)finite_or_zero_d(part[k * kTileRows + threadIdx.x]));
        d.moe_out[r] = moe;
        d.x[r] = d.x[r] + moe;
    }
}

// ---------------------------------------------------------------------------
// Final RMSNorm + Q6_K head + argmax (qx_compute_real_final_head,
// src/qx_format.c:3554-3738; greedy pick :3045-3057).  Persistent grid over
// groups of 2 tiles; logits compared as doubles (ties to the lower index, as
// the strict > scan does); the last CTA records the token and advances
// (token, pos) for the next step.
// ---------------------------------------------------------------------------
constexpr int kHeadStages = 3;
constexpr int kHeadTiles = 2;
// With the re-laid head (R8, the persistent step's copy: int8 weights, no
// decoding) a group is one 16-row tile, one block per warp, so the block
// partials add in block order as the persistent step's head adds them.
constexpr int kHeadStagesR8 = 2;   // small enough for two CTAs (16 warps) per SM

__host__ __device__ constexpr uint32_t head_row_bytes(bool r8, int H) {
    return r8 ? (uint32_t)r8_row_bytes(H) : (uint32_t)(H / 256) * 210u;
}

template <bool R8>
__global__ void __launch_bounds__(kThreads) k_head(Dev d) {
    constexpr int TILES = R8 ? 1 : kHeadTiles, STAGES = R8 ? kHeadStagesR8 : kHeadStages;
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kWarps];
    __shared__ double wbv[kWarps];
    __shared__ int wbi[kWarps];
    const int H = d.dm.hidden, V = d.dm.vocab;
    const int nblk = H / 256;
    const uint32_t rb = head_row_bytes(R8, H), tb = (uint32_t)kTileRows * rb, stage = TILES * tb;
    const uint8_t* src = R8 ? d.head_r : d.head;
    Carve cv(smem);
    uint8_t* ring = cv.take<uint8_t>(STAGES * stage);
    float* xs = cv.take<float>(H);
    uint32_t* xb = cv.take<uint32_t>(xq_words(H));
    int* sb = cv.take<int>(H / 256);
    double* part = cv.take<double>(kWarps * kTileRows);
    const int ngroups = V / (kTileRows * TILES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
    const int parts = kWarps / TILES, tile = warp / parts, p = warp % parts;
    // the first stages are issued before the norm + x quantization run
    const int first = blockIdx.x, step = gridDim.x;
    const int mine = first < ngroups ? (ngroups - first + step - 1) / step : 0;
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < mine) stage_copy(ring + (uint32_t)s * stage, src + (size_t)(first + s * step) * stage, stage);
        cp_async_commit();
    }
    rmsnorm_to_smem(d.x, d.out_norm, xs, H, scratch);
    build_xq(xs, H, xb, sb);
    __syncthreads();
    double bv = -1.0e300;
    int bi = 0x7fffffff;
    bool bad = false;
    for (int it = 0; it < mine; ++it) {
        const int nx = it + STAGES - 1;
        if (nx < mine) stage_copy(ring + (uint32_t)(nx % STAGES) * stage, src + (size_t)(first + nx * step) * stage, stage);
        cp_async_commit();
        cp_async_wait<STAGES - 1>();
        __syncthreads();
        const uint8_t* base = ring + (uint32_t)(it % STAGES) * stage + tile * tb;
        Acc acc{};
        if (R8)
            dot_r8_mma(base + g * rb, base + (g + 8) * rb, nblk, p * nblk / parts, (p + 1) * nblk / parts, XQ{xb, sb},
                       lane, acc);
        else
            dot_q6_k_mma(base + g * rb, base + (g + 8) * rb, p * nblk / parts, (p + 1) * nblk / parts, XQ{xb, sb},
                         lane, acc);
        store_tile_rows(part, warp, acc);
        __syncthreads();
        if (threadIdx.x < TILES * kTileRows) {
            const int tl = threadIdx.x / kTileRows, r = threadIdx.x % kTileRows;
            const int row = (first + it * step) * TILES * kTileRows + tl * kTileRows + r;
            const double v = sum_parts(part, tl, parts, r);
            if (!isfinite(v)) bad = true;
            d.logits[row] = (float)v;
            if (d.logits_d) d.logits_d[row] = v;
            if (v > bv || (v == bv && row < bi)) { bv = v; bi = row; }
        }
    }
    if (bad) atomicOr(d.err, kErrNonFinite);
    for (int o = 16; o; o >>= 1) {
        const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { wbv[warp] = bv; wbi[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < kWarps; ++i)
            if (wbv[i] > bv || (wbv[i] == bv && wbi[i] < bi)) { bv = wbv[i]; bi = wbi[i]; }
        d.best_val[blockIdx.x] = bv;
        d.best_idx[blockIdx.x] = bi;
    }
    if (!last_cta(d.counters + kCntHead, gridDim.x)) return;
    if (threadIdx.x == 0) {
        double v = d.best_val[0];
        int i = d.best_idx[0];
        for (int c = 1; c < (int)gridDim.x; ++c) {
            const double cv2 = d.best_val[c];
            const int ci = d.best_idx[c];
            if (cv2 > v || (cv2 == v && ci < i)) { v = cv2; i = ci; }
        }
        const int pos = *d.pos;
        if (pos >= 0 && pos < d.dm.ctx) d.tokens_out[pos] = i;
        *d.token = i;
        *d.pos = pos + 1;
        d.counters[kCntHead] = 0u;
    }
}

// Final RMSNorm alone (stage API output `normalized`).
__global__ void __launch_bounds__(256) k_final_norm(Dev d, float* out) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kWarps];
    float* xs = reinterpret_cast<float*>(smem);
    rmsnorm_to_smem(d.x, d.out_norm, xs, d.dm.hidden, scratch);
    for (int i = threadIdx.x; i < d.dm.hidden; i += blockDim.x) out[i] = xs[i];
}

// Top-N of the head's double logits in the order qx_compute_real_final_head
// keeps its list (:3715-3731): descending logit, the lower token first among
// equal logits.  Stage 1: each of kTopnParts CTAs takes a contiguous slice and
// picks its own top-N by N rounds of a block argmax; stage 2: one CTA picks
// the top-N of those candidates the same way.
__device__ void block_argmax(double v, int i, double* sv, int* si, double& bv, int& bi) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o; o >>= 1) {
        const double ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
    }
    __syncthreads();
    if (lane == 0) { sv[warp] = v; si[warp] = i; }
    __syncthreads();
    bv = sv[0];
    bi = si[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
}

// Each thread holds up to 8 candidates (values, indices); picks N in order.
template <int PER>
__device__ void select_top(const double* vals, const int* idxs, int count, int top_n, double* out_v, int* out_i) {
    __shared__ double sv[32];
    __shared__ int si[32];
    double v[PER];
    int ix[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int j = threadIdx.x + k * (int)blockDim.x;
        v[k] = j < count ? vals[j] : -1.0e300;
        ix[k] = j < count ? (idxs ? idxs[j] : j) : 0x7fffffff;
    }
    for (int r = 0; r < top_n; ++r) {
        double bv = -1.0e300;
        int bi = 0x7fffffff;
#pragma unroll
        for (int k = 0; k < PER; ++k)
            if (v[k] > bv || (v[k] == bv && ix[k] < bi)) { bv = v[k]; bi = ix[k]; }
        double gv;
        int gi;
        block_argmax(bv, bi, sv, si, gv, gi);
#pragma unroll
        for (int k = 0; k < PER; ++k)
            if (ix[k] == gi) { v[k] = -1.0e300; ix[k] = 0x7fffffff; }   // indices are unique
        if (threadIdx.x == 0) { out_v[r] = gv; out_i[r] = gi; }
    }
}

__global__ void __launch_bounds__(256) k_topn_part(Dev d, int top_n, double* cand_v, int* cand_i) {
    const int V = d.dm.vocab, b = blockIdx.x;
    const int r0 = (int)((long long)b * V / gridDim.x), r1 = (int)((long long)(b + 1) * V / gridDim.x);
    __shared__ int ids[2048];
    for (int j = threadIdx.x; j < r1 - r0 && j < 2048; j += blockDim.x) ids[j] = r0 + j;
    __syncthreads();
    select_top<8>(d.logits_d + r0, ids, r1 - r0, top_n, cand_v + (size_t)b * top_n, cand_i + (size_t)b * top_n);
}

__global__ void __launch_bounds__(1024) k_topn_merge(int parts, int top_n, const double* cand_v, const int* cand_i,
                                                     int* out_idx, float* out_val) {
    __shared__ double rv[32];
    __shared__ int ri[32];
    select_top<5>(cand_v, cand_i, parts * top_n, top_n, rv, ri);   // parts * top_n candidates, compact
    __syncthreads();
    if (threadIdx.x < top_n) {
        out_idx[threadIdx.x] = ri[threadIdx.x];
        out_val[threadIdx.x] = (float)rv[threadIdx.x];
    }
}

// ---------------------------------------------------------------------------
// launch configuration
// ---------------------------------------------------------------------------
namespace {
size_t a16(size_t v) { return (v + 15) / 16 * 16; }
size_t xq_bytes(int K) { return a16((size_t)K * 4) + a16(xq_words(K) * 4) + a16((size_t)K / 256 * 4); }
size_t part_bytes() { return a16((size_t)kWarps * kTileRows * 8); }
size_t smem_qkv(const Dims& m) { return 16 + a16((size_t)kQkvTiles * kTileRows * (m.hidden / 256) * 136) + xq_bytes(m.hidden) + part_bytes(); }
size_t smem_oproj(const Dims& m) { return 16 + a16((size_t)kTileRows * (m.q_dim() / 256) * 136) + xq_bytes(m.q_dim()) + part_bytes(); }
size_t smem_router(const Dims& m) { return (size_t)m.hidden * 4; }
size_t smem_gateup(const Dims& m, uint32_t bb = 74) {
    return 16 + a16(2 * (size_t)kTileRows * (m.hidden / 256) * bb) + a16(sizeof(IqTab)) + xq_bytes(m.hidden) + part_bytes();
}
size_t smem_proj(int K, uint32_t bb) { return 16 + a16(2 * (size_t)kTileRows * (K / 256) * bb) + xq_bytes(K) + part_bytes(); }
size_t smem_down(const Dims& m, uint32_t bb = 136) {
    return 16 + a16(8 * (size_t)kTileRows * (m.moe_inter / 256) * bb) + a16(sizeof(IqTab)) + a16((size_t)8 * m.moe_inter * 4) +
           a16(xq_words(8 * m.moe_inter) * 4) + a16((size_t)8 * m.moe_inter / 256 * 4) + part_bytes();
}
size_t smem_head(const Dims& m, bool r8 = false) {
    const size_t ring = r8 ? (size_t)kHeadStagesR8 * kTileRows * head_row_bytes(true, m.hidden)
                           : (size_t)kHeadStages * kHeadTiles * kTileRows * head_row_bytes(false, m.hidden);
    return 16 + a16(ring) + xq_bytes(m.hidden) + part_bytes();
}
}  // namespace

cudaError_t configure_kernels() {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    auto set = [&](const void* f) {
        cudaFuncAttributes a{};
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, f);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)a.sharedSizeBytes);
    };
    if (e == cudaSuccess) e = attn2_configure();
    if (e == cudaSuccess) e = q8_configure();
    set((const void*)k_qkv);
    set((const void*)k_oproj);
    set((const void*)k_router);
    set((const void*)k_gateup<17>);
    set((const void*)k_gateup<22>);
    set((const void*)k_down<18>);
    set((const void*)k_down<21>);
    set((const void*)k_down<23>);
    set((const void*)k_proj<23>);
    set((const void*)k_proj<14>);
    set((const void*)k_proj_q5k);
    set((const void*)k_head<false>);
    set((const void*)k_head<true>);
    set((const void*)k_final_norm);
    return e;
}

int head_grid_size(int device, const Dims& m, bool r8) {
    int sms = 0, per = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (r8) cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_head<true>, kThreads, smem_head(m, true));
    else cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_head<false>, kThreads, smem_head(m));
    if (per < 1) per = 1;
    const int groups = m.vocab / (kTileRows * (r8 ? 1 : kHeadTiles));
    const int grid = sms * per;
    return grid < groups ? grid : groups;
}

size_t attn_scores_bytes(const Dims& m) { return (size_t)m.q_heads * m.ctx * sizeof(double); }

bool geometry_supported(const Dims& m) {
    return m.hidden % 256 == 0 && m.q_dim() % 256 == 0 && m.kv_dim() <= 1024 && m.head_dim == 128 &&
           (m.q_dim() + 2 * m.kv_dim()) % (kQkvTiles * kTileRows) == 0 && m.moe_inter % 256 == 0 &&
           m.vocab % (kTileRows * kHeadTiles) == 0 && smem_down(m) <= 227 * 1024 && smem_oproj(m) <= 227 * 1024;
}

void launch_embed(const Dev& d, cudaStream_t st) { k_embed<<<1, 256, 0, st>>>(d); }

bool benchmark_mix(const LayerW* layers, int n) {
    for (int l = 0; l < n; ++l) {
        const LayerW& w = layers[l];
        if (w.tq != 23 || w.tk != 23 || w.tv != 23 || w.to != 23 || w.tgate != 17 || w.tup != 17 || w.tdown != 18)
            return false;
    }
    return true;
}

// One projection of any accepted attention type (rows of W, K inputs).
static void launch_proj(const Dev& d, int type, const float* in, const float* norm_w, const uint8_t* W, int rows, int K,
                        float* out, int residual, cudaStream_t st) {
    const int grid2 = (rows / kTileRows + 1) / 2;
    if (type == 23) k_proj<23><<<grid2, kThreads, smem_proj(K, 136), st>>>(d, in, norm_w, W, rows, K, out, residual);
    else if (type == 14) k_proj<14><<<grid2, kThreads, smem_proj(K, 210), st>>>(d, in, norm_w, W, rows, K, out, residual);
    else k_proj_q5k<<<(rows + kWarps - 1) / kWarps, kThreads, (size_t)K * 4, st>>>(d, in, norm_w, W, rows, K, out, residual);
}

int qkv_launches(const Dev& d, const LayerW& w) { return !d.q8 && w.tq == 23 && w.tk == 23 && w.tv == 23 ? 1 : 3; }

void launch_qkv(const Dev& d, const LayerW& w, cudaStream_t st) {
    if (d.q8) {
        const int H = d.dm.hidden, Q = d.dm.q_dim(), KV = d.dm.kv_dim();
        launch_q8_proj(d, w.tq, d.x, w.attn_norm, w.wq, Q, H, d.qkv, 0, st);
        launch_q8_proj(d, w.tk, d.x, w.attn_norm, w.wk, KV, H, d.qkv + Q, 0, st);
        launch_q8_proj(d, w.tv, d.x, w.attn_norm, w.wv, KV, H, d.qkv + Q + KV, 0, st);
        return;
    }
    if (qkv_launches(d, w) == 3) {              // another mix: one launch per tensor
        const int H = d.dm.hidden, Q = d.dm.q_dim(), KV = d.dm.kv_dim();
        launch_proj(d, w.tq, d.x, w.attn_norm, w.wq, Q, H, d.qkv, 0, st);
        launch_proj(d, w.tk, d.x, w.attn_norm, w.wk, KV, H, d.qkv + Q, 0, st);
        launch_proj(d, w.tv, d.x, w.attn_norm, w.wv, KV, H, d.qkv + Q + KV, 0, st);
        return;
    }
    const int nt = (d.dm.q_dim() + 2 * d.dm.kv_dim()) / kTileRows;
    k_qkv<<<(nt + kQkvTiles - 1) / kQkvTiles, kThreads, smem_qkv(d.dm), st>>>(d, w);
}

// The two-phase all-SM attention when it fits (attn2_supported), else one CTA
// per query head (any context length).
int attn_launches(const Dims& m) { return attn2_supported(m) ? 2 : 1; }

void launch_attn(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    if (attn2_supported(d.dm)) launch_attn2(d, w, layer, sms, st);
    else k_attn<<<d.dm.q_heads, 128, 0, st>>>(d, w, layer);
}

void launch_oproj(const Dev& d, const LayerW& w, cudaStream_t st) {
    if (d.q8) {
        launch_q8_proj(d, w.to, d.ctxv, nullptr, w.wo, d.dm.hidden, d.dm.q_dim(), nullptr, 1, st);
        return;
    }
    if (w.to != 23) {
        launch_proj(d, w.to, d.ctxv, nullptr, w.wo, d.dm.hidden, d.dm.q_dim(), nullptr, 1, st);
        return;
    }
    k_oproj<<<d.dm.hidden / kTileRows, kThreads, smem_oproj(d.dm), st>>>(d, w);
}

void launch_router(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    const int grid = (d.dm.experts + kRouterRowsPerCta - 1) / kRouterRowsPerCta;
    k_router<<<grid, kThreads, smem_router(d.dm), st>>>(d, w, layer);
}

void launch_gateup(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    if (d.q8) { launch_q8_gateup(d, w, layer, st); return; }
    const int grid = 8 * d.dm.moe_inter / kTileRows;
    if (w.tgate == 22) k_gateup<22><<<grid, kThreads, smem_gateup(d.dm, 82), st>>>(d, w, layer);
    else k_gateup<17><<<grid, kThreads, smem_gateup(d.dm, 74), st>>>(d, w, layer);
}

void launch_down(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    if (d.q8) { launch_q8_down(d, w, layer, st); return; }
    const int grid = d.dm.hidden / kTileRows;
    if (w.tdown == 21) k_down<21><<<grid, kThreads, smem_down(d.dm, 110), st>>>(d, w, layer);
    else if (w.tdown == 23) k_down<23><<<grid, kThreads, smem_down(d.dm, 136), st>>>(d, w, layer);
    else k_down<18><<<grid, kThreads, smem_down(d.dm, 98), st>>>(d, w, layer);
}

void launch_head(const Dev& d, cudaStream_t st) {
    if (d.q8) launch_q8_head(d, st);
    else if (d.head_r) k_head<true><<<d.head_grid_r8, kThreads, smem_head(d.dm, true), st>>>(d);
    else k_head<false><<<d.head_grid, kThreads, smem_head(d.dm), st>>>(d);
}

void launch_final_norm(const Dev& d, float* normalized, cudaStream_t st) {
    k_final_norm<<<1, 256, (size_t)d.dm.hidden * 4, st>>>(d, normalized);
}

void launch_topn(const Dev& d, int top_n, double* cand_v, int* cand_i, int* out_idx, float* out_val, cudaStream_t st) {
    k_topn_part<<<kTopnParts, 256, 0, st>>>(d, top_n, cand_v, cand_i);
    k_topn_merge<<<1, 1024, 0, st>>>(kTopnParts, top_n, cand_v, cand_i, out_idx, out_val);
}

}  // namespace qx
