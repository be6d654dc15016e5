// sm_100a kernels of one greedy decode step.  Every weight matrix is read in
// its native GGUF block layout: row tiles are streamed into shared memory with
// cp.async and decoded there by one warp per row.  Accumulation is F32 for the
// quantized matvecs; norms, the router, the softmax weights and SwiGLU use
// double where the reference does (src/qx_format.c cited per kernel).
#include <cfloat>

#include "qx_kernels.h"

namespace qx {

// ---------------------------------------------------------------------------
// shared helpers
// ---------------------------------------------------------------------------

// xs[i] = (float)((double)x[i] / rms) * w[i], rms = sqrt(sum x^2 / n + 1e-6)
// computed in double (qx_apply_f32_rmsnorm, src/qx_format.c:3358-3371).
__device__ void rmsnorm_to_smem(const float* x, const float* w, float* xs, int n, double* scratch) {
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        xs[i] = v;
        ss += (double)v * (double)v;
    }
    ss = block_sum_d(ss, scratch);
    const double rms = sqrt(ss / (double)n + 1.0e-6);
    for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = (float)((double)xs[i] / rms) * w[i];
    __syncthreads();
}

__device__ void copy_to_smem(const float* x, float* xs, int n) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
}

// CTA copy of a table (bytes a multiple of 4, both 4-byte aligned); the caller syncs.
__device__ __forceinline__ void copy_words(void* dst, const void* src, size_t bytes) {
    for (size_t i = threadIdx.x; i < bytes / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
}

__device__ __forceinline__ float finite_or_zero(float v) { return isfinite(v) ? v : 0.0f; }

__device__ __forceinline__ uint8_t* align16(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 15u) & ~(uintptr_t)15u);
}

// last-CTA ticket: returns true in exactly one CTA, after all `expected`
// CTAs have made their global writes visible.
__device__ __forceinline__ bool last_cta(unsigned* counter, unsigned expected) {
    __shared__ bool is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(counter, 1u) == expected - 1u;
    __syncthreads();
    if (is_last) __threadfence();
    return is_last;
}

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
    const int t = threadIdx.x;          // value index within each block
    const int c = t >> 6, l = t & 63;   // 64-value chunk, position inside it
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
        const float v = __fsub_rn(__fmul_rn(__fmul_rn(dd, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
        d.x[b * 256 + t] = v;
    }
}

// ---------------------------------------------------------------------------
// Q/K/V projections (qx_projection_matvec_fill_mode, src/qx_format.c:4207-4297)
// with the attention RMSNorm (:6283-6290) fused in the prologue.
// ---------------------------------------------------------------------------
constexpr int kSmallStages = 2;

__global__ void __launch_bounds__(kThreads) k_qkv(Dev d, LayerW w) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kWarps];
    __shared__ float kvals[16];
    const int H = d.dm.hidden, Q = d.dm.q_dim(), KV = d.dm.kv_dim();
    if (threadIdx.x < 16) kvals[threadIdx.x] = d.tables->kvalues[threadIdx.x];
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* ring = align16(smem + (size_t)H * 4);
    rmsnorm_to_smem(d.x, w.attn_norm, xs, H, scratch);
    const int nblk = H / 256;
    const uint32_t rb = (uint32_t)nblk * 136u, stage = (uint32_t)kTileRows * rb;
    const int ntiles = (Q + 2 * KV) / kTileRows;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    tile_pipeline<kSmallStages>(
        ntiles, stage, ring,
        [&](int t, uint8_t* dst) {
            const int r0 = t * kTileRows;
            const uint8_t* src = r0 < Q ? w.wq + (size_t)r0 * rb
                                 : r0 < Q + KV ? w.wk + (size_t)(r0 - Q) * rb
                                               : w.wv + (size_t)(r0 - Q - KV) * rb;
            stage_copy(dst, src, stage);
        },
        [&](int t, const uint8_t* s) {
            for (int r = warp; r < kTileRows; r += kWarps) {
                const float acc = dot_iq4_xs(s + r * rb, xs, nblk, kvals, lane);
                if (lane == 0) d.qkv[t * kTileRows + r] = finite_or_zero(acc);
            }
        });
}

// ---------------------------------------------------------------------------
// Split-KV GQA attention over the INT8 cache, with the per-head Q/K RMSNorm
// (:3740-3757), split-half RoPE (:4625-4641), the INT8 quantize-and-append of
// the current K/V (:4449-4463, :6343-6400) and the softmax/context of
// qx_rope_gqa_attention_partial (:5127-5172).  Grid: (kv_heads, nsplit); each
// CTA handles the 8 query heads of one KV head over one 64-position chunk;
// the last CTA of each KV head merges the chunks.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_attn(Dev d, LayerW w, int layer) {
    const int D = d.dm.head_dim, KVH = d.dm.kv_heads, QH = d.dm.q_heads, group = QH / KVH;
    const int Q = d.dm.q_dim(), KV = d.dm.kv_dim(), ctx = d.dm.ctx;
    const int g = blockIdx.x, split = blockIdx.y;
    const int pos = *d.pos;
    if (pos < 0 || pos >= ctx) {
        if (threadIdx.x == 0 && g == 0 && split == 0) atomicOr(d.err, kErrPosition);
        return;
    }
    if (split * kAttnChunk > pos) return;
    const int nact = pos / kAttnChunk + 1;
    extern __shared__ __align__(16) uint8_t smem[];
    float* kcur = reinterpret_cast<float*>(smem);        // [KV]
    float* vcur = kcur + KV;                               // [KV]
    float* qs = vcur + KV;                                 // [group][D]
    float* sc = qs + group * D;                            // [group][kAttnChunk]
    int8_t* k8 = reinterpret_cast<int8_t*>(sc + group * kAttnChunk);   // [KV]
    int8_t* v8 = k8 + KV;
    __shared__ float red[2][kWarps];
    __shared__ float scales[2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const double* rope = d.rope + (size_t)pos * (D / 2) * 2;

    for (int i = threadIdx.x; i < KV; i += blockDim.x) {
        kcur[i] = d.qkv[Q + i];
        vcur[i] = d.qkv[Q + KV + i];
    }
    for (int i = threadIdx.x; i < group * D; i += blockDim.x) qs[i] = d.qkv[(g * group) * D + i];
    __syncthreads();
    // head RMSNorm + RoPE: warps [0, KVH) take the K heads, the rest the Q heads of this group
    for (int hh = warp; hh < KVH + group; hh += nw) {
        float* v = hh < KVH ? kcur + hh * D : qs + (hh - KVH) * D;
        const float* nwt = hh < KVH ? w.k_norm : w.q_norm;
        double ss = 0.0;
        for (int i = lane; i < D; i += 32) ss += (double)v[i] * (double)v[i];
        ss = warp_sum_d(ss);
        const double inv = 1.0 / sqrt(ss / (double)D + 1.0e-6);
        for (int i = lane; i < D; i += 32) v[i] = (float)((double)v[i] * inv * (double)nwt[i]);
        __syncwarp();
        for (int i = lane; i < D / 2; i += 32) {
            const double c = rope[2 * i], s = rope[2 * i + 1];
            const float x0 = v[i], x1 = v[i + D / 2];
            v[i] = (float)((double)x0 * c - (double)x1 * s);
            v[i + D / 2] = (float)((double)x0 * s + (double)x1 * c);
        }
        __syncwarp();
    }
    __syncthreads();
    // one INT8 scale for all KV values of this token (K and V separately)
    float ka = 0.f, va = 0.f;
    for (int i = threadIdx.x; i < KV; i += blockDim.x) {
        ka = fmaxf(ka, isfinite(kcur[i]) ? fabsf(kcur[i]) : 0.f);
        va = fmaxf(va, isfinite(vcur[i]) ? fabsf(vcur[i]) : 0.f);
    }
    for (int o = 16; o; o >>= 1) {
        ka = fmaxf(ka, __shfl_xor_sync(0xffffffffu, ka, o));
        va = fmaxf(va, __shfl_xor_sync(0xffffffffu, va, o));
    }
    if (lane == 0) { red[0][warp] = ka; red[1][warp] = va; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.f, b = 0.f;
        for (int i = 0; i < nw; ++i) { a = fmaxf(a, red[0][i]); b = fmaxf(b, red[1][i]); }
        scales[0] = a > 0.f ? a / 127.0f : 1.0f;
        scales[1] = b > 0.f ? b / 127.0f : 1.0f;
    }
    __syncthreads();
    const float ksc = scales[0], vsc = scales[1];
    for (int i = threadIdx.x; i < KV; i += blockDim.x) {
        int qk = isfinite(kcur[i]) ? (int)lrintf(kcur[i] / ksc) : 0;
        int qv = isfinite(vcur[i]) ? (int)lrintf(vcur[i] / vsc) : 0;
        k8[i] = (int8_t)max(-127, min(127, qk));
        v8[i] = (int8_t)max(-127, min(127, qv));
    }
    __syncthreads();
    const size_t slot = (size_t)layer * ctx + pos;
    if (g == 0 && split == 0) {
        for (int i = threadIdx.x; i < KV; i += blockDim.x) {
            d.kcache[slot * KV + i] = k8[i];
            d.vcache[slot * KV + i] = v8[i];
        }
        if (threadIdx.x == 0) { d.kscale[slot] = ksc; d.vscale[slot] = vsc; }
    }
    // scores for this chunk: warp h <-> query head g*group + h
    const int t0 = split * kAttnChunk, n = min(kAttnChunk, pos + 1 - t0);
    const float inv_sqrt_d = (float)(1.0 / sqrt((double)D));
    for (int h = warp; h < group; h += nw) {
        const float* q = qs + h * D;
        for (int tt = 0; tt < n; ++tt) {
            const int t = t0 + tt;
            const size_t st = (size_t)layer * ctx + t;
            const int8_t* kp = t == pos ? k8 + g * D : d.kcache + st * KV + g * D;
            const float ks = t == pos ? ksc : d.kscale[st];
            float s = 0.f;
            for (int i = lane; i < D; i += 32) s = fmaf(q[i], (float)kp[i] * ks, s);
            s = warp_sum(s) * inv_sqrt_d;
            if (lane == 0) sc[h * kAttnChunk + tt] = isfinite(s) ? s : 0.f;
        }
    }
    __syncthreads();
    float* part = d.attn_part;
    const int stride = D + 2;
    for (int h = warp; h < group; h += nw) {
        float m = -FLT_MAX;
        for (int tt = lane; tt < n; tt += 32) m = fmaxf(m, sc[h * kAttnChunk + tt]);
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.f;
        for (int tt = lane; tt < n; tt += 32) {
            const float p = expf(sc[h * kAttnChunk + tt] - m);
            sc[h * kAttnChunk + tt] = p;
            l += p;
        }
        l = warp_sum(l);
        __syncwarp();
        float* out = part + ((size_t)(g * group + h) * d.nsplit + split) * stride;
        for (int i = lane; i < D; i += 32) {
            float acc = 0.f;
            for (int tt = 0; tt < n; ++tt) {
                const int t = t0 + tt;
                const size_t st = (size_t)layer * ctx + t;
                const int8_t* vp = t == pos ? v8 + g * D : d.vcache + st * KV + g * D;
                const float vs = t == pos ? vsc : d.vscale[st];
                acc = fmaf(sc[h * kAttnChunk + tt], (float)vp[i] * vs, acc);
            }
            out[2 + i] = acc;
        }
        if (lane == 0) { out[0] = m; out[1] = l; }
    }
    if (!last_cta(d.counters + kCntAttn + g, (unsigned)nact)) return;
    // merge the chunks of this KV head's query heads
    for (int h = warp; h < group; h += nw) {
        const float* base = part + (size_t)(g * group + h) * d.nsplit * stride;
        float M = -FLT_MAX;
        for (int s = 0; s < nact; ++s) M = fmaxf(M, base[(size_t)s * stride]);
        float L = 0.f;
        for (int s = 0; s < nact; ++s) L += base[(size_t)s * stride + 1] * expf(base[(size_t)s * stride] - M);
        for (int i = lane; i < D; i += 32) {
            float acc = 0.f;
            for (int s = 0; s < nact; ++s)
                acc = fmaf(base[(size_t)s * stride + 2 + i], expf(base[(size_t)s * stride] - M), acc);
            d.ctxv[(g * group + h) * D + i] = acc / L;
        }
    }
    if (threadIdx.x == 0) d.counters[kCntAttn + g] = 0u;
}

// ---------------------------------------------------------------------------
// O projection + residual add (:5183, :6420-6423)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_oproj(Dev d, LayerW w) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float kvals[16];
    const int H = d.dm.hidden, Q = d.dm.q_dim();
    if (threadIdx.x < 16) kvals[threadIdx.x] = d.tables->kvalues[threadIdx.x];
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* ring = align16(smem + (size_t)Q * 4);
    copy_to_smem(d.ctxv, xs, Q);
    const int nblk = Q / 256;
    const uint32_t rb = (uint32_t)nblk * 136u, stage = (uint32_t)kTileRows * rb;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    tile_pipeline<kSmallStages>(
        H / kTileRows, stage, ring, [&](int t, uint8_t* dst) { stage_copy(dst, w.wo + (size_t)t * stage, stage); },
        [&](int t, const uint8_t* s) {
            for (int r = warp; r < kTileRows; r += kWarps) {
                const float acc = dot_iq4_xs(s + r * rb, xs, nblk, kvals, lane);
                if (lane == 0) {
                    const int r0 = t * kTileRows + r;
                    const float o = finite_or_zero(acc);
                    d.attn_out[r0] = o;
                    d.x[r0] = d.x[r0] + o;
                }
            }
        });
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
    rmsnorm_to_smem(d.x, w.ffn_norm, xs, H, scratch);
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < H; i += blockDim.x) d.xn[i] = xs[i];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * kRouterRowsPerCta + warp;
    if (e < E) {
        const float* row = w.router + (size_t)e * H;
        double acc = 0.0;
        for (int i = lane * 4; i < H; i += 128) {
            const float4 wv = *reinterpret_cast<const float4*>(row + i);
            acc += (double)wv.x * (double)xs[i];
            acc += (double)wv.y * (double)xs[i + 1];
            acc += (double)wv.z * (double)xs[i + 2];
            acc += (double)wv.w * (double)xs[i + 3];
        }
        acc = warp_sum_d(acc);
        if (lane == 0) d.router_logits[e] = acc;
    }
    if (!last_cta(d.counters + kCntRouter, gridDim.x)) return;
    const int t = threadIdx.x;
    const double lg = t < E ? d.router_logits[t] : -1.0e300;
    // max
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
        // 8 rounds of argmax with strict > (lowest index wins ties)
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
// Tile = 16 rows of gate and the same 16 rows of up for one expert.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_gateup(Dev d, LayerW w, int layer) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float res[2][kTileRows];
    const int H = d.dm.hidden, I = d.dm.moe_inter;
    Tables* T = reinterpret_cast<Tables*>(smem);
    float* xs = reinterpret_cast<float*>(smem + sizeof(Tables));
    uint8_t* ring = align16(reinterpret_cast<uint8_t*>(xs + H));
    copy_words(T->iq2xs, d.tables->iq2xs, sizeof(T->iq2xs));
    copy_words(T->ksigns, d.tables->ksigns, sizeof(T->ksigns));
    copy_to_smem(d.xn, xs, H);
    const int nblk = H / 256;
    const uint32_t rb = (uint32_t)nblk * 74u, half = (uint32_t)kTileRows * rb, stage = 2u * half;
    const size_t slice = (size_t)I * rb;
    const int tiles_per_expert = I / kTileRows;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int* sel = d.sel + layer * 8;
    tile_pipeline<kSmallStages>(
        8 * tiles_per_expert, stage, ring,
        [&](int t, uint8_t* dst) {
            const int k = t / tiles_per_expert, i0 = (t % tiles_per_expert) * kTileRows;
            const size_t off = (size_t)sel[k] * slice + (size_t)i0 * rb;
            stage_copy(dst, w.gate + off, half);
            stage_copy(dst + half, w.up + off, half);
        },
        [&](int t, const uint8_t* s) {
            for (int r = warp; r < 2 * kTileRows; r += kWarps) {
                const float v = dot_iq2_xs(s + (r / kTileRows) * half + (r % kTileRows) * rb, xs, nblk, *T, lane);
                if (lane == 0) res[r / kTileRows][r % kTileRows] = finite_or_zero(v);
            }
            __syncthreads();
            if (threadIdx.x < kTileRows) {
                const int k = t / tiles_per_expert, i = (t % tiles_per_expert) * kTileRows + threadIdx.x;
                const double g = (double)res[0][threadIdx.x];
                d.hbuf[k * I + i] = (float)(g / (1.0 + exp(-g)) * (double)res[1][threadIdx.x]);
            }
        });
}

// ---------------------------------------------------------------------------
// IQ3_XXS down projections of the 8 experts with the rank-ordered weighted sum
// and the residual add fused (:5298-5309).  Tile = rows [16t, 16t+16) of all
// 8 selected experts, so each output row is finished inside one CTA.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_down(Dev d, LayerW w, int layer) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float y[8][kTileRows];
    const int H = d.dm.hidden, I = d.dm.moe_inter;
    Tables* T = reinterpret_cast<Tables*>(smem);
    float* hs = reinterpret_cast<float*>(smem + sizeof(Tables));
    uint8_t* ring = align16(reinterpret_cast<uint8_t*>(hs + 8 * I));
    copy_words(T->iq3xxs, d.tables->iq3xxs, sizeof(T->iq3xxs));
    copy_words(T->ksigns, d.tables->ksigns, sizeof(T->ksigns));
    copy_to_smem(d.hbuf, hs, 8 * I);
    const int nblk = I / 256;
    const uint32_t rb = (uint32_t)nblk * 98u, part = (uint32_t)kTileRows * rb, stage = 8u * part;
    const size_t slice = (size_t)H * rb;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int* sel = d.sel + layer * 8;
    tile_pipeline<kSmallStages>(
        H / kTileRows, stage, ring,
        [&](int t, uint8_t* dst) {
            for (int k = 0; k < 8; ++k)
                stage_copy(dst + k * part, w.down + (size_t)sel[k] * slice + (size_t)t * part, part);
        },
        [&](int t, const uint8_t* s) {
            for (int r = warp; r < 8 * kTileRows; r += kWarps) {
                const int k = r / kTileRows, rr = r % kTileRows;
                const float v = dot_iq3_xxs(s + k * part + rr * rb, hs + k * I, nblk, *T, lane);
                if (lane == 0) y[k][rr] = finite_or_zero(v);
            }
            __syncthreads();
            if (threadIdx.x < kTileRows) {
                const int r = t * kTileRows + threadIdx.x;
                float moe = 0.0f;
                for (int k = 0; k < 8; ++k) moe += (float)(d.selw_d[k] * (double)y[k][threadIdx.x]);
                d.moe_out[r] = moe;
                d.x[r] = d.x[r] + moe;
            }
        });
}

// ---------------------------------------------------------------------------
// Final RMSNorm + Q6_K head + argmax (qx_compute_real_final_head,
// src/qx_format.c:3554-3738; greedy pick :3045-3057).  Persistent grid; each
// CTA keeps its best (value, lowest index); the last CTA picks the token,
// records it at tokens_out[pos] and advances (token, pos) for the next step.
// ---------------------------------------------------------------------------
constexpr int kHeadStages = 4;

__global__ void __launch_bounds__(kThreads) k_head(Dev d) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kWarps];
    __shared__ float wbv[kWarps];
    __shared__ int wbi[kWarps];
    const int H = d.dm.hidden, V = d.dm.vocab;
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* ring = align16(smem + (size_t)H * 4);
    rmsnorm_to_smem(d.x, d.out_norm, xs, H, scratch);
    const int nblk = H / 256;
    const uint32_t rb = (uint32_t)nblk * 210u, stage = (uint32_t)kTileRows * rb;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    bool bad = false;
    tile_pipeline<kHeadStages>(
        V / kTileRows, stage, ring, [&](int t, uint8_t* dst) { stage_copy(dst, d.head + (size_t)t * stage, stage); },
        [&](int t, const uint8_t* s) {
            for (int r = warp; r < kTileRows; r += kWarps) {
                const float v = dot_q6_k(s + r * rb, xs, nblk, lane);
                const int row = t * kTileRows + r;
                if (lane == 0) {
                    d.logits[row] = v;
                    if (!isfinite(v)) bad = true;
                    if (v > bv || (v == bv && row < bi)) { bv = v; bi = row; }
                }
            }
        });
    if (lane == 0) { wbv[warp] = bv; wbi[warp] = bi; }
    if (bad) atomicOr(d.err, kErrNonFinite);
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < kWarps; ++i)
            if (wbv[i] > bv || (wbv[i] == bv && wbi[i] < bi)) { bv = wbv[i]; bi = wbi[i]; }
        d.best_val[blockIdx.x] = bv;
        d.best_idx[blockIdx.x] = bi;
    }
    if (!last_cta(d.counters + kCntHead, gridDim.x)) return;
    if (threadIdx.x == 0) {
        float v = d.best_val[0];
        int i = d.best_idx[0];
        for (int c = 1; c < (int)gridDim.x; ++c) {
            const float cv = d.best_val[c];
            const int ci = d.best_idx[c];
            if (cv > v || (cv == v && ci < i)) { v = cv; i = ci; }
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

// Top-N of the logits buffer by repeated argmax (ties to the lower index),
// the order qx_compute_real_final_head keeps (:3715-3731).
__global__ void __launch_bounds__(1024) k_topn(Dev d, int top_n, int* out_idx, float* out_val) {
    __shared__ float wv[32];
    __shared__ int wi[32];
    __shared__ int chosen[32];
    const int V = d.dm.vocab, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int k = 0; k < top_n; ++k) {
        float bv = -FLT_MAX;
        int bi = 0x7fffffff;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            bool taken = false;
            for (int j = 0; j < k; ++j) taken |= chosen[j] == i;
            const float v = d.logits[i];
            if (!taken && (v > bv || (v == bv && i < bi))) { bv = v; bi = i; }
        }
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { wv[warp] = bv; wi[warp] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
                if (wv[i] > bv || (wv[i] == bv && wi[i] < bi)) { bv = wv[i]; bi = wi[i]; }
            chosen[k] = bi;
            out_idx[k] = bi;
            out_val[k] = bv;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// launch configuration
// ---------------------------------------------------------------------------
static size_t smem_qkv(const Dims& m) { return (size_t)m.hidden * 4 + 16 + kSmallStages * (size_t)kTileRows * (m.hidden / 256) * 136; }
static size_t smem_oproj(const Dims& m) { return (size_t)m.q_dim() * 4 + 16 + kSmallStages * (size_t)kTileRows * (m.q_dim() / 256) * 136; }
static size_t smem_attn(const Dims& m) {
    const int group = m.q_heads / m.kv_heads;
    return (size_t)(2 * m.kv_dim() + group * m.head_dim + group * kAttnChunk) * 4 + 2 * (size_t)m.kv_dim() + 16;
}
static size_t smem_router(const Dims& m) { return (size_t)m.hidden * 4; }
static size_t smem_gateup(const Dims& m) { return sizeof(Tables) + (size_t)m.hidden * 4 + 16 + kSmallStages * 2 * (size_t)kTileRows * (m.hidden / 256) * 74; }
static size_t smem_down(const Dims& m) { return sizeof(Tables) + (size_t)8 * m.moe_inter * 4 + 16 + kSmallStages * 8 * (size_t)kTileRows * (m.moe_inter / 256) * 98; }
static size_t smem_head(const Dims& m) { return (size_t)m.hidden * 4 + 16 + kHeadStages * (size_t)kTileRows * (m.hidden / 256) * 210; }

cudaError_t configure_kernels() {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    // allow each kernel the opt-in maximum minus its static shared memory
    auto set = [&](const void* f) {
        cudaFuncAttributes a{};
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, f);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)a.sharedSizeBytes);
    };
    set((const void*)k_qkv);
    set((const void*)k_attn);
    set((const void*)k_oproj);
    set((const void*)k_router);
    set((const void*)k_gateup);
    set((const void*)k_down);
    set((const void*)k_head);
    set((const void*)k_final_norm);
    return e;
}

int head_grid_size(int device) {
    int sms = 0, per = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    Dims m{};
    m.hidden = 2048;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_head, kThreads, smem_head(m));
    if (per < 1) per = 1;
    return sms * per;
}

void launch_embed(const Dev& d, cudaStream_t st) { k_embed<<<1, 256, 0, st>>>(d); }

void launch_qkv(const Dev& d, const LayerW& w, cudaStream_t st) {
    const int nt = (d.dm.q_dim() + 2 * d.dm.kv_dim()) / kTileRows;
    k_qkv<<<nt, kThreads, smem_qkv(d.dm), st>>>(d, w);
}

void launch_attn(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    dim3 grid(d.dm.kv_heads, d.nsplit);
    k_attn<<<grid, 256, smem_attn(d.dm), st>>>(d, w, layer);
}

void launch_oproj(const Dev& d, const LayerW& w, cudaStream_t st) {
    k_oproj<<<d.dm.hidden / kTileRows, kThreads, smem_oproj(d.dm), st>>>(d, w);
}

void launch_router(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    const int grid = (d.dm.experts + kRouterRowsPerCta - 1) / kRouterRowsPerCta;
    k_router<<<grid, kThreads, smem_router(d.dm), st>>>(d, w, layer);
}

void launch_gateup(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    const int nt = 8 * d.dm.moe_inter / kTileRows;
    k_gateup<<<nt, kThreads, smem_gateup(d.dm), st>>>(d, w, layer);
}

void launch_down(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    k_down<<<d.dm.hidden / kTileRows, kThreads, smem_down(d.dm), st>>>(d, w, layer);
}

void launch_head(const Dev& d, cudaStream_t st) {
    k_head<<<d.head_grid, kThreads, smem_head(d.dm), st>>>(d);
}

void launch_final_norm(const Dev& d, float* normalized, cudaStream_t st) {
    k_final_norm<<<1, 256, (size_t)d.dm.hidden * 4, st>>>(d, normalized);
}

void launch_topn(const Dev& d, int top_n, int* out_idx, float* out_val, cudaStream_t st) {
    k_topn<<<1, 1024, 0, st>>>(d, top_n, out_idx, out_val);
}

}  // namespace qx
