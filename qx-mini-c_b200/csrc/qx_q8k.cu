// The reference's `q8_k_compat` activation mode (src/qx_format.c:3869-4205)
// on the per-stage path: activations are quantized per 256-value block to
// int8 with one float scale (Q8_K), every dot product is an exact int32 sum of
// integer weight codes times int8 activations, and the float epilogue of each
// quant type combines the block sums in the reference's order.
//
// Layout of the work: one warp per weight row; lane l takes values l + 32k
// (k = 0..7) of each block, so every value a lane touches has index = l (mod
// 8).  The types whose reference dot keeps eight partial sums by index mod 8
// (Q5_K, Q6_K) reduce lanes l, l+8, l+16, l+24; the others reduce the warp.
// Integer sums are exact in any order; the float steps run on one lane in the
// reference's order with explicit round-to-nearest operations (no FMA
// contraction, as the reference's ISO C build has none).
#include "qx_common.cuh"
#include "qx_kernels.h"

namespace qx {
namespace {

constexpr int kQ8Warps = 8;
constexpr int kQ8RowsPerWarp = 4;

struct Q8In {
    const int8_t* q;     // [K] quantized activations
    const float* d;      // [K/256] block scales
    const int* bs16;     // [K/16] sums of 16 consecutive q
};

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Quantize xs[0..K) (shared memory) to Q8_K (qx_quantize_q8_k, :3891-3927):
// the value of largest magnitude (first one on ties) sets iscale = -127/max,
// d = 1/iscale, q = round-to-nearest-even(iscale * x) clamped to [-128, 127].
// One warp per block; lane l holds values 8l..8l+7.  Non-finite input sets err.
__device__ void quantize_q8k(const float* xs, int K, int8_t* q, float* dq, int* bs16, int* err) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int blk = warp; blk < K / 256; blk += nw) {
        const float* x = xs + blk * 256;
        float best = 0.f;
        int bi = 0x7fffffff;
        bool bad = false;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = lane * 8 + j;
            const float v = x[i];
            bad |= !isfinite(v);
            const float a = fabsf(v);
            if (a > best) { best = a; bi = i; }   // in index order within the lane
        }
        for (int o = 16; o; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        bad = __any_sync(0xffffffffu, bad);
        if (bad) {
            if (lane == 0) atomicOr(err, kErrQ8Input);
            continue;
        }
        const float max_value = best > 0.f ? x[bi] : 0.f;
        const float iscale = max_value == 0.f ? 0.f : __fdiv_rn(-127.0f, max_value);
        if (lane == 0) dq[blk] = iscale == 0.f ? 0.f : __fdiv_rn(1.0f, iscale);
        int sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = lane * 8 + j;
            int v = iscale == 0.f ? 0 : __float2int_rn(__fmul_rn(iscale, x[i]));
            v = v > 127 ? 127 : v < -128 ? -128 : v;
            q[blk * 256 + i] = (int8_t)v;
            sum += v;
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);          // lanes 2m, 2m+1 cover one 16-value group
        if ((lane & 1) == 0) bs16[blk * 16 + lane / 2] = sum;
    }
    __syncthreads();
}

__device__ __forceinline__ float bcast(float v) { return __shfl_sync(0xffffffffu, v, 0); }

// ---- per-type dots: every lane returns the reference's float ----------------

// IQ4_XS (qx_dot_iq4_xs_q8_k, :3929-3951)
__device__ float q8_iq4_xs(const uint8_t* row, int nblk, const Q8In& a, const float* kvalues, int lane) {
    float total = 0.f;
    const int kv_lo = (int)kvalues[0];   // silence unused warnings for degenerate K
    (void)kv_lo;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 136;
        int dk[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint8_t byte = blk[8 + 16 * k + (lane & 15)];
            const int nib = lane < 16 ? byte & 15 : byte >> 4;
            dk[k] = warp_sum_i((int)kvalues[nib] * (int)a.q[b * 256 + lane + 32 * k]);
        }
        if (lane == 0) {
            const float d = __fmul_rn(h2f(ld16(blk)), a.d[b]);
            const uint32_t sh = ld16(blk + 2);
            for (int k = 0; k < 8; ++k) {
                const int s = ((blk[4 + k / 2] >> (4 * (k & 1))) & 15) | (((sh >> (2 * k)) & 3) << 4);
                total = __fadd_rn(total, __fmul_rn(__fmul_rn(d, (float)(s - 32)), (float)dk[k]));
            }
        }
    }
    return bcast(total);
}

// Q6_K (qx_dot_q6_k_q8_k, :3988-4021)
__device__ float q8_q6_k(const uint8_t* row, int nblk, const Q8In& a, int lane) {
    float sums = 0.f;                            // lane c < 8: sums[c]
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 210;
        int acc = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int idx = lane + 32 * k, h = k >> 2, s = k & 3;
            const uint8_t ql = blk[64 * h + (s & 1) * 32 + lane];
            const int nib = (s >> 1) ? ql >> 4 : ql & 15;
            const int hb = (blk[128 + 32 * h + lane] >> (2 * s)) & 3;
            const int quant = (nib | (hb << 4)) - 32;
            acc += (int)(int8_t)blk[192 + idx / 16] * (int)a.q[b * 256 + idx] * quant;
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 8);
        acc += __shfl_xor_sync(0xffffffffu, acc, 16);
        const float d = __fmul_rn(h2f(ld16(blk + 208)), a.d[b]);
        sums = __fadd_rn(sums, __fmul_rn(d, (float)acc));
    }
    float total = 0.f;
    for (int c = 0; c < 8; ++c) total = __fadd_rn(total, __shfl_sync(0xffffffffu, sums, c));
    return total;
}

// Q5_K (qx_dot_q5_k_q8_k, :3953-3986)
__device__ float q8_q5_k(const uint8_t* row, int nblk, const Q8In& a, int lane) {
    float sums = 0.f, sumf = 0.f;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 176;
        const uint8_t qh = blk[16 + lane];
        int acc = 0;
        int min_sum = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            uint32_t sc, m;
            q5k_scale_min(k, blk + 4, sc, m);
            const uint8_t packed = blk[48 + (k / 2) * 32 + lane];
            const int quant = ((k & 1) ? packed >> 4 : packed & 15) + (((qh >> k) & 1) ? 16 : 0);
            acc += (int)sc * quant * (int)a.q[b * 256 + lane + 32 * k];
            min_sum += (a.bs16[b * 16 + 2 * k] + a.bs16[b * 16 + 2 * k + 1]) * (int)m;
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 8);
        acc += __shfl_xor_sync(0xffffffffu, acc, 16);
        const float d = h2f(ld16(blk)), dmin = h2f(ld16(blk + 2));
        sums = __fadd_rn(sums, __fmul_rn(__fmul_rn(d, a.d[b]), (float)acc));
        sumf = __fsub_rn(sumf, __fmul_rn(__fmul_rn(dmin, a.d[b]), (float)min_sum));
    }
    for (int c = 0; c < 8; ++c) sumf = __fadd_rn(sumf, __shfl_sync(0xffffffffu, sums, c));
    return sumf;
}

// IQ2_XS / IQ2_S (qx_dot_iq2_xs_q8_k :4066, qx_dot_iq2_s_q8_k :4102): lane l
// takes entry 4k + l/8 (value l&7) of each 32-value group k.
template <bool S>
__device__ float q8_iq2(const uint8_t* row, int nblk, const Q8In& a, const Tables* tab, int lane) {
    float sumf = 0.f;
    const int le = lane >> 3, j = lane & 7;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * (S ? 82 : 74);
        int acc = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int e = 4 * k + le;
            int g, neg;
            uint8_t sbyte;
            if (S) {
                const uint32_t idx = blk[2 + e] | (((uint32_t)blk[66 + k] << (8 - 2 * le)) & 0x300u);
                g = (int)((__ldg(&tab->iq2s[idx][j >> 2]) >> (8 * (j & 3))) & 255u);
                neg = (blk[34 + e] >> j) & 1;
                sbyte = blk[74 + k];
            } else {
                const uint32_t q = ld16(blk + 2 + 2 * e);
                g = (int)tab->iq2xs[q & 511u][j];
                neg = (tab->ksigns[q >> 9] >> j) & 1;
                sbyte = blk[66 + k];
            }
            const int ls = le < 2 ? 2 * (sbyte & 15) + 1 : 2 * (sbyte >> 4) + 1;
            const int v = g * (int)a.q[b * 256 + lane + 32 * k] * ls;
            acc += neg ? -v : v;
        }
        const int bsum = warp_sum_i(acc);
        sumf = __fadd_rn(sumf, __fmul_rn(__fmul_rn(h2f(ld16(blk)), a.d[b]), (float)bsum));
    }
    return __fmul_rn(0.125f, sumf);
}

// IQ3_XXS / IQ3_S (qx_dot_iq3_xxs_q8_k :4135, qx_dot_iq3_s_q8_k :4168): lane
// l takes value l of each 32-value group k: 8-value part l/8, value l&7.
template <bool S>
__device__ float q8_iq3(const uint8_t* row, int nblk, const Q8In& a, const Tables* tab, int lane) {
    float sumf = 0.f;
    const int l = lane >> 3, jj = lane & 7, which = jj >> 2;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * (S ? 110 : 98);
        int acc = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            int g, neg, ls;
            if (S) {
                const uint32_t idx = blk[2 + 8 * k + 2 * l + which] | ((((uint32_t)blk[66 + k] >> (2 * l + which)) & 1u) << 8);
                g = (int)((__ldg(&tab->iq3s[idx]) >> (8 * (jj & 3))) & 255u);
                neg = (blk[74 + 4 * k + l] >> jj) & 1;
                ls = 2 * ((blk[106 + k / 2] >> (4 * (k & 1))) & 15) + 1;
            } else {
                const uint32_t aux = ld32u(blk + 66 + 4 * k);
                g = (int)tab->iq3xxs[blk[2 + 8 * k + 2 * l + which]][jj & 3];
                neg = (tab->ksigns[(aux >> (7 * l)) & 127u] >> jj) & 1;
                ls = 2 * (int)(aux >> 28) + 1;
            }
            const int v = g * (int)a.q[b * 256 + lane + 32 * k] * ls;
            acc += neg ? -v : v;
        }
        const int bsum = warp_sum_i(acc);
        sumf = __fadd_rn(sumf, __fmul_rn(__fmul_rn(h2f(ld16(blk)), a.d[b]), (float)bsum));
    }
    return S ? sumf : __fmul_rn(0.25f, sumf);
}

__device__ float q8_dot(int type, const uint8_t* row, int nblk, const Q8In& a, const Tables* tab, int lane) {
    switch (type) {
        case 13: return q8_q5_k(row, nblk, a, lane);
        case 14: return q8_q6_k(row, nblk, a, lane);
        case 17: return q8_iq2<false>(row, nblk, a, tab, lane);
        case 18: return q8_iq3<false>(row, nblk, a, tab, lane);
        case 21: return q8_iq3<true>(row, nblk, a, tab, lane);
        case 22: return q8_iq2<true>(row, nblk, a, tab, lane);
        default: return q8_iq4_xs(row, nblk, a, tab->kvalues, lane);
    }
}

__device__ uint32_t row_bytes_of(int type, int K) {
    const uint32_t bb = type == 13 ? 176u : type == 14 ? 210u : type == 17 ? 74u : type == 18 ? 98u
                      : type == 21 ? 110u : type == 22 ? 82u : 136u;
    return (uint32_t)(K / 256) * bb;
}

// Shared memory of one quantized input of K values.
struct Q8Smem {
    float* xs;
    int8_t* q;
    float* d;
    int* bs16;
};
__device__ Q8Smem q8_carve(uint8_t* smem, int K) {
    Carve cv(smem);
    Q8Smem s;
    s.xs = cv.take<float>(K);
    s.q = cv.take<int8_t>(K);
    s.d = cv.take<float>(K / 256);
    s.bs16 = cv.take<int>(K / 16);
    return s;
}

// Projection rows [row0, row0 + 32) of W (type) on the Q8_K of RMSNorm(in)
// (norm_w given) or of in; residual: attn_out = o, x += o; else out = o.
// Non-finite dots become 0 (qx_projection_matvec_fill_mode, :4290-4291).
__global__ void __launch_bounds__(kQ8Warps * 32) k_q8_proj(Dev d, int type, const float* in, const float* norm_w,
                                                         const uint8_t* W, int rows, int K, float* out, int residual) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kQ8Warps];
    const Q8Smem s = q8_carve(smem, K);
    if (norm_w) rmsnorm_to_smem(in, norm_w, s.xs, K, scratch);
    else copy_to_smem(in, s.xs, K);
    quantize_q8k(s.xs, K, s.q, s.d, s.bs16, d.err);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rb = row_bytes_of(type, K);
    const Q8In a{s.q, s.d, s.bs16};
    for (int j = 0; j < kQ8RowsPerWarp; ++j) {
        const int row = (blockIdx.x * kQ8Warps + warp) * kQ8RowsPerWarp + j;
        if (row >= rows) break;
        const float v = q8_dot(type, W + (size_t)row * rb, K / 256, a, d.tables, lane);
        if (lane == 0) {
            const float o = isfinite(v) ? v : 0.0f;
            if (residual) {
                d.attn_out[row] = o;
                d.x[row] = d.x[row] + o;
            } else {
                out[row] = o;
            }
        }
    }
}

// Gate/up rows of the 8 selected experts on the Q8_K of the FFN-normed input
// (:5290-5297): h = (float)(silu((double)g) * (double)u); a non-finite gate or
// up output is an error (:4771).
__global__ void __launch_bounds__(kQ8Warps * 32) k_q8_gateup(Dev d, LayerW w, int layer) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int H = d.dm.hidden, I = d.dm.moe_inter;
    const Q8Smem s = q8_carve(smem, H);
    copy_to_smem(d.xn, s.xs, H);
    quantize_q8k(s.xs, H, s.q, s.d, s.bs16, d.err);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rb = row_bytes_of(w.tgate, H);
    const Q8In a{s.q, s.d, s.bs16};
    for (int j = 0; j < kQ8RowsPerWarp; ++j) {
        const int item = (blockIdx.x * kQ8Warps + warp) * kQ8RowsPerWarp + j;   // slot * I + row
        if (item >= 8 * I) break;
        const int k = item / I, r = item % I;
        const size_t off = ((size_t)d.sel[layer * 8 + k] * I + r) * rb;
        const float g = q8_dot(w.tgate, w.gate + off, H / 256, a, d.tables, lane);
        const float u = q8_dot(w.tup, w.up + off, H / 256, a, d.tables, lane);
        if (lane == 0) {
            if (!isfinite(g) || !isfinite(u)) atomicOr(d.err, kErrQ8Expert);
            const double gd = (double)g;
            d.hbuf[item] = (float)(gd / (1.0 + exp(-gd)) * (double)u);
        }
    }
}

// Down rows of the 8 experts, each on the Q8_K of its own SwiGLU output
// (:5298-5303), then the rank-order weighted sum and the residual add.
__global__ void __launch_bounds__(kQ8Warps * 32) k_q8_down(Dev d, LayerW w, int layer) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int H = d.dm.hidden, I = d.dm.moe_inter;
    const Q8Smem s = q8_carve(smem, 8 * I);
    copy_to_smem(d.hbuf, s.xs, 8 * I);
    quantize_q8k(s.xs, 8 * I, s.q, s.d, s.bs16, d.err);     // expert k's blocks start at k * I / 256
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rb = row_bytes_of(w.tdown, I);
    for (int j = 0; j < kQ8RowsPerWarp; ++j) {
        const int row = (blockIdx.x * kQ8Warps + warp) * kQ8RowsPerWarp + j;
        if (row >= H) break;
        float moe = 0.0f;
        for (int k = 0; k < 8; ++k) {
            const Q8In a{s.q + k * I, s.d + k * (I / 256), s.bs16 + k * (I / 16)};
            const size_t off = ((size_t)d.sel[layer * 8 + k] * H + row) * rb;
            const float y = q8_dot(w.tdown, w.down + off, I / 256, a, d.tables, lane);
            if (lane == 0 && !isfinite(y)) atomicOr(d.err, kErrQ8Expert);
            moe += (float)(d.selw_d[k] * (double)y);
        }
        if (lane == 0) {
            d.moe_out[row] = moe;
            d.x[row] = d.x[row] + moe;
        }
    }
}

// Final RMSNorm + Q6_K head on the Q8_K of the normed input
// (qx_compute_real_final_head_q8_k, :4023-4058): float logits, the top entry
// by float value (ties to the lower token); the last CTA records the token.
__global__ void __launch_bounds__(kQ8Warps * 32) k_q8_head(Dev d) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kQ8Warps];
    __shared__ float wv[kQ8Warps];
    __shared__ int wi[kQ8Warps];
    const int H = d.dm.hidden, V = d.dm.vocab;
    const Q8Smem s = q8_carve(smem, H);
    rmsnorm_to_smem(d.x, d.out_norm, s.xs, H, scratch);
    quantize_q8k(s.xs, H, s.q, s.d, s.bs16, d.err);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rb = (uint32_t)(H / 256) * 210u;
    const Q8In a{s.q, s.d, s.bs16};
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int row = blockIdx.x * kQ8Warps + warp; row < V; row += gridDim.x * kQ8Warps) {
        const float v = q8_q6_k(d.head + (size_t)row * rb, H / 256, a, lane);
        if (lane == 0) {
            if (!isfinite(v)) atomicOr(d.err, kErrQ8Head);
            d.logits[row] = v;
            if (d.logits_d) d.logits_d[row] = (double)v;
            if (v > bv || (v == bv && row < bi)) { bv = v; bi = row; }
        }
    }
    if (lane == 0) { wv[warp] = bv; wi[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < kQ8Warps; ++i)
            if (wv[i] > bv || (wv[i] == bv && wi[i] < bi)) { bv = wv[i]; bi = wi[i]; }
        d.best_val[blockIdx.x] = (double)bv;
        d.best_idx[blockIdx.x] = bi;
    }
    if (!last_cta(d.counters + kCntHead, gridDim.x)) return;
    if (threadIdx.x == 0) {
        double v = d.best_val[0];
        int i = d.best_idx[0];
        for (int c = 1; c < (int)gridDim.x; ++c)
            if (d.best_val[c] > v || (d.best_val[c] == v && d.best_idx[c] < i)) { v = d.best_val[c]; i = d.best_idx[c]; }
        const int pos = *d.pos;
        if (pos >= 0 && pos < d.dm.ctx) d.tokens_out[pos] = i;
        *d.token = i;
        *d.pos = pos + 1;
        d.counters[kCntHead] = 0u;
    }
}

size_t q8_smem(int K) { return 64 + (size_t)K * 5 + (size_t)K / 256 * 4 + (size_t)K / 16 * 4 + 64; }

}  // namespace

cudaError_t q8_configure() {
    cudaError_t e = cudaFuncSetAttribute(k_q8_proj, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_q8_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_q8_down, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_q8_head, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
    return e;
}

static int q8_grid(int rows) { return (rows + kQ8Warps * kQ8RowsPerWarp - 1) / (kQ8Warps * kQ8RowsPerWarp); }

void launch_q8_proj(const Dev& d, int type, const float* in, const float* norm_w, const uint8_t* W, int rows, int K,
                    float* out, int residual, cudaStream_t st) {
    k_q8_proj<<<q8_grid(rows), kQ8Warps * 32, q8_smem(K), st>>>(d, type, in, norm_w, W, rows, K, out, residual);
}

void launch_q8_gateup(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    k_q8_gateup<<<q8_grid(8 * d.dm.moe_inter), kQ8Warps * 32, q8_smem(d.dm.hidden), st>>>(d, w, layer);
}

void launch_q8_down(const Dev& d, const LayerW& w, int layer, cudaStream_t st) {
    k_q8_down<<<q8_grid(d.dm.hidden), kQ8Warps * 32, q8_smem(8 * d.dm.moe_inter), st>>>(d, w, layer);
}

void launch_q8_head(const Dev& d, cudaStream_t st) {
    k_q8_head<<<d.head_grid, kQ8Warps * 32, q8_smem(d.dm.hidden), st>>>(d);
}

}  // namespace qx
