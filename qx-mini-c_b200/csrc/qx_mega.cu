// One greedy decode step as a single persistent cooperative kernel.
//
// Every CTA (one per SM) walks the same phase sequence: embedding, then per
// layer QKV -> attention -> O projection -> router -> gate/up -> down, then
// the head.  Phases are separated by a grid barrier (bounded spin, error flag
// on timeout).  Work items of a phase (16-row weight tiles) are assigned to
// CTAs round-robin; a CTA issues the cp.async copies of its NEXT phase's
// weight tiles into the other half of a double buffer before it computes the
// current phase, so the DRAM latency of the next phase and the barrier wait
// overlap.  The arithmetic is the same exact-integer tensor-core dot product
// and double-precision elementwise code as the per-stage kernels, so results
// are bit-identical to them (and to the reference's double accumulation).
#include <algorithm>
#include <cfloat>

#include "qx_common.cuh"

namespace qx {

struct MegaLayout {                      // byte offsets into dynamic shared memory
    uint32_t xs, xb, sb, tab, part, buf0, buf1, total, buf_bytes;
};

namespace {

constexpr int kMT = 256;                 // threads per CTA
constexpr int kMW = kMT / 32;
constexpr int kMaxTasks = 96;            // (tile, block) tasks per CTA per phase
constexpr long long kSpinLimit = 1ll << 24;   // ~1e7 L2 round trips: seconds
enum { QXH_IQ4_XS_F = 23, QXH_IQ2_XS_F = 17, QXH_IQ3_XXS_F = 18, QXH_Q6_K_F = 14 };

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier: every CTA arrives once per call; `epoch` counts calls.
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Trace buffer (optional, profiling only): [0, n) exit stamp of each barrier
// taken by CTA 0 (slot 0 = kernel start), [n, 9n) eight in-phase markers of
// CTA 0 per barrier epoch, [9n, 9n + n*grid) each CTA's arrival at each
// barrier; n = 3 + 6 * layers.
__device__ __forceinline__ size_t trace_n(const Dev& d) { return 3 + 6 * (size_t)d.dm.layers; }

__device__ __forceinline__ void mark(const Dev& d, unsigned epoch, int k) {
    if (d.trace && blockIdx.x == 0 && threadIdx.x == 0) d.trace[trace_n(d) + (size_t)(epoch + 1) * 8 + k] = global_ns();
}

__device__ __forceinline__ void grid_sync(unsigned* bar, unsigned& epoch, const Dev& d) {
    int* err = d.err;
    unsigned long long* trace = d.trace;
    __syncthreads();
    epoch += 1;
    if (threadIdx.x == 0) {
        if (trace) trace[9 * trace_n(d) + (size_t)epoch * gridDim.x + blockIdx.x] = global_ns();
        // the CTA's writes are ordered before this release by the bar.sync above
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        const unsigned target = epoch * gridDim.x;
        long long it = 0;
        while (ld_acquire(bar) < target) {
            if (++it > kSpinLimit) { atomicOr(err, kErrTimeout); break; }
        }
        if (trace && blockIdx.x == 0) trace[epoch] = global_ns();
    }
    __syncthreads();
}

// Items of a phase owned by this CTA: blockIdx.x, blockIdx.x + G, ...
__device__ __forceinline__ int my_items(int n) {
    return blockIdx.x < (unsigned)n ? (n - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
}
__device__ __forceinline__ int item_id(int k) { return (int)blockIdx.x + k * (int)gridDim.x; }

// Run (tile, block) tasks over `ntile` staged 16-row tiles of row size rb with
// nblk blocks; tile i uses activation xq[xsel(i)].  part[task][16] doubles.
template <int FMT, class XSel>
__device__ void run_tasks(const uint8_t* tiles, uint32_t tb, uint32_t rb, int ntile, int nblk, XSel xsel,
                          const uint32_t* K4, const IqTab* T, double* part) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
    const int ntask = ntile * nblk;
    for (int task = warp; task < ntask; task += kMW) {
        const int i = task / nblk, b = task % nblk;
        const uint8_t* base = tiles + (size_t)i * tb;
        const XQ x = xsel(i);
        Acc acc{};
        if (FMT == QXH_IQ4_XS_F) dot_iq4_xs_mma(base + g * rb, base + (g + 8) * rb, b, b + 1, x, K4, lane, acc);
        if (FMT == QXH_IQ2_XS_F) dot_iq2_xs_mma(base + g * rb, base + (g + 8) * rb, b, b + 1, x, *T, lane, acc);
        if (FMT == QXH_IQ3_XXS_F) dot_iq3_xxs_mma(base + g * rb, base + (g + 8) * rb, b, b + 1, x, *T, lane, acc);
        if (FMT == QXH_Q6_K_F) dot_q6_k_mma(base + g * rb, base + (g + 8) * rb, b, b + 1, x, lane, acc);
        store_tile_rows(part, task, acc);
    }
    __syncthreads();
}

// Sum the block partials of tile i, row r, in block order.
__device__ __forceinline__ double tile_row(const double* part, int i, int nblk, int r) {
    double v = 0.0;
    for (int b = 0; b < nblk; ++b) v += part[(i * nblk + b) * kTileRows + r];
    return v;
}

// ---- weight-tile issue per phase -------------------------------------------
__device__ void issue_qkv(const Dev& d, const LayerW& w, uint8_t* buf) {
    const int H = d.dm.hidden, Q = d.dm.q_dim(), KV = d.dm.kv_dim();
    const uint32_t rb = (uint32_t)(H / 256) * 136u, tb = (uint32_t)kTileRows * rb;
    const int n = (Q + 2 * KV) / kTileRows, mine = my_items(n);
    for (int k = 0; k < mine; ++k) {
        const int r0 = item_id(k) * kTileRows;
        const uint8_t* src = r0 < Q ? w.wq + (size_t)r0 * rb
                             : r0 < Q + KV ? w.wk + (size_t)(r0 - Q) * rb
                                           : w.wv + (size_t)(r0 - Q - KV) * rb;
        stage_copy(buf + (size_t)k * tb, src, tb);
    }
}

__device__ void issue_oproj(const Dev& d, const LayerW& w, uint8_t* buf) {
    const uint32_t rb = (uint32_t)(d.dm.q_dim() / 256) * 136u, tb = (uint32_t)kTileRows * rb;
    const int mine = my_items(d.dm.hidden / kTileRows);
    for (int k = 0; k < mine; ++k) stage_copy(buf + (size_t)k * tb, w.wo + (size_t)item_id(k) * tb, tb);
}

__device__ void issue_router(const Dev& d, const LayerW& w, uint8_t* buf) {
    const uint32_t rowb = (uint32_t)d.dm.hidden * 4u;
    const int mine = my_items(d.dm.experts);
    for (int k = 0; k < mine; ++k)
        stage_copy(buf + (size_t)k * rowb, reinterpret_cast<const uint8_t*>(w.router) + (size_t)item_id(k) * rowb, rowb);
}

__device__ void issue_gateup(const Dev& d, const LayerW& w, const int* sel, uint8_t* buf) {
    const int H = d.dm.hidden, I = d.dm.moe_inter;
    const uint32_t rb = (uint32_t)(H / 256) * 74u, tb = (uint32_t)kTileRows * rb;
    const int tpe = I / kTileRows, mine = my_items(8 * tpe);
    for (int k = 0; k < mine; ++k) {
        const int it = item_id(k), e = it / tpe, i0 = (it % tpe) * kTileRows;
        const size_t off = (size_t)sel[e] * ((size_t)I * rb) + (size_t)i0 * rb;
        stage_copy(buf + (size_t)(2 * k) * tb, w.gate + off, tb);
        stage_copy(buf + (size_t)(2 * k + 1) * tb, w.up + off, tb);
    }
}

__device__ void issue_down(const Dev& d, const LayerW& w, const int* sel, uint8_t* buf) {
    const int H = d.dm.hidden, I = d.dm.moe_inter;
    const uint32_t rb = (uint32_t)(I / 256) * 98u, tb = (uint32_t)kTileRows * rb;
    const size_t slice = (size_t)H * rb;
    const int mine = my_items(H / kTileRows);
    for (int k = 0; k < mine; ++k)
        for (int e = 0; e < 8; ++e)
            stage_copy(buf + (size_t)(8 * k + e) * tb, w.down + (size_t)sel[e] * slice + (size_t)item_id(k) * tb, tb);
}

constexpr int kHeadGroupTiles = 2;

__device__ void issue_head_group(const Dev& d, int grp, uint8_t* buf) {
    const uint32_t rb = (uint32_t)(d.dm.hidden / 256) * 210u, stage = (uint32_t)kHeadGroupTiles * kTileRows * rb;
    stage_copy(buf, d.head + (size_t)grp * stage, stage);
}

// ---- attention for one query head with 256 threads ----------------------------
struct AttnSmem {
    double sd[kMW];
    float sf[kMW];
    float qv[128];
    float kcur[1024];
    float vcur[1024];
    __align__(16) int8_t k8[1024];
    __align__(16) int8_t v8[1024];
};

constexpr int kVChunk = 128;   // positions of V staged per pass

// Attention of query head h (all 256 threads).  w_s: >= pos+1 doubles of
// shared scratch; v_s: kVChunk*128 bytes + kVChunk floats of shared scratch.
__device__ void attn_head(const Dev& d, const LayerW& w, int layer, int h, int pos, AttnSmem& S, double* w_s,
                          uint8_t* v_s, unsigned epoch) {
    const int D = 128, KVH = d.dm.kv_heads, group = d.dm.q_heads / KVH;
    const int Q = d.dm.q_dim(), KV = d.dm.kv_dim(), ctx = d.dm.ctx, g = h / group, i = threadIdx.x;
    const int warp = i >> 5, lane = i & 31;
    const double* rope = d.rope + (size_t)pos * 128;
    for (int j = i; j < KV; j += kMT) {
        S.kcur[j] = d.qkv[Q + j];
        S.vcur[j] = d.qkv[Q + KV + j];
    }
    if (i < 128) S.qv[i] = d.qkv[h * D + i];
    __syncthreads();
    for (int hh = warp; hh <= KVH; hh += kMW) {
        if (hh < KVH) warp_norm_rope(S.kcur + hh * D, w.k_norm, rope, lane);
        else warp_norm_rope(S.qv, w.q_norm, rope, lane);
    }
    __syncthreads();
    mark(d, epoch, 0);
    float ka = 0.f, va = 0.f;
    for (int j = i; j < KV; j += kMT) {
        ka = fmaxf(ka, isfinite(S.kcur[j]) ? fabsf(S.kcur[j]) : 0.f);
        va = fmaxf(va, isfinite(S.vcur[j]) ? fabsf(S.vcur[j]) : 0.f);
    }
    ka = block_max_f(ka, S.sf);
    va = block_max_f(va, S.sf);
    const float ksc = ka > 0.f ? ka / 127.0f : 1.0f, vsc = va > 0.f ? va / 127.0f : 1.0f;
    for (int j = i; j < KV; j += kMT) {
        const int qk = isfinite(S.kcur[j]) ? (int)lrintf(S.kcur[j] / ksc) : 0;
        const int qq = isfinite(S.vcur[j]) ? (int)lrintf(S.vcur[j] / vsc) : 0;
        S.k8[j] = (int8_t)max(-127, min(127, qk));
        S.v8[j] = (int8_t)max(-127, min(127, qq));
    }
    __syncthreads();
    mark(d, epoch, 1);
    const size_t slot = (size_t)layer * ctx + pos;
    if (h == 0) {
        for (int j = i; j < KV; j += kMT) {
            d.kcache[slot * KV + j] = S.k8[j];
            d.vcache[slot * KV + j] = S.v8[j];
        }
        if (i == 0) { d.kscale[slot] = ksc; d.vscale[slot] = vsc; }
    }
    // scores (double, dims in order) for positions i, i+256, ...
    const int T = pos + 1;
    const double sqrt_d = sqrt((double)D);
    double mloc = -1.0e300;
    for (int t = i; t < T; t += kMT) {
        const size_t st = (size_t)layer * ctx + t;
        const int8_t* kp = t == pos ? S.k8 + g * D : d.kcache + st * KV + g * D;
        const float ks = t == pos ? ksc : d.kscale[st];
        int4 raw[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) raw[j] = reinterpret_cast<const int4*>(kp)[j];
        double s = 0.0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int8_t* kb = reinterpret_cast<const int8_t*>(&raw[j]);
#pragma unroll
            for (int u = 0; u < 16; ++u) s += (double)S.qv[16 * j + u] * (double)((float)kb[u] * ks);
        }
        s /= sqrt_d;
        if (!isfinite(s)) s = 0.0;
        w_s[t] = s;
        mloc = fmax(mloc, s);
    }
    const double mx = block_max_d(mloc, S.sd);
    mark(d, epoch, 2);
    for (int t = i; t < T; t += kMT) w_s[t] = exp(w_s[t] - mx);
    double den = fixed_order_sum(w_s, T, S.sd);
    if (!isfinite(den) || den <= 0.0) den = 1.0;
    for (int t = i; t < T; t += kMT) w_s[t] = w_s[t] / den;
    mark(d, epoch, 3);
    // context: V of head g staged kVChunk positions at a time; thread i < 128
    // accumulates dim i over t in order, as the reference does.
    int8_t* vch = reinterpret_cast<int8_t*>(v_s);
    float* vsc_s = reinterpret_cast<float*>(v_s + kVChunk * 128);
    float acc = 0.0f;
    for (int t0 = 0; t0 < T; t0 += kVChunk) {
        const int n = min(kVChunk, T - t0);
        __syncthreads();
        for (int j = i; j < n * 8; j += kMT) {          // 8 x 16 bytes per position
            const int t = t0 + j / 8, part = j % 8;
            const int4* src = t == pos ? reinterpret_cast<const int4*>(S.v8 + g * D)
                                       : reinterpret_cast<const int4*>(d.vcache + ((size_t)layer * ctx + t) * KV + g * D);
            reinterpret_cast<int4*>(vch + (size_t)(j / 8) * 128)[part] = src[part];
        }
        for (int j = i; j < n; j += kMT) vsc_s[j] = t0 + j == pos ? vsc : d.vscale[(size_t)layer * ctx + t0 + j];
        __syncthreads();
        if (i < 128) {
#pragma unroll 8
            for (int j = 0; j < n; ++j) {
                const float vv = (float)vch[j * 128 + i] * vsc_s[j];
                acc += (float)(w_s[t0 + j] * (double)vv);
            }
        }
    }
    if (i < 128) d.ctxv[h * D + i] = acc;
    __syncthreads();
}

// Router softmax + top-8 over the logits in global memory (every CTA; the
// result is identical everywhere).  sel/w in shared memory.
__device__ void top8(const Dev& d, int layer, int* sel, double* wsel, double* probs, double* scratch) {
    const int E = d.dm.experts, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const double lg = t < E ? d.router_logits[t] : -1.0e300;
    const double m = block_max_d(lg, scratch);
    const double ex = t < E ? exp(lg - m) : 0.0;
    const double den = block_sum_d(ex, scratch);
    probs[t] = t < E ? ex / den : -1.0;
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
            if (lane == 0) { sel[k] = bi; wsel[k] = bv; probs[bi] = -1.0; }
            __syncwarp();
        }
        if (lane == 0) {
            double sum = 0.0;
            for (int k = 0; k < 8; ++k) sum += wsel[k];
            if (!(sum > 0.0) || !isfinite(sum)) atomicOr(d.err, kErrRouter);
            for (int k = 0; k < 8; ++k) {
                wsel[k] = wsel[k] / sum;
                if (blockIdx.x == 0) {
                    d.sel[layer * 8 + k] = sel[k];
                    d.selw[layer * 8 + k] = (float)wsel[k];
                }
            }
        }
    }
    __syncthreads();
}

}  // namespace

__global__ void __launch_bounds__(kMT, 1) k_decode_step(Dev d, const LayerW* __restrict__ layers, MegaLayout L) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kMW];
    __shared__ double probs[256];
    __shared__ double wsel[8];
    __shared__ int sel[8];
    __shared__ AttnSmem attn;
    __shared__ double hbv[kMW];
    __shared__ int hbi[kMW];
    float* xs = reinterpret_cast<float*>(smem + L.xs);
    uint32_t* xb = reinterpret_cast<uint32_t*>(smem + L.xb);
    int* sb = reinterpret_cast<int*>(smem + L.sb);
    IqTab* T = reinterpret_cast<IqTab*>(smem + L.tab);
    double* part = reinterpret_cast<double*>(smem + L.part);
    uint8_t* buf[2] = {smem + L.buf0, smem + L.buf1};
    const Dims& m = d.dm;
    const int H = m.hidden, Q = m.q_dim(), KV = m.kv_dim(), I = m.moe_inter, E = m.experts;
    unsigned epoch = 0;
    unsigned* bar = d.counters + kCntBarrier;
    const int tok = *d.token, pos = *d.pos;
    if (tok < 0 || tok >= m.vocab || pos < 0 || pos >= m.ctx) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(d.err, tok < 0 || tok >= m.vocab ? kErrToken : kErrPosition);
        return;   // uniform across the grid: no barrier is entered
    }
    if (d.trace && blockIdx.x == 0 && threadIdx.x == 0) d.trace[0] = global_ns();
    uint32_t K4[4];
    load_kv_regs(d.tables, K4);
    load_iq_tables(T, d.tables, true, true);
    int qb = 0;
    issue_qkv(d, layers[0], buf[qb]);
    cp_async_commit();
    // embedding (every CTA into its own xs; CTA 0 also writes the residual)
    {
        const int nblk = H / 256;
        const uint8_t* row = d.tok_embd + (size_t)tok * (size_t)(nblk * 144);
        const int t = threadIdx.x, c = t >> 6, l = t & 63;
        for (int b = 0; b < nblk; ++b) {
            const uint8_t* blk = row + b * 144;
            const float dd = h2f(ld16(blk)), dmin = h2f(ld16(blk + 2));
            const uint8_t* s = blk + 4;
            const int j = 2 * c + (l >= 32);
            uint32_t scv, mn;
            if (j < 4) { scv = s[j] & 63u; mn = s[j + 4] & 63u; }
            else { scv = (s[j + 4] & 15u) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
            const uint8_t qbt = blk[16 + 32 * c + (l & 31)];
            const uint32_t q = l < 32 ? (qbt & 15u) : (qbt >> 4);
            const float v = __fsub_rn(__fmul_rn(__fmul_rn(dd, (float)scv), (float)q), __fmul_rn(dmin, (float)mn));
            xs[b * 256 + t] = v;
            if (blockIdx.x == 0) d.x[b * 256 + t] = v;
        }
        __syncthreads();
    }
    for (int layer = 0; layer < m.layers; ++layer) {
        const LayerW& w = layers[layer];
        // ---------------- QKV (weights in buf[qb]) ----------------
        {
            if (layer > 0) copy_to_smem(d.x, xs, H);
            // attention RMSNorm of xs in place
            double ss = 0.0;
            for (int i = threadIdx.x; i < H; i += kMT) ss += (double)xs[i] * (double)xs[i];
            ss = block_sum_d(ss, scratch);
            const double rms = sqrt(ss / (double)H + 1.0e-6);
            for (int i = threadIdx.x; i < H; i += kMT) xs[i] = (float)((double)xs[i] / rms) * w.attn_norm[i];
            __syncthreads();
            mark(d, epoch, 0);
            build_xq(xs, H, xb, sb);
            issue_oproj(d, w, buf[1 - qb]);
            cp_async_commit();
            __syncthreads();
            mark(d, epoch, 1);
            cp_async_wait<1>();
            __syncthreads();
            mark(d, epoch, 2);
            const uint32_t rb = (uint32_t)(H / 256) * 136u, tb = (uint32_t)kTileRows * rb;
            const int mine = my_items((Q + 2 * KV) / kTileRows), nblk = H / 256;
            run_tasks<QXH_IQ4_XS_F>(buf[qb], tb, rb, mine, nblk, [&](int) { return XQ{xb, sb}; }, K4, T, part);
            mark(d, epoch, 3);
            for (int r = threadIdx.x; r < mine * kTileRows; r += kMT)
                d.qkv[item_id(r / kTileRows) * kTileRows + r % kTileRows] =
                    finite_or_zero_d(tile_row(part, r / kTileRows, nblk, r % kTileRows));
            grid_sync(bar, epoch, d);
        }
        // ---------------- attention (CTAs 0..Hq-1) ----------------
        issue_router(d, w, buf[qb]);
        cp_async_commit();
        for (int h = blockIdx.x; h < m.q_heads; h += gridDim.x)
            attn_head(d, w, layer, h, pos, attn, reinterpret_cast<double*>(smem + L.xb), smem + L.xs, epoch);
        grid_sync(bar, epoch, d);
        // ---------------- O projection (weights in buf[1-qb]) ----------------
        {
            copy_to_smem(d.ctxv, xs, Q);
            mark(d, epoch, 0);
            build_xq(xs, Q, xb, sb);
            __syncthreads();
            mark(d, epoch, 1);
            cp_async_wait<1>();
            __syncthreads();
            mark(d, epoch, 2);
            const uint32_t rb = (uint32_t)(Q / 256) * 136u, tb = (uint32_t)kTileRows * rb;
            const int mine = my_items(H / kTileRows), nblk = Q / 256;
            run_tasks<QXH_IQ4_XS_F>(buf[1 - qb], tb, rb, mine, nblk, [&](int) { return XQ{xb, sb}; }, K4, T, part);
            mark(d, epoch, 3);
            for (int r = threadIdx.x; r < mine * kTileRows; r += kMT) {
                const int row = item_id(r / kTileRows) * kTileRows + r % kTileRows;
                const float o = finite_or_zero_d(tile_row(part, r / kTileRows, nblk, r % kTileRows));
                d.attn_out[row] = o;
                d.x[row] = d.x[row] + o;
            }
            grid_sync(bar, epoch, d);
        }
        // ---------------- router (weights in buf[qb]) ----------------
        {
            copy_to_smem(d.x, xs, H);
            double ss = 0.0;
            for (int i = threadIdx.x; i < H; i += kMT) ss += (double)xs[i] * (double)xs[i];
            ss = block_sum_d(ss, scratch);
            const double rms = sqrt(ss / (double)H + 1.0e-6);
            for (int i = threadIdx.x; i < H; i += kMT) xs[i] = (float)((double)xs[i] / rms) * w.ffn_norm[i];
            __syncthreads();
            if (blockIdx.x == 0)
                for (int i = threadIdx.x; i < H; i += kMT) d.xn[i] = xs[i];
            mark(d, epoch, 0);
            cp_async_wait<0>();
            __syncthreads();
            mark(d, epoch, 1);
            const int mine = my_items(E);
            const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            for (int k = 0; k < mine; ++k) {
                const float* row = reinterpret_cast<const float*>(buf[qb] + (size_t)k * H * 4);
                double acc = 0.0;
                for (int i = (warp * 32 + lane) * 4; i < H; i += kMT * 4) {
                    const float4 v = *reinterpret_cast<const float4*>(row + i);
                    acc += (double)v.x * (double)xs[i] + (double)v.y * (double)xs[i + 1];
                    acc += (double)v.z * (double)xs[i + 2] + (double)v.w * (double)xs[i + 3];
                }
                acc = block_sum_d(acc, scratch);
                if (threadIdx.x == 0) d.router_logits[item_id(k)] = acc;
            }
            grid_sync(bar, epoch, d);
        }
        // ---------------- top-8 + gate/up (weights in buf[1-qb]) ----------------
        {
            top8(d, layer, sel, wsel, probs, scratch);
            mark(d, epoch, 0);
            issue_gateup(d, w, sel, buf[1 - qb]);
            cp_async_commit();
            issue_down(d, w, sel, buf[qb]);
            cp_async_commit();
            build_xq(xs, H, xb, sb);            // xs still holds the FFN-normed input
            __syncthreads();
            mark(d, epoch, 1);
            cp_async_wait<1>();
            __syncthreads();
            mark(d, epoch, 2);
            const uint32_t rb = (uint32_t)(H / 256) * 74u, tb = (uint32_t)kTileRows * rb;
            const int mine = my_items(8 * (I / kTileRows)), nblk = H / 256;
            run_tasks<QXH_IQ2_XS_F>(buf[1 - qb], tb, rb, 2 * mine, nblk, [&](int) { return XQ{xb, sb}; }, K4, T, part);
            mark(d, epoch, 3);
            const int tpe = I / kTileRows;
            for (int r = threadIdx.x; r < mine * kTileRows; r += kMT) {
                const int k = r / kTileRows, rr = r % kTileRows, it = item_id(k);
                const float gv = finite_or_zero_d(tile_row(part, 2 * k, nblk, rr));
                const float uv = finite_or_zero_d(tile_row(part, 2 * k + 1, nblk, rr));
                const double gd = (double)gv;
                d.hbuf[(it / tpe) * I + (it % tpe) * kTileRows + rr] = (float)(gd / (1.0 + exp(-gd)) * (double)uv);
            }
            grid_sync(bar, epoch, d);
        }
        // ---------------- down (weights in buf[qb]) ----------------
        {
            copy_to_smem(d.hbuf, xs, 8 * I);
            mark(d, epoch, 0);
            build_xq(xs, 8 * I, xb, sb);     // expert e's groups start at e * I / 16 (I % 256 == 0)
            if (layer + 1 < m.layers) issue_qkv(d, layers[layer + 1], buf[1 - qb]);
            else if ((int)blockIdx.x < m.vocab / (kTileRows * kHeadGroupTiles)) issue_head_group(d, blockIdx.x, buf[1 - qb]);
            cp_async_commit();
            __syncthreads();
            mark(d, epoch, 1);
            cp_async_wait<1>();
            __syncthreads();
            mark(d, epoch, 2);
            const uint32_t rb = (uint32_t)(I / 256) * 98u, tb = (uint32_t)kTileRows * rb;
            const int mine = my_items(H / kTileRows), nblk = I / 256;
            run_tasks<QXH_IQ3_XXS_F>(buf[qb], tb, rb, 8 * mine, nblk,
                                     [&](int i) { return XQ{xb + (i % 8) * xq_words(I), sb + (i % 8) * (I / 256)}; },
                                     K4, T, part);
            mark(d, epoch, 3);
            for (int r = threadIdx.x; r < mine * kTileRows; r += kMT) {
                const int k = r / kTileRows, rr = r % kTileRows, row = item_id(k) * kTileRows + rr;
                float moe = 0.0f;
                for (int e = 0; e < 8; ++e)
                    moe += (float)(wsel[e] * (double)finite_or_zero_d(tile_row(part, 8 * k + e, nblk, rr)));
                d.moe_out[row] = moe;
                d.x[row] = d.x[row] + moe;
            }
            grid_sync(bar, epoch, d);
        }
        qb = 1 - qb;
    }
    // ---------------- head (2-stage ring over buf[qb], buf[1-qb]) ----------------
    {
        copy_to_smem(d.x, xs, H);
        double ss = 0.0;
        for (int i = threadIdx.x; i < H; i += kMT) ss += (double)xs[i] * (double)xs[i];
        ss = block_sum_d(ss, scratch);
        const double rms = sqrt(ss / (double)H + 1.0e-6);
        for (int i = threadIdx.x; i < H; i += kMT) xs[i] = (float)((double)xs[i] / rms) * d.out_norm[i];
        __syncthreads();
        build_xq(xs, H, xb, sb);
        __syncthreads();
        const int ngroups = m.vocab / (kTileRows * kHeadGroupTiles), mine = my_items(ngroups), nblk = H / 256;
        const uint32_t rb = (uint32_t)nblk * 210u, tb = (uint32_t)kTileRows * rb;
        double bv = -1.0e300;
        int bi = 0x7fffffff;
        bool bad = false;
        for (int k = 0; k < mine; ++k) {
            uint8_t* cur = buf[(qb + k) & 1];
            if (k + 1 < mine) issue_head_group(d, item_id(k + 1), buf[(qb + k + 1) & 1]);
            cp_async_commit();
            cp_async_wait<1>();
            __syncthreads();
            run_tasks<QXH_Q6_K_F>(cur, tb, rb, kHeadGroupTiles, nblk, [&](int) { return XQ{xb, sb}; }, K4, T, part);
            if (threadIdx.x < kHeadGroupTiles * kTileRows) {
                const int i = threadIdx.x / kTileRows, r = threadIdx.x % kTileRows;
                const int row = item_id(k) * kHeadGroupTiles * kTileRows + i * kTileRows + r;
                const double v = tile_row(part, i, nblk, r);
                if (!isfinite(v)) bad = true;
                d.logits[row] = (float)v;
                if (v > bv || (v == bv && row < bi)) { bv = v; bi = row; }
            }
            __syncthreads();   // the buffer is refilled two iterations later
        }
        if (bad) atomicOr(d.err, kErrNonFinite);
        for (int o = 16; o; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if ((threadIdx.x & 31) == 0) { hbv[threadIdx.x >> 5] = bv; hbi[threadIdx.x >> 5] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int i = 1; i < kMW; ++i)
                if (hbv[i] > bv || (hbv[i] == bv && hbi[i] < bi)) { bv = hbv[i]; bi = hbi[i]; }
            d.best_val[blockIdx.x] = bv;
            d.best_idx[blockIdx.x] = bi;
        }
        grid_sync(bar, epoch, d);
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            double v = d.best_val[0];
            int i = d.best_idx[0];
            for (int c = 1; c < (int)gridDim.x; ++c) {
                const double cv = d.best_val[c];
                const int ci = d.best_idx[c];
                if (cv > v || (cv == v && ci < i)) { v = cv; i = ci; }
            }
            d.tokens_out[pos] = i;
            *d.token = i;
            *d.pos = pos + 1;
        }
    }
}

namespace {
MegaLayout g_layout;
uint32_t a16u(size_t v) { return (uint32_t)((v + 15) / 16 * 16); }
}  // namespace

// Shared-memory layout for the model geometry on `grid` CTAs.
static MegaLayout mega_layout(const Dims& m, int grid) {
    auto cdiv = [](int a, int b) { return (a + b - 1) / b; };
    const int H = m.hidden, Q = m.q_dim(), KV = m.kv_dim(), I = m.moe_inter;
    const size_t t_qkv = (size_t)kTileRows * (H / 256) * 136, t_o = (size_t)kTileRows * (Q / 256) * 136;
    const size_t t_gu = (size_t)kTileRows * (H / 256) * 74, t_dn = (size_t)kTileRows * (I / 256) * 98;
    const size_t t_hd = (size_t)kHeadGroupTiles * kTileRows * (H / 256) * 210;
    size_t bufb = 0;
    bufb = std::max(bufb, cdiv((Q + 2 * KV) / kTileRows, grid) * t_qkv);
    bufb = std::max(bufb, cdiv(H / kTileRows, grid) * t_o);
    bufb = std::max(bufb, (size_t)cdiv(m.experts, grid) * H * 4);
    bufb = std::max(bufb, cdiv(8 * (I / kTileRows), grid) * 2 * t_gu);
    bufb = std::max(bufb, cdiv(H / kTileRows, grid) * 8 * t_dn);
    bufb = std::max(bufb, t_hd);
    const int XS = std::max(std::max(H, Q), 8 * I);
    MegaLayout L{};
    uint32_t off = 0;
    L.xs = off; off += a16u(std::max((size_t)XS * 4, (size_t)kVChunk * 132));
    L.xb = off; off += a16u(xq_words(XS) * 4);
    L.sb = off; off += a16u((size_t)XS / 256 * 4 + 32);
    L.tab = off; off += a16u(sizeof(IqTab));
    L.part = off; off += a16u((size_t)kMaxTasks * kTileRows * 8);
    L.buf_bytes = a16u(bufb);
    L.buf0 = off; off += L.buf_bytes;
    L.buf1 = off; off += L.buf_bytes;
    L.total = off;
    return L;
}

// Tasks per CTA must fit the partial buffer.
static bool mega_tasks_fit(const Dims& m, int grid) {
    auto cdiv = [](int a, int b) { return (a + b - 1) / b; };
    const int H = m.hidden, Q = m.q_dim(), KV = m.kv_dim(), I = m.moe_inter;
    const int t[] = {cdiv((Q + 2 * KV) / kTileRows, grid) * (H / 256), cdiv(H / kTileRows, grid) * (Q / 256),
                     cdiv(8 * (I / kTileRows), grid) * 2 * (H / 256), cdiv(H / kTileRows, grid) * 8 * (I / 256),
                     kHeadGroupTiles * (H / 256)};
    for (int v : t)
        if (v > kMaxTasks) return false;
    return m.experts <= 256;
}

int mega_setup(int device, const Dims& m, int* grid_out) {
    int sms = 0, optin = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, k_decode_step) != cudaSuccess) return 0;
    const MegaLayout L = mega_layout(m, sms);
    if (L.total + a.sharedSizeBytes > (size_t)optin || !mega_tasks_fit(m, sms)) return 0;
    if ((size_t)m.ctx * 8 > L.sb - L.xb || (size_t)kVChunk * 132 > L.xb - L.xs) return 0;
    if (cudaFuncSetAttribute(k_decode_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total) != cudaSuccess)
        return 0;
    int per = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_decode_step, kMT, L.total);
    if (per < 1) return 0;
    g_layout = L;
    *grid_out = sms;
    return 1;
}

cudaError_t launch_decode_step(const Dev& d, const LayerW* layers_dev, int grid, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(d.counters + kCntBarrier, 0, sizeof(unsigned), st);
    if (e != cudaSuccess) return e;
    MegaLayout L = mega_layout(d.dm, grid);
    Dev dd = d;
    const LayerW* lw = layers_dev;
    void* args[] = {&dd, &lw, &L};
    return cudaLaunchCooperativeKernel((const void*)k_decode_step, dim3(grid), dim3(kMT), args, L.total, st);
}

}  // namespace qx
