// One greedy decode step as a single persistent cooperative kernel.
//
// Every CTA (one per SM) walks the same phase sequence: embedding, then per
// layer QKV -> attention -> O projection -> router -> gate/up -> down, then
// the head.  Phases are separated by a grid barrier (bounded spin, error flag
// on timeout).  Work items of a phase (16-row weight tiles) are assigned to
// CTAs round-robin; a CTA's tiles of a later phase are copied into a free
// weight buffer by bulk copies (mbarrier completion) while it computes and
// waits, so the DRAM latency of a phase overlaps the ones before it.  The
// weights are in the kernel's own layouts (IQ2R, R4, R8: re-laid once at
// engine creation, same integers and scales as the GGUF blocks); the
// arithmetic is the same exact-integer tensor-core dot product and
// double-precision elementwise code as the per-stage kernels, so results are
// bit-identical to them (and agree with the reference's double accumulation).
#include <algorithm>
#include <cfloat>
#include <mutex>

#include "qx_common.cuh"

#ifndef QX_MEGA_THREADS
#define QX_MEGA_THREADS 512
#endif

namespace qx {

struct MegaLayout {                      // byte offsets into dynamic shared memory
    uint32_t xs, xb, sb, tab, part, buf0, buf1, total, buf_bytes;
    uint32_t norm;                       // offset inside a weight buffer of the RMSNorm vector
    uint32_t iq2r_rb;                    // bytes per IQ2R gate/up row (tiles span buf0 + buf1)
};

namespace {

constexpr int kMT = QX_MEGA_THREADS;     // threads per CTA (a multiple of 256)
constexpr int kMW = kMT / 32;
constexpr int kMaxTasks = 96;            // (tile, block) tasks per CTA per phase
constexpr long long kSpinLimit = 1ll << 26;             // polls of one barrier wait, at most
constexpr unsigned long long kBarrierTimeoutNs = 2000000000ull;   // 2 s; a healthy wait is microseconds
enum { QXH_IQ4_XS_F = 23, QXH_IQ2_XS_F = 17, QXH_IQ3_XXS_F = 18, QXH_Q6_K_F = 14, QXH_IQ2R_F = 117, QXH_R4_IQ4_F = 123,
       QXH_R4_IQ3_F = 118, QXH_R8_F = 114 };

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
// barrier; n = 3 + kPhasesPerLayer * layers.
__device__ __forceinline__ size_t trace_n(const Dev& d) { return 3 + kPhasesPerLayer * (size_t)d.dm.layers; }

__device__ __forceinline__ void mark(const Dev& d, unsigned epoch, int k) {
    if (d.trace && blockIdx.x == 0 && threadIdx.x == 0) d.trace[trace_n(d) + (size_t)(epoch + 1) * 8 + k] = global_ns();
}

// `epoch` numbers phases (trace slots); `nsync` counts the barriers actually
// entered, which sets the arrival target.  A CTA waits at most
// kBarrierTimeoutNs (or kSpinLimit polls); then it sets kErrTimeout and
// returns, and every later barrier returns at once when it sees that flag, so
// a broken step ends quickly with an error the host reports.  (Measured on
// B200 against a flag word per CTA polled by several warps, and against a
// counter plus a generation word: this single counter with one polling
// thread per CTA was the fastest, 1.23 us per barrier for 148 CTAs.)
__device__ __forceinline__ void grid_arrive(unsigned* bar, unsigned& epoch, unsigned& nsync, const Dev& d) {
    __syncthreads();
    epoch += 1;
    nsync += 1;
    if (threadIdx.x == 0) {
        if (d.trace) d.trace[9 * trace_n(d) + (size_t)epoch * gridDim.x + blockIdx.x] = global_ns();
        // the CTA's writes are ordered before this release by the bar.sync above
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
    }
}

// Second half of a split barrier: between grid_arrive and grid_wait a CTA may
// only do work that touches its own shared memory (or issues cp.async reads of
// data that no CTA writes in the current phase).
__device__ __forceinline__ void grid_wait(unsigned* bar, unsigned epoch, unsigned nsync, const Dev& d) {
    int* err = d.err;
    if (threadIdx.x == 0) {
        const unsigned target = nsync * gridDim.x;
        const unsigned long long t0 = global_ns();
        for (long long it = 0; ld_acquire(bar) < target; ++it) {
            if ((it & 63) == 63) {
                if (*reinterpret_cast<volatile int*>(err) & kErrTimeout) break;
                if (global_ns() - t0 > kBarrierTimeoutNs || it > kSpinLimit) {
                    atomicOr(err, kErrTimeout);
                    break;
                }
            }
        }
        if (d.trace && blockIdx.x == 0) d.trace[epoch] = global_ns();
    }
    __syncthreads();
}

__device__ __forceinline__ void grid_sync(unsigned* bar, unsigned& epoch, unsigned& nsync, const Dev& d) {
    grid_arrive(bar, epoch, nsync, d);
    grid_wait(bar, epoch, nsync, d);
}

// Advance the barrier numbering without synchronising (a phase that is
// merged into the previous one); the trace records a zero-length phase.
__device__ __forceinline__ void skip_sync(unsigned& epoch, const Dev& d) {
    epoch += 1;
    if (d.trace && blockIdx.x == 0 && threadIdx.x == 0) d.trace[epoch] = global_ns();
}

// Items of a phase owned by this CTA: blockIdx.x, blockIdx.x + G, ...
__device__ __forceinline__ int my_items(int n) {
    return blockIdx.x < (unsigned)n ? (n - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
}
__device__ __forceinline__ int item_id(int k) { return (int)blockIdx.x + k * (int)gridDim.x; }

// Run (tile, block) tasks over `ntile` staged 16-row tiles of row size rb with
// nblk blocks; tile i uses activation xq[xsel(i)].  part[task][16] doubles.
// Bounded wait on an mbarrier phase: gives up (error flag set) after
// kBarrierTimeoutNs, or at once when another wait of the step timed out.
__device__ __forceinline__ bool bounded_mbar_wait(uint64_t* bar, unsigned parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (int it = 0; !mbar_try_wait(bar, parity); ++it) {
        if ((it & 15) == 15 && (*reinterpret_cast<volatile int*>(err) & kErrTimeout)) return false;
        if (global_ns() - t0 > kBarrierTimeoutNs) {
            atomicOr(err, kErrTimeout);
            return false;
        }
    }
    return true;
}

// Tile i of a phase whose tiles each complete on their own mbarrier
// (tbar[i], phase parity bit i of tpar): a warp waits only for the tile of
// its current task, so work starts while later tiles are still landing.
struct TileWait {
    uint64_t* tbar;
    unsigned tpar;
    int* err;
};

// Every tile uses the same activation (one run_tasks instantiation per format).
struct SameXQ {
    XQ x;
    __device__ __forceinline__ XQ operator()(int) const { return x; }
};

template <int FMT, class XSel>
__device__ void run_tasks(const uint8_t* tiles, uint32_t tb, uint32_t rb, int ntile, int nblk, XSel xsel,
                          const uint32_t* K4, const IqTab* T, double* part, TileWait tw = TileWait{nullptr, 0u, nullptr}) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
    const int ntask = ntile * nblk;
    for (int task = warp; task < ntask; task += kMW) {
        const int i = task / nblk, b = task % nblk;
        if (tw.tbar) bounded_mbar_wait(tw.tbar + i, (tw.tpar >> i) & 1u, tw.err);
        const uint8_t* base = tiles + (size_t)i * tb;
        const XQ x = xsel(i);
        Acc acc{};
        if (FMT == QXH_IQ4_XS_F) dot_iq4_xs_mma(base + g * rb, base + (g + 8) * rb, b, b + 1, x, K4, lane, acc);
        if (FMT == QXH_IQ2_XS_F) dot_iq2_xs_mma(base + g * rb, base + (g + 8) * rb, b, b + 1, x, *T, lane, acc);
        if (FMT == QXH_IQ2R_F)
            dot_iq2r_mma(base + g * rb, base + (g + 8) * rb, (int)rb - nblk * kIq2rBlock, b, b + 1, x, lane, acc);
        if (FMT == QXH_R4_IQ4_F) dot_r4_mma<true>(base + g * rb, base + (g + 8) * rb, nblk, b, b + 1, 0, x, K4, lane, acc);
        if (FMT == QXH_R4_IQ3_F) {
            const uint32_t K3[4] = {0x1c140c04u, 0x3e342c24u, 0xe4ecf4fcu, 0xc2ccd4dcu};   // 4..62, -4..-62
            dot_r4_mma<false>(base + g * rb, base + (g + 8) * rb, nblk, b, b + 1, -2, x, K3, lane, acc);
        }
        if (FMT == QXH_IQ3_XXS_F) dot_iq3_xxs_mma(base + g * rb, base + (g + 8) * rb, b, b + 1, x, *T, lane, acc);
        if (FMT == QXH_Q6_K_F) dot_q6_k_mma(base + g * rb, base + (g + 8) * rb, b, b + 1, x, lane, acc);
        if (FMT == QXH_R8_F) dot_r8_mma(base + g * rb, base + (g + 8) * rb, nblk, b, b + 1, x, lane, acc);
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

// ---- weight-tile staging per phase -----------------------------------------
// Each phase's weight tiles move as one bulk-copy group (qx_dev.cuh) into half
// of a double buffer, completing on that group's mbarrier.  All threads call
// the issue and wait functions (the bookkeeping is uniform); warp 1 issues the
// copies (thread 0 spins on the grid barrier meanwhile): lane 0 announces the
// group's bytes, then the lanes take the spans round-robin.
//
// The attention, gate/up and down tiles are in the kernel's own layouts (R4,
// IQ2R: re-laid once at engine creation), whose row sizes keep the 8 rows a
// warp reads at once in different shared-memory banks; a tile of 16 rows is
// one contiguous copy.
enum { kGQkv, kGOproj, kGRouter, kGGateup, kGDown, kGHead0, kGHead1, kGHead2, kGroups };
constexpr int kHeadStages = 3;             // head tiles in flight: a ring of 3 one-tile stages
constexpr int kIssueWarp = 1;

struct Groups {
    uint64_t* bar;       // kGroups mbarriers (static shared memory)
    unsigned parity;     // bit g: parity of group g's next phase
    unsigned pending;    // bit g: issued, not yet waited for
    unsigned stuck;      // bit g: a wait gave up (error already reported)
    uint64_t* tbar;      // kTileBars per-tile mbarriers: gate/up tiles at 0, down tiles at kTileBars / 2
    unsigned tparity;    // bit i: parity of tile barrier i's next phase
    unsigned tused;      // bit i: tile barrier i has been issued on
};
constexpr int kTileBars = 32;

// One copy per tile, each completing on its own tile barrier base + c.
template <class Span>
__device__ __forceinline__ void issue_tiles(Groups& G, int base, int count, Span span) {
    G.tused |= (count >= 32 ? 0xffffffffu : ((1u << count) - 1u)) << base;
    if ((int)(threadIdx.x >> 5) != kIssueWarp) return;
    bulk_fence();
    for (int c = threadIdx.x & 31; c < count; c += 32) {
        uint8_t* dst;
        const void* src;
        uint32_t bytes;
        span(c, dst, src, bytes);
        bulk_group_begin(G.tbar + base + c, bytes);
        bulk_copy(dst, src, bytes, G.tbar + base + c);
    }
}
__device__ __forceinline__ TileWait tile_waits(const Groups& G, int base, const Dev& d) {
    return TileWait{G.tbar + base, G.tparity >> base, d.err};
}
// After the phase's run_tasks: every tile phase has completed (or timed out).
__device__ __forceinline__ void tiles_done(Groups& G, int base, int count) {
    G.tparity ^= (count >= 32 ? 0xffffffffu : ((1u << count) - 1u)) << base;
}

// span(c, dst, src, bytes) describes copy c of `count`.
template <class Span>
__device__ __forceinline__ void issue_group(Groups& G, int g, uint32_t total, int count, Span span) {
    G.pending |= 1u << g;
    if ((int)(threadIdx.x >> 5) != kIssueWarp) return;
    const int lane = threadIdx.x & 31;
    if (lane == 0) bulk_group_begin(G.bar + g, total);
    __syncwarp();
    bulk_fence();
    for (int c = lane; c < count; c += 32) {
        uint8_t* dst;
        const void* src;
        uint32_t bytes;
        span(c, dst, src, bytes);
        bulk_copy(dst, src, bytes, G.bar + g);
    }
}

// Wait for group g's bytes (bounded: after kBarrierTimeoutNs the error flag
// is set and the wait returns; the group is then drained at kernel exit).
__device__ void group_wait(Groups& G, int g, const Dev& d) {
    if (!((G.pending >> g) & 1u)) return;
    const unsigned par = (G.parity >> g) & 1u;
    if (!bounded_mbar_wait(G.bar + g, par, d.err)) G.stuck |= 1u << g;
    if (!((G.stuck >> g) & 1u)) G.parity ^= 1u << g;
    G.pending &= ~(1u << g);
}

// Kernel exit: no copy may still be writing this CTA's shared memory.  A
// tile barrier's last issued phase has parity (tparity bit) ^ 1.
__device__ void group_drain(Groups& G, const Dev& d) {
    for (int g = 0; g < kGroups; ++g) {
        if (((G.pending | G.stuck) >> g) & 1u) {
            const unsigned par = (G.parity >> g) & 1u;
            const unsigned long long t0 = global_ns();
            while (!mbar_try_wait(G.bar + g, par) && global_ns() - t0 < kBarrierTimeoutNs) {
            }
        }
    }
    for (int i = 0; i < kTileBars; ++i) {
        if ((G.tused >> i) & 1u) {
            const unsigned par = ((G.tparity >> i) & 1u) ^ 1u;
            const unsigned long long t0 = global_ns();
            while (!mbar_try_wait(G.tbar + i, par) && global_ns() - t0 < kBarrierTimeoutNs) {
            }
        }
    }
}

// The QKV and router groups also carry the layer's RMSNorm weights (H floats)
// to offset `norm` of the buffer.
__device__ void issue_qkv(const Dev& d, const LayerW& w, uint8_t* buf, uint32_t norm, Groups& G) {
    const int H = d.dm.hidden, Q = d.dm.q_dim(), KV = d.dm.kv_dim();
    const uint32_t rb = (uint32_t)r4_row_bytes(H), tb = (uint32_t)kTileRows * rb;
    const int mine = my_items((Q + 2 * KV) / kTileRows);
    issue_group(G, kGQkv, (uint32_t)H * 4u + (uint32_t)mine * tb, 1 + mine,
                [&](int c, uint8_t*& dst, const void*& src, uint32_t& bytes) {
                    if (c == 0) {
                        dst = buf + norm, src = w.attn_norm, bytes = (uint32_t)H * 4u;
                        return;
                    }
                    const int r0 = item_id(c - 1) * kTileRows;
                    dst = buf + (size_t)(c - 1) * tb;
                    src = r0 < Q ? w.wq_r + (size_t)r0 * rb
                          : r0 < Q + KV ? w.wk_r + (size_t)(r0 - Q) * rb
                                        : w.wv_r + (size_t)(r0 - Q - KV) * rb;
                    bytes = tb;
                });
}

__device__ void issue_oproj(const Dev& d, const LayerW& w, uint8_t* buf, Groups& G) {
    const uint32_t rb = (uint32_t)r4_row_bytes(d.dm.q_dim()), tb = (uint32_t)kTileRows * rb;
    const int mine = my_items(d.dm.hidden / kTileRows);
    issue_group(G, kGOproj, (uint32_t)mine * tb, mine, [&](int c, uint8_t*& dst, const void*& src, uint32_t& bytes) {
        dst = buf + (size_t)c * tb, src = w.wo_r + (size_t)item_id(c) * tb, bytes = tb;
    });
}

__device__ void issue_router(const Dev& d, const LayerW& w, uint8_t* buf, uint32_t norm, Groups& G) {
    const uint32_t rowb = (uint32_t)d.dm.hidden * 4u;
    const int mine = my_items(d.dm.experts);
    issue_group(G, kGRouter, rowb * (uint32_t)(1 + mine), 1 + mine,
                [&](int c, uint8_t*& dst, const void*& src, uint32_t& bytes) {
                    bytes = rowb;
                    if (c == 0) {
                        dst = buf + norm, src = w.ffn_norm;
                        return;
                    }
                    dst = buf + (size_t)(c - 1) * rowb;
                    src = reinterpret_cast<const uint8_t*>(w.router) + (size_t)item_id(c - 1) * rowb;
                });
}

// own[0..n_own): the top-8 slots (rank order) whose expert this GPU computes
// (all 8 on one GPU).
// Gate/up tiles in the IQ2R layout (rb = iq2r_row_bytes(H)); `buf` spans both
// weight buffers.
__device__ void issue_gateup(const Dev& d, const LayerW& w, const int* sel, const int* own, int n_own, uint8_t* buf,
                             uint32_t rb, Groups& G) {
    const int I = d.dm.moe_inter;
    const uint32_t tb = (uint32_t)kTileRows * rb;
    const int tpe = I / kTileRows, mine = my_items(n_own * tpe);
    issue_tiles(G, 0, 2 * mine, [&](int c, uint8_t*& dst, const void*& src, uint32_t& bytes) {
                    const int it = item_id(c >> 1), e = own[it / tpe], i0 = (it % tpe) * kTileRows;
                    const size_t off = (size_t)sel[e] * ((size_t)I * rb) + (size_t)i0 * rb;
                    dst = buf + (size_t)c * tb;
                    src = ((c & 1) ? w.up_r : w.gate_r) + off;
                    bytes = tb;
                });
}

__device__ void issue_down(const Dev& d, const LayerW& w, const int* sel, const int* own, int n_own, uint8_t* buf,
                           Groups& G) {
    const int H = d.dm.hidden, I = d.dm.moe_inter;
    const uint32_t rb = (uint32_t)r4_row_bytes(I), tb = (uint32_t)kTileRows * rb;
    const size_t slice = (size_t)H * rb;
    const int mine = my_items(H / kTileRows);
    issue_tiles(G, kTileBars / 2, mine * n_own, [&](int c, uint8_t*& dst, const void*& src, uint32_t& bytes) {
                    const int k = c / max(n_own, 1), j = c % max(n_own, 1);
                    dst = buf + (size_t)c * tb;
                    src = w.down_r + (size_t)sel[own[j]] * slice + (size_t)item_id(k) * tb;
                    bytes = tb;
                });
}

// ---- expert-parallel exchange ------------------------------------------------
__device__ __forceinline__ float* ep_terms(uint8_t* base, int parity, int slot, int H) {
    return reinterpret_cast<float*>(base) + ((size_t)parity * 8 + slot) * H;
}
__device__ __forceinline__ EpTail* ep_tail(uint8_t* base, int H) {
    return reinterpret_cast<EpTail*>(base + ep_terms_bytes(H));
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread waits until flags[p] >= want for every rank p (wrap-safe), with
// the grid barrier's bounds: on timeout it sets kErrTimeout and returns.
__device__ void ep_wait_flags(const unsigned* flags, int world, unsigned want, int* err) {
    const unsigned long long t0 = global_ns();
    for (int p = 0; p < world; ++p)
        for (long long it = 0; (int)(ld_acquire_sys(flags + p) - want) < 0; ++it)
            if ((it & 63) == 63) {
                if (*reinterpret_cast<volatile int*>(err) & kErrTimeout) return;
                if (global_ns() - t0 > kBarrierTimeoutNs || it > kSpinLimit) {
                    atomicOr(err, kErrTimeout);
                    return;
                }
            }
}

// x + the MoE output of the previous layer (all 8 slots, rank order, float),
// into xs[0..H): the single-GPU down phase's `moe` and residual add.
__device__ void ep_combine(const Dev& d, int prev_layer, float* xs) {
    const int H = d.dm.hidden;
    for (int i = threadIdx.x; i < H; i += kMT) {
        float moe = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) moe += __ldcg(ep_terms(d.ep_local, prev_layer & 1, k, H) + i);   // peer-written: skip L1
        xs[i] = d.x[i] + moe;
    }
    __syncthreads();
}

// CTA-wide: wait for every rank's MoE terms of `prev_layer`: every CTA of
// every rank adds 1 to this rank's layer_cnt[rank] per layer, so after layer
// L of step s the count is (s * layers + L + 1) * grid.
__device__ void ep_wait_layer(const Dev& d, unsigned seqb, int prev_layer) {
    if (threadIdx.x == 0) {
        const unsigned want = ((seqb / 64u) * (unsigned)d.dm.layers + (unsigned)prev_layer + 1u) * gridDim.x;
        ep_wait_flags(ep_tail(d.ep_local, d.dm.hidden)->layer_cnt, d.ep_world, want, d.err);
    }
    __syncthreads();
}


// Head tile `tile` (16 R8 rows) into ring stage `st` (mbarrier kGHead0 + st).
__device__ void issue_head_tile(const Dev& d, int tile, uint8_t* ring, int st, Groups& G) {
    const uint32_t tb = (uint32_t)kTileRows * (uint32_t)r8_row_bytes(d.dm.hidden);
    issue_group(G, kGHead0 + st, tb, 1, [&](int, uint8_t*& dst, const void*& src, uint32_t& bytes) {
        dst = ring + (size_t)st * tb, src = d.head_r + (size_t)tile * tb, bytes = tb;
    });
}

// ---- attention over every CTA ---------------------------------------------
struct AttnSmem {
    double sd[kMW];
    float sf[kMW];
    float kcur[1024];
    float vcur[1024];
    __align__(16) int8_t k8[1024];
    __align__(16) int8_t v8[1024];
};

__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

constexpr int kVChunk = 128;   // positions per context pass
constexpr int kCtxSlices = 4;  // 32-dim slices of a head's context
constexpr int kQdStride = 130; // doubles per staged query head (conflict-free rows)

// Two-phase context: chunks of kRingChunk positions.  Product thread j (the
// threads after warp 0) owns position j / 8 of every chunk, dimensions
// 4 (j % 8) .. + 3: 60 positions x 8 quads = one quad for each of the 480
// threads.  Each copies its own 4 V bytes and the position's scale into a
// ring of kRing slots (cp.async groups, kRing - 1 chunks ahead), so it needs
// no other thread's copies; slot: 480 V words, then 480 scales.  Products go
// to kProdBufs buffers that warp 0 consumes in order.
constexpr int kCtxChunk = 64;
constexpr int kRingChunk = 60;
constexpr int kRing = 5;
constexpr int kProdBufs = 3;
constexpr uint32_t kRingSlot = (kMT - 32) * 8;
constexpr uint32_t kProdBytes = kProdBufs * kRingChunk * 32 * 4;

// Shared-memory staging of the attention phases (the activation region, free
// while attention runs).  Scores: RoPE row, Q/K norm vectors, this CTA's cached
// K rows and scales (rows beyond the capacity are read from global memory).
// Context: softmax weights w_s[ctx], then the V ring.
struct AttnStage {
    double* rope;
    float* qn;
    float* kn;
    float* kscl;
    int8_t* krows;
    int kcap;
    double* w_s;
    uint8_t* ring;
};

// Bytes of the context staging at a given context capacity.
__host__ __device__ constexpr uint32_t attn_ctx_bytes(int ctx) {
    return (uint32_t)((ctx * 8 + 15) & ~15) + kRing * kRingSlot;
}

__device__ __forceinline__ int attn_cpg(const Dev& d) { return (int)gridDim.x / d.dm.kv_heads; }

__device__ AttnStage attn_stage(const Dev& d, int pos, uint8_t* base, uint32_t bytes) {
    AttnStage st;
    const int cpg = attn_cpg(d);
    st.rope = reinterpret_cast<double*>(base);
    st.qn = reinterpret_cast<float*>(base + 1024);
    st.kn = reinterpret_cast<float*>(base + 1536);
    const int krows = (pos + cpg - 1) / cpg;                  // most positions < pos one CTA scores
    const int kfit = ((int)bytes - 2048 - 16) / 132;
    st.kcap = max(0, min(krows, kfit));
    st.kscl = reinterpret_cast<float*>(base + 2048);
    st.krows = reinterpret_cast<int8_t*>(base + 2048 + ((st.kcap * 4 + 15) & ~15));
    st.w_s = reinterpret_cast<double*>(base);
    st.ring = base + ((d.dm.ctx * 8 + 15) & ~15);
    return st;
}

__device__ void issue_attn_scores(const Dev& d, const LayerW& w, int layer, int pos, const AttnStage& st) {
    const int KVH = d.dm.kv_heads, cpg = attn_cpg(d), KV = d.dm.kv_dim(), ctx = d.dm.ctx;
    if ((int)blockIdx.x >= cpg * KVH) return;
    const int g = blockIdx.x / cpg, r = blockIdx.x % cpg;
    stage_copy(reinterpret_cast<uint8_t*>(st.rope), reinterpret_cast<const uint8_t*>(d.rope + (size_t)pos * 128), 1024);
    stage_copy(reinterpret_cast<uint8_t*>(st.qn), reinterpret_cast<const uint8_t*>(w.q_norm), 512);
    stage_copy(reinterpret_cast<uint8_t*>(st.kn), reinterpret_cast<const uint8_t*>(w.k_norm), 512);
    const int rows = r < pos ? min(st.kcap, (pos - r + cpg - 1) / cpg) : 0;
    for (int c = threadIdx.x; c < rows * 8; c += kMT) {
        const int mrow = c >> 3, part = c & 7, t = r + mrow * cpg;
        cp_async16(st.krows + mrow * 128 + part * 16, d.kcache + ((size_t)layer * ctx + t) * KV + g * 128 + part * 16);
    }
    for (int mrow = threadIdx.x; mrow < rows; mrow += kMT)
        cp_async4(st.kscl + mrow, d.kscale + (size_t)layer * ctx + r + mrow * cpg);
}

// This product thread's copies of context chunk c (V slice (g, sl)) into ring
// slot c % kRing; every product thread commits one group per call (an empty
// one past the end), so the group counts agree.
__device__ __forceinline__ void ring_issue(const Dev& d, int layer, int g, int sl, int T, int c, uint8_t* ring) {
    const int j = (int)threadIdx.x - 32, t = c * kRingChunk + (j >> 3);
    if (t < T) {
        uint8_t* slot = ring + (c % kRing) * kRingSlot;
        const size_t row = (size_t)layer * d.dm.ctx + t;
        cp_async4(slot + j * 4, d.vcache + row * d.dm.kv_dim() + g * 128 + sl * 32 + (j & 7) * 4);
        cp_async4(slot + (kMT - 32) * 4 + j * 4, d.vscale + row);
    }
    cp_async_commit();
}

// Context of 32 dims over positions 0..T-1: acc_d = sum_t (float)(w_t * v_t,d)
// in float, t in order (src/qx_format.c:5152-5172).  The products of a
// 64-position chunk are computed by warps 1.. into one half of `prod` while
// warp 0 (lane = dim) adds the previous chunk from the other half.
// vv(t, dd) returns the dequantized V value; prod: 2 * 64 * 32 floats.
// acc + src[0] + src[32] + ... in position order (one lane = one dimension);
// a full chunk's loads go out 20 at a time ahead of the dependent adds.
__device__ __forceinline__ float chunk_sum(const float* src, int n, float acc) {
    if (n == kRingChunk) {
        float v[20];
#pragma unroll
        for (int q = 0; q < kRingChunk; q += 20) {
#pragma unroll
            for (int u = 0; u < 20; ++u) v[u] = src[(q + u) * 32];
#pragma unroll
            for (int u = 0; u < 20; ++u) acc += v[u];
        }
    } else {
#pragma unroll 8
        for (int tt = 0; tt < n; ++tt) acc += src[tt * 32];
    }
    return acc;
}

template <class VV>
__device__ float context_chain(int T, const double* w_s, float* prod, VV vv) {
    const int SW = 32, i = threadIdx.x, nch = (T + kCtxChunk - 1) / kCtxChunk;
    auto products = [&](int c) {
        float* dst = prod + (c & 1) * kCtxChunk * SW;
        const int t0 = c * kCtxChunk, n = min(kCtxChunk, T - t0);
        for (int idx = i - 32; idx < n * SW; idx += kMT - 32) {
            const int t = t0 + idx / SW;
            dst[idx] = (float)(w_s[t] * (double)vv(t, idx % SW));
        }
    };
    float acc = 0.0f;
    if (i >= 32) products(0);
    __syncthreads();
    for (int c = 0; c < nch; ++c) {
        if (i < 32) {
            acc = chunk_sum(prod + (c & 1) * kCtxChunk * SW + i, min(kCtxChunk, T - c * kCtxChunk), acc);
        } else if (c + 1 < nch) {
            products(c + 1);
        }
        __syncthreads();
    }
    return acc;
}

// context_chain over V streamed through the ring: the same products and the
// same position order, with warp 0 and the product threads decoupled.  The
// product threads fill buffer c % kProdBufs with chunk c and arrive on its
// "full" barrier; warp 0 waits there, adds the chunk and, while a later chunk
// will reuse the buffer, arrives on its "empty" barrier, which the product
// threads wait on first.  Arrivals and waits pair up exactly (named barriers
// 2 .. 2 + 2 kProdBufs, all kMT threads).  The caller issued chunks
// 0 .. kRing - 2 with ring_issue.
__device__ float context_ring(const Dev& d, int layer, int g, int sl, int T, const double* w_s, float* prod,
                              uint8_t* ring) {
    static_assert(kRingChunk * 8 == kMT - 32, "one quad per product thread");
    const int i = threadIdx.x, nch = (T + kRingChunk - 1) / kRingChunk;
    float acc = 0.0f;
    if (i >= 32) {
        const int j = i - 32, tt = j >> 3, q4 = (j & 7) * 4;
        for (int c = 0; c < nch; ++c) {
            const int b = c % kProdBufs, t = c * kRingChunk + tt;
            ring_issue(d, layer, g, sl, T, c + kRing - 1, ring);
            cp_async_wait<kRing - 1>();
            if (c >= kProdBufs) named_sync(2 + kProdBufs + b, kMT);
            if (t < T) {
                const uint8_t* slot = ring + (c % kRing) * kRingSlot;
                const uint32_t raw = *reinterpret_cast<const uint32_t*>(slot + j * 4);
                const float vs = *reinterpret_cast<const float*>(slot + (kMT - 32) * 4 + j * 4);
                const double w = w_s[t];
                float4 o;
                o.x = (float)(w * (double)(i8_to_f32((int)(raw << 24) >> 24) * vs));
                o.y = (float)(w * (double)(i8_to_f32((int)(raw << 16) >> 24) * vs));
                o.z = (float)(w * (double)(i8_to_f32((int)(raw << 8) >> 24) * vs));
                o.w = (float)(w * (double)(i8_to_f32((int)raw >> 24) * vs));
                *reinterpret_cast<float4*>(prod + b * kRingChunk * 32 + tt * 32 + q4) = o;
            }
            named_arrive(2 + b, kMT);
        }
    } else {
        for (int c = 0; c < nch; ++c) {
            const int b = c % kProdBufs;
            named_sync(2 + b, kMT);
            acc = chunk_sum(prod + b * kRingChunk * 32 + i, min(kRingChunk, T - c * kRingChunk), acc);
            if (c + kProdBufs < nch) named_arrive(2 + kProdBufs + b, kMT);
        }
    }
    __syncthreads();
    return acc;
}

// score_row of one key row against the G query heads of its KV group (rows
// kQdStride doubles apart), stored to out[h * stride]: each head's sum in
// dimension order exactly as score_row adds it; the key values are widened
// once for all G heads.
template <int G>
__device__ __forceinline__ void score_rows_group(const double* qd, const int8_t* kp, float ks, double sqrt_d,
                                                 double* out, int stride) {
    double s[G];
#pragma unroll
    for (int h = 0; h < G; ++h) s[h] = 0.0;
#pragma unroll 1
    for (int j = 0; j < 128; j += 8) {
        const int2 raw = *reinterpret_cast<const int2*>(kp + j);
        const int8_t* kb = reinterpret_cast<const int8_t*>(&raw);
        double kd[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) kd[u] = (double)(i8_to_f32(kb[u]) * ks);
#pragma unroll
        for (int h = 0; h < G; ++h)
#pragma unroll
            for (int u = 0; u < 8; u += 2) {
                const double2 q = *reinterpret_cast<const double2*>(qd + h * kQdStride + j + u);
                s[h] = fma(q.x, kd[u], s[h]);
                s[h] = fma(q.y, kd[u + 1], s[h]);
            }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const double v = s[h] / sqrt_d;
        out[(size_t)h * stride] = isfinite(v) ? v : 0.0;
    }
}

// Scores.  The CTAs form kv_heads groups of G/kv_heads; group g serves the
// query heads of KV head g, CTA r of the group positions r, r + cpg, ...;
// thread i scores query head i % group at one of those positions.  Every CTA
// of a group repeats the per-head Q/K RMSNorm + RoPE of its heads and the INT8
// quantization of the current K/V (one scale per token over all KV values,
// src/qx_format.c:4449-4463); CTA 0 appends them to the cache.  qd: shared
// scratch of group * kQdStride doubles.  The staged group must be the second
// most recent cp.async group.
__device__ void attn_scores(const Dev& d, const LayerW& w, int layer, int pos, AttnSmem& S, double* qd,
                            const AttnStage& st, unsigned epoch) {
    const int D = 128, KVH = d.dm.kv_heads, group = d.dm.q_heads / KVH;
    const int Q = d.dm.q_dim(), KV = d.dm.kv_dim(), ctx = d.dm.ctx, i = threadIdx.x;
    const int warp = i >> 5, lane = i & 31, cpg = attn_cpg(d);
    const bool active = (int)blockIdx.x < cpg * KVH;
    const int g = blockIdx.x / max(cpg, 1), r = blockIdx.x % max(cpg, 1);
    float* qf = reinterpret_cast<float*>(qd);             // group * 128 floats, widened below
    if (active) {
        for (int j = i; j < KV; j += kMT) {
            S.kcur[j] = d.qkv[Q + j];
            S.vcur[j] = d.qkv[Q + KV + j];
        }
        for (int j = i; j < group * D; j += kMT) qf[j] = d.qkv[(size_t)g * group * D + j];
    }
    __syncthreads();
    mark(d, epoch, 3);
    // the staging copies start once the phase's inputs are in, so they do not
    // queue ahead of those loads
    issue_attn_scores(d, w, layer, pos, st);
    cp_async_commit();
    if (!active) return;
    cp_async_wait<0>();
    __syncthreads();
    mark(d, epoch, 4);
    for (int hh = warp; hh < KVH + group; hh += kMW) {
        if (hh < KVH) warp_norm_rope(S.kcur + hh * D, st.kn, st.rope, lane);
        else warp_norm_rope(qf + (hh - KVH) * D, st.qn, st.rope, lane);
    }
    __syncthreads();
    mark(d, epoch, 5);
    float ka = 0.f, va = 0.f;
    for (int j = i; j < KV; j += kMT) {
        ka = fmaxf(ka, isfinite(S.kcur[j]) ? fabsf(S.kcur[j]) : 0.f);
        va = fmaxf(va, isfinite(S.vcur[j]) ? fabsf(S.vcur[j]) : 0.f);
    }
    // widen the query heads (exact) into padded double rows; every float is
    // read into registers before the first double is written over them
    float qreg[8];
    const int nq = group * D;
#pragma unroll
    for (int k = 0; k < 8; ++k) qreg[k] = (i + k * kMT < nq) ? qf[i + k * kMT] : 0.f;
    ka = block_max_f(ka, S.sf);
    va = block_max_f(va, S.sf);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int j = i + k * kMT;
        if (j < nq) qd[(j / D) * kQdStride + j % D] = (double)qreg[k];
    }
    mark(d, epoch, 0);
    const float ksc = ka > 0.f ? ka / 127.0f : 1.0f, vsc = va > 0.f ? va / 127.0f : 1.0f;
    const float krc = 1.0f / ksc, vrc = 1.0f / vsc;   // one division each; divf_by per value
    for (int j = i; j < KV; j += kMT) {
        const float kq = ksc >= FLT_MIN ? divf_by(S.kcur[j], ksc, krc) : S.kcur[j] / ksc;
        const float vq = vsc >= FLT_MIN ? divf_by(S.vcur[j], vsc, vrc) : S.vcur[j] / vsc;
        const int qk = isfinite(S.kcur[j]) ? (int)lrintf(kq) : 0;
        const int qq = isfinite(S.vcur[j]) ? (int)lrintf(vq) : 0;
        S.k8[j] = (int8_t)max(-127, min(127, qk));
        S.v8[j] = (int8_t)max(-127, min(127, qq));
    }
    __syncthreads();
    const size_t slot = (size_t)layer * ctx + pos;
    if (blockIdx.x == 0) {
        for (int j = i; j < KV; j += kMT) {
            d.kcache[slot * KV + j] = S.k8[j];
            d.vcache[slot * KV + j] = S.v8[j];
        }
        if (i == 0) { d.kscale[slot] = ksc; d.vscale[slot] = vsc; }
    }
    mark(d, epoch, 1);
    const int T = pos + 1, per = kMT / group, hj = i % group;
    const double sqrt_d = sqrt((double)D);
    auto key_row = [&](int mrow, int t, const int8_t*& kp, float& ks) {
        const size_t stt = (size_t)layer * ctx + t;
        kp = t == pos ? S.k8 + g * D : mrow < st.kcap ? st.krows + mrow * 128 : d.kcache + stt * KV + g * D;
        ks = t == pos ? ksc : mrow < st.kcap ? st.kscl[mrow] : d.kscale[stt];
    };
    if (group % 2 == 0) {                 // thread: one position, two heads (the key widened once for both)
        const int sub = group / 2, h0 = 2 * (i % sub);
        double* out = d.attn_scores + (size_t)(g * group + h0) * ctx;
        for (int mrow = i / sub; r + mrow * cpg < T; mrow += kMT / sub) {
            const int t = r + mrow * cpg;
            const int8_t* kp;
            float ks;
            key_row(mrow, t, kp, ks);
            score_rows_group<2>(qd + h0 * kQdStride, kp, ks, sqrt_d, out + t, ctx);
        }
        __syncthreads();
        mark(d, epoch, 2);
        return;
    }
    const double* q = qd + hj * kQdStride;
    double* out = d.attn_scores + (size_t)(g * group + hj) * ctx;
    for (int mrow = i / group; r + mrow * cpg < T; mrow += per) {
        const int t = r + mrow * cpg;
        const size_t stt = (size_t)layer * ctx + t;
        // pick the row first so the lanes of a warp run one chain together
        const int8_t* kp = t == pos ? S.k8 + g * D : mrow < st.kcap ? st.krows + mrow * 128 : d.kcache + stt * KV + g * D;
        const float ks = t == pos ? ksc : mrow < st.kcap ? st.kscl[mrow] : d.kscale[stt];
        out[t] = score_row(q, kp, ks, sqrt_d);
    }
    __syncthreads();
    mark(d, epoch, 2);
}

// Softmax and context.  Item (h, slice) = 32 context dims of query head h:
// the head's softmax in double (max, exp, fixed-order sum, divide), then the
// products (float)(w_t * v_t) by every thread into prod, then one warp adds
// them per dimension in position order in float (src/qx_format.c:5152-5172).
// prod: kVChunk * 32 floats of shared scratch.  The staged V group must be the
// most recent cp.async group.
__device__ void attn_context(const Dev& d, int layer, int pos, AttnSmem& S, float* prod, const AttnStage& st,
                             unsigned epoch) {
    const int D = 128, SW = D / kCtxSlices, group = d.dm.q_heads / d.dm.kv_heads;
    const int KV = d.dm.kv_dim(), ctx = d.dm.ctx, T = pos + 1, i = threadIdx.x;
    double* w_s = st.w_s;
    for (int item = blockIdx.x; item < d.dm.q_heads * kCtxSlices; item += gridDim.x) {
        const int h = item / kCtxSlices, sl = item % kCtxSlices, g = h / group;
        if (i >= 32)                       // V streams from here
            for (int c = 0; c < kRing - 1; ++c) ring_issue(d, layer, g, sl, T, c, st.ring);
        const double* sc = d.attn_scores + (size_t)h * ctx;
        double mloc = -1.0e300;
        for (int t = i; t < T; t += kMT) {
            const double s = sc[t];
            w_s[t] = s;
            mloc = fmax(mloc, s);
        }
        const double mx = block_max_d(mloc, S.sd);
        mark(d, epoch, 3);
        for (int t = i; t < T; t += kMT) w_s[t] = exp(w_s[t] - mx);
        double den = fixed_order_sum(w_s, T, S.sd);
        mark(d, epoch, 4);
        if (!isfinite(den) || den <= 0.0) den = 1.0;
        for (int t = i; t < T; t += kMT) w_s[t] = w_s[t] / den;
        __syncthreads();
        mark(d, epoch, 5);
        mark(d, epoch, 0);
        const float acc = context_ring(d, layer, g, sl, T, w_s, prod, st.ring);
        if (i < SW) d.ctxv[h * D + sl * SW + i] = acc;
        mark(d, epoch, 1);
        __syncthreads();
    }
}

// ---- single-phase attention (history fits in shared memory) ----------------
// Item (h, slice) computes every score of query head h itself (the 4 slice
// CTAs of a head repeat the same exact arithmetic), then its 32 context dims;
// no scores round trip through global memory and one grid barrier fewer.
// Staged at the end of the QKV phase into the activation region: RoPE row,
// Q/K norm vectors, K rows of the item's KV head (16-byte chunk j of row t at
// chunk j ^ (t & 7), so lanes scoring consecutive positions read different
// banks), K scales, the item's 32-byte V slices and V scales.
struct FusedStage {
    double* rope;
    float* qn;
    float* kn;
    double* qd;
    double* w_s;
    float* kscl;
    float* vscl;
    int8_t* krows;
    int8_t* vrows;
};

constexpr uint32_t kFusedFixed = 1024 + 512 + 512 + 1040;        // rope, norms, qd (bytes, 16-aligned)
constexpr uint32_t kFusedPerPos = 8 + 4 + 4 + 128 + 32;          // w_s, scales, K row, V slice

__device__ __forceinline__ int fused_cap(uint32_t bytes) {
    return bytes > kFusedFixed + 64 ? min(1024, (int)((bytes - kFusedFixed - 64) / kFusedPerPos)) : 0;
}

__device__ FusedStage fused_stage(uint8_t* base, uint32_t bytes) {
    const int cap = fused_cap(bytes);
    FusedStage f;
    f.rope = reinterpret_cast<double*>(base);
    f.qn = reinterpret_cast<float*>(base + 1024);
    f.kn = reinterpret_cast<float*>(base + 1536);
    f.qd = reinterpret_cast<double*>(base + 2048);
    uint8_t* p = base + kFusedFixed;
    f.w_s = reinterpret_cast<double*>(p);
    p += ((size_t)cap * 8 + 15) & ~(size_t)15;
    f.kscl = reinterpret_cast<float*>(p);
    p += ((size_t)cap * 4 + 15) & ~(size_t)15;
    f.vscl = reinterpret_cast<float*>(p);
    p += ((size_t)cap * 4 + 15) & ~(size_t)15;
    f.krows = reinterpret_cast<int8_t*>(p);
    p += (size_t)cap * 128;
    f.vrows = reinterpret_cast<int8_t*>(p);
    return f;
}

// Copies for the fused phase of `layer` at `pos` (history rows t < pos).
__device__ void issue_attn_fused(const Dev& d, const LayerW& w, int layer, int pos, const FusedStage& f) {
    const int D = 128, SW = D / kCtxSlices, group = d.dm.q_heads / d.dm.kv_heads;
    const int KV = d.dm.kv_dim(), ctx = d.dm.ctx, item = blockIdx.x;
    if (item >= d.dm.q_heads * kCtxSlices) return;
    const int h = item / kCtxSlices, sl = item % kCtxSlices, g = h / group;
    stage_copy(reinterpret_cast<uint8_t*>(f.rope), reinterpret_cast<const uint8_t*>(d.rope + (size_t)pos * 128), 1024);
    stage_copy(reinterpret_cast<uint8_t*>(f.qn), reinterpret_cast<const uint8_t*>(w.q_norm), 512);
    stage_copy(reinterpret_cast<uint8_t*>(f.kn), reinterpret_cast<const uint8_t*>(w.k_norm), 512);
    const int8_t* kb = d.kcache + (size_t)layer * ctx * KV + g * D;
    const int8_t* vb = d.vcache + (size_t)layer * ctx * KV + g * D + sl * SW;
    for (int c = threadIdx.x; c < pos * 8; c += kMT) {
        const int t = c >> 3, j = c & 7;
        cp_async16(f.krows + t * 128 + 16 * (j ^ (t & 7)), kb + (size_t)t * KV + 16 * j);
    }
    for (int c = threadIdx.x; c < pos * 2; c += kMT)
        cp_async16(f.vrows + (c >> 1) * SW + (c & 1) * 16, vb + (size_t)(c >> 1) * KV + (c & 1) * 16);
    for (int t = threadIdx.x; t < pos; t += kMT) {
        cp_async4(f.kscl + t, d.kscale + (size_t)layer * ctx + t);
        cp_async4(f.vscl + t, d.vscale + (size_t)layer * ctx + t);
    }
}

// The fused phase.  The staged group must be the second most recent
// cp.async group (the router rows follow it).
__device__ void attn_fused(const Dev& d, int layer, int pos, AttnSmem& S, const FusedStage& f, float* prod,
                           unsigned epoch) {
    const int D = 128, SW = D / kCtxSlices, KVH = d.dm.kv_heads, group = d.dm.q_heads / KVH;
    const int Q = d.dm.q_dim(), KV = d.dm.kv_dim(), ctx = d.dm.ctx, i = threadIdx.x;
    const int warp = i >> 5, lane = i & 31, item = blockIdx.x, T = pos + 1;
    const bool active = item < d.dm.q_heads * kCtxSlices;
    const int h = item / kCtxSlices, sl = item % kCtxSlices, g = h / group;
    float* qf = reinterpret_cast<float*>(prod);                   // 128 floats of scratch
    if (active) {
        for (int j = i; j < KV; j += kMT) {
            S.kcur[j] = d.qkv[Q + j];
            S.vcur[j] = d.qkv[Q + KV + j];
        }
        if (i < D) qf[i] = d.qkv[h * D + i];
    }
    __syncthreads();
    if (!active) return;
    cp_async_wait<0>();
    __syncthreads();
    mark(d, epoch, 1);
    // one warp per head: K heads (RMSNorm + RoPE, then max |k|), V heads
    // (max |v|), the query head (RMSNorm + RoPE, widened to double); the
    // row maxima (non-finite values count as 0) meet in S.sf[0..8) / [8..16)
    for (int hh = warp; hh < 2 * KVH + 1; hh += kMW) {
        if (hh < 2 * KVH) {
            float* v = hh < KVH ? S.kcur + hh * D : S.vcur + (hh - KVH) * D;
            if (hh < KVH) warp_norm_rope(v, f.kn, f.rope, lane);
            float mx = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float e = v[lane + 32 * k];            // the lane's own dims (written by it above)
                mx = fmaxf(mx, isfinite(e) ? fabsf(e) : 0.f);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0) S.sf[hh < KVH ? hh : 8 + hh - KVH] = mx;
        } else {
            warp_norm_rope(qf, f.qn, f.rope, lane);
#pragma unroll
            for (int k = 0; k < 4; ++k) f.qd[lane + 32 * k] = (double)qf[lane + 32 * k];
        }
    }
    __syncthreads();
    float ka = 0.f, va = 0.f;
    for (int k = 0; k < KVH; ++k) {
        ka = fmaxf(ka, S.sf[k]);
        va = fmaxf(va, S.sf[8 + k]);
    }
    const float ksc = ka > 0.f ? ka / 127.0f : 1.0f, vsc = va > 0.f ? va / 127.0f : 1.0f;
    const float krc = 1.0f / ksc, vrc = 1.0f / vsc;   // one division each; divf_by per value
    for (int j = i; j < KV; j += kMT) {
        const float kq = ksc >= FLT_MIN ? divf_by(S.kcur[j], ksc, krc) : S.kcur[j] / ksc;
        const float vq = vsc >= FLT_MIN ? divf_by(S.vcur[j], vsc, vrc) : S.vcur[j] / vsc;
        const int qk = isfinite(S.kcur[j]) ? (int)lrintf(kq) : 0;
        const int qq = isfinite(S.vcur[j]) ? (int)lrintf(vq) : 0;
        S.k8[j] = (int8_t)max(-127, min(127, qk));
        S.v8[j] = (int8_t)max(-127, min(127, qq));
    }
    __syncthreads();
    if (item == 0) {
        const size_t slot = (size_t)layer * ctx + pos;
        for (int j = i; j < KV; j += kMT) {
            d.kcache[slot * KV + j] = S.k8[j];
            d.vcache[slot * KV + j] = S.v8[j];
        }
        if (i == 0) { d.kscale[slot] = ksc; d.vscale[slot] = vsc; }
    }
    mark(d, epoch, 3);
    // scores of every position (the current one from the fresh INT8 row)
    const double sqrt_d = sqrt((double)D);
    double mloc = -1.0e300;
    for (int t = i; t < T; t += kMT) {
        const bool cur = t == pos;
        const double s = score_row_sw(f.qd, cur ? S.k8 + g * D : f.krows + t * 128, cur ? 0 : (t & 7),
                                      cur ? ksc : f.kscl[t], sqrt_d);
        f.w_s[t] = s;
        mloc = fmax(mloc, s);
    }
    const double mx = block_max_d(mloc, S.sd);
    mark(d, epoch, 4);
    for (int t = i; t < T; t += kMT) f.w_s[t] = exp(f.w_s[t] - mx);
    double den = fixed_order_sum(f.w_s, T, S.sd);
    if (!isfinite(den) || den <= 0.0) den = 1.0;
    for (int t = i; t < T; t += kMT) f.w_s[t] = f.w_s[t] / den;
    __syncthreads();
    const float acc = context_chain(T, f.w_s, prod, [&](int t, int dd) {
        return t == pos ? i8_to_f32(S.v8[g * D + sl * SW + dd]) * vsc : i8_to_f32(f.vrows[t * SW + dd]) * f.vscl[t];
    });
    if (i < SW) d.ctxv[h * D + sl * SW + i] = acc;
    __syncthreads();
    mark(d, epoch, 6);
}

// Router softmax + top-8 over the logits in global memory (every CTA; the
// result is identical everywhere).  The reference picks the 8 largest
// probabilities one at a time, ties to the lower expert index
// (src/qx_format.c:5272-5285); the same list comes from ranking every expert
// by (probability descending, index ascending).
//
// Softmax: thread e < E holds expert e; the first ceil(E/32) warps reduce
// with shuffles and meet at a named barrier, in the same order in every CTA.
// Probabilities are >= 0, so their bit patterns order like the values.  The
// fast ranks compare only the upper 32 bits and count strictly larger keys;
// equal upper halves share a rank, which leaves one of the eight slots empty
// or doubly filled, and then the exact 64-bit (key, index) ranking runs.  A
// NaN makes the weight sum NaN, reported as an error in top8_weights.
__device__ void top8_select(const Dev& d, int* sel, double* wsel, long long* keys, double* red, int* cnt) {
    const int E = d.dm.experts, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int sw = (E + 31) >> 5, st = sw * 32;       // softmax warps / threads
    uint32_t* hk = reinterpret_cast<uint32_t*>(keys + kMT / 2);   // upper halves, after the full keys
    if (t < st) {
        const double lg = t < E ? __ldcg(d.router_logits + t) : -1.0e300;
        double m = lg;
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) red[warp] = m;
        named_sync(1, st);
        m = red[0];
        for (int k = 1; k < sw; ++k) m = fmax(m, red[k]);
        const double ex = t < E ? exp(lg - m) : 0.0;
        double s = ex;
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) red[8 + warp] = s;
        named_sync(1, st);
        double den = red[8];
        for (int k = 1; k < sw; ++k) den += red[8 + k];
        if (t < E) {
            const long long key = __double_as_longlong(ex / den);
            keys[t] = key;
            hk[t] = (uint32_t)(key >> 32);
        }
        if (t == 0) cnt[0] = cnt[1] = 0;
    }
    __syncthreads();
    // P adjacent threads per expert, each over a contiguous chunk of candidates
    const int P = E <= kMT / 4 ? 4 : (E <= kMT / 2 ? 2 : 1);
    const int e = t / P, q = t % P, chunk = (E + P - 1) / P;
    const uint32_t he = e < E ? hk[e] : 0u;
    int rank = 0;
    if (e < E) {
        if (E == 128) {
            const uint4* kp = reinterpret_cast<const uint4*>(hk + 32 * q);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 v = kp[(i + q) & 7];      // rotated start: the quad's loads hit different banks
                rank += (v.x > he) + (v.y > he) + (v.z > he) + (v.w > he);
            }
        } else {
            for (int u = q * chunk; u < min(E, (q + 1) * chunk); ++u) rank += hk[u] > he;
        }
    }
    if (P >= 2) rank += __shfl_xor_sync(0xffffffffu, rank, 1);
    if (P >= 4) rank += __shfl_xor_sync(0xffffffffu, rank, 2);
    if (e < E && q == 0 && rank < 8) {
        sel[rank] = e;
        wsel[rank] = __longlong_as_double(keys[e]);
        atomicAdd(cnt, 1);
        atomicOr(cnt + 1, 1 << rank);
    }
    __syncthreads();
    if (cnt[0] != 8 || cnt[1] != 0xff) {          // near-equal probabilities at the top: exact ranks
        const long long ke = e < E ? keys[e] : 0;
        rank = 0;
        if (e < E)
            for (int u = q; u < E; u += P) {
                const long long k2 = keys[u];
                rank += (k2 > ke) | ((k2 == ke) & (u < e));
            }
        if (P >= 2) rank += __shfl_xor_sync(0xffffffffu, rank, 1);
        if (P >= 4) rank += __shfl_xor_sync(0xffffffffu, rank, 2);
        if (e < E && q == 0 && rank < 8) {
            sel[rank] = e;
            wsel[rank] = __longlong_as_double(ke);
        }
        __syncthreads();
    }
}

// Normalise the 8 selected probabilities (rank-order sum, :5287); CTA 0
// records the selection.  Readers of wsel sync before they read it.
__device__ void top8_weights(const Dev& d, int layer, const int* sel, double* wsel) {
    const int t = threadIdx.x;
    if (t < 8) {
        double sum = 0.0;
        for (int k = 0; k < 8; ++k) sum += wsel[k];
        if (t == 0 && (!(sum > 0.0) || !isfinite(sum))) atomicOr(d.err, kErrRouter);
        const double wk = wsel[t] / sum;
        __syncwarp(0xffu);
        wsel[t] = wk;
        if (blockIdx.x == 0) {
            d.sel[layer * 8 + t] = sel[t];
            d.selw[layer * 8 + t] = (float)wk;
        }
    }
}

}  // namespace

__global__ void __launch_bounds__(kMT, 1) k_decode_step(Dev d, const LayerW* __restrict__ layers, MegaLayout L) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kMW];
    __shared__ __align__(16) double probs[kMT];
    __shared__ int top_cnt[2];
    __shared__ uint64_t gbar[kGroups];
    __shared__ uint64_t tbar_s[kTileBars];
    __shared__ double wsel[8];
    __shared__ int sel[8];
    __shared__ int own[8];
    __shared__ int n_own_s;
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
    unsigned epoch = 0, nsync = 0;
    unsigned* bar = d.counters + kCntBarrier;
    const int tok = *d.token, pos = *d.pos;
    if (tok < 0 || tok >= m.vocab || pos < 0 || pos >= m.ctx) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(d.err, tok < 0 || tok >= m.vocab ? kErrToken : kErrPosition);
        return;   // uniform across the grid: no barrier is entered
    }
    if (d.trace && blockIdx.x == 0 && threadIdx.x == 0) d.trace[0] = global_ns();
    // expert parallelism: this rank's experts [e0, e1) and head groups [hg0, hg1)
    // (qx_cuda_ep_partition); flags of this step are seqb + layer + 1 (MoE
    // terms) and seqb + 63 (head)
    const bool ep = d.ep_world > 1;
    const unsigned seqb = ep ? *d.ep_seq * 64u : 0u;
    const int e0 = d.ep_e0, e1 = d.ep_e1, hg0 = d.ep_hg0, hg1 = d.ep_hg1;
    uint32_t K4[4];
    load_kv_regs(d.tables, K4);
    load_iq_tables(T, d.tables, true, true);
    // attention in one phase when the whole history of a head fits in shared memory
    const bool fused = pos + 1 <= fused_cap(L.sb - L.xb);
    const FusedStage fz = fused_stage(smem + L.xb, L.sb - L.xb);
    int qb = 0;
    // Weight groups: each is issued once its buffer is free and early enough
    // to land before use, but not ahead of the activation reads that start a
    // phase (the fills share the SM's L2 path with them): down(l) at the end
    // of gate/up(l), QKV(l+1) in down(l) after its input is read, O-proj(l) in
    // QKV(l) after the norm, router(l) at the end of QKV(l), gate/up(l) after
    // top-8.
    Groups G{gbar, 0u, 0u, 0u, tbar_s, 0u, 0u};
    if (threadIdx.x == 0) {
        for (int g = 0; g < kGroups; ++g) mbar_init(gbar + g, 1);
        for (int i = 0; i < kTileBars; ++i) mbar_init(tbar_s + i, 1);
        mbar_init_fence();
    }
    __syncthreads();
    issue_qkv(d, layers[0], buf[qb], L.norm, G);
    // embedding (every CTA into its own xs; CTA 0 also writes the residual)
    {
        const int nblk = H / 256;
        const uint8_t* row = d.tok_embd + (size_t)tok * (size_t)(nblk * 144);
        const int t = threadIdx.x & 255, c = t >> 6, l = t & 63;
        for (int b = threadIdx.x >> 8; b < nblk; b += kMT / 256) {
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
    // The residual rows this CTA updates in the O-projection and down
    // epilogues (the same 16-row items in both phases): thread r keeps row
    // item_id(0) * 16 + r in a register, so the epilogues need no L2 read.
    const int own_rows = my_items(H / kTileRows) * kTileRows;
    float xown = threadIdx.x < own_rows ? xs[item_id(threadIdx.x / kTileRows) * kTileRows + threadIdx.x % kTileRows] : 0.0f;
    for (int layer = 0; layer < m.layers; ++layer) {
        const LayerW& w = layers[layer];
        // ---------------- QKV (weights in buf[qb]) ----------------
        {
            group_wait(G, kGQkv, d);             // this phase's tiles and norm vector
            if (layer > 0 && ep) {
                ep_wait_layer(d, seqb, layer - 1);
                ep_combine(d, layer - 1, xs);
            } else if (layer > 0) {
                copy_to_smem(d.x, xs, H);
            } else {
                __syncthreads();
            }
            // attention RMSNorm of xs in place
            const float* nw = reinterpret_cast<const float*>(buf[qb] + L.norm);
            const double ss = sum_sq_fixed(xs, H, scratch);
            const double rms = sqrt(ss / (double)H + 1.0e-6), rinv = 1.0 / rms;
            if (isfinite(rms))
                for (int i = threadIdx.x; i < H; i += kMT) xs[i] = (float)div_by((double)xs[i], rms, rinv) * nw[i];
            else
                for (int i = threadIdx.x; i < H; i += kMT) xs[i] = (float)((double)xs[i] / rms) * nw[i];
            __syncthreads();
            mark(d, epoch, 2);
            issue_oproj(d, w, buf[1 - qb], G);  // the previous layer's down tiles are consumed
            build_xq(xs, H, xb, sb);
            __syncthreads();
            mark(d, epoch, 3);
            const uint32_t rb = (uint32_t)r4_row_bytes(H), tb = (uint32_t)kTileRows * rb;
            const int mine = my_items((Q + 2 * KV) / kTileRows), nblk = H / 256;
            run_tasks<QXH_R4_IQ4_F>(buf[qb], tb, rb, mine, nblk, SameXQ{XQ{xb, sb}}, K4, T, part);
            mark(d, epoch, 4);
            for (int r = threadIdx.x; r < mine * kTileRows; r += kMT)
                d.qkv[item_id(r / kTileRows) * kTileRows + r % kTileRows] =
                    finite_or_zero_d(tile_row(part, r / kTileRows, nblk, r % kTileRows));
            grid_arrive(bar, epoch, nsync, d);
            if (fused) issue_attn_fused(d, w, layer, pos, fz);   // the activation region is free again
            cp_async_commit();
            issue_router(d, w, buf[qb], L.norm, G);               // the QKV tiles are consumed
            grid_wait(bar, epoch, nsync, d);
        }
        // ---------------- attention (CTAs 0..Hq-1) ----------------
        if (fused) {
            attn_fused(d, layer, pos, attn, fz, reinterpret_cast<float*>(smem + L.xs), epoch);
            skip_sync(epoch, d);
            grid_sync(bar, epoch, nsync, d);
        } else {
            const AttnStage stg = attn_stage(d, pos, smem + L.xb, L.sb - L.xb);
            attn_scores(d, w, layer, pos, attn, reinterpret_cast<double*>(smem + L.xs), stg, epoch);
            grid_sync(bar, epoch, nsync, d);
            attn_context(d, layer, pos, attn, reinterpret_cast<float*>(smem + L.xs), stg, epoch);
            grid_sync(bar, epoch, nsync, d);
        }
        // ---------------- O projection (weights in buf[1-qb]) ----------------
        {
            copy_to_smem(d.ctxv, xs, Q);
            build_xq(xs, Q, xb, sb);
            __syncthreads();
            mark(d, epoch, 1);
            group_wait(G, kGOproj, d);
            const uint32_t rb = (uint32_t)r4_row_bytes(Q), tb = (uint32_t)kTileRows * rb;
            const int mine = my_items(H / kTileRows), nblk = Q / 256;
            run_tasks<QXH_R4_IQ4_F>(buf[1 - qb], tb, rb, mine, nblk, SameXQ{XQ{xb, sb}}, K4, T, part);
            mark(d, epoch, 3);
            for (int r = threadIdx.x; r < mine * kTileRows; r += kMT) {
                const int row = item_id(r / kTileRows) * kTileRows + r % kTileRows;
                const float o = finite_or_zero_d(tile_row(part, r / kTileRows, nblk, r % kTileRows));
                d.attn_out[row] = o;
                float xr = xown;                 // == d.x[row]
                if (ep && layer > 0) {           // the previous layer's MoE add, as ep_combine does it
                    float moe = 0.0f;
#pragma unroll
                    for (int k = 0; k < 8; ++k) moe += __ldcg(ep_terms(d.ep_local, (layer - 1) & 1, k, H) + row);
                    xr = xr + moe;
                }
                xown = xr + o;
                d.x[row] = xown;
            }
            grid_sync(bar, epoch, nsync, d);
        }
        // ---------------- router (weights in buf[qb]) ----------------
        {
            group_wait(G, kGRouter, d);          // router rows and norm vector
            copy_to_smem(d.x, xs, H);
            const float* nw = reinterpret_cast<const float*>(buf[qb] + L.norm);
            const double ss = sum_sq_fixed(xs, H, scratch);
            const double rms = sqrt(ss / (double)H + 1.0e-6), rinv = 1.0 / rms;
            if (isfinite(rms))
                for (int i = threadIdx.x; i < H; i += kMT) xs[i] = (float)div_by((double)xs[i], rms, rinv) * nw[i];
            else
                for (int i = threadIdx.x; i < H; i += kMT) xs[i] = (float)((double)xs[i] / rms) * nw[i];
            __syncthreads();
            if (blockIdx.x == 0)
                for (int i = threadIdx.x; i < H; i += kMT) d.xn[i] = xs[i];
            __syncthreads();
            mark(d, epoch, 2);
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
            mark(d, epoch, 3);
            grid_arrive(bar, epoch, nsync, d);
            build_xq(xs, H, xb, sb);   // the FFN input for gate/up, while the grid gathers
            grid_wait(bar, epoch, nsync, d);
        }
        // ---------------- top-8 + gate/up (weights in buf[1-qb]) ----------------
        {
            top8_select(d, sel, wsel, reinterpret_cast<long long*>(probs), scratch, top_cnt);
            mark(d, epoch, 0);
            if (threadIdx.x < 32) {              // the slots whose expert this rank owns, in rank order
                const unsigned mine_mask =
                    __ballot_sync(0xffffffffu, threadIdx.x < 8 && sel[threadIdx.x & 7] >= e0 && sel[threadIdx.x & 7] < e1);
                if (threadIdx.x < 8 && ((mine_mask >> threadIdx.x) & 1u))
                    own[__popc(mine_mask & ((1u << threadIdx.x) - 1u))] = threadIdx.x;
                if (threadIdx.x == 0) n_own_s = __popc(mine_mask);
            }
            __syncthreads();
            const int n_own = n_own_s;
            issue_gateup(d, w, sel, own, n_own, smem + L.buf0, L.iq2r_rb, G);   // both buffers: free now
            top8_weights(d, layer, sel, wsel);  // read in the down phase, after several block syncs
            const uint32_t rb = L.iq2r_rb, tb = (uint32_t)kTileRows * rb;
            const int mine = my_items(n_own * (I / kTileRows)), nblk = H / 256;
            run_tasks<QXH_IQ2R_F>(smem + L.buf0, tb, rb, 2 * mine, nblk, SameXQ{XQ{xb, sb}}, K4, T, part,
                                    tile_waits(G, 0, d));
            tiles_done(G, 0, 2 * mine);
            mark(d, epoch, 3);
            const int tpe = I / kTileRows;
            for (int r = threadIdx.x; r < mine * kTileRows; r += kMT) {
                const int k = r / kTileRows, rr = r % kTileRows, it = item_id(k);
                const float gv = finite_or_zero_d(tile_row(part, 2 * k, nblk, rr));
                const float uv = finite_or_zero_d(tile_row(part, 2 * k + 1, nblk, rr));
                const double gd = (double)gv;
                d.hbuf[(it / tpe) * I + (it % tpe) * kTileRows + rr] = (float)(gd / (1.0 + exp(-gd)) * (double)uv);
            }
            grid_arrive(bar, epoch, nsync, d);
            issue_down(d, w, sel, own, n_own, buf[qb], G);
            grid_wait(bar, epoch, nsync, d);
        }
        // ---------------- down (weights in buf[qb]) ----------------
        {
            const int n_own = n_own_s;
            copy_to_smem(d.hbuf, xs, n_own * I);
            // into the free gate/up buffer: next layer's QKV tiles (or the first head group)
            if (layer + 1 < m.layers) issue_qkv(d, layers[layer + 1], buf[1 - qb], L.norm, G);
            build_xq(xs, n_own * I, xb, sb);   // slot j's groups start at j * I / 16 (I % 256 == 0)
            __syncthreads();
            mark(d, epoch, 2);
            const uint32_t rb = (uint32_t)r4_row_bytes(I), tb = (uint32_t)kTileRows * rb;
            const int mine = my_items(H / kTileRows), nblk = I / 256;
            run_tasks<QXH_R4_IQ3_F>(buf[qb], tb, rb, n_own * mine, nblk,
                                     [&](int i) {
                                         return XQ{xb + (i % n_own) * xq_words(I), sb + (i % n_own) * (I / 256)};
                                     },
                                     K4, T, part, tile_waits(G, kTileBars / 2, d));
            tiles_done(G, kTileBars / 2, n_own * mine);
            mark(d, epoch, 3);
            // the weighted terms (float)(w_j * y_j) of every (row, slot) in
            // parallel (xs is free again), then per row in rank order
            float* terms = xs;
            auto term_of = [&](int r, int j) {
                return (float)(wsel[own[j]] *
                               (double)finite_or_zero_d(tile_row(part, n_own * (r / kTileRows) + j, nblk, r % kTileRows)));
            };
            if (!ep) {
                for (int u = threadIdx.x; u < mine * kTileRows * n_own; u += kMT) terms[u] = term_of(u / n_own, u % n_own);
            } else {
                // this rank's slots into every rank's exchange buffer, 4 rows per
                // 16-byte store; then the CTA's release on every rank's counter
                const int quads = mine * kTileRows / 4;
                for (int u = threadIdx.x; u < quads * n_own; u += kMT) {
                    const int j = u / quads, r = (u % quads) * 4;
                    const float4 v = make_float4(term_of(r, j), term_of(r + 1, j), term_of(r + 2, j), term_of(r + 3, j));
                    const int row = item_id(r / kTileRows) * kTileRows + r % kTileRows;
                    for (int p = 0; p < d.ep_world; ++p)
                        *reinterpret_cast<float4*>(ep_terms(d.ep_peers[p], layer & 1, own[j], H) + row) = v;
                }
                __syncthreads();
                if (threadIdx.x == 0)            // the CTA's stores happen before (bar.sync), so they are released
                    for (int p = 0; p < d.ep_world; ++p) red_release_sys_add(&ep_tail(d.ep_peers[p], H)->layer_cnt[d.ep_rank], 1u);
            }
            if (!ep) {
                __syncthreads();
                for (int r = threadIdx.x; r < mine * kTileRows; r += kMT) {
                    const int row = item_id(r / kTileRows) * kTileRows + r % kTileRows;
                    float moe = 0.0f;
                    for (int j = 0; j < n_own; ++j) moe += terms[r * n_own + j];
                    d.moe_out[row] = moe;
                    xown = xown + moe;
                    d.x[row] = xown;
                }
            }
            if (ep) skip_sync(epoch, d);         // the next layer waits on every rank's counters instead
            else grid_sync(bar, epoch, nsync, d);
        }
        qb = 1 - qb;
    }
    // ---------------- head (R8 tiles through a ring of kHeadStages stages) ----------------
    {
        if (ep) {
            ep_wait_layer(d, seqb, m.layers - 1);
            ep_combine(d, m.layers - 1, xs);
            if (blockIdx.x == 0)                // the final residual; d.x is still being read
                for (int i = threadIdx.x; i < H; i += kMT) d.hbuf[i] = xs[i];
        } else {
            copy_to_smem(d.x, xs, H);
        }
        const double ss = sum_sq_fixed(xs, H, scratch);
        const double rms = sqrt(ss / (double)H + 1.0e-6), rinv = 1.0 / rms;
        if (isfinite(rms))
            for (int i = threadIdx.x; i < H; i += kMT) xs[i] = (float)div_by((double)xs[i], rms, rinv) * d.out_norm[i];
        else
            for (int i = threadIdx.x; i < H; i += kMT) xs[i] = (float)((double)xs[i] / rms) * d.out_norm[i];
        __syncthreads();
        build_xq(xs, H, xb, sb);
        __syncthreads();
        // this rank's head rows [32 hg0, 32 hg1) as 16-row tiles; the ring spans
        // both weight buffers (free: no layer tiles are in flight)
        const int t0 = 2 * hg0, mine = my_items(2 * (hg1 - hg0)), nblk = H / 256;
        const uint32_t rb = (uint32_t)r8_row_bytes(H), tb = (uint32_t)kTileRows * rb;
        uint8_t* ring = smem + L.buf0;
        for (int k = 0; k < kHeadStages - 1 && k < mine; ++k) issue_head_tile(d, t0 + item_id(k), ring, k, G);
        double bv = -1.0e300;
        int bi = 0x7fffffff;
        bool bad = false;
        for (int k = 0; k < mine; ++k) {
            const int st = k % kHeadStages;
            if (k + kHeadStages - 1 < mine)    // the stage freed by tile k - 1 (synced below)
                issue_head_tile(d, t0 + item_id(k + kHeadStages - 1), ring, (k + kHeadStages - 1) % kHeadStages, G);
            group_wait(G, kGHead0 + st, d);
            run_tasks<QXH_R8_F>(ring + (size_t)st * tb, tb, rb, 1, nblk, SameXQ{XQ{xb, sb}}, K4, T, part);
            if (threadIdx.x < kTileRows) {
                const int r = threadIdx.x, row = (t0 + item_id(k)) * kTileRows + r;
                const double v = tile_row(part, 0, nblk, r);
                if (!isfinite(v)) bad = true;
                d.logits[row] = (float)v;
                if (v > bv || (v == bv && row < bi)) { bv = v; bi = row; }
            }
            __syncthreads();   // stage st is refilled in the next iteration
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
        grid_sync(bar, epoch, nsync, d);
        if (ep && blockIdx.x == 0)
            for (int i = threadIdx.x; i < H; i += kMT) d.x[i] = d.hbuf[i];
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            double v = d.best_val[0];
            int i = d.best_idx[0];
            for (int c = 1; c < (int)gridDim.x; ++c) {
                const double cv = d.best_val[c];
                const int ci = d.best_idx[c];
                if (cv > v || (cv == v && ci < i)) { v = cv; i = ci; }
            }
            if (ep) {                             // every rank's shard maximum, lowest index on ties
                for (int p = 0; p < d.ep_world; ++p) {
                    EpTail* t = ep_tail(d.ep_peers[p], H);
                    t->best_val[d.ep_rank] = v;
                    t->best_idx[d.ep_rank] = i;
                }
                __threadfence_system();
                for (int p = 0; p < d.ep_world; ++p)
                    st_release_sys(&ep_tail(d.ep_peers[p], H)->head_flag[d.ep_rank], seqb + 63u);
                EpTail* mine_t = ep_tail(d.ep_local, H);
                ep_wait_flags(mine_t->head_flag, d.ep_world, seqb + 63u, d.err);
                v = __ldcg(&mine_t->best_val[0]);
                i = __ldcg(&mine_t->best_idx[0]);
                for (int p = 1; p < d.ep_world; ++p) {
                    const double cv = __ldcg(&mine_t->best_val[p]);
                    const int ci = __ldcg(&mine_t->best_idx[p]);
                    if (cv > v || (cv == v && ci < i)) { v = cv; i = ci; }
                }
                *d.ep_seq = seqb / 64u + 1u;
            }
            d.tokens_out[pos] = i;
            *d.token = i;
            *d.pos = pos + 1;
        }
    }
    group_drain(G, d);
}

// ---- the same two-phase attention as stand-alone kernels (per-stage path) ----
// Used by the stage entry point and the per-stage decode path, so both share
// the one-launch kernel's attention arithmetic.  Shared memory: the staging
// region (kAttnStageBytes) followed by the query / product scratch.
constexpr uint32_t kAttnStageBytes = 192 * 1024;   // scores: K rows; context: 8 B per position + the V ring
constexpr uint32_t kAttnScratchBytes =
    std::max<uint32_t>(std::max<uint32_t>(kVChunk * 132, kProdBytes), 16 * kQdStride * 8);

__global__ void __launch_bounds__(kMT, 1) k_attn_scores(Dev d, LayerW w, int layer) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ AttnSmem attn;
    const int pos = *d.pos;
    if (pos < 0 || pos >= d.dm.ctx) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(d.err, kErrPosition);
        return;
    }
    const AttnStage stg = attn_stage(d, pos, smem, kAttnStageBytes);
    attn_scores(d, w, layer, pos, attn, reinterpret_cast<double*>(smem + kAttnStageBytes), stg, 0);
}

__global__ void __launch_bounds__(kMT, 1) k_attn_context(Dev d, int layer) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ AttnSmem attn;
    const int pos = *d.pos;
    if (pos < 0 || pos >= d.dm.ctx) return;
    const AttnStage stg = attn_stage(d, pos, smem, kAttnStageBytes);
    attn_context(d, layer, pos, attn, reinterpret_cast<float*>(smem + kAttnStageBytes), stg, 0);
}

namespace {
uint32_t a16u(size_t v) { return (uint32_t)((v + 15) / 16 * 16); }
// The step kernel's dynamic shared-memory limit is a per-device attribute of
// the function, shared by every engine on that device: only ever raise it, so
// an engine with a smaller model created later cannot lower it below what an
// earlier engine's launches need.
std::mutex g_smem_mu;
int g_smem_limit[64];
}  // namespace

// (tile, block) tasks one CTA runs in its largest dot phase.
static int mega_max_tasks(const Dims& m, int grid) {
    auto cdiv = [](int a, int b) { return (a + b - 1) / b; };
    const int H = m.hidden, Q = m.q_dim(), KV = m.kv_dim(), I = m.moe_inter;
    const int t[] = {cdiv((Q + 2 * KV) / kTileRows, grid) * (H / 256), cdiv(H / kTileRows, grid) * (Q / 256),
                     cdiv(8 * (I / kTileRows), grid) * 2 * (H / 256), cdiv(H / kTileRows, grid) * 8 * (I / 256),
                     H / 256};
    int mx = 0;
    for (int v : t) mx = std::max(mx, v);
    return mx;
}

// Shared-memory layout for the model geometry on `grid` CTAs.
static MegaLayout mega_layout(const Dims& m, int grid) {
    auto cdiv = [](int a, int b) { return (a + b - 1) / b; };
    const int H = m.hidden, Q = m.q_dim(), KV = m.kv_dim(), I = m.moe_inter;
    const size_t t_qkv = (size_t)kTileRows * r4_row_bytes(H), t_o = (size_t)kTileRows * r4_row_bytes(Q);
    const size_t t_dn = (size_t)kTileRows * r4_row_bytes(I);
    const size_t t_hd = ((size_t)kHeadStages * kTileRows * r8_row_bytes(H) + 1) / 2;   // the ring spans both buffers
    size_t bufb = 0;
    bufb = std::max(bufb, cdiv((Q + 2 * KV) / kTileRows, grid) * t_qkv + (size_t)H * 4);
    bufb = std::max(bufb, cdiv(H / kTileRows, grid) * t_o);
    bufb = std::max(bufb, (size_t)cdiv(m.experts, grid) * H * 4 + (size_t)H * 4);
    bufb = std::max(bufb, (cdiv(8 * (I / kTileRows), grid) * 2 * kTileRows * iq2r_row_bytes(H) + 1) / 2);   // spans both
    bufb = std::max(bufb, cdiv(H / kTileRows, grid) * 8 * t_dn);
    bufb = std::max(bufb, t_hd);
    const int XS = std::max(std::max(H, Q), 8 * I);
    MegaLayout L{};
    uint32_t off = 0;
    L.xs = off; off += a16u(std::max({(size_t)XS * 4, (size_t)kVChunk * 132, (size_t)kProdBytes}));
    L.xb = off; off += a16u(std::max(xq_words(XS) * 4, (size_t)attn_ctx_bytes(m.ctx)));   // also the attention staging
    L.sb = off; off += a16u((size_t)XS / 256 * 4 + 32);
    L.tab = off; off += a16u(sizeof(IqTab));
    L.part = off; off += a16u((size_t)mega_max_tasks(m, grid) * kTileRows * 8);
    L.buf_bytes = a16u(bufb);
    L.norm = L.buf_bytes - (uint32_t)H * 4u;
    L.buf0 = off; off += L.buf_bytes;
    L.buf1 = off; off += L.buf_bytes;
    L.total = off;
    L.iq2r_rb = (uint32_t)iq2r_row_bytes(H);
    return L;
}

// Tasks per CTA must fit the per-task bookkeeping.
static bool mega_tasks_fit(const Dims& m, int grid) { return mega_max_tasks(m, grid) <= kMaxTasks && m.experts <= kMT; }

int mega_setup(int device, const Dims& m, int* grid_out) {
    int sms = 0, optin = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, k_decode_step) != cudaSuccess) return 0;
    if (m.vocab % 32) return 0;               // head rows in groups of 32 (the expert-parallel unit)
    const MegaLayout L = mega_layout(m, sms);
    if (L.total + a.sharedSizeBytes > (size_t)optin || !mega_tasks_fit(m, sms)) return 0;
    if (attn_ctx_bytes(m.ctx) > L.sb - L.xb || std::max((size_t)kVChunk * 132, (size_t)kProdBytes) > L.xb - L.xs) return 0;
    const int group = m.q_heads / m.kv_heads;
    if (kMT % group || group * 128 > 8 * kMT || (size_t)group * kQdStride * 8 > L.xb - L.xs || sms < m.kv_heads ||
        m.kv_heads > 8)
        return 0;
    auto cdiv = [](int a, int b) { return (a + b - 1) / b; };
    if ((size_t)2 * cdiv(8 * (m.moe_inter / kTileRows), sms) * kTileRows * L.iq2r_rb > (size_t)2 * L.buf_bytes ||
        2 * cdiv(8 * (m.moe_inter / kTileRows), sms) > kTileBars / 2 || 8 * cdiv(m.hidden / kTileRows, sms) > kTileBars / 2)
        return 0;                             // gate/up and down tiles of one CTA each fit half the tile barriers
    if (cdiv(m.hidden / kTileRows, sms) * kTileRows > kMT) return 0;   // one residual row per thread (xown)
    {
        std::lock_guard<std::mutex> lk(g_smem_mu);
        int& cur = g_smem_limit[device & 63];
        if ((int)L.total > cur) {
            if (cudaFuncSetAttribute(k_decode_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total) !=
                cudaSuccess)
                return 0;
            cur = (int)L.total;
        }
    }
    int per = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_decode_step, kMT, L.total);
    if (per < 1) return 0;
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

// ---- IQ2_XS -> IQ2R re-lay (once, at engine creation) ----------------------
__host__ __device__ inline size_t iq2r_rb(int H) {
    const size_t nblk = (size_t)H / 256;
    return (2 * nblk + 15) / 16 * 16 + nblk * kIq2rBlock;
}
size_t iq2r_row_bytes(int H) { return iq2r_rb(H); }

// One thread per (row, 256-value block).  Value v of the block comes from grid
// entry e = v / 8 (qs[e]: 9-bit lattice index, 7 sign bits + parity from
// ksigns), position v % 8; its code is 1..3 for magnitude 8, 25, 43, plus 4
// when negative (src/qx_format.c:1994-2030 decodes the same fields).
__global__ void k_iq2r_repack(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, size_t rows, int H,
                              const Tables* __restrict__ t) {
    const int nblk = H / 256;
    const size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= rows * (size_t)nblk) return;
    const size_t row = id / nblk;
    const int b = (int)(id % nblk);
    const size_t rb = iq2r_rb(H), hdr = rb - (size_t)nblk * kIq2rBlock;
    const uint8_t* blk = src + (row * nblk + b) * 74;
    uint8_t* orow = dst + row * rb;
    orow[2 * b] = blk[0];
    orow[2 * b + 1] = blk[1];
    uint8_t* ob = orow + hdr + (size_t)b * kIq2rBlock;
    for (int gq = 0; gq < 16; ++gq) ob[gq] = (uint8_t)(1 + 2 * ((blk[66 + (gq >> 1)] >> (4 * (gq & 1))) & 15));
    for (int gq = 0; gq < 16; ++gq)
        for (int tt = 0; tt < 4; ++tt) {
            uint32_t codes = 0;
            for (int j = 0; j < 4; ++j) {
                const int v = 16 * gq + 4 * tt + j, e = v >> 3, k = v & 7;
                const uint32_t q = (uint32_t)blk[2 + 2 * e] | ((uint32_t)blk[3 + 2 * e] << 8);
                const float mag = t->iq2xs[q & 511u][k];
                const bool neg = (t->ksigns[q >> 9] >> k) & 1u;
                const uint32_t c = mag == 8.0f ? 1u : mag == 25.0f ? 2u : mag == 43.0f ? 3u : 0u;
                codes |= (c | (neg && c ? 4u : 0u)) << (4 * j);
            }
            ob[16 + 32 * tt + 2 * gq] = (uint8_t)codes;
            ob[16 + 32 * tt + 2 * gq + 1] = (uint8_t)(codes >> 8);
        }
    if (b == 0)
        for (size_t i = 2 * (size_t)nblk; i < hdr; ++i) orow[i] = 0;
}

size_t r4_bytes_per_row(int K) { return r4_row_bytes(K); }
size_t r8_bytes_per_row(int K) { return r8_row_bytes(K); }

// One thread per (row, 256-value block) of Q6_K (210 B: ql[128], qh[64],
// int8 scales[16], fp16 d).  Value v = 128h + 32s + l has the low 4 bits from
// ql[64h + 32(s & 1) + l] (high nibble for s >= 2) and the high 2 bits from
// qh[32h + l] >> 2s, weight q - 32, group scale scales[v / 16]
// (src/qx_format.c decodes the same fields; so does dot_q6_k_mma).
__global__ void k_r8_repack(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, size_t rows, int K) {
    const int nblk = K / 256;
    const size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= rows * (size_t)nblk) return;
    const size_t row = id / nblk;
    const int b = (int)(id % nblk);
    const size_t rb = r8_row_bytes(K);
    const int hdr = r4_hdr(nblk);
    const uint8_t* blk = src + (row * nblk + b) * 210;
    uint8_t* orow = dst + row * rb;
    orow[2 * b] = blk[208];
    orow[2 * b + 1] = blk[209];
    uint8_t* ob = orow + hdr + 272 * b;
    for (int gq = 0; gq < 16; ++gq) ob[gq] = blk[192 + gq];
    for (int v = 0; v < 256; ++v) {
        const int h = v >> 7, sct = (v >> 5) & 3, l = v & 31;
        const uint8_t qlb = blk[64 * h + 32 * (sct & 1) + l];
        const int lo = sct >= 2 ? (qlb >> 4) : (qlb & 15);
        const int hi = (blk[128 + 32 * h + l] >> (2 * sct)) & 3;
        const int gq = v >> 4, t = (v >> 2) & 3, j = v & 3;
        ob[16 + 64 * (gq >> 2) + 16 * t + 4 * (gq & 3) + j] = (uint8_t)(int8_t)((lo | (hi << 4)) - 32);
    }
    if (b == 0) {
        for (int i = 2 * nblk; i < hdr; ++i) orow[i] = 0;
        for (size_t i = (size_t)hdr + 272 * (size_t)nblk; i < rb; ++i) orow[i] = 0;
    }
}

cudaError_t launch_r8_repack(const uint8_t* src, uint8_t* dst, size_t rows, int K, cudaStream_t st) {
    const size_t n = rows * (size_t)(K / 256);
    k_r8_repack<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(src, dst, rows, K);
    return cudaGetLastError();
}

// One thread per (row, 256-value block).  IQ4_XS (136 B: d, scales_h, scales_l,
// 128 B of nibbles: byte j of group ib holds values 32ib + j (low) and
// 32ib + 16 + j (high)): the code is the nibble, the group scale ls - 32.
// IQ3_XXS (98 B: d, 64 lattice indices of 4 values, 8 x u32 of four 7-bit
// sign codes and the group scale nibble): the code is the magnitude's index in
// {4, 12, ..., 52, 62} plus 8 when negative, the group scale 1 + 2s
// (src/qx_format.c:1914-1960, 2060-2110 decode the same fields).
__global__ void k_r4_repack(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, size_t rows, int K, int type,
                            const Tables* __restrict__ t) {
    const int nblk = K / 256;
    const size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= rows * (size_t)nblk) return;
    const size_t row = id / nblk;
    const int b = (int)(id % nblk);
    const size_t rb = r4_row_bytes(K);
    const int hdr = r4_hdr(nblk), cod = r4_codes(nblk);
    uint8_t* orow = dst + row * rb;
    uint8_t code[256];
    uint8_t scale[8];
    if (type == QXH_IQ4_XS_F) {
        const uint8_t* blk = src + (row * nblk + b) * 136;
        orow[2 * b] = blk[0];
        orow[2 * b + 1] = blk[1];
        const uint32_t sh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8);
        const uint32_t sl = (uint32_t)blk[4] | ((uint32_t)blk[5] << 8) | ((uint32_t)blk[6] << 16) | ((uint32_t)blk[7] << 24);
        for (int ib = 0; ib < 8; ++ib) {
            const int ls = (int)(((sl >> (4 * ib)) & 15u) | (((sh >> (2 * ib)) & 3u) << 4));
            scale[ib] = (uint8_t)(int8_t)(ls - 32);
            for (int j = 0; j < 16; ++j) {
                const uint8_t q = blk[8 + 16 * ib + j];
                code[32 * ib + j] = q & 15u;
                code[32 * ib + 16 + j] = q >> 4;
            }
        }
    } else {
        const uint8_t* blk = src + (row * nblk + b) * 98;
        orow[2 * b] = blk[0];
        orow[2 * b + 1] = blk[1];
        for (int ib = 0; ib < 8; ++ib) {
            const uint8_t* a = blk + 66 + 4 * ib;
            const uint32_t aux = (uint32_t)a[0] | ((uint32_t)a[1] << 8) | ((uint32_t)a[2] << 16) | ((uint32_t)a[3] << 24);
            scale[ib] = (uint8_t)(1 + 2 * (aux >> 28));
            for (int k = 0; k < 8; ++k) {
                const int idx = blk[2 + 8 * ib + k];
                const uint32_t signs = t->ksigns[(aux >> (7 * (k >> 1))) & 127u];
                for (int j = 0; j < 4; ++j) {
                    const int mag = (int)t->iq3xxs[idx][j];
                    const int mi = mag == 62 ? 7 : (mag - 4) / 8;
                    const uint32_t neg = (signs >> (4 * (k & 1) + j)) & 1u;
                    code[32 * ib + 4 * k + j] = (uint8_t)(mi + 8 * neg);
                }
            }
        }
    }
    for (int ib = 0; ib < 8; ++ib) orow[hdr + 8 * b + ib] = scale[ib];
    for (int tt = 0; tt < 4; ++tt)
        for (int ib = 0; ib < 8; ++ib) {
            uint32_t w = 0;
            for (int j = 0; j < 4; ++j) {
                w |= (uint32_t)code[32 * ib + 4 * tt + j] << (4 * j);
                w |= (uint32_t)code[32 * ib + 16 + 4 * tt + j] << (16 + 4 * j);
            }
            uint8_t* o = orow + cod + 128 * b + 32 * tt + 4 * ib;
            o[0] = (uint8_t)w, o[1] = (uint8_t)(w >> 8), o[2] = (uint8_t)(w >> 16), o[3] = (uint8_t)(w >> 24);
        }
    if (b == 0) {                              // the row's padding
        for (int i = 2 * nblk; i < hdr; ++i) orow[i] = 0;
        for (int i = hdr + 8 * nblk; i < cod; ++i) orow[i] = 0;
        for (size_t i = (size_t)cod + 128 * (size_t)nblk; i < rb; ++i) orow[i] = 0;
    }
}

cudaError_t launch_r4_repack(const uint8_t* src, uint8_t* dst, size_t rows, int K, int type, const Tables* t,
                             cudaStream_t st) {
    if (type != QXH_IQ4_XS_F && type != QXH_IQ3_XXS_F) return cudaErrorInvalidValue;
    const size_t n = rows * (size_t)(K / 256);
    k_r4_repack<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(src, dst, rows, K, type, t);
    return cudaGetLastError();
}

cudaError_t launch_iq2r_repack(const uint8_t* src, uint8_t* dst, size_t rows, int H, const Tables* t, cudaStream_t st) {
    const size_t n = rows * (size_t)(H / 256);
    k_iq2r_repack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, dst, rows, H, t);
    return cudaGetLastError();
}

}  // namespace qx

namespace qx {

// The stand-alone two-phase attention fits when the softmax weights of the
// whole context fit the staging region and the query heads fit the scratch.
bool attn2_supported(const Dims& m) {
    const int group = m.q_heads / m.kv_heads;
    return (size_t)m.ctx * 8 + 2048 <= kAttnStageBytes && attn_ctx_bytes(m.ctx) <= kAttnStageBytes &&
           kMT % group == 0 && group * 128 <= 8 * kMT &&
           (size_t)group * kQdStride * 8 <= kAttnScratchBytes;
}

cudaError_t attn2_configure() {
    const int bytes = (int)(kAttnStageBytes + kAttnScratchBytes);
    cudaError_t e = cudaFuncSetAttribute(k_attn_scores, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_attn_context, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    return e;
}

void launch_attn2(const Dev& d, const LayerW& w, int layer, int sms, cudaStream_t st) {
    const size_t bytes = kAttnStageBytes + kAttnScratchBytes;
    k_attn_scores<<<sms, kMT, bytes, st>>>(d, w, layer);
    k_attn_context<<<std::min(sms, d.dm.q_heads * kCtxSlices), kMT, bytes, st>>>(d, layer);
}

}  // namespace qx
