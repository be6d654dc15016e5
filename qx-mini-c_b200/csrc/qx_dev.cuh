// Device-side building blocks of the decode engine: GGUF block decoders that
// reproduce the reference's float weight values, warp row-dot products over
// row tiles staged in shared memory, and the cp.async tile pipeline.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace qx {

constexpr int kThreads = 256;          // 8 warps per CTA for every GEMV kernel
constexpr int kWarps = kThreads / 32;
constexpr int kTileRows = 16;          // rows per staged tile (16*row_bytes is 16-byte aligned for every format)

// Error bits written to Dev::err (read by the host after each call).
enum : int {
    kErrToken = 1, kErrPosition = 2, kErrNonFinite = 4, kErrRouter = 8, kErrTimeout = 16,
    kErrQ8Input = 32,     // q8_k_compat: non-finite activation
    kErrQ8Expert = 64,    // q8_k_compat: non-finite expert output
    kErrQ8Head = 128      // q8_k_compat: non-finite logit
};

// Lattice / codebook tables, built on the host (qx_host.c) and uploaded once.
struct Tables {
    float iq2xs[512][8];     // IQ2_XS lattice magnitudes {8,25,43} as floats
    float iq3xxs[256][4];    // IQ3_XXS lattice magnitudes as floats
    uint8_t ksigns[128];     // 7 stored sign bits + even-parity 8th bit
    float kvalues[16];       // IQ4_NL codebook
    uint32_t iq2s[1024][2];  // IQ2_S lattice: 8 magnitude bytes per entry (value order)
    uint32_t iq3s[512];      // IQ3_S lattice: 4 magnitude bytes per entry
};

// binary16 -> binary32 with the reference's Inf/NaN rule (exp==31 -> +-65504),
// src/qx_format.c:1854-1876.  Finite values and subnormals convert exactly.
__device__ __forceinline__ float h2f(uint16_t h) {
    if (((h >> 10) & 31u) == 31u) return __uint_as_float(((uint32_t)(h & 0x8000u) << 16) | 0x477fe000u);
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint16_t ld16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
__device__ __forceinline__ uint32_t ld32u(const uint8_t* p) {   // 2-byte aligned 32-bit load
    return (uint32_t)ld16(p) | ((uint32_t)ld16(p + 2) << 16);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide double sum (all threads get the result). scratch: >= kWarps doubles.
__device__ __forceinline__ double block_sum_d(double v, double* scratch) {
    v = warp_sum_d(v);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) scratch[w] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += scratch[i];
    return t;
}

// ---- row dots: one warp, one row staged in shared memory ------------------
// Each lane owns 8 consecutive input positions (8*lane .. 8*lane+7) of every
// 256-value block, so x reads are contiguous per lane.

// IQ2_XS (74 B/block), src/qx_format.c:1914-1933.
__device__ __forceinline__ float dot_iq2_xs(const uint8_t* row, const float* x, int nblk, const Tables& T, int lane) {
    float acc = 0.f;
    const int ib = lane >> 2, sub = lane & 3;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 74;
        const float d = h2f(ld16(blk));
        const uint8_t sc = blk[66 + ib];
        const float db = d * (0.5f + (float)(sub < 2 ? (sc & 15) : (sc >> 4))) * 0.25f;
        const uint16_t q = ld16(blk + 2 + 2 * lane);
        const float* g = T.iq2xs[q & 511u];
        const uint32_t s = T.ksigns[q >> 9];
        const float4 x0 = *reinterpret_cast<const float4*>(x + b * 256 + 8 * lane);
        const float4 x1 = *reinterpret_cast<const float4*>(x + b * 256 + 8 * lane + 4);
        const float4 g0 = *reinterpret_cast<const float4*>(g);
        const float4 g1 = *reinterpret_cast<const float4*>(g + 4);
        float t = 0.f;
        t = fmaf(g0.x, (s & 1u) ? -x0.x : x0.x, t);
        t = fmaf(g0.y, (s & 2u) ? -x0.y : x0.y, t);
        t = fmaf(g0.z, (s & 4u) ? -x0.z : x0.z, t);
        t = fmaf(g0.w, (s & 8u) ? -x0.w : x0.w, t);
        t = fmaf(g1.x, (s & 16u) ? -x1.x : x1.x, t);
        t = fmaf(g1.y, (s & 32u) ? -x1.y : x1.y, t);
        t = fmaf(g1.z, (s & 64u) ? -x1.z : x1.z, t);
        t = fmaf(g1.w, (s & 128u) ? -x1.w : x1.w, t);
        acc = fmaf(db, t, acc);
    }
    return warp_sum(acc);
}

// IQ3_XXS (98 B/block), src/qx_format.c:1935-1959.
__device__ __forceinline__ float dot_iq3_xxs(const uint8_t* row, const float* x, int nblk, const Tables& T, int lane) {
    float acc = 0.f;
    const int ib = lane >> 2, l = lane & 3;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 98;
        const float d = h2f(ld16(blk));
        const uint32_t aux = ld32u(blk + 66 + 4 * ib);
        const float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
        const uint32_t s = T.ksigns[(aux >> (7 * l)) & 127u];
        const float* g1 = T.iq3xxs[blk[2 + 8 * ib + 2 * l]];
        const float* g2 = T.iq3xxs[blk[2 + 8 * ib + 2 * l + 1]];
        const float4 x0 = *reinterpret_cast<const float4*>(x + b * 256 + 8 * lane);
        const float4 x1 = *reinterpret_cast<const float4*>(x + b * 256 + 8 * lane + 4);
        const float4 a = *reinterpret_cast<const float4*>(g1);
        const float4 c = *reinterpret_cast<const float4*>(g2);
        float t = 0.f;
        t = fmaf(a.x, (s & 1u) ? -x0.x : x0.x, t);
        t = fmaf(a.y, (s & 2u) ? -x0.y : x0.y, t);
        t = fmaf(a.z, (s & 4u) ? -x0.z : x0.z, t);
        t = fmaf(a.w, (s & 8u) ? -x0.w : x0.w, t);
        t = fmaf(c.x, (s & 16u) ? -x1.x : x1.x, t);
        t = fmaf(c.y, (s & 32u) ? -x1.y : x1.y, t);
        t = fmaf(c.z, (s & 64u) ? -x1.z : x1.z, t);
        t = fmaf(c.w, (s & 128u) ? -x1.w : x1.w, t);
        acc = fmaf(db, t, acc);
    }
    return warp_sum(acc);
}

// IQ4_XS (136 B/block), src/qx_format.c:2036-2077.
__device__ __forceinline__ float dot_iq4_xs(const uint8_t* row, const float* x, int nblk, const float* kv, int lane) {
    float acc = 0.f;
    const int ib = lane >> 2, part = lane & 3;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 136;
        const float d = h2f(ld16(blk));
        const uint32_t sh = ld16(blk + 2);
        const int ls = ((blk[4 + (ib >> 1)] >> (4 * (ib & 1))) & 15) | (((sh >> (2 * ib)) & 3) << 4);
        const float dl = d * (float)(ls - 32);
        const uint32_t q = *reinterpret_cast<const uint32_t*>(blk + 8 + 16 * ib + 4 * part);
        const float4 xl = *reinterpret_cast<const float4*>(x + b * 256 + 32 * ib + 4 * part);
        const float4 xh = *reinterpret_cast<const float4*>(x + b * 256 + 32 * ib + 16 + 4 * part);
        float t = 0.f;
        t = fmaf(kv[q & 15u], xl.x, t);
        t = fmaf(kv[(q >> 8) & 15u], xl.y, t);
        t = fmaf(kv[(q >> 16) & 15u], xl.z, t);
        t = fmaf(kv[(q >> 24) & 15u], xl.w, t);
        t = fmaf(kv[(q >> 4) & 15u], xh.x, t);
        t = fmaf(kv[(q >> 12) & 15u], xh.y, t);
        t = fmaf(kv[(q >> 20) & 15u], xh.z, t);
        t = fmaf(kv[(q >> 28) & 15u], xh.w, t);
        acc = fmaf(dl, t, acc);
    }
    return warp_sum(acc);
}

// Q6_K (210 B/block), src/qx_format.c:2147-2169.  Lane l owns position l of
// each 32-value section of each 128-value half.
__device__ __forceinline__ float dot_q6_k(const uint8_t* row, const float* x, int nblk, int lane) {
    float acc = 0.f;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 210;
        const float d = h2f(ld16(blk + 208));
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t l0 = blk[64 * h + lane], l1 = blk[64 * h + 32 + lane], qh = blk[128 + 32 * h + lane];
            const float* xv = x + b * 256 + 128 * h + lane;
            const int si = 8 * h + (lane >> 4);
            const int q1 = (int)((l0 & 15u) | ((qh & 3u) << 4)) - 32;
            const int q2 = (int)((l1 & 15u) | (((qh >> 2) & 3u) << 4)) - 32;
            const int q3 = (int)((l0 >> 4) | (((qh >> 4) & 3u) << 4)) - 32;
            const int q4 = (int)((l1 >> 4) | (((qh >> 6) & 3u) << 4)) - 32;
            acc = fmaf(d * (float)sc[si], (float)q1 * xv[0], acc);
            acc = fmaf(d * (float)sc[si + 2], (float)q2 * xv[32], acc);
            acc = fmaf(d * (float)sc[si + 4], (float)q3 * xv[64], acc);
            acc = fmaf(d * (float)sc[si + 6], (float)q4 * xv[96], acc);
        }
    }
    return warp_sum(acc);
}

// ---- cp.async row-tile pipeline --------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}

// ---- bulk copies on the copy engine ------------------------------------------
// cp.async.bulk (no tensor map, no multicast): one instruction moves a
// contiguous span global -> shared (both 16-byte aligned, size a multiple of
// 16) and counts its bytes down on an mbarrier of this CTA.  A "group" is one
// mbarrier phase: the issuing thread announces the group's byte total with
// arrive.expect_tx, then issues the spans; the phase completes when all bytes
// have landed, and every thread that waits on its parity sees them.
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// The group's byte total (one arrival of the issuing warp's lane 0).
__device__ __forceinline__ void bulk_group_begin(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Each issuing thread: its earlier generic-proxy accesses of the destination
// (made visible to it by a block barrier) come before the copy engine's writes.
__device__ __forceinline__ void bulk_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Copy `bytes` (multiple of 16, both pointers 16-byte aligned) with the whole CTA.
__device__ __forceinline__ void stage_copy(uint8_t* dst, const uint8_t* src, uint32_t bytes) {
    for (uint32_t c = threadIdx.x; c < bytes / 16u; c += blockDim.x) cp_async16(dst + 16u * c, src + 16u * c);
}


}  // namespace qx
