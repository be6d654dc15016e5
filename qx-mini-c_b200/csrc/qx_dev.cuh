// Device-side building blocks of the decode engine: error bits, the lattice
// tables, the reference's fp16 conversion, warp/block reductions, and the
// asynchronous copy primitives (cp.async, bulk copies on mbarriers).
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

// Correctly rounded quotients a / b for many a and one b, without a
// division per element: r = RN(1 / b) once, then q = RN(a * r) is within one
// ulp of a / b, the remainder a - b*q is exact in one FMA, and RN(q + rem*r)
// is the correctly rounded quotient (P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
// 1990).  Valid for finite a and finite, nonzero b when the quotient is a
// normal number; callers keep the plain division for a non-finite b.  Checked
// on the B200 against the IEEE division over 2^31 random double and float
// quotients (no difference).
__device__ __forceinline__ double div_by(double a, double b, double r) {
    const double q = a * r;
    return fma(fma(-q, b, a), r, q);
}
__device__ __forceinline__ float divf_by(float a, float b, float r) {
    const float q = a * r;
    return fmaf(fmaf(-q, b, a), r, q);
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

// Sum of x[i]^2 over n floats (n % 4 == 0, 16-byte aligned) in the one order
// every RMSNorm of this library uses, whatever its block size (>= 256):
// thread i < 256 adds the float4 groups i, i + 256, ... as (a^2 + b^2) then
// (c^2 + d^2), then block_sum_d adds the warp sums in warp order; threads
// beyond 256 add 0.0, which changes no sum.  (Each square is exact in double;
// only the additions round, so every path that uses this rounds alike.)
__device__ __forceinline__ double sum_sq_fixed(const float* x, int n, double* scratch) {
    double ss = 0.0;
    if (threadIdx.x < 256)
        for (int i = threadIdx.x * 4; i < n; i += 256 * 4) {
            const float4 v = *reinterpret_cast<const float4*>(x + i);
            ss += (double)v.x * (double)v.x + (double)v.y * (double)v.y;
            ss += (double)v.z * (double)v.z + (double)v.w * (double)v.w;
        }
    return block_sum_d(ss, scratch);
}

// ---- asynchronous copies into shared memory ------------------------------
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
