// Device helpers shared by the per-stage kernels (qx_kernels.cu) and the
// persistent decode-step kernel (qx_mega.cu).
#pragma once
#include <cfloat>

#include "qx_imma.cuh"
#include "qx_kernels.h"

namespace qx {

// ---------------------------------------------------------------------------
// shared helpers
// ---------------------------------------------------------------------------

// xs[i] = (float)((double)x[i] / rms) * w[i], rms = sqrt(sum x^2 / n + 1e-6)
// in double (qx_apply_f32_rmsnorm, src/qx_format.c:3358-3371).
__device__ inline void rmsnorm_to_smem(const float* x, const float* w, float* xs, int n, double* scratch) {
    for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
        *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(x + i);
    __syncthreads();
    const double rms = sqrt(sum_sq_fixed(xs, n, scratch) / (double)n + 1.0e-6);
    for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) {
        const float4 wv = *reinterpret_cast<const float4*>(w + i);
        float4 v = *reinterpret_cast<float4*>(xs + i);
        v.x = (float)((double)v.x / rms) * wv.x;
        v.y = (float)((double)v.y / rms) * wv.y;
        v.z = (float)((double)v.z / rms) * wv.z;
        v.w = (float)((double)v.w / rms) * wv.w;
        *reinterpret_cast<float4*>(xs + i) = v;
    }
    __syncthreads();
}

// Global (L2) -> shared copy of n floats (n % 4 == 0, 16-byte aligned), all of
// a thread's loads issued before its stores so the L2 round trips overlap.
__device__ inline void copy_to_smem(const float* x, float* xs, int n) {
    constexpr int U = 2;
    const int step = blockDim.x * 4;
    for (int i0 = threadIdx.x * 4; i0 < n; i0 += U * step) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i0 + u * step < n) v[u] = __ldcg(reinterpret_cast<const float4*>(x + i0 + u * step));
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i0 + u * step < n) *reinterpret_cast<float4*>(xs + i0 + u * step) = v[u];
    }
    __syncthreads();
}

__device__ __forceinline__ float finite_or_zero_d(double v) { return isfinite(v) ? (float)v : 0.0f; }

__device__ __forceinline__ uint8_t* align16(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 15u) & ~(uintptr_t)15u);
}

// last-CTA ticket: true in exactly one CTA, after all `expected` CTAs made
// their global writes visible.
__device__ __forceinline__ bool last_cta(unsigned* counter, unsigned expected) {
    __shared__ bool is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(counter, 1u) == expected - 1u;
    __syncthreads();
    if (is_last) __threadfence();
    return is_last;
}

// Shared-memory carve-up helper.
struct Carve {
    uint8_t* p;
    __device__ explicit Carve(uint8_t* base) : p(base) {}
    template <class T>
    __device__ T* take(size_t count) {
        p = align16(p);
        T* r = reinterpret_cast<T*>(p);
        p += count * sizeof(T);
        return r;
    }
};

__device__ __forceinline__ void load_kv_regs(const Tables* t, uint32_t K[4]) {
    // IQ4_NL codebook as 16 signed bytes in 4 registers
    for (int j = 0; j < 4; ++j) {
        uint32_t w = 0;
        for (int k = 0; k < 4; ++k) w |= ((uint32_t)(uint8_t)(int8_t)t->kvalues[4 * j + k]) << (8 * k);
        K[j] = w;
    }
}

// Sum the per-part tile partials in part order and return the row value.
__device__ __forceinline__ double sum_parts(const double* part, int tile, int parts, int row) {
    double v = 0.0;
    for (int p = 0; p < parts; ++p) v += part[(tile * parts + p) * kTileRows + row];
    return v;
}

// Store the two rows a warp finished (lane t = 0 of each group g).
__device__ __forceinline__ void store_tile_rows(double* part, int warp, const Acc& acc) {
    double lo, hi;
    acc.finish(lo, hi);
    const int lane = threadIdx.x & 31;
    if ((lane & 3) == 0) {
        part[warp * kTileRows + (lane >> 2)] = lo;
        part[warp * kTileRows + (lane >> 2) + 8] = hi;
    }
}

__device__ __forceinline__ double block_max_d(double v, double* scratch) {
    for (int o = 16; o; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    double m = scratch[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = fmax(m, scratch[i]);
    return m;
}

__device__ __forceinline__ float block_max_f(float v, float* scratch) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = scratch[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, scratch[i]);
    return m;
}

// Head RMSNorm (double) + RoPE (double, host table) of one 128-wide head held
// in v[0..127] (shared memory); all 128 threads call.
__device__ inline void head_norm_rope(float* v, const float* nw, const double* rope, double* scratch) {
    const int i = threadIdx.x;
    const double x = (double)v[i];
    const double ss = block_sum_d(x * x, scratch);
    const double inv = 1.0 / sqrt(ss / 128.0 + 1.0e-6);
    const float y = (float)(x * inv * (double)nw[i]);
    __syncthreads();
    v[i] = y;
    __syncthreads();
    if (i < 64) {
        const double c = rope[2 * i], s = rope[2 * i + 1];
        const float x0 = v[i], x1 = v[i + 64];
        v[i] = (float)__dsub_rn(__dmul_rn((double)x0, c), __dmul_rn((double)x1, s));   // no contraction
        v[i + 64] = (float)__dadd_rn(__dmul_rn((double)x0, s), __dmul_rn((double)x1, c));
    }
    __syncthreads();
}

__device__ inline void load_iq_tables(IqTab* T, const Tables* G, bool want2, bool want3) {
    if (want2)
        for (int i = threadIdx.x; i < 512 * 2; i += blockDim.x) {
            const float* g = G->iq2xs[i >> 1] + 4 * (i & 1);
            T->grid2[i >> 1][i & 1] =
                (uint32_t)g[0] | ((uint32_t)g[1] << 8) | ((uint32_t)g[2] << 16) | ((uint32_t)g[3] << 24);
        }
    if (want3)
        for (int i = threadIdx.x; i < 256; i += blockDim.x) {
            const float* g = G->iq3xxs[i];
            T->grid3[i] = (uint32_t)g[0] | ((uint32_t)g[1] << 8) | ((uint32_t)g[2] << 16) | ((uint32_t)g[3] << 24);
        }
    for (int i = threadIdx.x; i < 128; i += blockDim.x) T->ksigns[i] = G->ksigns[i];
}

// Head RMSNorm (double) + RoPE of one 128-wide head by one warp; lane owns
// dims lane, lane+32, lane+64, lane+96 (RoPE pairs (i, i+64) stay in-lane).
__device__ __forceinline__ void warp_norm_rope(float* v, const float* nw, const double* rope, int lane) {
    double x[4], ss = 0.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) { x[k] = (double)v[lane + 32 * k]; ss += x[k] * x[k]; }
    ss = warp_sum_d(ss);
    const double inv = 1.0 / sqrt(ss / 128.0 + 1.0e-6);
    float y[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) y[k] = (float)(x[k] * inv * (double)nw[lane + 32 * k]);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int i = lane + 32 * k;
        const double c = rope[2 * i], s = rope[2 * i + 1];
        const float x0 = y[k], x1 = y[k + 2];
        v[i] = (float)__dsub_rn(__dmul_rn((double)x0, c), __dmul_rn((double)x1, s));   // no contraction
        v[i + 64] = (float)__dadd_rn(__dmul_rn((double)x0, s), __dmul_rn((double)x1, c));
    }
}

// (float)k for an INT8 value, exactly, as one FP32 add instead of an integer
// conversion: 1.5 * 2^23 + k has k in its last mantissa bits (ulp 1 there),
// and subtracting 1.5 * 2^23 is exact (Sterbenz).  Valid for |k| < 2^22.
__device__ __forceinline__ float i8_to_f32(int k) { return __fsub_rn(__int_as_float(0x4b400000 + k), 12582912.0f); }

// Attention score of one cached INT8 key row (128 dims) against a query head
// held as doubles: the dot product in dimension order in double, exactly as the
// reference accumulates it (src/qx_format.c:5127-5150): each product of two
// floats is exact in double, so the fused multiply-add rounds like the
// reference's multiply-then-add.  Divided by sqrt(128); non-finite -> 0.
__device__ __forceinline__ double score_row(const double* qd, const int8_t* kp, float ks, double sqrt_d) {
    double s = 0.0;
#pragma unroll 2
    for (int j = 0; j < 128; j += 16) {
        const int4 raw = *reinterpret_cast<const int4*>(kp + j);
        const int8_t* kb = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
        for (int u = 0; u < 16; ++u) s = fma(qd[j + u], (double)(i8_to_f32(kb[u]) * ks), s);
    }
    s /= sqrt_d;
    return isfinite(s) ? s : 0.0;
}

// score_row over a key row whose 16-byte chunk j is stored at chunk j ^ key
// (a shared-memory swizzle; key 0 = plain row).  Same arithmetic and order.
__device__ __forceinline__ double score_row_sw(const double* qd, const int8_t* kp, int key, float ks, double sqrt_d) {
    double s = 0.0;
#pragma unroll 2
    for (int j = 0; j < 8; ++j) {
        const int4 raw = *reinterpret_cast<const int4*>(kp + 16 * (j ^ key));
        const int8_t* kb = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
        for (int u = 0; u < 16; ++u) s = fma(qd[16 * j + u], (double)(i8_to_f32(kb[u]) * ks), s);
    }
    s /= sqrt_d;
    return isfinite(s) ? s : 0.0;
}

// Sum of w[0..n) in a fixed order that does not depend on the CTA size:
// lane l adds w[l], w[l+32], ... then the 32 lane sums are combined by a
// butterfly.  All threads call; the result is broadcast.
__device__ inline double fixed_order_sum(const double* w, int n, double* slot) {
    __syncthreads();
    if (threadIdx.x < 32) {
        double s = 0.0;
        for (int t = threadIdx.x; t < n; t += 32) s += w[t];
        s = warp_sum_d(s);
        if (threadIdx.x == 0) *slot = s;
    }
    __syncthreads();
    return *slot;
}

}  // namespace qx
