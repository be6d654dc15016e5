// Exact integer dot products on the tensor cores (mma.sync int8, sm_100a).
//
// Every weight of the GGUF block formats on the decode path is a small
// integer times per-block scales:
//   IQ2_XS  w = d/8 * (1+2s) * g,   g in +-{8,25,43},   s 4-bit per 16 values
//   IQ3_XXS w = d/4 * (1+2s) * g,   g in +-{4..62},     s 4-bit per 32 values
//   IQ4_XS  w = d * (ls-32) * kv,   kv in [-127,113],   ls 6-bit per 32 values
//   Q6_K    w = d * sc * (q-32),    q 6-bit,            sc int8 per 16 values
// (src/qx_format.c:1914-2169).  The activation x of each 256-value block is
// turned into a 56-bit fixed-point integer X = round(x * 2^S_b) (exact for
// every element within 2^31 of the block maximum), offset to X' = X + 2^55 >= 0
// and split into 7 unsigned bytes ("limbs").  One m16n8k{16,32} s8*u8 MMA then
// gives, per row, the exact integer sums of (integer weight) * (limb) for the
// 7 limbs in columns 0..6, and in column 7 (a column of ones) the integer sum
// of the weights, which removes the offset.  The per-group integer scales are
// applied to the int32 results with IMAD, and each block's result is folded
// into a double accumulator with its (exact) block factor d * 2^-S_b.  The
// only roundings are the double additions, so the result agrees with the
// reference's double accumulation to ~1e-16 and rounds to the same float.
#pragma once
#include <cstdint>

#include "qx_dev.cuh"

namespace qx {

constexpr int kLimbs = 7;           // 56-bit fixed point
constexpr int kOffsetBits = 55;

// B operand in shared memory: for each 16-value group G, kXG words of which
// the first 32 are in lane order; lane 4n+t holds limb n of values
// 16G+4t .. 16G+4t+3 (one byte each, value order).  Lane group n = 7 holds the
// constant 1 (offset column).  The stride of 36 words (not 32) makes the
// quantizer's stores conflict-free: the 8 groups a warp writes at once start
// in banks 0, 4, ..., 28.
constexpr int kXG = 36;
__host__ __device__ constexpr size_t xq_words(int K) { return (size_t)K / 16 * kXG; }

struct XQ {
    const uint32_t* b;   // [K/16][kXG]
    const int* s;        // [K/256] block exponents S_b
};

// Exact 2^e as a double for -1022 <= e <= 1023.
__device__ __forceinline__ double pow2d(int e) { return __longlong_as_double((long long)(1023 + e) << 52); }

// Block exponent recorded for a 256-value block that holds a NaN or an
// infinity.  The reference's dot products with such an input are not finite
// (and then zeroed, src/qx_format.c:4284, :4783, or reported, :3715); the
// block's factor becomes NaN so every row's result is NaN here too.
constexpr int kSbNonFinite = 0x40000000;
__device__ __forceinline__ double blk_pow2(int S, int k) {
    return S == kSbNonFinite ? __longlong_as_double(0x7ff8000000000000ll) : pow2d(k - S);
}

// ---- activation quantization ------------------------------------------------

// X' = round(x * 2^S) + 2^55 (halfway cases away from zero), split in two
// words.  S = 54 - E(block max) lies in [-73, 180]; the scale is applied as two
// exact power-of-two factors in [2^-37, 2^90], so y = x * 2^S is exact (a
// product that underflows has |x * 2^S| < 2^-126 and rounds to 0 either way)
// and |y| < 2^55 converts to int64 exactly.  Rounding: truncate, then step
// away from zero when the (exact) dropped fraction is at least 1/2.
__device__ __forceinline__ void to_fixed(float x, int S, uint32_t& hi, uint32_t& lo) {
    const int s1 = S >> 1, s2 = S - s1;
    const float y = __fmul_rn(__fmul_rn(x, __int_as_float((s1 + 127) << 23)), __int_as_float((s2 + 127) << 23));
    long long X = __float2ll_rz(y);
    if (fabsf(__fsub_rn(y, truncf(y))) >= 0.5f) X += y < 0.f ? -1 : 1;
    const uint64_t Xp = (uint64_t)(X + (1ll << kOffsetBits));
    hi = (uint32_t)(Xp >> 32);
    lo = (uint32_t)Xp;
}

// 4x4 byte transpose: out[n] = byte n of in[0..3], in value order.
__device__ __forceinline__ void transpose4(uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t out[4]) {
    const uint32_t t0 = __byte_perm(a, b, 0x5140), t1 = __byte_perm(a, b, 0x7362);
    const uint32_t t2 = __byte_perm(c, d, 0x5140), t3 = __byte_perm(c, d, 0x7362);
    out[0] = __byte_perm(t0, t2, 0x5410);
    out[1] = __byte_perm(t0, t2, 0x7632);
    out[2] = __byte_perm(t1, t3, 0x5410);
    out[3] = __byte_perm(t1, t3, 0x7632);
}

// Quantize xs[0..K) (shared memory floats, 16-byte aligned, K a multiple of
// 256) into the B layout.  One warp per 256-value block: lane 4*gl + t
// converts values 16G+4t..+3 of groups G = gl and gl + 8 of the block.
__device__ __forceinline__ void build_xq(const float* xs, int K, uint32_t* xb, int* sb) {
    const int lane = threadIdx.x & 31, t = lane & 3, gl = lane >> 2;
    for (int blk = threadIdx.x >> 5; blk < K / 256; blk += blockDim.x >> 5) {
        const float4 u = reinterpret_cast<const float4*>(xs + blk * 256)[lane];
        const float4 v = reinterpret_cast<const float4*>(xs + blk * 256 + 128)[lane];
        float mx = fmaxf(fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w))),
                         fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const bool fin = isfinite(u.x) && isfinite(u.y) && isfinite(u.z) && isfinite(u.w) && isfinite(v.x) &&
                         isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
        const int E = mx > 0.f ? (int)((__float_as_uint(mx) >> 23) & 255u) - 127 : -126;
        const int S = __all_sync(0xffffffffu, fin) ? 54 - (E < -126 ? -126 : E) : kSbNonFinite;
        if (lane == 0) sb[blk] = S;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float4 q = h ? v : u;
            uint32_t hi[4], lo[4], w[4];
            const int Sq = S == kSbNonFinite ? 0 : S;   // the limbs are unused then (factor NaN)
            to_fixed(q.x, Sq, hi[0], lo[0]);
            to_fixed(q.y, Sq, hi[1], lo[1]);
            to_fixed(q.z, Sq, hi[2], lo[2]);
            to_fixed(q.w, Sq, hi[3], lo[3]);
            uint32_t* dst = xb + (size_t)(blk * 16 + 8 * h + gl) * kXG + t;
            transpose4(lo[0], lo[1], lo[2], lo[3], w);
#pragma unroll
            for (int n = 0; n < 4; ++n) dst[4 * n] = w[n];
            transpose4(hi[0], hi[1], hi[2], hi[3], w);
#pragma unroll
            for (int n = 0; n < 3; ++n) dst[4 * (4 + n)] = w[n];
            dst[28] = 0x01010101u;
        }
    }
}

// Weight of accumulator register r of lane (g,t): limb n = 2t + (r & 1)
// carries 2^(8n).  Column 7 (sum of the integer weights) is folded into limb
// 6 in the int32 domain before conversion (Acc::flush), so its weight is 0.
__device__ __forceinline__ double limb_weight(int lane, int r) {
    const int n = 2 * (lane & 3) + (r & 1);
    return n < kLimbs ? pow2d(8 * n) : 0.0;
}

// ---- tensor-core primitives -------------------------------------------------
__device__ __forceinline__ void mma_k32(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_k16(int d[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Per-lane accumulation state of one 16-row tile: int32 per block, double overall.
struct Acc {
    int i[4];
    double d[4];
    __device__ __forceinline__ void zero_block() { i[0] = i[1] = i[2] = i[3] = 0; }
    __device__ __forceinline__ void add(const int D[4], int s_lo, int s_hi) {   // s_lo: row g, s_hi: row g+8
        i[0] += s_lo * D[0];
        i[1] += s_lo * D[1];
        i[2] += s_hi * D[2];
        i[3] += s_hi * D[3];
    }
    // fold this block: f_lo / f_hi = block factor of rows g / g+8 (d * 2^-S / c)
    __device__ __forceinline__ void flush(double f_lo, double f_hi, const double lw[2]) {
        // lane t = 3 holds limb 6 (offset bit 7 of that byte) and column 7:
        // remove 2^55 * sum(w) exactly: limb6 -= 128 * column7.
        if ((threadIdx.x & 3) == 3) {
            i[0] -= 128 * i[1];
            i[2] -= 128 * i[3];
        }
        d[0] = fma((double)i[0], f_lo * lw[0], d[0]);
        d[1] = fma((double)i[1], f_lo * lw[1], d[1]);
        d[2] = fma((double)i[2], f_hi * lw[0], d[2]);
        d[3] = fma((double)i[3], f_hi * lw[1], d[3]);
    }
    // After the last block: lane (g, 0) returns rows g (lo) and g+8 (hi).
    __device__ __forceinline__ void finish(double& lo, double& hi) const {
        double a = d[0] + d[1], b = d[2] + d[3];
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        b += __shfl_xor_sync(0xffffffffu, b, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        b += __shfl_xor_sync(0xffffffffu, b, 2);
        lo = a;
        hi = b;
    }
};

// Small lattice tables staged in shared memory by the expert kernels.
struct IqTab {
    uint32_t grid2[512][2];      // IQ2_XS lattice, 8 magnitude bytes per entry     4 KB
    uint32_t grid3[256];         // IQ3_XXS lattice, 4 magnitude bytes per entry    1 KB
    uint8_t ksigns[128];         // 7 stored sign bits + even parity bit
};

// Negate byte k of `mag` when bit k of `nib` is set (|values| < 128, no carries).
__device__ __forceinline__ uint32_t signed_bytes(uint32_t mag, uint32_t nib) {
    const uint32_t m1 = ((nib & 15u) * 0x00204081u) & 0x01010101u;
    return (mag ^ (m1 * 255u)) + m1;
}

// ---- per-format tile dots ---------------------------------------------------
// One warp; rows r0 (= g) and r1 (= g+8) of a 16-row tile staged in shared
// memory; blocks [b0, b1) of the row.  Accumulates into acc.

// Codebook lookup of all eight nibbles of q: lo = entries of the low nibbles
// of bytes 0..3, hi = entries of the high nibbles.  __byte_perm reads only the
// low 3 bits of each selector nibble, so the first two permutes fetch entries
// n & 7 from the lower and upper halves of the 16-byte table; a third picks
// the half by bit 3 of each nibble; two more split low and high nibbles.
__device__ __forceinline__ void kv_lookup8(uint32_t q, const uint32_t K[4], uint32_t& lo, uint32_t& hi) {
    const uint32_t pick = ((q & 0x88888888u) >> 1) | 0x32103210u;   // nibble k -> byte k or 4 + k
    const uint32_t r0 = __byte_perm(__byte_perm(K[0], K[1], q), __byte_perm(K[2], K[3], q), pick);
    const uint32_t r1 = __byte_perm(__byte_perm(K[0], K[1], q >> 16), __byte_perm(K[2], K[3], q >> 16), pick >> 16);
    lo = __byte_perm(r0, r1, 0x6420);
    hi = __byte_perm(r0, r1, 0x7531);
}

// IQ4_XS: m16n8k32, natural order (lane t: bytes 4t..4t+3 of each 16-byte
// group -> values 4t.. (low nibbles) and 16+4t.. (high nibbles)).
__device__ __forceinline__ void dot_iq4_xs_mma(const uint8_t* r0, const uint8_t* r1, int b0, int b1, const XQ& x,
                                               const uint32_t K[4], int lane, Acc& acc) {
    const double lw[2] = {limb_weight(lane, 0), limb_weight(lane, 1)};
    const int t = lane & 3;
    for (int b = b0; b < b1; ++b) {
        const uint8_t* p0 = r0 + b * 136;
        const uint8_t* p1 = r1 + b * 136;
        const uint32_t sh0 = ld16(p0 + 2), sh1 = ld16(p1 + 2);
        const uint32_t sl0 = *reinterpret_cast<const uint32_t*>(p0 + 4);
        const uint32_t sl1 = *reinterpret_cast<const uint32_t*>(p1 + 4);
        acc.zero_block();
#pragma unroll 4
        for (int ib = 0; ib < 8; ++ib) {
            const int ls0 = ((sl0 >> (4 * ib)) & 15) | (((sh0 >> (2 * ib)) & 3) << 4);
            const int ls1 = ((sl1 >> (4 * ib)) & 15) | (((sh1 >> (2 * ib)) & 3) << 4);
            const uint32_t q0 = *reinterpret_cast<const uint32_t*>(p0 + 8 + 16 * ib + 4 * t);
            const uint32_t q1 = *reinterpret_cast<const uint32_t*>(p1 + 8 + 16 * ib + 4 * t);
            uint32_t a0, a1, a2, a3;
            kv_lookup8(q0, K, a0, a2);
            kv_lookup8(q1, K, a1, a3);
            const int G = b * 16 + 2 * ib;
            int D[4];
            mma_k32(D, a0, a1, a2, a3, x.b[G * kXG + lane], x.b[(G + 1) * kXG + lane]);
            acc.add(D, ls0 - 32, ls1 - 32);
        }
        const double sc = blk_pow2(x.s[b], 0);
        acc.flush((double)h2f(ld16(p0)) * sc, (double)h2f(ld16(p1)) * sc, lw);
    }
}

// IQ2_XS: m16n8k16 per 16-value scale group; lane t takes values 4t..4t+3 =
// half (t&1) of grid entry 2G' + (t>>1).
__device__ __forceinline__ void dot_iq2_xs_mma(const uint8_t* r0, const uint8_t* r1, int b0, int b1, const XQ& x,
                                               const IqTab& T, int lane, Acc& acc) {
    const double lw[2] = {limb_weight(lane, 0), limb_weight(lane, 1)};
    const int t = lane & 3, half = t & 1, sub = t >> 1;
    for (int b = b0; b < b1; ++b) {
        const uint8_t* p0 = r0 + b * 74;
        const uint8_t* p1 = r1 + b * 74;
        acc.zero_block();
#pragma unroll 4
        for (int gq = 0; gq < 16; ++gq) {       // 16-value group: ib32 = gq/2, scale nibble gq&1
            const int e = 2 * gq + sub;           // grid entry index within the block
            const uint32_t q0 = ld16(p0 + 2 + 2 * e), q1 = ld16(p1 + 2 + 2 * e);
            const uint32_t s0 = T.ksigns[q0 >> 9], s1 = T.ksigns[q1 >> 9];
            const uint32_t a0 = signed_bytes(T.grid2[q0 & 511u][half], s0 >> (4 * half));
            const uint32_t a1 = signed_bytes(T.grid2[q1 & 511u][half], s1 >> (4 * half));
            const int sc0 = 1 + 2 * ((p0[66 + (gq >> 1)] >> (4 * (gq & 1))) & 15);
            const int sc1 = 1 + 2 * ((p1[66 + (gq >> 1)] >> (4 * (gq & 1))) & 15);
            int D[4];
            mma_k16(D, a0, a1, x.b[(b * 16 + gq) * kXG + lane]);
            acc.add(D, sc0, sc1);
        }
        const double sc = blk_pow2(x.s[b], -3);
        acc.flush((double)h2f(ld16(p0)) * sc, (double)h2f(ld16(p1)) * sc, lw);
    }
}

// IQ2R (the persistent kernel's re-laid IQ2_XS, qx_mega.cu): row = fp16
// block scales d (hdr bytes), then per block 16 scale bytes (1 + 2s of each
// 16-value group) and 4 chunks of 32 bytes; chunk t holds, for groups
// gq = 0..15, the u16 of nibble codes of values 16gq+4t..+3.  A code indexes
// the signed lattice values {0, 8, 25, 43, 0, -8, -25, -43} (bytes of T0:T1;
// code = 1..3 for magnitude 8, 25, 43, plus 4 when negative),
// so one byte permute decodes 4 weights.  Same integer sums and block factors
// as dot_iq2_xs_mma (d/8 * (1+2s) * sign * grid).
constexpr uint32_t kIq2rT0 = 0x2b190800u, kIq2rT1 = 0xd5e7f800u;
constexpr int kIq2rBlock = 144;
__device__ __forceinline__ void dot_iq2r_mma(const uint8_t* r0, const uint8_t* r1, int hdr, int b0, int b1, const XQ& x,
                                             int lane, Acc& acc) {
    const double lw[2] = {limb_weight(lane, 0), limb_weight(lane, 1)};
    const int t = lane & 3;
    for (int b = b0; b < b1; ++b) {
        const uint8_t* p0 = r0 + hdr + b * kIq2rBlock;
        const uint8_t* p1 = r1 + hdr + b * kIq2rBlock;
        const uint4 s0 = *reinterpret_cast<const uint4*>(p0), s1 = *reinterpret_cast<const uint4*>(p1);
        const uint4 c0a = *reinterpret_cast<const uint4*>(p0 + 16 + 32 * t);
        const uint4 c0b = *reinterpret_cast<const uint4*>(p0 + 32 + 32 * t);
        const uint4 c1a = *reinterpret_cast<const uint4*>(p1 + 16 + 32 * t);
        const uint4 c1b = *reinterpret_cast<const uint4*>(p1 + 32 + 32 * t);
        const uint32_t w0[8] = {c0a.x, c0a.y, c0a.z, c0a.w, c0b.x, c0b.y, c0b.z, c0b.w};
        const uint32_t w1[8] = {c1a.x, c1a.y, c1a.z, c1a.w, c1b.x, c1b.y, c1b.z, c1b.w};
        const uint32_t sv0[4] = {s0.x, s0.y, s0.z, s0.w}, sv1[4] = {s1.x, s1.y, s1.z, s1.w};
        acc.zero_block();
#pragma unroll
        for (int gq = 0; gq < 16; ++gq) {
            const uint32_t q0 = (gq & 1) ? (w0[gq >> 1] >> 16) : w0[gq >> 1];
            const uint32_t q1 = (gq & 1) ? (w1[gq >> 1] >> 16) : w1[gq >> 1];
            const uint32_t a0 = __byte_perm(kIq2rT0, kIq2rT1, q0), a1 = __byte_perm(kIq2rT0, kIq2rT1, q1);
            const int sc0 = (int)__byte_perm(sv0[gq >> 2], 0u, 0x4440u | (gq & 3));
            const int sc1 = (int)__byte_perm(sv1[gq >> 2], 0u, 0x4440u | (gq & 3));
            int D[4];
            mma_k16(D, a0, a1, x.b[(b * 16 + gq) * kXG + lane]);
            acc.add(D, sc0, sc1);
        }
        const double sc = blk_pow2(x.s[b], -3);
        acc.flush((double)h2f(ld16(r0 + 2 * b)) * sc, (double)h2f(ld16(r1 + 2 * b)) * sc, lw);
    }
}

// R4 (the persistent kernel's re-laid IQ4_XS and IQ3_XXS, qx_mega.cu): each
// weight is a 4-bit index into a 16-entry signed byte table K (IQ4_NL values,
// or +-IQ3_XXS lattice magnitudes), every 32-value group has one scale byte
// (IQ4_XS: ls - 32, signed; IQ3_XXS: 1 + 2s).  Row = fp16 block scales d
// (r4_hdr bytes), the 8 scale bytes of every block, then from r4_codes
// (16-byte aligned) per block 4 chunks
// of 32 bytes: chunk t holds for groups ib = 0..7 the u32 whose nibbles 0..3
// index values 32ib+4t..+3 and nibbles 4..7 values 32ib+16+4t..+3 (the A
// fragments a0/a2 of lane t for m16n8k32).  Row bytes are 16 mod 32 so the
// 16-byte code loads of the 8 rows a warp reads are conflict-free.
__host__ __device__ constexpr int r4_hdr(int nblk) { return (2 * nblk + 15) / 16 * 16; }
__host__ __device__ constexpr int r4_codes(int nblk) { return (r4_hdr(nblk) + 8 * nblk + 15) / 16 * 16; }
__host__ __device__ constexpr size_t r4_row_bytes(int K) {
    return ((size_t)r4_codes(K / 256) + (size_t)(K / 256) * 128 + 47) / 32 * 32 - 16;
}
constexpr uint32_t kIq3rK[4] = {0x1c140c04u, 0x3e342c24u, 0xe4ecf4fcu, 0xc2ccd4dcu};   // 4..62, -4..-62

// 8 codes -> lo = table bytes of nibbles 0..3, hi = of nibbles 4..7.
__device__ __forceinline__ void r4_lookup8(uint32_t q, const uint32_t K[4], uint32_t& lo, uint32_t& hi) {
    const uint32_t pick = ((q >> 1) & 0x44444444u) | 0x32103210u;   // nibble n -> byte n or 4 + n
    lo = __byte_perm(__byte_perm(K[0], K[1], q), __byte_perm(K[2], K[3], q), pick);
    const uint32_t q2 = q >> 16;
    hi = __byte_perm(__byte_perm(K[0], K[1], q2), __byte_perm(K[2], K[3], q2), pick >> 16);
}

template <bool SIGNED_SCALE>
__device__ __forceinline__ void dot_r4_mma(const uint8_t* r0, const uint8_t* r1, int nblk, int b0, int b1, int fexp,
                                           const XQ& x, const uint32_t K[4], int lane, Acc& acc) {
    const double lw[2] = {limb_weight(lane, 0), limb_weight(lane, 1)};
    const int t = lane & 3, hdr = r4_hdr(nblk), cod = r4_codes(nblk);
    for (int b = b0; b < b1; ++b) {
        const uint2 s0 = *reinterpret_cast<const uint2*>(r0 + hdr + 8 * b);
        const uint2 s1 = *reinterpret_cast<const uint2*>(r1 + hdr + 8 * b);
        const uint4 c0a = *reinterpret_cast<const uint4*>(r0 + cod + 128 * b + 32 * t);
        const uint4 c0b = *reinterpret_cast<const uint4*>(r0 + cod + 128 * b + 32 * t + 16);
        const uint4 c1a = *reinterpret_cast<const uint4*>(r1 + cod + 128 * b + 32 * t);
        const uint4 c1b = *reinterpret_cast<const uint4*>(r1 + cod + 128 * b + 32 * t + 16);
        const uint32_t w0[8] = {c0a.x, c0a.y, c0a.z, c0a.w, c0b.x, c0b.y, c0b.z, c0b.w};
        const uint32_t w1[8] = {c1a.x, c1a.y, c1a.z, c1a.w, c1b.x, c1b.y, c1b.z, c1b.w};
        acc.zero_block();
#pragma unroll
        for (int ib = 0; ib < 8; ++ib) {
            uint32_t a0, a1, a2, a3;
            r4_lookup8(w0[ib], K, a0, a2);
            r4_lookup8(w1[ib], K, a1, a3);
            const uint32_t v0 = ((ib < 4 ? s0.x : s0.y) >> (8 * (ib & 3))) & 0xffu;
            const uint32_t v1 = ((ib < 4 ? s1.x : s1.y) >> (8 * (ib & 3))) & 0xffu;
            const int sc0 = SIGNED_SCALE ? (int)(int8_t)v0 : (int)v0, sc1 = SIGNED_SCALE ? (int)(int8_t)v1 : (int)v1;
            const int G = b * 16 + 2 * ib;
            int D[4];
            mma_k32(D, a0, a1, a2, a3, x.b[G * kXG + lane], x.b[(G + 1) * kXG + lane]);
            acc.add(D, sc0, sc1);
        }
        const double sc = blk_pow2(x.s[b], fexp);
        acc.flush((double)h2f(ld16(r0 + 2 * b)) * sc, (double)h2f(ld16(r1 + 2 * b)) * sc, lw);
    }
}

// IQ3_XXS: m16n8k32 per 32-value group; lane t: grid index bytes t (values
// 4t..) and 4+t (values 16+4t..); sign group = t>>1 resp. 2+(t>>1), half t&1.
__device__ __forceinline__ void dot_iq3_xxs_mma(const uint8_t* r0, const uint8_t* r1, int b0, int b1, const XQ& x,
                                                const IqTab& T, int lane, Acc& acc) {
    const double lw[2] = {limb_weight(lane, 0), limb_weight(lane, 1)};
    const int t = lane & 3, half = t & 1, sg = t >> 1;
    for (int b = b0; b < b1; ++b) {
        const uint8_t* p0 = r0 + b * 98;
        const uint8_t* p1 = r1 + b * 98;
        acc.zero_block();
#pragma unroll 2
        for (int ib = 0; ib < 8; ++ib) {
            const uint32_t aux0 = ld32u(p0 + 66 + 4 * ib), aux1 = ld32u(p1 + 66 + 4 * ib);
            const uint32_t sA0 = T.ksigns[(aux0 >> (7 * sg)) & 127u], sB0 = T.ksigns[(aux0 >> (7 * (2 + sg))) & 127u];
            const uint32_t sA1 = T.ksigns[(aux1 >> (7 * sg)) & 127u], sB1 = T.ksigns[(aux1 >> (7 * (2 + sg))) & 127u];
            const uint32_t a0 = signed_bytes(T.grid3[p0[2 + 8 * ib + t]], sA0 >> (4 * half));
            const uint32_t a2 = signed_bytes(T.grid3[p0[2 + 8 * ib + 4 + t]], sB0 >> (4 * half));
            const uint32_t a1 = signed_bytes(T.grid3[p1[2 + 8 * ib + t]], sA1 >> (4 * half));
            const uint32_t a3 = signed_bytes(T.grid3[p1[2 + 8 * ib + 4 + t]], sB1 >> (4 * half));
            const int G = b * 16 + 2 * ib;
            int D[4];
            mma_k32(D, a0, a1, a2, a3, x.b[G * kXG + lane], x.b[(G + 1) * kXG + lane]);
            acc.add(D, 1 + 2 * (int)(aux0 >> 28), 1 + 2 * (int)(aux1 >> 28));
        }
        const double sc = blk_pow2(x.s[b], -2);
        acc.flush((double)h2f(ld16(p0)) * sc, (double)h2f(ld16(p1)) * sc, lw);
    }
}

// IQ2_S (82-byte blocks: d, qs[32] low index bytes, signs[32], qh[8], scales[8];
// src/qx_format.c:1961-1984): w = d/8 * (1+2s) * g * sign, g from the
// 1024-entry lattice, index = qs[e] | (2 bits of qh).  Same lane mapping as
// IQ2_XS: m16n8k16 per 16-value group, lane t takes half (t&1) of entry
// 2gq + (t>>1).  grid: the lattice in global memory (read through L1).
__device__ __forceinline__ void dot_iq2_s_mma(const uint8_t* r0, const uint8_t* r1, int b0, int b1, const XQ& x,
                                              const uint32_t (*grid)[2], int lane, Acc& acc) {
    const double lw[2] = {limb_weight(lane, 0), limb_weight(lane, 1)};
    const int t = lane & 3, half = t & 1, sub = t >> 1;
    for (int b = b0; b < b1; ++b) {
        const uint8_t* p0 = r0 + b * 82;
        const uint8_t* p1 = r1 + b * 82;
        acc.zero_block();
#pragma unroll 4
        for (int gq = 0; gq < 16; ++gq) {
            const int e = 2 * gq + sub, ib = e >> 2, l = e & 3;
            const uint32_t i0 = p0[2 + e] | (((uint32_t)p0[66 + ib] << (8 - 2 * l)) & 0x300u);
            const uint32_t i1 = p1[2 + e] | (((uint32_t)p1[66 + ib] << (8 - 2 * l)) & 0x300u);
            const uint32_t a0 = signed_bytes(__ldg(&grid[i0][half]), (uint32_t)p0[34 + e] >> (4 * half));
            const uint32_t a1 = signed_bytes(__ldg(&grid[i1][half]), (uint32_t)p1[34 + e] >> (4 * half));
            const int sc0 = 1 + 2 * ((p0[74 + (gq >> 1)] >> (4 * (gq & 1))) & 15);
            const int sc1 = 1 + 2 * ((p1[74 + (gq >> 1)] >> (4 * (gq & 1))) & 15);
            int D[4];
            mma_k16(D, a0, a1, x.b[(b * 16 + gq) * kXG + lane]);
            acc.add(D, sc0, sc1);
        }
        const double sc = blk_pow2(x.s[b], -3);
        acc.flush((double)h2f(ld16(p0)) * sc, (double)h2f(ld16(p1)) * sc, lw);
    }
}

// IQ3_S (110-byte blocks: d, qs[64], qh[8], signs[32], scales[4];
// src/qx_format.c:1987-2030): w = d * (1+2s) * g * sign, g from the 512-entry
// lattice; in 32-value group ib the 4-value quad q has index qs[8ib+q] | bit q
// of qh[ib] << 8 and sign nibble q&1 of signs[4ib + q/2]; s is nibble ib&1 of
// scales[ib/2].  m16n8k32 per group, lane t: quads t and 4+t.
__device__ __forceinline__ void dot_iq3_s_mma(const uint8_t* r0, const uint8_t* r1, int b0, int b1, const XQ& x,
                                              const uint32_t* grid, int lane, Acc& acc) {
    const double lw[2] = {limb_weight(lane, 0), limb_weight(lane, 1)};
    const int t = lane & 3;
    for (int b = b0; b < b1; ++b) {
        const uint8_t* p0 = r0 + b * 110;
        const uint8_t* p1 = r1 + b * 110;
        acc.zero_block();
#pragma unroll 2
        for (int ib = 0; ib < 8; ++ib) {
            uint32_t a[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {                 // a0: row 0 quad t, a1: row 1 quad t, a2/a3: quad 4+t
                const uint8_t* p = (k & 1) ? p1 : p0;
                const int q = (k >> 1) * 4 + t;
                const uint32_t idx = p[2 + 8 * ib + q] | ((((uint32_t)p[66 + ib] >> q) & 1u) << 8);
                a[k] = signed_bytes(__ldg(&grid[idx]), (uint32_t)p[74 + 4 * ib + (q >> 1)] >> (4 * (q & 1)));
            }
            const int s0 = 1 + 2 * ((p0[106 + (ib >> 1)] >> (4 * (ib & 1))) & 15);
            const int s1 = 1 + 2 * ((p1[106 + (ib >> 1)] >> (4 * (ib & 1))) & 15);
            const int G = b * 16 + 2 * ib;
            int D[4];
            mma_k32(D, a[0], a[1], a[2], a[3], x.b[G * kXG + lane], x.b[(G + 1) * kXG + lane]);
            acc.add(D, s0, s1);
        }
        const double sc = blk_pow2(x.s[b], 0);
        acc.flush((double)h2f(ld16(p0)) * sc, (double)h2f(ld16(p1)) * sc, lw);
    }
}

// Q5_K (176-byte blocks: d, dmin, scales[12], qh[32], qs[128];
// src/qx_format.c:2112-2145): w = d*sc*q - dmin*m is affine, and the
// subtraction rounds, so w is not an exact integer multiple: each weight is
// decoded to the reference's float with the same operations (no contraction)
// and multiplied into a double accumulator (the product is exact, the FMA
// rounds like the reference's add).  One warp per row; lane l takes values
// 64j+l and 64j+32+l of every block.  Returns the warp's double sum.
__device__ __forceinline__ void q5k_scale_min(int j, const uint8_t* q, uint32_t& sc, uint32_t& m) {
    if (j < 4) { sc = q[j] & 63u; m = q[j + 4] & 63u; }
    else { sc = (q[j + 4] & 15u) | ((q[j - 4] >> 6) << 4); m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
}

__device__ inline double dot_q5_k_row(const uint8_t* row, int nblk, const float* xs, int lane) {
    double acc = 0.0;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + (size_t)b * 176;
        const float d = h2f(ld16(blk)), dmin = h2f(ld16(blk + 2));
        const uint8_t qh = blk[16 + lane];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint8_t qv = blk[48 + 32 * j + lane];
            uint32_t sc, m;
            q5k_scale_min(2 * j, blk + 4, sc, m);
            const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
            q5k_scale_min(2 * j + 1, blk + 4, sc, m);
            const float d2 = __fmul_rn(d, (float)sc), m2 = __fmul_rn(dmin, (float)m);
            const int qa = (qv & 15) | (((qh >> (2 * j)) & 1) << 4), qb = (qv >> 4) | (((qh >> (2 * j + 1)) & 1) << 4);
            const float wa = __fsub_rn(__fmul_rn(d1, (float)qa), m1), wb = __fsub_rn(__fmul_rn(d2, (float)qb), m2);
            const int ia = b * 256 + 64 * j + lane;
            acc = fma((double)wa, (double)xs[ia], acc);
            acc = fma((double)wb, (double)xs[ia + 32], acc);
        }
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

// R8 (the persistent kernel's re-laid Q6_K head, qx_mega.cu): row = fp16
// block scales d (r4_hdr bytes), then per block 16 int8 group scales and 16
// units of 16 bytes; unit 4 q4 + t holds for groups gq = 4q4..4q4+3 the int8
// weights q - 32 of values 16gq+4t..+3 (lane t's A fragments of m16n8k16).
// Block = 272 bytes; row bytes 64 mod 128, so the 8 units a quarter warp
// loads (rows g, g+1; t = 0..3) fall in 8 different bank groups.  The same
// integer weights, group scales and block factors as dot_q6_k_mma, with no
// decoding.
__host__ __device__ constexpr size_t r8_row_bytes(int K) {
    return ((size_t)r4_hdr(K / 256) + (size_t)(K / 256) * 272 + 63) / 128 * 128 + 64;
}
__device__ __forceinline__ void dot_r8_mma(const uint8_t* r0, const uint8_t* r1, int nblk, int b0, int b1, const XQ& x,
                                           int lane, Acc& acc) {
    const double lw[2] = {limb_weight(lane, 0), limb_weight(lane, 1)};
    const int t = lane & 3, hdr = r4_hdr(nblk);
    for (int b = b0; b < b1; ++b) {
        const uint8_t* p0 = r0 + hdr + 272 * b;
        const uint8_t* p1 = r1 + hdr + 272 * b;
        const uint4 s0 = *reinterpret_cast<const uint4*>(p0), s1 = *reinterpret_cast<const uint4*>(p1);
        const uint32_t sv0[4] = {s0.x, s0.y, s0.z, s0.w}, sv1[4] = {s1.x, s1.y, s1.z, s1.w};
        acc.zero_block();
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
            const uint4 v0 = *reinterpret_cast<const uint4*>(p0 + 16 + 64 * q4 + 16 * t);
            const uint4 v1 = *reinterpret_cast<const uint4*>(p1 + 16 + 64 * q4 + 16 * t);
            const uint32_t w0[4] = {v0.x, v0.y, v0.z, v0.w}, w1[4] = {v1.x, v1.y, v1.z, v1.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int gq = 4 * q4 + j;
                const int sc0 = (int)(int8_t)((sv0[q4] >> (8 * j)) & 0xffu);
                const int sc1 = (int)(int8_t)((sv1[q4] >> (8 * j)) & 0xffu);
                int D[4];
                mma_k16(D, w0[j], w1[j], x.b[(b * 16 + gq) * kXG + lane]);
                acc.add(D, sc0, sc1);
            }
        }
        const double sc = blk_pow2(x.s[b], 0);
        acc.flush((double)h2f(ld16(r0 + 2 * b)) * sc, (double)h2f(ld16(r1 + 2 * b)) * sc, lw);
    }
}

// Q6_K: m16n8k16 per 16-value scale group.  Values of a 128-value half:
// pos = 32*s + l (section s, l in 0..31); lane t takes l = 16*lh + 4t .. +3.
__device__ __forceinline__ uint32_t q6_word(uint32_t ql, uint32_t qh, int s) {
    const uint32_t lo = (s < 2 ? ql : ql >> 4) & 0x0f0f0f0fu;
    const uint32_t hb = ((qh >> (2 * s)) & 0x03030303u) << 4;
    return ((lo | hb | 0x80808080u) - 0x20202020u) ^ 0x80808080u;   // bytewise q - 32
}

__device__ __forceinline__ void dot_q6_k_mma(const uint8_t* r0, const uint8_t* r1, int b0, int b1, const XQ& x,
                                             int lane, Acc& acc) {
    const double lw[2] = {limb_weight(lane, 0), limb_weight(lane, 1)};
    const int t = lane & 3;
    for (int b = b0; b < b1; ++b) {
        const uint8_t* p0 = r0 + b * 210;
        const uint8_t* p1 = r1 + b * 210;
        const int8_t* c0 = reinterpret_cast<const int8_t*>(p0 + 192);
        const int8_t* c1 = reinterpret_cast<const int8_t*>(p1 + 192);
        acc.zero_block();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int lh = 0; lh < 2; ++lh) {
                const int l = 16 * lh + 4 * t;
                const uint32_t qlA0 = ld32u(p0 + 64 * h + l), qlB0 = ld32u(p0 + 64 * h + 32 + l);
                const uint32_t qh0 = ld32u(p0 + 128 + 32 * h + l);
                const uint32_t qlA1 = ld32u(p1 + 64 * h + l), qlB1 = ld32u(p1 + 64 * h + 32 + l);
                const uint32_t qh1 = ld32u(p1 + 128 + 32 * h + l);
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint32_t a0 = q6_word((s & 1) ? qlB0 : qlA0, qh0, s);
                    const uint32_t a1 = q6_word((s & 1) ? qlB1 : qlA1, qh1, s);
                    const int gq = 8 * h + 2 * s + lh;      // 16-value group index in the block
                    int D[4];
                    mma_k16(D, a0, a1, x.b[(b * 16 + gq) * kXG + lane]);
                    const int si = 8 * h + lh + 2 * s;
                    acc.add(D, (int)c0[si], (int)c1[si]);
                }
            }
        }
        const double sc = blk_pow2(x.s[b], 0);
        acc.flush((double)h2f(ld16(p0 + 208)) * sc, (double)h2f(ld16(p1 + 208)) * sc, lw);
    }
}

}  // namespace qx
