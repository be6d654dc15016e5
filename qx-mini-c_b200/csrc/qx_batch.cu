// Batched MoE FFN for many tokens at once (prefill / batched decode): the
// grouped-expert contraction on the 5th-generation tensor cores.
//
// The reference has no batched path: its prefill and decode run
// qx_apply_real_moe_layer (src/qx_format.c:5198-5310) one token at a time.
// For N tokens this file computes the same per-token result -
//   RMSNorm(ffn_norm) -> F32 router in double -> softmax -> top-8 (strict >,
//   lowest index on ties) -> renormalised weights -> per selected expert
//   IQ2_XS gate/up, SwiGLU in double, IQ3_XXS down -> rank-order weighted sum
//   -> residual add
// - with the expert projections done as grouped GEMMs: the tokens routed to
// an expert form the columns of one contraction against that expert's rows.
//
// Exact integer contraction (the same arithmetic as the decode path,
// qx_imma.cuh): each weight is an integer A = (1 + 2s) * g times the block
// factor d; each activation block is a 56-bit fixed-point integer split into
// 7 unsigned byte limbs plus a column of ones.  A (up to +-1922) does not fit
// an int8 operand, so it is split into two int8 digits, A = 64 * hi + lo
// (hi = A >> 6, lo = A & 63), and tcgen05.mma kind::i8 (s8 x u8 -> s32)
// forms both digit products for a 128-row x 16-token tile (N = 16 x 8 limb
// columns) of one 256-value block into two TMEM accumulators.  The epilogue
// reads them back (tcgen05.ld), rebuilds the exact block integer per row and
// token, and folds it into a double accumulator with the block factor
// d * 2^-S.  Operands are staged in shared memory in the UMMA K-major
// no-swizzle layout: core matrices of 8 rows x 16 bytes, 128 B apart along K
// (LBO) and 256 B apart along M/N (SBO), one 4 KB slab per 32 values of K.
//
// The weights come from the step kernel's re-laid copies (IQ2R gate/up, R4
// down: the same integers and scales as the GGUF blocks); each CTA decodes
// its 128 rows of one block into the hi/lo slabs with byte-permute table
// lookups, stages its tokens' limbs, and one thread issues the MMAs.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdio>
#include <vector>

#include "qx_batch.h"
#include "qx_common.cuh"

namespace qx {
namespace {

constexpr int kGemmThreads = 128;   // 4 warps: one TMEM lane quarter each
constexpr int kTokTile = 16;        // tokens (or expert slots) per tile: N = 128 columns
constexpr int kTiles = 2;           // column tiles per CTA: each decoded weight block serves both
constexpr int kRowTile = 128;       // weight rows per tile: M = 128
constexpr int kSlab = 4096;         // bytes of one 32-value K step of a 128-row operand
constexpr int kTmemCols = 256;      // hi accumulator in columns [0, 128), lo in [128, 256)
constexpr int kMaxBlk = 16;         // 256-value blocks per row (K <= 4096)
constexpr uint32_t kSmemGemm = 3 * 8 * kSlab + 128;    // A hi, A lo, B (8 K steps each) + alignment

// ---- tcgen05 primitives (PTX ISA 8.7, sm_100a) ------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory matrix descriptor, K-major, no swizzle: start address, leading
// byte offset (next core matrix along K), stride byte offset (next 8-row group
// along M/N), version 1 (bits 46-47), layout type 0.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// Instruction descriptor for kind::i8: D s32 (bits 4-5 = 2), A s8 (bits 7-9 =
// 1), B u8 (bits 10-12 = 0), both K-major, N >> 3 at bits 17-22, M >> 4 at 24-28.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ---- operand decoding ---------------------------------------------------------
// Byte offset of (row r, value k) of a 128-row x 256-value operand in the
// K-major no-swizzle layout: slab k / 32, 8-row group r / 8 (256 B), core
// matrix (k % 32) / 16 (128 B), row r % 8 (16 B), byte k % 16.
__device__ __forceinline__ uint32_t op_off(int r, int k) {
    return (uint32_t)((k >> 5) * kSlab + (r >> 3) * 256 + ((k >> 4) & 1) * 128 + (r & 7) * 16 + (k & 15));
}

// Word w (a compile-time index once unrolled) of a register array of uint4.
template <int N>
__device__ __forceinline__ uint32_t word_of(const uint4 (&v)[N], int w) {
    const uint4 q = v[w >> 2];
    return (w & 3) == 0 ? q.x : (w & 3) == 1 ? q.y : (w & 3) == 2 ? q.z : q.w;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) | ((uint32_t)(d & 255) << 24);
}

// IQ2R block (16 group-scale bytes 1 + 2s, then for tt = 0..3 and group gq a
// u16 of four 3-bit codes: magnitude index 1..3 for {8, 25, 43} plus 4 when
// negative, of values 16 gq + 4 tt + j): the 256 integers (1 + 2s) * g of one
// row as hi/lo digits into the operand slabs.
// One row's source bytes of one block: the group scales and the 128 code
// bytes, loaded a block ahead so the global latency hides behind the MMAs.
template <int NW>
struct RowSrcN {
    uint4 sv;
    uint4 cw[NW];
};
using RowSrc = RowSrcN<8>;

template <int NW>
__device__ __forceinline__ void load_src(const uint8_t* scales, const uint8_t* codes, bool scales16, RowSrcN<NW>& s) {
    if (scales16) {
        s.sv = *reinterpret_cast<const uint4*>(scales);
    } else {
        const uint2 v = *reinterpret_cast<const uint2*>(scales);
        s.sv = make_uint4(v.x, v.y, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < NW; ++i) s.cw[i] = *reinterpret_cast<const uint4*>(codes + 16 * i);
}

// R8 block (the re-laid Q6_K head: 16 int8 group scales, then 16 units of 16
// bytes; unit 4 (gq >> 2) + t holds the int8 weights q - 32 of values
// 16 gq + 4 t .. + 3 at byte 4 (gq & 3)): A = scale * (q - 32) per value,
// |A| <= 4096, as hi/lo digits.
__device__ __forceinline__ void decode_r8_row(const RowSrcN<16>& src, int r, uint8_t* ahi, uint8_t* alo) {
    const uint32_t sw[4] = {src.sv.x, src.sv.y, src.sv.z, src.sv.w};
#pragma unroll
    for (int gq = 0; gq < 16; ++gq) {
        const int sc = (int)(int8_t)(uint8_t)(sw[gq >> 2] >> (8 * (gq & 3)));
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t W = word_of(src.cw, 16 * (gq >> 2) + 4 * t + (gq & 3));
            const int a0 = sc * (int)(int8_t)(uint8_t)W, a1 = sc * (int)(int8_t)(uint8_t)(W >> 8);
            const int a2 = sc * (int)(int8_t)(uint8_t)(W >> 16), a3 = sc * (int)(int8_t)(uint8_t)(W >> 24);
            hw[t] = pack4(a0 >> 6, a1 >> 6, a2 >> 6, a3 >> 6);
            lw[t] = pack4(a0 & 63, a1 & 63, a2 & 63, a3 & 63);
        }
        const uint32_t o = op_off(r, 16 * gq);
        *reinterpret_cast<uint4*>(ahi + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(alo + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
}

__device__ __forceinline__ void decode_iq2r_row(const RowSrc& src, int r, uint8_t* ahi, uint8_t* alo) {
    const uint4 sv = src.sv;
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
    const uint4 (&cw)[8] = src.cw;
    // u16 (tt, gq) at halfword 16 tt + gq
#pragma unroll
    for (int gq = 0; gq < 16; ++gq) {
        const int s = (int)((sw[gq >> 2] >> (8 * (gq & 3))) & 255u);
        const int v1 = s * 8, v2 = s * 25, v3 = s * 43;
        const uint32_t h0 = pack4(0, v1 >> 6, v2 >> 6, v3 >> 6), h1 = pack4(0, (-v1) >> 6, (-v2) >> 6, (-v3) >> 6);
        const uint32_t l0 = pack4(0, v1 & 63, v2 & 63, v3 & 63), l1 = pack4(0, (-v1) & 63, (-v2) & 63, (-v3) & 63);
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
            const int hwi = 16 * tt + gq;   // halfword index
            const uint32_t q = (word_of(cw, hwi >> 1) >> (16 * (hwi & 1))) & 0xffffu;
            hw[tt] = __byte_perm(h0, h1, q);
            lw[tt] = __byte_perm(l0, l1, q);
        }
        const uint32_t o = op_off(r, 16 * gq);
        *reinterpret_cast<uint4*>(ahi + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(alo + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
}

// R4 block of IQ3_XXS origin (8 group-scale bytes 1 + 2s; then for tt = 0..3
// and group ib a u32 whose nibbles 0..3 / 4..7 index values 32 ib + 4 tt + j /
// 32 ib + 16 + 4 tt + j in {4, 12, ..., 52, 62} plus 8 when negative).
__device__ __forceinline__ void lut16(uint32_t q, const uint32_t T[4], uint32_t& lo, uint32_t& hi) {
    const uint32_t pick = ((q >> 1) & 0x44444444u) | 0x32103210u;
    lo = __byte_perm(__byte_perm(T[0], T[1], q), __byte_perm(T[2], T[3], q), pick);
    const uint32_t q2 = q >> 16;
    hi = __byte_perm(__byte_perm(T[0], T[1], q2), __byte_perm(T[2], T[3], q2), pick >> 16);
}

// IQ4 (R4 of IQ4_XS origin): the code is an index into the IQ4_NL values
// (src/qx_format.c:2032), the scale byte is ls - 32 (signed).
__device__ constexpr int kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

template <bool IQ4>
__device__ __forceinline__ void decode_r4_row(const RowSrc& src, int r, uint8_t* ahi, uint8_t* alo) {
    const uint4 sv = src.sv;
    const uint4 (&cw)[8] = src.cw;
    // u32 (tt, ib) at word 8 tt + ib
    constexpr int kMag[8] = {4, 12, 20, 28, 36, 44, 52, 62};
#pragma unroll
    for (int ib = 0; ib < 8; ++ib) {
        const uint32_t sb = ((ib < 4 ? sv.x : sv.y) >> (8 * (ib & 3))) & 255u;
        const int s = IQ4 ? (int)(int8_t)sb : (int)sb;
        int v[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] = IQ4 ? s * kIq4nl[c] : (c < 8 ? s * kMag[c] : -(s * kMag[c - 8]));
        const uint32_t Th[4] = {pack4(v[0] >> 6, v[1] >> 6, v[2] >> 6, v[3] >> 6),
                                pack4(v[4] >> 6, v[5] >> 6, v[6] >> 6, v[7] >> 6),
                                pack4(v[8] >> 6, v[9] >> 6, v[10] >> 6, v[11] >> 6),
                                pack4(v[12] >> 6, v[13] >> 6, v[14] >> 6, v[15] >> 6)};
        const uint32_t Tl[4] = {pack4(v[0] & 63, v[1] & 63, v[2] & 63, v[3] & 63),
                                pack4(v[4] & 63, v[5] & 63, v[6] & 63, v[7] & 63),
                                pack4(v[8] & 63, v[9] & 63, v[10] & 63, v[11] & 63),
                                pack4(v[12] & 63, v[13] & 63, v[14] & 63, v[15] & 63)};
        uint32_t h0[4], h1[4], l0[4], l1[4];
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
            const uint32_t q = word_of(cw, 8 * tt + ib);
            lut16(q, Th, h0[tt], h1[tt]);
            lut16(q, Tl, l0[tt], l1[tt]);
        }
        const uint32_t o = op_off(r, 32 * ib);
        *reinterpret_cast<uint4*>(ahi + o) = make_uint4(h0[0], h0[1], h0[2], h0[3]);
        *reinterpret_cast<uint4*>(ahi + o + 128) = make_uint4(h1[0], h1[1], h1[2], h1[3]);
        *reinterpret_cast<uint4*>(alo + o) = make_uint4(l0[0], l0[1], l0[2], l0[3]);
        *reinterpret_cast<uint4*>(alo + o + 128) = make_uint4(l1[0], l1[1], l1[2], l1[3]);
    }
}

// ---- the grouped GEMM ---------------------------------------------------------
// One CTA: 128 rows [row0, row0 + 128) of one expert matrix against up to 16
// columns (expert slots, or tokens for gate/up) of the item.  Per 256-value
// block: decode A (hi/lo), stage B, 16 MMAs (8 K steps x 2 digits), commit,
// fold the accumulators.  Output out[col * out_stride + row] = the dot
// product as a float (non-finite -> 0, src/qx_format.c:4783).
template <int FMT>
__global__ void __launch_bounds__(kGemmThreads, 1) k_moe_gemm(GemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem) + 127) & ~(uintptr_t)127);
    uint8_t* ahi = base;
    uint8_t* alo = base + 8 * kSlab;
    uint8_t* bop = base + 16 * kSlab;
    __shared__ __align__(8) uint64_t mbar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int cols_s[kTiles * kTokTile], bidx_s[kTiles * kTokTile];
    __shared__ int sexp_s[kTiles * kTokTile][kMaxBlk];
    if (a.nitems && (int)blockIdx.x >= *a.nitems) return;     // past a device-built list
    const GemmItem it = a.items[blockIdx.x];
    const int r = threadIdx.x, warp = r >> 5, ncol = it.ncols, ntile = (ncol + kTokTile - 1) / kTokTile;
    if (r < kTiles * kTokTile) {
        const int c = r < ncol ? a.cols[it.col0 + r] : -1;
        cols_s[r] = c;
        bidx_s[r] = c < 0 ? -1 : (a.b_by_token ? c / 8 : c);
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base_s)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (r == 0) {
        asm volatile("mbarrier.init.shared.b64 [%0], 1;" ::"r"(smem_addr(&mbar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // columns beyond the item stay zero in every block (no limbs, no ones)
    for (int i = r; i < 8 * kSlab / 16; i += kGemmThreads) reinterpret_cast<uint4*>(bop)[i] = make_uint4(0, 0, 0, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = tmem_base_s;
    for (int i = r; i < kTiles * kTokTile * a.nblk; i += kGemmThreads) {
        const int j = i / a.nblk, b = i % a.nblk;
        sexp_s[j][b] = bidx_s[j] < 0 ? 0 : a.sexp[(size_t)bidx_s[j] * a.nblk + b];
    }
    const uint8_t* mat = a.weights + (size_t)it.expert * a.expert_stride + (size_t)(it.row0 + r) * a.row_bytes;
    const uint32_t idesc = idesc_i8(kRowTile, 8 * kTokTile);
    double acc[kTiles * kTokTile];
#pragma unroll
    for (int j = 0; j < kTiles * kTokTile; ++j) acc[j] = 0.0;
    unsigned phase = 0;
    bool ok = true;
    using Src = RowSrcN<FMT == kGemmR8 ? 16 : 8>;
    auto src_at = [&](int b, Src& s) {
        if (FMT == kGemmIq2r) load_src(mat + a.hdr + (size_t)b * 144, mat + a.hdr + (size_t)b * 144 + 16, true, s);
        else if (FMT == kGemmR8) load_src(mat + a.hdr + (size_t)b * 272, mat + a.hdr + (size_t)b * 272 + 16, true, s);
        else load_src(mat + a.hdr + 8 * b, mat + a.codes + 128 * b, false, s);
    };
    Src src;
    src_at(0, src);
    // B of column tile t: each column's 2 KB of a block (8 slabs x 256 B:
    // limbs 0-6 and the ones column of 32 values) to slab s, 8-row group j.
    // Rows of columns past the item keep whatever they held: their MMA
    // columns are never folded into a stored result.
    auto stage_b = [&](int b, int t) {
        for (int i = r; i < kTokTile * 128; i += kGemmThreads) {
            const int j = i >> 7, c16 = i & 127, col = t * kTokTile + j;
            if (bidx_s[col] < 0) continue;
            const int s = c16 >> 4, w = c16 & 15;
            cp_async16(bop + s * kSlab + j * 256 + w * 16,
                       a.bq + ((size_t)bidx_s[col] * a.nblk + b) * 2048 + s * 256 + w * 16);
        }
        cp_async_commit();
    };
    stage_b(0, 0);
    for (int b = 0; b < a.nblk && ok; ++b) {
        // A: this thread's row of block b (source loaded during the previous block)
        if constexpr (FMT == kGemmIq2r) decode_iq2r_row(src, r, ahi, alo);
        else if constexpr (FMT == kGemmR4Iq4) decode_r4_row<true>(src, r, ahi, alo);
        else if constexpr (FMT == kGemmR8) decode_r8_row(src, r, ahi, alo);
        else decode_r4_row<false>(src, r, ahi, alo);
        const double dfac = (double)h2f(*reinterpret_cast<const uint16_t*>(mat + 2 * b));
#pragma unroll
        for (int t = 0; t < kTiles; ++t) {
            if (t >= ntile || !ok) break;
            cp_async_wait<0>();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic-proxy writes -> tensor core
            __syncthreads();
            if (r == 0) {
                tc_fence_after();
                const uint32_t ah = smem_addr(ahi), al = smem_addr(alo), bb = smem_addr(bop);
#pragma unroll
                for (int s = 0; s < 8; ++s) {
                    const uint64_t bd = umma_desc(bb + s * kSlab, 128, 256);
                    mma_i8(tbase, umma_desc(ah + s * kSlab, 128, 256), bd, idesc, s > 0);
                    mma_i8(tbase + 128, umma_desc(al + s * kSlab, 128, 256), bd, idesc, s > 0);
                }
                mma_commit(&mbar);
            }
            if (t == 0 && b + 1 < a.nblk) src_at(b + 1, src);   // in flight during the MMAs and the folds
            // bounded wait for the MMAs (2 s; a healthy block takes microseconds);
            // every thread agrees on the outcome before it touches TMEM
            {
                const unsigned long long t0 = gtimer();
                uint32_t done = 0;
                while (!done) {
                    asm volatile(
                        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
                        : "=r"(done)
                        : "r"(smem_addr(&mbar)), "r"(phase)
                        : "memory");
                    if (!done && gtimer() - t0 > 2000000000ull) break;
                }
                ok = __syncthreads_and((int)done) != 0;
                if (!ok && r == 0) atomicOr(a.err, kErrTimeout);
                phase ^= 1u;
            }
            tc_fence_after();
            if (ok) {
                // the MMAs have read B: refill it with the next tile (or the
                // next block's first tile) during the fold
                if (t + 1 < ntile) stage_b(b, t + 1);
                else if (b + 1 < a.nblk) stage_b(b + 1, 0);
                // fold: column j's exact block integer X = sum_n c_n 2^(8n) (limb 6
                // minus 128 x the ones column removes the 2^55 offset) times
                // d * 2^(fexp - S_j)
                const uint32_t lane_addr = tbase + ((uint32_t)(32 * warp) << 16);
#pragma unroll
                for (int p = 0; p < kTokTile / 2; ++p) {
                    uint32_t hv[16], lv[16];
                    tmem_ld16(lane_addr + 16 * p, hv);
                    tmem_ld16(lane_addr + 128 + 16 * p, lv);
                    tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        int c[8];
#pragma unroll
                        for (int n = 0; n < 8; ++n) c[n] = 64 * (int)hv[8 * h + n] + (int)lv[8 * h + n];
                        c[6] -= 128 * c[7];
                        const long long plo = (long long)c[0] + ((long long)c[1] << 8) + ((long long)c[2] << 16) +
                                              ((long long)c[3] << 24);
                        const long long phi = (long long)c[4] + ((long long)c[5] << 8) + ((long long)c[6] << 16);
                        const int j = t * kTokTile + 2 * p + h;
                        const double f = dfac * blk_pow2(sexp_s[j][b], a.fexp);
                        acc[j] = fma((double)phi, f * 4294967296.0, acc[j]);
                        acc[j] = fma((double)plo, f, acc[j]);
                    }
                }
            }
            tc_fence_before();
            __syncthreads();   // the accumulators (and, after the last tile, the slabs) are free
        }
    }
    if (ok) {
#pragma unroll
        for (int j = 0; j < kTiles * kTokTile; ++j) {
            const double v = acc[j];
            if (j < ncol) {
                const size_t o = (size_t)cols_s[j] * a.out_stride + a.out_off + it.row0 + r;
                if (a.out_d) a.out_d[o] = v;                       // the head: double logits
                else a.out[o] = isfinite(v) ? (float)v : 0.0f;
            }
        }
    }
    tc_fence_after();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols) : "memory");
}

// ---- expert slot lists ----------------------------------------------------------
__global__ void k_slot_count(const int* sel, int nslots, int E, int* count) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s < nslots) {
        const int e = sel[s];
        if (e >= 0 && e < E) atomicAdd(count + e, 1);
    }
}

// CTA e (256 threads): expert e's start and item offsets from the counts, its
// slots compacted in slot order (ballot per warp, warp offsets per pass), and
// its work items.
__global__ void __launch_bounds__(256) k_slot_lists(const int* sel, int nslots, int E, const int* count, int* cols,
                                                    GemmItem* items_gu, int rows_gu, GemmItem* items_dn, int rows_dn,
                                                    int* nitems) {
    __shared__ int wsum[8];
    __shared__ int base_s[4];
    const int e = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    if (warp == 0) {                      // exclusive prefixes over the experts before e
        int st = 0, ct = 0, tot_ct = 0;
        for (int k = lane; k < E; k += 32) {
            const int c = count[k], n = (c + kGemmItemCols - 1) / kGemmItemCols;
            if (k < e) { st += c; ct += n; }
            tot_ct += n;
        }
        for (int o = 16; o; o >>= 1) {
            st += __shfl_xor_sync(0xffffffffu, st, o);
            ct += __shfl_xor_sync(0xffffffffu, ct, o);
            tot_ct += __shfl_xor_sync(0xffffffffu, tot_ct, o);
        }
        if (lane == 0) {
            base_s[0] = st;
            base_s[1] = ct;
            if (e == 0) {
                nitems[0] = tot_ct * (rows_gu / kRowTile);
                nitems[1] = tot_ct * (rows_dn / kRowTile);
            }
        }
    }
    __syncthreads();
    const int start = base_s[0], ct0 = base_s[1], cnt = count[e];
    int done = 0;
    for (int s0 = 0; s0 < nslots; s0 += 256) {
        const int s = s0 + t;
        const bool mine = s < nslots && sel[s] == e;
        const unsigned m = __ballot_sync(0xffffffffu, mine);
        if (lane == 0) wsum[warp] = __popc(m);
        __syncthreads();
        int before = done;
        for (int w = 0; w < warp; ++w) before += wsum[w];
        if (mine) cols[start + before + __popc(m & ((1u << lane) - 1u))] = s;
        int all = 0;
        for (int w = 0; w < 8; ++w) all += wsum[w];
        done += all;
        __syncthreads();
    }
    const int nct = (cnt + kGemmItemCols - 1) / kGemmItemCols, rgu = rows_gu / kRowTile, rdn = rows_dn / kRowTile;
    for (int i = t; i < nct * rgu; i += 256) {
        const int c = i / rgu, rt = i % rgu;
        items_gu[(size_t)(ct0 + c) * rgu + rt] =
            GemmItem{e, start + c * kGemmItemCols, min(kGemmItemCols, cnt - c * kGemmItemCols), rt * kRowTile};
    }
    for (int i = t; i < nct * rdn; i += 256) {
        const int c = i / rdn, rt = i % rdn;
        items_dn[(size_t)(ct0 + c) * rdn + rt] =
            GemmItem{e, start + c * kGemmItemCols, min(kGemmItemCols, cnt - c * kGemmItemCols), rt * kRowTile};
    }
}

// ---- activations -------------------------------------------------------------
// RMSNorm (ffn_norm, src/qx_format.c:3358-3371) of every token, CTA per token.
__global__ void __launch_bounds__(256) k_batch_norm(const float* x, const float* w, float* xn, int H) {
    __shared__ double scratch[8];
    const float* xt = x + (size_t)blockIdx.x * H;
    float* yt = xn + (size_t)blockIdx.x * H;
    const double ss = sum_sq_fixed(xt, H, scratch);
    const double rms = sqrt(ss / (double)H + 1.0e-6);
    for (int i = threadIdx.x; i < H; i += blockDim.x) yt[i] = (float)((double)xt[i] / rms) * w[i];
}

// Fixed-point limbs of every 256-value block of rows x[n][K] in the GEMM's B
// layout: per row and block 2 KB = 8 slabs (32 values) of 8 limb rows x 32
// bytes (two 16-byte core-matrix rows), limb 7 the ones column; one warp per
// (row, half block), the same rounding as build_xq.
__global__ void __launch_bounds__(256) k_batch_limbs(const float* x, int K, int nrows, uint8_t* bq, int* sexp) {
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nblk = K / 256;
    if (item >= nrows * nblk * 2) return;
    const int h = item & 1, b = (item >> 1) % nblk, t = (item >> 1) / nblk;
    const float* xs = x + (size_t)t * K + b * 256;
    const float4 u = reinterpret_cast<const float4*>(xs)[lane];
    const float4 v = reinterpret_cast<const float4*>(xs + 128)[lane];
    float mx = fmaxf(fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w))),
                     fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const bool fin = isfinite(u.x) && isfinite(u.y) && isfinite(u.z) && isfinite(u.w) && isfinite(v.x) &&
                     isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
    const int E = mx > 0.f ? (int)((__float_as_uint(mx) >> 23) & 255u) - 127 : -126;
    const int S = __all_sync(0xffffffffu, fin) ? 54 - (E < -126 ? -126 : E) : kSbNonFinite;
    if (lane == 0 && h == 0) sexp[(size_t)t * nblk + b] = S;
    const float4 q = h ? v : u;
    const int Sq = S == kSbNonFinite ? 0 : S;
    uint32_t hi[4], lo[4], w[4];
    to_fixed(q.x, Sq, hi[0], lo[0]);
    to_fixed(q.y, Sq, hi[1], lo[1]);
    to_fixed(q.z, Sq, hi[2], lo[2]);
    to_fixed(q.w, Sq, hi[3], lo[3]);
    const int k0 = 128 * h + 4 * lane;   // values k0 .. k0 + 3 of the block
    uint8_t* dst = bq + ((size_t)t * nblk + b) * 2048 + (k0 >> 5) * 256 + ((k0 >> 4) & 1) * 128 + (k0 & 15);
    transpose4(lo[0], lo[1], lo[2], lo[3], w);
#pragma unroll
    for (int n = 0; n < 4; ++n) *reinterpret_cast<uint32_t*>(dst + 16 * n) = w[n];
    transpose4(hi[0], hi[1], hi[2], hi[3], w);
#pragma unroll
    for (int n = 0; n < 3; ++n) *reinterpret_cast<uint32_t*>(dst + 16 * (4 + n)) = w[n];
    *reinterpret_cast<uint32_t*>(dst + 16 * 7) = 0x01010101u;
}

// F32 router in double, softmax in double, top-8 by repeated strict-> scans
// (lowest index on ties) and renormalisation, per token
// (src/qx_format.c:5253-5287).  A CTA takes kRouterTok tokens (widened to
// double in shared memory, so each router row read from L2 serves all of
// them); warp w forms the logits of experts w, w + 8, ... (lane-strided
// partial dots, then a butterfly), then warp j ranks token j's experts.
constexpr int kRouterTok = 8;

__global__ void __launch_bounds__(256) k_batch_router(const float* xn, const float* router, int H, int E, int ntok,
                                                      int* sel, double* wsel, int* err) {
    extern __shared__ __align__(16) uint8_t rsm[];
    double* xd = reinterpret_cast<double*>(rsm);                    // [kRouterTok][H]
    double* logit = xd + (size_t)kRouterTok * H;                    // [kRouterTok][E]
    double* prob = logit + (size_t)kRouterTok * E;
    const int t0 = blockIdx.x * kRouterTok, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nt = min(kRouterTok, ntok - t0);
    for (int i = threadIdx.x; i < kRouterTok * H; i += blockDim.x) {
        const int j = i / H;
        xd[i] = j < nt ? (double)xn[(size_t)(t0 + j) * H + i % H] : 0.0;
    }
    __syncthreads();
    // warp w: experts 4 w' .. 4 w' + 3 for w' = w, w + 8, ...; each x value
    // read from shared memory feeds four FMAs
    for (int e0 = 4 * warp; e0 < E; e0 += 4 * (blockDim.x >> 5)) {
        double acc[4][kRouterTok];
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int j = 0; j < kRouterTok; ++j) acc[q][j] = 0.0;
#pragma unroll 4
        for (int i = lane; i < H; i += 32) {
            double wv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) wv[q] = e0 + q < E ? (double)router[(size_t)(e0 + q) * H + i] : 0.0;
#pragma unroll
            for (int j = 0; j < kRouterTok; ++j) {
                const double xv = xd[j * H + i];
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[q][j] = fma(wv[q], xv, acc[q][j]);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int j = 0; j < kRouterTok; ++j) {
                const double v = warp_sum_d(acc[q][j]);
                if (lane == 0 && e0 + q < E) logit[j * E + e0 + q] = v;
            }
    }
    __syncthreads();
    if (warp >= nt) return;
    const int t = t0 + warp;
    const double* lg = logit + warp * E;
    double* pr = prob + warp * E;
    double m = -1.0e300;
    for (int e = lane; e < E; e += 32) m = fmax(m, lg[e]);
    for (int o = 16; o; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    double s = 0.0;
    for (int e = lane; e < E; e += 32) {
        const double p = exp(lg[e] - m);
        pr[e] = p;
        s += p;
    }
    s = warp_sum_d(s);
    for (int e = lane; e < E; e += 32) pr[e] /= s;
    __syncwarp();
    double ws[8];
    int picked = 0;   // bit q: expert lane + 32 q is taken
    double sum = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        double bv = -1.0;
        int bi = 0x7fffffff;
        for (int e = lane, q = 0; e < E; e += 32, ++q)
            if (!((picked >> q) & 1) && (pr[e] > bv || (pr[e] == bv && e < bi))) { bv = pr[e]; bi = e; }
        for (int o = 16; o; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (bi != 0x7fffffff && (bi & 31) == lane) picked |= 1 << (bi >> 5);
        ws[k] = bv;
        sum += bv;
        if (lane == 0) sel[t * 8 + k] = bi;
    }
    if (lane == 0) {
        if (!(sum > 0.0) || !isfinite(sum)) atomicOr(err, kErrRouter);
        for (int k = 0; k < 8; ++k) wsel[t * 8 + k] = ws[k] / sum;
    }
}

// SwiGLU in double (src/qx_format.c:5297, qx_silu :2511-2513) of every expert
// slot: gu[slot][0 .. I) = gate, [I .. 2I) = up.
__global__ void k_batch_swiglu(const float* gu, int I, int nslots, float* h) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)nslots * I) return;
    const size_t s = i / I, k = i % I;
    const double gd = (double)gu[s * 2 * I + k];
    h[i] = (float)(gd / (1.0 + exp(-gd)) * (double)gu[s * 2 * I + I + k]);
}

// out = residual + sum over ranks k = 0..7 (in order) of (float)(w_k * y_k)
// (src/qx_format.c:5303-5309).
__global__ void k_batch_combine(const float* x, const float* y, const double* wsel, int H, int ntok, float* moe,
                                float* out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)ntok * H) return;
    const size_t t = i / H, c = i % H;
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) m += (float)(wsel[t * 8 + k] * (double)y[(t * 8 + k) * H + c]);
    if (moe) moe[i] = m;
    out[i] = x[i] + m;
}

// ---- prompt prefill: the attention half for many tokens ----------------------
// Embedding rows (Q4_K, d * sc * q - dmin * m with each product rounded to
// float, src/qx_format.c:2089-2110, :3759-3819), one CTA per token.
__global__ void __launch_bounds__(256) k_batch_embed(const uint32_t* tokens, const uint8_t* emb, int H, int V,
                                                     float* x, int* err) {
    const uint32_t tok = tokens[blockIdx.x];
    if (tok >= (uint32_t)V) {
        if (threadIdx.x == 0) atomicOr(err, kErrToken);
        return;
    }
    const int nblk = H / 256;
    const uint8_t* row = emb + (size_t)tok * (size_t)(nblk * 144);
    float* xt = x + (size_t)blockIdx.x * H;
    const int t = threadIdx.x, c = t >> 6, l = t & 63;
    for (int b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 144;
        const float dd = h2f(ld16(blk)), dmin = h2f(ld16(blk + 2));
        const uint8_t* sc = blk + 4;
        const int j = 2 * c + (l >= 32);
        uint32_t scv, mn;
        if (j < 4) { scv = sc[j] & 63u; mn = sc[j + 4] & 63u; }
        else { scv = (sc[j + 4] & 15u) | ((sc[j - 4] >> 6) << 4); mn = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4); }
        const uint8_t qb = blk[16 + 32 * c + (l & 31)];
        const uint32_t q = l < 32 ? (qb & 15u) : (qb >> 4);
        xt[b * 256 + t] = __fsub_rn(__fmul_rn(__fmul_rn(dd, (float)scv), (float)q), __fmul_rn(dmin, (float)mn));
    }
}

// Per token (CTA): per-head Q/K RMSNorm + split-half RoPE at the token's
// position (src/qx_format.c:3740-3757, :4625-4641), the normed Q to qn, and
// the INT8 K/V row (one scale per token over all KV values, :4449-4463)
// appended to the cache at (layer, p0 + t) (:6343-6400).
__global__ void __launch_bounds__(256) k_batch_qkv_post(const float* qkv, const float* q_norm, const float* k_norm,
                                                        const double* rope, int layer, const int* tpos,
                                                        const int* tslot, KvView kv, int QH, int KVH, float* qn) {
    constexpr int D = 128;
    __shared__ float v[4096 + 2 * 1024];
    __shared__ float scratch_f[8];
    const int Q = QH * D, KV = KVH * D, t = blockIdx.x, pos = tpos[t], ctx = kv.ctx;
    int8_t* kcache = kv.k + (size_t)tslot[t] * kv.slot_rows * KV;
    int8_t* vcache = kv.v + (size_t)tslot[t] * kv.slot_rows * KV;
    float* kscale = kv.ks + (size_t)tslot[t] * kv.slot_rows;
    float* vscale = kv.vs + (size_t)tslot[t] * kv.slot_rows;
    const float* src = qkv + (size_t)t * (Q + 2 * KV);
    for (int j = threadIdx.x; j < Q + 2 * KV; j += blockDim.x) v[j] = src[j];
    __syncthreads();
    const double* rp = rope + (size_t)pos * 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int hh = warp; hh < QH + KVH; hh += blockDim.x >> 5) {
        if (hh < QH) warp_norm_rope(v + hh * D, q_norm, rp, lane);
        else warp_norm_rope(v + Q + (hh - QH) * D, k_norm, rp, lane);
    }
    __syncthreads();
    for (int j = threadIdx.x; j < Q; j += blockDim.x) qn[(size_t)t * Q + j] = v[j];
    const float* kc = v + Q;
    const float* vc = v + Q + KV;
    float ka = 0.f, va = 0.f;
    for (int j = threadIdx.x; j < KV; j += blockDim.x) {
        ka = fmaxf(ka, isfinite(kc[j]) ? fabsf(kc[j]) : 0.f);
        va = fmaxf(va, isfinite(vc[j]) ? fabsf(vc[j]) : 0.f);
    }
    ka = block_max_f(ka, scratch_f);
    va = block_max_f(va, scratch_f);
    const float ksc = ka > 0.f ? ka / 127.0f : 1.0f, vsc = va > 0.f ? va / 127.0f : 1.0f;
    const size_t slot = (size_t)layer * ctx + pos;
    for (int j = threadIdx.x; j < KV; j += blockDim.x) {
        const int qk = isfinite(kc[j]) ? (int)lrintf(kc[j] / ksc) : 0;
        const int qq = isfinite(vc[j]) ? (int)lrintf(vc[j] / vsc) : 0;
        kcache[slot * KV + j] = (int8_t)max(-127, min(127, qk));
        vcache[slot * KV + j] = (int8_t)max(-127, min(127, qq));
    }
    if (threadIdx.x == 0) { kscale[slot] = ksc; vscale[slot] = vsc; }
}

// Causal GQA attention of token t (grid.x) and query head h (grid.y) over
// positions 0..p0 + t of the cache: scores in double in dimension order,
// softmax with the max subtracted and a fixed-order sum, context accumulated
// in float over positions in order (src/qx_format.c:5127-5172) - the same
// arithmetic as the decode step's attention.  128 threads; dynamic shared
// memory: (p0 + t + 1) doubles.
__global__ void __launch_bounds__(128) k_batch_attn(const float* qn, KvView kv, int layer, const int* tpos,
                                                    const int* tslot, int QH, int KVH, float* ctx_out) {
    constexpr int D = 128;
    extern __shared__ __align__(16) double w_s[];
    __shared__ double qd[D];
    __shared__ double scratch_d[4];
    const int t = blockIdx.x, h = blockIdx.y, i = threadIdx.x, g = h / (QH / KVH);
    const int Q = QH * D, KV = KVH * D, T = tpos[t] + 1, ctx = kv.ctx;
    const int8_t* kcache = kv.k + (size_t)tslot[t] * kv.slot_rows * KV;
    const int8_t* vcache = kv.v + (size_t)tslot[t] * kv.slot_rows * KV;
    const float* kscale = kv.ks + (size_t)tslot[t] * kv.slot_rows;
    const float* vscale = kv.vs + (size_t)tslot[t] * kv.slot_rows;
    qd[i] = (double)qn[(size_t)t * Q + h * D + i];
    __syncthreads();
    const double sqrt_d = sqrt((double)D);
    double mloc = -1.0e300;
    for (int p = i; p < T; p += D) {
        const size_t st = (size_t)layer * ctx + p;
        const double sc = score_row(qd, kcache + st * KV + g * D, kscale[st], sqrt_d);
        w_s[p] = sc;
        mloc = fmax(mloc, sc);
    }
    const double mx = block_max_d(mloc, scratch_d);
    for (int p = i; p < T; p += D) w_s[p] = exp(w_s[p] - mx);
    double den = fixed_order_sum(w_s, T, scratch_d);
    if (!isfinite(den) || den <= 0.0) den = 1.0;
    for (int p = i; p < T; p += D) w_s[p] = w_s[p] / den;
    __syncthreads();
    const int8_t* vb = vcache + (size_t)layer * ctx * KV + g * D + i;
    const float* vs = vscale + (size_t)layer * ctx;
    float acc = 0.0f;
    constexpr int U = 16;                 // positions whose loads go out together
    int p = 0;
    for (; p + U <= T; p += U) {
        int8_t vq[U];
        float vsc[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            vq[u] = vb[(size_t)(p + u) * KV];
            vsc[u] = vs[p + u];
        }
#pragma unroll
        for (int u = 0; u < U; ++u) acc += (float)(w_s[p + u] * (double)(i8_to_f32(vq[u]) * vsc[u]));
    }
    for (; p < T; ++p) acc += (float)(w_s[p] * (double)(i8_to_f32(vb[(size_t)p * KV]) * vs[p]));
    ctx_out[(size_t)t * Q + h * D + i] = acc;
}

// vd[r][j] = (double)((float)v[r][j] * vs[r]) for rows r < rows: the widened
// value every context product of row r uses (the same expression).
__global__ void k_widen_v(const int8_t* v, const float* vs, int rows, int KV, double* vd) {
    const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < (size_t)rows * KV) vd[e] = (double)(i8_to_f32(v[e]) * vs[e / KV]);
}

// k_batch_attn for all G query heads of one KV group at once: CTA = (token,
// KV group), 256 threads.  Every scalar operation and its order are those of
// the per-token step (score_row's dimension-order FMA chain, fmax, exp,
// fixed_order_sum's lane-strided denominator, one division, the position-order
// float context sum), so the results are bit-identical; what changes is that
// a key or value is widened to double once for all the heads that use it.
// Scores: thread -> positions i, i + 512, ... for all G heads; softmax: warp h
// forms head h's denominator; context: thread -> dimension i % 128 for heads
// (i / 128) * G/4 .. + G/4 - 1.  w_s: [T][G] doubles (dynamic shared memory).
// Tokens t0 + blockIdx.x.  vd (optional, slot 0 only): the layer's V rows
// already widened, vd[p][j] = (double)((float)v * vscale) (k_widen_v), read
// in place of the INT8 rows.
template <int G>
__global__ void __launch_bounds__(512, 2) k_batch_attn_grp(const float* qn, KvView kv, int layer, const int* tpos,
                                                        const int* tslot, int QH, int KVH, float* ctx_out, int t0,
                                                        const double* vd) {
    constexpr int D = 128, NT = 512, HH = G / 4;
    extern __shared__ __align__(16) double w_s[];
    __shared__ __align__(16) double qd[G * D];
    __shared__ double red[NT / 32][G];
    __shared__ double hv[2][G];
    const int t = t0 + blockIdx.x, g = blockIdx.y, i = threadIdx.x, warp = i >> 5, lane = i & 31;
    const int Q = QH * D, KV = KVH * D, T = tpos[t] + 1, ctx = kv.ctx;
    const size_t srow = (size_t)tslot[t] * kv.slot_rows;
    const int8_t* kcache = kv.k + srow * KV;
    const int8_t* vcache = kv.v + srow * KV;
    const float* kscale = kv.ks + srow;
    const float* vscale = kv.vs + srow;
    for (int j = i; j < G * D; j += NT) qd[j] = (double)qn[(size_t)t * Q + (size_t)g * G * D + j];
    __syncthreads();
    const double sqrt_d = sqrt((double)D);
    double mloc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) mloc[h] = -1.0e300;
    for (int p = i; p < T; p += NT) {
        const size_t st = (size_t)layer * ctx + p;
        const int8_t* kp = kcache + st * KV + g * D;
        const float ks = kscale[st];
        double s[G];
#pragma unroll
        for (int h = 0; h < G; ++h) s[h] = 0.0;
#pragma unroll 1
        for (int j = 0; j < D; j += 8) {
            const int2 raw = *reinterpret_cast<const int2*>(kp + j);
            const int8_t* kb = reinterpret_cast<const int8_t*>(&raw);
            double kd[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) kd[u] = (double)(i8_to_f32(kb[u]) * ks);
#pragma unroll
            for (int h = 0; h < G; ++h)
#pragma unroll
                for (int u = 0; u < 8; ++u) s[h] = fma(qd[h * D + j + u], kd[u], s[h]);
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
            double v = s[h] / sqrt_d;
            v = isfinite(v) ? v : 0.0;
            w_s[p * G + h] = v;
            mloc[h] = fmax(mloc[h], v);
        }
    }
    // per-head maxima (fmax: the order does not matter)
#pragma unroll
    for (int h = 0; h < G; ++h) {
        double m = mloc[h];
        for (int o = 16; o; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) red[warp][h] = m;
    }
    __syncthreads();
    if (i < G) {
        double m = red[0][i];
        for (int k = 1; k < NT / 32; ++k) m = fmax(m, red[k][i]);
        hv[0][i] = m;
    }
    __syncthreads();
    for (int e = i; e < T * G; e += NT) w_s[e] = exp(w_s[e] - hv[0][e % G]);
    __syncthreads();
    if (warp < G) {                       // head `warp`: fixed_order_sum's order
        double sum = 0.0;
        for (int p = lane; p < T; p += 32) sum += w_s[p * G + warp];
        sum = warp_sum_d(sum);
        if (lane == 0) hv[1][warp] = (!isfinite(sum) || sum <= 0.0) ? 1.0 : sum;
    }
    __syncthreads();
    for (int e = i; e < T * G; e += NT) w_s[e] = w_s[e] / hv[1][e % G];
    __syncthreads();
    const int d = i & (D - 1), h0 = (i >> 7) * HH;
    const int8_t* vb = vcache + (size_t)layer * ctx * KV + g * D + d;
    const float* vs = vscale + (size_t)layer * ctx;
    float acc[HH];
#pragma unroll
    for (int k = 0; k < HH; ++k) acc[k] = 0.0f;
    constexpr int U = 16;                 // positions whose loads go out together
    int p = 0;
    if (vd) {
        const double* vp = vd + g * D + d;
        for (; p + U <= T; p += U) {
            double vv[U];
#pragma unroll
            for (int u = 0; u < U; ++u) vv[u] = vp[(size_t)(p + u) * KV];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int k = 0; k < HH; ++k) acc[k] += (float)(w_s[(p + u) * G + h0 + k] * vv[u]);
        }
        for (; p < T; ++p)
#pragma unroll
            for (int k = 0; k < HH; ++k) acc[k] += (float)(w_s[p * G + h0 + k] * vp[(size_t)p * KV]);
    }
    for (; p + U <= T; p += U) {
        int8_t vq[U];
        float vsc[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            vq[u] = vb[(size_t)(p + u) * KV];
            vsc[u] = vs[p + u];
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const double vd = (double)(i8_to_f32(vq[u]) * vsc[u]);
#pragma unroll
            for (int k = 0; k < HH; ++k) acc[k] += (float)(w_s[(p + u) * G + h0 + k] * vd);
        }
    }
    for (; p < T; ++p) {
        const double vd = (double)(i8_to_f32(vb[(size_t)p * KV]) * vs[p]);
#pragma unroll
        for (int k = 0; k < HH; ++k) acc[k] += (float)(w_s[p * G + h0 + k] * vd);
    }
#pragma unroll
    for (int k = 0; k < HH; ++k) ctx_out[(size_t)t * Q + (size_t)(g * G + h0 + k) * D + d] = acc[k];
}

// Greedy pick per token over double logits [ntok][V]: the largest, lowest
// index on ties (src/qx_format.c:3723-3730); a non-finite logit is an error
// (:3715).
__global__ void __launch_bounds__(1024) k_batch_argmax(const double* logits, int V, uint32_t* out, int* err) {
    __shared__ double bv_s[32];
    __shared__ int bi_s[32];
    const double* lg = logits + (size_t)blockIdx.x * V;
    double bv = -1.0e300;
    int bi = 0x7fffffff;
    bool bad = false;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const double v = lg[i];
        if (!isfinite(v)) bad = true;
        if (v > bv) { bv = v; bi = i; }
    }
    for (int o = 16; o; o >>= 1) {
        const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (bad) atomicOr(err, kErrNonFinite);
    if ((threadIdx.x & 31) == 0) { bv_s[threadIdx.x >> 5] = bv; bi_s[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (bv_s[w] > bv || (bv_s[w] == bv && bi_s[w] < bi)) { bv = bv_s[w]; bi = bi_s[w]; }
        out[blockIdx.x] = (uint32_t)bi;
    }
}

// x[i] += y[i] (the residual adds, float, src/qx_format.c:6420-6423).
__global__ void k_batch_add(float* x, const float* y, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = x[i] + y[i];
}

}  // namespace

// Dynamic shared memory the grouped attention kernel may use (set once by
// moe_batch_configure; 0 until then, which selects the per-head kernel).
size_t g_attn_grp_smem = 0;
constexpr int kAttnBucket = 256;

void launch_batch_embed(const uint32_t* tokens, const uint8_t* emb, int H, int V, int ntok, float* x, int* err,
                        cudaStream_t st) {
    k_batch_embed<<<ntok, 256, 0, st>>>(tokens, emb, H, V, x, err);
}

void launch_batch_qkv_post(const float* qkv, const float* q_norm, const float* k_norm, const double* rope, int layer,
                           const int* tpos, const int* tslot, const KvView& kv, int ntok, int QH, int KVH, float* qn,
                           cudaStream_t st) {
    k_batch_qkv_post<<<ntok, 256, 0, st>>>(qkv, q_norm, k_norm, rope, layer, tpos, tslot, kv, QH, KVH, qn);
}

void launch_batch_attn(const float* qn, const KvView& kv, int layer, const int* tpos, const int* tslot, int max_pos,
                       int ntok, int QH, int KVH, float* ctx_out, cudaStream_t st, int first_pos, double* vd) {
    const int G = QH / KVH;
    if ((G == 8 || G == 4) && (size_t)(max_pos + 1) * G * 8 <= g_attn_grp_smem) {   // CTA per (token, KV group)
        // consecutive positions (a prompt): buckets of kAttnBucket tokens, each
        // with the shared memory of its own longest context
        const int bucket = first_pos >= 0 ? kAttnBucket : ntok;
        const double* vdp = nullptr;
        if (first_pos >= 0 && vd) {      // a prompt in slot 0: widen rows 0..max_pos once
            const int KV = KVH * 128;
            const size_t n = (size_t)(max_pos + 1) * KV;
            k_widen_v<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(kv.v + (size_t)layer * kv.ctx * KV,
                                                                  kv.vs + (size_t)layer * kv.ctx, max_pos + 1, KV, vd);
            vdp = vd;
        }
        for (int b0 = 0; b0 < ntok; b0 += bucket) {
            const int n = std::min(bucket, ntok - b0);
            const int mp = first_pos >= 0 ? first_pos + b0 + n - 1 : max_pos;
            const size_t sm = (size_t)(mp + 1) * G * 8;
            if (G == 8)
                k_batch_attn_grp<8><<<dim3(n, KVH), 512, sm, st>>>(qn, kv, layer, tpos, tslot, QH, KVH, ctx_out, b0, vdp);
            else
                k_batch_attn_grp<4><<<dim3(n, KVH), 512, sm, st>>>(qn, kv, layer, tpos, tslot, QH, KVH, ctx_out, b0, vdp);
        }
        return;
    }
    const size_t smem = (size_t)(max_pos + 1) * 8;
    k_batch_attn<<<dim3(ntok, QH), 128, smem, st>>>(qn, kv, layer, tpos, tslot, QH, KVH, ctx_out);
}

void launch_batch_argmax(const double* logits, int V, int ntok, uint32_t* out, int* err, cudaStream_t st) {
    k_batch_argmax<<<ntok, 1024, 0, st>>>(logits, V, out, err);
}

void launch_batch_add(float* x, const float* y, size_t n, cudaStream_t st) {
    k_batch_add<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, y, n);
}

uint32_t moe_gemm_smem_bytes() { return kSmemGemm; }
size_t batch_router_smem_bytes(int H, int E) { return (size_t)kRouterTok * (H + 2 * E) * 8; }

cudaError_t moe_batch_configure() {
    cudaError_t e = cudaSuccess;
    for (const void* f : {(const void*)k_moe_gemm<kGemmIq2r>, (const void*)k_moe_gemm<kGemmR4Iq3>,
                          (const void*)k_moe_gemm<kGemmR4Iq4>, (const void*)k_moe_gemm<kGemmR8>})
        if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemGemm);
    int dev = 0, optin = 0;
    if (e == cudaSuccess) e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_batch_router, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_batch_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - 2048);
    // the grouped kernel: its static arrays (query heads, reductions) take < 10 KB
    const int grp = optin - 10 * 1024;
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_batch_attn_grp<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, grp);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_batch_attn_grp<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, grp);
    if (e == cudaSuccess) g_attn_grp_smem = (size_t)grp;
    return e;
}

void launch_batch_norm(const float* x, const float* w, float* xn, int H, int ntok, cudaStream_t st) {
    k_batch_norm<<<ntok, 256, 0, st>>>(x, w, xn, H);
}

void launch_batch_limbs(const float* x, int K, int nrows, uint8_t* bq, int* sexp, cudaStream_t st) {
    const int warps = nrows * (K / 256) * 2;
    k_batch_limbs<<<(warps + 7) / 8, 256, 0, st>>>(x, K, nrows, bq, sexp);
}

void launch_batch_router(const float* xn, const float* router, int H, int E, int ntok, int* sel, double* wsel, int* err,
                         cudaStream_t st) {
    const size_t smem = (size_t)kRouterTok * (H + 2 * E) * 8;
    k_batch_router<<<(ntok + kRouterTok - 1) / kRouterTok, 256, smem, st>>>(xn, router, H, E, ntok, sel, wsel, err);
}

void launch_moe_gemm(const GemmArgs& a, int nitems, cudaStream_t st) {
    if (nitems <= 0) return;
    switch (a.fmt) {
        case kGemmIq2r: k_moe_gemm<kGemmIq2r><<<nitems, kGemmThreads, kSmemGemm, st>>>(a); break;
        case kGemmR4Iq3: k_moe_gemm<kGemmR4Iq3><<<nitems, kGemmThreads, kSmemGemm, st>>>(a); break;
        case kGemmR4Iq4: k_moe_gemm<kGemmR4Iq4><<<nitems, kGemmThreads, kSmemGemm, st>>>(a); break;
        default: k_moe_gemm<kGemmR8><<<nitems, kGemmThreads, kSmemGemm, st>>>(a); break;
    }
}

void launch_slot_lists(const int* sel, int nslots, int E, int* count, int* cols, GemmItem* items_gu, int rows_gu,
                       GemmItem* items_dn, int rows_dn, int* nitems, cudaStream_t st) {
    cudaMemsetAsync(count, 0, (size_t)E * 4, st);
    k_slot_count<<<(nslots + 255) / 256, 256, 0, st>>>(sel, nslots, E, count);
    k_slot_lists<<<E, 256, 0, st>>>(sel, nslots, E, count, cols, items_gu, rows_gu, items_dn, rows_dn, nitems);
}

void launch_batch_swiglu(const float* gu, int I, int nslots, float* h, cudaStream_t st) {
    const size_t n = (size_t)nslots * I;
    k_batch_swiglu<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(gu, I, nslots, h);
}

void launch_batch_combine(const float* x, const float* y, const double* wsel, int H, int ntok, float* moe, float* out,
                          cudaStream_t st) {
    const size_t n = (size_t)ntok * H;
    k_batch_combine<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, y, wsel, H, ntok, moe, out);
}

}  // namespace qx
