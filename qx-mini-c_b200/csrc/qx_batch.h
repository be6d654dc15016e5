// Batched MoE FFN (qx_batch.cu): the grouped-expert GEMMs on tcgen05 and the
// per-token kernels around them.  Internal to the engine; not part of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace qx {

// One CTA of the grouped GEMM: rows [row0, row0 + 128) of expert `expert`
// against the columns cols[col0 .. col0 + ncols) (ncols <= 16).
struct GemmItem {
    int expert, col0, ncols, row0;   // ncols <= kGemmItemCols
};
constexpr int kGemmItemCols = 32;    // columns (tokens or slots) per work item: two 16-column tiles
enum { kGemmIq2r = 0, kGemmR4Iq3 = 1, kGemmR4Iq4 = 2, kGemmR8 = 3 };

struct GemmArgs {
    const GemmItem* items;
    const int* cols;              // column ids: expert slots t * 8 + k, grouped by expert
    const uint8_t* weights;       // re-laid expert stack (IQ2R or R4 rows)
    size_t expert_stride;         // bytes per expert
    uint32_t row_bytes;
    int hdr;                      // IQ2R: first block; R4: first scale byte
    int codes;                    // R4: first code byte
    int nblk;                     // 256-value blocks per row (K / 256)
    int fmt;                      // kGemmIq2r or kGemmR4Iq3
    int fexp;                     // block factor d * 2^(fexp - S): -3 (IQ2_XS), -2 (IQ3_XXS), 0 (IQ4_XS, Q6_K)
    const uint8_t* bq;            // limbs [rows][nblk][2048 B] (k_batch_limbs)
    const int* sexp;              // block exponents [rows][nblk]
    int b_by_token;               // 1: B row = column id / 8 (the token), 0: B row = column id
    float* out;                   // out[col * out_stride + out_off + row] (non-finite -> 0)
    double* out_d;                // if set: the double results there instead (the head's logits)
    size_t out_stride;
    int out_off;
    int* err;
    const int* nitems;            // if set: the number of valid items (device-built lists); CTAs past it exit
};

// An INT8 KV cache of `slots` sequences: [slot][layer][ctx][kv] bytes and
// [slot][layer][ctx] scales, slot_rows = layers * ctx.
struct KvView {
    int8_t* k;
    int8_t* v;
    float* ks;
    float* vs;
    size_t slot_rows;
    int ctx;
};

uint32_t moe_gemm_smem_bytes();
size_t batch_router_smem_bytes(int H, int E);
cudaError_t moe_batch_configure();
void launch_batch_norm(const float* x, const float* w, float* xn, int H, int ntok, cudaStream_t st);
void launch_batch_limbs(const float* x, int K, int nrows, uint8_t* bq, int* sexp, cudaStream_t st);
void launch_batch_router(const float* xn, const float* router, int H, int E, int ntok, int* sel, double* wsel, int* err,
                         cudaStream_t st);
void launch_moe_gemm(const GemmArgs& a, int nitems, cudaStream_t st);
void launch_batch_swiglu(const float* gu, int I, int nslots, float* h, cudaStream_t st);
void launch_batch_embed(const uint32_t* tokens, const uint8_t* emb, int H, int V, int ntok, float* x, int* err,
                        cudaStream_t st);
void launch_batch_qkv_post(const float* qkv, const float* q_norm, const float* k_norm, const double* rope, int layer,
                           const int* tpos, const int* tslot, const KvView& kv, int ntok, int QH, int KVH, float* qn,
                           cudaStream_t st);
// The expert slot lists on the device: count[e] = slots that chose expert e
// (count zeroed first), then cols = the slots grouped by expert in slot order,
// and the GEMM work items of the gate/up (rows_gu weight rows) and down
// (rows_dn) projections in expert, column-pair, row-tile order, with their
// counts in nitems[0], nitems[1].  Slots with an expert outside [0, E) (a
// failed router, which raised its error flag) are left out.
void launch_slot_lists(const int* sel, int nslots, int E, int* count, int* cols, GemmItem* items_gu, int rows_gu,
                       GemmItem* items_dn, int rows_dn, int* nitems, cudaStream_t st);

// first_pos >= 0: token t is at position first_pos + t of KV slot 0 (a
// prompt), which lets the launch size each bucket of tokens for its own
// context length and, given vd ([max_pos + 1][kv_dim] doubles of scratch),
// widen the layer's V rows once for every head.
void launch_batch_attn(const float* qn, const KvView& kv, int layer, const int* tpos, const int* tslot, int max_pos,
                       int ntok, int QH, int KVH, float* ctx_out, cudaStream_t st, int first_pos = -1,
                       double* vd = nullptr);
void launch_batch_argmax(const double* logits, int V, int ntok, uint32_t* out, int* err, cudaStream_t st);
void launch_batch_add(float* x, const float* y, size_t n, cudaStream_t st);
void launch_batch_combine(const float* x, const float* y, const double* wsel, int H, int ntok, float* moe, float* out,
                          cudaStream_t st);

}  // namespace qx
