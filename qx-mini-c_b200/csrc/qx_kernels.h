// Internal interface between the engine runtime (qx_engine.cu) and the
// kernels (qx_kernels.cu).  Not part of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "qx_dev.cuh"
#include "qx_imma.cuh"

namespace qx {

struct LayerW {                  // device pointers into the weight arena (native GGUF layouts)
    const float* attn_norm;      // F32 [H]
    const uint8_t* wq;           // IQ4_XS [Q rows][H]
    const uint8_t* wk;           // IQ4_XS [KV rows][H]
    const uint8_t* wv;           // IQ4_XS [KV rows][H]
    const uint8_t* wo;           // IQ4_XS [H rows][Q]
    const float* q_norm;         // F32 [D]
    const float* k_norm;         // F32 [D]
    const float* ffn_norm;       // F32 [H]
    const float* router;         // F32 [E rows][H]
    const uint8_t* gate;         // IQ2_XS [E][I rows][H]
    const uint8_t* up;           // IQ2_XS [E][I rows][H]
    const uint8_t* down;         // IQ3_XXS [E][H rows][I]
    // ggml types of the quantized tensors: the benchmark mix is IQ4_XS (23)
    // attention, IQ2_XS (17) gate/up, IQ3_XXS (18) down; the per-stage kernels
    // also take Q5_K (13) / Q6_K (14) attention, IQ2_S (22) gate/up and
    // IQ3_S (21) / IQ4_XS (23) down
    int tq, tk, tv, to, tgate, tup, tdown;
    // IQ2_XS gate/up re-laid for the persistent step kernel (iq2r_row_bytes per
    // row; null when that kernel is not used)
    const uint8_t* gate_r;
    const uint8_t* up_r;
    // IQ4_XS attention and IQ3_XXS down re-laid for the persistent kernel
    // (r4_bytes_per_row per row; null when that kernel is not used)
    const uint8_t* wq_r;
    const uint8_t* wk_r;
    const uint8_t* wv_r;
    const uint8_t* wo_r;
    const uint8_t* down_r;
};

// Bytes per row of the persistent kernel's IQ2_XS layout ("IQ2R") for a row of
// H values: fp16 block scales, then per 256-value block 16 group-scale bytes
// (1 + 2s) and 128 bytes of 3-bit signed-lattice codes in nibbles.
size_t iq2r_row_bytes(int H);
// Re-lay `rows` IQ2_XS rows of H values (src) into IQ2R rows (dst).
cudaError_t launch_iq2r_repack(const uint8_t* src, uint8_t* dst, size_t rows, int H, const Tables* t, cudaStream_t st);
// The persistent kernel's layout ("R4") of IQ4_XS (type 23) and IQ3_XXS (18)
// rows of K values: 4-bit indices into a 16-entry signed byte table, one scale
// byte per 32 values, fp16 block scales.
size_t r4_bytes_per_row(int K);
// The persistent kernel's layout ("R8") of Q6_K rows of K values: int8 weights
// q - 32 in per-lane chunks, int8 group scales, fp16 block scales.
size_t r8_bytes_per_row(int K);
cudaError_t launch_r8_repack(const uint8_t* src, uint8_t* dst, size_t rows, int K, cudaStream_t st);
cudaError_t launch_r4_repack(const uint8_t* src, uint8_t* dst, size_t rows, int K, int type, const Tables* t,
                             cudaStream_t st);

// True when every layer uses the benchmark mix (the one-launch kernel's types).
bool benchmark_mix(const LayerW* layers, int n);

struct Dims {
    int layers, hidden, q_heads, kv_heads, head_dim, vocab, experts, moe_inter, ctx;
    __host__ __device__ int q_dim() const { return q_heads * head_dim; }
    __host__ __device__ int kv_dim() const { return kv_heads * head_dim; }
};

// Per-engine device state (all device pointers).
struct Dev {
    Dims dm;
    const Tables* tables;
    const uint8_t* tok_embd;     // Q4_K [V rows][H]
    const float* out_norm;       // F32 [H]
    const uint8_t* head;         // Q6_K [V rows][H]
    const uint8_t* head_r;       // the head re-laid for the persistent kernel (R8; null otherwise)
    const double* rope;          // [ctx][D/2][2] cos, sin (host libm, double)
    float* x;                    // residual [H]
    float* xn;                   // normed input of the current projection [max(H,Q)]
    float* qkv;                  // raw Q|K|V projections [Q + 2KV]
    int8_t* kcache;              // [L][ctx][KV]
    int8_t* vcache;
    float* kscale;               // [L][ctx]
    float* vscale;
    double* attn_scores;         // softmax scratch [Hq][ctx] (double)
    float* ctxv;                 // attention context [Q]
    float* attn_out;             // O projection output [H] (stage API)
    float* moe_out;              // MoE output [H] (stage API)
    double* router_logits;       // [E]
    int* sel;                    // [L][8] selected experts, rank order
    float* selw;                 // [L][8] renormalised weights (float copies)
    double* selw_d;              // [8] weights of the current layer (double)
    float* hbuf;                 // SwiGLU outputs [8][I]
    float* logits;               // [V]
    double* logits_d;            // optional [V]: the head's double logits (top-N of the stage entry point)
    int q8;                      // 1: q8_k_compat activations (per-stage kernels, qx_q8k.cu)
    double* best_val;            // per-CTA argmax partials (double logits, as the reference compares)
    int* best_idx;
    unsigned* counters;          // ticket counters for last-CTA reductions
    int* token;                  // current input token (device scalar)
    int* pos;                    // current position (device scalar)
    int* tokens_out;             // [ctx] argmax written at index pos
    int* err;                    // error bits
    int head_grid;               // CTAs of the head kernel (partials length)
    int head_grid_r8;            // CTAs of the head kernel on the re-laid (R8) head
    unsigned long long* trace;   // optional: global-timer stamp per grid barrier (CTA 0)
    // expert parallelism (ep_world > 1; persistent step kernel only)
    int ep_rank, ep_world;
    uint8_t* ep_local;           // this rank's exchange buffer (peers store into it)
    uint8_t* const* ep_peers;    // [ep_world] every rank's exchange buffer as mapped on this device
    unsigned* ep_seq;            // decode steps run so far (the same count on every rank)
    int ep_e0, ep_e1;            // experts this rank computes: [ep_e0, ep_e1)
    int ep_hg0, ep_hg1;          // head row groups (32 rows each) this rank scans
};

// Exchange buffer of one rank: MoE terms [2 layer parities][8 top-8 slots][H]
// floats written by the rank that owns each slot, then per-source flags and
// the head's per-rank (max logit, index).
constexpr int kEpMaxRanks = 8;
__host__ __device__ inline size_t ep_terms_bytes(int hidden) { return (size_t)2 * 8 * hidden * 4; }
__host__ __device__ inline size_t ep_xchg_bytes(int hidden) { return ep_terms_bytes(hidden) + 4096; }
struct EpTail {                  // at offset ep_terms_bytes(H)
    unsigned layer_cnt[kEpMaxRanks];     // per source rank: its CTAs' releases of MoE terms
    unsigned head_flag[kEpMaxRanks];
    double best_val[kEpMaxRanks];
    int best_idx[kEpMaxRanks];
};

enum CounterSlot { kCntRouter = 8, kCntHead = 9, kCntBarrier = 10, kCntTotal = 16 };

// Launchers.  All run on `st` and read pos/token from device memory, so they
// can be captured once into a CUDA graph.
void launch_embed(const Dev& d, cudaStream_t st);
void launch_qkv(const Dev& d, const LayerW& w, cudaStream_t st);
void launch_attn(const Dev& d, const LayerW& w, int layer, cudaStream_t st);
void launch_oproj(const Dev& d, const LayerW& w, cudaStream_t st);
void launch_router(const Dev& d, const LayerW& w, int layer, cudaStream_t st);
void launch_gateup(const Dev& d, const LayerW& w, int layer, cudaStream_t st);
void launch_down(const Dev& d, const LayerW& w, int layer, cudaStream_t st);
void launch_head(const Dev& d, cudaStream_t st);
// Top-N (N <= 32) of the double logits: per-CTA candidates, then one merge.
constexpr int kTopnParts = 148;
void launch_topn(const Dev& d, int top_n, double* cand_v, int* cand_i, int* out_idx, float* out_val, cudaStream_t st);
void launch_final_norm(const Dev& d, float* normalized, cudaStream_t st);
int head_grid_size(int device, const Dims& m, bool r8 = false);
size_t attn_scores_bytes(const Dims& m);
// Grid barriers per layer of the persistent step kernel: QKV, attention
// scores, attention context, O projection, router, gate/up, down.
constexpr int kPhasesPerLayer = 7;
bool geometry_supported(const Dims& m);
cudaError_t configure_kernels();
// Persistent one-launch decode step (qx_mega.cu).
int mega_setup(int device, const Dims& m, int* grid_out);
// Stand-alone two-phase attention (the one-launch kernel's attention code, qx_mega.cu).
bool attn2_supported(const Dims& m);
int attn_launches(const Dims& m);             // kernels launch_attn starts (1 or 2)
int qkv_launches(const Dev& d, const LayerW& w);   // kernels launch_qkv starts (1, or 3 for other mixes / q8)
// q8_k_compat kernels (qx_q8k.cu)
cudaError_t q8_configure();
void launch_q8_proj(const Dev& d, int type, const float* in, const float* norm_w, const uint8_t* W, int rows, int K,
                    float* out, int residual, cudaStream_t st);
void launch_q8_gateup(const Dev& d, const LayerW& w, int layer, cudaStream_t st);
void launch_q8_down(const Dev& d, const LayerW& w, int layer, cudaStream_t st);
void launch_q8_head(const Dev& d, cudaStream_t st);
cudaError_t attn2_configure();
void launch_attn2(const Dev& d, const LayerW& w, int layer, int sms, cudaStream_t st);
cudaError_t launch_decode_step(const Dev& d, const LayerW* layers_dev, int grid, cudaStream_t st);

}  // namespace qx
