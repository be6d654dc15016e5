// Engine runtime behind include/qx_cuda.h: tensor table, one-time HBM upload
// of the QXF1 tensors in their native block layouts, persistent INT8 KV,
// per-token CUDA graph, and the C entry points.
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <unordered_map>
#include <initializer_list>
#include <thread>
#include <atomic>
#include <algorithm>
#include <vector>

#include "qx_cuda.h"
#include "qx_host.h"
#include "qx_batch.h"
#include "qx_kernels.h"

#define QX_API extern "C" __attribute__((visibility("default")))

namespace {

using qx::Dev;
using qx::Dims;
using qx::LayerW;

struct Op {                  // one launch of the per-token sequence
    const char* name;
    int layer;
    int kind;
};

enum OpKind { kEmbed, kQkv, kAttn, kOproj, kRouter, kGateup, kDown, kHead, kStep };
const char* kOpNames[] = {"embed_q4k", "qkv_iq4xs", "attn_int8kv", "oproj_iq4xs",
                          "router_top8", "gateup_iq2xs_swiglu", "down_iq3xxs_wsum", "head_q6k_argmax",
                          "decode_step_persistent"};

}  // namespace

struct qx_cuda_engine {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    Dims dm{};
    Dev dev{};
    std::vector<LayerW> layers;
    void* weights = nullptr;     // one arena for every tensor
    size_t weight_bytes = 0;
    void* work = nullptr;        // activations, KV, tables
    size_t work_bytes = 0;
    qx::Tables* tables = nullptr;
    int* h_io = nullptr;         // pinned host staging: [0]=token [1]=pos [2]=next [3]=err
    cudaGraphExec_t graph = nullptr;
    bool use_graph = true;
    std::vector<Op> ops;
    LayerW* layers_dev = nullptr;   // device copy of the layer table (persistent step kernel)
    uint8_t* relay = nullptr;        // weights re-laid for the persistent step kernel (IQ2R, R4, R8)
    int mega_grid = 0;               // 0 = per-stage kernels
    int* d_topi = nullptr;
    double* d_logits_d = nullptr;    // final_head: double logits for the top-N
    double* d_cand_v = nullptr;      // top-N candidates per part
    int* d_cand_i = nullptr;
    uint8_t* h_stage = nullptr;      // pinned bounce buffer for large device-to-host copies
    size_t h_stage_bytes = 0, h_stage_used = 0;
    struct Pending { void* dst; size_t off, bytes; };
    std::vector<Pending> pending;    // bounce-buffer copies to finish after the stream syncs
    // expert parallelism
    uint8_t* ep_xchg = nullptr;      // this rank's exchange buffer (its own allocation, exported by IPC)
    uint8_t** ep_peers_dev = nullptr;
    std::vector<void*> ep_opened;    // peer buffers mapped by qx_cuda_ep_connect
    bool ep_connected = false;
    float* d_topv = nullptr;
    float* d_norm = nullptr;
    qx_cuda_profile prof{};
    // batched MoE (qx_cuda_moe_batch): one allocation sized for `cap` tokens
    struct Batch {
        size_t cap = 0;
        void* mem = nullptr;
        float *x, *xn, *gu, *h, *y, *out, *moe, *qkv, *qn, *ctxo, *ao;
        uint8_t *bqx, *bqh;
        int *sx, *sh, *sel, *cols, *tcols, *tpos, *tslot;
        int *count, *nitems;             // device-built expert slot lists: per-expert counts, item counts
        uint32_t *tok, *next;
        double* logits;                  // [cap][vocab] (batched decode's head)
        double* wsel;
        double* vd;                      // [ctx][kv_dim] widened V rows of a prompt's layer
        qx::GemmItem* items;
        size_t item_cap;
        // sequence slots of qx_cuda_decode_batch: their own INT8 KV caches
        void* slot_mem = nullptr;
        qx::KvView slots{};
    } batch;
};

namespace {

void set_err(char* err, uint64_t n, const std::string& m) {
    if (err && n) snprintf(err, (size_t)n, "%s", m.c_str());
}

// Kernels one per-stage decode step launches (attention may be two kernels).
size_t stage_launches(const qx_cuda_engine* E) {
    size_t k = 0;
    for (const Op& op : E->ops)
        k += op.kind == kAttn ? (size_t)qx::attn_launches(E->dm)
             : op.kind == kQkv ? (size_t)qx::qkv_launches(E->dev, E->layers[op.layer]) : 1u;
    return k;
}

bool cuda_ok(cudaError_t e, const char* what, char* err, uint64_t n) {
    if (e == cudaSuccess) return true;
    set_err(err, n, std::string(what) + ": " + cudaGetErrorString(e));
    return false;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

void run_op(qx_cuda_engine* E, const Op& op) {
    const Dev& d = E->dev;
    cudaStream_t st = E->stream;
    switch (op.kind) {
        case kEmbed: qx::launch_embed(d, st); break;
        case kQkv: qx::launch_qkv(d, E->layers[op.layer], st); break;
        case kAttn: qx::launch_attn(d, E->layers[op.layer], op.layer, st); break;
        case kOproj: qx::launch_oproj(d, E->layers[op.layer], st); break;
        case kRouter: qx::launch_router(d, E->layers[op.layer], op.layer, st); break;
        case kGateup: qx::launch_gateup(d, E->layers[op.layer], op.layer, st); break;
        case kDown: qx::launch_down(d, E->layers[op.layer], op.layer, st); break;
        case kHead: qx::launch_head(d, st); break;
        case kStep: qx::launch_decode_step(d, E->layers_dev, E->mega_grid, st); break;
    }
}

void build_ops(qx_cuda_engine* E) {
    E->ops.clear();
    if (E->mega_grid) {
        E->ops.push_back({kOpNames[kStep], -1, kStep});
        return;
    }
    E->ops.push_back({kOpNames[kEmbed], -1, kEmbed});
    for (int l = 0; l < E->dm.layers; ++l)
        for (int k = kQkv; k <= kDown; ++k) E->ops.push_back({kOpNames[k], l, k});
    E->ops.push_back({kOpNames[kHead], -1, kHead});
}

bool run_step(qx_cuda_engine* E, char* err, uint64_t n) {
    if (E->use_graph && E->graph) {
        if (!cuda_ok(cudaGraphLaunch(E->graph, E->stream), "cudaGraphLaunch", err, n)) return false;
        E->prof.graph_replays++;
    } else {
        for (const Op& op : E->ops) run_op(E, op);
        if (!cuda_ok(cudaGetLastError(), "kernel launch", err, n)) return false;
    }
    E->prof.kernel_launches += E->mega_grid ? 1 : stage_launches(E);
    E->prof.decode_steps++;
    return true;
}

struct Tensor {
    const qx_cuda_tensor* t;
    size_t offset;               // in the weight arena
};

// `types`: the accepted ggml types (the first is the benchmark mix's).
bool check_tensor(const std::unordered_map<std::string, const qx_cuda_tensor*>& by, const std::string& name,
                  std::initializer_list<uint32_t> types, uint32_t rank, uint64_t d0, uint64_t d1, uint64_t d2,
                  char* err, uint64_t n) {
    auto it = by.find(name);
    if (it == by.end()) { set_err(err, n, "tensor not found: " + name); return false; }
    const qx_cuda_tensor* t = it->second;
    const uint32_t type = t->ggml_type;
    bool accepted = false;
    std::string list;
    for (uint32_t a : types) {
        accepted |= a == type;
        list += (list.empty() ? "" : "/") + std::to_string(a);
    }
    if (!accepted) {
        set_err(err, n, "unsupported ggml type " + std::to_string(t->ggml_type) + " for " + name +
                            " (engine path expects " + list + ")");
        return false;
    }
    if (t->rank != rank || t->dims[0] != d0 || (rank > 1 && t->dims[1] != d1) || (rank > 2 && t->dims[2] != d2)) {
        set_err(err, n, "unexpected dimensions for " + name);
        return false;
    }
    uint32_t bv = 1, bb = 4;
    qxh_block_info(type, &bv, &bb);
    uint64_t elems = d0 * (rank > 1 ? d1 : 1) * (rank > 2 ? d2 : 1);
    if (t->byte_size != elems / bv * bb || !t->data) { set_err(err, n, "byte size inconsistent for " + name); return false; }
    return true;
}

}  // namespace

// ---------------------------------------------------------------------------
QX_API void qx_cuda_engine_destroy(qx_cuda_engine* E) {
    if (!E) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(E->device);
    if (E->stream) cudaStreamSynchronize(E->stream);
    if (E->graph) cudaGraphExecDestroy(E->graph);
    if (E->weights) cudaFree(E->weights);
    if (E->work) cudaFree(E->work);
    if (E->layers_dev) cudaFree(E->layers_dev);
    if (E->relay) cudaFree(E->relay);
    if (E->batch.mem) cudaFree(E->batch.mem);
    if (E->batch.slot_mem) cudaFree(E->batch.slot_mem);
    for (void* p : E->ep_opened) cudaIpcCloseMemHandle(p);
    if (E->ep_xchg) cudaFree(E->ep_xchg);
    if (E->ep_peers_dev) cudaFree(E->ep_peers_dev);
    if (E->h_io) cudaFreeHost(E->h_io);
    if (E->h_stage) cudaFreeHost(E->h_stage);
    if (E->own_stream && E->stream) cudaStreamDestroy(E->stream);
    cudaSetDevice(prev);
    delete E;
}

// The persistent kernel's re-laid weights store each IQ2_XS weight as an
// index into {8, 25, 43} and each IQ3_XXS weight as an index into
// {4, 12, ..., 52, 62} (times a sign); the lattices must hold exactly those.
static bool relay_tables_ok(const qxh_iq_tables* T) {
    for (int i = 0; i < 512; ++i)
        for (int j = 0; j < 8; ++j) {
            const int v = T->iq2xs[i][j];
            if (v != 8 && v != 25 && v != 43) return false;
        }
    for (int i = 0; i < 256; ++i)
        for (int j = 0; j < 4; ++j) {
            const int v = T->iq3xxs[i][j];
            if (!(v == 62 || (v >= 4 && v <= 52 && (v - 4) % 8 == 0))) return false;
        }
    return true;
}

QX_API int qx_cuda_engine_create(const qx_cuda_model* model, const qx_cuda_tensor* tensors, uint32_t count,
                                 const qx_cuda_options* opt, qx_cuda_engine** out, char* err, uint64_t n) {
    if (!model || !tensors || !count || !out) { set_err(err, n, "invalid argument"); return 0; }
    *out = nullptr;
    qx_cuda_options o{};
    o.device = -1;
    o.ctx_tokens = 4096;
    if (opt) o = *opt;
    if (o.nccl_comm) { set_err(err, n, "nccl_comm is reserved and must be NULL"); return 0; }
    if (o.ep_world > (uint32_t)qx::kEpMaxRanks || (o.ep_world > 1 && o.ep_rank >= o.ep_world)) {
        set_err(err, n, "invalid expert-parallel rank or world size");
        return 0;
    }
    Dims dm{};
    dm.layers = (int)model->layers; dm.hidden = (int)model->hidden; dm.q_heads = (int)model->q_heads;
    dm.kv_heads = (int)model->kv_heads; dm.head_dim = (int)model->head_dim; dm.vocab = (int)model->vocab;
    dm.experts = (int)model->experts; dm.moe_inter = (int)model->moe_intermediate; dm.ctx = (int)o.ctx_tokens;
    if (dm.layers < 1 || dm.hidden < 256 || dm.hidden % 256 || dm.hidden > 8192 || dm.kv_heads < 1 ||
        dm.q_heads % dm.kv_heads || dm.q_heads / dm.kv_heads > 8 || dm.head_dim != 128 || dm.q_dim() % 256 ||
        dm.q_dim() > 8192 || dm.vocab < 16 || dm.vocab % 16 || dm.experts < 8 || dm.experts > 256 ||
        model->experts_per_token != 8 || dm.moe_inter < 256 || dm.moe_inter % 256 || dm.moe_inter > 2048 ||
        dm.ctx < 1 || dm.ctx > 65536 || !qx::geometry_supported(dm)) {
        set_err(err, n, "unsupported model geometry for the B200 engine");
        return 0;
    }
    std::unordered_map<std::string, const qx_cuda_tensor*> by;
    for (uint32_t i = 0; i < count; ++i)
        if (tensors[i].name) by[tensors[i].name] = &tensors[i];
    const uint64_t H = dm.hidden, Q = dm.q_dim(), KV = dm.kv_dim(), Ee = dm.experts, I = dm.moe_inter;
    std::vector<std::string> names;
    auto need = [&](const std::string& nm, std::initializer_list<uint32_t> types, uint32_t rank, uint64_t d0,
                    uint64_t d1, uint64_t d2) {
        names.push_back(nm);
        return check_tensor(by, nm, types, rank, d0, d1, d2, err, n);
    };
    const std::initializer_list<uint32_t> kAttnT = {QXH_IQ4_XS, QXH_Q5_K, QXH_Q6_K};
    const std::initializer_list<uint32_t> kGateT = {QXH_IQ2_XS, QXH_IQ2_S};
    const std::initializer_list<uint32_t> kDownT = {QXH_IQ3_XXS, QXH_IQ3_S, QXH_IQ4_XS};
    bool ok = need("token_embd.weight", {QXH_Q4_K}, 2, H, dm.vocab, 0) &&
              need("output_norm.weight", {QXH_F32}, 1, H, 0, 0) && need("output.weight", {QXH_Q6_K}, 2, H, dm.vocab, 0);
    for (int l = 0; ok && l < dm.layers; ++l) {
        std::string p = "blk." + std::to_string(l) + ".";
        ok = need(p + "attn_norm.weight", {QXH_F32}, 1, H, 0, 0) && need(p + "attn_q.weight", kAttnT, 2, H, Q, 0) &&
             need(p + "attn_k.weight", kAttnT, 2, H, KV, 0) && need(p + "attn_v.weight", kAttnT, 2, H, KV, 0) &&
             need(p + "attn_output.weight", kAttnT, 2, Q, H, 0) &&
             need(p + "attn_q_norm.weight", {QXH_F32}, 1, dm.head_dim, 0, 0) &&
             need(p + "attn_k_norm.weight", {QXH_F32}, 1, dm.head_dim, 0, 0) &&
             need(p + "ffn_norm.weight", {QXH_F32}, 1, H, 0, 0) &&
             need(p + "ffn_gate_inp.weight", {QXH_F32}, 2, H, Ee, 0) &&
             need(p + "ffn_gate_exps.weight", kGateT, 3, H, I, Ee) && need(p + "ffn_up_exps.weight", kGateT, 3, H, I, Ee) &&
             need(p + "ffn_down_exps.weight", kDownT, 3, I, H, Ee);
        if (ok && by[p + "ffn_gate_exps.weight"]->ggml_type != by[p + "ffn_up_exps.weight"]->ggml_type) {
            set_err(err, n, "gate and up experts must share one type: " + p);
            ok = false;
        }
    }
    if (!ok) return 0;
    if (o.flags & QX_CUDA_VERIFY_CHECKSUMS) {
        // FNV-1a is sequential within a tensor, independent across tensors:
        // verify on every host core, largest tensors first; report the first
        // mismatch in directory order
        std::vector<const qx_cuda_tensor*> tp(names.size());   // resolved here: the workers only read
        for (size_t i = 0; i < names.size(); ++i) tp[i] = by[names[i]];
        std::vector<size_t> order(names.size());
        for (size_t i = 0; i < order.size(); ++i) order[i] = i;
        std::sort(order.begin(), order.end(), [&](size_t a, size_t b) { return tp[a]->byte_size > tp[b]->byte_size; });
        std::vector<char> bad(names.size(), 0);
        std::atomic<size_t> next{0};
        const unsigned nt = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
        std::vector<std::thread> pool;
        for (unsigned k = 0; k < nt; ++k)
            pool.emplace_back([&]() {
                for (size_t j; (j = next.fetch_add(1)) < order.size();) {
                    const qx_cuda_tensor* t = tp[order[j]];
                    bad[order[j]] = qxh_fnv1a64(t->data, t->byte_size) != t->checksum;
                }
            });
        for (auto& th : pool) th.join();
        for (size_t i = 0; i < names.size(); ++i)
            if (bad[i]) { set_err(err, n, "tensor checksum mismatch: " + names[i]); return 0; }
    }

    auto* E = new qx_cuda_engine();
    E->dm = dm;
    int dev = o.device;
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    E->device = dev;
    E->use_graph = !(o.flags & QX_CUDA_NO_GRAPH);
    auto fail = [&](cudaError_t e, const char* what) {
        cuda_ok(e, what, err, n);
        qx_cuda_engine_destroy(E);
        return 0;
    };
    cudaError_t ce = cudaSetDevice(dev);
    if (ce != cudaSuccess) return fail(ce, "cudaSetDevice");
    if (o.stream) E->stream = (cudaStream_t)o.stream;
    else {
        ce = cudaStreamCreateWithFlags(&E->stream, cudaStreamNonBlocking);
        if (ce != cudaSuccess) return fail(ce, "cudaStreamCreate");
        E->own_stream = true;
    }
    ce = qx::configure_kernels();
    if (ce == cudaSuccess) ce = qx::moe_batch_configure();
    if (ce != cudaSuccess) return fail(ce, "cudaFuncSetAttribute");

    // weight arena: every tensor, 256-byte aligned, in its native layout
    std::map<std::string, size_t> off;
    size_t wb = 0;
    for (const auto& nm : names) {
        off[nm] = wb;
        wb = align_up(wb + by[nm]->byte_size, 256);
    }
    E->weight_bytes = wb;
    ce = cudaMalloc(&E->weights, wb);
    if (ce != cudaSuccess) return fail(ce, "cudaMalloc(weights)");
    {
        // two pinned staging buffers: the host copy of chunk i+1 (4 threads)
        // overlaps the DMA of chunk i
        const size_t kChunk = (size_t)64 << 20;
        uint8_t* pin[2] = {nullptr, nullptr};
        cudaEvent_t done[2] = {nullptr, nullptr};
        ce = cudaHostAlloc((void**)&pin[0], 2 * kChunk, cudaHostAllocDefault);
        if (ce == cudaSuccess) { pin[1] = pin[0] + kChunk; ce = cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming); }
        if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming);
        int slot = 0;
        bool used[2] = {false, false};
        for (size_t i = 0; ce == cudaSuccess && i < names.size(); ++i) {
            const qx_cuda_tensor* t = by[names[i]];
            for (size_t pos = 0; ce == cudaSuccess && pos < t->byte_size; pos += kChunk) {
                const size_t len = std::min(kChunk, (size_t)t->byte_size - pos);
                if (used[slot]) ce = cudaEventSynchronize(done[slot]);     // its previous DMA is finished
                if (ce != cudaSuccess) break;
                const uint8_t* src = static_cast<const uint8_t*>(t->data) + pos;
                const size_t part = (len + 3) / 4;
                std::thread cp[4];
                for (int k = 0; k < 4; ++k) {
                    const size_t a = std::min(len, k * part), b = std::min(len, (k + 1) * part);
                    cp[k] = std::thread([=]() { if (b > a) memcpy(pin[slot] + a, src + a, b - a); });
                }
                for (auto& th : cp) th.join();
                ce = cudaMemcpyAsync((uint8_t*)E->weights + off[names[i]] + pos, pin[slot], len, cudaMemcpyHostToDevice,
                                     E->stream);
                if (ce == cudaSuccess) ce = cudaEventRecord(done[slot], E->stream);
                used[slot] = true;
                slot ^= 1;
            }
            E->prof.host_to_device_bytes += t->byte_size;
        }
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(E->stream);
        for (auto ev : done) if (ev) cudaEventDestroy(ev);
        if (pin[0]) cudaFreeHost(pin[0]);
        if (ce != cudaSuccess) return fail(ce, "upload weights");
    }
    auto W = [&](const std::string& nm) { return (const uint8_t*)E->weights + off[nm]; };
    for (int l = 0; l < dm.layers; ++l) {
        std::string p = "blk." + std::to_string(l) + ".";
        LayerW lw{};
        lw.attn_norm = (const float*)W(p + "attn_norm.weight");
        lw.wq = W(p + "attn_q.weight");
        lw.wk = W(p + "attn_k.weight");
        lw.wv = W(p + "attn_v.weight");
        lw.wo = W(p + "attn_output.weight");
        lw.q_norm = (const float*)W(p + "attn_q_norm.weight");
        lw.k_norm = (const float*)W(p + "attn_k_norm.weight");
        lw.ffn_norm = (const float*)W(p + "ffn_norm.weight");
        lw.router = (const float*)W(p + "ffn_gate_inp.weight");
        lw.gate = W(p + "ffn_gate_exps.weight");
        lw.up = W(p + "ffn_up_exps.weight");
        lw.down = W(p + "ffn_down_exps.weight");
        lw.tq = (int)by[p + "attn_q.weight"]->ggml_type;
        lw.tk = (int)by[p + "attn_k.weight"]->ggml_type;
        lw.tv = (int)by[p + "attn_v.weight"]->ggml_type;
        lw.to = (int)by[p + "attn_output.weight"]->ggml_type;
        lw.tgate = (int)by[p + "ffn_gate_exps.weight"]->ggml_type;
        lw.tup = (int)by[p + "ffn_up_exps.weight"]->ggml_type;
        lw.tdown = (int)by[p + "ffn_down_exps.weight"]->ggml_type;
        E->layers.push_back(lw);
    }

    // work buffers
    Dev& d = E->dev;
    d.dm = dm;
    d.tok_embd = W("token_embd.weight");
    d.out_norm = (const float*)W("output_norm.weight");
    d.head = W("output.weight");
    d.head_grid = qx::head_grid_size(dev, dm);
    d.head_grid_r8 = qx::head_grid_size(dev, dm, true);
    const size_t L = dm.layers, C = dm.ctx, D = dm.head_dim;
    struct Slot { void** p; size_t bytes; };
    std::vector<Slot> slots;
    size_t wk = 0;
    auto add = [&](void** p, size_t bytes) { slots.push_back({p, bytes}); wk = align_up(wk + bytes, 256); };
    add((void**)&E->tables, sizeof(qx::Tables));
    add((void**)&d.rope, C * (D / 2) * 2 * sizeof(double));
    add((void**)&d.x, H * 4);
    add((void**)&d.xn, std::max(H, Q) * 4);
    add((void**)&d.qkv, (Q + 2 * KV) * 4);
    add((void**)&d.kcache, L * C * KV);
    add((void**)&d.vcache, L * C * KV);
    add((void**)&d.kscale, L * C * 4);
    add((void**)&d.vscale, L * C * 4);
    add((void**)&d.attn_scores, qx::attn_scores_bytes(dm));
    add((void**)&d.ctxv, Q * 4);
    add((void**)&d.attn_out, H * 4);
    add((void**)&d.moe_out, H * 4);
    add((void**)&d.router_logits, Ee * 8);
    add((void**)&d.sel, L * 8 * 4);
    add((void**)&d.selw, L * 8 * 4);
    add((void**)&d.selw_d, 8 * 8);
    add((void**)&d.hbuf, 8 * I * 4);
    add((void**)&d.logits, (size_t)dm.vocab * 4);
    // argmax partials: one per CTA of the per-stage head (either layout) or
    // of the persistent step kernel (one CTA per SM), whichever is largest
    int sm_count = 0;
    cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
    const size_t partials = (size_t)std::max({d.head_grid, d.head_grid_r8, sm_count});
    add((void**)&d.best_val, partials * sizeof(double));
    add((void**)&d.best_idx, partials * 4);
    add((void**)&d.counters, qx::kCntTotal * 4);
    add((void**)&d.token, 4);
    add((void**)&d.pos, 4);
    add((void**)&d.tokens_out, C * 4);
    add((void**)&d.err, 4);
    add((void**)&d.ep_seq, 4);
    add((void**)&E->d_logits_d, (size_t)dm.vocab * 8);
    add((void**)&E->d_cand_v, (size_t)qx::kTopnParts * 32 * 8);
    add((void**)&E->d_cand_i, (size_t)qx::kTopnParts * 32 * 4);
    add((void**)&E->d_topi, 32 * 4);
    add((void**)&E->d_topv, 32 * 4);
    add((void**)&E->d_norm, H * 4);
    E->work_bytes = wk;
    ce = cudaMalloc(&E->work, wk);
    if (ce != cudaSuccess) return fail(ce, "cudaMalloc(work)");
    ce = cudaMemsetAsync(E->work, 0, wk, E->stream);
    if (ce != cudaSuccess) return fail(ce, "cudaMemset(work)");
    size_t cur = 0;
    for (auto& s : slots) {
        *s.p = (uint8_t*)E->work + cur;
        cur = align_up(cur + s.bytes, 256);
    }
    d.tables = E->tables;

    // lattice tables and RoPE table (host libm, double, as src/qx_format.c:4630-4634)
    qx::Tables ht{};
    const qxh_iq_tables* T = qxh_tables();
    for (int i = 0; i < 512; ++i) for (int j = 0; j < 8; ++j) ht.iq2xs[i][j] = (float)T->iq2xs[i][j];
    for (int i = 0; i < 256; ++i) for (int j = 0; j < 4; ++j) ht.iq3xxs[i][j] = (float)T->iq3xxs[i][j];
    memcpy(ht.ksigns, T->ksigns, 128);
    for (int i = 0; i < 1024; ++i) memcpy(ht.iq2s[i], T->iq2s[i], 8);
    for (int i = 0; i < 512; ++i) memcpy(&ht.iq3s[i], T->iq3s[i], 4);
    static const int8_t kv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
    for (int i = 0; i < 16; ++i) ht.kvalues[i] = (float)kv[i];
    std::vector<double> rope(C * (D / 2) * 2);
    for (size_t p = 0; p < C; ++p)
        for (size_t i = 0; i < D / 2; ++i) {
            const double f = pow(1000000.0, -(2.0 * (double)i) / (double)D);
            const double a = (double)p * f;
            rope[(p * (D / 2) + i) * 2] = cos(a);
            rope[(p * (D / 2) + i) * 2 + 1] = sin(a);
        }
    ce = cudaMemcpyAsync(E->tables, &ht, sizeof(ht), cudaMemcpyHostToDevice, E->stream);
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync((void*)d.rope, rope.data(), rope.size() * sizeof(double), cudaMemcpyHostToDevice, E->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(E->stream);
    if (ce != cudaSuccess) return fail(ce, "upload tables");
    ce = cudaHostAlloc((void**)&E->h_io, 64, cudaHostAllocDefault);
    if (ce == cudaSuccess) {
        E->h_stage_bytes = (size_t)dm.vocab * 4 + (size_t)64 * 1024;   // logits + the small outputs of one call
        ce = cudaHostAlloc((void**)&E->h_stage, E->h_stage_bytes, cudaHostAllocDefault);
    }
    if (ce != cudaSuccess) return fail(ce, "cudaHostAlloc");
    // the one-launch kernel covers the benchmark mix; any other mix runs per stage
    d.q8 = (o.flags & QX_CUDA_Q8K_COMPAT) ? 1 : 0;
    if (d.q8 && o.ep_world > 1) {
        set_err(err, n, "q8_k_compat runs on the per-stage path, without expert parallelism");
        qx_cuda_engine_destroy(E);
        return 0;
    }
    bool mega = !(o.flags & QX_CUDA_PER_STAGE) && !d.q8 && qx::benchmark_mix(E->layers.data(), dm.layers) &&
                relay_tables_ok(qxh_tables()) && qx::mega_setup(dev, dm, &E->mega_grid);
    size_t relay_per = 0;                    // re-laid bytes per layer
    if (mega) {
        // the re-laid copies need ~17 GB for the full model: without the room,
        // the engine runs the per-stage path on the GGUF layouts instead
        const int H = dm.hidden, Q = dm.q_dim(), KV = dm.kv_dim(), I = dm.moe_inter;
        relay_per = 2 * (size_t)dm.experts * I * qx::iq2r_row_bytes(H) + (size_t)(Q + 2 * KV) * qx::r4_bytes_per_row(H) +
                    (size_t)H * qx::r4_bytes_per_row(Q) + (size_t)dm.experts * H * qx::r4_bytes_per_row(I);
        const size_t relay_bytes = relay_per * (size_t)dm.layers + (size_t)dm.vocab * qx::r8_bytes_per_row(H);
        if (cudaMalloc((void**)&E->relay, relay_bytes) != cudaSuccess) {
            (void)cudaGetLastError();
            E->relay = nullptr;
            mega = false;
        }
    }
    if (mega) {
        // the persistent kernel reads its weights in its own layouts (one
        // table index per weight, decoded by byte permutes): re-lay them once
        const int H = dm.hidden, Q = dm.q_dim(), KV = dm.kv_dim(), I = dm.moe_inter;
        const size_t gu = (size_t)dm.experts * I * qx::iq2r_row_bytes(H);
        const size_t qkv = (size_t)(Q + 2 * KV) * qx::r4_bytes_per_row(H), wo = (size_t)H * qx::r4_bytes_per_row(Q);
        const size_t per = relay_per;            // = 2 gu + qkv + wo + down
        d.head_r = E->relay + per * (size_t)dm.layers;
        ce = qx::launch_r8_repack(d.head, const_cast<uint8_t*>(d.head_r), (size_t)dm.vocab, H, E->stream);
        for (int l = 0; l < dm.layers && ce == cudaSuccess; ++l) {
            LayerW& w = E->layers[l];
            uint8_t* p = E->relay + (size_t)l * per;
            const size_t rbh = qx::r4_bytes_per_row(H);
            w.gate_r = p, w.up_r = p + gu, p += 2 * gu;
            w.wq_r = p, w.wk_r = p + (size_t)Q * rbh, w.wv_r = p + (size_t)(Q + KV) * rbh, p += qkv;
            w.wo_r = p, p += wo;
            w.down_r = p;
            const qx::Tables* T = E->tables;
            ce = qx::launch_iq2r_repack(w.gate, const_cast<uint8_t*>(w.gate_r), (size_t)dm.experts * I, H, T, E->stream);
            if (ce == cudaSuccess) ce = qx::launch_iq2r_repack(w.up, const_cast<uint8_t*>(w.up_r), (size_t)dm.experts * I, H, T, E->stream);
            if (ce == cudaSuccess) ce = qx::launch_r4_repack(w.wq, const_cast<uint8_t*>(w.wq_r), Q, H, 23, T, E->stream);
            if (ce == cudaSuccess) ce = qx::launch_r4_repack(w.wk, const_cast<uint8_t*>(w.wk_r), KV, H, 23, T, E->stream);
            if (ce == cudaSuccess) ce = qx::launch_r4_repack(w.wv, const_cast<uint8_t*>(w.wv_r), KV, H, 23, T, E->stream);
            if (ce == cudaSuccess) ce = qx::launch_r4_repack(w.wo, const_cast<uint8_t*>(w.wo_r), H, Q, 23, T, E->stream);
            if (ce == cudaSuccess)
                ce = qx::launch_r4_repack(w.down, const_cast<uint8_t*>(w.down_r), (size_t)dm.experts * H, I, 18, T, E->stream);
        }
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(E->stream);
        if (ce != cudaSuccess) return fail(ce, "weight re-lay");
        ce = cudaMalloc((void**)&E->layers_dev, E->layers.size() * sizeof(LayerW));
        if (ce == cudaSuccess)
            ce = cudaMemcpy(E->layers_dev, E->layers.data(), E->layers.size() * sizeof(LayerW), cudaMemcpyHostToDevice);
        if (ce != cudaSuccess) return fail(ce, "layer table");
    } else {
        E->mega_grid = 0;
    }
    d.ep_world = o.ep_world > 1 ? (int)o.ep_world : 1;
    d.ep_rank = o.ep_world > 1 ? (int)o.ep_rank : 0;
    {
        // all experts and head rows when the partition does not apply (the
        // persistent kernel, the only user, requires vocab % 32 == 0)
        uint32_t r[4] = {0u, (uint32_t)dm.experts, 0u, (uint32_t)dm.vocab / 32u * 32u};
        qx_cuda_ep_partition((uint32_t)dm.experts, (uint32_t)dm.vocab, (uint32_t)d.ep_world, (uint32_t)d.ep_rank, r);
        d.ep_e0 = (int)r[0];
        d.ep_e1 = (int)r[1];
        d.ep_hg0 = (int)(r[2] / 32);
        d.ep_hg1 = (int)(r[3] / 32);
    }
    if (d.ep_world > 1) {
        // the exchange lives in its own allocation so that peers can map it (CUDA IPC)
        if (!E->mega_grid || dm.hidden > 8 * dm.moe_inter) {
            set_err(err, n, "expert parallelism needs the persistent step kernel for this geometry");
            qx_cuda_engine_destroy(E);
            return 0;
        }
        ce = cudaMalloc((void**)&E->ep_xchg, qx::ep_xchg_bytes(dm.hidden));
        if (ce == cudaSuccess) ce = cudaMemset(E->ep_xchg, 0, qx::ep_xchg_bytes(dm.hidden));
        if (ce == cudaSuccess) ce = cudaMalloc((void**)&E->ep_peers_dev, qx::kEpMaxRanks * sizeof(uint8_t*));
        if (ce == cudaSuccess) ce = cudaMemset(E->ep_peers_dev, 0, qx::kEpMaxRanks * sizeof(uint8_t*));
        if (ce != cudaSuccess) return fail(ce, "expert-parallel exchange buffer");
        d.ep_local = E->ep_xchg;
        d.ep_peers = E->ep_peers_dev;
    }
    build_ops(E);

    if (E->use_graph) {
        cudaGraph_t g = nullptr;
        ce = cudaStreamBeginCapture(E->stream, cudaStreamCaptureModeThreadLocal);
        if (ce != cudaSuccess) return fail(ce, "cudaStreamBeginCapture");
        for (const Op& op : E->ops) run_op(E, op);
        cudaError_t le = cudaGetLastError();
        ce = cudaStreamEndCapture(E->stream, &g);
        if (le != cudaSuccess) { if (g) cudaGraphDestroy(g); return fail(le, "capture launch"); }
        if (ce != cudaSuccess) return fail(ce, "cudaStreamEndCapture");
        ce = cudaGraphInstantiate(&E->graph, g, 0);
        cudaGraphDestroy(g);
        if (ce != cudaSuccess) return fail(ce, "cudaGraphInstantiate");
    }
    E->prof.device_bytes = wb + wk;
    snprintf(E->prof.backend, sizeof(E->prof.backend), "b200-sm100a");
    *out = E;
    return 1;
}

namespace {

int create_from_file(const qxh_file& f, const qx_cuda_options* opt, qx_cuda_engine** out, char* err, uint64_t n) {
    const qxh_manifest& m = f.header.manifest;
    qx_cuda_model model{m.layers, m.hidden, m.q_heads, m.kv_heads, m.head_dim, m.vocab, m.experts,
                        m.experts_per_token, m.moe_intermediate};
    std::vector<qx_cuda_tensor> ts(f.header.tensor_count);
    for (uint32_t i = 0; i < f.header.tensor_count; ++i) {
        const qxh_dir_entry& e = f.dir[i];
        qx_cuda_tensor& t = ts[i];
        t.name = e.name;
        t.ggml_type = e.flags;
        t.rank = e.rank;
        for (int k = 0; k < 4; ++k) t.dims[k] = e.dims[k];
        t.byte_size = e.byte_size;
        t.checksum = e.checksum;
        t.data = f.base + e.offset;
    }
    return qx_cuda_engine_create(&model, ts.data(), (uint32_t)ts.size(), opt, out, err, n);
}

}  // namespace

QX_API int qx_cuda_engine_create_from_qxf(const char* path, const qx_cuda_options* opt, qx_cuda_engine** out,
                                          char* err, uint64_t n) {
    qxh_file f;
    if (!qxh_open_path(path, &f, err, n)) return 0;
    int ok = create_from_file(f, opt, out, err, n);
    qxh_close(&f);
    return ok;
}

QX_API int qx_cuda_engine_create_from_image(const void* image, uint64_t size, const qx_cuda_options* opt,
                                            qx_cuda_engine** out, char* err, uint64_t n) {
    qxh_file f;
    if (!qxh_open_image(image, size, &f, err, n)) return 0;
    return create_from_file(f, opt, out, err, n);
}

namespace {

struct DeviceGuard {
    int prev = 0;
    explicit DeviceGuard(int d) { cudaGetDevice(&prev); cudaSetDevice(d); }
    ~DeviceGuard() { cudaSetDevice(prev); }
};

// Copy the error bits back, clear them, and turn them into a message.
bool finish(qx_cuda_engine* E, char* err, uint64_t n) {
    cudaError_t ce = cudaMemcpyAsync(E->h_io + 3, E->dev.err, 4, cudaMemcpyDeviceToHost, E->stream);
    E->prof.device_to_host_bytes += 4;
    if (ce == cudaSuccess) ce = cudaMemsetAsync(E->dev.err, 0, 4, E->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(E->stream);
    const bool copied = ce == cudaSuccess;
    for (const auto& p : E->pending)
        if (copied) memcpy(p.dst, E->h_stage + p.off, p.bytes);
    E->pending.clear();
    E->h_stage_used = 0;
    if (!cuda_ok(ce, "device execution", err, n)) return false;
    const int bits = E->h_io[3];
    if (bits & qx::kErrToken) { set_err(err, n, "token id out of range"); return false; }
    if (bits & qx::kErrPosition) { set_err(err, n, "steps exceed ctx"); return false; }
    if (bits & qx::kErrNonFinite) { set_err(err, n, "non-finite final logit"); return false; }
    if (bits & qx::kErrRouter) { set_err(err, n, "invalid selected router weights"); return false; }
    if (bits & qx::kErrTimeout) { set_err(err, n, "device grid barrier timed out"); return false; }
    if (bits & qx::kErrQ8Input) { set_err(err, n, "Q8_K activation contains NaN or Inf"); return false; }
    if (bits & qx::kErrQ8Expert) { set_err(err, n, "non-finite packed expert Q8_K output"); return false; }
    if (bits & qx::kErrQ8Head) { set_err(err, n, "non-finite final Q6_K Q8_K logit"); return false; }
    return true;
}

// An expert-parallel engine runs decode steps only once every peer is mapped.
bool ep_ready(const qx_cuda_engine* E, char* err, uint64_t n) {
    if (E->dev.ep_world > 1 && !E->ep_connected) {
        set_err(err, n, "expert-parallel engine is not connected to its peers");
        return false;
    }
    return true;
}

bool set_scalars(qx_cuda_engine* E, uint32_t token, uint32_t pos, char* err, uint64_t n) {
    E->h_io[0] = (int)token;
    E->h_io[1] = (int)pos;
    cudaError_t ce = cudaMemcpyAsync(E->dev.token, E->h_io, 4, cudaMemcpyHostToDevice, E->stream);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(E->dev.pos, E->h_io + 1, 4, cudaMemcpyHostToDevice, E->stream);
    E->prof.host_to_device_bytes += 8;
    return cuda_ok(ce, "cudaMemcpyAsync(scalars)", err, n);
}

// Device-to-host copy of a call's output; large ones go through the pinned
// bounce buffer (a pageable destination is copied at pageable speed) and land
// in `dst` when finish() has synchronised.
bool d2h(qx_cuda_engine* E, void* dst, const void* src, size_t bytes, char* err, uint64_t n) {
    if (!dst) return true;
    E->prof.device_to_host_bytes += bytes;
    // through the pinned staging arena whenever it fits: a copy into pageable
    // memory would wait for the stream on the spot; finish() (or kv_read)
    // delivers the staged bytes after its one synchronisation
    const size_t off = (E->h_stage_used + 255) / 256 * 256;
    if (E->h_stage && off + bytes <= E->h_stage_bytes) {
        if (!cuda_ok(cudaMemcpyAsync(E->h_stage + off, src, bytes, cudaMemcpyDeviceToHost, E->stream),
                     "cudaMemcpyAsync(d2h)", err, n)) {
            E->pending.clear();               // the call fails: none of its outputs is delivered
            E->h_stage_used = 0;
            return false;
        }
        E->h_stage_used = off + bytes;
        E->pending.push_back({dst, off, bytes});
        return true;
    }
    if (cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, E->stream), "cudaMemcpyAsync(d2h)", err, n))
        return true;
    E->pending.clear();
    E->h_stage_used = 0;
    return false;
}

// Inputs that fit the pinned arena are copied into it first, so the transfer
// is asynchronous; every caller synchronises the stream before it returns
// (finish(), kv_write, kv_read), and only then is the arena reused.
bool h2d(qx_cuda_engine* E, void* dst, const void* src, size_t bytes, char* err, uint64_t n) {
    E->prof.host_to_device_bytes += bytes;
    const size_t off = (E->h_stage_used + 255) / 256 * 256;
    if (E->h_stage && bytes && off + bytes <= E->h_stage_bytes) {
        memcpy(E->h_stage + off, src, bytes);
        E->h_stage_used = off + bytes;
        src = E->h_stage + off;
    }
    return cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, E->stream), "cudaMemcpyAsync(h2d)", err, n);
}

}  // namespace

QX_API int qx_cuda_reset(qx_cuda_engine* E, char* err, uint64_t n) {
    if (!E) { set_err(err, n, "invalid argument"); return 0; }
    DeviceGuard g(E->device);
    const size_t L = E->dm.layers, C = E->dm.ctx, KV = E->dm.kv_dim();
    cudaError_t ce = cudaMemsetAsync(E->dev.kcache, 0, L * C * KV, E->stream);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(E->dev.vcache, 0, L * C * KV, E->stream);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(E->dev.kscale, 0, L * C * 4, E->stream);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(E->dev.vscale, 0, L * C * 4, E->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(E->stream);
    return cuda_ok(ce, "reset", err, n) ? 1 : 0;
}

QX_API int qx_cuda_decode_step(qx_cuda_engine* E, uint32_t token, uint32_t position, uint32_t* next_token,
                               float* logits, float* final_residual, uint32_t* experts, float* routing, char* err,
                               uint64_t n) {
    if (!E || !next_token) { set_err(err, n, "invalid argument"); return 0; }
    if (token >= (uint32_t)E->dm.vocab) { set_err(err, n, "prompt token out of range"); return 0; }
    if (position >= (uint32_t)E->dm.ctx) { set_err(err, n, "steps exceed ctx"); return 0; }
    DeviceGuard g(E->device);
    if (!ep_ready(E, err, n) || !set_scalars(E, token, position, err, n) || !run_step(E, err, n)) return 0;
    if (!d2h(E, E->h_io + 2, E->dev.token, 4, err, n)) return 0;
    const size_t L = E->dm.layers;
    if (!d2h(E, logits, E->dev.logits, (size_t)E->dm.vocab * 4, err, n) ||
        !d2h(E, final_residual, E->dev.x, (size_t)E->dm.hidden * 4, err, n) ||
        !d2h(E, experts, E->dev.sel, L * 8 * 4, err, n) || !d2h(E, routing, E->dev.selw, L * 8 * 4, err, n))
        return 0;
    if (!finish(E, err, n)) return 0;
    *next_token = (uint32_t)E->h_io[2];
    return 1;
}

QX_API int qx_cuda_generate(qx_cuda_engine* E, uint32_t token, uint32_t position, uint32_t steps,
                            uint32_t* tokens_out, char* err, uint64_t n) {
    if (!E || !tokens_out || !steps) { set_err(err, n, "invalid argument"); return 0; }
    if (token >= (uint32_t)E->dm.vocab) { set_err(err, n, "prompt token out of range"); return 0; }
    if ((uint64_t)position + steps > (uint64_t)E->dm.ctx) { set_err(err, n, "steps exceed ctx"); return 0; }
    DeviceGuard g(E->device);
    if (!ep_ready(E, err, n) || !set_scalars(E, token, position, err, n)) return 0;
    for (uint32_t s = 0; s < steps; ++s)
        if (!run_step(E, err, n)) return 0;
    if (!d2h(E, tokens_out, E->dev.tokens_out + position, (size_t)steps * 4, err, n)) return 0;
    return finish(E, err, n) ? 1 : 0;
}

QX_API int qx_cuda_final_head(qx_cuda_engine* E, const float* residual, float* normalized, float* logits,
                              uint32_t top_n, uint32_t* top_tokens, float* top_logits, char* err, uint64_t n) {
    if (!E || !residual) { set_err(err, n, "invalid final head argument"); return 0; }
    if (top_n > 32) top_n = 32;
    DeviceGuard g(E->device);
    if (!h2d(E, E->dev.x, residual, (size_t)E->dm.hidden * 4, err, n)) return 0;
    E->h_io[1] = 0;
    if (!cuda_ok(cudaMemcpyAsync(E->dev.pos, E->h_io + 1, 4, cudaMemcpyHostToDevice, E->stream), "h2d", err, n)) return 0;
    if (top_n && E->dm.vocab > qx::kTopnParts * 2048) { set_err(err, n, "vocabulary too large for the top-N"); return 0; }
    Dev dh = E->dev;
    dh.logits_d = top_n ? E->d_logits_d : nullptr;
    qx::launch_head(dh, E->stream);
    E->prof.kernel_launches++;
    if (normalized) { qx::launch_final_norm(E->dev, E->d_norm, E->stream); E->prof.kernel_launches++; }
    if (top_n) {
        qx::launch_topn(dh, (int)top_n, E->d_cand_v, E->d_cand_i, E->d_topi, E->d_topv, E->stream);
        E->prof.kernel_launches += 2;
    }
    if (!cuda_ok(cudaGetLastError(), "kernel launch", err, n)) return 0;
    if (!d2h(E, normalized, E->d_norm, (size_t)E->dm.hidden * 4, err, n) ||
        !d2h(E, logits, E->dev.logits, (size_t)E->dm.vocab * 4, err, n) ||
        !d2h(E, top_n ? top_tokens : nullptr, E->d_topi, top_n * 4, err, n) ||
        !d2h(E, top_n ? top_logits : nullptr, E->d_topv, top_n * 4, err, n))
        return 0;
    return finish(E, err, n) ? 1 : 0;
}

QX_API int qx_cuda_moe_layer(qx_cuda_engine* E, uint32_t layer, const float* x, float* layer_output,
                             float* moe_output, uint32_t selected[8], float weights[8], char* err, uint64_t n) {
    if (!E || !x || layer >= (uint32_t)E->dm.layers) { set_err(err, n, "invalid packed expert matvec argument"); return 0; }
    DeviceGuard g(E->device);
    const LayerW& w = E->layers[layer];
    if (!h2d(E, E->dev.x, x, (size_t)E->dm.hidden * 4, err, n)) return 0;
    qx::launch_router(E->dev, w, (int)layer, E->stream);
    qx::launch_gateup(E->dev, w, (int)layer, E->stream);
    qx::launch_down(E->dev, w, (int)layer, E->stream);
    E->prof.kernel_launches += 3;
    if (!cuda_ok(cudaGetLastError(), "kernel launch", err, n)) return 0;
    if (!d2h(E, layer_output, E->dev.x, (size_t)E->dm.hidden * 4, err, n) ||
        !d2h(E, moe_output, E->dev.moe_out, (size_t)E->dm.hidden * 4, err, n) ||
        !d2h(E, selected, E->dev.sel + layer * 8, 32, err, n) || !d2h(E, weights, E->dev.selw + layer * 8, 32, err, n))
        return 0;
    return finish(E, err, n) ? 1 : 0;
}

// ---- batched MoE: N tokens through one MoE layer on the grouped tcgen05 GEMM ----
namespace {

bool batch_reserve(qx_cuda_engine* E, size_t ntok, char* err, uint64_t n) {
    auto& B = E->batch;
    if (B.cap >= ntok) return true;
    if (B.mem) { cudaFree(B.mem); B.mem = nullptr; B.cap = 0; }
    const size_t H = E->dm.hidden, I = E->dm.moe_inter, S = ntok * 8;
    const size_t Q = E->dm.q_dim(), KV = E->dm.kv_dim(), K = std::max(H, Q);
    const size_t V = E->dm.vocab;
    const size_t nhead = std::min<size_t>(ntok, QX_CUDA_MAX_SLOTS);   // tokens the batched head serves
    const size_t items = std::max(std::max((S / qx::kGemmItemCols + (size_t)E->dm.experts) * (I / 128 + H / 128),
                                           (ntok / 16 + 1) * std::max(Q / 128, H / 128)),
                                  (nhead / 16 + 1) * (V / 128));
    size_t off = 0;
    std::vector<std::pair<void**, size_t>> parts = {
        {(void**)&B.x, ntok * H * 4}, {(void**)&B.xn, ntok * H * 4}, {(void**)&B.out, ntok * H * 4},
        {(void**)&B.moe, ntok * H * 4}, {(void**)&B.gu, S * 2 * I * 4}, {(void**)&B.h, S * I * 4},
        {(void**)&B.y, S * H * 4}, {(void**)&B.bqx, ntok * (K / 256) * 2048}, {(void**)&B.bqh, S * (I / 256) * 2048},
        {(void**)&B.sx, ntok * (K / 256) * 4}, {(void**)&B.sh, S * (I / 256) * 4}, {(void**)&B.sel, S * 4},
        {(void**)&B.cols, S * 4}, {(void**)&B.wsel, S * 8}, {(void**)&B.items, items * sizeof(qx::GemmItem)},
        {(void**)&B.qkv, ntok * (Q + 2 * KV) * 4}, {(void**)&B.qn, ntok * Q * 4}, {(void**)&B.ctxo, ntok * Q * 4},
        {(void**)&B.ao, ntok * H * 4}, {(void**)&B.tcols, ntok * 4}, {(void**)&B.tok, ntok * 4},
        {(void**)&B.tpos, ntok * 4}, {(void**)&B.tslot, ntok * 4}, {(void**)&B.next, ntok * 4},
        {(void**)&B.logits, nhead * V * 8}, {(void**)&B.count, (size_t)E->dm.experts * 4}, {(void**)&B.nitems, 8}, {(void**)&B.vd, (size_t)E->dm.ctx * KV * 8}};
    for (auto& p : parts) off = align_up(off + p.second, 256);
    if (!cuda_ok(cudaMalloc(&B.mem, off), "cudaMalloc(batch)", err, n)) return false;
    off = 0;
    for (auto& p : parts) {
        *p.first = (uint8_t*)B.mem + off;
        off = align_up(off + p.second, 256);
    }
    B.cap = ntok;
    B.item_cap = items;
    return true;
}

}  // namespace

namespace {

bool batch_supported(const qx_cuda_engine* E, const LayerW& w, bool attention, char* err, uint64_t n) {
    const int H = E->dm.hidden, I = E->dm.moe_inter, EX = E->dm.experts;
    bool ok = w.gate_r && w.up_r && w.down_r && w.tgate == 17 && w.tup == 17 && w.tdown == 18 && H % 128 == 0 &&
              I % 128 == 0 && EX <= 256 && qx::batch_router_smem_bytes(H, EX) <= 200 * 1024;
    if (attention)
        ok = ok && w.wq_r && w.wk_r && w.wv_r && w.wo_r && w.tq == 23 && w.tk == 23 && w.tv == 23 && w.to == 23 &&
             E->dm.head_dim == 128 && E->dm.q_dim() <= 4096 && E->dm.kv_dim() <= 1024 && E->dm.q_dim() % 128 == 0 &&
             E->dm.kv_dim() % 128 == 0;
    if (!ok) set_err(err, n, "batched path needs the benchmark quant mix in the one-launch step kernel's layouts");
    return ok;
}

// GEMM arguments for an R4-laid IQ4_XS matrix of `rows` x K (one "expert"),
// columns = tokens 0..N-1 (ids in B.tcols), B rows = tokens.
qx::GemmArgs proj_args(qx_cuda_engine* E, const uint8_t* weights, int K, float* out, size_t out_stride, int out_off) {
    auto& B = E->batch;
    const size_t rb = qx::r4_bytes_per_row(K);
    qx::GemmArgs a{};
    a.items = B.items;
    a.cols = B.tcols;
    a.weights = weights;
    a.expert_stride = 0;
    a.row_bytes = (uint32_t)rb;
    a.hdr = (2 * (K / 256) + 15) / 16 * 16;
    a.codes = (a.hdr + 8 * (K / 256) + 15) / 16 * 16;
    a.nblk = K / 256;
    a.fmt = qx::kGemmR4Iq4;
    a.fexp = 0;
    a.bq = B.bqx;
    a.sexp = B.sx;
    a.b_by_token = 0;
    a.out = out;
    a.out_stride = out_stride;
    a.out_off = out_off;
    a.err = E->dev.err;
    return a;
}

// Work items of a projection over N tokens: column tiles x 128-row tiles.  A
// prompt-sized batch takes two 16-token tiles per item (one weight decode for
// both); a small one keeps one tile per item, for twice the CTAs.
bool proj_items(qx_cuda_engine* E, int N, int rows, int* count, char* err, uint64_t n) {
    std::vector<qx::GemmItem> items;
    const int w = N >= 512 ? qx::kGemmItemCols : 16;
    for (int c0 = 0; c0 < N; c0 += w)
        for (int r0 = 0; r0 < rows; r0 += 128) items.push_back({0, c0, std::min(w, N - c0), r0});
    if (items.size() > E->batch.item_cap) { set_err(err, n, "batched work list too long"); return false; }
    *count = (int)items.size();
    return h2d(E, E->batch.items, items.data(), items.size() * sizeof(qx::GemmItem), err, n);
}

// One MoE layer for the N residuals in B.x: B.out = B.x + moe (B.moe), the
// selections in B.sel / B.wsel.  Leaves the stream running.
bool moe_batch_run(qx_cuda_engine* E, uint32_t layer, int N, char* err, uint64_t n) {
    auto& B = E->batch;
    const LayerW& w = E->layers[layer];
    const int H = E->dm.hidden, I = E->dm.moe_inter, EX = E->dm.experts, S = N * 8;
    // norm, activation limbs, router + top-8 (every token)
    qx::launch_batch_norm(B.x, w.ffn_norm, B.xn, H, N, E->stream);
    qx::launch_batch_limbs(B.xn, H, N, B.bqx, B.sx, E->stream);
    qx::launch_batch_router(B.xn, w.router, H, EX, N, B.sel, B.wsel, E->dev.err, E->stream);
    E->prof.kernel_launches += 3;
    // the slots (token, rank) of every expert in token order and both GEMMs'
    // work items, built on the device (no host round trip)
    const size_t max_ct = (size_t)S / qx::kGemmItemCols + (size_t)EX;   // bounds sum_e ceil(count_e / 32)
    const int max_gu = (int)(max_ct * (size_t)(I / 128)), max_dn = (int)(max_ct * (size_t)(H / 128));
    if ((size_t)max_gu + (size_t)max_dn > B.item_cap) { set_err(err, n, "batched expert work list too long"); return false; }
    qx::launch_slot_lists(B.sel, S, EX, B.count, B.cols, B.items, I, B.items + max_gu, H, B.nitems, E->stream);
    const size_t rb2 = qx::iq2r_row_bytes(H);
    qx::GemmArgs ga{};
    ga.items = B.items;
    ga.nitems = B.nitems;
    ga.cols = B.cols;
    ga.expert_stride = (size_t)I * rb2;
    ga.row_bytes = (uint32_t)rb2;
    ga.hdr = (int)(rb2 - (size_t)(H / 256) * 144);
    ga.nblk = H / 256;
    ga.fmt = qx::kGemmIq2r;
    ga.fexp = -3;
    ga.bq = B.bqx;
    ga.sexp = B.sx;
    ga.b_by_token = 1;
    ga.out = B.gu;
    ga.out_stride = (size_t)2 * I;
    ga.err = E->dev.err;
    ga.weights = w.gate_r;
    ga.out_off = 0;
    qx::launch_moe_gemm(ga, max_gu, E->stream);
    ga.weights = w.up_r;
    ga.out_off = I;
    qx::launch_moe_gemm(ga, max_gu, E->stream);
    // SwiGLU, then the down input's limbs per slot
    qx::launch_batch_swiglu(B.gu, I, S, B.h, E->stream);
    qx::launch_batch_limbs(B.h, I, S, B.bqh, B.sh, E->stream);
    // down: rows of H values of K = I, columns = slots, B = the slot's limbs
    const size_t rb4 = qx::r4_bytes_per_row(I);
    qx::GemmArgs gd = ga;
    gd.items = B.items + max_gu;
    gd.nitems = B.nitems + 1;
    gd.weights = w.down_r;
    gd.expert_stride = (size_t)H * rb4;
    gd.row_bytes = (uint32_t)rb4;
    gd.hdr = (2 * (I / 256) + 15) / 16 * 16;
    gd.codes = (gd.hdr + 8 * (I / 256) + 15) / 16 * 16;
    gd.nblk = I / 256;
    gd.fmt = qx::kGemmR4Iq3;
    gd.fexp = -2;
    gd.bq = B.bqh;
    gd.sexp = B.sh;
    gd.b_by_token = 0;
    gd.out = B.y;
    gd.out_stride = (size_t)H;
    gd.out_off = 0;
    qx::launch_moe_gemm(gd, max_dn, E->stream);
    qx::launch_batch_combine(B.x, B.y, B.wsel, H, N, B.moe, B.out, E->stream);
    E->prof.kernel_launches += 8;   // slot count + lists, gate, up, SwiGLU, limbs, down, combine
    return cuda_ok(cudaGetLastError(), "kernel launch", err, n);
}

}  // namespace

QX_API int qx_cuda_moe_batch(qx_cuda_engine* E, uint32_t layer, uint32_t ntok, const float* x, float* layer_output,
                             float* moe_output, uint32_t* selected, float* weights, char* err, uint64_t n) {
    if (!E || !x || !layer_output || layer >= (uint32_t)E->dm.layers || ntok == 0 || ntok > QX_CUDA_MAX_BATCH) {
        set_err(err, n, "invalid batched expert argument");
        return 0;
    }
    if (!batch_supported(E, E->layers[layer], false, err, n)) return 0;
    DeviceGuard g(E->device);
    if (!batch_reserve(E, ntok, err, n)) return 0;
    auto& B = E->batch;
    const int N = (int)ntok, S = N * 8, H = E->dm.hidden;
    if (!h2d(E, B.x, x, (size_t)N * H * 4, err, n)) return 0;
    if (!moe_batch_run(E, layer, N, err, n)) return 0;
    if (!d2h(E, layer_output, B.out, (size_t)N * H * 4, err, n) ||
        !d2h(E, moe_output, B.moe, (size_t)N * H * 4, err, n) ||
        !d2h(E, selected, B.sel, (size_t)S * 4, err, n))
        return 0;
    if (weights) {
        std::vector<double> wd(S);
        if (!d2h(E, wd.data(), B.wsel, (size_t)S * 8, err, n) || !finish(E, err, n)) return 0;
        for (int s = 0; s < S; ++s) weights[s] = (float)wd[s];
        return 1;
    }
    return finish(E, err, n) ? 1 : 0;
}

namespace {

// The attention half of one layer for the N tokens in B.x (positions B.tpos,
// KV slots B.tslot of `kv`): attention RMSNorm, Q/K/V on the tensor cores,
// head norms + RoPE + the K/V rows into the cache, causal attention, O
// projection, residual add.  Leaves the stream running.
bool attn_batch_run(qx_cuda_engine* E, int layer, int N, const qx::KvView& kv, int max_pos, int first_pos, char* err,
                    uint64_t n) {
    auto& B = E->batch;
    const LayerW& w = E->layers[layer];
    const int H = E->dm.hidden, Q = E->dm.q_dim(), KV = E->dm.kv_dim(), QH = E->dm.q_heads, KVH = E->dm.kv_heads;
    int cnt = 0;
    qx::launch_batch_norm(B.x, w.attn_norm, B.xn, H, N, E->stream);
    qx::launch_batch_limbs(B.xn, H, N, B.bqx, B.sx, E->stream);
    if (!proj_items(E, N, Q, &cnt, err, n)) return false;
    qx::launch_moe_gemm(proj_args(E, w.wq_r, H, B.qkv, (size_t)(Q + 2 * KV), 0), cnt, E->stream);
    if (!proj_items(E, N, KV, &cnt, err, n)) return false;
    qx::launch_moe_gemm(proj_args(E, w.wk_r, H, B.qkv, (size_t)(Q + 2 * KV), Q), cnt, E->stream);
    qx::launch_moe_gemm(proj_args(E, w.wv_r, H, B.qkv, (size_t)(Q + 2 * KV), Q + KV), cnt, E->stream);
    qx::launch_batch_qkv_post(B.qkv, w.q_norm, w.k_norm, E->dev.rope, layer, B.tpos, B.tslot, kv, N, QH, KVH, B.qn,
                              E->stream);
    qx::launch_batch_attn(B.qn, kv, layer, B.tpos, B.tslot, max_pos, N, QH, KVH, B.ctxo, E->stream, first_pos, B.vd);
    qx::launch_batch_limbs(B.ctxo, Q, N, B.bqx, B.sx, E->stream);
    if (!proj_items(E, N, H, &cnt, err, n)) return false;
    qx::launch_moe_gemm(proj_args(E, w.wo_r, Q, B.ao, (size_t)H, 0), cnt, E->stream);
    qx::launch_batch_add(B.x, B.ao, (size_t)N * H, E->stream);
    E->prof.kernel_launches += 10;
    return cuda_ok(cudaGetLastError(), "kernel launch", err, n);
}

}  // namespace

QX_API int qx_cuda_prefill(qx_cuda_engine* E, const uint32_t* tokens, uint32_t ntok, uint32_t position,
                           uint32_t* next_token, float* final_residual, char* err, uint64_t n) {
    if (!E || !tokens || !next_token || ntok == 0 || ntok > QX_CUDA_MAX_BATCH) {
        set_err(err, n, "invalid prefill argument");
        return 0;
    }
    if ((uint64_t)position + ntok > (uint64_t)E->dm.ctx) { set_err(err, n, "steps exceed ctx"); return 0; }
    for (uint32_t t = 0; t < ntok; ++t)
        if (tokens[t] >= (uint32_t)E->dm.vocab) { set_err(err, n, "prompt token out of range"); return 0; }
    for (const auto& w : E->layers)
        if (!batch_supported(E, w, true, err, n)) return 0;
    DeviceGuard g(E->device);
    if (!batch_reserve(E, ntok, err, n)) return 0;
    auto& B = E->batch;
    const int N = (int)ntok, H = E->dm.hidden, C = E->dm.ctx;
    Dev& d = E->dev;
    {
        std::vector<int> ids(N);
        for (int t = 0; t < N; ++t) ids[t] = t;
        if (!h2d(E, B.tcols, ids.data(), (size_t)N * 4, err, n) || !h2d(E, B.tok, tokens, (size_t)N * 4, err, n))
            return 0;
    }
    {
        std::vector<int> pos(N), zero(N, 0);
        for (int t = 0; t < N; ++t) pos[t] = (int)position + t;
        if (!h2d(E, B.tpos, pos.data(), (size_t)N * 4, err, n) || !h2d(E, B.tslot, zero.data(), (size_t)N * 4, err, n))
            return 0;
    }
    const qx::KvView kv{d.kcache, d.vcache, d.kscale, d.vscale, 0, C};
    qx::launch_batch_embed(B.tok, d.tok_embd, H, E->dm.vocab, N, B.x, d.err, E->stream);
    E->prof.kernel_launches++;
    for (int layer = 0; layer < E->dm.layers; ++layer) {
        if (!attn_batch_run(E, layer, N, kv, (int)position + N - 1, (int)position, err, n)) return 0;
        // the MoE FFN, then its output is the next layer's residual
        if (!moe_batch_run(E, (uint32_t)layer, N, err, n)) return 0;
        std::swap(B.x, B.out);
    }
    // the head for the last prompt token only (the reference skips it for the
    // others, src/qx_format.c:6533-6547): greedy next token at position p0 + N - 1
    E->h_io[1] = (int)(position + ntok - 1);
    if (!cuda_ok(cudaMemcpyAsync(d.x, B.x + (size_t)(N - 1) * H, (size_t)H * 4, cudaMemcpyDeviceToDevice, E->stream),
                 "d2d", err, n) ||
        !cuda_ok(cudaMemcpyAsync(d.pos, E->h_io + 1, 4, cudaMemcpyHostToDevice, E->stream), "h2d", err, n))
        return 0;
    Dev dh = d;
    dh.logits_d = nullptr;
    qx::launch_head(dh, E->stream);
    E->prof.kernel_launches++;
    if (!cuda_ok(cudaGetLastError(), "kernel launch", err, n)) return 0;
    if (!d2h(E, E->h_io + 2, d.token, 4, err, n) || !d2h(E, final_residual, d.x, (size_t)H * 4, err, n)) return 0;
    if (!finish(E, err, n)) return 0;
    *next_token = (uint32_t)E->h_io[2];
    E->prof.decode_steps += ntok;
    return 1;
}

QX_API int qx_cuda_decode_batch(qx_cuda_engine* E, uint32_t nseq, const uint32_t* slots, const uint32_t* tokens,
                                const uint32_t* positions, uint32_t* next_tokens, char* err, uint64_t n) {
    if (!E || !slots || !tokens || !positions || !next_tokens || nseq == 0 || nseq > QX_CUDA_MAX_SLOTS) {
        set_err(err, n, "invalid batched decode argument");
        return 0;
    }
    int max_pos = 0;
    for (uint32_t i = 0; i < nseq; ++i) {
        if (slots[i] >= QX_CUDA_MAX_SLOTS) { set_err(err, n, "invalid batched decode argument"); return 0; }
        for (uint32_t j = 0; j < i; ++j)
            if (slots[j] == slots[i]) { set_err(err, n, "a sequence slot appears twice in one batch"); return 0; }
        if (tokens[i] >= (uint32_t)E->dm.vocab) { set_err(err, n, "prompt token out of range"); return 0; }
        if (positions[i] >= (uint32_t)E->dm.ctx) { set_err(err, n, "steps exceed ctx"); return 0; }
        max_pos = std::max(max_pos, (int)positions[i]);
    }
    for (const auto& w : E->layers)
        if (!batch_supported(E, w, true, err, n)) return 0;
    if (!E->dev.head_r || E->dm.vocab % 128) { set_err(err, n, "batched decode needs the re-laid head"); return 0; }
    DeviceGuard g(E->device);
    if (!batch_reserve(E, std::max<uint32_t>(nseq, 16), err, n)) return 0;
    auto& B = E->batch;
    const size_t L = E->dm.layers, C = E->dm.ctx, KV = E->dm.kv_dim(), rows = L * C;
    if (!B.slot_mem) {                    // every slot's KV, zeroed once (positions beyond a slot's are not read)
        const size_t bytes = (size_t)QX_CUDA_MAX_SLOTS * rows * (2 * KV + 8);
        if (!cuda_ok(cudaMalloc(&B.slot_mem, bytes), "cudaMalloc(sequence slots)", err, n)) return 0;
        if (!cuda_ok(cudaMemsetAsync(B.slot_mem, 0, bytes, E->stream), "memset", err, n)) return 0;
        int8_t* p = (int8_t*)B.slot_mem;
        B.slots.k = p;
        B.slots.v = p + (size_t)QX_CUDA_MAX_SLOTS * rows * KV;
        B.slots.ks = (float*)(p + (size_t)QX_CUDA_MAX_SLOTS * rows * 2 * KV);
        B.slots.vs = B.slots.ks + (size_t)QX_CUDA_MAX_SLOTS * rows;
        B.slots.slot_rows = rows;
        B.slots.ctx = (int)C;
    }
    const int N = (int)nseq, H = E->dm.hidden, V = E->dm.vocab;
    Dev& d = E->dev;
    {
        std::vector<int> ids(N), pos(N), sl(N);
        for (int t = 0; t < N; ++t) ids[t] = t, pos[t] = (int)positions[t], sl[t] = (int)slots[t];
        if (!h2d(E, B.tcols, ids.data(), (size_t)N * 4, err, n) || !h2d(E, B.tok, tokens, (size_t)N * 4, err, n) ||
            !h2d(E, B.tpos, pos.data(), (size_t)N * 4, err, n) || !h2d(E, B.tslot, sl.data(), (size_t)N * 4, err, n))
            return 0;
    }
    qx::launch_batch_embed(B.tok, d.tok_embd, H, V, N, B.x, d.err, E->stream);
    E->prof.kernel_launches++;
    for (int layer = 0; layer < E->dm.layers; ++layer) {
        if (!attn_batch_run(E, layer, N, B.slots, max_pos, -1, err, n)) return 0;
        if (!moe_batch_run(E, (uint32_t)layer, N, err, n)) return 0;
        std::swap(B.x, B.out);
    }
    // the head of every sequence: final RMSNorm, Q6_K rows on the tensor cores
    // (double logits), greedy pick
    int cnt = 0;
    qx::launch_batch_norm(B.x, d.out_norm, B.xn, H, N, E->stream);
    qx::launch_batch_limbs(B.xn, H, N, B.bqx, B.sx, E->stream);
    if (!proj_items(E, N, V, &cnt, err, n)) return 0;
    qx::GemmArgs ha = proj_args(E, d.head_r, H, nullptr, (size_t)V, 0);
    ha.row_bytes = (uint32_t)qx::r8_bytes_per_row(H);
    ha.hdr = (2 * (H / 256) + 15) / 16 * 16;
    ha.fmt = qx::kGemmR8;
    ha.out_d = B.logits;
    qx::launch_moe_gemm(ha, cnt, E->stream);
    qx::launch_batch_argmax(B.logits, V, N, B.next, d.err, E->stream);
    E->prof.kernel_launches += 4;
    if (!cuda_ok(cudaGetLastError(), "kernel launch", err, n)) return 0;
    if (!d2h(E, next_tokens, B.next, (size_t)N * 4, err, n) || !finish(E, err, n)) return 0;
    E->prof.decode_steps += nseq;
    return 1;
}

QX_API int qx_cuda_attention_layer(qx_cuda_engine* E, uint32_t layer, uint32_t position, float* residual,
                                   float* attn_out, float* context, char* err, uint64_t n) {
    if (!E || !residual || layer >= (uint32_t)E->dm.layers) { set_err(err, n, "invalid argument"); return 0; }
    if (position >= (uint32_t)E->dm.ctx) { set_err(err, n, "steps exceed ctx"); return 0; }
    DeviceGuard g(E->device);
    const LayerW& w = E->layers[layer];
    if (!h2d(E, E->dev.x, residual, (size_t)E->dm.hidden * 4, err, n)) return 0;
    E->h_io[1] = (int)position;
    if (!cuda_ok(cudaMemcpyAsync(E->dev.pos, E->h_io + 1, 4, cudaMemcpyHostToDevice, E->stream), "h2d", err, n)) return 0;
    qx::launch_qkv(E->dev, w, E->stream);
    qx::launch_attn(E->dev, w, (int)layer, E->stream);
    qx::launch_oproj(E->dev, w, E->stream);
    E->prof.kernel_launches += 1 + qx::qkv_launches(E->dev, w) + qx::attn_launches(E->dm);
    if (!cuda_ok(cudaGetLastError(), "kernel launch", err, n)) return 0;
    if (!d2h(E, residual, E->dev.x, (size_t)E->dm.hidden * 4, err, n) ||
        !d2h(E, attn_out, E->dev.attn_out, (size_t)E->dm.hidden * 4, err, n) ||
        !d2h(E, context, E->dev.ctxv, (size_t)E->dm.q_dim() * 4, err, n))
        return 0;
    return finish(E, err, n) ? 1 : 0;
}

QX_API int qx_cuda_embed(qx_cuda_engine* E, uint32_t token, float* out, char* err, uint64_t n) {
    if (!E || !out) { set_err(err, n, "invalid residual vector argument"); return 0; }
    if (token >= (uint32_t)E->dm.vocab) { set_err(err, n, "token id out of range"); return 0; }
    DeviceGuard g(E->device);
    if (!set_scalars(E, token, 0, err, n)) return 0;
    qx::launch_embed(E->dev, E->stream);
    E->prof.kernel_launches++;
    if (!cuda_ok(cudaGetLastError(), "kernel launch", err, n)) return 0;
    if (!d2h(E, out, E->dev.x, (size_t)E->dm.hidden * 4, err, n)) return 0;
    return finish(E, err, n) ? 1 : 0;
}

QX_API int qx_cuda_kv_write(qx_cuda_engine* E, uint32_t layer, uint32_t first, uint32_t count, const int8_t* k,
                            const int8_t* v, const float* ks, const float* vs, char* err, uint64_t n) {
    if (!E || !k || !v || !ks || !vs || layer >= (uint32_t)E->dm.layers || (uint64_t)first + count > (uint64_t)E->dm.ctx) {
        set_err(err, n, "invalid KV range"); return 0;
    }
    DeviceGuard g(E->device);
    const size_t KV = E->dm.kv_dim(), base = (size_t)layer * E->dm.ctx + first;
    bool ok = h2d(E, E->dev.kcache + base * KV, k, count * KV, err, n) &&
              h2d(E, E->dev.vcache + base * KV, v, count * KV, err, n) &&
              h2d(E, E->dev.kscale + base, ks, count * 4, err, n) && h2d(E, E->dev.vscale + base, vs, count * 4, err, n);
    const cudaError_t ce = ok ? cudaStreamSynchronize(E->stream) : cudaSuccess;
    E->h_stage_used = 0;                  // the staged inputs have been consumed (or the call failed)
    if (!ok) return 0;
    return cuda_ok(ce, "kv write", err, n) ? 1 : 0;
}

QX_API int qx_cuda_kv_read(qx_cuda_engine* E, uint32_t layer, uint32_t first, uint32_t count, int8_t* k, int8_t* v,
                           float* ks, float* vs, char* err, uint64_t n) {
    if (!E || layer >= (uint32_t)E->dm.layers || (uint64_t)first + count > (uint64_t)E->dm.ctx) {
        set_err(err, n, "invalid KV range"); return 0;
    }
    DeviceGuard g(E->device);
    const size_t KV = E->dm.kv_dim(), base = (size_t)layer * E->dm.ctx + first;
    bool ok = d2h(E, k, E->dev.kcache + base * KV, count * KV, err, n) &&
              d2h(E, v, E->dev.vcache + base * KV, count * KV, err, n) &&
              d2h(E, ks, E->dev.kscale + base, count * 4, err, n) && d2h(E, vs, E->dev.vscale + base, count * 4, err, n);
    if (!ok) return 0;
    // wait, then move the staged copies into the caller's buffers
    const cudaError_t ce = cudaStreamSynchronize(E->stream);
    for (const auto& p : E->pending)
        if (ce == cudaSuccess) memcpy(p.dst, E->h_stage + p.off, p.bytes);
    E->pending.clear();
    E->h_stage_used = 0;
    return cuda_ok(ce, "kv read", err, n) ? 1 : 0;
}

QX_API int qx_cuda_profile_get(const qx_cuda_engine* E, qx_cuda_profile* out) {
    if (!E || !out) return 0;
    *out = E->prof;
    return 1;
}

QX_API void* qx_cuda_stream(const qx_cuda_engine* E) { return E ? (void*)E->stream : nullptr; }

QX_API int qx_cuda_time_kernels(qx_cuda_engine* E, uint32_t token, uint32_t position, uint32_t steps, char* names,
                                uint64_t names_len, float* ms_avg, uint32_t* launches, uint32_t max_kernels,
                                uint32_t* kernel_count, char* err, uint64_t n) {
    if (!E || !steps || (uint64_t)position + steps > (uint64_t)E->dm.ctx) { set_err(err, n, "invalid argument"); return 0; }
    DeviceGuard g(E->device);
    if (!ep_ready(E, err, n) || !set_scalars(E, token, position, err, n)) return 0;
    const size_t nops = E->ops.size();
    std::vector<cudaEvent_t> ev(nops * steps + 1);
    for (auto& e : ev) cudaEventCreate(&e);
    size_t k = 0;
    cudaEventRecord(ev[k++], E->stream);
    for (uint32_t s = 0; s < steps; ++s)
        for (const Op& op : E->ops) {
            run_op(E, op);
            cudaEventRecord(ev[k++], E->stream);
        }
    bool ok = cuda_ok(cudaGetLastError(), "kernel launch", err, n) && finish(E, err, n);
    std::vector<std::string> order;
    std::map<std::string, std::pair<double, uint32_t>> acc;
    if (ok) {
        k = 0;
        for (uint32_t s = 0; s < steps; ++s)
            for (const Op& op : E->ops) {
                float ms = 0.f;
                cudaEventElapsedTime(&ms, ev[k], ev[k + 1]);
                ++k;
                if (!acc.count(op.name)) order.push_back(op.name);
                acc[op.name].first += ms;
                acc[op.name].second += 1;
            }
    }
    for (auto& e : ev) cudaEventDestroy(e);
    if (!ok) return 0;
    std::string joined;
    uint32_t c = 0;
    for (const auto& nm : order) {
        if (c < max_kernels) {
            ms_avg[c] = (float)(acc[nm].first / acc[nm].second);
            launches[c] = acc[nm].second;
        }
        joined += (c ? ";" : "") + nm;
        ++c;
    }
    if (kernel_count) *kernel_count = c;
    if (names && names_len) snprintf(names, (size_t)names_len, "%s", joined.c_str());
    E->prof.kernel_launches += (E->mega_grid ? nops : stage_launches(E)) * steps;
    return 1;
}

QX_API int qx_cuda_phase_trace(qx_cuda_engine* E, uint32_t token, uint32_t position, uint64_t* stamps_ns,
                               uint32_t max_stamps, uint32_t* count, char* err, uint64_t n) {
    if (!E || !stamps_ns || !count || !max_stamps) { set_err(err, n, "invalid argument"); return 0; }
    if (!E->mega_grid) { set_err(err, n, "phase trace needs the persistent step kernel"); return 0; }
    if (position >= (uint32_t)E->dm.ctx || token >= (uint32_t)E->dm.vocab) { set_err(err, n, "invalid argument"); return 0; }
    DeviceGuard g(E->device);
    const uint32_t nst = 2u + (uint32_t)qx::kPhasesPerLayer * (uint32_t)E->dm.layers + 1u;
    const uint32_t total = nst * (9u + (uint32_t)E->mega_grid);
    unsigned long long* tr = nullptr;
    if (!cuda_ok(cudaMalloc((void**)&tr, (size_t)total * 8), "cudaMalloc(trace)", err, n)) return 0;
    cudaMemsetAsync(tr, 0, (size_t)total * 8, E->stream);
    bool ok = ep_ready(E, err, n) && set_scalars(E, token, position, err, n);
    if (ok) {
        Dev d = E->dev;
        d.trace = tr;
        ok = cuda_ok(qx::launch_decode_step(d, E->layers_dev, E->mega_grid, E->stream), "launch", err, n) && finish(E, err, n);
    }
    const uint32_t c = total < max_stamps ? total : max_stamps;
    if (ok) ok = cuda_ok(cudaMemcpy(stamps_ns, tr, c * 8, cudaMemcpyDeviceToHost), "trace d2h", err, n);
    cudaFree(tr);
    if (ok) *count = c;
    return ok ? 1 : 0;
}

// ---- expert parallelism: the split and the mapping of the peers' buffers ----

QX_API int qx_cuda_ep_partition(uint32_t experts, uint32_t vocab, uint32_t world, uint32_t rank, uint32_t out[4]) {
    if (!out || world < 1 || rank >= world || vocab % 32) return 0;
    const uint32_t groups = vocab / 32;                      // head rows go in groups of 32 (two 16-row tiles)
    out[0] = (uint32_t)((uint64_t)rank * experts / world);
    out[1] = (uint32_t)((uint64_t)(rank + 1) * experts / world);
    out[2] = (uint32_t)((uint64_t)rank * groups / world) * 32u;
    out[3] = (uint32_t)((uint64_t)(rank + 1) * groups / world) * 32u;
    return 1;
}

QX_API int qx_cuda_ep_handle(qx_cuda_engine* E, void* handle, uint64_t handle_size, char* err, uint64_t n) {
    if (!E || !handle || handle_size < sizeof(cudaIpcMemHandle_t)) { set_err(err, n, "invalid argument"); return 0; }
    if (E->dev.ep_world <= 1) { set_err(err, n, "engine is not expert-parallel"); return 0; }
    DeviceGuard g(E->device);
    cudaIpcMemHandle_t h;
    if (!cuda_ok(cudaIpcGetMemHandle(&h, E->ep_xchg), "cudaIpcGetMemHandle", err, n)) return 0;
    memset(handle, 0, (size_t)handle_size);
    memcpy(handle, &h, sizeof(h));
    return 1;
}

QX_API int qx_cuda_ep_connect(qx_cuda_engine* E, const void* handles, uint64_t handle_size, uint32_t world, char* err,
                              uint64_t n) {
    if (!E || !handles || handle_size < sizeof(cudaIpcMemHandle_t)) { set_err(err, n, "invalid argument"); return 0; }
    if (E->dev.ep_world <= 1 || (int)world != E->dev.ep_world) {
        set_err(err, n, "peer count does not match the engine's expert-parallel world size");
        return 0;
    }
    if (E->ep_connected) { set_err(err, n, "expert-parallel engine is already connected"); return 0; }
    DeviceGuard g(E->device);
    uint8_t* ptrs[qx::kEpMaxRanks] = {};
    for (uint32_t p = 0; p < world; ++p) {
        if ((int)p == E->dev.ep_rank) { ptrs[p] = E->ep_xchg; continue; }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)p * handle_size, sizeof(h));
        void* mapped = nullptr;
        if (!cuda_ok(cudaIpcOpenMemHandle(&mapped, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle", err, n))
            return 0;
        E->ep_opened.push_back(mapped);
        ptrs[p] = static_cast<uint8_t*>(mapped);
    }
    if (!cuda_ok(cudaMemcpy(E->ep_peers_dev, ptrs, sizeof(ptrs), cudaMemcpyHostToDevice), "peer table", err, n))
        return 0;
    E->ep_connected = true;
    return 1;
}

// ---- QXKVSNP1 snapshot of the persistent INT8 KV ----------------------------

QX_API int qx_cuda_kv_export(qx_cuda_engine* E, const char* path, uint32_t positions, uint32_t next_token,
                             uint32_t seed, char* err, uint64_t n) {
    if (!E || !path || positions == 0 || positions > (uint32_t)E->dm.ctx) {
        set_err(err, n, "invalid accumulated KV snapshot output");
        return 0;
    }
    DeviceGuard g(E->device);
    const size_t L = E->dm.layers, C = E->dm.ctx, KV = E->dm.kv_dim();
    std::vector<int8_t> k(L * C * KV), v(L * C * KV);
    std::vector<float> ks(L * C), vs(L * C);
    cudaError_t ce = cudaStreamSynchronize(E->stream);
    if (ce == cudaSuccess) ce = cudaMemcpy(k.data(), E->dev.kcache, k.size(), cudaMemcpyDeviceToHost);
    if (ce == cudaSuccess) ce = cudaMemcpy(v.data(), E->dev.vcache, v.size(), cudaMemcpyDeviceToHost);
    if (ce == cudaSuccess) ce = cudaMemcpy(ks.data(), E->dev.kscale, ks.size() * 4, cudaMemcpyDeviceToHost);
    if (ce == cudaSuccess) ce = cudaMemcpy(vs.data(), E->dev.vscale, vs.size() * 4, cudaMemcpyDeviceToHost);
    if (!cuda_ok(ce, "KV snapshot d2h", err, n)) return 0;
    E->prof.device_to_host_bytes += 2 * (k.size() + ks.size() * 4);
    return qxh_kv_snapshot_write(path, (uint32_t)L, positions, (uint32_t)C, (uint32_t)E->dm.kv_heads,
                                 (uint32_t)E->dm.head_dim, next_token, seed, k.data(), v.data(), ks.data(), vs.data(),
                                 err, n);
}

QX_API int qx_cuda_kv_import(qx_cuda_engine* E, const char* path, uint32_t seed, uint32_t* positions,
                             uint32_t* next_token, char* err, uint64_t n) {
    if (!E || !path || !positions || !next_token) { set_err(err, n, "invalid argument"); return 0; }
    DeviceGuard g(E->device);
    const size_t L = E->dm.layers, C = E->dm.ctx, KV = E->dm.kv_dim();
    std::vector<int8_t> k(L * C * KV, 0), v(L * C * KV, 0);
    std::vector<float> ks(L * C, 0.f), vs(L * C, 0.f);
    uint32_t pos = 0, nt = 0;
    if (!qxh_kv_snapshot_read(path, (uint32_t)L, (uint32_t)C, (uint32_t)E->dm.kv_heads, (uint32_t)E->dm.head_dim, seed,
                              k.data(), v.data(), ks.data(), vs.data(), &pos, &nt, err, n))
        return 0;                         // the device KV is untouched on failure
    cudaError_t ce = cudaStreamSynchronize(E->stream);
    if (ce == cudaSuccess) ce = cudaMemcpy(E->dev.kcache, k.data(), k.size(), cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMemcpy(E->dev.vcache, v.data(), v.size(), cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMemcpy(E->dev.kscale, ks.data(), ks.size() * 4, cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMemcpy(E->dev.vscale, vs.data(), vs.size() * 4, cudaMemcpyHostToDevice);
    if (!cuda_ok(ce, "KV snapshot h2d", err, n)) return 0;
    E->prof.host_to_device_bytes += 2 * (k.size() + ks.size() * 4);
    *positions = pos;
    *next_token = nt;
    return 1;
}
