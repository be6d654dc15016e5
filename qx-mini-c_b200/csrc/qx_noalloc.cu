// Final RMSNorm + Q6_K head + argmax for callers that cannot allocate device
// memory: a plugin running inside a host that owns every allocation (its own
// pool or arena, a sandbox without cudaMalloc rights), or code that must not
// allocate between stream-ordered steps.  The caller supplies every input and
// output buffer; the per-CTA argmax partials and the completion counter that
// the engine's head kernel keeps in engine-allocated scratch live here in a
// file-scope __device__ array instead.
//
// Limits: at most kNoAllocMaxCtas CTAs (the grid is clamped to it), hidden a
// multiple of 256 up to 2048, vocab a multiple of 32.  The array is shared by
// every call on a device and keeps the last call's contents; calls that
// overlap on the GPU (different streams, no ordering) race on it.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdio>
#include <mutex>

#include "qx_cuda.h"
#include "qx_imma.cuh"

namespace {

constexpr int kNoAllocMaxCtas = 1024;
constexpr int kTiles = 2;      // tiles per pipeline stage
constexpr int kStages = 3;
constexpr int kMaxDevices = 64;

struct HeadScratch {
    double best_val[kNoAllocMaxCtas];
    int best_idx[kNoAllocMaxCtas];
    unsigned counter;          // must be 0 when a call starts; cleared by every call
};

// Every GPU that loads the library holds this array until the process exits.
static __device__ __align__(256) HeadScratch g_head_scratch;

HeadScratch* g_scratch_ptr[kMaxDevices];
bool g_ready[kMaxDevices];
std::mutex g_mutex;

using namespace qx;

__device__ __forceinline__ uint8_t* align16(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 15u) & ~(uintptr_t)15u);
}

__global__ void __launch_bounds__(kThreads) k_head_noalloc(const float* x, const float* nw, const uint8_t* head,
                                                            int H, int V, float* logits, uint32_t* argmax,
                                                            HeadScratch* scr) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ double scratch[kWarps];
    __shared__ double wbv[kWarps];
    __shared__ int wbi[kWarps];
    __shared__ bool is_last;
    const int nblk = H / 256;
    const uint32_t rb = (uint32_t)nblk * 210u, tb = (uint32_t)kTileRows * rb, stage = kTiles * tb;
    uint8_t* ring = align16(smem);
    float* xs = reinterpret_cast<float*>(align16(ring + (size_t)kStages * stage));
    uint32_t* xb = reinterpret_cast<uint32_t*>(align16(reinterpret_cast<uint8_t*>(xs + H)));
    int* sb = reinterpret_cast<int*>(align16(reinterpret_cast<uint8_t*>(xb + xq_words(H))));
    double* part = reinterpret_cast<double*>(align16(reinterpret_cast<uint8_t*>(sb + H / 256)));
    const int ngroups = V / (kTileRows * kTiles);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
    const int parts = kWarps / kTiles, tile = warp / parts, p = warp % parts;
    const int first = blockIdx.x, step = gridDim.x;
    const int mine = first < ngroups ? (ngroups - first + step - 1) / step : 0;
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < mine) stage_copy(ring + (uint32_t)s * stage, head + (size_t)(first + s * step) * stage, stage);
        cp_async_commit();
    }
    // RMSNorm in double (qx_apply_f32_rmsnorm, src/qx_format.c:3358-3371)
    for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    const double ss = sum_sq_fixed(xs, H, scratch);
    const double rms = sqrt(ss / (double)H + 1.0e-6);
    for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = (float)((double)xs[i] / rms) * nw[i];
    __syncthreads();
    build_xq(xs, H, xb, sb);
    __syncthreads();
    double bv = -1.0e300;
    int bi = 0x7fffffff;
    bool bad = false;
    for (int it = 0; it < mine; ++it) {
        const int nx = it + kStages - 1;
        if (nx < mine)
            stage_copy(ring + (uint32_t)(nx % kStages) * stage, head + (size_t)(first + nx * step) * stage, stage);
        cp_async_commit();
        cp_async_wait<kStages - 1>();
        __syncthreads();
        const uint8_t* base = ring + (uint32_t)(it % kStages) * stage + tile * tb;
        Acc acc{};
        dot_q6_k_mma(base + g * rb, base + (g + 8) * rb, p * nblk / parts, (p + 1) * nblk / parts, XQ{xb, sb}, lane,
                     acc);
        double lo, hi;
        acc.finish(lo, hi);
        if ((lane & 3) == 0) {
            part[warp * kTileRows + g] = lo;
            part[warp * kTileRows + g + 8] = hi;
        }
        __syncthreads();
        if (threadIdx.x < kTiles * kTileRows) {
            const int tl = threadIdx.x / kTileRows, r = threadIdx.x % kTileRows;
            const int row = (first + it * step) * kTiles * kTileRows + tl * kTileRows + r;
            double v = 0.0;
            for (int q = 0; q < parts; ++q) v += part[(tl * parts + q) * kTileRows + r];
            if (!isfinite(v)) bad = true;
            if (logits) logits[row] = (float)v;
            if (v > bv || (v == bv && row < bi)) { bv = v; bi = row; }
        }
    }
    for (int o = 16; o; o >>= 1) {
        const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const bool wbad = __any_sync(0xffffffffu, bad);
    if (lane == 0) { wbv[warp] = bv; wbi[warp] = wbad ? -1 : bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        bool anybad = false;
        for (int i = 0; i < kWarps; ++i) anybad |= wbi[i] == -1;
        for (int i = 1; i < kWarps; ++i)
            if (wbi[i] != -1 && (wbv[i] > bv || (wbv[i] == bv && wbi[i] < bi))) { bv = wbv[i]; bi = wbi[i]; }
        scr->best_val[blockIdx.x] = bv;
        scr->best_idx[blockIdx.x] = anybad ? -1 : bi;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(&scr->counter, 1u) == gridDim.x - 1u;
    __syncthreads();
    if (!is_last || threadIdx.x != 0) return;
    __threadfence();
    double v = -1.0e300;
    int idx = 0x7fffffff;
    bool failed = false;
    for (int c = 0; c < (int)gridDim.x; ++c) {
        const double cv = scr->best_val[c];
        const int ci = scr->best_idx[c];
        if (ci == -1) { failed = true; continue; }
        if (cv > v || (cv == v && ci < idx)) { v = cv; idx = ci; }
    }
    *argmax = failed ? 0xffffffffu : (uint32_t)idx;
    scr->counter = 0u;
}

size_t smem_bytes(int H) {
    auto a16 = [](size_t v) { return (v + 15) / 16 * 16; };
    return 16 + a16((size_t)kStages * kTiles * kTileRows * (H / 256) * 210) + a16((size_t)H * 4) +
           a16(xq_words(H) * 4) + a16((size_t)H / 256 * 4) + a16((size_t)kWarps * kTileRows * 8);
}

void set_err(char* err, uint64_t n, const char* m) {
    if (err && n) snprintf(err, (size_t)n, "%s", m);
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int qx_cuda_final_head_noalloc(
    const float* residual_dev, const float* norm_weight_dev, const void* head_q6k_dev, uint32_t hidden, uint32_t vocab,
    float* logits_dev, uint32_t* argmax_dev, void* stream, char* err, uint64_t err_len) {
    if (!residual_dev || !norm_weight_dev || !head_q6k_dev || !argmax_dev) {
        set_err(err, err_len, "invalid final head argument");
        return 0;
    }
    // The head rows are staged into shared memory with 16-byte asynchronous
    // copies, so the head must start on a 16-byte boundary; the float and
    // uint32 buffers need their natural 4-byte alignment.  A pointer carved
    // from a caller's arena at another offset is refused here, before any
    // launch, instead of faulting on the device.
    if (reinterpret_cast<uintptr_t>(head_q6k_dev) & 15u) {
        set_err(err, err_len, "head_q6k_dev must be 16-byte aligned");
        return 0;
    }
    if ((reinterpret_cast<uintptr_t>(residual_dev) | reinterpret_cast<uintptr_t>(norm_weight_dev) |
         reinterpret_cast<uintptr_t>(logits_dev) | reinterpret_cast<uintptr_t>(argmax_dev)) & 3u) {
        set_err(err, err_len, "residual, norm weight, logits and argmax buffers must be 4-byte aligned");
        return 0;
    }
    if (hidden == 0 || hidden % 256 || hidden > 2048) {
        set_err(err, err_len, "hidden size must be a multiple of 256 and at most 2048");
        return 0;
    }
    if (vocab == 0 || vocab % (kTileRows * kTiles) || vocab > 0x7fffffffu) {
        set_err(err, err_len, "vocab must be a positive multiple of 32");
        return 0;
    }
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_err(err, err_len, ce != cudaSuccess ? cudaGetErrorString(ce) : "device ordinal too large");
        return 0;
    }
    HeadScratch* scr = nullptr;
    {
        // One-time set-up per device (run it before any stream capture): the
        // device address of the file-scope scratch and the shared-memory limit.
        std::lock_guard<std::mutex> lock(g_mutex);
        if (!g_ready[dev]) {
            ce = cudaGetSymbolAddress((void**)&g_scratch_ptr[dev], g_head_scratch);
            if (ce == cudaSuccess)
                ce = cudaFuncSetAttribute((const void*)k_head_noalloc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem_bytes(2048));
            if (ce != cudaSuccess) {
                set_err(err, err_len, cudaGetErrorString(ce));
                return 0;
            }
            g_ready[dev] = true;
        }
        scr = g_scratch_ptr[dev];
    }
    cudaStream_t st = (cudaStream_t)stream;
    int sms = 0, per = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_head_noalloc, kThreads, smem_bytes((int)hidden));
    int grid = sms * (per < 1 ? 1 : per);
    const int groups = (int)(vocab / (kTileRows * kTiles));
    if (grid > groups) grid = groups;
    if (grid > kNoAllocMaxCtas) grid = kNoAllocMaxCtas;
    // the completion counter must start at zero
    ce = cudaMemsetAsync(&scr->counter, 0, sizeof(unsigned), st);
    if (ce != cudaSuccess) {
        set_err(err, err_len, cudaGetErrorString(ce));
        return 0;
    }
    k_head_noalloc<<<grid, kThreads, smem_bytes((int)hidden), st>>>(
        residual_dev, norm_weight_dev, (const uint8_t*)head_q6k_dev, (int)hidden, (int)vocab, logits_dev, argmax_dev,
        scr);
    ce = cudaGetLastError();
    if (ce != cudaSuccess) {
        set_err(err, err_len, cudaGetErrorString(ce));
        return 0;
    }
    return 1;
}
