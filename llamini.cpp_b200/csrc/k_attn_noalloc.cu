// k_attn_noalloc.cu -- decode attention over caller-owned device buffers that
// allocates nothing.
//
// llamini_causal_mha_noalloc computes what causal_mha (model.c:217-260) computes
// for one query position, on device pointers, splitting the positions 0..pos
// across CTAs like the session's attention kernel. The split partials and the
// per-head completion counters live in one fixed array in device global memory
// (g_scratch below) that the module loader reserves with the library, so a call
// makes no device allocation and frees nothing. It is meant for callers that
// must not allocate on their path: an engine that has already handed nearly all
// of HBM to its own page pool (a cudaMalloc there fails or fragments that pool),
// or a loop that cannot absorb the implicit device synchronisation of cudaFree.
//
// Limits: n_heads <= 256 (one counter each), head_dim <= 256, and the partials
// of one call, n_heads x splits x (head_dim + 2) floats, within 1 MiB; the call
// uses as many position splits (up to 32, each of 64 positions or more) as fit
// and is rejected only when a limit on heads or head_dim is exceeded.
//
// What must start at zero: the counters. The loader zero-fills g_scratch, and
// the last CTA of every head sets its counter back to zero before the kernel
// ends, so each call leaves them as it found them. The partials need no
// initial value (every split writes its own before the merge reads it).
//
// Calls that overlap in time on one device -- issued on two streams, or from two
// host threads without ordering -- share the scratch and race: their results
// are undefined. Issue the calls of one device on one stream (or order them).
//
// The first call on each device does the set-up (looks up the scratch address
// with cudaGetSymbolAddress and raises the kernel's shared-memory limit); make
// that first call before any stream capture.
#include "internal.h"

#include <cuda_runtime.h>
#include <math.h>
#include <mutex>

namespace lm {
namespace {

constexpr int kThreads = 128;
constexpr uint32_t kChunk = 64;                  // positions staged in shared memory at a time
constexpr uint32_t kMaxHeads = 256;
constexpr uint32_t kMaxHeadDim = 256;            // two output dims per thread
constexpr uint32_t kMaxSplits = 32;
constexpr size_t kPartFloats = (size_t)1 << 18;  // 1 MiB of split partials
constexpr size_t kScratchFloats = kPartFloats + kMaxHeads;  // + counters
constexpr int kMaxDevices = 64;

// Split partials [head][split][m, l, o(head_dim)] followed by the counters.
static __device__ __align__(256) float g_scratch[kScratchFloats];

float* g_base[kMaxDevices];                      // per-device address of g_scratch
std::mutex g_base_mu;                            // first calls from several host threads

struct NoAllocArgs {
    const float* q;        // [n_heads * hd]
    const float* kc;       // [pos + 1][n_kv * hd], position pos already stored
    const float* vc;
    float* out;            // [n_heads * hd]
    float* part;
    uint32_t* counter;
    uint32_t pos, n_heads, n_kv, hd, n_split;
};

// One CTA per (query head, position split): stage 64 key/value rows of the
// head's kv head (model.c:220) with a padded stride, score one position per
// thread, keep an online softmax across chunks, accumulate two output dims per
// thread. The last CTA of a head merges the splits in split order.
__global__ void __launch_bounds__(kThreads) mha_noalloc_kernel(const NoAllocArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ int is_last;
    __shared__ float s_m, s_l;
    const uint32_t G = a.n_heads / a.n_kv;
    const uint32_t hd = a.hd, hp = hd + 1, kvd = a.n_kv * hd;
    const uint32_t h = blockIdx.x, g = h / G, split = blockIdx.y;
    const uint32_t L = a.pos + 1, ns = a.n_split;
    const uint32_t chunk = (L + ns - 1) / ns;
    const uint32_t t0 = min(split * chunk, L);
    const uint32_t t1 = min(t0 + chunk, L);
    const uint32_t tid = threadIdx.x;

    float* qs = sm;                  // [hd]
    float* ks = qs + hp;             // [kChunk][hd+1]
    float* vs = ks + kChunk * hp;    // [kChunk][hd+1]
    float* sc = vs + kChunk * hp;    // [kChunk + 4] probabilities, reductions, merge weights

    for (uint32_t i = tid; i < hd; i += kThreads) qs[i] = a.q[(uint64_t)h * hd + i];
    if (tid == 0) { s_m = -INFINITY; s_l = 0.f; }
    const float rscale = sqrtf((float)hd);     // model.c:243
    float o[2] = {0.f, 0.f};

    for (uint32_t c0 = t0; c0 < t1; c0 += kChunk) {
        const uint32_t n = min(kChunk, t1 - c0);
        __syncthreads();
        for (uint32_t i = tid; i < n * hd; i += kThreads) {
            const uint32_t t = i / hd, d = i - t * hd;
            const uint64_t src = (uint64_t)(c0 + t) * kvd + (uint64_t)g * hd + d;
            ks[t * hp + d] = a.kc[src];
            vs[t * hp + d] = a.vc[src];
        }
        __syncthreads();
        float sv = -INFINITY;
        if (tid < n) {
            float s = 0.f;
            const float* kr = ks + tid * hp;
            for (uint32_t d = 0; d < hd; d++) s = fmaf(qs[d], kr[d], s);
            sv = s / rscale;
        }
        if (tid < 64) {
            float m = sv;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
            if ((tid & 31u) == 0) sc[kChunk + (tid >> 5)] = m;
        }
        __syncthreads();
        const float mprev = s_m;
        const float mnew = fmaxf(mprev, fmaxf(sc[kChunk], sc[kChunk + 1]));
        const float p = tid < n ? expf(sv - mnew) : 0.f;
        if (tid < kChunk) sc[tid] = p;
        if (tid < 64) {
            float l = p;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
            if ((tid & 31u) == 0) sc[kChunk + 2 + (tid >> 5)] = l;
        }
        __syncthreads();
        const float corr = expf(mprev - mnew);
        if (tid == 0) {
            s_l = s_l * corr + sc[kChunk + 2] + sc[kChunk + 3];
            s_m = mnew;
        }
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const uint32_t d = tid + kThreads * j;
            if (d < hd) {
                float acc = o[j] * corr;
                for (uint32_t t = 0; t < n; t++) acc = fmaf(sc[t], vs[t * hp + d], acc);
                o[j] = acc;
            }
        }
    }
    __syncthreads();
    if (ns == 1) {
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const uint32_t d = tid + kThreads * j;
            if (d < hd) a.out[(uint64_t)h * hd + d] = o[j] / s_l;
        }
        return;
    }
    const uint32_t stride = hd + 2;
    float* dst = a.part + ((uint64_t)h * ns + split) * stride;
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const uint32_t d = tid + kThreads * j;
        if (d < hd) dst[2 + d] = o[j];
    }
    if (tid == 0) { dst[0] = s_m; dst[1] = s_l; }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&a.counter[h], 1u) == ns - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const float* src = a.part + (uint64_t)h * ns * stride;
    if (tid < 32) {
        float M = -INFINITY;
        for (uint32_t s = tid; s < ns; s += 32) M = fmaxf(M, __ldcg(src + s * stride));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float Ls = 0.f;
        for (uint32_t s = tid; s < ns; s += 32) {
            const float w = expf(__ldcg(src + s * stride) - M);
            sc[s] = w;
            Ls += w * __ldcg(src + s * stride + 1);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, off);
        if (tid == 0) s_l = Ls;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const uint32_t d = tid + kThreads * j;
        if (d < hd) {
            float acc = 0.f;
            for (uint32_t s = 0; s < ns; s++) acc = fmaf(__ldcg(src + s * stride + 2 + d), sc[s], acc);
            a.out[(uint64_t)h * hd + d] = acc / s_l;
        }
    }
    if (tid == 0) a.counter[h] = 0u;
}

size_t smem_bytes(uint32_t hd) { return ((size_t)(hd + 1) * (1 + 2 * kChunk) + kChunk + 4) * sizeof(float); }

// Once per device, with that device current: the scratch address and the
// kernel's shared-memory limit. No allocation.
float* scratch_base(int dev) {
    std::lock_guard<std::mutex> lock(g_base_mu);
    if (g_base[dev]) return g_base[dev];
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("causal_mha_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        return nullptr;
    }
    if (!LM_CUDA(cudaFuncSetAttribute(mha_noalloc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem_bytes(kMaxHeadDim))))
        return nullptr;
    g_base[dev] = static_cast<float*>(p);
    return g_base[dev];
}

}  // namespace
}  // namespace lm

extern "C" int llamini_causal_mha_noalloc(const f32* d_q, const f32* d_key, const f32* d_val, f32* d_out, u32 pos,
                                          u32 n_heads, u32 n_heads_kv, u32 head_dim, void* stream) {
    using namespace lm;
    if (!d_q || !d_key || !d_val || !d_out) { set_error("causal_mha_noalloc: null pointer"); return -1; }
    if (n_heads == 0 || n_heads_kv == 0 || n_heads % n_heads_kv != 0 || head_dim == 0) {
        set_error("causal_mha_noalloc: bad shape heads=%u kv_heads=%u head_dim=%u", n_heads, n_heads_kv, head_dim);
        return -1;
    }
    if (n_heads > kMaxHeads || head_dim > kMaxHeadDim) {
        set_error("causal_mha_noalloc: heads=%u head_dim=%u exceed the fixed scratch limits (%u heads, head_dim %u)",
                  n_heads, head_dim, kMaxHeads, kMaxHeadDim);
        return -1;
    }
    int dev = -1;
    if (!LM_CUDA(cudaGetDevice(&dev))) return -1;
    if (dev < 0 || dev >= kMaxDevices) { set_error("causal_mha_noalloc: device %d out of range", dev); return -1; }
    float* base = scratch_base(dev);
    if (!base) return -1;
    const uint64_t L = (uint64_t)pos + 1;
    uint64_t ns = (L + kChunk - 1) / kChunk;
    if (ns > kMaxSplits) ns = kMaxSplits;
    const uint64_t fit = kPartFloats / ((uint64_t)n_heads * (head_dim + 2));
    if (ns > fit) ns = fit;
    if (ns < 1) ns = 1;
    NoAllocArgs a;
    a.q = d_q; a.kc = d_key; a.vc = d_val; a.out = d_out;
    a.part = base;
    a.counter = reinterpret_cast<uint32_t*>(base + kPartFloats);
    a.pos = pos; a.n_heads = n_heads; a.n_kv = n_heads_kv; a.hd = head_dim; a.n_split = (uint32_t)ns;
    mha_noalloc_kernel<<<dim3(n_heads, (uint32_t)ns), kThreads, smem_bytes(head_dim),
                         static_cast<cudaStream_t>(stream)>>>(a);
    return LM_CUDA(cudaGetLastError()) ? 0 : -1;
}
