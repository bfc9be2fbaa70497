// k_attn.cu -- decode attention over the device KV cache.
//
// Replaces llamini.cpp causal_mha() (model.c:217-260) and the rope() calls that
// precede it (generate.c:100-101, model.c:31-58) for one new token. The cache
// lives on the device in [kv_head][position][head_dim] order (f32 by default,
// fp16 on request), so a head's keys and values are contiguous.
//
// Grid = (kv heads) x (position splits). A CTA takes one kv head, all query
// heads that share it (the GQA group, model.c:220) and a contiguous slice of
// positions 0..pos; only as many splits as the context needs (16 positions or
// more each) do work. The CTA rotates the queries itself (angle = pos * theta_j
// with theta_j = base^(-2j/hd) computed on the host with the C library's powf,
// exactly the reference's value); the CTA whose slice holds `pos` also rotates
// the new key and stores the new key/value before reading them back. Each CTA
// writes (running max, sum of exponentials, weighted value sum) per head; the
// last CTA of a kv head (atomic ticket) merges them with all of its threads.
#include "internal.h"
#include "pdl.cuh"

#include <cuda_fp16.h>

namespace lm {

constexpr int kAttnThreads = 128;
constexpr uint32_t kMinSplitLen = 16;     // positions per split before another split is used

__device__ __forceinline__ float kv_load(const float* p) { return *p; }
__device__ __forceinline__ float kv_load(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ void kv_store(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_store(__half* p, float v) { *p = __float2half_rn(v); }

// Rotate the pairs of `nvec` head vectors of length hd held in shared memory
// (model.c:31-58): NORM pairs (2j, 2j+1), NEOX pairs (j, j+hd/2); both use
// theta_j for pair j.
__device__ void rope_vecs(float* v, uint32_t nvec, uint32_t hd, uint32_t pos, uint32_t mode, const float* theta) {
    if (mode == 0) return;
    const uint32_t half = hd / 2;
    for (uint32_t t = threadIdx.x; t < nvec * half; t += blockDim.x) {
        const uint32_t h = t / half, j = t % half;
        float s, c;
        sincosf((float)pos * theta[j], &s, &c);
        float* a = v + h * hd + (mode == 2 ? j : 2 * j);
        float* b = mode == 2 ? a + half : a + 1;
        const float x = *a, y = *b;
        *a = x * c - y * s;
        *b = x * s + y * c;
    }
}

template <typename KV>
__global__ void __launch_bounds__(kAttnThreads)
attn_decode_kernel(const AttnArgs a) {
    extern __shared__ float sm[];
    __shared__ int is_last;
    pdl_trigger();
    pdl_wait();                                   // q/k/v come from the QKV projection
    const uint32_t G = a.n_heads / a.n_kv;        // query heads per kv head
    const uint32_t hd = a.hd;
    const uint32_t g = blockIdx.x, split = blockIdx.y;
    const uint32_t pos = a.st->pos;
    const uint32_t L = pos + 1;
    // splits in use: enough that each has >= kMinSplitLen positions
    uint32_t ns = (L + kMinSplitLen - 1) / kMinSplitLen;
    ns = ns < a.n_split ? ns : a.n_split;
    if (split >= ns) return;
    const uint32_t chunk = (L + ns - 1) / ns;
    const uint32_t t0 = min(split * chunk, L);
    const uint32_t t1 = min(t0 + chunk, L);
    const uint32_t maxc = (a.max_seq + a.n_split - 1) / a.n_split;
    const uint32_t cap = maxc > kMinSplitLen ? maxc : kMinSplitLen;   // score slots per head

    float* qs = sm;                 // [G][hd]
    float* kv = qs + G * hd;        // [hd] new key, [hd] new value
    float* sc = kv + 2 * hd;        // [G][cap] scores, then probabilities

    const float* q = a.qkv + (uint64_t)g * G * hd;
    for (uint32_t i = threadIdx.x; i < G * hd; i += blockDim.x) qs[i] = q[i];
    const bool has_new = t0 <= pos && pos < t1;
    if (has_new) {
        const float* kn = a.qkv + (uint64_t)a.n_heads * hd + (uint64_t)g * hd;
        const float* vn = kn + (uint64_t)a.n_kv * hd;
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) { kv[i] = kn[i]; kv[hd + i] = vn[i]; }
    }
    __syncthreads();
    rope_vecs(qs, G, hd, pos, a.rope, a.theta);
    if (has_new) rope_vecs(kv, 1, hd, pos, a.rope, a.theta);
    __syncthreads();
    KV* kc = reinterpret_cast<KV*>(a.kc) + (uint64_t)g * a.max_seq * hd;
    KV* vc = reinterpret_cast<KV*>(a.vc) + (uint64_t)g * a.max_seq * hd;
    if (has_new) {
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
            kv_store(kc + (uint64_t)pos * hd + i, kv[i]);
            kv_store(vc + (uint64_t)pos * hd + i, kv[hd + i]);
        }
    }
    __syncthreads();

    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float rscale = sqrtf((float)hd);        // model.c:243

    // scores: warp per position, lanes over head_dim, all G heads
    for (uint32_t t = t0 + warp; t < t1; t += nw) {
        const KV* kt = kc + (uint64_t)t * hd;
        float kr[4];
#pragma unroll
        for (int j = 0; j < 4; j++) kr[j] = (lane + 32 * j < hd) ? kv_load(kt + lane + 32 * j) : 0.f;
        for (uint32_t i = 0; i < G; i++) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) if (lane + 32 * j < hd) s = fmaf(qs[i * hd + lane + 32 * j], kr[j], s);
            for (uint32_t d = lane + 128; d < hd; d += 32) s = fmaf(qs[i * hd + d], kv_load(kt + d), s);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) sc[i * cap + (t - t0)] = s / rscale;
        }
    }
    __syncthreads();

    const uint32_t stride = hd + 2;
    const uint32_t n = t1 - t0;
    for (uint32_t i = warp; i < G; i += nw) {
        const uint32_t h = g * G + i;
        float m = -INFINITY;
        for (uint32_t t = lane; t < n; t += 32) m = fmaxf(m, sc[i * cap + t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.f;
        for (uint32_t t = lane; t < n; t += 32) {
            const float p = expf(sc[i * cap + t] - m);
            sc[i * cap + t] = p;
            l += p;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        __syncwarp();
        float* dst = a.part + ((uint64_t)h * a.n_split + split) * stride;
        for (uint32_t d = lane; d < hd; d += 32) {
            float o = 0.f;
            for (uint32_t t = 0; t < n; t++) o = fmaf(sc[i * cap + t], kv_load(vc + (uint64_t)(t0 + t) * hd + d), o);
            if (ns == 1) a.out[(uint64_t)h * hd + d] = o / l;
            else dst[2 + d] = o;
        }
        if (ns > 1 && lane == 0) { dst[0] = m; dst[1] = l; }
    }
    if (ns == 1) return;

    // the last CTA of this kv head merges the partials of its G heads
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(&a.counter[g], 1u) == ns - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    float* wts = sc;                               // [G][ns] merge weights, then [G] totals
    float* tot = sc + G * ns;
    for (uint32_t t = threadIdx.x; t < G; t += blockDim.x) {
        const float* src = a.part + (uint64_t)(g * G + t) * a.n_split * stride;
        float M = -INFINITY;
        for (uint32_t s = 0; s < ns; s++) M = fmaxf(M, __ldcg(src + s * stride));
        float Ls = 0.f;
        for (uint32_t s = 0; s < ns; s++) {
            const float w = expf(__ldcg(src + s * stride) - M);
            wts[t * ns + s] = w;
            Ls += w * __ldcg(src + s * stride + 1);
        }
        tot[t] = Ls;
    }
    __syncthreads();
    for (uint32_t idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
        const uint32_t t = idx / hd, d = idx % hd;
        const float* src = a.part + (uint64_t)(g * G + t) * a.n_split * stride + 2 + d;
        float o = 0.f;
        for (uint32_t s = 0; s < ns; s++) o = fmaf(__ldcg(src + s * stride), wts[t * ns + s], o);
        a.out[(uint64_t)(g * G + t) * hd + d] = o / tot[t];
    }
    if (threadIdx.x == 0) a.counter[g] = 0u;
}

bool attn_init() {
    return LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
}

bool launch_attention(const AttnArgs& a, cudaStream_t st) {
    if (a.n_kv == 0 || a.n_heads % a.n_kv != 0 || a.hd == 0 || a.hd % 2 != 0 || a.n_split == 0) {
        set_error("attention: bad shape heads=%u kv=%u hd=%u", a.n_heads, a.n_kv, a.hd);
        return false;
    }
    const uint32_t G = a.n_heads / a.n_kv;
    const uint32_t maxc = (a.max_seq + a.n_split - 1) / a.n_split;
    const uint32_t cap = maxc > kMinSplitLen ? maxc : kMinSplitLen;
    // scores need G*cap floats; the merge reuses them for G*n_split + G floats
    const size_t tail = (size_t)G * cap > (size_t)G * a.n_split + G ? (size_t)G * cap : (size_t)G * a.n_split + G;
    const size_t smem = ((size_t)G * a.hd + 2 * a.hd + tail) * sizeof(float);
    if (smem > 200 * 1024) { set_error("attention: shared memory %zu too large", smem); return false; }
    const dim3 grid(a.n_kv, a.n_split);
    if (a.kv_f16) return LM_CUDA(launch_k(attn_decode_kernel<__half>, grid, dim3(kAttnThreads), smem, st, a));
    return LM_CUDA(launch_k(attn_decode_kernel<float>, grid, dim3(kAttnThreads), smem, st, a));
}

}  // namespace lm
