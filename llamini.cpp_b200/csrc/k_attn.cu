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

constexpr uint32_t kChunk = 64;           // positions staged in shared memory at a time
constexpr uint32_t kMaxHeadsPerWarp = 4;  // G <= 16 query heads per kv head
constexpr uint32_t kMaxDimPerLane = 8;    // head_dim <= 256

// Stage rows [t0, t0+n) of one kv head's cache (row length hd) as f32.
__device__ __forceinline__ void stage_rows(float* dst, const float* src, uint32_t n, uint32_t hd) {
    if ((hd & 3u) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (uint32_t i = threadIdx.x; i < n * hd / 4; i += blockDim.x) d4[i] = s4[i];
    } else {
        for (uint32_t i = threadIdx.x; i < n * hd; i += blockDim.x) dst[i] = src[i];
    }
}
__device__ __forceinline__ void stage_rows(float* dst, const __half* src, uint32_t n, uint32_t hd) {
    if ((hd & 3u) == 0) {
        const uint2* s2 = reinterpret_cast<const uint2*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (uint32_t i = threadIdx.x; i < n * hd / 4; i += blockDim.x) {
            const uint2 v = s2[i];
            const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
            const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
            d4[i] = make_float4(lo.x, lo.y, hi.x, hi.y);
        }
    } else {
        for (uint32_t i = threadIdx.x; i < n * hd; i += blockDim.x) dst[i] = __half2float(src[i]);
    }
}

template <typename KV>
__global__ void __launch_bounds__(kAttnThreads)
attn_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
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

    const uint32_t hd4 = (hd + 3u) & ~3u;
    float* qs = sm;                      // [G][hd]
    float* kvn = qs + G * hd4;           // [2][hd] new key, new value
    float* ks = kvn + 2 * hd4;           // [kChunk][hd]
    float* vs = ks + kChunk * hd;        // [kChunk][hd]
    float* sc = vs + kChunk * hd;        // [G][kChunk] scores / probabilities (and merge scratch)

    const float* q = a.qkv + (uint64_t)g * G * hd;
    for (uint32_t i = threadIdx.x; i < G * hd; i += blockDim.x) qs[(i / hd) * hd4 + i % hd] = q[i];
    const bool has_new = t0 <= pos && pos < t1;
    if (has_new) {
        const float* kn = a.qkv + (uint64_t)a.n_heads * hd + (uint64_t)g * hd;
        const float* vn = kn + (uint64_t)a.n_kv * hd;
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) { kvn[i] = kn[i]; kvn[hd4 + i] = vn[i]; }
    }
    __syncthreads();
    for (uint32_t i = 0; i < G; i++) rope_vecs(qs + i * hd4, 1, hd, pos, a.rope, a.theta);
    if (has_new) rope_vecs(kvn, 1, hd, pos, a.rope, a.theta);
    __syncthreads();
    KV* kc = reinterpret_cast<KV*>(a.kc) + (uint64_t)g * a.max_seq * hd;
    KV* vc = reinterpret_cast<KV*>(a.vc) + (uint64_t)g * a.max_seq * hd;
    if (has_new) {
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
            kv_store(kc + (uint64_t)pos * hd + i, kvn[i]);
            kv_store(vc + (uint64_t)pos * hd + i, kvn[hd4 + i]);
        }
    }
    __syncthreads();                               // the new row is visible to the staging loads

    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float rscale = sqrtf((float)hd);        // model.c:243
    // online softmax state of the heads this warp owns (i = warp + nw * j)
    float mrun[kMaxHeadsPerWarp], lrun[kMaxHeadsPerWarp], o[kMaxHeadsPerWarp][kMaxDimPerLane];
#pragma unroll
    for (uint32_t j = 0; j < kMaxHeadsPerWarp; j++) {
        mrun[j] = -INFINITY;
        lrun[j] = 0.f;
#pragma unroll
        for (uint32_t d = 0; d < kMaxDimPerLane; d++) o[j][d] = 0.f;
    }

    for (uint32_t c0 = t0; c0 < t1; c0 += kChunk) {
        const uint32_t n = min(kChunk, t1 - c0);
        __syncthreads();                           // previous chunk fully consumed
        stage_rows(ks, kc + (uint64_t)c0 * hd, n, hd);
        stage_rows(vs, vc + (uint64_t)c0 * hd, n, hd);
        __syncthreads();
        // scores: warp per position, lanes over head_dim, all G heads
        for (uint32_t t = warp; t < n; t += nw) {
            for (uint32_t i = 0; i < G; i++) {
                float s = 0.f;
                for (uint32_t d = lane; d < hd; d += 32) s = fmaf(qs[i * hd4 + d], ks[t * hd + d], s);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                if (lane == 0) sc[i * kChunk + t] = s / rscale;
            }
        }
        __syncthreads();
#pragma unroll
        for (uint32_t j = 0; j < kMaxHeadsPerWarp; j++) {
            const uint32_t i = warp + nw * j;
            if (i >= G) break;
            float* si = sc + i * kChunk;
            float cm = -INFINITY;
            for (uint32_t t = lane; t < n; t += 32) cm = fmaxf(cm, si[t]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, off));
            const float mnew = fmaxf(mrun[j], cm);
            const float corr = expf(mrun[j] - mnew);      // 0 on the first chunk
            float cl = 0.f;
            for (uint32_t t = lane; t < n; t += 32) {
                const float p = expf(si[t] - mnew);
                si[t] = p;
                cl += p;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) cl += __shfl_xor_sync(0xffffffffu, cl, off);
            __syncwarp();
            lrun[j] = lrun[j] * corr + cl;
            mrun[j] = mnew;
#pragma unroll
            for (uint32_t dd = 0; dd < kMaxDimPerLane; dd++) {
                const uint32_t d = lane + 32 * dd;
                if (d >= hd) break;
                float acc = o[j][dd] * corr;
                for (uint32_t t = 0; t < n; t++) acc = fmaf(si[t], vs[t * hd + d], acc);
                o[j][dd] = acc;
            }
        }
    }

    const uint32_t stride = hd + 2;
#pragma unroll
    for (uint32_t j = 0; j < kMaxHeadsPerWarp; j++) {
        const uint32_t i = warp + nw * j;
        if (i >= G) break;
        const uint32_t h = g * G + i;
        float* dst = a.part + ((uint64_t)h * a.n_split + split) * stride;
#pragma unroll
        for (uint32_t dd = 0; dd < kMaxDimPerLane; dd++) {
            const uint32_t d = lane + 32 * dd;
            if (d >= hd) break;
            if (ns == 1) a.out[(uint64_t)h * hd + d] = o[j][dd] / lrun[j];
            else dst[2 + d] = o[j][dd];
        }
        if (ns > 1 && lane == 0) { dst[0] = mrun[j]; dst[1] = lrun[j]; }
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
        float acc = 0.f;
        for (uint32_t s = 0; s < ns; s++) acc = fmaf(__ldcg(src + s * stride), wts[t * ns + s], acc);
        a.out[(uint64_t)(g * G + t) * hd + d] = acc / tot[t];
    }
    if (threadIdx.x == 0) a.counter[g] = 0u;
}

bool attn_init() {
    return LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributePreferredSharedMemoryCarveout, 100)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
}

bool launch_attention(const AttnArgs& a, cudaStream_t st) {
    if (a.n_kv == 0 || a.n_heads % a.n_kv != 0 || a.hd == 0 || a.hd % 2 != 0 || a.n_split == 0) {
        set_error("attention: bad shape heads=%u kv=%u hd=%u", a.n_heads, a.n_kv, a.hd);
        return false;
    }
    const uint32_t G = a.n_heads / a.n_kv;
    if (G > kMaxHeadsPerWarp * (kAttnThreads / 32) || a.hd > 32 * kMaxDimPerLane) {
        set_error("attention: %u query heads per kv head / head_dim %u not supported", G, a.hd);
        return false;
    }
    const size_t hd4 = (a.hd + 3u) & ~3u;
    // scores need G*kChunk floats; the merge reuses them for G*n_split + G floats
    const size_t tail = (size_t)G * kChunk > (size_t)G * a.n_split + G ? (size_t)G * kChunk : (size_t)G * a.n_split + G;
    const size_t smem = ((size_t)G * hd4 + 2 * hd4 + 2 * (size_t)kChunk * a.hd + tail) * sizeof(float);
    if (smem > 200 * 1024) { set_error("attention: shared memory %zu too large", smem); return false; }
    const dim3 grid(a.n_kv, a.n_split);
    if (a.kv_f16) return LM_CUDA(launch_k(attn_decode_kernel<__half>, grid, dim3(kAttnThreads), smem, st, a));
    return LM_CUDA(launch_k(attn_decode_kernel<float>, grid, dim3(kAttnThreads), smem, st, a));
}

}  // namespace lm
