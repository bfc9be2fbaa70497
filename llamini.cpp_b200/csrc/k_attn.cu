// k_attn.cu -- decode attention over the device fp16 KV cache.
//
// Replaces llamini.cpp causal_mha() (model.c:217-260) and the rope() calls that
// precede it (generate.c:100-101, model.c:31-58) for one new token. The cache
// lives on the device as fp16 in [kv_head][position][head_dim] order so that a
// head's keys and values are contiguous.
//
// Grid = (kv heads) x (position splits). A CTA takes one kv head, all query
// heads that share it (GQA group, model.c:220), and one contiguous slice of
// positions 0..pos. It rotates the queries itself; the CTA whose slice holds
// `pos` also rotates the new key and stores the new key/value into the cache
// before reading it back. Each CTA writes an unnormalised partial (running max,
// sum of exponentials, weighted value sum); the last CTA of a kv head (atomic
// ticket) merges the partials and writes the attention output.
#include "internal.h"

#include <cuda_fp16.h>

namespace lm {

constexpr int kAttnThreads = 128;

// Cache element access: f32 keeps the reference's precision (model.c:222-224
// stores f32), fp16 halves the cache traffic.
__device__ __forceinline__ float kv_load(const float* p) { return *p; }
__device__ __forceinline__ float kv_load(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ void kv_store(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_store(__half* p, float v) { *p = __float2half_rn(v); }

// Rotate one (a, b) pair of element index `i` of a head (model.c:31-58).
__device__ __forceinline__ void rope_pair(float* a, float* b, uint32_t pos, uint32_t expo_num,
                                          uint32_t hd, float base) {
    const float th = powf(base, -(float)expo_num / (float)hd);
    const float ang = (float)pos * th;
    const float c = cosf(ang), s = sinf(ang);
    const float x = *a, y = *b;
    *a = x * c - y * s;
    *b = x * s + y * c;
}

// Apply RoPE in place to one head vector v[hd] held in shared memory.
__device__ void rope_head(float* v, uint32_t hd, uint32_t pos, uint32_t mode, float base) {
    if (mode == 0) return;
    const uint32_t half = hd / 2;
    for (uint32_t j = threadIdx.x; j < half; j += blockDim.x) {
        if (mode == 2) rope_pair(&v[j], &v[j + half], pos, 2 * j, hd, base);      // NEOX
        else rope_pair(&v[2 * j], &v[2 * j + 1], pos, 2 * j, hd, base);           // NORM
    }
}

template <typename KV>
__global__ void __launch_bounds__(kAttnThreads)
attn_decode_kernel(const AttnArgs a) {
    extern __shared__ float sm[];
    const uint32_t G = a.n_heads / a.n_kv;       // query heads per kv head
    const uint32_t hd = a.hd;
    const uint32_t g = blockIdx.x, split = blockIdx.y;
    const uint32_t pos = a.st->pos;
    const uint32_t L = pos + 1;
    const uint32_t chunk = (L + a.n_split - 1) / a.n_split;
    // Slices past the end are empty (t1 == t0); later splits may start past L.
    const uint32_t t0 = min(split * chunk, L);
    const uint32_t t1 = min(t0 + chunk, L);
    const uint32_t maxc = (a.max_seq + a.n_split - 1) / a.n_split;

    float* qs = sm;                 // [G][hd]
    float* kv = qs + G * hd;        // [hd] new key, then [hd] new value
    float* sc = kv + 2 * hd;        // [G][maxc] scores / probabilities
    __shared__ int is_last;

    const float* q = a.qkv + (uint64_t)g * G * hd;
    for (uint32_t i = threadIdx.x; i < G * hd; i += blockDim.x) qs[i] = q[i];
    const bool has_new = t0 <= pos && pos < t1;
    if (has_new) {
        const float* kn = a.qkv + (uint64_t)a.n_heads * hd + (uint64_t)g * hd;
        const float* vn = kn + (uint64_t)a.n_kv * hd;
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) { kv[i] = kn[i]; kv[hd + i] = vn[i]; }
    }
    __syncthreads();
    for (uint32_t i = 0; i < G; i++) rope_head(qs + i * hd, hd, pos, a.rope, a.rope_base);
    if (has_new) rope_head(kv, hd, pos, a.rope, a.rope_base);
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
    const float rscale = sqrtf((float)hd);

    // scores: warp per position, lanes over head_dim, all G heads at once
    for (uint32_t t = t0 + warp; t < t1; t += nw) {
        const KV* kt = kc + (uint64_t)t * hd;
        for (uint32_t i = 0; i < G; i++) {
            float s = 0.f;
            for (uint32_t d = lane; d < hd; d += 32) s = fmaf(qs[i * hd + d], kv_load(kt + d), s);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) sc[i * maxc + (t - t0)] = s / rscale;
        }
    }
    __syncthreads();

    const uint32_t stride = hd + 2;
    for (uint32_t i = warp; i < G; i += nw) {
        const uint32_t h = g * G + i;
        float m = -INFINITY;
        for (uint32_t t = lane; t < t1 - t0; t += 32) m = fmaxf(m, sc[i * maxc + t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.f;
        for (uint32_t t = lane; t < t1 - t0; t += 32) {
            float p = expf(sc[i * maxc + t] - m);
            sc[i * maxc + t] = p;
            l += p;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        __syncwarp();
        float* dst = a.part + ((uint64_t)h * a.n_split + split) * stride;
        for (uint32_t d = lane; d < hd; d += 32) {
            float o = 0.f;
            for (uint32_t t = t0; t < t1; t++) o = fmaf(sc[i * maxc + (t - t0)], kv_load(vc + (uint64_t)t * hd + d), o);
            if (a.n_split == 1) a.out[(uint64_t)h * hd + d] = o / l;
            else dst[2 + d] = o;
        }
        if (a.n_split > 1 && lane == 0) { dst[0] = m; dst[1] = l; }
    }
    if (a.n_split == 1) return;

    // last CTA of this kv head merges the partials
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t prev = atomicAdd(&a.counter[g], 1u);
        is_last = prev == a.n_split - 1;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (uint32_t i = warp; i < G; i += nw) {
        const uint32_t h = g * G + i;
        const float* src = a.part + (uint64_t)h * a.n_split * stride;
        float M = -INFINITY;
        for (uint32_t s = 0; s < a.n_split; s++) M = fmaxf(M, __ldcg(src + s * stride));
        float Lsum = 0.f;
        for (uint32_t s = 0; s < a.n_split; s++) {
            float ms = __ldcg(src + s * stride);
            if (ms != -INFINITY) Lsum += __ldcg(src + s * stride + 1) * expf(ms - M);
        }
        for (uint32_t d = lane; d < hd; d += 32) {
            float o = 0.f;
            for (uint32_t s = 0; s < a.n_split; s++) {
                float ms = __ldcg(src + s * stride);
                if (ms != -INFINITY) o += __ldcg(src + s * stride + 2 + d) * expf(ms - M);
            }
            a.out[(uint64_t)h * hd + d] = o / Lsum;
        }
    }
    if (threadIdx.x == 0) a.counter[g] = 0u;
}

bool attn_init() {
    return LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
}

bool launch_attention(const AttnArgs& a, cudaStream_t st) {
    if (a.n_kv == 0 || a.n_heads % a.n_kv != 0 || a.hd == 0 || a.n_split == 0) {
        set_error("attention: bad shape heads=%u kv=%u hd=%u", a.n_heads, a.n_kv, a.hd);
        return false;
    }
    const uint32_t G = a.n_heads / a.n_kv;
    const uint32_t maxc = (a.max_seq + a.n_split - 1) / a.n_split;
    size_t smem = ((size_t)G * a.hd + 2 * a.hd + (size_t)G * maxc) * sizeof(float);
    if (smem > 200 * 1024) { set_error("attention: shared memory %zu too large", smem); return false; }
    dim3 grid(a.n_kv, a.n_split);
    if (a.kv_f16) attn_decode_kernel<__half><<<grid, kAttnThreads, smem, st>>>(a);
    else attn_decode_kernel<float><<<grid, kAttnThreads, smem, st>>>(a);
    return LM_CUDA(cudaGetLastError());
}

}  // namespace lm
