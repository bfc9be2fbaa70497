// k_attn.cu -- decode attention over the device KV cache.
//
// Replaces llamini.cpp causal_mha() (model.c:217-260) and the rope() calls that
// precede it (generate.c:100-101, model.c:31-58) for one new token. The cache
// lives on the device in [kv_head][position][head_dim] order (f32 by default,
// fp16 on request), so a head's keys and values are contiguous.
//
// Grid = (query heads) x (position splits). A CTA takes one query head and a
// contiguous slice of positions 0..pos; only as many splits as the context
// needs (64 positions or more each) do work. It stages the slice's keys and
// values of the head's kv head (the GQA group, model.c:220) in shared memory
// 64 positions at a time, scores one position per thread and keeps an online
// softmax across chunks. The CTA rotates its query itself (angle = pos * theta_j
// with theta_j = base^(-2j/hd) computed on the host with the C library's powf,
// exactly the reference's value); the CTA whose slice holds `pos` also rotates
// the new key and uses the new key/value from shared memory, and the group's
// first head stores them into the cache. Each CTA writes (running max, sum of
// exponentials, weighted value sum); the last CTA of a head (atomic ticket)
// merges them with all of its threads.
#include "internal.h"
#include "pdl.cuh"

#include <cuda_fp16.h>

namespace lm {

constexpr int kAttnThreads = 128;

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

// Stage rows [c0, c0+n) of one kv head's cache (row length hd) as f32 with a
// row stride of hd+1 floats, so that "thread t reads row t" is conflict-free.
template <typename KV>
__device__ __forceinline__ void stage_rows(float* dst, const KV* src, uint32_t n, uint32_t hd) {
    for (uint32_t i = threadIdx.x; i < n * hd; i += blockDim.x) {
        const uint32_t t = i / hd, d = i - t * hd;
        dst[t * (hd + 1) + d] = kv_load(src + i);
    }
}

// One CTA per (query head, position split). q, and for the split holding
// `pos` the new key/value, are rotated locally; the new key/value rows are used
// from shared memory and written to the cache by the group's first head only,
// so no CTA reads a cache row another CTA of this launch writes.
template <typename KV>
__global__ void __launch_bounds__(kAttnThreads)
attn_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ int is_last;
    __shared__ float s_m, s_l;
    pdl_trigger();
    pdl_wait();                                   // q/k/v come from the QKV projection
    const uint32_t G = a.n_heads / a.n_kv;        // query heads per kv head (model.c:220)
    const uint32_t hd = a.hd, hp = hd + 1;
    const uint32_t h = blockIdx.x, g = h / G, split = blockIdx.y;
    const uint32_t pos = a.st->pos;
    const uint32_t L = pos + 1;
    // splits in use: each covers >= kChunk positions
    uint32_t ns = (L + kChunk - 1) / kChunk;
    ns = ns < a.n_split ? ns : a.n_split;
    if (split >= ns) return;
    const uint32_t chunk = (L + ns - 1) / ns;
    const uint32_t t0 = min(split * chunk, L);
    const uint32_t t1 = min(t0 + chunk, L);
    const uint32_t tid = threadIdx.x;

    float* qs = sm;                  // [hd]
    float* kn = qs + hp;             // [hd] new key
    float* vn = kn + hp;             // [hd] new value
    float* ks = vn + hp;             // [kChunk][hd+1]
    float* vs = ks + kChunk * hp;    // [kChunk][hd+1]
    float* sc = vs + kChunk * hp;    // [kChunk] probabilities (and merge weights)

    const bool has_new = t0 <= pos && pos < t1;
    for (uint32_t i = tid; i < hd; i += blockDim.x) {
        qs[i] = a.qkv[(uint64_t)h * hd + i];
        if (has_new) {
            kn[i] = a.qkv[(uint64_t)a.n_heads * hd + (uint64_t)g * hd + i];
            vn[i] = a.qkv[(uint64_t)(a.n_heads + a.n_kv) * hd + (uint64_t)g * hd + i];
        }
    }
    __syncthreads();
    rope_vecs(qs, 1, hd, pos, a.rope, a.theta);
    if (has_new) rope_vecs(kn, 1, hd, pos, a.rope, a.theta);
    __syncthreads();
    KV* kc = reinterpret_cast<KV*>(a.kc) + (uint64_t)g * a.max_seq * hd;
    KV* vc = reinterpret_cast<KV*>(a.vc) + (uint64_t)g * a.max_seq * hd;
    if (has_new && h == g * G) {                  // one writer per kv head
        for (uint32_t i = tid; i < hd; i += blockDim.x) {
            kv_store(kc + (uint64_t)pos * hd + i, kn[i]);
            kv_store(vc + (uint64_t)pos * hd + i, vn[i]);
        }
    }
    const float rscale = sqrtf((float)hd);        // model.c:243
    float o[2] = {0.f, 0.f};                      // thread owns dims tid, tid + 128
    if (tid == 0) { s_m = -INFINITY; s_l = 0.f; }

    for (uint32_t c0 = t0; c0 < t1; c0 += kChunk) {
        const uint32_t n = min(kChunk, t1 - c0);
        __syncthreads();                           // previous chunk consumed
        // rows < pos come from the cache (written by earlier steps); row pos
        // is this step's key/value, taken from shared memory
        const uint32_t nold = (c0 + n > pos) ? pos - c0 : n;
        stage_rows(ks, kc + (uint64_t)c0 * hd, nold, hd);
        stage_rows(vs, vc + (uint64_t)c0 * hd, nold, hd);
        if (nold < n)
            for (uint32_t i = tid; i < hd; i += blockDim.x) { ks[nold * hp + i] = kn[i]; vs[nold * hp + i] = vn[i]; }
        __syncthreads();
        // scores: thread t takes position t
        float sv = -INFINITY;
        if (tid < n) {
            float s = 0.f;
            const float* kr = ks + tid * hp;
            for (uint32_t d = 0; d < hd; d++) s = fmaf(qs[d], kr[d], s);
            sv = s / rscale;
        }
        // chunk max / sum over the first two warps (kChunk = 64 positions)
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
        const float corr = expf(mprev - mnew);    // 0 on the first chunk
        if (tid == 0) {
            s_l = s_l * corr + sc[kChunk + 2] + sc[kChunk + 3];
            s_m = mnew;
        }
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const uint32_t d = tid + 128 * j;
            if (d < hd) {
                float acc = o[j] * corr;
                for (uint32_t t = 0; t < n; t++) acc = fmaf(sc[t], vs[t * hp + d], acc);
                o[j] = acc;
            }
        }
    }
    __syncthreads();
    const uint32_t stride = hd + 2;
    float* dst = a.part + ((uint64_t)h * a.n_split + split) * stride;
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const uint32_t d = tid + 128 * j;
        if (d < hd) {
            if (ns == 1) a.out[(uint64_t)h * hd + d] = o[j] / s_l;
            else dst[2 + d] = o[j];
        }
    }
    if (ns == 1) return;
    if (tid == 0) { dst[0] = s_m; dst[1] = s_l; }

    // the last CTA of this head merges the splits (model.c:247-257 in one pass)
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&a.counter[h], 1u) == ns - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const float* src = a.part + (uint64_t)h * a.n_split * stride;
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
        const uint32_t d = tid + 128 * j;
        if (d < hd) {
            float acc = 0.f;
            for (uint32_t s = 0; s < ns; s++) acc = fmaf(__ldcg(src + s * stride + 2 + d), sc[s], acc);
            a.out[(uint64_t)h * hd + d] = acc / s_l;
        }
    }
    if (tid == 0) a.counter[h] = 0u;
}

bool attn_init() {
    return LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributePreferredSharedMemoryCarveout, 100)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
}

bool launch_attention(const AttnArgs& a, cudaStream_t st) {
    if (a.n_kv == 0 || a.n_heads % a.n_kv != 0 || a.hd == 0 || a.hd % 2 != 0 || a.n_split == 0 || a.hd > 256) {
        set_error("attention: bad shape heads=%u kv=%u hd=%u", a.n_heads, a.n_kv, a.hd);
        return false;
    }
    const size_t hp = a.hd + 1;
    const size_t tail = kChunk + 4 > a.n_split ? kChunk + 4 : a.n_split;
    const size_t smem = (3 * hp + 2 * (size_t)kChunk * hp + tail) * sizeof(float);
    if (smem > 200 * 1024) { set_error("attention: shared memory %zu too large", smem); return false; }
    const dim3 grid(a.n_heads, a.n_split);
    if (a.kv_f16) return LM_CUDA(launch_k(attn_decode_kernel<__half>, grid, dim3(kAttnThreads), smem, st, a));
    return LM_CUDA(launch_k(attn_decode_kernel<float>, grid, dim3(kAttnThreads), smem, st, a));
}

}  // namespace lm
