// k_attn.cu -- decode attention over the device KV cache.
//
// Replaces llamini.cpp causal_mha() (model.c:217-260) and the rope() calls that
// precede it (generate.c:100-101, model.c:31-58) for one new token. The cache
// lives on the device in [kv_head][position][head_dim] order (f32 by default,
// fp16 on request), so a head's keys and values are contiguous.
//
// Grid = (query heads) x (position splits); each CTA computes one split of one
// head with the shared core in attn_core.cuh (chunked cp.async staging of the
// cached K/V rows, online softmax). The CTA rotates its query itself (angle =
// pos * theta_j with theta_j = base^(-2j/hd) computed on the host with the C
// library's powf, exactly the reference's value); the CTA whose split holds
// `pos` also rotates the new key, uses the new key/value from shared memory,
// and -- for the group's first head -- stores them into the cache. The last
// CTA of a head (atomic ticket) merges the splits in split order.
#include "internal.h"
#include "pdl.cuh"
#include "attn_core.cuh"

#include <cuda_fp16.h>

namespace lm {

constexpr int kAttnThreads = 128;

// Split `split` of head h for the sequence whose buffers `a` points at.
template <typename KV>
__device__ __forceinline__ void attn_one(const AttnArgs& a, uint32_t h, uint32_t split, uint8_t* smem, int& is_last,
                                         float& s_ls) {
    const uint32_t G = a.n_heads / a.n_kv;        // query heads per kv head (model.c:220)
    const uint32_t hd = a.hd;
    const uint32_t g = h / G;
    const uint32_t pos = a.st->pos;
    const SplitRange r = split_range(pos, a.n_split, split);
    if (split >= r.ns) return;
    const uint32_t tid = threadIdx.x;
    const bool f16 = sizeof(KV) == 2;
    const AttnSm sm = attn_carve(smem, hd, f16);
    float* wts = reinterpret_cast<float*>(smem + attn_core_bytes(hd, f16));   // [n_split] merge weights

    const bool has_new = r.t0 <= pos && pos < r.t1;
    for (uint32_t i = tid; i < hd; i += blockDim.x) {
        sm.qs[i] = a.qkv[(uint64_t)h * hd + i];
        if (has_new) {
            sm.kn[i] = a.qkv[(uint64_t)a.n_heads * hd + (uint64_t)g * hd + i];
            sm.vn[i] = a.qkv[(uint64_t)(a.n_heads + a.n_kv) * hd + (uint64_t)g * hd + i];
        }
    }
    __syncthreads();
    rope_pairs(sm.qs, hd, pos, a.rope, a.theta, tid, blockDim.x);
    if (has_new) rope_pairs(sm.kn, hd, pos, a.rope, a.theta, tid, blockDim.x);
    __syncthreads();
    KV* kc = reinterpret_cast<KV*>(a.kc) + (uint64_t)g * a.max_seq * hd;
    KV* vc = reinterpret_cast<KV*>(a.vc) + (uint64_t)g * a.max_seq * hd;
    if (has_new && h == g * G) {                  // one writer per kv head
        for (uint32_t i = tid; i < hd; i += blockDim.x) {
            kv_put(kc + (uint64_t)pos * hd + i, sm.kn[i]);
            kv_put(vc + (uint64_t)pos * hd + i, sm.vn[i]);
        }
    }
    const float o = attn_chunks<KV>(sm, kc, vc, pos, r.t0, r.t1, hd, tid, blockDim.x, false,
                                    [] { __syncthreads(); });
    const float m = sm.sc[kAttnChunk + 4], l = sm.sc[kAttnChunk + 5];
    if (r.ns == 1) {
        if (tid < hd) a.out[(uint64_t)h * hd + tid] = merged_single(o, m, l);
        return;
    }
    const uint32_t stride = attn_part_stride(hd);
    float* dst = a.part + ((uint64_t)h * a.n_split + split) * stride;
    if (tid < hd) dst[4 + tid] = o;
    if (tid == 0) { dst[0] = m; dst[1] = l; }
    // the last CTA of this head merges the splits (model.c:247-257 in one pass)
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&a.counter[h], 1u) == r.ns - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const float* src = a.part + (uint64_t)h * a.n_split * stride;
    if (tid == 0) s_ls = merge_weights(src, r.ns, stride, wts);
    __syncthreads();
    if (tid < hd) a.out[(uint64_t)h * hd + tid] = merged_value(src, r.ns, stride, wts, s_ls, tid);
    if (tid == 0) a.counter[h] = 0u;
}

template <typename KV>
__global__ void __launch_bounds__(kAttnThreads)
attn_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ int is_last;
    __shared__ float s_ls;
    pdl_trigger();
    pdl_wait();                                   // q/k/v come from the QKV projection
    attn_one<KV>(a, blockIdx.x, blockIdx.y, smem, is_last, s_ls);
}

// Batched decode: blockIdx.z = sequence; each sequence has its own q/k/v row,
// cache, output row, split partials and tickets, all at fixed strides.
template <typename KV>
__global__ void __launch_bounds__(kAttnThreads)
attn_batch_kernel(const AttnArgs a, const AttnBatch bt) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ int is_last;
    __shared__ float s_ls;
    pdl_trigger();
    pdl_wait();                                   // q/k/v come from the q/k/v finish
    const uint32_t b = blockIdx.z;
    AttnArgs s = a;
    s.qkv = a.qkv + (uint64_t)b * bt.qkv_stride;
    s.kc = reinterpret_cast<uint8_t*>(a.kc) + (uint64_t)b * bt.cache_stride;
    s.vc = reinterpret_cast<uint8_t*>(a.vc) + (uint64_t)b * bt.cache_stride;
    s.out = a.out + (uint64_t)b * bt.out_stride;
    s.part = a.part + (uint64_t)b * bt.part_stride;
    s.counter = a.counter + (uint64_t)b * a.n_heads;
    attn_one<KV>(s, blockIdx.x, blockIdx.y, smem, is_last, s_ls);
}

bool attn_init() {
    return LM_CUDA(cudaFuncSetAttribute(attn_batch_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_batch_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributePreferredSharedMemoryCarveout, 100)) &&
           LM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
}

bool launch_attention(const AttnArgs& a, cudaStream_t st) {
    if (a.n_kv == 0 || a.n_heads % a.n_kv != 0 || a.hd == 0 || a.hd % 2 != 0 || a.n_split == 0 || a.hd > 256) {
        set_error("attention: bad shape heads=%u kv=%u hd=%u", a.n_heads, a.n_kv, a.hd);
        return false;
    }
    const size_t smem = attn_core_bytes(a.hd, a.kv_f16 != 0) + (size_t)a.n_split * 4;
    if (smem > 200 * 1024) { set_error("attention: shared memory %zu too large", smem); return false; }
    const dim3 grid(a.n_heads, a.n_split);
    if (a.kv_f16) return LM_CUDA(launch_k(attn_decode_kernel<__half>, grid, dim3(kAttnThreads), smem, st, a));
    return LM_CUDA(launch_k(attn_decode_kernel<float>, grid, dim3(kAttnThreads), smem, st, a));
}

bool launch_attention_batch(const AttnArgs& a, const AttnBatch& bt, uint32_t B, cudaStream_t st) {
    if (a.n_kv == 0 || a.n_heads % a.n_kv != 0 || a.hd == 0 || a.hd % 2 != 0 || a.n_split == 0 || a.hd > 256) {
        set_error("attention: bad shape heads=%u kv=%u hd=%u", a.n_heads, a.n_kv, a.hd);
        return false;
    }
    const size_t smem = attn_core_bytes(a.hd, a.kv_f16 != 0) + (size_t)a.n_split * 4;
    const dim3 grid(a.n_heads, a.n_split, B);
    if (a.kv_f16) return LM_CUDA(launch_k(attn_batch_kernel<__half>, grid, dim3(kAttnThreads), smem, st, a, bt));
    return LM_CUDA(launch_k(attn_batch_kernel<float>, grid, dim3(kAttnThreads), smem, st, a, bt));
}

}  // namespace lm
