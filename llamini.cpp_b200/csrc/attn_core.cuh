// attn_core.cuh -- one (query head, position split) of decode attention,
// shared by the per-op attention kernel (k_attn.cu) and the persistent decode
// kernel (k_decode.cu), so both compute the same bits.
//
// causal_mha (model.c:217-260) for one query position: scores q.k / sqrt(hd),
// max-subtracted softmax, weighted sum of V. A split of positions [t0, t1) is
// processed in chunks of kAttnChunk positions: the chunk's cached K/V rows are
// copied into shared memory with 16-byte cp.async (L2 only: other SMs wrote
// them), padded to a row stride that keeps "thread t reads row t" free of bank
// conflicts; thread t scores position t; an online softmax carries (max, sum)
// across chunks; thread d accumulates output dimension d. A split leaves
// (max m, sum l, unnormalised o); merge_weights() / merged_value() combine the
// splits of a head in split order.
#pragma once

#include "internal.h"

#include <cuda_fp16.h>

namespace lm {

constexpr uint32_t kAttnChunk = 64;

// Row stride in shared memory (elements): +16 bytes per row.
template <typename KV> struct KvPad;
template <> struct KvPad<float> { static constexpr uint32_t v = 4; };
template <> struct KvPad<__half> { static constexpr uint32_t v = 8; };

__host__ __device__ __forceinline__ uint32_t attn_stride(uint32_t hd, bool f16) { return hd + (f16 ? 8u : 4u); }

// Shared memory of one split (bytes): q, new k, new v (f32), K and V chunk
// buffers (cache element type), scores + reduction slots.
__host__ __device__ __forceinline__ size_t attn_core_bytes(uint32_t hd, bool f16) {
    return (size_t)3 * hd * 4 + (size_t)2 * kAttnChunk * attn_stride(hd, f16) * (f16 ? 2 : 4) +
           (size_t)(kAttnChunk + 8) * 4;
}

struct AttnSm {
    float* qs;
    float* kn;
    float* vn;
    void* ks;
    void* vs;
    float* sc;     // [kAttnChunk] probabilities, then max x2, sum x2, running m, running l
};

__device__ __forceinline__ AttnSm attn_carve(void* base, uint32_t hd, bool f16) {
    AttnSm s;
    s.qs = reinterpret_cast<float*>(base);
    s.kn = s.qs + hd;
    s.vn = s.kn + hd;
    uint8_t* p = reinterpret_cast<uint8_t*>(s.vn + hd);
    const size_t kvb = (size_t)kAttnChunk * attn_stride(hd, f16) * (f16 ? 2 : 4);
    s.ks = p;
    s.vs = p + kvb;
    s.sc = reinterpret_cast<float*>(p + 2 * kvb);
    return s;
}

// Positions of split `split` out of the ns = min(NS, ceil(L / chunk)) splits in use.
struct SplitRange {
    uint32_t ns, t0, t1;
};
__device__ __forceinline__ SplitRange split_range(uint32_t pos, uint32_t NS, uint32_t split) {
    const uint32_t L = pos + 1;
    uint32_t ns = (L + kAttnChunk - 1) / kAttnChunk;
    ns = ns < NS ? ns : NS;
    const uint32_t chunk = (L + ns - 1) / ns;
    const uint32_t t0 = min(split * chunk, L);
    return SplitRange{ns, t0, min(t0 + chunk, L)};
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n"
                 :: "r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Rows whose size is a multiple of 16 bytes move with cp.async; others (small
// or odd head sizes) with plain L2 loads.
template <typename KV>
__host__ __device__ __forceinline__ bool attn_vec_rows(uint32_t hd) { return (hd * sizeof(KV)) % 16 == 0; }

// Issue the copies of cache rows [c0, c0 + n) of one kv head (kc, vc point at
// the head's row 0; rows are hd elements) into the chunk buffers.
template <typename KV>
__device__ __forceinline__ void attn_stage_async(const AttnSm& s, const KV* kc, const KV* vc, uint32_t c0, uint32_t n,
                                                 uint32_t hd, uint32_t tid, uint32_t nt) {
    constexpr uint32_t E16 = 16 / sizeof(KV);              // elements per 16 bytes
    const uint32_t stride = hd + KvPad<KV>::v;
    KV* ks = reinterpret_cast<KV*>(s.ks);
    KV* vs = reinterpret_cast<KV*>(s.vs);
    const KV* k0 = kc + (uint64_t)c0 * hd;
    const KV* v0 = vc + (uint64_t)c0 * hd;
    if (attn_vec_rows<KV>(hd)) {
        const uint32_t upr = hd / E16;
        for (uint32_t u = tid; u < n * upr; u += nt) {
            const uint32_t t = u / upr, j = u - t * upr;
            cp_async16(ks + t * stride + j * E16, k0 + (uint64_t)t * hd + j * E16);
            cp_async16(vs + t * stride + j * E16, v0 + (uint64_t)t * hd + j * E16);
        }
    } else {
        for (uint32_t i = tid; i < n * hd; i += nt) {
            const uint32_t t = i / hd, d = i - t * hd;
            ks[t * stride + d] = __ldcg(k0 + i);
            vs[t * stride + d] = __ldcg(v0 + i);
        }
    }
}

// RoPE of one head vector in shared memory (model.c:31-58): NORM rotates pairs
// (2j, 2j+1), NEOX pairs (j, j + hd/2), both by pos * theta_j.
__device__ __forceinline__ void rope_pairs(float* v, uint32_t hd, uint32_t pos, uint32_t mode, const float* theta,
                                           uint32_t tid, uint32_t nt) {
    if (mode == 0) return;
    const uint32_t half = hd / 2;
    for (uint32_t j = tid; j < half; j += nt) {
        float sn, cs;
        sincosf((float)pos * theta[j], &sn, &cs);
        float* a = v + (mode == 2 ? j : 2 * j);
        float* b = mode == 2 ? a + half : a + 1;
        const float x = *a, y = *b;
        *a = x * cs - y * sn;
        *b = x * sn + y * cs;
    }
}

__device__ __forceinline__ float kv_f(float v) { return v; }
__device__ __forceinline__ float kv_f(__half v) { return __half2float(v); }
__device__ __forceinline__ void kv_put(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_put(__half* p, float v) { *p = __float2half_rn(v); }

__device__ __forceinline__ float dot_row(const float* qs, const float* r, uint32_t hd) {
    float s = 0.f;
    if (hd % 4 == 0) {
        for (uint32_t d = 0; d < hd; d += 4) {
            const float4 k = *reinterpret_cast<const float4*>(r + d);
            s = fmaf(qs[d], k.x, s);
            s = fmaf(qs[d + 1], k.y, s);
            s = fmaf(qs[d + 2], k.z, s);
            s = fmaf(qs[d + 3], k.w, s);
        }
    } else {
        for (uint32_t d = 0; d < hd; d++) s = fmaf(qs[d], r[d], s);
    }
    return s;
}
__device__ __forceinline__ float dot_row(const float* qs, const __half* r, uint32_t hd) {
    float s = 0.f;
    if (hd % 8 == 0) {
        for (uint32_t d = 0; d < hd; d += 8) {
            const uint4 k = *reinterpret_cast<const uint4*>(r + d);
            const __half2* h = reinterpret_cast<const __half2*>(&k);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 f = __half22float2(h[i]);
                s = fmaf(qs[d + 2 * i], f.x, s);
                s = fmaf(qs[d + 2 * i + 1], f.y, s);
            }
        }
    } else {
        for (uint32_t d = 0; d < hd; d++) s = fmaf(qs[d], __half2float(r[d]), s);
    }
    return s;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// The chunk loop of one split: qs holds the rotated query, kn/vn this step's
// rotated key and value (used for row `pos` when it falls in the split). If
// `staged` is set, the first chunk's cached rows were already issued with
// attn_stage_async. Returns thread d's unnormalised output; the split's max
// and sum are left in s.sc[kAttnChunk + 4], s.sc[kAttnChunk + 5]. `bar` is the
// barrier of the nt participating threads (nt >= 64).
template <typename KV, class Bar>
__device__ float attn_chunks(const AttnSm& s, const KV* kc, const KV* vc, uint32_t pos, uint32_t t0, uint32_t t1,
                             uint32_t hd, uint32_t tid, uint32_t nt, bool staged, Bar bar) {
    const uint32_t stride = hd + KvPad<KV>::v;
    const KV* ks = reinterpret_cast<const KV*>(s.ks);
    const KV* vs = reinterpret_cast<const KV*>(s.vs);
    float* sc = s.sc;
    const float rscale = sqrtf((float)hd);     // model.c:243
    float o = 0.f;
    if (tid == 0) { sc[kAttnChunk + 4] = -INFINITY; sc[kAttnChunk + 5] = 0.f; }
    for (uint32_t c0 = t0; c0 < t1; c0 += kAttnChunk) {
        const uint32_t n = min(kAttnChunk, t1 - c0);
        const uint32_t nold = (c0 + n > pos) ? pos - c0 : n;     // cached rows; row pos is this step's
        if (!(staged && c0 == t0)) {
            bar();                                                // previous chunk consumed
            attn_stage_async<KV>(s, kc, vc, c0, nold, hd, tid, nt);
        }
        if (nold < n) {
            KV* kw = reinterpret_cast<KV*>(s.ks) + nold * stride;
            KV* vw = reinterpret_cast<KV*>(s.vs) + nold * stride;
            for (uint32_t i = tid; i < hd; i += nt) { kv_put(kw + i, s.kn[i]); kv_put(vw + i, s.vn[i]); }
        }
        cp_async_wait_all();
        bar();
        float sv = -INFINITY;
        if (tid < n) sv = dot_row(s.qs, ks + tid * stride, hd) / rscale;
        if (tid < 64) {
            const float m = warp_max(sv);
            if ((tid & 31u) == 0) sc[kAttnChunk + (tid >> 5)] = m;
        }
        bar();
        const float mprev = sc[kAttnChunk + 4];
        const float mnew = fmaxf(mprev, fmaxf(sc[kAttnChunk], sc[kAttnChunk + 1]));
        const float p = tid < n ? expf(sv - mnew) : 0.f;
        if (tid < kAttnChunk) sc[tid] = p;
        if (tid < 64) {
            const float l = warp_sum(p);
            if ((tid & 31u) == 0) sc[kAttnChunk + 2 + (tid >> 5)] = l;
        }
        bar();
        const float corr = expf(mprev - mnew);
        if (tid < hd) {
            float acc = o * corr;
            for (uint32_t t = 0; t < n; t++) acc = fmaf(sc[t], kv_f(vs[t * stride + tid]), acc);
            o = acc;
        }
        bar();                                                    // every thread has read mprev
        if (tid == 0) {
            sc[kAttnChunk + 5] = sc[kAttnChunk + 5] * corr + sc[kAttnChunk + 2] + sc[kAttnChunk + 3];
            sc[kAttnChunk + 4] = mnew;
        }
    }
    bar();
    return o;
}

// Split partials: one row of attn_part_stride(hd) floats per (head, split):
// m, l, two unused words, then o[hd] (16-byte aligned for vector loads).
__host__ __device__ __forceinline__ uint32_t attn_part_stride(uint32_t hd) { return hd + 4; }

// Merge of a head's splits, in split order (src: the head's ns partial rows):
// w_s = exp(m_s - max m), returns sum_s w_s l_s.
__device__ __forceinline__ float merge_weights(const float* src, uint32_t ns, uint32_t stride, float* w) {
    float M = -INFINITY;
    for (uint32_t s = 0; s < ns; s++) M = fmaxf(M, __ldcg(src + s * stride));
    float Ls = 0.f;
    for (uint32_t s = 0; s < ns; s++) {
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(src + s * stride));
        const float ws = expf(ml.x - M);
        w[s] = ws;
        Ls = fmaf(ws, ml.y, Ls);
    }
    return Ls;
}
__device__ __forceinline__ float merged_value(const float* src, uint32_t ns, uint32_t stride, const float* w, float Ls,
                                              uint32_t d) {
    float acc = 0.f;
    for (uint32_t s = 0; s < ns; s++) acc = fmaf(__ldcg(src + s * stride + 4 + d), w[s], acc);
    return acc / Ls;
}
// Four consecutive dimensions d..d+3 (d % 4 == 0) of merged_value.
__device__ __forceinline__ float4 merged_value4(const float* src, uint32_t ns, uint32_t stride, const float* w,
                                                float Ls, uint32_t d) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (uint32_t s = 0; s < ns; s++) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src + s * stride + 4 + d));
        const float ws = w[s];
        acc.x = fmaf(v.x, ws, acc.x);
        acc.y = fmaf(v.y, ws, acc.y);
        acc.z = fmaf(v.z, ws, acc.z);
        acc.w = fmaf(v.w, ws, acc.w);
    }
    return make_float4(acc.x / Ls, acc.y / Ls, acc.z / Ls, acc.w / Ls);
}
// merged_value4 with the weights computed in place (same operations in the
// same order as merge_weights + merged_value4); for ns <= 4 every load is
// issued before the first use, so the merge costs one round trip to L2.
__device__ __forceinline__ float4 merge_head4(const float* src, uint32_t ns, uint32_t stride, uint32_t d) {
    if (ns <= 4) {
        float2 ml[4];
        float4 v[4];
#pragma unroll
        for (uint32_t s = 0; s < 4; s++) {
            if (s < ns) {
                ml[s] = __ldcg(reinterpret_cast<const float2*>(src + s * stride));
                v[s] = __ldcg(reinterpret_cast<const float4*>(src + s * stride + 4 + d));
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (uint32_t s = 0; s < 4; s++)
            if (s < ns) M = fmaxf(M, ml[s].x);
        float Ls = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (uint32_t s = 0; s < 4; s++) {
            if (s < ns) {
                const float ws = expf(ml[s].x - M);
                Ls = fmaf(ws, ml[s].y, Ls);
                acc.x = fmaf(v[s].x, ws, acc.x);
                acc.y = fmaf(v[s].y, ws, acc.y);
                acc.z = fmaf(v[s].z, ws, acc.z);
                acc.w = fmaf(v[s].w, ws, acc.w);
            }
        }
        return make_float4(acc.x / Ls, acc.y / Ls, acc.z / Ls, acc.w / Ls);
    }
    float M = -INFINITY;
    for (uint32_t s = 0; s < ns; s++) M = fmaxf(M, __ldcg(src + s * stride));
    float Ls = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t s = 0; s < ns; s++) {
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(src + s * stride));
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src + s * stride + 4 + d));
        const float ws = expf(ml.x - M);
        Ls = fmaf(ws, ml.y, Ls);
        acc.x = fmaf(v.x, ws, acc.x);
        acc.y = fmaf(v.y, ws, acc.y);
        acc.z = fmaf(v.z, ws, acc.z);
        acc.w = fmaf(v.w, ws, acc.w);
    }
    return make_float4(acc.x / Ls, acc.y / Ls, acc.z / Ls, acc.w / Ls);
}
// The same merge for a single split held in registers.
__device__ __forceinline__ float merged_single(float o, float m, float l) {
    const float M = fmaxf(-INFINITY, m);
    const float ws = expf(m - M);
    const float Ls = fmaf(ws, l, 0.f);
    return fmaf(o, ws, 0.f) / Ls;
}

}  // namespace lm
