// k_prefill.cu -- prompt positions in chunks (prefill).
//
// generate_autoregressive (generate.c:122-167) runs every prompt position
// through the decode step and discards the logits of all but the last one.
// Here up to 64 prompt positions go through each layer together (p0 .. p0 +
// C - 1 of one sequence, or cp consecutive positions of each of ns sequences
// of a batch: column b is position p0 + b % cp of sequence b / cp): the matrices as tcgen05 GEMMs with the C positions as the
// columns (k_tgemm.cu, same staging and finish kernels as batched decode), the
// rotation and KV-cache writes of all C positions, then causal attention of
// every position over the cache up to itself -- per position the arithmetic of
// model.c:217-260 (scores (q . k) / sqrtf(hd), max-subtracted expf, weighted
// sum of V), evaluated as an online softmax over 64-key tiles. No lm_head for
// a prompt: its last position runs through the decode step, which produces
// the logits and the first generated token. Teacher-forced perplexity adds the
// final norm and lm_head of every chunk position (a tensor-core GEMM) and
// scores each position's next token (pnll_kernel).
#include "internal.h"
#include "rows.cuh"
#include "attn_core.cuh"

#include <cuda_fp16.h>

namespace lm {

// grid C, 256 threads: column b embeds its position's token (tensor_get_row,
// tensor.c:24-30; GPT-2 adds the learned position row, gpt2.c:155-160).
__global__ void pembed_kernel(const PEmbedArgs a) {
    const uint32_t b = blockIdx.x, i = b / a.cp, p = a.p0 + (b - i * a.cp);
    uint32_t t = a.tokens[(uint64_t)i * a.tok_stride + p];
    if (t >= a.tok.rows) t = 0;                    // out-of-range ids read row 0
    float* h = a.hidden + (uint64_t)b * a.dim;
    decode_row_part(a.tok, t, h, a.scale, false, threadIdx.x, blockDim.x);
    if (a.pos.ptr != nullptr) {
        __syncthreads();
        const uint32_t pp = p < a.pos.rows ? p : a.pos.rows - 1;
        decode_row_part(a.pos, pp, h, 1.0f, true, threadIdx.x, blockDim.x);
    }
}

// grid (C, n_heads + n_kv): query head h of column b rotated in place, or kv
// head h - n_heads rotated and written with its V row to the column's
// sequence's cache at its position (model.c:31-58 then 222-224).
__global__ void prope_kernel(const PRopeArgs a) {
    const uint32_t b = blockIdx.x, h = blockIdx.y, i = b / a.cp, p = a.p0 + (b - i * a.cp), hd = a.hd;
    float* row = a.qkv + (uint64_t)b * a.qkv_stride;
    if (h < a.n_heads) {
        rope_pairs(row + (uint64_t)h * hd, hd, p, a.rope, a.theta, threadIdx.x, blockDim.x);
        return;
    }
    const uint32_t j = h - a.n_heads;
    float* k = row + (uint64_t)a.n_heads * hd + (uint64_t)j * hd;
    const float* v = row + (uint64_t)(a.n_heads + a.n_kv) * hd + (uint64_t)j * hd;
    rope_pairs(k, hd, p, a.rope, a.theta, threadIdx.x, blockDim.x);
    __syncthreads();                               // the rotated row, written by other threads
    const uint64_t off = (uint64_t)i * a.seq_elems + ((uint64_t)j * a.max_seq + p) * hd;
    for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
        if (a.kv_f16) {
            reinterpret_cast<__half*>(a.kc)[off + i] = __float2half_rn(k[i]);
            reinterpret_cast<__half*>(a.vc)[off + i] = __float2half_rn(v[i]);
        } else {
            reinterpret_cast<float*>(a.kc)[off + i] = k[i];
            reinterpret_cast<float*>(a.vc)[off + i] = v[i];
        }
    }
}

constexpr uint32_t kPQ = 16;                       // query positions per CTA
constexpr uint32_t kPK = 64;                       // keys per tile
constexpr uint32_t kPThreads = 256;                // 16 lanes per query
constexpr uint32_t kPMaxHd = 256;

__host__ __device__ __forceinline__ size_t pattn_smem(uint32_t hd) {
    return ((size_t)kPQ * hd + (size_t)kPK * (hd + 1) + (size_t)kPK * hd + (size_t)kPQ * kPK) * sizeof(float);
}

// grid (n_heads, ns * ceil(cp / kPQ)): a CTA takes up to kPQ consecutive
// positions of one sequence. Thread t serves query t / 16 of the CTA: scores
// of keys t % 16 + 16 u (u < 4) of each tile, then output elements t % 16 +
// 16 k of the head.
template <typename KV>
__global__ void __launch_bounds__(kPThreads) pattn_kernel(const PAttnArgs a) {
    extern __shared__ __align__(16) float psm[];
    const uint32_t hd = a.hd, h = blockIdx.x, g = h / (a.n_heads / a.n_kv);
    const uint32_t qb = (a.cp + kPQ - 1) / kPQ, si = blockIdx.y / qb;
    const uint32_t q0 = (blockIdx.y - si * qb) * kPQ, nq = min(kPQ, a.cp - q0);
    const uint32_t c0col = si * a.cp + q0;         // the CTA's first column
    float* qs = psm;                               // [kPQ][hd]
    float* ks = qs + kPQ * hd;                     // [kPK][hd + 1]
    float* vs = ks + kPK * (hd + 1);               // [kPK][hd]
    float* ps = vs + kPK * hd;                     // [kPQ][kPK]
    const uint32_t tid = threadIdx.x, qi = tid >> 4, lj = tid & 15u;
    for (uint32_t i = tid; i < kPQ * hd; i += kPThreads) {
        const uint32_t r = i / hd, d = i - r * hd;
        qs[i] = r < nq ? a.qkv[(uint64_t)(c0col + r) * a.qkv_stride + (uint64_t)h * hd + d] : 0.f;
    }
    const KV* kc = reinterpret_cast<const KV*>(a.kc) + (uint64_t)si * a.seq_elems + (uint64_t)g * a.max_seq * hd;
    const KV* vc = reinterpret_cast<const KV*>(a.vc) + (uint64_t)si * a.seq_elems + (uint64_t)g * a.max_seq * hd;
    const uint32_t my_pos = a.p0 + q0 + qi;        // this lane group's query position
    const uint32_t last = a.p0 + q0 + nq - 1;      // last key any query here needs
    const float rscale = sqrtf((float)hd);         // model.c:243
    float m = -INFINITY, l = 0.f;
    float o[kPMaxHd / 16];
#pragma unroll
    for (uint32_t k = 0; k < kPMaxHd / 16; k++) o[k] = 0.f;
    for (uint32_t c0 = 0; c0 <= last; c0 += kPK) {
        const uint32_t n = min(kPK, last + 1 - c0);
        __syncthreads();                           // the previous tile is consumed (and q is loaded)
        for (uint32_t i = tid; i < n * hd; i += kPThreads) {
            const uint32_t r = i / hd, d = i - r * hd;
            ks[r * (hd + 1) + d] = kv_f(kc[(uint64_t)(c0 + r) * hd + d]);
            vs[r * hd + d] = kv_f(vc[(uint64_t)(c0 + r) * hd + d]);
        }
        __syncthreads();
        float sc[4];
        float mx = -INFINITY;
#pragma unroll
        for (uint32_t u = 0; u < 4; u++) {
            const uint32_t key = lj + 16 * u;
            float v = -INFINITY;
            if (qi >= nq) v = 0.f;                 // padding query: finite, never stored
            else if (key < n && c0 + key <= my_pos) {
                const float* qr = qs + qi * hd;
                const float* kr = ks + key * (hd + 1);
                float s = 0.f;
                for (uint32_t d = 0; d < hd; d++) s = fmaf(qr[d], kr[d], s);
                v = s / rscale;
            }
            sc[u] = v;
            mx = fmaxf(mx, v);
        }
#pragma unroll
        for (int o2 = 8; o2 > 0; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
        const float mnew = fmaxf(m, mx);           // finite: key 0 is in every query's range
        float sum = 0.f;
#pragma unroll
        for (uint32_t u = 0; u < 4; u++) {
            const float p = sc[u] == -INFINITY ? 0.f : expf(sc[u] - mnew);
            ps[qi * kPK + lj + 16 * u] = p;
            sum += p;
        }
#pragma unroll
        for (int o2 = 8; o2 > 0; o2 >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o2);
        const float corr = m == -INFINITY ? 0.f : expf(m - mnew);
        l = l * corr + sum;
        m = mnew;
        __syncwarp();                              // this query's probabilities, from its 16 lanes
#pragma unroll
        for (uint32_t k = 0; k < kPMaxHd / 16; k++) {
            const uint32_t d = lj + 16 * k;
            if (d < hd) {
                float acc = o[k] * corr;
                for (uint32_t t = 0; t < n; t++) acc = fmaf(ps[qi * kPK + t], vs[t * hd + d], acc);
                o[k] = acc;
            }
        }
    }
    if (qi < nq) {
        float* out = a.out + (uint64_t)(c0col + qi) * a.out_stride + (uint64_t)h * hd;
#pragma unroll
        for (uint32_t k = 0; k < kPMaxHd / 16; k++) {
            const uint32_t d = lj + 16 * k;
            if (d < hd) out[d] = o[k] / l;
        }
    }
}

// grid C, 1024 threads: position p0 + b's log-probability of the next token,
// (logit[t] - max) - log(sum exp(logit - max)) as generate.c:182-188 computes
// it (the sums in a tree order rather than the reference's left-to-right).
__global__ void __launch_bounds__(1024) pnll_kernel(const PNllArgs a) {
    __shared__ float red[32];
    __shared__ float bval;
    const uint32_t b = blockIdx.x, pos = a.p0 + b;
    if (pos > a.last) return;                      // the whole block: no next token to score
    const float* lg = a.logits + (uint64_t)b * a.ld;
    const uint32_t tid = threadIdx.x, nw = blockDim.x >> 5;
    float m = -INFINITY;
    for (uint32_t i = tid; i < a.vocab; i += blockDim.x) m = fmaxf(m, lg[i]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31u) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
        float t = red[0];
        for (uint32_t i = 1; i < nw; i++) t = fmaxf(t, red[i]);
        bval = t;
    }
    __syncthreads();
    const float mx = bval;
    float e = 0.f;
    for (uint32_t i = tid; i < a.vocab; i += blockDim.x) e += expf(lg[i] - mx);
    for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    __syncthreads();                               // bval read by every thread before red is reused
    if ((tid & 31u) == 0) red[tid >> 5] = e;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (uint32_t i = 0; i < nw; i++) t += red[i];
        const uint32_t tgt = a.tokens[pos + 1];
        a.lp[pos] = (lg[tgt < a.vocab ? tgt : 0] - mx) - logf(t);
    }
}

bool launch_pnll(const PNllArgs& a, cudaStream_t st) {
    pnll_kernel<<<a.C, 1024, 0, st>>>(a);
    return LM_CUDA(cudaGetLastError());
}

bool prefill_init() {
    return LM_CUDA(cudaFuncSetAttribute(pattn_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)pattn_smem(kPMaxHd))) &&
           LM_CUDA(cudaFuncSetAttribute(pattn_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)pattn_smem(kPMaxHd)));
}

bool launch_pembed(const PEmbedArgs& a, cudaStream_t st) {
    if (a.cp == 0 || a.C % a.cp != 0) { set_error("prefill: %u columns are not whole runs of %u positions", a.C, a.cp); return false; }
    pembed_kernel<<<a.C, 256, 0, st>>>(a);
    return LM_CUDA(cudaGetLastError());
}

bool launch_prope(const PRopeArgs& a, uint32_t C, cudaStream_t st) {
    if (a.cp == 0 || C % a.cp != 0) { set_error("prefill: %u columns are not whole runs of %u positions", C, a.cp); return false; }
    const uint32_t nt = a.hd < 32 ? 32u : (a.hd + 31) / 32 * 32;
    prope_kernel<<<dim3(C, a.n_heads + a.n_kv), nt > 1024 ? 1024 : nt, 0, st>>>(a);
    return LM_CUDA(cudaGetLastError());
}

bool launch_pattn(const PAttnArgs& a, cudaStream_t st) {
    if (a.hd == 0 || a.hd > kPMaxHd || a.n_kv == 0 || a.n_heads % a.n_kv != 0) {
        set_error("prefill attention: head size %u (at most %u), heads %u / %u", a.hd, kPMaxHd, a.n_heads, a.n_kv);
        return false;
    }
    if (a.cp == 0 || a.C % a.cp != 0) {
        set_error("prefill attention: %u columns are not whole runs of %u positions", a.C, a.cp);
        return false;
    }
    const dim3 grid(a.n_heads, a.C / a.cp * ((a.cp + kPQ - 1) / kPQ));
    if (a.kv_f16) pattn_kernel<__half><<<grid, kPThreads, pattn_smem(a.hd), st>>>(a);
    else pattn_kernel<float><<<grid, kPThreads, pattn_smem(a.hd), st>>>(a);
    return LM_CUDA(cudaGetLastError());
}

}  // namespace lm
