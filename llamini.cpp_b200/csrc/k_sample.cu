// k_sample.cu -- sample_token (generate.c:25-60) on the device.
//
// The reference: p_i = expf((logit_i - max) / temp), sort by p descending (a
// stable sort, so equal p keep index order), keep the smallest prefix whose
// mass reaches top_p * sum, draw r = u * (prefix mass) with u = rand() /
// (RAND_MAX + 1), return the first kept id whose running mass passes r.
//
// The sums are the reference's own f32 arithmetic: thread 0 adds the p_i in
// index order (generate.c:40-43) while the other threads locate the nucleus.
// Give element i the 64-bit key (bits of p_i) << 32 | (2^32 - 1 - i): the
// reference's sorted order is descending key order and mass(K), the sum of p_i
// over keys >= K, is the mass of every prefix of it. A most-significant-digit
// search over the key (four bits a pass, per-digit masses in double) finds the
// largest K with mass(K) >= top_p * sum * (1 + 2^-10); the elements at or
// above it (the candidates) contain the reference's nucleus, since its f32
// sums are within far less than that margin of the exact ones. Up to
// kCand candidates are sorted in shared memory and thread 0 replays the
// reference's cumulative loop and draw over them in f32 (generate.c:45-59), so
// the pick is the reference's. A larger nucleus (a flat distribution) is
// resolved by the same key search in double instead: the nucleus end is the
// largest K with mass(K) >= top_p * sum and the pick the element whose key is
// the largest K with mass(K) > u * mass(K*); that pick can differ from the
// reference's where its f32 rounding moves a boundary.
//
// p_i is exp evaluated in double and rounded to float (a correctly rounded
// expf), computed once into a global scratch array of vocab floats (the
// caller's).
#include "internal.h"

#include <cuda_runtime.h>
#include <math.h>

namespace lm {
namespace {

constexpr int kST = 1024;
constexpr int kSW = kST / 32;
constexpr uint32_t kCand = 8192;        // candidates sorted in shared memory (64 KB of keys)

__device__ __forceinline__ uint64_t skey(float p, uint32_t i) {
    return ((uint64_t)__float_as_uint(p) << 32) | (uint64_t)(0xFFFFFFFFu - i);
}

// Block sum of 17 doubles per thread (acc[0..16]) into out[0..16] (every thread).
__device__ void block_sum17(double* acc, double* red, double* out) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
#pragma unroll
    for (int k = 0; k < 17; k++) {
        double v = acc[k];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp * 17 + k] = v;
    }
    __syncthreads();
    if (threadIdx.x < 17) {
        double v = 0.0;
        for (int w = 0; w < kSW; w++) v += red[w * 17 + threadIdx.x];
        out[threadIdx.x] = v;
    }
    __syncthreads();
}

// The largest key K (most significant digit first) whose mass(K) satisfies
// mass(K) >= thr (strict = false) or mass(K) > thr (strict = true); mass(0) is
// the total, which satisfies the test by the caller's choice of thr.
__device__ uint64_t key_search(const float* p, uint32_t V, double thr, bool strict, double* red, double* tot,
                               double* mass_out) {
    uint64_t P = 0;
    double massP = 0.0;                 // mass(P) (set on the first pass)
    for (int shift = 60; shift >= 0; shift -= 4) {
        // per-digit mass of the keys that share P's digits above `shift`,
        // and the mass of keys strictly above that prefix
        double acc[17];
#pragma unroll
        for (int k = 0; k < 17; k++) acc[k] = 0.0;
        const uint64_t hi = shift == 60 ? 0ull : (P >> (shift + 4));
        for (uint32_t i = threadIdx.x; i < V; i += kST) {
            const float pi = p[i];
            const uint64_t k = skey(pi, i);
            const uint64_t kh = shift == 60 ? 0ull : (k >> (shift + 4));
            if (kh > hi) {
                acc[16] += pi;
            } else if (kh == hi) {
                acc[(k >> shift) & 15u] += pi;     // a small per-thread table
            }
        }
        block_sum17(acc, red, tot);
        // mass(P | d << shift) = above + sum of digits >= d; the largest d that
        // passes (d = 0, mass(P), when none does: the whole remaining range)
        double m = tot[16];
        uint32_t best = 0;
        double mbest = -1.0;
        for (int d = 15; d >= 0; d--) {
            m += tot[d];
            const bool ok = strict ? m > thr : m >= thr;
            if (ok) {
                best = (uint32_t)d;
                mbest = m;
                break;
            }
        }
        if (mbest < 0.0) mbest = m;
        P |= (uint64_t)best << shift;
        massP = mbest;
    }
    *mass_out = massP;
    return P;
}

__global__ void __launch_bounds__(kST) sample_kernel(const float* logits, uint32_t V, float temp, float top_p, float u,
                                                    float* p, uint32_t* tok_out) {
    extern __shared__ unsigned long long cand[];           // kCand keys
    __shared__ double red[kSW * 17];
    __shared__ double tot[17];
    __shared__ float smax[kSW];
    __shared__ float s_f32;
    __shared__ uint32_t n_cand;
    // max logit (generate.c:35-36)
    float mx = -INFINITY;
    for (uint32_t i = threadIdx.x; i < V; i += kST) mx = fmaxf(mx, logits[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31u) == 0) smax[threadIdx.x >> 5] = mx;
    if (threadIdx.x == 0) n_cand = 0;
    __syncthreads();
    mx = smax[0];
    for (int w = 1; w < kSW; w++) mx = fmaxf(mx, smax[w]);
    // p_i (generate.c:38-43) and their exact sum
    double acc[17];
#pragma unroll
    for (int k = 0; k < 17; k++) acc[k] = 0.0;
    for (uint32_t i = threadIdx.x; i < V; i += kST) {
        const float x = (logits[i] - mx) / temp;
        const float pi = (float)exp((double)x);
        p[i] = pi;
        acc[0] += pi;
    }
    __syncthreads();                    // p is written by this CTA's threads; reads follow a barrier
    block_sum17(acc, red, tot);
    const double sum = tot[0];
    // the reference's f32 sum, in index order (thread 0, alongside the search)
    if (threadIdx.x == 0) {
        float sf = 0.0f;
        for (uint32_t i = 0; i < V; i++) sf += p[i];
        s_f32 = sf;
    }
    // candidates: every key at or above the largest K whose mass reaches the
    // target with margin (the whole vocabulary when the margin passes the sum)
    double cmass = 0.0;
    const double want = (double)top_p * sum * (1.0 + 1.0 / 1024.0);
    const uint64_t Kc = want >= sum ? 0ull : key_search(p, V, want, false, red, tot, &cmass);
    for (uint32_t i = threadIdx.x; i < V; i += kST) {
        const uint64_t k = skey(p[i], i);
        if (k >= Kc) {
            const uint32_t slot = atomicAdd(&n_cand, 1u);
            if (slot < kCand) cand[slot] = k;
        }
    }
    __syncthreads();
    const uint32_t nc = n_cand;
    if (nc <= kCand) {
        // bitonic sort, descending, over the next power of two (padding keys 0)
        uint32_t n2 = 1;
        while (n2 < nc) n2 <<= 1;
        for (uint32_t i = nc + threadIdx.x; i < n2; i += kST) cand[i] = 0ull;
        __syncthreads();
        for (uint32_t k = 2; k <= n2; k <<= 1) {
            for (uint32_t j = k >> 1; j > 0; j >>= 1) {
                for (uint32_t i = threadIdx.x; i < n2; i += kST) {
                    const uint32_t l = i ^ j;
                    if (l > i) {
                        const unsigned long long a = cand[i], b = cand[l];
                        const bool desc = (i & k) == 0;
                        if (desc ? a < b : a > b) {
                            cand[i] = b;
                            cand[l] = a;
                        }
                    }
                }
                __syncthreads();
            }
        }
        if (threadIdx.x == 0) {
            // generate.c:45-59 in f32, over the sorted candidates
            const float sf = s_f32;
            float cum = 0.0f;
            uint32_t keep = 0;
            bool reached = false;
            while (keep < nc) {
                cum += __uint_as_float((uint32_t)(cand[keep] >> 32));
                keep++;
                if (cum >= top_p * sf) {
                    reached = true;
                    break;
                }
            }
            // the candidates end before the nucleus does only when the margin
            // covered the whole vocabulary (then keep == V as in the reference)
            if (reached || nc == V) {
                const float r = u * cum;
                float a = 0.0f;
                uint32_t pick = 0xFFFFFFFFu - (uint32_t)(cand[0] & 0xFFFFFFFFull);
                for (uint32_t i = 0; i < keep; i++) {
                    a += __uint_as_float((uint32_t)(cand[i] >> 32));
                    if (r < a) {
                        pick = 0xFFFFFFFFu - (uint32_t)(cand[i] & 0xFFFFFFFFull);
                        break;
                    }
                }
                *tok_out = pick;
                n_cand = 0xFFFFFFFFu;        // done
            }
        }
        __syncthreads();
        if (n_cand == 0xFFFFFFFFu) return;
    }
    // a nucleus beyond the shared-memory candidates: the double-precision search
    double cum = 0.0;
    key_search(p, V, (double)top_p * sum, false, red, tot, &cum);
    double mpick = 0.0;
    const uint64_t K = key_search(p, V, (double)u * cum, true, red, tot, &mpick);
    if (threadIdx.x == 0) *tok_out = 0xFFFFFFFFu - (uint32_t)(K & 0xFFFFFFFFull);
}

}  // namespace

bool launch_sample(const float* d_logits, uint32_t vocab, float temp, float top_p, float u, float* d_scratch,
                   uint32_t* d_tok, cudaStream_t st) {
    static bool attr = false;                          // 64 KB of dynamic shared memory (once per process)
    if (!attr) {
        if (!LM_CUDA(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)(kCand * sizeof(unsigned long long)))))
            return false;
        attr = true;
    }
    sample_kernel<<<1, kST, kCand * sizeof(unsigned long long), st>>>(d_logits, vocab, temp, top_p, u, d_scratch, d_tok);
    return LM_CUDA(cudaGetLastError());
}

}  // namespace lm

extern "C" u32 llamini_sample_host(const f32* logits, u32 vocab, f32 temp, f32 top_p, f32 u) {
    using namespace lm;
    if (!logits || vocab == 0 || !(temp > 0.0f)) {
        set_error("sample_host: needs logits, vocab > 0 and temp > 0");
        return 0xFFFFFFFFu;
    }
    if (!ensure_device()) return 0xFFFFFFFFu;
    float *d_l = nullptr, *d_p = nullptr;
    uint32_t* d_t = nullptr;
    u32 tok = 0xFFFFFFFFu;
    cudaStream_t st = stream();
    if (LM_CUDA(cudaMalloc(&d_l, (size_t)vocab * 4)) && LM_CUDA(cudaMalloc(&d_p, (size_t)vocab * 4)) &&
        LM_CUDA(cudaMalloc(&d_t, 4)) &&
        LM_CUDA(cudaMemcpyAsync(d_l, logits, (size_t)vocab * 4, cudaMemcpyHostToDevice, st)) &&
        launch_sample(d_l, vocab, temp, top_p, u, d_p, d_t, st) &&
        LM_CUDA(cudaMemcpyAsync(&tok, d_t, 4, cudaMemcpyDeviceToHost, st)) && LM_CUDA(cudaStreamSynchronize(st))) {
    } else {
        tok = 0xFFFFFFFFu;
    }
    cudaFree(d_l);
    cudaFree(d_p);
    cudaFree(d_t);
    return tok;
}

