// k_bgemm.cu -- dequant GEMM for a batch of input vectors.
//
// Batched decode multiplies every weight matrix by up to 64 sequences' vectors
// at once (model.c:66-176 per sequence). Layout of one op:
//
//   bstage_kernel   per sequence: optional RMSNorm / LayerNorm, then the input
//                   split into fp16 hi/lo halves of x * 2^E_b, 16-element sums,
//                   and the output scale 2^(24 - E_b) (the same arithmetic as the
//                   single-vector kernel's staging, per sequence)
//   bgemm_kernel    CTA = 128 rows (8 warps x 16-row tiles) x all sequences x one
//                   K range; the K range is walked in units (one super-block, or
//                   32-element blocks), each unit's weight rows and staged inputs
//                   double-buffered in shared memory with cp.async; per-lane f32
//                   accumulators; raw partial sums to part[ksplit][B][rows]
//   bfinish_kernel  per (sequence, row): the K-range partials summed in order,
//                   scaled, then bias / residual / gate x up / GELU and an
//                   optional argmax per sequence
#include "internal.h"
#include "bgemm.cuh"
#include "pdl.cuh"

#include <cuda_fp16.h>

namespace lm {

constexpr int kBWarps = 8;
constexpr uint32_t kBThreads = kBWarps * 32;
constexpr uint32_t kBRows = 16 * kBWarps;

__device__ __forceinline__ void cpa16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cpa8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// ---------------------------------------------------------------- staging

__device__ float bblock_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (uint32_t i = 0; i < (blockDim.x >> 5); i++) t += red[i];
    return t;
}
__device__ float bblock_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (uint32_t i = 0; i < (blockDim.x >> 5); i++) t = fmaxf(t, red[i]);
    return t;
}

// Stage sequence b's K values, already in shared memory xf (complete on
// entry): RMSNorm (model.c:4-10) or LayerNorm (gpt2.c:130-139) in place, then
// x * 2^E_b split into fp16 hi/lo. Called by every thread of the CTA.
__device__ void stage_core(const BStageArgs& a, float* xf, uint32_t b, float* red) {
    const uint32_t K = a.K, tid = threadIdx.x;
    float f = 1.0f;
    if (a.norm == NORM_RMS) {
        float s = 0.f;
        for (uint32_t i = tid; i < K; i += blockDim.x) {
            const float v = xf[i];
            s = fmaf(v, v, s);
            xf[i] = v * a.norm_w[i];
        }
        s = bblock_sum(s, red);
        f = 1.0f / sqrtf(s / (float)K + a.eps);
    } else if (a.norm == NORM_LAYER) {                   // two passes: mean, then variance
        float s = 0.f;
        for (uint32_t i = tid; i < K; i += blockDim.x) s += xf[i];
        s = bblock_sum(s, red);
        const float mean = s / (float)K;
        float vs = 0.f;
        for (uint32_t i = tid; i < K; i += blockDim.x) {
            const float c = xf[i] - mean;
            vs = fmaf(c, c, vs);
        }
        vs = bblock_sum(vs, red);
        const float inv = 1.0f / sqrtf(vs / (float)K + a.eps);
        for (uint32_t i = tid; i < K; i += blockDim.x) xf[i] = (xf[i] - mean) * inv * a.norm_w[i] + a.norm_b[i];
    }
    float m = 0.f;
    for (uint32_t i = tid; i < K; i += blockDim.x) m = fmaxf(m, fabsf(xf[i]));
    m = bblock_max(m, red);                              // ends with a barrier: xf is complete
    const float mx = m * f;
    int e = 0;
    if (mx > 0.f && mx < INFINITY) frexpf(mx, &e);
    int E = 14 - e;
    E = E > 100 ? 100 : (E < -100 ? -100 : E);
    const float F = f * __int_as_float((E + 127) << 23);
    __half* xh = reinterpret_cast<__half*>(a.xh) + (uint64_t)b * K;
    __half* xl = reinterpret_cast<__half*>(a.xl) + (uint64_t)b * K;
    float* sx = a.sx + (uint64_t)b * (K / 16);
    // thread t takes 4 consecutive elements; a 16-element run is 4 consecutive lanes
    const uint32_t n4 = K / 4, n4r = (n4 + 31u) & ~31u;
    for (uint32_t i = tid; i < n4r; i += blockDim.x) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (i < n4) {
#pragma unroll
            for (int j = 0; j < 4; j++) v[j] = xf[4 * i + j] * F;
        }
        const float s4 = (v[0] + v[1]) + (v[2] + v[3]);
        float rs = s4 * 5.9604644775390625e-08f;        // units of 2^(E-24)
        rs += __shfl_xor_sync(0xffffffffu, rs, 1);
        rs += __shfl_xor_sync(0xffffffffu, rs, 2);
        if (a.np && K % 256 == 0) {
            // 32-element sums (lanes 8t .. 8t + 7) for the tensor-core GEMM's
            // K-quant min terms: x * 2^(E-5) split into fp16 hi + lo, after the
            // staged inputs at xh + K np, per super-block u the K-major chunk
            // [2][np/8][8][8]: element (b, k) at half 16np u + 8np (k/8) + 8b + k%8
            // with k = j (hi) or 8 + j (lo) for sub-block j
            float s32 = s4 + __shfl_xor_sync(0xffffffffu, s4, 1);
            s32 += __shfl_xor_sync(0xffffffffu, s32, 2);
            s32 += __shfl_xor_sync(0xffffffffu, s32, 4);
            if (i < n4 && (i & 7u) == 0) {
                const float sv = s32 * 0.03125f;
                const __half sh = __float2half_rn(sv), sl = __float2half_rn(sv - __half2float(sh));
                __half* gs = reinterpret_cast<__half*>(a.xh) + (uint64_t)K * a.np + (uint64_t)(i >> 6) * 16u * a.np +
                             8u * b + ((i >> 3) & 7u);
                gs[0] = sh;
                gs[8u * a.np] = sl;
            }
        }
        if (i < n4 && a.np) {
            // tensor-core layout: element (b, k) at half (k/8) * 8np + 8b + k%8
            __half h[4], l[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                h[j] = __float2half_rn(v[j]);
                l[j] = __float2half_rn(v[j] - __half2float(h[j]));
            }
            const uint64_t o = (uint64_t)(i >> 1) * 8u * a.np + 8u * b + 4u * (i & 1u);
            __half* gh = reinterpret_cast<__half*>(a.xh) + o;
            __half* gl = reinterpret_cast<__half*>(a.xl) + o;
            reinterpret_cast<__half2*>(gh)[0] = __halves2half2(h[0], h[1]);
            reinterpret_cast<__half2*>(gh)[1] = __halves2half2(h[2], h[3]);
            reinterpret_cast<__half2*>(gl)[0] = __halves2half2(l[0], l[1]);
            reinterpret_cast<__half2*>(gl)[1] = __halves2half2(l[2], l[3]);
        } else if (i < n4) {
            // fragment order within the 4-group: elements 0, 2, 1, 3
            __half h[4], l[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                h[j] = __float2half_rn(v[j]);
                l[j] = __float2half_rn(v[j] - __half2float(h[j]));
            }
            const __half2 h0 = __halves2half2(h[0], h[2]), h1 = __halves2half2(h[1], h[3]);
            const __half2 l0 = __halves2half2(l[0], l[2]), l1 = __halves2half2(l[1], l[3]);
            reinterpret_cast<__half2*>(xh)[2 * i] = h0;
            reinterpret_cast<__half2*>(xh)[2 * i + 1] = h1;
            reinterpret_cast<__half2*>(xl)[2 * i] = l0;
            reinterpret_cast<__half2*>(xl)[2 * i + 1] = l1;
            if ((i & 3u) == 0) sx[i >> 2] = rs;
        }
    }
    if (tid == 0) a.oscale[b] = __int_as_float((127 + 24 - E) << 23);   // 2^(24-E)
}

// One sequence per CTA (blockIdx.x).
__global__ void __launch_bounds__(1024) bstage_kernel(const BStageArgs a) {
    extern __shared__ __align__(16) float xf[];          // K floats
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();                                          // x comes from the previous kernel
    const uint32_t b = blockIdx.x;
    const float* x = a.x + (uint64_t)b * a.ldx;
    for (uint32_t i = threadIdx.x; i < a.K; i += blockDim.x) xf[i] = x[i];
    __syncthreads();
    stage_core(a, xf, b, red);
}

// ---------------------------------------------------------------- GEMM

struct BBuf {
    uint8_t* w;
    uint16_t* xh;
    uint16_t* xl;
    float* sx;
};

__host__ __device__ __forceinline__ uint32_t bbuf_bytes(const BGemmArgs& a) {
    const uint32_t wbytes = kBRows * a.wrs;
    const uint32_t xbytes = a.bpad * a.xs * 2;
    const uint32_t sbytes = a.bpad * (a.ue / 16) * 4;
    return (wbytes + a.xlo + ((xbytes + 15) & ~15u) + sbytes + 127) & ~127u;
}

// Buffer i: weight rows, then the high halves, the low halves a.xlo bytes
// further (so hi and lo fall in different banks), then the 16-element sums.
__device__ __forceinline__ BBuf bbuf(uint8_t* base, const BGemmArgs& a, uint32_t i) {
    const uint32_t wbytes = kBRows * a.wrs;
    const uint32_t xbytes = (a.bpad * a.xs * 2 + 15) & ~15u;
    uint8_t* p = base + i * bbuf_bytes(a);
    uint8_t* xh = p + wbytes;
    return BBuf{p, reinterpret_cast<uint16_t*>(xh), reinterpret_cast<uint16_t*>(xh + a.xlo),
                reinterpret_cast<float*>(xh + a.xlo + xbytes)};
}

// Issue the copies of K unit u into buffer `buf`.
__device__ __forceinline__ void bstage_unit(const BGemmArgs& a, const BSeg& S, uint32_t row0, uint32_t u, const BBuf& buf) {
    const uint32_t tid = threadIdx.x;
    // weight rows: bytes [o, o + ub) of each row, from the 16-byte boundary below o
    const uint32_t ub = S.ub;
    const uint32_t pieces = (ub + 15) / 16 + 1;
    for (uint32_t i = tid; i < kBRows * pieces; i += kBThreads) {
        const uint32_t r = i / pieces, p = i - r * pieces;
        if (row0 + r >= S.rows) continue;
        const uint64_t o = (uint64_t)(row0 + r) * S.row_bytes + (uint64_t)u * ub;
        const uint64_t a16 = o & ~uint64_t(15);
        if (a16 + 16 * p >= o + ub) continue;
        cpa16(buf.w + r * S.wrs + 16 * p, S.w + a16 + 16 * p);
    }
    // staged inputs of every sequence for elements [u * ue, (u + 1) * ue)
    const uint32_t xp = a.ue / 8;                          // 16-byte pieces per sequence
    for (uint32_t i = tid; i < a.B * xp; i += kBThreads) {
        const uint32_t b = i / xp, p = i - b * xp;
        const uint64_t src = (uint64_t)b * a.K + (uint64_t)u * a.ue + 8 * p;
        cpa16(buf.xh + b * a.xs + 8 * p, a.xh + src);
        cpa16(buf.xl + b * a.xs + 8 * p, a.xl + src);
    }
    const uint32_t sn = a.ue / 16;                         // sums per sequence per unit
    if (sn >= 4) {
        const uint32_t sp = sn / 4;
        for (uint32_t i = tid; i < a.B * sp; i += kBThreads) {
            const uint32_t b = i / sp, p = i - b * sp;
            cpa16(buf.sx + b * sn + 4 * p, a.sx + (uint64_t)b * (a.K / 16) + (uint64_t)u * sn + 4 * p);
        }
    } else {
        for (uint32_t b = tid; b < a.B; b += kBThreads)
            cpa8(buf.sx + b * sn, a.sx + (uint64_t)b * (a.K / 16) + (uint64_t)u * sn);
    }
    cpa_commit();
}

template <uint32_t NQ>
__device__ __forceinline__ void bcompute_unit(const BGemmArgs& a, const BSeg& S, uint32_t row0, uint32_t u,
                                              const BBuf& buf, const BLane& L, uint32_t warp, BAcc<NQ>& acc) {
    const uint32_t rt = row0 + 16 * warp;                  // this warp's first row
    if (rt >= S.rows) return;
    BX X;
    X.h = buf.xh;
    X.l = buf.xl;
    X.sx = buf.sx;
    X.xs = a.xs;
    X.sxs = a.ue / 16;
    const uint32_t nq = (a.B + 3) / 4;
    const uint64_t ob = (uint64_t)u * S.ub;
    const uint32_t rg = rt + L.g, rg8 = rt + L.g + 8;
    const uint8_t* bg = buf.w + (16 * warp + L.g) * S.wrs + (uint32_t)(((uint64_t)rg * S.row_bytes + ob) & 15u);
    const uint8_t* bg8 = buf.w + (16 * warp + L.g + 8) * S.wrs + (uint32_t)(((uint64_t)rg8 * S.row_bytes + ob) & 15u);
    switch (S.type) {
    case T_Q4_K: bq4k<NQ>(bg, bg8, 0, nq, L, X, acc); break;
    case T_Q6_K: bq6k<NQ>(bg, bg8, 0, nq, L, X, acc); break;
    case T_Q8_0:
        for (uint32_t k = 0; k < a.ue / 32; k++) bq80<NQ>(bg + 34 * k, bg8 + 34 * k, 32 * k, nq, L, X, acc);
        break;
    case T_Q4_0:
        for (uint32_t k = 0; k < a.ue / 32; k++) bq40<NQ>(bg + 18 * k, bg8 + 18 * k, 32 * k, nq, L, X, acc);
        break;
    default:   // F16
        for (uint32_t k = 0; k < a.ue / 32; k++) bf16w<NQ>(bg + 64 * k, bg8 + 64 * k, 32 * k, nq, L, X, acc);
        break;
    }
}

template <uint32_t NQ>
__global__ void __launch_bounds__(kBThreads, 1) bgemm_kernel(const __grid_constant__ BGemmArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint32_t s = 0;
#pragma unroll
    for (uint32_t i = 1; i < 3; i++)
        if (i < a.nseg && blockIdx.x >= a.seg[i].rb0) s = i;
    const BSeg& S = a.seg[s];
    const uint32_t row0 = (blockIdx.x - S.rb0) * kBRows;
    const uint32_t units = a.K / a.ue;
    const uint32_t ks = blockIdx.y;
    const uint32_t u0 = ks * a.ups, u1 = min(units, u0 + a.ups);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    BLane L;
    L.g = lane >> 2;
    L.tig = lane & 3u;
    BAcc<NQ> acc;
#pragma unroll
    for (uint32_t q = 0; q < NQ; q++) acc.v[q][0] = acc.v[q][1] = 0.f;
    if (u0 < u1) {
        bstage_unit(a, S, row0, u0, bbuf(smem, a, 0));
        for (uint32_t u = u0; u < u1; u++) {
            const uint32_t cur = (u - u0) & 1u;
            if (u + 1 < u1) {
                bstage_unit(a, S, row0, u + 1, bbuf(smem, a, cur ^ 1u));
                cpa_wait<1>();
            } else {
                cpa_wait<0>();
            }
            __syncthreads();
            bcompute_unit<NQ>(a, S, row0, u, bbuf(smem, a, cur), L, warp, acc);
            __syncthreads();                               // buffer `cur` is refilled next
        }
    }
    // raw sums for rows g, g+8 of this warp's tile, sequence 4q + tig
    const uint32_t rt = row0 + 16 * warp;
#pragma unroll
    for (uint32_t q = 0; q < NQ; q++) {
        const uint32_t b = 4 * q + L.tig;
        if (b >= a.B) continue;
        float* dst = S.part + ((uint64_t)ks * a.B + b) * S.rows;
        if (rt + L.g < S.rows) dst[rt + L.g] = acc.v[q][0];
        if (rt + L.g + 8 < S.rows) dst[rt + L.g + 8] = acc.v[q][1];
    }
}

// ---------------------------------------------------------------- finish

__device__ __forceinline__ float bgelu(float x) {
    const float k0 = 0.79788456080286535587989211986876f, k1 = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(k0 * x * (1.0f + k1 * x * x)));
}
__device__ __forceinline__ unsigned long long bkey(float v, uint32_t idx) {
    if (v != v) return idx == 0 ? ~0ull : 0ull;
    if (v == 0.0f) v = 0.0f;
    const uint32_t bb = __float_as_uint(v);
    const uint32_t o = (bb & 0x80000000u) ? ~bb : (bb | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

// Row r of sequence b of a single-segment finish: the K-range partials summed
// in order, scaled by sc, then the epilogue; stores and returns the value.
__device__ __forceinline__ float bfin_row(const BFinishArgs& a, uint32_t b, uint32_t r, float sc) {
    float v = 0.f, w = 0.f;
    for (uint32_t k = 0; k < a.ksplit; k++) v += a.part[((uint64_t)k * a.B + b) * a.rows + r];
    v *= sc;
    if (a.part2) {
        for (uint32_t k = 0; k < a.ksplit; k++) w += a.part2[((uint64_t)k * a.B + b) * a.rows + r];
        w *= sc;
    }
    float* o = a.out + (uint64_t)b * a.ldo + r;
    switch (a.epi) {
    case EPI_STORE: if (a.bias) v += a.bias[r]; break;
    case EPI_RESID: if (a.bias) v += a.bias[r]; v = *o + v; break;
    case EPI_GLU_SILU: v = v / (1.0f + expf(-v)) * w; break;       // model.c:22
    case EPI_GLU_GELU: v = bgelu(v) * w; break;
    case EPI_GELU: if (a.bias) v += a.bias[r]; v = bgelu(v); break;
    }
    *o = v;
    return v;
}

// grid (ceil((rows + rows_b + rows_c) / 256), B)
__global__ void __launch_bounds__(256) bfinish_kernel(const BFinishArgs a) {
    pdl_trigger();
    pdl_wait();                                          // the partial sums come from the GEMM
    const uint32_t b = blockIdx.y, r = blockIdx.x * blockDim.x + threadIdx.x;
    unsigned long long key = 0ull;
    const float sc = a.oscale[b];
    if (r < a.rows) {
        const float v = bfin_row(a, b, r, sc);
        if (a.keys) key = bkey(v, r);
    } else if (r < a.rows + a.rows_b + a.rows_c) {
        // a further segment: its own partials, rows and bias; plain store
        const bool sb = r < a.rows + a.rows_b;
        const uint32_t rr = sb ? r - a.rows : r - a.rows - a.rows_b, n = sb ? a.rows_b : a.rows_c;
        const float* part = sb ? a.part_b : a.part_c;
        const float* bias = sb ? a.bias_b : a.bias_c;
        float v = 0.f;
        for (uint32_t k = 0; k < a.ksplit; k++) v += part[((uint64_t)k * a.B + b) * n + rr];
        v *= sc;
        if (bias) v += bias[rr];
        a.out[(uint64_t)b * a.ldo + r] = v;
    }
    if (a.keys) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
            key = k2 > key ? k2 : key;
        }
        if ((threadIdx.x & 31u) == 0 && key != 0ull) atomicMax(a.keys + b, key);
    }
}

// ---------------------------------------------------------------- host side



bool bgemm_type(uint32_t t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0 || t == T_Q4_0 || t == T_F16; }

static uint32_t unit_bytes(uint32_t type, uint32_t ue) {
    switch (type) {
    case T_Q4_K: return 144;
    case T_Q6_K: return 210;
    case T_Q8_0: return ue / 32 * 34;
    case T_Q4_0: return ue / 32 * 18;
    default: return ue * 2;                                // F16
    }
}

size_t bgemm_smem(const BGemmArgs& a) { return 2 * (size_t)bbuf_bytes(a); }

constexpr size_t kBSmemMax = 226 * 1024;

bool bgemm_init() {
    return LM_CUDA(cudaFuncSetAttribute(bgemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBSmemMax)) &&
           LM_CUDA(cudaFuncSetAttribute(bgemm_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBSmemMax)) &&
           LM_CUDA(cudaFuncSetAttribute(bgemm_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBSmemMax)) &&
           LM_CUDA(cudaFuncSetAttribute(bgemm_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBSmemMax)) &&
           LM_CUDA(cudaFuncSetAttribute(bstage_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
}

// Fill the launch geometry of `a` (segments, B, K and partial buffers set by
// the caller): unit size, K split and shared-memory strides. False (no error
// set) when a segment's format or shape is not supported here.
bool bgemm_plan(BGemmArgs& a, uint32_t target_ctas) {
    if (a.B == 0 || a.B > 64 || a.nseg == 0 || a.nseg > 3 || a.K % 32 != 0) return false;
    uint32_t rbs = 0;
    bool kquant = false;
    for (uint32_t i = 0; i < a.nseg; i++) {
        BSeg& S = a.seg[i];
        if (!bgemm_type(S.type)) return false;
        if (reinterpret_cast<uintptr_t>(S.w) % 16 != 0) return false;
        if (S.type == T_F16 && a.K % 4 != 0) return false;
        kquant = kquant || S.type == T_Q4_K || S.type == T_Q6_K;
        S.rb0 = rbs;
        rbs += (S.rows + kBRows - 1) / kBRows;
    }
    a.bpad = (a.B + 3) & ~3u;                              // the last quad's MMA reads 4 sequence rows
    const uint32_t units_max = a.K % 256 == 0 ? 256u : 32u;
    for (uint32_t ue = units_max; ue >= 32; ue /= 8) {     // 256, then 32 for block formats
        if (kquant && ue != 256) return false;
        a.ue = ue;
        a.wrs = 0;
        for (uint32_t i = 0; i < a.nseg; i++) {
            BSeg& S = a.seg[i];
            S.ub = unit_bytes(S.type, ue);
            uint32_t wrs = (S.ub + 15 + 16 + 15) & ~15u;   // slack: alignment delta + word reads
            if ((wrs / 16) % 2 == 0) wrs += 16;           // odd number of 16-byte units: rows spread over banks
            S.wrs = wrs;
            a.wrs = a.wrs > wrs ? a.wrs : wrs;
        }
        // input rows: a stride of 64 (mod 128) bytes between sequences, and the
        // low halves 64 (Q4_K: one 16-byte load per lane) or 32 (8-byte loads)
        // bytes (mod 128) after the high halves, so a warp's fragment loads
        // fall in distinct banks
        a.xs = a.ue % 64 == 0 ? a.ue + 32 : a.ue + 64;
        const uint32_t xbytes = (a.bpad * a.xs * 2 + 15) & ~15u;
        a.xlo = ((xbytes + 127) & ~127u) + (a.seg[0].type == T_Q4_K ? 64u : 32u);
        if (bgemm_smem(a) <= kBSmemMax) break;
        if (ue == 32) return false;
    }
    const uint32_t units = a.K / a.ue;
    uint32_t ks = target_ctas / (rbs ? rbs : 1);
    if (ks < 1) ks = 1;
    if (ks > units) ks = units;
    a.ups = (units + ks - 1) / ks;
    a.ksplit = (units + a.ups - 1) / a.ups;
    a.rblocks = rbs;
    return true;
}

bool launch_bgemm(const BGemmArgs& a, cudaStream_t st) {
    const dim3 grid(a.rblocks, a.ksplit);
    const size_t smem = bgemm_smem(a);
    if (a.B <= 8) bgemm_kernel<2><<<grid, kBThreads, smem, st>>>(a);
    else if (a.B <= 16) bgemm_kernel<4><<<grid, kBThreads, smem, st>>>(a);
    else if (a.B <= 32) bgemm_kernel<8><<<grid, kBThreads, smem, st>>>(a);
    else bgemm_kernel<16><<<grid, kBThreads, smem, st>>>(a);
    return LM_CUDA(cudaGetLastError());
}

bool launch_bstage(const BStageArgs& a, cudaStream_t st) {
    if (a.K % 4 != 0 || a.K > 16384) { set_error("batch staging: K %u", a.K); return false; }
    return LM_CUDA(launch_k(bstage_kernel, dim3(a.B), dim3(1024), (size_t)a.K * 4, st, a));
}


bool launch_bfinish(const BFinishArgs& a, cudaStream_t st) {
    return LM_CUDA(launch_k(bfinish_kernel, dim3((a.rows + a.rows_b + a.rows_c + 255) / 256, a.B), dim3(256), 0, st, a));
}

}  // namespace lm
