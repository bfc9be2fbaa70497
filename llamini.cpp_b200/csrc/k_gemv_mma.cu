// k_gemv_mma.cu -- dequant-GEMV on the tensor cores (Q4_K / Q6_K / Q8_0 / Q4_0).
//
// Same contract as the CUDA-core kernel in k_gemv.cu (llamini.cpp linear(),
// model.c:66-176, with the fused prologues/epilogues), computed differently:
//
//  * Every block format is affine per group of 16 or 32 weights:
//      w = alpha * q - beta     (q a small unsigned integer, gguf.c:427-590)
//    so  sum_i w_i x_i = alpha * sum_i q_i x_i - beta * sum_i x_i.
//  * sum_i q_i x_i for 16 rows at a time is one mma.sync.m16n8k16: the integers
//    q (< 1024) enter the A operand as exact fp16 subnormals q * 2^-24, made
//    with one AND (or byte permute) on the packed bytes; x enters the B operand
//    as two fp16 columns x_hi + x_lo (22 significant bits) after the whole
//    vector is scaled by a power of two into fp16's range. Accumulation is f32.
//  * alpha, beta and the per-16 sums of x are applied in f32 by the lanes that
//    hold columns 0/1 of the accumulator; the result is scaled back at the end.
//
// CTA = one tile of 16 output rows (16 gate + 16 up rows for the gated FFN);
// its 8 warps split the row's blocks between them and combine partial sums in
// shared memory. Latency is what limits a batch-1 GEMV, so each warp loads its
// first blocks of weights into registers before anything else (before waiting
// for the previous kernel, which produces x), and keeps one iteration of loads
// in flight while it computes the previous one.
#include "internal.h"
#include "quant.cuh"
#include "pdl.cuh"

#include <cuda_fp16.h>

namespace lm {

constexpr int kMWarps = 8;
constexpr int kMThreads = kMWarps * 32;

bool mma_type(uint32_t t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0 || t == T_Q4_0; }

struct MmaSmem {
    float* xf;          // staged x (f32, before the final scale for RMSNorm)
    uint32_t* xh;       // x * 2^E as fp16 pairs, high part   (K/2 words)
    uint32_t* xl;       // low part
    float* sx;          // per 16-element run: sum(x) * 2^(E-24)
    float* red;         // [2 * kMWarps] reduction scratch
    float* part;        // [kMWarps][16] partial row sums
};

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// B fragment for the 4 consecutive elements e0..e0+3 (e0 % 4 == 0): k slots
// (2t, 2t+1) take elements (e0, e0+2), slots (2t+8, 2t+9) take (e0+1, e0+3),
// matching how the A pairs are cut from packed bytes. Column 0 = x_hi,
// column 1 = x_lo, other columns zero.
struct BFrag { uint32_t b0, b1; };

struct Lane {
    uint32_t g, tig;
    bool bact;                 // provides a B column (g < 2)
    const uint32_t* xpart;     // xh for g == 0, xl for g == 1
};

__device__ __forceinline__ BFrag bfrag(const Lane& L, uint32_t e0) {
    BFrag f{0u, 0u};
    if (L.bact) {
        const uint2 v = *reinterpret_cast<const uint2*>(L.xpart + (e0 >> 1));
        f.b0 = __byte_perm(v.x, v.y, 0x5410);
        f.b1 = __byte_perm(v.x, v.y, 0x7632);
    }
    return f;
}

// acc[0] (row g) and acc[1] (row g+8) += alpha * P - beta * S, lanes tig == 0.
__device__ __forceinline__ void scale_add(float* acc, const float* c, float a_g, float b_g, float a_g8, float b_g8,
                                          float sx) {
    acc[0] = fmaf(a_g, c[0] + c[1], fmaf(-b_g, sx, acc[0]));
    acc[1] = fmaf(a_g8, c[2] + c[3], fmaf(-b_g8, sx, acc[1]));
}

// ------------------------------------------------------------------ formats
// Each format: Raw (the words one lane needs for one iteration of rows g and
// g+8), SB (elements per iteration), load(), compute().

// Q4_K (gguf.c:504-529): 256-element super-block, 4 groups of 64; in group j
// the low nibbles of qs[32j..32j+32) are sub-block 2j, the high nibbles 2j+1.
// Lane tig takes bytes 8*tig..8*tig+8 of each group: two MMAs per sub-block.
struct FQ4K {
    static constexpr uint32_t SB = 256, SBB = 144;
    struct Raw { uint32_t h[4], h8[4]; uint2 q[4], q8[4]; };
    static __device__ __forceinline__ void load(Raw& r, const uint8_t* bg, const uint8_t* bg8, uint32_t, const Lane& L) {
        ld_v4(bg, r.h);
        ld_v4(bg8, r.h8);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            r.q[j] = __ldg(reinterpret_cast<const uint2*>(bg + 16 + 32 * j + 8 * L.tig));
            r.q8[j] = __ldg(reinterpret_cast<const uint2*>(bg8 + 16 + 32 * j + 8 * L.tig));
        }
    }
    static __device__ __forceinline__ void compute(const Raw& r, uint32_t e_blk, uint32_t, const Lane& L,
                                                   const MmaSmem& sm, float* acc) {
        const float dg = f16_bits(r.h[0] & 0xFFFFu), mg = f16_bits(r.h[0] >> 16);
        const float dg8 = f16_bits(r.h8[0] & 0xFFFFu), mg8 = f16_bits(r.h8[0] >> 16);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t e = e_blk + 64 * j + 8 * L.tig;
            const BFrag lo0 = bfrag(L, e), lo1 = bfrag(L, e + 4), hi0 = bfrag(L, e + 32), hi1 = bfrag(L, e + 36);
            const uint32_t w0 = r.q[j].x, w1 = r.q[j].y, v0 = r.q8[j].x, v1 = r.q8[j].y;
            const uint32_t w0s = w0 >> 8, w1s = w1 >> 8, v0s = v0 >> 8, v1s = v1 >> 8;
            float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(cl, w0 & 0x000F000Fu, v0 & 0x000F000Fu, w0s & 0x000F000Fu, v0s & 0x000F000Fu, lo0.b0, lo0.b1);
            mma16816(cl, w1 & 0x000F000Fu, v1 & 0x000F000Fu, w1s & 0x000F000Fu, v1s & 0x000F000Fu, lo1.b0, lo1.b1);
            // high nibbles in place (16 q): alpha of sub-block 2j+1 scaled by 1/16
            mma16816(ch, w0 & 0x00F000F0u, v0 & 0x00F000F0u, w0s & 0x00F000F0u, v0s & 0x00F000F0u, hi0.b0, hi0.b1);
            mma16816(ch, w1 & 0x00F000F0u, v1 & 0x00F000F0u, w1s & 0x00F000F0u, v1s & 0x00F000F0u, hi1.b0, hi1.b1);
            if (L.tig == 0) {
                uint32_t s0, m0, s1, m1, t0, n0, t1, n1;
                k4_scale_min(r.h + 1, 2 * j, &s0, &m0);
                k4_scale_min(r.h + 1, 2 * j + 1, &s1, &m1);
                k4_scale_min(r.h8 + 1, 2 * j, &t0, &n0);
                k4_scale_min(r.h8 + 1, 2 * j + 1, &t1, &n1);
                const uint32_t q = (e_blk + 64 * j) >> 4;
                const float sxl = sm.sx[q] + sm.sx[q + 1], sxh = sm.sx[q + 2] + sm.sx[q + 3];
                scale_add(acc, cl, dg * (float)s0, mg * (float)m0, dg8 * (float)t0, mg8 * (float)n0, sxl);
                scale_add(acc, ch, dg * (float)s1 * 0.0625f, mg * (float)m1, dg8 * (float)t1 * 0.0625f,
                          mg8 * (float)n1, sxh);
            }
        }
    }
};

// Q6_K (gguf.c:561-590): per 128-half H, byte l of ql[64H..], ql[64H+32..] and
// qh[32H..] give elements 128H + 32c + l (c = 0..3), scale sc[8H + l/16 + 2c].
// One MMA per 16-element scale group; lane tig takes l = 16u + 4tig .. +4.
// Blocks are 210 bytes, so words are read with funnel shifts (ld_u32).
struct FQ6K {
    static constexpr uint32_t SB = 256, SBB = 210;
    struct Raw { uint32_t a[4], b[4], h[4], a8[4], b8[4], h8[4], sc[4], sc8[4]; uint32_t d; };
    static __device__ __forceinline__ void load(Raw& r, const uint8_t* bg, const uint8_t* bg8, uint32_t, const Lane& L) {
#pragma unroll
        for (int H = 0; H < 2; H++) {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const uint32_t off = 16 * u + 4 * L.tig, i = 2 * H + u;
                r.a[i] = ld_u32(bg + 64 * H + off);
                r.b[i] = ld_u32(bg + 64 * H + 32 + off);
                r.h[i] = ld_u32(bg + 128 + 32 * H + off);
                r.a8[i] = ld_u32(bg8 + 64 * H + off);
                r.b8[i] = ld_u32(bg8 + 64 * H + 32 + off);
                r.h8[i] = ld_u32(bg8 + 128 + 32 * H + off);
            }
        }
        if (L.tig == 0) {
            ld_words<4>(bg + 192, r.sc);
            ld_words<4>(bg8 + 192, r.sc8);
        }
        r.d = ld_u16(bg + 208) | (ld_u16(bg8 + 208) << 16);
    }
    static __device__ __forceinline__ uint32_t word(uint32_t n, uint32_t hbits) { return (n & 0x0F0F0F0Fu) | hbits; }
    static __device__ __forceinline__ void compute(const Raw& r, uint32_t e_blk, uint32_t, const Lane& L,
                                                   const MmaSmem& sm, float* acc) {
        const float dg = f16_bits(r.d & 0xFFFFu), dg8 = f16_bits(r.d >> 16);
#pragma unroll
        for (int H = 0; H < 2; H++) {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int i = 2 * H + u;
                uint32_t wq[4], wm[4];
                wq[0] = word(r.a[i], (r.h[i] << 4) & 0x30303030u);
                wq[1] = word(r.b[i], (r.h[i] << 2) & 0x30303030u);
                wq[2] = word(r.a[i] >> 4, r.h[i] & 0x30303030u);
                wq[3] = word(r.b[i] >> 4, (r.h[i] >> 2) & 0x30303030u);
                wm[0] = word(r.a8[i], (r.h8[i] << 4) & 0x30303030u);
                wm[1] = word(r.b8[i], (r.h8[i] << 2) & 0x30303030u);
                wm[2] = word(r.a8[i] >> 4, r.h8[i] & 0x30303030u);
                wm[3] = word(r.b8[i] >> 4, (r.h8[i] >> 2) & 0x30303030u);
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const uint32_t e = e_blk + 128 * H + 32 * c + 16 * u + 4 * L.tig;
                    const BFrag b = bfrag(L, e);
                    float cc[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(cc, __byte_perm(wq[c], 0, 0x4240), __byte_perm(wm[c], 0, 0x4240),
                             __byte_perm(wq[c], 0, 0x4341), __byte_perm(wm[c], 0, 0x4341), b.b0, b.b1);
                    if (L.tig == 0) {
                        const uint32_t si = 8 * H + u + 2 * c;           // scale byte index
                        const float sg = (float)(int8_t)(uint8_t)((r.sc[si >> 2] >> (8 * (si & 3))) & 0xFFu);
                        const float sg8 = (float)(int8_t)(uint8_t)((r.sc8[si >> 2] >> (8 * (si & 3))) & 0xFFu);
                        const float ag = dg * sg, ag8 = dg8 * sg8;
                        scale_add(acc, cc, ag, 32.0f * ag, ag8, 32.0f * ag8,
                                  sm.sx[(e_blk + 128 * H + 32 * c + 16 * u) >> 4]);
                    }
                }
            }
        }
    }
};

// 32-element formats, 4 blocks per iteration (the last one may be partial;
// nb32 = number of blocks in the row).
// Q8_0 (gguf.c:489-503): w = d q, q int8; with u = q ^ 0x80, w = d u - 128 d.
struct FQ80 {
    static constexpr uint32_t SB = 128, SBB = 136, BB = 34;
    struct Raw { uint32_t w[4][2], v[4][2], d[4]; };
    static __device__ __forceinline__ void load(Raw& r, const uint8_t* bg, const uint8_t* bg8, uint32_t nvalid,
                                                const Lane& L) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k < nvalid) {
                const uint8_t* p = bg + k * BB;
                const uint8_t* q = bg8 + k * BB;
                r.w[k][0] = ld_u32(p + 2 + 4 * L.tig);
                r.w[k][1] = ld_u32(p + 18 + 4 * L.tig);
                r.v[k][0] = ld_u32(q + 2 + 4 * L.tig);
                r.v[k][1] = ld_u32(q + 18 + 4 * L.tig);
                r.d[k] = ld_u16(p) | (ld_u16(q) << 16);
            }
        }
    }
    static __device__ __forceinline__ void compute(const Raw& r, uint32_t e_blk, uint32_t nvalid, const Lane& L,
                                                   const MmaSmem& sm, float* acc) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k >= nvalid) break;
            const float dg = f16_bits(r.d[k] & 0xFFFFu), dg8 = f16_bits(r.d[k] >> 16);
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const uint32_t w = r.w[k][u] ^ 0x80808080u, v = r.v[k][u] ^ 0x80808080u;
                const uint32_t e = e_blk + 32 * k + 16 * u + 4 * L.tig;
                const BFrag b = bfrag(L, e);
                float cc[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(cc, __byte_perm(w, 0, 0x4240), __byte_perm(v, 0, 0x4240),
                         __byte_perm(w, 0, 0x4341), __byte_perm(v, 0, 0x4341), b.b0, b.b1);
                if (L.tig == 0)
                    scale_add(acc, cc, dg, 128.0f * dg, dg8, 128.0f * dg8, sm.sx[(e_blk + 32 * k + 16 * u) >> 4]);
            }
        }
    }
};

// Q4_0 (gguf.c:427-444): w = (q - 8) d; low nibbles are elements 0..15, high
// nibbles 16..31.
struct FQ40 {
    static constexpr uint32_t SB = 128, SBB = 72, BB = 18;
    struct Raw { uint32_t w[4], v[4], d[4]; };
    static __device__ __forceinline__ void load(Raw& r, const uint8_t* bg, const uint8_t* bg8, uint32_t nvalid,
                                                const Lane& L) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k < nvalid) {
                r.w[k] = ld_u32(bg + k * BB + 2 + 4 * L.tig);
                r.v[k] = ld_u32(bg8 + k * BB + 2 + 4 * L.tig);
                r.d[k] = ld_u16(bg + k * BB) | (ld_u16(bg8 + k * BB) << 16);
            }
        }
    }
    static __device__ __forceinline__ void compute(const Raw& r, uint32_t e_blk, uint32_t nvalid, const Lane& L,
                                                   const MmaSmem& sm, float* acc) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k >= nvalid) break;
            const float dg = f16_bits(r.d[k] & 0xFFFFu), dg8 = f16_bits(r.d[k] >> 16);
            const uint32_t w = r.w[k], v = r.v[k], ws = w >> 8, vs = v >> 8;
            const uint32_t e = e_blk + 32 * k;
            const BFrag lo = bfrag(L, e + 4 * L.tig), hi = bfrag(L, e + 16 + 4 * L.tig);
            float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(cl, w & 0x000F000Fu, v & 0x000F000Fu, ws & 0x000F000Fu, vs & 0x000F000Fu, lo.b0, lo.b1);
            mma16816(ch, w & 0x00F000F0u, v & 0x00F000F0u, ws & 0x00F000F0u, vs & 0x00F000F0u, hi.b0, hi.b1);
            if (L.tig == 0) {
                const uint32_t q = e >> 4;
                scale_add(acc, cl, dg, 8.0f * dg, dg8, 8.0f * dg8, sm.sx[q]);
                scale_add(acc, ch, dg * 0.0625f, 8.0f * dg, dg8 * 0.0625f, 8.0f * dg8, sm.sx[q + 1]);
            }
        }
    }
};

// ------------------------------------------------------------------ reductions

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Block-wide (sum of s, max of m) in one round.
__device__ void block_sum_max(float& s, float& m, float* red) {
    s = wsum(s);
    m = wmax(m);
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) { red[threadIdx.x >> 5] = s; red[kMWarps + (threadIdx.x >> 5)] = m; }
    __syncthreads();
    float ts = 0.f, tm = 0.f;
#pragma unroll
    for (int i = 0; i < kMWarps; i++) { ts += red[i]; tm = fmaxf(tm, red[kMWarps + i]); }
    s = ts;
    m = tm;
}

__device__ __forceinline__ float m_gelu(float x) {
    const float k0 = 0.79788456080286535587989211986876f, k1 = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(k0 * x * (1.0f + k1 * x * x)));
}
__device__ __forceinline__ unsigned long long m_key(float v, uint32_t idx) {
    if (v != v) return idx == 0 ? ~0ull : 0ull;
    if (v == 0.0f) v = 0.0f;
    const uint32_t b = __float_as_uint(v);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

// ------------------------------------------------------------------ prologue
// Stage the input vector: normalise (RMSNorm model.c:4-10 / LayerNorm
// gpt2.c:130-139), choose E with max|x| * 2^E < 2^14, write the fp16 hi/lo
// split and the scaled 16-element sums. Threads own runs of 16 elements; the
// loads of a run are issued together, so x costs one round trip.
__device__ void stage_x(const GemvArgs& a, const MmaSmem& sm, float* s_scale) {
    const uint32_t K = a.K, nrun = K / 16;
    float s = 0.f, m = 0.f;
    if (a.norm == NORM_LAYER) {
        // two-pass mean / variance like the reference
        for (uint32_t r = threadIdx.x; r < nrun; r += blockDim.x) {
            const float4* xp = reinterpret_cast<const float4*>(a.x + 16 * r);
            float4 v[4];
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = xp[i];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                reinterpret_cast<float4*>(sm.xf + 16 * r)[i] = v[i];
                s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
            }
        }
        block_sum_max(s, m, sm.red);
        const float mean = s / (float)K;
        float vs = 0.f;
        for (uint32_t r = threadIdx.x; r < nrun; r += blockDim.x)
            for (int i = 0; i < 16; i++) { const float c = sm.xf[16 * r + i] - mean; vs = fmaf(c, c, vs); }
        float dummy = 0.f;
        block_sum_max(vs, dummy, sm.red);
        const float inv = 1.0f / sqrtf(vs / (float)K + a.eps);
        m = 0.f;
        for (uint32_t r = threadIdx.x; r < nrun; r += blockDim.x) {
            for (int i = 0; i < 16; i++) {
                const uint32_t k = 16 * r + i;
                const float v = (sm.xf[k] - mean) * inv * a.norm_w[k] + a.norm_b[k];
                sm.xf[k] = v;
                m = fmaxf(m, fabsf(v));
            }
        }
        s = 0.f;
        block_sum_max(s, m, sm.red);
        s = 1.0f;                                  // xf already final
    } else {
        const bool rms = a.norm == NORM_RMS;
        for (uint32_t r = threadIdx.x; r < nrun; r += blockDim.x) {
            const float4* xp = reinterpret_cast<const float4*>(a.x + 16 * r);
            float4 v[4], w[4];
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = xp[i];
            if (rms) {
                const float4* wp = reinterpret_cast<const float4*>(a.norm_w + 16 * r);
#pragma unroll
                for (int i = 0; i < 4; i++) w[i] = wp[i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                float4 o = v[i];
                if (rms) {
                    s = fmaf(v[i].x, v[i].x, fmaf(v[i].y, v[i].y, fmaf(v[i].z, v[i].z, fmaf(v[i].w, v[i].w, s))));
                    o.x *= w[i].x; o.y *= w[i].y; o.z *= w[i].z; o.w *= w[i].w;
                }
                m = fmaxf(m, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
                reinterpret_cast<float4*>(sm.xf + 16 * r)[i] = o;
            }
        }
        block_sum_max(s, m, sm.red);
        // RMSNorm: xf holds x*w; the common factor 1/rms is applied below
        s = rms ? 1.0f / sqrtf(s / (float)K + a.eps) : 1.0f;
    }
    const float f = s;                             // factor still to apply to xf
    const float mx = m * f;
    int e = 0;
    if (mx > 0.f && mx < INFINITY) frexpf(mx, &e);
    const int E = 14 - e;
    for (uint32_t r = threadIdx.x; r < nrun; r += blockDim.x) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 t = reinterpret_cast<const float4*>(sm.xf + 16 * r)[i];
            v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
        }
        float sum = 0.f;
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            const float x0 = v[i] * f, x1 = v[i + 1] * f;
            sum += x0 + x1;
            const float s0 = ldexpf(x0, E), s1 = ldexpf(x1, E);
            const __half h0 = __float2half_rn(s0), h1 = __float2half_rn(s1);
            const __half l0 = __float2half_rn(s0 - __half2float(h0)), l1 = __float2half_rn(s1 - __half2float(h1));
            hw[i / 2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            lw[i / 2] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        uint4* hp = reinterpret_cast<uint4*>(sm.xh + 8 * r);
        uint4* lp = reinterpret_cast<uint4*>(sm.xl + 8 * r);
        hp[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        hp[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
        lp[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        lp[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
        sm.sx[r] = ldexpf(sum, E - 24);
    }
    if (threadIdx.x == 0) *s_scale = ldexpf(1.0f, 24 - E);
    __syncthreads();
}

// ------------------------------------------------------------------ tile runner

// Rows g and g+8 of one matrix: this warp takes iterations first, first+step,
// ... The first iteration's weights are loaded before waiting for the producer
// of x; afterwards one iteration of loads stays in flight.
template <class F>
__device__ __forceinline__ void run_tile(const GemvArgs& a, const uint8_t* w, uint64_t row_bytes, uint32_t ra,
                                         uint32_t rb, const Lane& L, uint32_t first, uint32_t step,
                                         const MmaSmem& sm, float* s_scale, float* acc) {
    const uint32_t K = a.K;
    const uint32_t nblk32 = K / 32;                        // only used by the 32-block formats
    const uint32_t nit = (K + F::SB - 1) / F::SB;
    const uint8_t* ga = w + (uint64_t)ra * row_bytes;
    const uint8_t* gb = w + (uint64_t)rb * row_bytes;
    auto nvalid = [&](uint32_t it) -> uint32_t { return F::SB == 256 ? 1u : min(4u, nblk32 - it * 4); };
    typename F::Raw r0;
    uint32_t it = first;
    if (it < nit) F::load(r0, ga + (uint64_t)it * F::SBB, gb + (uint64_t)it * F::SBB, nvalid(it), L);
    pdl_wait();                                            // x comes from the previous kernel
    stage_x(a, sm, s_scale);
    for (; it < nit; it += step) {
        typename F::Raw r1;
        const uint32_t nx = it + step;
        if (nx < nit) F::load(r1, ga + (uint64_t)nx * F::SBB, gb + (uint64_t)nx * F::SBB, nvalid(nx), L);
        F::compute(r0, it * F::SB, nvalid(it), L, sm, acc);
        r0 = r1;
    }
}

// ------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kMThreads)
gemv_mma_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float s_scale;
    pdl_trigger();
    const uint32_t K = a.K;
    MmaSmem sm;
    sm.xf = smem;
    sm.xh = reinterpret_cast<uint32_t*>(smem + K);
    sm.xl = sm.xh + K / 2;
    sm.sx = reinterpret_cast<float*>(sm.xl + K / 2);
    sm.red = sm.sx + K / 16;
    sm.part = sm.red + 2 * kMWarps;

    uint32_t s = 0;
#pragma unroll
    for (uint32_t i = 1; i < kMaxSegs; i++)
        if (i < a.nseg && blockIdx.x >= a.seg[i].tile0) s = i;
    const GemvSeg& G = a.seg[s];
    const uint32_t row0 = (blockIdx.x - G.tile0) * 16;
    const bool glu = G.epi == EPI_GLU_SILU || G.epi == EPI_GLU_GELU;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    Lane L;
    L.g = lane >> 2;
    L.tig = lane & 3u;
    L.bact = L.g < 2;
    L.xpart = L.g == 0 ? sm.xh : sm.xl;
    // rows past the end of the matrix read its last row; their results are dropped
    const uint32_t ra = min(row0 + L.g, G.rows - 1), rb = min(row0 + L.g + 8, G.rows - 1);

    // A gated tile gives the gate matrix to warps 0..3 and the up matrix to
    // warps 4..7; otherwise all 8 warps share the one matrix.
    const uint32_t half = kMWarps / 2;
    const bool up = glu && warp >= half;
    const uint8_t* wm = up ? G.w2 : G.w;
    const uint64_t rbytes = up ? G.row_bytes2 : G.row_bytes;
    const uint32_t first = glu ? warp % half : warp, step = glu ? half : kMWarps;
    float acc[2] = {0.f, 0.f};
    switch (G.type) {
    case T_Q4_K: run_tile<FQ4K>(a, wm, rbytes, ra, rb, L, first, step, sm, &s_scale, acc); break;
    case T_Q6_K: run_tile<FQ6K>(a, wm, rbytes, ra, rb, L, first, step, sm, &s_scale, acc); break;
    case T_Q8_0: run_tile<FQ80>(a, wm, rbytes, ra, rb, L, first, step, sm, &s_scale, acc); break;
    default:     run_tile<FQ40>(a, wm, rbytes, ra, rb, L, first, step, sm, &s_scale, acc); break;
    }

    if (L.tig == 0) {
        sm.part[warp * 16 + L.g] = acc[0];
        sm.part[warp * 16 + L.g + 8] = acc[1];
    }
    __syncthreads();

    // epilogue: thread r < 16 finishes row row0 + r
    unsigned long long key = 0ull;
    if (threadIdx.x < 16) {
        const uint32_t r = threadIdx.x, row = row0 + r;
        float v = 0.f, u = 0.f;
#pragma unroll
        for (uint32_t w = 0; w < kMWarps; w++) {
            if (glu && w >= half) u += sm.part[w * 16 + r];
            else v += sm.part[w * 16 + r];
        }
        v *= s_scale;
        u *= s_scale;
        if (row < G.rows) {
            switch (G.epi) {
            case EPI_STORE: if (G.bias) v += G.bias[row]; G.out[row] = v; break;
            case EPI_RESID: if (G.bias) v += G.bias[row]; G.out[row] += v; break;
            case EPI_GLU_SILU: v = v / (1.0f + expf(-v)) * u; G.out[row] = v; break;   // model.c:22
            case EPI_GLU_GELU: v = m_gelu(v) * u; G.out[row] = v; break;
            case EPI_GELU: if (G.bias) v += G.bias[row]; v = m_gelu(v); G.out[row] = v; break;
            }
            if (G.argmax) key = m_key(v, row);
        }
    }
    if (a.argmax_key != nullptr && warp == 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
            key = k2 > key ? k2 : key;
        }
        if (lane == 0 && key != 0ull) atomicMax(a.argmax_key, key);
    }
}

size_t gemv_mma_smem(uint32_t K) {
    // xf (4K) + xh, xl (2K each) + sx (K/4) bytes, then red and part
    return (size_t)K * 8 + (size_t)K / 16 * 4 + 2 * kMWarps * 4 + kMWarps * 2 * 16 * 4;
}

bool gemv_mma_init() {
    return LM_CUDA(cudaFuncSetAttribute(gemv_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
}

// Launch when every segment is a tensor-core format (and a gated pair shares
// one format); *handled = false otherwise, and the caller uses k_gemv.cu.
bool launch_gemv_mma(const GemvArgs& in, cudaStream_t st, bool* handled) {
    *handled = false;
    // the 32-block formats iterate in runs of 4 blocks, the last run may be partial
    if (in.K % 32 != 0) return true;
    for (uint32_t i = 0; i < in.nseg; i++) {
        const GemvSeg& g = in.seg[i];
        const bool glu = g.epi == EPI_GLU_SILU || g.epi == EPI_GLU_GELU;
        if (!mma_type(g.type) || (glu && g.type2 != g.type)) return true;
        if (type_bytes(g.type, in.K) == 0) return true;
    }
    if (in.norm != NORM_NONE && (reinterpret_cast<uintptr_t>(in.norm_w) % 16 != 0 ||
                                 (in.norm == NORM_LAYER && reinterpret_cast<uintptr_t>(in.norm_b) % 16 != 0)))
        return true;
    if (reinterpret_cast<uintptr_t>(in.x) % 16 != 0) return true;
    GemvArgs a = in;
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < a.nseg; i++) {
        a.seg[i].tile0 = tiles;
        tiles += (a.seg[i].rows + 15) / 16;
    }
    const size_t smem = gemv_mma_smem(a.K);
    if (smem > 200 * 1024) return true;
    *handled = true;
    return LM_CUDA(launch_k(gemv_mma_kernel, dim3(tiles), dim3(kMThreads), smem, st, a));
}

}  // namespace lm
