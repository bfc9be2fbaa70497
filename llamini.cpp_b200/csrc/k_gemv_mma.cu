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
    float* xf;          // staged x before the final scale (K floats)
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

// Lane roles. For the A operand lane (g, tig) supplies rows g and g+8 at the k
// slots of its tig. For B, lane (g, tig) supplies column g; the column pair
// (2s, 2s+1) of an MMA carries (x_hi, x_lo) of "slot" s (a group, scale group
// or block, depending on the format) and is zero in every other slot's MMA.
// Chaining the MMAs of 4 slots into one accumulator therefore leaves slot s's
// sums in the lanes with tig == s (accumulator columns 2tig, 2tig+1), so the
// four lanes of a quad apply the scales of four different slots in parallel.
struct Lane {
    uint32_t g, tig;
    uint32_t slot;             // g >> 1: the slot whose x this lane supplies
    const uint32_t* xpart;     // xh for even g (x_hi column), xl for odd g
};

struct BFrag { uint32_t b0, b1; };

// B values of this lane for elements e0..e0+3 (e0 % 4 == 0): k slots (2t, 2t+1)
// take elements (e0, e0+2), slots (2t+8, 2t+9) take (e0+1, e0+3), matching how
// the A pairs are cut from packed bytes.
__device__ __forceinline__ BFrag bfrag(const Lane& L, uint32_t e0) {
    const uint2 v = *reinterpret_cast<const uint2*>(L.xpart + (e0 >> 1));
    return BFrag{__byte_perm(v.x, v.y, 0x5410), __byte_perm(v.x, v.y, 0x7632)};
}
__device__ __forceinline__ BFrag bmask(const BFrag& f, uint32_t slot, uint32_t s) {
    const uint32_t m = slot == s ? 0xFFFFFFFFu : 0u;
    return BFrag{f.b0 & m, f.b1 & m};
}

// Exact small-integer to float (v < 2^23) without the conversion unit.
__device__ __forceinline__ float u2f(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.0f; }

// acc[0] (row g) and acc[1] (row g+8) += alpha * P - beta * S.
__device__ __forceinline__ void scale_add(float* acc, const float* c, float a_g, float b_g, float a_g8, float b_g8,
                                          float sx) {
    acc[0] = fmaf(a_g, c[0] + c[1], fmaf(-b_g, sx, acc[0]));
    acc[1] = fmaf(a_g8, c[2] + c[3], fmaf(-b_g8, sx, acc[1]));
}

// ------------------------------------------------------------------ formats
// Each format: Raw (the words one lane needs for one iteration of rows g and
// g+8), SB (elements per iteration), SBB (bytes per iteration), load(),
// compute().

// Q4_K (gguf.c:504-529): 256-element super-block, 4 groups of 64; in group j
// the low nibbles of qs[32j..32j+32) are sub-block 2j, the high nibbles 2j+1.
// Lane tig takes bytes 8tig..8tig+8 of each group (two MMAs per sub-block);
// slot = group.
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
    // scale and min of sub-blocks 2t and 2t+1 (gguf.c:391-399), all 16 six-bit
    // fields unpacked with word-wide masks
    static __device__ __forceinline__ void scales(const uint32_t* h, uint32_t t, float* sl, float* ml, float* sh,
                                                  float* mh) {
        const uint32_t lo = t < 2;
        const uint32_t wsc = lo ? (h[1] & 0x3F3F3F3Fu) : ((h[3] & 0x0F0F0F0Fu) | ((h[1] >> 2) & 0x30303030u));
        const uint32_t wm = lo ? (h[2] & 0x3F3F3F3Fu) : (((h[3] >> 4) & 0x0F0F0F0Fu) | ((h[2] >> 2) & 0x30303030u));
        const uint32_t sh16 = 16 * (t & 1);
        *sl = u2f((wsc >> sh16) & 0xFFu);
        *sh = u2f((wsc >> (sh16 + 8)) & 0xFFu);
        *ml = u2f((wm >> sh16) & 0xFFu);
        *mh = u2f((wm >> (sh16 + 8)) & 0xFFu);
    }
    static __device__ __forceinline__ void compute(const Raw& r, uint32_t e_blk, uint32_t, const Lane& L,
                                                   const MmaSmem& sm, float* acc) {
        const uint32_t eb = e_blk + 64 * L.slot + 8 * L.tig;
        const BFrag f00 = bfrag(L, eb), f01 = bfrag(L, eb + 4), f10 = bfrag(L, eb + 32), f11 = bfrag(L, eb + 36);
        float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t w0 = r.q[j].x, w1 = r.q[j].y, v0 = r.q8[j].x, v1 = r.q8[j].y;
            const uint32_t w0s = w0 >> 8, w1s = w1 >> 8, v0s = v0 >> 8, v1s = v1 >> 8;
            const BFrag b00 = bmask(f00, L.slot, j), b01 = bmask(f01, L.slot, j);
            const BFrag b10 = bmask(f10, L.slot, j), b11 = bmask(f11, L.slot, j);
            mma16816(cl, w0 & 0x000F000Fu, v0 & 0x000F000Fu, w0s & 0x000F000Fu, v0s & 0x000F000Fu, b00.b0, b00.b1);
            mma16816(cl, w1 & 0x000F000Fu, v1 & 0x000F000Fu, w1s & 0x000F000Fu, v1s & 0x000F000Fu, b01.b0, b01.b1);
            // high nibbles in place (16 q): alpha scaled by 1/16 below
            mma16816(ch, w0 & 0x00F000F0u, v0 & 0x00F000F0u, w0s & 0x00F000F0u, v0s & 0x00F000F0u, b10.b0, b10.b1);
            mma16816(ch, w1 & 0x00F000F0u, v1 & 0x00F000F0u, w1s & 0x00F000F0u, v1s & 0x00F000F0u, b11.b0, b11.b1);
        }
        // this lane: group tig of rows g and g+8
        float sl, ml, sh, mh, tl, nl, th, nh;
        scales(r.h, L.tig, &sl, &ml, &sh, &mh);
        scales(r.h8, L.tig, &tl, &nl, &th, &nh);
        const float dg = __half2float(__ushort_as_half((unsigned short)(r.h[0] & 0xFFFFu)));
        const float mg = __half2float(__ushort_as_half((unsigned short)(r.h[0] >> 16)));
        const float dg8 = __half2float(__ushort_as_half((unsigned short)(r.h8[0] & 0xFFFFu)));
        const float mg8 = __half2float(__ushort_as_half((unsigned short)(r.h8[0] >> 16)));
        const uint32_t q = (e_blk + 64 * L.tig) >> 4;
        const float sxl = sm.sx[q] + sm.sx[q + 1], sxh = sm.sx[q + 2] + sm.sx[q + 3];
        scale_add(acc, cl, dg * sl, mg * ml, dg8 * tl, mg8 * nl, sxl);
        scale_add(acc, ch, dg * sh * 0.0625f, mg * mh, dg8 * th * 0.0625f, mg8 * nh, sxh);
    }
};

// Q6_K (gguf.c:561-590): per 128-half H, byte l of ql[64H..], ql[64H+32..] and
// qh[32H..] give elements 128H + 32c + l (c = 0..3), scale sc[8H + l/16 + 2c].
// For each (H, u = l/16) the four scale groups c are one MMA each, slot = c.
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
        ld_words<4>(bg + 192, r.sc);
        ld_words<4>(bg8 + 192, r.sc8);
        r.d = ld_u16(bg + 208) | (ld_u16(bg8 + 208) << 16);
    }
    static __device__ __forceinline__ uint32_t word(uint32_t n, uint32_t hbits) { return (n & 0x0F0F0F0Fu) | hbits; }
    // signed scale byte i of the 16-byte field (i is lane dependent: words are
    // picked with selects, not a dynamically indexed array)
    static __device__ __forceinline__ float sbyte(const uint32_t* w, uint32_t i) {
        const uint32_t q = i >> 2;
        const uint32_t x = q == 0 ? w[0] : (q == 1 ? w[1] : (q == 2 ? w[2] : w[3]));
        return (float)(int)(int8_t)(uint8_t)((x >> (8 * (i & 3))) & 0xFFu);
    }
    static __device__ __forceinline__ void compute(const Raw& r, uint32_t e_blk, uint32_t, const Lane& L,
                                                   const MmaSmem& sm, float* acc) {
        const float dg = __half2float(__ushort_as_half((unsigned short)(r.d & 0xFFFFu)));
        const float dg8 = __half2float(__ushort_as_half((unsigned short)(r.d >> 16)));
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
                const BFrag f = bfrag(L, e_blk + 128 * H + 32 * L.slot + 16 * u + 4 * L.tig);
                float cc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const BFrag b = bmask(f, L.slot, c);
                    mma16816(cc, __byte_perm(wq[c], 0, 0x4240), __byte_perm(wm[c], 0, 0x4240),
                             __byte_perm(wq[c], 0, 0x4341), __byte_perm(wm[c], 0, 0x4341), b.b0, b.b1);
                }
                // this lane: scale group c = tig of rows g, g+8
                const uint32_t si = 8 * H + u + 2 * L.tig;
                const float ag = dg * sbyte(r.sc, si), ag8 = dg8 * sbyte(r.sc8, si);
                scale_add(acc, cc, ag, 32.0f * ag, ag8, 32.0f * ag8,
                          sm.sx[(e_blk + 128 * H + 32 * L.tig + 16 * u) >> 4]);
            }
        }
    }
};

// 32-element formats, 4 blocks per iteration (slot = block; the last iteration
// of a row may hold fewer blocks).
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
        const uint32_t es = e_blk + 32 * L.slot + 4 * L.tig;
        const BFrag f0 = L.slot < nvalid ? bfrag(L, es) : BFrag{0u, 0u};
        const BFrag f1 = L.slot < nvalid ? bfrag(L, es + 16) : BFrag{0u, 0u};
        float cc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k >= nvalid) break;
            const BFrag b0 = bmask(f0, L.slot, k), b1 = bmask(f1, L.slot, k);
            const uint32_t w = r.w[k][0] ^ 0x80808080u, v = r.v[k][0] ^ 0x80808080u;
            const uint32_t w2 = r.w[k][1] ^ 0x80808080u, v2 = r.v[k][1] ^ 0x80808080u;
            mma16816(cc, __byte_perm(w, 0, 0x4240), __byte_perm(v, 0, 0x4240),
                     __byte_perm(w, 0, 0x4341), __byte_perm(v, 0, 0x4341), b0.b0, b0.b1);
            mma16816(cc, __byte_perm(w2, 0, 0x4240), __byte_perm(v2, 0, 0x4240),
                     __byte_perm(w2, 0, 0x4341), __byte_perm(v2, 0, 0x4341), b1.b0, b1.b1);
        }
        if (L.tig < nvalid) {
            uint32_t dd = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) if ((uint32_t)k == L.tig) dd = r.d[k];
            const float dg = __half2float(__ushort_as_half((unsigned short)(dd & 0xFFFFu)));
            const float dg8 = __half2float(__ushort_as_half((unsigned short)(dd >> 16)));
            const uint32_t q = (e_blk + 32 * L.tig) >> 4;
            scale_add(acc, cc, dg, 128.0f * dg, dg8, 128.0f * dg8, sm.sx[q] + sm.sx[q + 1]);
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
        const uint32_t es = e_blk + 32 * L.slot + 4 * L.tig;
        const BFrag fl = L.slot < nvalid ? bfrag(L, es) : BFrag{0u, 0u};
        const BFrag fh = L.slot < nvalid ? bfrag(L, es + 16) : BFrag{0u, 0u};
        float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k >= nvalid) break;
            const uint32_t w = r.w[k], v = r.v[k], ws = w >> 8, vs = v >> 8;
            const BFrag bl = bmask(fl, L.slot, k), bh = bmask(fh, L.slot, k);
            mma16816(cl, w & 0x000F000Fu, v & 0x000F000Fu, ws & 0x000F000Fu, vs & 0x000F000Fu, bl.b0, bl.b1);
            mma16816(ch, w & 0x00F000F0u, v & 0x00F000F0u, ws & 0x00F000F0u, vs & 0x00F000F0u, bh.b0, bh.b1);
        }
        if (L.tig < nvalid) {
            uint32_t dd = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) if ((uint32_t)k == L.tig) dd = r.d[k];
            const float dg = __half2float(__ushort_as_half((unsigned short)(dd & 0xFFFFu)));
            const float dg8 = __half2float(__ushort_as_half((unsigned short)(dd >> 16)));
            const uint32_t q = (e_blk + 32 * L.tig) >> 4;
            scale_add(acc, cl, dg, 8.0f * dg, dg8, 8.0f * dg8, sm.sx[q]);
            scale_add(acc, ch, dg * 0.0625f, 8.0f * dg, dg8 * 0.0625f, 8.0f * dg8, sm.sx[q + 1]);
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
// gpt2.c:130-139), choose E with max|x| 2^E < 2^14, write the fp16 hi/lo split
// and the scaled 16-element sums. Thread t owns float4s t, t+256, ...; all its
// loads are issued before any is used, so x costs one round trip.
__device__ void stage_x(const GemvArgs& a, const MmaSmem& sm, float* s_scale) {
    const uint32_t K = a.K, n4 = K / 4, tid = threadIdx.x;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    float4* xf4 = reinterpret_cast<float4*>(sm.xf);
    float s = 0.f, m = 0.f, f = 1.0f;
    // pass 1: x (times the RMSNorm weight) into shared memory, sum of squares, max
    if (a.norm == NORM_RMS) {
        const float4* w4 = reinterpret_cast<const float4*>(a.norm_w);
#pragma unroll 4
        for (uint32_t i = tid; i < n4; i += kMThreads) {
            const float4 v = x4[i], w = w4[i];
            s = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, s))));
            const float4 o = make_float4(v.x * w.x, v.y * w.y, v.z * w.z, v.w * w.w);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
            xf4[i] = o;
        }
        block_sum_max(s, m, sm.red);
        f = 1.0f / sqrtf(s / (float)K + a.eps);    // model.c:7-8; applied to x*w below
    } else if (a.norm == NORM_LAYER) {
#pragma unroll 4
        for (uint32_t i = tid; i < n4; i += kMThreads) {
            const float4 v = x4[i];
            s += (v.x + v.y) + (v.z + v.w);
            xf4[i] = v;
        }
        block_sum_max(s, m, sm.red);
        const float mean = s / (float)K;          // two passes like gpt2.c:131-136
        float vs = 0.f;
        for (uint32_t i = tid; i < n4; i += kMThreads) {
            const float4 v = xf4[i];
            const float c0 = v.x - mean, c1 = v.y - mean, c2 = v.z - mean, c3 = v.w - mean;
            vs = fmaf(c0, c0, fmaf(c1, c1, fmaf(c2, c2, fmaf(c3, c3, vs))));
        }
        float dummy = 0.f;
        block_sum_max(vs, dummy, sm.red);
        const float inv = 1.0f / sqrtf(vs / (float)K + a.eps);
        const float4* w4 = reinterpret_cast<const float4*>(a.norm_w);
        const float4* b4 = reinterpret_cast<const float4*>(a.norm_b);
        m = 0.f;
#pragma unroll 4
        for (uint32_t i = tid; i < n4; i += kMThreads) {
            const float4 v = xf4[i], w = w4[i], b = b4[i];
            const float4 o = make_float4((v.x - mean) * inv * w.x + b.x, (v.y - mean) * inv * w.y + b.y,
                                         (v.z - mean) * inv * w.z + b.z, (v.w - mean) * inv * w.w + b.w);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
            xf4[i] = o;
        }
        float ds = 0.f;
        block_sum_max(ds, m, sm.red);
    } else {
#pragma unroll 4
        for (uint32_t i = tid; i < n4; i += kMThreads) {
            const float4 v = x4[i];
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            xf4[i] = v;
        }
        float ds = 0.f;
        block_sum_max(ds, m, sm.red);
    }
    // pass 2: x_final = xf * f, scaled by 2^E so that max|x| 2^E < 2^14
    const float mx = m * f;
    int e = 0;
    if (mx > 0.f && mx < INFINITY) frexpf(mx, &e);
    int E = 14 - e;
    E = E > 100 ? 100 : (E < -100 ? -100 : E);
    const float F = f * __int_as_float((E + 127) << 23);
    // each lane takes whole float4s; the runs of 16 are 4 consecutive lanes
    const uint32_t n4r = (n4 + 31u) & ~31u;            // whole warps in the loop
    for (uint32_t i = tid; i < n4r; i += kMThreads) {
        const float4 v = i < n4 ? xf4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float x0 = v.x * F, x1 = v.y * F, x2 = v.z * F, x3 = v.w * F;
        const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
        const __half h2 = __float2half_rn(x2), h3 = __float2half_rn(x3);
        const __half l0 = __float2half_rn(x0 - __half2float(h0)), l1 = __float2half_rn(x1 - __half2float(h1));
        const __half l2 = __float2half_rn(x2 - __half2float(h2)), l3 = __float2half_rn(x3 - __half2float(h3));
        float rs = ((x0 + x1) + (x2 + x3)) * 5.9604644775390625e-08f;     // units of 2^(E-24)
        rs += __shfl_xor_sync(0xffffffffu, rs, 1);
        rs += __shfl_xor_sync(0xffffffffu, rs, 2);
        if (i < n4) {
            *reinterpret_cast<uint2*>(sm.xh + 2 * i) =
                make_uint2((uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16),
                           (uint32_t)__half_as_ushort(h2) | ((uint32_t)__half_as_ushort(h3) << 16));
            *reinterpret_cast<uint2*>(sm.xl + 2 * i) =
                make_uint2((uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16),
                           (uint32_t)__half_as_ushort(l2) | ((uint32_t)__half_as_ushort(l3) << 16));
            if ((i & 3u) == 0) sm.sx[i >> 2] = rs;
        }
    }
    if (tid == 0) *s_scale = __int_as_float((127 + 24 - E) << 23);   // 2^(24-E)
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
    L.slot = L.g >> 1;
    L.xpart = (L.g & 1u) ? sm.xl : sm.xh;
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
    // xf (4K bytes), xh, xl (2K bytes each), sx (K/4 bytes), then red and part
    return (size_t)K * 8 + (size_t)K / 16 * 4 + 2 * kMWarps * 4 + kMWarps * 16 * 4;
}

bool gemv_mma_init() {
    return LM_CUDA(cudaFuncSetAttribute(gemv_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(gemv_mma_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
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
