// mma_gemv.cuh -- building blocks of the tensor-core dequant-GEMV, shared by
// the per-matrix kernel (k_gemv_mma.cu) and the persistent decode-step kernel
// (k_decode.cu): mbarrier/bulk-copy helpers, the m16n8k16 fragment layout with
// "slot" columns, and the per-format tile compute for Q4_K, Q6_K, Q8_0, Q4_0, Q4_1, Q5_0.
//
// Every block format is affine per group of 16 or 32 weights,
//     w = alpha * q - beta      (q a small unsigned integer, gguf.c:427-590),
// so sum_i w_i x_i = alpha * sum_i q_i x_i - beta * sum_i x_i. The integers enter
// the A operand as exact fp16 subnormals (q * 2^-24), x enters B as an fp16
// hi/lo pair after scaling by a power of two, accumulation is f32; alpha, beta
// and the 16-element sums of x are applied in f32 afterwards.
#pragma once

#include "internal.h"
#include "quant.cuh"

#include <cuda_fp16.h>

namespace lm {

constexpr uint32_t kMaxWait = 1u << 26;      // polls of an mbarrier before giving up

// ------------------------------------------------------------------ TMA / mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// this GPU's global memory into this CTA's shared memory. No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// Bounded wait for the phase with the given parity; false if it never came.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t i = 0; i < kMaxWait; i++) {
        uint32_t done;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                     " selp.u32 %0, 1, 0, p;\n}\n" : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

// ------------------------------------------------------------------ MMA helpers

struct MmaSmem {
    float* xf;          // staged x before the final scale (K floats)
    uint32_t* xh;       // x * 2^E as fp16 pairs, high part   (K/2 words)
    uint32_t* xl;       // low part
    float* sx;          // per 16-element run: sum(x) * 2^(E-24)
    float* red;         // [2 * warps] reduction scratch
    float* part;        // [warps][16] partial row sums
};

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Lane roles. For A, lane (g, tig) supplies rows g and g+8 at the k slots of
// its tig. For B, lane (g, tig) supplies column g: column pair (2s, 2s+1) of
// an MMA carries (x_hi, x_lo) of slot s and is zero in other slots' MMAs.
struct Lane {
    uint32_t g, tig;
    uint32_t slot;             // g >> 1: the slot whose x this lane supplies
    const uint32_t* xpart;     // xh for even g (x_hi column), xl for odd g
};

struct BFrag { uint32_t b0, b1; };

// B values for elements e0..e0+3 (e0 % 4 == 0): k slots (2t, 2t+1) take
// elements (e0, e0+2), slots (2t+8, 2t+9) take (e0+1, e0+3), matching how the
// A pairs are cut from packed bytes.
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
__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }

// acc[0] (row g) and acc[1] (row g+8) += alpha * P - beta * S.
__device__ __forceinline__ void scale_add(float* acc, const float* c, float a_g, float b_g, float a_g8, float b_g8,
                                          float sx) {
    acc[0] = fmaf(a_g, c[0] + c[1], fmaf(-b_g, sx, acc[0]));
    acc[1] = fmaf(a_g8, c[2] + c[3], fmaf(-b_g8, sx, acc[1]));
}

// Shared-memory word loads at any 2-byte alignment (funnel shift of the two
// aligned words around the address; the stage buffer has slack at its end).
__device__ __forceinline__ uint32_t lds_u32(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t s = (uint32_t)(a & 3u) * 8u;
    const uint32_t lo = w[0];
    return s ? __funnelshift_r(lo, w[1], s) : lo;
}
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return lds_u32(p) & 0xFFFFu; }

// ------------------------------------------------------------------ formats
// compute(bg, bg8, e_blk, nvalid, L, sm, acc): one iteration (SB elements) of
// rows g (bytes at bg) and g+8 (bg8), both in shared memory.

// Q4_K (gguf.c:504-529): 256-element super-block, 4 groups of 64; in group j
// the low nibbles of qs[32j..32j+32) are sub-block 2j, the high nibbles 2j+1.
// Lane tig takes bytes 8tig..8tig+8 of each group; slot = group.
struct FQ4K {
    static constexpr uint32_t SB = 256, SBB = 144;
    // scale and min of sub-blocks 2t and 2t+1 (gguf.c:391-399): all 16 six-bit
    // fields unpacked with word-wide masks, then the pair for group t picked
    static __device__ __forceinline__ void scales(uint32_t s0, uint32_t s1, uint32_t s2, uint32_t t, float* sl,
                                                  float* ml, float* sh, float* mh) {
        const bool lo = t < 2;
        const uint32_t wsc = lo ? (s0 & 0x3F3F3F3Fu) : ((s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u));
        const uint32_t wm = lo ? (s1 & 0x3F3F3F3Fu) : (((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u));
        const uint32_t sh16 = 16 * (t & 1);
        *sl = u2f((wsc >> sh16) & 0xFFu);
        *sh = u2f((wsc >> (sh16 + 8)) & 0xFFu);
        *ml = u2f((wm >> sh16) & 0xFFu);
        *mh = u2f((wm >> (sh16 + 8)) & 0xFFu);
    }
    static __device__ __forceinline__ void compute(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk, uint32_t,
                                                   const Lane& L, const MmaSmem& sm, float* acc) {
        const uint4 h = *reinterpret_cast<const uint4*>(bg), h8 = *reinterpret_cast<const uint4*>(bg8);
        const uint32_t eb = e_blk + 64 * L.slot + 8 * L.tig;
        const BFrag f00 = bfrag(L, eb), f01 = bfrag(L, eb + 4), f10 = bfrag(L, eb + 32), f11 = bfrag(L, eb + 36);
        float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint2 q = *reinterpret_cast<const uint2*>(bg + 16 + 32 * j + 8 * L.tig);
            const uint2 q8 = *reinterpret_cast<const uint2*>(bg8 + 16 + 32 * j + 8 * L.tig);
            const uint32_t w0 = q.x, w1 = q.y, v0 = q8.x, v1 = q8.y;
            const uint32_t w0s = w0 >> 8, w1s = w1 >> 8, v0s = v0 >> 8, v1s = v1 >> 8;
            const BFrag b00 = bmask(f00, L.slot, j), b01 = bmask(f01, L.slot, j);
            const BFrag b10 = bmask(f10, L.slot, j), b11 = bmask(f11, L.slot, j);
            mma16816(cl, w0 & 0x000F000Fu, v0 & 0x000F000Fu, w0s & 0x000F000Fu, v0s & 0x000F000Fu, b00.b0, b00.b1);
            mma16816(cl, w1 & 0x000F000Fu, v1 & 0x000F000Fu, w1s & 0x000F000Fu, v1s & 0x000F000Fu, b01.b0, b01.b1);
            // high nibbles in place (16 q): alpha scaled by 1/16 below
            mma16816(ch, w0 & 0x00F000F0u, v0 & 0x00F000F0u, w0s & 0x00F000F0u, v0s & 0x00F000F0u, b10.b0, b10.b1);
            mma16816(ch, w1 & 0x00F000F0u, v1 & 0x00F000F0u, w1s & 0x00F000F0u, v1s & 0x00F000F0u, b11.b0, b11.b1);
        }
        float sl, ml, sh, mh, tl, nl, th, nh;
        scales(h.y, h.z, h.w, L.tig, &sl, &ml, &sh, &mh);
        scales(h8.y, h8.z, h8.w, L.tig, &tl, &nl, &th, &nh);
        const float dg = h2f(h.x & 0xFFFFu), mg = h2f(h.x >> 16);
        const float dg8 = h2f(h8.x & 0xFFFFu), mg8 = h2f(h8.x >> 16);
        const uint32_t q = (e_blk + 64 * L.tig) >> 4;
        const float sxl = sm.sx[q] + sm.sx[q + 1], sxh = sm.sx[q + 2] + sm.sx[q + 3];
        scale_add(acc, cl, dg * sl, mg * ml, dg8 * tl, mg8 * nl, sxl);
        scale_add(acc, ch, dg * sh * 0.0625f, mg * mh, dg8 * th * 0.0625f, mg8 * nh, sxh);
    }
};

// Q5_K (gguf.c:530-560): Q4_K's layout (d, dmin, 12 scale bytes) with qh[32]
// before qs[128]: bit 2j of qh[l] is the fifth bit of element 64j + l, bit
// 2j + 1 that of 64j + 32 + l. The bits are merged into the fp16 halves (bit 4
// under a low nibble, bit 8 under a high nibble kept in place as 16 q).
struct FQ5K {
    static constexpr uint32_t SB = 256, SBB = 176;
    static __device__ __forceinline__ void compute(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk, uint32_t,
                                                   const Lane& L, const MmaSmem& sm, float* acc) {
        const uint4 h = *reinterpret_cast<const uint4*>(bg), h8 = *reinterpret_cast<const uint4*>(bg8);
        const uint2 hq = *reinterpret_cast<const uint2*>(bg + 16 + 8 * L.tig);
        const uint2 hq8 = *reinterpret_cast<const uint2*>(bg8 + 16 + 8 * L.tig);
        const uint32_t eb = e_blk + 64 * L.slot + 8 * L.tig;
        const BFrag f00 = bfrag(L, eb), f01 = bfrag(L, eb + 4), f10 = bfrag(L, eb + 32), f11 = bfrag(L, eb + 36);
        float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
        constexpr uint32_t L4 = 0x000F000Fu, H4 = 0x00F000F0u, B1 = 0x01010101u;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint2 q = *reinterpret_cast<const uint2*>(bg + 48 + 32 * j + 8 * L.tig);
            const uint2 q8 = *reinterpret_cast<const uint2*>(bg8 + 48 + 32 * j + 8 * L.tig);
            const uint32_t w0 = q.x, w1 = q.y, v0 = q8.x, v1 = q8.y;
            const uint32_t w0s = w0 >> 8, w1s = w1 >> 8, v0s = v0 >> 8, v1s = v1 >> 8;
            // fifth bits of bytes 0..3 of each word at bits 0, 8, 16, 24
            const uint32_t lw0 = (hq.x >> (2 * j)) & B1, lw1 = (hq.y >> (2 * j)) & B1;
            const uint32_t lv0 = (hq8.x >> (2 * j)) & B1, lv1 = (hq8.y >> (2 * j)) & B1;
            const uint32_t uw0 = (hq.x >> (2 * j + 1)) & B1, uw1 = (hq.y >> (2 * j + 1)) & B1;
            const uint32_t uv0 = (hq8.x >> (2 * j + 1)) & B1, uv1 = (hq8.y >> (2 * j + 1)) & B1;
            const BFrag b00 = bmask(f00, L.slot, j), b01 = bmask(f01, L.slot, j);
            const BFrag b10 = bmask(f10, L.slot, j), b11 = bmask(f11, L.slot, j);
            // low nibbles: bytes 0, 2 (bits 0, 16 -> 4, 20), bytes 1, 3 (bits 8, 24 -> 4, 20)
            mma16816(cl, (w0 & L4) | ((lw0 << 4) & 0x00100010u), (v0 & L4) | ((lv0 << 4) & 0x00100010u),
                     (w0s & L4) | ((lw0 >> 4) & 0x00100010u), (v0s & L4) | ((lv0 >> 4) & 0x00100010u), b00.b0, b00.b1);
            mma16816(cl, (w1 & L4) | ((lw1 << 4) & 0x00100010u), (v1 & L4) | ((lv1 << 4) & 0x00100010u),
                     (w1s & L4) | ((lw1 >> 4) & 0x00100010u), (v1s & L4) | ((lv1 >> 4) & 0x00100010u), b01.b0, b01.b1);
            // high nibbles in place (16 q): bytes 0, 2 (bits 0, 16 -> 8, 24), bytes 1, 3 (bits 8, 24 stay)
            mma16816(ch, (w0 & H4) | ((uw0 << 8) & 0x01000100u), (v0 & H4) | ((uv0 << 8) & 0x01000100u),
                     (w0s & H4) | (uw0 & 0x01000100u), (v0s & H4) | (uv0 & 0x01000100u), b10.b0, b10.b1);
            mma16816(ch, (w1 & H4) | ((uw1 << 8) & 0x01000100u), (v1 & H4) | ((uv1 << 8) & 0x01000100u),
                     (w1s & H4) | (uw1 & 0x01000100u), (v1s & H4) | (uv1 & 0x01000100u), b11.b0, b11.b1);
        }
        float sl, ml, sh, mh, tl, nl, th, nh;
        FQ4K::scales(h.y, h.z, h.w, L.tig, &sl, &ml, &sh, &mh);
        FQ4K::scales(h8.y, h8.z, h8.w, L.tig, &tl, &nl, &th, &nh);
        const float dg = h2f(h.x & 0xFFFFu), mg = h2f(h.x >> 16);
        const float dg8 = h2f(h8.x & 0xFFFFu), mg8 = h2f(h8.x >> 16);
        const uint32_t q = (e_blk + 64 * L.tig) >> 4;
        const float sxl = sm.sx[q] + sm.sx[q + 1], sxh = sm.sx[q + 2] + sm.sx[q + 3];
        scale_add(acc, cl, dg * sl, mg * ml, dg8 * tl, mg8 * nl, sxl);
        scale_add(acc, ch, dg * sh * 0.0625f, mg * mh, dg8 * th * 0.0625f, mg8 * nh, sxh);
    }
};

// Q6_K (gguf.c:561-590): per 128-half H, byte l of ql[64H..], ql[64H+32..] and
// qh[32H..] give elements 128H + 32c + l (c = 0..3), scale sc[8H + l/16 + 2c].
// For each (H, u = l/16) the four scale groups c are one MMA each, slot = c.
struct FQ6K {
    static constexpr uint32_t SB = 256, SBB = 210;
    static __device__ __forceinline__ uint32_t word(uint32_t n, uint32_t hbits) { return (n & 0x0F0F0F0Fu) | hbits; }
    static __device__ __forceinline__ void compute(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk, uint32_t,
                                                   const Lane& L, const MmaSmem& sm, float* acc) {
        const float dg = h2f(lds_u16(bg + 208)), dg8 = h2f(lds_u16(bg8 + 208));
#pragma unroll
        for (int H = 0; H < 2; H++) {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const uint32_t off = 16 * u + 4 * L.tig;
                const uint32_t a = lds_u32(bg + 64 * H + off), b = lds_u32(bg + 64 * H + 32 + off);
                const uint32_t hq = lds_u32(bg + 128 + 32 * H + off);
                const uint32_t a8 = lds_u32(bg8 + 64 * H + off), b8 = lds_u32(bg8 + 64 * H + 32 + off);
                const uint32_t h8 = lds_u32(bg8 + 128 + 32 * H + off);
                uint32_t wq[4], wm[4];
                wq[0] = word(a, (hq << 4) & 0x30303030u);
                wq[1] = word(b, (hq << 2) & 0x30303030u);
                wq[2] = word(a >> 4, hq & 0x30303030u);
                wq[3] = word(b >> 4, (hq >> 2) & 0x30303030u);
                wm[0] = word(a8, (h8 << 4) & 0x30303030u);
                wm[1] = word(b8, (h8 << 2) & 0x30303030u);
                wm[2] = word(a8 >> 4, h8 & 0x30303030u);
                wm[3] = word(b8 >> 4, (h8 >> 2) & 0x30303030u);
                const BFrag f = bfrag(L, e_blk + 128 * H + 32 * L.slot + 16 * u + 4 * L.tig);
                float cc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const BFrag bb = bmask(f, L.slot, c);
                    mma16816(cc, __byte_perm(wq[c], 0, 0x4240), __byte_perm(wm[c], 0, 0x4240),
                             __byte_perm(wq[c], 0, 0x4341), __byte_perm(wm[c], 0, 0x4341), bb.b0, bb.b1);
                }
                // this lane: scale group c = tig of rows g, g+8
                const uint32_t si = 192 + 8 * H + u + 2 * L.tig;
                const float ag = dg * (float)(int8_t)bg[si], ag8 = dg8 * (float)(int8_t)bg8[si];
                scale_add(acc, cc, ag, 32.0f * ag, ag8, 32.0f * ag8,
                          sm.sx[(e_blk + 128 * H + 32 * L.tig + 16 * u) >> 4]);
            }
        }
    }
};

// 32-element formats, 4 blocks per iteration (slot = block; the last
// iteration of a row may hold fewer blocks).
// Q8_0 (gguf.c:489-503): w = d q, q int8; with u = q ^ 0x80, w = d u - 128 d.
struct FQ80 {
    static constexpr uint32_t SB = 128, SBB = 136, BB = 34;
    static __device__ __forceinline__ void compute(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk,
                                                   uint32_t nvalid, const Lane& L, const MmaSmem& sm, float* acc) {
        const uint32_t es = e_blk + 32 * L.slot + 4 * L.tig;
        const BFrag f0 = L.slot < nvalid ? bfrag(L, es) : BFrag{0u, 0u};
        const BFrag f1 = L.slot < nvalid ? bfrag(L, es + 16) : BFrag{0u, 0u};
        float cc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k >= nvalid) break;
            const uint8_t* p = bg + k * BB + 2 + 4 * L.tig;
            const uint8_t* q = bg8 + k * BB + 2 + 4 * L.tig;
            const uint32_t w = lds_u32(p) ^ 0x80808080u, v = lds_u32(q) ^ 0x80808080u;
            const uint32_t w2 = lds_u32(p + 16) ^ 0x80808080u, v2 = lds_u32(q + 16) ^ 0x80808080u;
            const BFrag b0 = bmask(f0, L.slot, k), b1 = bmask(f1, L.slot, k);
            mma16816(cc, __byte_perm(w, 0, 0x4240), __byte_perm(v, 0, 0x4240),
                     __byte_perm(w, 0, 0x4341), __byte_perm(v, 0, 0x4341), b0.b0, b0.b1);
            mma16816(cc, __byte_perm(w2, 0, 0x4240), __byte_perm(v2, 0, 0x4240),
                     __byte_perm(w2, 0, 0x4341), __byte_perm(v2, 0, 0x4341), b1.b0, b1.b1);
        }
        if (L.tig < nvalid) {
            const float dg = h2f(lds_u16(bg + L.tig * BB)), dg8 = h2f(lds_u16(bg8 + L.tig * BB));
            const uint32_t q = (e_blk + 32 * L.tig) >> 4;
            scale_add(acc, cc, dg, 128.0f * dg, dg8, 128.0f * dg8, sm.sx[q] + sm.sx[q + 1]);
        }
    }
};

// Q4_0 (gguf.c:427-444): w = (q - 8) d; low nibbles are elements 0..15, high
// nibbles 16..31.
struct FQ40 {
    static constexpr uint32_t SB = 128, SBB = 72, BB = 18;
    static __device__ __forceinline__ void compute(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk,
                                                   uint32_t nvalid, const Lane& L, const MmaSmem& sm, float* acc) {
        const uint32_t es = e_blk + 32 * L.slot + 4 * L.tig;
        const BFrag fl = L.slot < nvalid ? bfrag(L, es) : BFrag{0u, 0u};
        const BFrag fh = L.slot < nvalid ? bfrag(L, es + 16) : BFrag{0u, 0u};
        float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k >= nvalid) break;
            const uint32_t w = lds_u32(bg + k * BB + 2 + 4 * L.tig), v = lds_u32(bg8 + k * BB + 2 + 4 * L.tig);
            const uint32_t ws = w >> 8, vs = v >> 8;
            const BFrag bl = bmask(fl, L.slot, k), bh = bmask(fh, L.slot, k);
            mma16816(cl, w & 0x000F000Fu, v & 0x000F000Fu, ws & 0x000F000Fu, vs & 0x000F000Fu, bl.b0, bl.b1);
            mma16816(ch, w & 0x00F000F0u, v & 0x00F000F0u, ws & 0x00F000F0u, vs & 0x00F000F0u, bh.b0, bh.b1);
        }
        if (L.tig < nvalid) {
            const float dg = h2f(lds_u16(bg + L.tig * BB)), dg8 = h2f(lds_u16(bg8 + L.tig * BB));
            const uint32_t q = (e_blk + 32 * L.tig) >> 4;
            scale_add(acc, cl, dg, 8.0f * dg, dg8, 8.0f * dg8, sm.sx[q]);
            scale_add(acc, ch, dg * 0.0625f, 8.0f * dg, dg8 * 0.0625f, 8.0f * dg8, sm.sx[q + 1]);
        }
    }
};

// Q4_1 (gguf.c:445-462): w = d q + m; nibbles as Q4_0, qs after d and m.
struct FQ41 {
    static constexpr uint32_t SB = 128, SBB = 80, BB = 20;
    static __device__ __forceinline__ void compute(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk,
                                                   uint32_t nvalid, const Lane& L, const MmaSmem& sm, float* acc) {
        const uint32_t es = e_blk + 32 * L.slot + 4 * L.tig;
        const BFrag fl = L.slot < nvalid ? bfrag(L, es) : BFrag{0u, 0u};
        const BFrag fh = L.slot < nvalid ? bfrag(L, es + 16) : BFrag{0u, 0u};
        float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k >= nvalid) break;
            const uint32_t w = lds_u32(bg + k * BB + 4 + 4 * L.tig), v = lds_u32(bg8 + k * BB + 4 + 4 * L.tig);
            const uint32_t ws = w >> 8, vs = v >> 8;
            const BFrag bl = bmask(fl, L.slot, k), bh = bmask(fh, L.slot, k);
            mma16816(cl, w & 0x000F000Fu, v & 0x000F000Fu, ws & 0x000F000Fu, vs & 0x000F000Fu, bl.b0, bl.b1);
            mma16816(ch, w & 0x00F000F0u, v & 0x00F000F0u, ws & 0x00F000F0u, vs & 0x00F000F0u, bh.b0, bh.b1);
        }
        if (L.tig < nvalid) {
            const uint32_t h = lds_u32(bg + L.tig * BB), h8 = lds_u32(bg8 + L.tig * BB);
            const float dg = h2f(h & 0xFFFFu), mg = h2f(h >> 16), dg8 = h2f(h8 & 0xFFFFu), mg8 = h2f(h8 >> 16);
            const uint32_t q = (e_blk + 32 * L.tig) >> 4;
            scale_add(acc, cl, dg, -mg, dg8, -mg8, sm.sx[q]);
            scale_add(acc, ch, dg * 0.0625f, -mg, dg8 * 0.0625f, -mg8, sm.sx[q + 1]);
        }
    }
};

// Q5_0 (gguf.c:463-488): w = (q - 16) d, q = nibble | (bit e of qh) << 4; low
// nibbles are elements 0..15, high nibbles 16..31. The fifth bit is merged
// into each fp16 half: bit 4 under a low nibble, bit 8 under a high nibble kept
// in place (16 q).
struct FQ50 {
    static constexpr uint32_t SB = 128, SBB = 88, BB = 22;
    static __device__ __forceinline__ uint32_t lo_even(uint32_t w, uint32_t h) {   // elements e, e + 2
        return (w & 0x000F000Fu) | ((h << 4) & 0x10u) | ((h << 18) & 0x100000u);
    }
    static __device__ __forceinline__ uint32_t lo_odd(uint32_t ws, uint32_t h) {   // elements e + 1, e + 3
        return (ws & 0x000F000Fu) | ((h << 3) & 0x10u) | ((h << 17) & 0x100000u);
    }
    static __device__ __forceinline__ uint32_t hi_even(uint32_t w, uint32_t h) {
        return (w & 0x00F000F0u) | ((h << 8) & 0x100u) | ((h << 22) & 0x1000000u);
    }
    static __device__ __forceinline__ uint32_t hi_odd(uint32_t ws, uint32_t h) {
        return (ws & 0x00F000F0u) | ((h << 7) & 0x100u) | ((h << 21) & 0x1000000u);
    }
    static __device__ __forceinline__ void compute(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk,
                                                   uint32_t nvalid, const Lane& L, const MmaSmem& sm, float* acc) {
        const uint32_t es = e_blk + 32 * L.slot + 4 * L.tig;
        const BFrag fl = L.slot < nvalid ? bfrag(L, es) : BFrag{0u, 0u};
        const BFrag fh = L.slot < nvalid ? bfrag(L, es + 16) : BFrag{0u, 0u};
        float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k >= nvalid) break;
            const uint8_t* p = bg + k * BB;
            const uint8_t* r = bg8 + k * BB;
            const uint32_t w = lds_u32(p + 6 + 4 * L.tig), v = lds_u32(r + 6 + 4 * L.tig);
            // high bits of this lane's elements: bits 0..3 = 4 tig .. 4 tig + 3, bits 16..19 = 16 + those
            const uint32_t hw = lds_u32(p + 2) >> (4 * L.tig), hv = lds_u32(r + 2) >> (4 * L.tig);
            const uint32_t ws = w >> 8, vs = v >> 8, hw2 = hw >> 16, hv2 = hv >> 16;
            const BFrag bl = bmask(fl, L.slot, k), bh = bmask(fh, L.slot, k);
            mma16816(cl, lo_even(w, hw), lo_even(v, hv), lo_odd(ws, hw), lo_odd(vs, hv), bl.b0, bl.b1);
            mma16816(ch, hi_even(w, hw2), hi_even(v, hv2), hi_odd(ws, hw2), hi_odd(vs, hv2), bh.b0, bh.b1);
        }
        if (L.tig < nvalid) {
            const float dg = h2f(lds_u16(bg + L.tig * BB)), dg8 = h2f(lds_u16(bg8 + L.tig * BB));
            const uint32_t q = (e_blk + 32 * L.tig) >> 4;
            scale_add(acc, cl, dg, 16.0f * dg, dg8, 16.0f * dg8, sm.sx[q]);
            scale_add(acc, ch, dg * 0.0625f, 16.0f * dg, dg8 * 0.0625f, 16.0f * dg8, sm.sx[q + 1]);
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

template <class F>
__device__ __forceinline__ void tile_rows(const uint8_t* base, uint64_t rb, uint32_t K, const Lane& L,
                                          uint32_t first, uint32_t step, const MmaSmem& sm, float* acc) {
    const uint32_t nblk32 = K / 32;
    const uint32_t nit = (K + F::SB - 1) / F::SB;
    const uint8_t* rg = base + (uint64_t)L.g * rb;
    const uint8_t* rg8 = base + (uint64_t)(L.g + 8) * rb;
    for (uint32_t it = first; it < nit; it += step) {
        const uint32_t nvalid = F::SB == 256 ? 1u : min(4u, nblk32 - it * 4);
        F::compute(rg + (uint64_t)it * F::SBB, rg8 + (uint64_t)it * F::SBB, it * F::SB, nvalid, L, sm, acc);
    }
}

// Iterations [it0, it1) of one K-chunk of a tile (rows at stride rb from base,
// the chunk's first byte at base): warps first, first + step, ...
// mis, mis8: where rows g and g + 8 start in their slots (copies of rows whose
// chunk does not start on a 16-byte boundary bring the aligned window around it).
template <class F>
__device__ __forceinline__ void chunk_rows(const uint8_t* base, uint64_t rb, uint32_t mis, uint32_t mis8, uint32_t K,
                                           const Lane& L, uint32_t first, uint32_t step, uint32_t it0, uint32_t it1,
                                           const MmaSmem& sm, float* acc) {
    const uint32_t nblk32 = K / 32;
    const uint8_t* rg = base + (uint64_t)L.g * rb + mis;
    const uint8_t* rg8 = base + (uint64_t)(L.g + 8) * rb + mis8;
    for (uint32_t it = it0 + first; it < it1; it += step) {
        const uint32_t nvalid = F::SB == 256 ? 1u : min(4u, nblk32 - it * 4);
        const uint64_t o = (uint64_t)(it - it0) * F::SBB;
        F::compute(rg + o, rg8 + o, it * F::SB, nvalid, L, sm, acc);
    }
}

// ------------------------------------------------------------------ tiles

struct TileRef {
    uint32_t seg, row0, nrows;
};

__device__ __forceinline__ TileRef tile_of(const GemvArgs& a, uint32_t t) {
    uint32_t s = 0;
#pragma unroll
    for (uint32_t i = 1; i < kMaxSegs; i++)
        if (i < a.nseg && t >= a.seg[i].tile0) s = i;
    const GemvSeg& G = a.seg[s];
    const uint32_t row0 = (t - G.tile0) * 16;
    return TileRef{s, row0, min(16u, G.rows - row0)};
}

__host__ __device__ __forceinline__ uint32_t align16(uint64_t v) { return (uint32_t)((v + 15) & ~uint64_t(15)); }

// Row stride of a tile in shared memory. Rows that are an even number of
// 16-byte units long would all start in the same bank group, so the 8 rows an
// MMA fragment reads at once would conflict 8 ways; such rows are copied one
// by one to a stride of one more unit. Other row sizes stay contiguous and
// move in one copy.
__host__ __device__ __forceinline__ uint64_t smem_rs(uint64_t rb) {
    return (rb % 16 == 0 && (rb / 16) % 2 == 0) ? rb + 16 : rb;
}
// Shared-memory bytes of one 16-row tile.
__host__ __device__ __forceinline__ uint32_t tile_bytes(uint64_t rb) { return align16(16 * smem_rs(rb)); }
// Offset of the up matrix's rows in a gated tile.
__host__ __device__ __forceinline__ uint32_t up_offset(const GemvSeg& G) { return tile_bytes(G.row_bytes); }
// Bytes the copies of `nrows` rows deliver (what the mbarrier expects).
__host__ __device__ __forceinline__ uint32_t rows_tx(uint64_t rb, uint32_t nrows) {
    return smem_rs(rb) == rb ? align16((uint64_t)nrows * rb) : (uint32_t)(nrows * rb);
}
// Rows copied through a tensor map: an even number of 16-byte units (their
// shared-memory stride is padded by one unit). Copying such rows one bulk copy
// per row is slow (the copy engine handles small copies at a few GB/s per SM),
// so their tiles move as one TMA tensor copy whose box is a unit wider than
// the row (encode_tile_map), which lands the rows at the padded stride.
__host__ __device__ __forceinline__ bool padded_rows(uint64_t rb) { return smem_rs(rb) != rb; }

// TMA tensor copy of a K-chunk of a 16-row tile: the map's box starting at
// unit y of each row. No multicast.
__device__ __forceinline__ void tma_box(void* dst, const CUtensorMap* map, int32_t y, int32_t row0, uint64_t* bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3, %4}], [%5];\n"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(row0),
                   "r"(smem_u32(bar)) : "memory");
}

// TMA tensor copy of one 16-row tile: box {8 halves, units + 1, 16 rows} of a
// rank-3 view {8, units per row, rows} at row row0, written densely; the extra
// unit and rows past the end read as zeros. dst 128-byte aligned. No multicast.
__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* map, int32_t row0, uint64_t* bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3, %4}], [%5];\n"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(0), "r"(row0),
                   "r"(smem_u32(bar)) : "memory");
}
// Bytes one tile of rows of rb bytes brings into shared memory (a tensor copy
// delivers the whole box).
__host__ __device__ __forceinline__ uint32_t tile_tx(uint64_t rb, uint32_t nrows, bool tensor) {
    return tensor ? 16u * (uint32_t)smem_rs(rb) : rows_tx(rb, nrows);
}

// One thread: copy rows [0, nrows) at src (row size rb) into dst at stride smem_rs(rb).
__device__ __forceinline__ void copy_rows(uint8_t* dst, const uint8_t* src, uint64_t rb, uint32_t nrows,
                                          uint64_t* bar) {
    const uint64_t rs = smem_rs(rb);
    if (rs == rb) {
        bulk_g2s(dst, src, align16((uint64_t)nrows * rb), bar);
        return;
    }
    for (uint32_t r = 0; r < nrows; r++) bulk_g2s(dst + r * rs, src + (uint64_t)r * rb, (uint32_t)rb, bar);
}

}  // namespace lm
