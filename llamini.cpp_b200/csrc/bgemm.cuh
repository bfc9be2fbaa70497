// bgemm.cuh -- per-format compute of the batched dequant-GEMM (k_bgemm.cu).
//
// Y[b][r] = sum_k W[r][k] X[b][k] for up to 64 input vectors. The weight side is
// the same exact-integer A fragment as the single-vector kernel (mma_gemv.cuh):
// q enters mma.sync.m16n8k16 as an fp16 subnormal, w = alpha * q - beta is
// applied per 16/32-element group in f32 afterwards. The input side differs:
// the 8 B columns of one MMA carry 4 sequences, each as an fp16 (hi, lo) pair of
// its own scaled x, so a lane (g, tig) of the result holds sequence 4q + tig's
// sums for rows g and g + 8 (columns 2tig, 2tig + 1 = hi + lo). No column is
// wasted, and every group's scale is applied by every lane.
#pragma once

#include "mma_gemv.cuh"

namespace lm {

constexpr uint32_t kBMaxQuads = 16;       // 64 input vectors

// Staged input of the CTA's current K unit in shared memory: fp16 hi and lo of
// x * 2^E per sequence (row stride xs halves) and 16-element sums (stride sxs).
// Within every aligned group of 4 elements the halves are stored in fragment
// order (e, e+2, e+1, e+3), so a lane's 8-byte load is its B fragment as is.
struct BX {
    const uint16_t* h;
    const uint16_t* l;
    const float* sx;
    uint32_t xs, sxs;
};

struct BLane {
    uint32_t g, tig;
};

// B fragment of quad q at local element e0 (e0 % 4 == 0): lane (g, tig) gives
// column g = (sequence 4q + g/2, hi for even g, lo for odd g), elements e0..e0+3.
__device__ __forceinline__ BFrag bq(const BX& X, const BLane& L, uint32_t q, uint32_t e0) {
    const uint16_t* p = ((L.g & 1u) ? X.l : X.h) + (4 * q + (L.g >> 1)) * X.xs + e0;
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    return BFrag{v.x, v.y};
}
// Both fragments of elements e0..e0+7 (e0 % 8 == 0) in one 16-byte load.
__device__ __forceinline__ void bq2(const BX& X, const BLane& L, uint32_t q, uint32_t e0, BFrag& f0, BFrag& f1) {
    const uint16_t* p = ((L.g & 1u) ? X.l : X.h) + (4 * q + (L.g >> 1)) * X.xs + e0;
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    f0 = BFrag{v.x, v.y};
    f1 = BFrag{v.z, v.w};
}
__device__ __forceinline__ float bsx(const BX& X, const BLane& L, uint32_t q, uint32_t i16) {
    return X.sx[(4 * q + L.tig) * X.sxs + i16];
}

template <uint32_t NQ>
struct BAcc {
    float v[NQ][2];
};

// Q4_K super-block (gguf.c:504-529) at local element eb; bg/bg8 are rows g, g+8.
template <uint32_t NQ>
__device__ __forceinline__ void bq4k(const uint8_t* bg, const uint8_t* bg8, uint32_t eb, uint32_t nq, const BLane& L,
                                     const BX& X, BAcc<NQ>& acc) {
    const uint4 h = *reinterpret_cast<const uint4*>(bg), h8 = *reinterpret_cast<const uint4*>(bg8);
    const float dg = h2f(h.x & 0xFFFFu), mg = h2f(h.x >> 16);
    const float dg8 = h2f(h8.x & 0xFFFFu), mg8 = h2f(h8.x >> 16);
#pragma unroll
    for (uint32_t j = 0; j < 4; j++) {
        const uint2 q = *reinterpret_cast<const uint2*>(bg + 16 + 32 * j + 8 * L.tig);
        const uint2 q8 = *reinterpret_cast<const uint2*>(bg8 + 16 + 32 * j + 8 * L.tig);
        float sl, ml, sh, mh, tl, nl, th, nh;
        FQ4K::scales(h.y, h.z, h.w, j, &sl, &ml, &sh, &mh);
        FQ4K::scales(h8.y, h8.z, h8.w, j, &tl, &nl, &th, &nh);
        const float al = dg * sl, bl = mg * ml, ah = dg * sh * 0.0625f, bh = mg * mh;
        const float al8 = dg8 * tl, bl8 = mg8 * nl, ah8 = dg8 * th * 0.0625f, bh8 = mg8 * nh;
        const uint32_t w0 = q.x, w1 = q.y, v0 = q8.x, v1 = q8.y;
        const uint32_t w0s = w0 >> 8, w1s = w1 >> 8, v0s = v0 >> 8, v1s = v1 >> 8;
        const uint32_t e = eb + 64 * j + 8 * L.tig;
        const uint32_t i16 = (eb + 64 * j) >> 4;
#pragma unroll
        for (uint32_t qq = 0; qq < NQ; qq++) {
            if (qq < nq) {
                BFrag f0, f1, g0, g1;
                bq2(X, L, qq, e, f0, f1);
                bq2(X, L, qq, e + 32, g0, g1);
                float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(cl, w0 & 0x000F000Fu, v0 & 0x000F000Fu, w0s & 0x000F000Fu, v0s & 0x000F000Fu, f0.b0, f0.b1);
                mma16816(cl, w1 & 0x000F000Fu, v1 & 0x000F000Fu, w1s & 0x000F000Fu, v1s & 0x000F000Fu, f1.b0, f1.b1);
                mma16816(ch, w0 & 0x00F000F0u, v0 & 0x00F000F0u, w0s & 0x00F000F0u, v0s & 0x00F000F0u, g0.b0, g0.b1);
                mma16816(ch, w1 & 0x00F000F0u, v1 & 0x00F000F0u, w1s & 0x00F000F0u, v1s & 0x00F000F0u, g1.b0, g1.b1);
                const float sxl = bsx(X, L, qq, i16) + bsx(X, L, qq, i16 + 1);
                const float sxh = bsx(X, L, qq, i16 + 2) + bsx(X, L, qq, i16 + 3);
                scale_add(acc.v[qq], cl, al, bl, al8, bl8, sxl);
                scale_add(acc.v[qq], ch, ah, bh, ah8, bh8, sxh);
            }
        }
    }
}

// Q6_K super-block (gguf.c:561-590): 16 scale groups of 16 elements.
template <uint32_t NQ>
__device__ __forceinline__ void bq6k(const uint8_t* bg, const uint8_t* bg8, uint32_t eb, uint32_t nq, const BLane& L,
                                     const BX& X, BAcc<NQ>& acc) {
    const float dg = h2f(lds_u16(bg + 208)), dg8 = h2f(lds_u16(bg8 + 208));
#pragma unroll
    for (uint32_t H = 0; H < 2; H++) {
#pragma unroll
        for (uint32_t u = 0; u < 2; u++) {
            const uint32_t off = 16 * u + 4 * L.tig;
            const uint32_t a = lds_u32(bg + 64 * H + off), b = lds_u32(bg + 64 * H + 32 + off);
            const uint32_t hq = lds_u32(bg + 128 + 32 * H + off);
            const uint32_t a8 = lds_u32(bg8 + 64 * H + off), b8 = lds_u32(bg8 + 64 * H + 32 + off);
            const uint32_t h8 = lds_u32(bg8 + 128 + 32 * H + off);
            uint32_t wq[4], wm[4];
            wq[0] = FQ6K::word(a, (hq << 4) & 0x30303030u);
            wq[1] = FQ6K::word(b, (hq << 2) & 0x30303030u);
            wq[2] = FQ6K::word(a >> 4, hq & 0x30303030u);
            wq[3] = FQ6K::word(b >> 4, (hq >> 2) & 0x30303030u);
            wm[0] = FQ6K::word(a8, (h8 << 4) & 0x30303030u);
            wm[1] = FQ6K::word(b8, (h8 << 2) & 0x30303030u);
            wm[2] = FQ6K::word(a8 >> 4, h8 & 0x30303030u);
            wm[3] = FQ6K::word(b8 >> 4, (h8 >> 2) & 0x30303030u);
#pragma unroll
            for (uint32_t c = 0; c < 4; c++) {
                const uint32_t si = 192 + 8 * H + u + 2 * c;
                const float ag = dg * (float)(int8_t)bg[si], ag8 = dg8 * (float)(int8_t)bg8[si];
                const uint32_t a0 = __byte_perm(wq[c], 0, 0x4240), a1 = __byte_perm(wm[c], 0, 0x4240);
                const uint32_t a2 = __byte_perm(wq[c], 0, 0x4341), a3 = __byte_perm(wm[c], 0, 0x4341);
                const uint32_t e = eb + 128 * H + 32 * c + 16 * u;
#pragma unroll
                for (uint32_t qq = 0; qq < NQ; qq++) {
                    if (qq < nq) {
                        const BFrag f = bq(X, L, qq, e + 4 * L.tig);
                        float cc[4] = {0.f, 0.f, 0.f, 0.f};
                        mma16816(cc, a0, a1, a2, a3, f.b0, f.b1);
                        scale_add(acc.v[qq], cc, ag, 32.0f * ag, ag8, 32.0f * ag8, bsx(X, L, qq, e >> 4));
                    }
                }
            }
        }
    }
}

// Q8_0 block (gguf.c:489-503) at local element eb: w = d (q ^ 0x80) - 128 d.
template <uint32_t NQ>
__device__ __forceinline__ void bq80(const uint8_t* bg, const uint8_t* bg8, uint32_t eb, uint32_t nq, const BLane& L,
                                     const BX& X, BAcc<NQ>& acc) {
    const uint8_t* p = bg + 2 + 4 * L.tig;
    const uint8_t* p8 = bg8 + 2 + 4 * L.tig;
    const uint32_t w = lds_u32(p) ^ 0x80808080u, v = lds_u32(p8) ^ 0x80808080u;
    const uint32_t w2 = lds_u32(p + 16) ^ 0x80808080u, v2 = lds_u32(p8 + 16) ^ 0x80808080u;
    const float dg = h2f(lds_u16(bg)), dg8 = h2f(lds_u16(bg8));
    const uint32_t a0 = __byte_perm(w, 0, 0x4240), a1 = __byte_perm(v, 0, 0x4240);
    const uint32_t a2 = __byte_perm(w, 0, 0x4341), a3 = __byte_perm(v, 0, 0x4341);
    const uint32_t c0 = __byte_perm(w2, 0, 0x4240), c1 = __byte_perm(v2, 0, 0x4240);
    const uint32_t c2 = __byte_perm(w2, 0, 0x4341), c3 = __byte_perm(v2, 0, 0x4341);
    const uint32_t e = eb + 4 * L.tig;
#pragma unroll
    for (uint32_t qq = 0; qq < NQ; qq++) {
        if (qq < nq) {
            const BFrag f0 = bq(X, L, qq, e), f1 = bq(X, L, qq, e + 16);
            float cc[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(cc, a0, a1, a2, a3, f0.b0, f0.b1);
            mma16816(cc, c0, c1, c2, c3, f1.b0, f1.b1);
            scale_add(acc.v[qq], cc, dg, 128.0f * dg, dg8, 128.0f * dg8,
                      bsx(X, L, qq, eb >> 4) + bsx(X, L, qq, (eb >> 4) + 1));
        }
    }
}

// Q4_0 block (gguf.c:427-444): low nibbles are elements 0..15, high 16..31.
template <uint32_t NQ>
__device__ __forceinline__ void bq40(const uint8_t* bg, const uint8_t* bg8, uint32_t eb, uint32_t nq, const BLane& L,
                                     const BX& X, BAcc<NQ>& acc) {
    const uint32_t w = lds_u32(bg + 2 + 4 * L.tig), v = lds_u32(bg8 + 2 + 4 * L.tig);
    const uint32_t ws = w >> 8, vs = v >> 8;
    const float dg = h2f(lds_u16(bg)), dg8 = h2f(lds_u16(bg8));
    const uint32_t e = eb + 4 * L.tig;
#pragma unroll
    for (uint32_t qq = 0; qq < NQ; qq++) {
        if (qq < nq) {
            const BFrag fl = bq(X, L, qq, e), fh = bq(X, L, qq, e + 16);
            float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(cl, w & 0x000F000Fu, v & 0x000F000Fu, ws & 0x000F000Fu, vs & 0x000F000Fu, fl.b0, fl.b1);
            mma16816(ch, w & 0x00F000F0u, v & 0x00F000F0u, ws & 0x00F000F0u, vs & 0x00F000F0u, fh.b0, fh.b1);
            scale_add(acc.v[qq], cl, dg, 8.0f * dg, dg8, 8.0f * dg8, bsx(X, L, qq, eb >> 4));
            scale_add(acc.v[qq], ch, dg * 0.0625f, 8.0f * dg, dg8 * 0.0625f, 8.0f * dg8, bsx(X, L, qq, (eb >> 4) + 1));
        }
    }
}

// F16 rows (GPT-2's tied lm_head): 32 elements; the fp16 weights enter the MMA
// unchanged, so the sums carry an extra 2^24 relative to the integer formats.
template <uint32_t NQ>
__device__ __forceinline__ void bf16w(const uint8_t* bg, const uint8_t* bg8, uint32_t eb, uint32_t nq, const BLane& L,
                                      const BX& X, BAcc<NQ>& acc) {
    const uint2 r0 = *reinterpret_cast<const uint2*>(bg + 8 * L.tig);
    const uint2 r8 = *reinterpret_cast<const uint2*>(bg8 + 8 * L.tig);
    const uint2 s0 = *reinterpret_cast<const uint2*>(bg + 32 + 8 * L.tig);
    const uint2 s8 = *reinterpret_cast<const uint2*>(bg8 + 32 + 8 * L.tig);
    const uint32_t a0 = __byte_perm(r0.x, r0.y, 0x5410), a1 = __byte_perm(r8.x, r8.y, 0x5410);
    const uint32_t a2 = __byte_perm(r0.x, r0.y, 0x7632), a3 = __byte_perm(r8.x, r8.y, 0x7632);
    const uint32_t c0 = __byte_perm(s0.x, s0.y, 0x5410), c1 = __byte_perm(s8.x, s8.y, 0x5410);
    const uint32_t c2 = __byte_perm(s0.x, s0.y, 0x7632), c3 = __byte_perm(s8.x, s8.y, 0x7632);
    const uint32_t e = eb + 4 * L.tig;
    const float k = 5.9604644775390625e-08f;   // 2^-24
#pragma unroll
    for (uint32_t qq = 0; qq < NQ; qq++) {
        if (qq < nq) {
            const BFrag f0 = bq(X, L, qq, e), f1 = bq(X, L, qq, e + 16);
            float cc[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(cc, a0, a1, a2, a3, f0.b0, f0.b1);
            mma16816(cc, c0, c1, c2, c3, f1.b0, f1.b1);
            scale_add(acc.v[qq], cc, k, 0.f, k, 0.f, 0.f);
        }
    }
}

}  // namespace lm
