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
//    with a single AND on the packed bytes; x enters the B operand as two fp16
//    columns, x_hi + x_lo (22 significant bits), after scaling the whole vector
//    by a power of two so that it fits fp16's range. The accumulator is f32.
//  * alpha, beta and the per-group sums of x are applied in f32 by the lanes
//    that hold column 0/1 of the accumulator; the result is scaled back by the
//    same power of two.
//
// CTA = one tile of 16 output rows (32 for a gated pair); its 8 warps split the
// row's blocks between them and combine their partial sums in shared memory.
#include "internal.h"
#include "quant.cuh"

#include <cuda_fp16.h>

namespace lm {

constexpr int kMWarps = 8;
constexpr int kMThreads = kMWarps * 32;

bool mma_type(uint32_t t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0 || t == T_Q4_0; }

struct MmaSmem {
    float* xf;          // normalised x (f32)
    uint32_t* xh;       // x * 2^E as fp16 pairs, high part   (K/2 words)
    uint32_t* xl;       // low part
    float* sx;          // per 16-element run: sum(x) * 2^(E-24)
};

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// B fragment of this lane for the 4 consecutive elements starting at e0 (a
// multiple of 4): k slots (2t, 2t+1) take elements (e0, e0+2) and slots
// (2t+8, 2t+9) take (e0+1, e0+3), matching how the A pairs are cut from packed
// bytes. Column 0 is x_hi, column 1 x_lo, the other columns are zero.
struct BFrag { uint32_t b0, b1; };

__device__ __forceinline__ BFrag bfrag(const uint32_t* xpart, uint32_t e0, bool active) {
    BFrag f{0u, 0u};
    if (active) {
        const uint2 v = *reinterpret_cast<const uint2*>(xpart + (e0 >> 1));   // halves e0..e0+3
        f.b0 = __byte_perm(v.x, v.y, 0x5410);     // (e0, e0+2)
        f.b1 = __byte_perm(v.x, v.y, 0x7632);     // (e0+1, e0+3)
    }
    return f;
}

// ------------------------------------------------------------------ formats
// Each process() handles one block (or run of blocks) of rows g and g+8 for
// this warp and adds alpha*P - beta*S to acc[0] (row g) and acc[1] (row g+8)
// in the scaled domain. Only lanes with tig == 0 hold meaningful acc.

struct Lane {
    uint32_t g, tig;
    bool bact;                 // provides a B column (g < 2)
    const uint32_t* xpart;     // xh for g == 0, xl for g == 1
};

__device__ __forceinline__ void scale_add(float* acc, const float* c, float a_g, float b_g, float a_g8, float b_g8,
                                          float sx) {
    acc[0] = fmaf(a_g, c[0] + c[1], fmaf(-b_g, sx, acc[0]));
    acc[1] = fmaf(a_g8, c[2] + c[3], fmaf(-b_g8, sx, acc[1]));
}

// Q4_K (gguf.c:504-529): super-block of 256, 4 groups of 64; in group j the
// low nibbles of qs[32j..32j+32) are sub-block 2j, the high nibbles 2j+1.
// Lane tig takes bytes 8*tig..8*tig+8 of each group: two words, i.e. two MMAs
// per sub-block that share its (scale, min).
__device__ __forceinline__ void q4k_block(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk,
                                          const Lane& L, const MmaSmem& sm, float* acc) {
    uint32_t hg[4], hg8[4];
    ld_v4(bg, hg);
    ld_v4(bg8, hg8);
    const float dg = f16_bits(hg[0] & 0xFFFFu), mg = f16_bits(hg[0] >> 16);
    const float dg8 = f16_bits(hg8[0] & 0xFFFFu), mg8 = f16_bits(hg8[0] >> 16);
    uint2 q[4], q8[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        q[j] = __ldg(reinterpret_cast<const uint2*>(bg + 16 + 32 * j + 8 * L.tig));
        q8[j] = __ldg(reinterpret_cast<const uint2*>(bg8 + 16 + 32 * j + 8 * L.tig));
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t e = e_blk + 64 * j + 8 * L.tig;
        const BFrag lo0 = bfrag(L.xpart, e, L.bact), lo1 = bfrag(L.xpart, e + 4, L.bact);
        const BFrag hi0 = bfrag(L.xpart, e + 32, L.bact), hi1 = bfrag(L.xpart, e + 36, L.bact);
        const uint32_t w0 = q[j].x, w1 = q[j].y, v0 = q8[j].x, v1 = q8[j].y;
        const uint32_t w0s = w0 >> 8, w1s = w1 >> 8, v0s = v0 >> 8, v1s = v1 >> 8;
        float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
        // low nibbles: sub-block 2j
        mma16816(cl, w0 & 0x000F000Fu, v0 & 0x000F000Fu, w0s & 0x000F000Fu, v0s & 0x000F000Fu, lo0.b0, lo0.b1);
        mma16816(cl, w1 & 0x000F000Fu, v1 & 0x000F000Fu, w1s & 0x000F000Fu, v1s & 0x000F000Fu, lo1.b0, lo1.b1);
        // high nibbles in place (16*q): sub-block 2j+1, alpha scaled by 1/16
        mma16816(ch, w0 & 0x00F000F0u, v0 & 0x00F000F0u, w0s & 0x00F000F0u, v0s & 0x00F000F0u, hi0.b0, hi0.b1);
        mma16816(ch, w1 & 0x00F000F0u, v1 & 0x00F000F0u, w1s & 0x00F000F0u, v1s & 0x00F000F0u, hi1.b0, hi1.b1);
        if (L.tig == 0) {
            uint32_t s0, m0, s1, m1, t0, n0, t1, n1;
            k4_scale_min(hg + 1, 2 * j, &s0, &m0);
            k4_scale_min(hg + 1, 2 * j + 1, &s1, &m1);
            k4_scale_min(hg8 + 1, 2 * j, &t0, &n0);
            k4_scale_min(hg8 + 1, 2 * j + 1, &t1, &n1);
            const uint32_t r = (e_blk + 64 * j) >> 4;
            const float sxl = sm.sx[r] + sm.sx[r + 1], sxh = sm.sx[r + 2] + sm.sx[r + 3];
            scale_add(acc, cl, dg * (float)s0, mg * (float)m0, dg8 * (float)t0, mg8 * (float)n0, sxl);
            scale_add(acc, ch, dg * (float)s1 * 0.0625f, mg * (float)m1, dg8 * (float)t1 * 0.0625f, mg8 * (float)n1, sxh);
        }
    }
}

// Q6_K (gguf.c:561-590): per 128-half H, byte l of ql[64H..], ql[64H+32..] and
// qh[32H..] give elements 128H + 32c + l (c = 0..3) with scale sc[8H + l/16 + 2c].
// One MMA per 16-element scale group: lane tig takes l = 16u + 4*tig .. +4.
__device__ __forceinline__ uint32_t q6_word(uint32_t n, uint32_t hbits) {
    return (n & 0x0F0F0F0Fu) | hbits;        // 6-bit values in each byte
}

__device__ __forceinline__ void q6k_block(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk,
                                          const Lane& L, const MmaSmem& sm, float* acc) {
    const float dg = f16_bits(ld_u16(bg + 208)), dg8 = f16_bits(ld_u16(bg8 + 208));
#pragma unroll
    for (int H = 0; H < 2; H++) {
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const uint32_t off = 16 * u + 4 * L.tig;
            const uint32_t la = ld_u32(bg + 64 * H + off), lb = ld_u32(bg + 64 * H + 32 + off);
            const uint32_t qh = ld_u32(bg + 128 + 32 * H + off);
            const uint32_t ma = ld_u32(bg8 + 64 * H + off), mb = ld_u32(bg8 + 64 * H + 32 + off);
            const uint32_t mh = ld_u32(bg8 + 128 + 32 * H + off);
            uint32_t wq[4], wm[4];
            wq[0] = q6_word(la, (qh << 4) & 0x30303030u);
            wq[1] = q6_word(lb, (qh << 2) & 0x30303030u);
            wq[2] = q6_word(la >> 4, qh & 0x30303030u);
            wq[3] = q6_word(lb >> 4, (qh >> 2) & 0x30303030u);
            wm[0] = q6_word(ma, (mh << 4) & 0x30303030u);
            wm[1] = q6_word(mb, (mh << 2) & 0x30303030u);
            wm[2] = q6_word(ma >> 4, mh & 0x30303030u);
            wm[3] = q6_word(mb >> 4, (mh >> 2) & 0x30303030u);
            int8_t scg[4], scg8[4];
            if (L.tig == 0) {
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    scg[c] = (int8_t)bg[192 + 8 * H + u + 2 * c];
                    scg8[c] = (int8_t)bg8[192 + 8 * H + u + 2 * c];
                }
            }
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const uint32_t e = e_blk + 128 * H + 32 * c + 16 * u + 4 * L.tig;
                const BFrag b = bfrag(L.xpart, e, L.bact);
                float cc[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(cc, __byte_perm(wq[c], 0, 0x4240), __byte_perm(wm[c], 0, 0x4240),
                         __byte_perm(wq[c], 0, 0x4341), __byte_perm(wm[c], 0, 0x4341), b.b0, b.b1);
                if (L.tig == 0) {
                    const float sx = sm.sx[(e_blk + 128 * H + 32 * c + 16 * u) >> 4];
                    const float ag = dg * (float)scg[c], ag8 = dg8 * (float)scg8[c];
                    scale_add(acc, cc, ag, 32.0f * ag, ag8, 32.0f * ag8, sx);
                }
            }
        }
    }
}

// Q8_0 (gguf.c:489-503): 32 int8 per block, w = d * q. With u = q ^ 0x80 the
// value is d*u - 128*d, u in [0, 255].
__device__ __forceinline__ void q8_block(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk,
                                         const Lane& L, const MmaSmem& sm, float* acc) {
    const float dg = f16_bits(ld_u16(bg)), dg8 = f16_bits(ld_u16(bg8));
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const uint32_t w = ld_u32(bg + 2 + 16 * u + 4 * L.tig) ^ 0x80808080u;
        const uint32_t v = ld_u32(bg8 + 2 + 16 * u + 4 * L.tig) ^ 0x80808080u;
        const uint32_t e = e_blk + 16 * u + 4 * L.tig;
        const BFrag b = bfrag(L.xpart, e, L.bact);
        float cc[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(cc, __byte_perm(w, 0, 0x4240), __byte_perm(v, 0, 0x4240),
                 __byte_perm(w, 0, 0x4341), __byte_perm(v, 0, 0x4341), b.b0, b.b1);
        if (L.tig == 0) {
            const float sx = sm.sx[(e_blk + 16 * u) >> 4];
            scale_add(acc, cc, dg, 128.0f * dg, dg8, 128.0f * dg8, sx);
        }
    }
}

// Q4_0 (gguf.c:427-444): w = (q - 8) * d; low nibbles are elements 0..15,
// high nibbles 16..31 of the block.
__device__ __forceinline__ void q40_block(const uint8_t* bg, const uint8_t* bg8, uint32_t e_blk,
                                          const Lane& L, const MmaSmem& sm, float* acc) {
    const float dg = f16_bits(ld_u16(bg)), dg8 = f16_bits(ld_u16(bg8));
    const uint32_t w = ld_u32(bg + 2 + 4 * L.tig), v = ld_u32(bg8 + 2 + 4 * L.tig);
    const uint32_t ws = w >> 8, vs = v >> 8;
    const BFrag lo = bfrag(L.xpart, e_blk + 4 * L.tig, L.bact);
    const BFrag hi = bfrag(L.xpart, e_blk + 16 + 4 * L.tig, L.bact);
    float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816(cl, w & 0x000F000Fu, v & 0x000F000Fu, ws & 0x000F000Fu, vs & 0x000F000Fu, lo.b0, lo.b1);
    mma16816(ch, w & 0x00F000F0u, v & 0x00F000F0u, ws & 0x00F000F0u, vs & 0x00F000F0u, hi.b0, hi.b1);
    if (L.tig == 0) {
        const uint32_t r = e_blk >> 4;
        scale_add(acc, cl, dg, 8.0f * dg, dg8, 8.0f * dg8, sm.sx[r]);
        scale_add(acc, ch, dg * 0.0625f, 8.0f * dg, dg8 * 0.0625f, 8.0f * dg8, sm.sx[r + 1]);
    }
}

// All blocks of rows g and g+8 that belong to warp `warp` (blocks warp,
// warp+W, ...), accumulated into acc.
template <uint32_t T>
__device__ __forceinline__ void mma_rows(const uint8_t* rg, const uint8_t* rg8, uint32_t K, uint32_t warp,
                                         const Lane& L, const MmaSmem& sm, float* acc) {
    using F = Fmt<T>;
    const uint32_t nb = K / F::BE;
    for (uint32_t b = warp; b < nb; b += kMWarps) {
        const uint8_t* bg = rg + (uint64_t)b * F::BB;
        const uint8_t* bg8 = rg8 + (uint64_t)b * F::BB;
        if (T == T_Q4_K) q4k_block(bg, bg8, b * F::BE, L, sm, acc);
        else if (T == T_Q6_K) q6k_block(bg, bg8, b * F::BE, L, sm, acc);
        else if (T == T_Q8_0) q8_block(bg, bg8, b * F::BE, L, sm, acc);
        else q40_block(bg, bg8, b * F::BE, L, sm, acc);
    }
}

__device__ __forceinline__ void mma_dispatch(uint32_t type, const uint8_t* rg, const uint8_t* rg8, uint32_t K,
                                             uint32_t warp, const Lane& L, const MmaSmem& sm, float* acc) {
    switch (type) {
    case T_Q4_K: mma_rows<T_Q4_K>(rg, rg8, K, warp, L, sm, acc); break;
    case T_Q6_K: mma_rows<T_Q6_K>(rg, rg8, K, warp, L, sm, acc); break;
    case T_Q8_0: mma_rows<T_Q8_0>(rg, rg8, K, warp, L, sm, acc); break;
    case T_Q4_0: mma_rows<T_Q4_0>(rg, rg8, K, warp, L, sm, acc); break;
    default: break;
    }
}

// ------------------------------------------------------------------ shared helpers

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
__device__ float bsum(float v, float* red) {
    v = wsum(v);
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (uint32_t i = 0; i < kMWarps; i++) t += red[i];
    return t;
}
__device__ float bmax(float v, float* red) {
    v = wmax(v);
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (uint32_t i = 0; i < kMWarps; i++) t = fmaxf(t, red[i]);
    return t;
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

// ------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kMThreads)
gemv_mma_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(16) float smem[];
    const uint32_t K = a.K;                       // multiple of 32 (checked by the launcher)
    MmaSmem sm;
    sm.xf = smem;
    sm.xh = reinterpret_cast<uint32_t*>(smem + K);
    sm.xl = sm.xh + K / 2;
    sm.sx = reinterpret_cast<float*>(sm.xl + K / 2);
    float* red = sm.sx + K / 16;                  // [kMWarps] scratch
    float* part = red + kMWarps;                  // [kMWarps][2][16] partial rows
    __shared__ float s_scale;

    // ---- prologue: x (normalised), its power-of-two scale, fp16 split, run sums
    if (a.norm == NORM_NONE) {
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) sm.xf[i] = a.x[i];
    } else if (a.norm == NORM_RMS) {
        float ss = 0.f;
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) { float v = a.x[i]; sm.xf[i] = v; ss = fmaf(v, v, ss); }
        ss = bsum(ss, red);
        const float inv = 1.0f / sqrtf(ss / (float)K + a.eps);          // model.c:7-9
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) sm.xf[i] = sm.xf[i] * inv * a.norm_w[i];
    } else {
        float s = 0.f;
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) { float v = a.x[i]; sm.xf[i] = v; s += v; }
        const float mean = bsum(s, red) / (float)K;                     // gpt2.c:131-138
        float vs = 0.f;
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) { float c = sm.xf[i] - mean; vs = fmaf(c, c, vs); }
        const float inv = 1.0f / sqrtf(bsum(vs, red) / (float)K + a.eps);
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x)
            sm.xf[i] = (sm.xf[i] - mean) * inv * a.norm_w[i] + a.norm_b[i];
    }
    __syncthreads();
    float mx = 0.f;
    for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) mx = fmaxf(mx, fabsf(sm.xf[i]));
    mx = bmax(mx, red);
    int e = 0;
    if (mx > 0.f && mx < INFINITY) frexpf(mx, &e);                   // mx < 2^e
    const int E = 14 - e;                                              // |x * 2^E| < 2^14
    for (uint32_t i = threadIdx.x; i < K / 2; i += blockDim.x) {
        const float v0 = ldexpf(sm.xf[2 * i], E), v1 = ldexpf(sm.xf[2 * i + 1], E);
        const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
        const __half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
        sm.xh[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        sm.xl[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    for (uint32_t r = threadIdx.x; r < K / 16; r += blockDim.x) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++) s += sm.xf[16 * r + i];
        sm.sx[r] = ldexpf(s, E - 24);
    }
    if (threadIdx.x == 0) s_scale = ldexpf(1.0f, 24 - E);
    __syncthreads();
    if (a.x_out != nullptr && blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) a.x_out[i] = sm.xf[i];

    // ---- which tile
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
    // rows past the end of the matrix read row `rows-1` (results discarded)
    const uint32_t ra = min(row0 + L.g, G.rows - 1), rb = min(row0 + L.g + 8, G.rows - 1);

    float acc[2] = {0.f, 0.f};
    mma_dispatch(G.type, G.w + (uint64_t)ra * G.row_bytes, G.w + (uint64_t)rb * G.row_bytes, K, warp, L, sm, acc);
    float acc2[2] = {0.f, 0.f};
    if (glu) mma_dispatch(G.type2, G.w2 + (uint64_t)ra * G.row_bytes2, G.w2 + (uint64_t)rb * G.row_bytes2, K, warp, L, sm, acc2);

    if (L.tig == 0) {
        part[(warp * 2 + 0) * 16 + L.g] = acc[0];
        part[(warp * 2 + 0) * 16 + L.g + 8] = acc[1];
        part[(warp * 2 + 1) * 16 + L.g] = acc2[0];
        part[(warp * 2 + 1) * 16 + L.g + 8] = acc2[1];
    }
    __syncthreads();

    // ---- epilogue: thread r < 16 finishes row row0 + r
    unsigned long long key = 0ull;
    if (threadIdx.x < 16) {
        const uint32_t r = threadIdx.x, row = row0 + r;
        float v = 0.f, u = 0.f;
        for (uint32_t w = 0; w < kMWarps; w++) { v += part[(w * 2) * 16 + r]; u += part[(w * 2 + 1) * 16 + r]; }
        v *= s_scale;
        u *= s_scale;
        if (row < G.rows) {
            switch (G.epi) {
            case EPI_STORE: if (G.bias) v += G.bias[row]; G.out[row] = v; break;
            case EPI_RESID: if (G.bias) v += G.bias[row]; G.out[row] += v; break;
            case EPI_GLU_SILU: v = v / (1.0f + expf(-v)) * u; G.out[row] = v; break;
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
    return (size_t)K * 4 + (size_t)K * 4 + (size_t)K / 16 * 4 + kMWarps * 4 + kMWarps * 2 * 16 * 4;
}

bool gemv_mma_init() {
    return LM_CUDA(cudaFuncSetAttribute(gemv_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
}

// Launch when every segment is a tensor-core format; returns false with
// *handled = false otherwise (the caller then uses the CUDA-core kernel).
bool launch_gemv_mma(const GemvArgs& in, cudaStream_t st, bool* handled) {
    *handled = false;
    if (in.K % 256 != 0 && in.K % 32 != 0) return true;
    for (uint32_t i = 0; i < in.nseg; i++) {
        const GemvSeg& g = in.seg[i];
        const bool glu = g.epi == EPI_GLU_SILU || g.epi == EPI_GLU_GELU;
        if (!mma_type(g.type) || (glu && !mma_type(g.type2))) return true;
        if (type_bytes(g.type, in.K) == 0 || (glu && type_bytes(g.type2, in.K) == 0)) return true;
    }
    GemvArgs a = in;
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < a.nseg; i++) {
        a.seg[i].tile0 = tiles;
        tiles += (a.seg[i].rows + 15) / 16;
    }
    const size_t smem = gemv_mma_smem(a.K);
    if (smem > 200 * 1024) return true;
    *handled = true;
    gemv_mma_kernel<<<tiles, kMThreads, smem, st>>>(a);
    return LM_CUDA(cudaGetLastError());
}

}  // namespace lm
