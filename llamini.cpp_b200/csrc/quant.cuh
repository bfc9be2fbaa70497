// quant.cuh -- register-level decoders for the GGUF block formats.
//
// Every format is handled in "units" of 32 elements: a unit is the smallest
// piece of a block whose weights share their scale fields and whose bytes a
// thread can fetch on its own. decode() yields the 32 dequantized weights of one
// unit in the unit's own order and elem() says which element of the block each
// one is. The weights are bit-identical to llamini.cpp gguf.c:409-594: every
// product and sum is written with the _rn intrinsics so the compiler cannot fuse
// them into FMAs, which would change the rounding.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace lm {

enum : uint32_t {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q8_0 = 8,
    T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14
};

// Half -> float from the bit pattern, with the reference's exact handling of
// subnormals, infinities and NaN payloads (gguf.c:364-386).
__device__ __forceinline__ float f16_bits(uint32_t h) {
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 31u;
    uint32_t m = h & 1023u;
    uint32_t bits;
    if (e == 31u) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e != 0u) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0u) {
        bits = sign;
    } else {
        // subnormal: normalise so that bit 10 is set; each shift lowers the exponent
        uint32_t sh = __clz(m) - 21;      // m < 1024 -> clz >= 22; shift to bit 10
        m = (m << sh) & 1023u;
        bits = sign | ((113u - sh) << 23) | (m << 13);
    }
    return __uint_as_float(bits);
}

// Loads that tolerate any byte alignment: the surrounding aligned words are
// read and funnel-shifted. Reads at most 3 bytes past the requested range,
// which the weight store pads for.
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    uint32_t s = (uint32_t)(a & 3u) * 8u;
    uint32_t lo = __ldg(w);
    if (s == 0) return lo;
    return __funnelshift_r(lo, __ldg(w + 1), s);
}
__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
    return ld_u32(p) & 0xFFFFu;
}
__device__ __forceinline__ uint32_t byte_of(const uint32_t* w, uint32_t i) {
    return (w[i >> 2] >> ((i & 3u) * 8u)) & 0xFFu;
}
// n bytes (n a multiple of 4) from any alignment into words.
template <int NW>
__device__ __forceinline__ void ld_words(const uint8_t* p, uint32_t* w) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* b = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    uint32_t s = (uint32_t)(a & 3u) * 8u;
    if (s == 0) {
#pragma unroll
        for (int i = 0; i < NW; i++) w[i] = __ldg(b + i);
    } else {
        uint32_t prev = __ldg(b);
#pragma unroll
        for (int i = 0; i < NW; i++) {
            uint32_t nx = __ldg(b + i + 1);
            w[i] = __funnelshift_r(prev, nx, s);
            prev = nx;
        }
    }
}
// 16-byte aligned vector load.
__device__ __forceinline__ void ld_v4(const uint8_t* p, uint32_t* w) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
}

// gguf.c:391-399: six-bit scale and min of sub-block j from the 12 scale bytes
// (given as 3 little-endian words).
__device__ __forceinline__ void k4_scale_min(const uint32_t* s, uint32_t j, uint32_t* sc, uint32_t* mn) {
    if (j < 4) {
        *sc = byte_of(s, j) & 63u;
        *mn = byte_of(s, j + 4) & 63u;
    } else {
        *sc = (byte_of(s, j + 4) & 15u) | ((byte_of(s, j - 4) >> 6) << 4);
        *mn = (byte_of(s, j + 4) >> 4) | ((byte_of(s, j) >> 6) << 4);
    }
}

template <uint32_t T> struct Fmt;

// ---- 32-element block formats: one unit per block, natural element order.
template <> struct Fmt<T_Q4_0> {           // gguf.c:427-444
    static constexpr uint32_t BE = 32, BB = 18, UPB = 1;
    static __device__ __forceinline__ uint32_t elem(uint32_t, uint32_t i) { return i; }
    static __device__ __forceinline__ void decode(const uint8_t* b, uint32_t, float* y) {
        float d = f16_bits(ld_u16(b));
        uint32_t q[4];
        ld_words<4>(b + 2, q);
#pragma unroll
        for (uint32_t i = 0; i < 16; i++) {
            uint32_t v = byte_of(q, i);
            y[i]      = __fmul_rn(__fsub_rn((float)(v & 15u), 8.0f), d);
            y[i + 16] = __fmul_rn(__fsub_rn((float)(v >> 4), 8.0f), d);
        }
    }
};

template <> struct Fmt<T_Q4_1> {           // gguf.c:445-462
    static constexpr uint32_t BE = 32, BB = 20, UPB = 1;
    static __device__ __forceinline__ uint32_t elem(uint32_t, uint32_t i) { return i; }
    static __device__ __forceinline__ void decode(const uint8_t* b, uint32_t, float* y) {
        uint32_t dm = ld_u32(b);
        float d = f16_bits(dm & 0xFFFFu), m = f16_bits(dm >> 16);
        uint32_t q[4];
        ld_words<4>(b + 4, q);
#pragma unroll
        for (uint32_t i = 0; i < 16; i++) {
            uint32_t v = byte_of(q, i);
            y[i]      = __fadd_rn(__fmul_rn((float)(v & 15u), d), m);
            y[i + 16] = __fadd_rn(__fmul_rn((float)(v >> 4), d), m);
        }
    }
};

template <> struct Fmt<T_Q5_0> {           // gguf.c:463-488
    static constexpr uint32_t BE = 32, BB = 22, UPB = 1;
    static __device__ __forceinline__ uint32_t elem(uint32_t, uint32_t i) { return i; }
    static __device__ __forceinline__ void decode(const uint8_t* b, uint32_t, float* y) {
        float d = f16_bits(ld_u16(b));
        uint32_t hb = ld_u32(b + 2);
        uint32_t q[4];
        ld_words<4>(b + 6, q);
#pragma unroll
        for (uint32_t i = 0; i < 16; i++) {
            uint32_t v = byte_of(q, i);
            int lo = (int)((v & 15u) | (((hb >> i) & 1u) << 4)) - 16;
            int hi = (int)((v >> 4) | (((hb >> (i + 16)) & 1u) << 4)) - 16;
            y[i]      = __fmul_rn((float)lo, d);
            y[i + 16] = __fmul_rn((float)hi, d);
        }
    }
};

template <> struct Fmt<T_Q8_0> {           // gguf.c:489-503
    static constexpr uint32_t BE = 32, BB = 34, UPB = 1;
    static __device__ __forceinline__ uint32_t elem(uint32_t, uint32_t i) { return i; }
    static __device__ __forceinline__ void decode(const uint8_t* b, uint32_t, float* y) {
        float d = f16_bits(ld_u16(b));
        uint32_t q[8];
        ld_words<8>(b + 2, q);
#pragma unroll
        for (uint32_t i = 0; i < 32; i++) {
            int v = (int)(int8_t)(uint8_t)byte_of(q, i);
            y[i] = __fmul_rn((float)v, d);
        }
    }
};

// ---- K-quants: 256-element super-blocks split into 8 units.
// Q4_K unit v (g = v/2 selects the 64-element group, h = v%2 its half) covers
// qs bytes [32g+16h, +16): their low nibbles are elements 64g+16h+j and their
// high nibbles elements 64g+32+16h+j (gguf.c:504-529).
template <> struct Fmt<T_Q4_K> {
    static constexpr uint32_t BE = 256, BB = 144, UPB = 8;
    static __device__ __forceinline__ uint32_t elem(uint32_t v, uint32_t i) {
        return 64u * (v >> 1) + 16u * (v & 1u) + (i & 15u) + ((i >> 4) << 5);
    }
    static __device__ __forceinline__ void decode(const uint8_t* b, uint32_t v, float* y) {
        uint32_t hdr[4], q[4];
        ld_v4(b, hdr);                                  // d, dmin, scales[12]
        uint32_t g = v >> 1, h = v & 1u;
        ld_v4(b + 16 + 32 * g + 16 * h, q);
        float d = f16_bits(hdr[0] & 0xFFFFu), dmin = f16_bits(hdr[0] >> 16);
        uint32_t s0, m0, s1, m1;
        k4_scale_min(hdr + 1, 2 * g, &s0, &m0);
        k4_scale_min(hdr + 1, 2 * g + 1, &s1, &m1);
        float d0 = __fmul_rn(d, (float)s0), n0 = __fmul_rn(dmin, (float)m0);
        float d1 = __fmul_rn(d, (float)s1), n1 = __fmul_rn(dmin, (float)m1);
#pragma unroll
        for (uint32_t j = 0; j < 16; j++) {
            uint32_t x = byte_of(q, j);
            y[j]      = __fsub_rn(__fmul_rn(d0, (float)(x & 15u)), n0);
            y[j + 16] = __fsub_rn(__fmul_rn(d1, (float)(x >> 4)), n1);
        }
    }
};

// Q5_K: Q4_K plus a high-bit plane qh[32]; element 64g+l takes bit 2g of qh[l],
// element 64g+32+l bit 2g+1 (gguf.c:530-560).
template <> struct Fmt<T_Q5_K> {
    static constexpr uint32_t BE = 256, BB = 176, UPB = 8;
    static __device__ __forceinline__ uint32_t elem(uint32_t v, uint32_t i) {
        return 64u * (v >> 1) + 16u * (v & 1u) + (i & 15u) + ((i >> 4) << 5);
    }
    static __device__ __forceinline__ void decode(const uint8_t* b, uint32_t v, float* y) {
        uint32_t hdr[4], q[4], hb[4];
        ld_v4(b, hdr);
        uint32_t g = v >> 1, h = v & 1u;
        ld_v4(b + 16 + 16 * h, hb);
        ld_v4(b + 48 + 32 * g + 16 * h, q);
        float d = f16_bits(hdr[0] & 0xFFFFu), dmin = f16_bits(hdr[0] >> 16);
        uint32_t s0, m0, s1, m1;
        k4_scale_min(hdr + 1, 2 * g, &s0, &m0);
        k4_scale_min(hdr + 1, 2 * g + 1, &s1, &m1);
        float d0 = __fmul_rn(d, (float)s0), n0 = __fmul_rn(dmin, (float)m0);
        float d1 = __fmul_rn(d, (float)s1), n1 = __fmul_rn(dmin, (float)m1);
#pragma unroll
        for (uint32_t j = 0; j < 16; j++) {
            uint32_t x = byte_of(q, j), hh = byte_of(hb, j);
            uint32_t lo = (x & 15u) + (((hh >> (2 * g)) & 1u) << 4);
            uint32_t hi = (x >> 4) + (((hh >> (2 * g + 1)) & 1u) << 4);
            y[j]      = __fsub_rn(__fmul_rn(d0, (float)lo), n0);
            y[j + 16] = __fsub_rn(__fmul_rn(d1, (float)hi), n1);
        }
    }
};

// Q6_K unit v (H = v/4 picks the 128-element half, k = v%4 a run of 8 l values):
// for l in [8k, 8k+8) it yields elements 128H + l + 32c, c = 0..3, built from
// ql[64H + l], ql[64H + 32 + l] and qh[32H + l] with scale sc[8H + l/16 + 2c]
// (gguf.c:561-590). Output order: y[8c + j] is element 128H + 8k + j + 32c.
template <> struct Fmt<T_Q6_K> {
    static constexpr uint32_t BE = 256, BB = 210, UPB = 8;
    static __device__ __forceinline__ uint32_t elem(uint32_t v, uint32_t i) {
        return 128u * (v >> 2) + 8u * (v & 3u) + (i & 7u) + ((i >> 3) << 5);
    }
    static __device__ __forceinline__ void decode(const uint8_t* b, uint32_t v, float* y) {
        uint32_t H = v >> 2, k = v & 3u;
        uint32_t la[2], lb[2], qh[2], sw;
        ld_words<2>(b + 64 * H + 8 * k, la);
        ld_words<2>(b + 64 * H + 32 + 8 * k, lb);
        ld_words<2>(b + 128 + 32 * H + 8 * k, qh);
        float d = f16_bits(ld_u16(b + 208));
        const uint8_t* scp = b + 192 + 8 * H + (k >> 1);
        sw = ld_u32(scp);                              // sc[is], sc[is+1..3]
        uint32_t sw2 = ld_u32(scp + 4);                // sc[is+4..7]
        float sc0 = (float)(int)(int8_t)(uint8_t)(sw & 0xFFu);
        float sc1 = (float)(int)(int8_t)(uint8_t)((sw >> 16) & 0xFFu);
        float sc2 = (float)(int)(int8_t)(uint8_t)(sw2 & 0xFFu);
        float sc3 = (float)(int)(int8_t)(uint8_t)((sw2 >> 16) & 0xFFu);
        float ds0 = __fmul_rn(d, sc0), ds1 = __fmul_rn(d, sc1);
        float ds2 = __fmul_rn(d, sc2), ds3 = __fmul_rn(d, sc3);
#pragma unroll
        for (uint32_t j = 0; j < 8; j++) {
            uint32_t a = byte_of(la, j), c = byte_of(lb, j), hh = byte_of(qh, j);
            int q0 = (int)((a & 15u) | ((hh & 3u) << 4)) - 32;
            int q1 = (int)((c & 15u) | (((hh >> 2) & 3u) << 4)) - 32;
            int q2 = (int)((a >> 4) | (((hh >> 4) & 3u) << 4)) - 32;
            int q3 = (int)((c >> 4) | (((hh >> 6) & 3u) << 4)) - 32;
            y[j]      = __fmul_rn(ds0, (float)q0);
            y[j + 8]  = __fmul_rn(ds1, (float)q1);
            y[j + 16] = __fmul_rn(ds2, (float)q2);
            y[j + 24] = __fmul_rn(ds3, (float)q3);
        }
    }
};

}  // namespace lm
