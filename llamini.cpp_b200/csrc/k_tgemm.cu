// k_tgemm.cu -- tensor-core (tcgen05) dequant GEMM for a batch of input vectors.
//
// y[b][r] = sum_k W[r][k] x[b][k] for up to 64 vectors at once: the matrix
// products of batched decode (model.c:66-176 and gpt2.c's forward, once per
// sequence) and of the batch columns of the GEMV entry points. The weights stay
// in their GGUF block layout in HBM. A CTA owns 128 rows of one matrix and a K
// range, and runs five roles:
//
//   raw warp       bulk copies (cp.async.bulk, the TMA engine) of each row's
//                  bytes of the current unit -- one 256-element super-block for
//                  Q4_K/Q6_K, 64 elements otherwise -- into a ring of raw buffers
//   x warp         bulk copies of the staged inputs of each 64-element slab
//   8 dequant      decode a slab (128 rows x 64 elements) to f32 exactly as
//   warps          gguf.c:409-594 does, split each weight into fp16 hi + lo
//                  (22 significant bits) and store both in the UMMA K-major,
//                  no-swizzle layout
//   MMA warp       allocates tensor memory; one thread issues tcgen05.mma
//                  kind::f16 (M = 128, N = batch padded to 16, K = 16, f32
//                  accumulators in tensor memory): w_hi x_hi + w_hi x_lo +
//                  w_lo x_hi per 16-element step; tcgen05.commit frees each
//                  stage and finally hands the accumulators to the epilogue
//   epilogue       the dequant warps read the accumulators (tcgen05.ld) and
//                  store raw sums to part[ksplit][B][rows] in the units that
//                  bfinish_kernel (k_bgemm.cu) scales and finishes
//
// Inputs are staged by bstage_kernel as x * 2^E (per sequence) split into fp16
// hi + lo, laid out [K/8][NP/8][8 sequences][8 elements], the same UMMA layout,
// so one slab of every sequence is one contiguous bulk copy. The accumulator is
// sum w * x * 2^E; the partial stored is that times 2^-24, which bfinish
// multiplies by 2^(24 - E).
//
// UMMA shared-memory layout (K-major, no swizzle): 8 x 16-byte rows form a
// core matrix; for a tile of R rows and one 64-element slab, element (r, k)
// sits at byte (k / 8) * 16R + 16r + 2(k % 8). A 16-element K step of the tile
// starts at 32R * step; its descriptor has leading byte offset (next 8 K
// elements) 16R and stride byte offset (next 8 rows) 128.
//
// Every mbarrier wait is bounded (kTWaitNs); a wait that runs out sets an error
// bit in *err, and every role then leaves its loop, drains the copies and
// tensor-core work it started, and the CTA frees its tensor memory and exits.
#include "internal.h"
#include "mma_gemv.cuh"
#include "quant.cuh"

#include <cuda_fp16.h>

namespace lm {

constexpr uint32_t kTRows = 128;                 // MMA M: matrix rows per CTA
constexpr uint32_t kTSlab = 64;                  // K elements per stage
constexpr uint32_t kTATile = kTRows * kTSlab * 2;   // bytes of one fp16 A tile (hi or lo)
constexpr uint32_t kTDeqWarps = 8;
constexpr uint32_t kTWarpMma = 8, kTWarpRaw = 9, kTWarpX = 10;
constexpr uint32_t kTThreads = 11 * 32;
constexpr uint32_t kTRaw = 2;                    // raw buffers
constexpr uint32_t kTMaxStages = 4;
constexpr uint64_t kTWaitNs = 2000000000ull;     // 2 s
constexpr size_t kTSmemMax = 226 * 1024;

constexpr uint32_t kTErrWait = 1u;               // *err bits
constexpr uint32_t kTErrRange = 2u;              // a weight outside the fp16 range

struct TShared {
    uint64_t raw_full[kTRaw], raw_empty[kTRaw];
    uint64_t xfull[kTMaxStages], afull[kTMaxStages], sempty[kTMaxStages];
    uint64_t accf;
    uint32_t tmem;
    uint32_t abort;
};

// ---------------------------------------------------------------- primitives

__device__ __forceinline__ uint64_t tg_time() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool tg_try(uint32_t adr, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n" : "=r"(done) : "r"(adr), "r"(parity) : "memory");
    return done != 0;
}
__device__ __forceinline__ bool tg_aborted(TShared& S) { return *reinterpret_cast<volatile uint32_t*>(&S.abort) != 0; }

// Bounded wait for the phase of `bar` with this parity. False when the CTA
// aborted meanwhile, or when the wait ran out (which aborts the CTA).
__device__ bool tg_wait(TShared& S, uint64_t* bar, uint32_t parity, uint32_t* err) {
    const uint32_t adr = smem_u32(bar);
    const uint64_t t0 = tg_time();
    for (uint32_t i = 0;; i++) {
        if (tg_try(adr, parity)) return true;
        if ((i & 15u) == 15u) {
            if (tg_aborted(S)) return false;
            if (tg_time() - t0 > kTWaitNs) {
                *reinterpret_cast<volatile uint32_t*>(&S.abort) = 1u;
                if (err) atomicOr(err, kTErrWait);
                return false;
            }
        }
    }
}
// Bounded wait that ignores an abort: used to drain work already started.
__device__ void tg_drain(uint64_t* bar, uint32_t parity) {
    const uint32_t adr = smem_u32(bar);
    const uint64_t t0 = tg_time();
    while (!tg_try(adr, parity) && tg_time() - t0 < kTWaitNs) {
    }
}
// The same wait by every lane of a warp, with one outcome for the whole warp
// (the warp's later .sync.aligned instructions need it to stay converged).
__device__ __forceinline__ bool tg_wait_warp(TShared& S, uint64_t* bar, uint32_t parity, uint32_t* err) {
    return __all_sync(0xffffffffu, tg_wait(S, bar, parity, err));
}
__device__ __forceinline__ void tg_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// UMMA shared-memory descriptor, K-major without swizzle: start address,
// leading byte offset (K direction) and stride byte offset (M/N direction),
// all in 16-byte units; version 1 at bits 46-47; layout type 0 (no swizzle).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::f16: f32 accumulator (bits 4-5 = 1), A and B
// fp16 (format 0), both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t M, uint32_t N) {
    return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                 ::"r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
// The mbarrier completes one arrival once every tcgen05.mma this thread issued
// before has finished (its shared-memory reads included).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n"
                 ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// 16 consecutive f32 columns of this warp's 32 tensor-memory lanes, waited for.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n"
                 "tcgen05.wait::ld.sync.aligned;\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr) : "memory");
}

// NW little-endian words from a 2-byte aligned shared-memory address (the
// aligned words around it, funnel-shifted; reads one word past the range).
template <int NW>
__device__ __forceinline__ void sm_words(const uint8_t* p, uint32_t* w) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* b = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t s = (uint32_t)(a & 3u) * 8u;
    uint32_t prev = b[0];
#pragma unroll
    for (int i = 0; i < NW; i++) {
        const uint32_t nx = b[i + 1];
        w[i] = s ? __funnelshift_r(prev, nx, s) : prev;
        prev = nx;
    }
}

// ---------------------------------------------------------------- decoders
// Each yields the 32 weights of run j of a unit in natural K order, bit-exact
// with gguf.c. p is the row's first byte of the unit in shared memory.

// Q4_K (gguf.c:504-529): run j = sub-block j; its quants are the low (j even)
// or high (j odd) nibbles of qs[32 (j/2) + l], weight d*sc_j*q - dmin*m_j.
// d*sc_j*q is exact in f32 (at most 21 significant bits), so one fused
// multiply-add rounds exactly as the reference's multiply-then-subtract.
__device__ __forceinline__ void dq_q4k(const uint8_t* p, uint32_t j, float* w) {
    const uint4 h = *reinterpret_cast<const uint4*>(p);
    const uint4 q0 = *reinterpret_cast<const uint4*>(p + 16 + 32 * (j >> 1));
    const uint4 q1 = *reinterpret_cast<const uint4*>(p + 32 + 32 * (j >> 1));
    const uint32_t hs[3] = {h.y, h.z, h.w};
    uint32_t sc, mn;
    k4_scale_min(hs, j, &sc, &mn);
    const float d1 = __fmul_rn(f16_bits(h.x & 0xFFFFu), u2f(sc));
    const float m1 = __fmul_rn(f16_bits(h.x >> 16), u2f(mn));
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint32_t sh = (j & 1u) * 4u;
#pragma unroll
    for (int i = 0; i < 8; i++) {
#pragma unroll
        for (int b = 0; b < 4; b++) w[4 * i + b] = __fmaf_rn(d1, u2f((qw[i] >> (8 * b + sh)) & 15u), -m1);
    }
}

// Q6_K (gguf.c:561-590): run j covers elements 128H + 32c + l (H = j/4,
// c = j%4, l < 32): low 4 bits from nibble c/2 of ql[64H + 32(c%2) + l], high
// 2 bits from bits 2c of qh[32H + l], scale sc[8H + 2c + l/16]; weight
// (d*sc)*(q - 32), exact in f32.
__device__ __forceinline__ void dq_q6k(const uint8_t* p, uint32_t j, float* w) {
    const uint32_t H = j >> 2, c = j & 3u;
    uint32_t ql[8], qh[8];
    sm_words<8>(p + 64 * H + 32 * (c & 1u), ql);
    sm_words<8>(p + 128 + 32 * H, qh);
    const uint32_t sw = lds_u32(p + 192 + 8 * H + 2 * c);
    const float d = f16_bits(lds_u16(p + 208));
    const float ds0 = __fmul_rn(d, (float)(int)(int8_t)(uint8_t)(sw & 0xFFu));
    const float ds1 = __fmul_rn(d, (float)(int)(int8_t)(uint8_t)((sw >> 8) & 0xFFu));
    const uint32_t ns = (c >> 1) * 4u, hs = 2u * c;
#pragma unroll
    for (int l = 0; l < 32; l++) {
        const uint32_t nib = (ql[l >> 2] >> (8 * (l & 3) + ns)) & 15u;
        const uint32_t hb = (qh[l >> 2] >> (8 * (l & 3) + hs)) & 3u;
        const float q = __uint_as_float(0x4B000000u | (nib | (hb << 4))) - 8388640.0f;   // (q6 - 32), exact
        w[l] = __fmul_rn(l < 16 ? ds0 : ds1, q);
    }
}

// Q8_0 (gguf.c:489-503): run j = block j of the unit, weight q * d.
__device__ __forceinline__ void dq_q80(const uint8_t* p, uint32_t j, float* w) {
    const uint8_t* b = p + 34 * j;
    const float d = f16_bits(lds_u16(b));
    uint32_t q[8];
    sm_words<8>(b + 2, q);
#pragma unroll
    for (int i = 0; i < 32; i++) w[i] = __fmul_rn((float)(int)(int8_t)(uint8_t)((q[i >> 2] >> (8 * (i & 3))) & 0xFFu), d);
}

// Q4_0 (gguf.c:427-444): run j = block j; element l < 16 is the low nibble of
// qs[l], element l + 16 its high nibble; weight (q - 8) * d.
__device__ __forceinline__ void dq_q40(const uint8_t* p, uint32_t j, float* w) {
    const uint8_t* b = p + 18 * j;
    const float d = f16_bits(lds_u16(b));
    uint32_t q[4];
    sm_words<4>(b + 2, q);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const uint32_t v = (q[i >> 2] >> (8 * (i & 3))) & 0xFFu;
        w[i] = __fmul_rn(u2f(v & 15u) - 8.0f, d);
        w[i + 16] = __fmul_rn(u2f(v >> 4) - 8.0f, d);
    }
}

// Split 32 weights into fp16 hi and lo and store them as four 8-element
// K slices (16 bytes each, 16R bytes apart) of the A tiles.
__device__ __forceinline__ void tstore(uint8_t* ahi, uint8_t* alo, const float* w) {
#pragma unroll
    for (int sl = 0; sl < 4; sl++) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float a = w[8 * sl + 2 * q], b = w[8 * sl + 2 * q + 1];
            const __half2 hh = __floats2half2_rn(a, b);
            const float2 hf = __half22float2(hh);
            const __half2 ll = __floats2half2_rn(__fsub_rn(a, hf.x), __fsub_rn(b, hf.y));
            h[q] = *reinterpret_cast<const uint32_t*>(&hh);
            l[q] = *reinterpret_cast<const uint32_t*>(&ll);
        }
        *reinterpret_cast<uint4*>(ahi + sl * (16 * kTRows)) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(alo + sl * (16 * kTRows)) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// ---------------------------------------------------------------- kernel

__host__ __device__ __forceinline__ uint32_t tg_stage_bytes(uint32_t np) { return 2 * kTATile + 2 * (128 * np); }

__global__ void __launch_bounds__(kTThreads, 1) tgemm_kernel(const __grid_constant__ TGemmArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ TShared S;
    uint32_t sgi = 0;
#pragma unroll
    for (uint32_t i = 1; i < 3; i++)
        if (i < a.nseg && blockIdx.x >= a.seg[i].rb0) sgi = i;
    const TSeg& G = a.seg[sgi];
    const uint32_t row0 = (blockIdx.x - G.rb0) * kTRows;
    const uint32_t ks = blockIdx.y;
    const uint32_t units = a.K / a.ue;
    const uint32_t u0 = ks * a.ups, u1 = min(units, u0 + a.ups);
    const uint32_t sl0 = u0 * (a.ue / kTSlab), sl1 = u1 * (a.ue / kTSlab);   // slabs [sl0, sl1)
    const uint32_t ru = G.ru, spr = ru / kTSlab;                             // slabs per raw unit
    const uint32_t ur0 = sl0 / spr;
    const uint32_t NS = a.stages, NP = a.NP;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;

    uint8_t* const abase = smem;                                      // NS x (A hi, A lo)
    uint8_t* const xbase = smem + NS * 2 * kTATile;                   // NS x (x hi, x lo)
    uint8_t* const rbase = xbase + NS * 2 * (128 * NP);               // kTRaw raw buffers

    if (tid == 0) {
        for (uint32_t i = 0; i < kTRaw; i++) { mbar_init(&S.raw_full[i], 1); mbar_init(&S.raw_empty[i], kTDeqWarps); }
        for (uint32_t i = 0; i < NS; i++) {
            mbar_init(&S.xfull[i], 1);
            mbar_init(&S.afull[i], kTDeqWarps);
            mbar_init(&S.sempty[i], 1);
        }
        mbar_init(&S.accf, 1);
        S.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        fence_async_smem();
    }
    if (warp == kTWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n"
                     ::"r"(smem_u32(&S.tmem)), "r"(a.tcols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem;

    if (warp == kTWarpRaw) {
        // ------------------------------------------------ raw weight bytes
        const uint32_t nru = (sl1 - sl0) / spr;
        uint32_t armed = 0;                                            // raw units issued
        for (uint32_t lr = 0; lr < nru; lr++) {
            const uint32_t buf = lr % kTRaw, t = lr / kTRaw;
            if (t > 0 && !tg_wait_warp(S, &S.raw_empty[buf], (t - 1) & 1u, a.err)) break;
            const uint64_t ur = ur0 + lr;
            uint8_t* dst = rbase + buf * a.raw_bytes;
            uint32_t len[4], tot = 0;
            uint64_t src[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t r = lane + 32u * i;
                len[i] = 0;
                src[i] = 0;
                if (row0 + r < G.rows) {
                    const uint64_t o = (uint64_t)(row0 + r) * G.row_bytes + ur * G.ub;
                    src[i] = o & ~uint64_t(15);
                    len[i] = (uint32_t)(((o + G.ub + 15) & ~uint64_t(15)) - src[i]);
                    tot += len[i];
                }
            }
            tot = __reduce_add_sync(0xffffffffu, tot);
            if (lane == 0) mbar_expect_tx(&S.raw_full[buf], tot);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; i++)
                if (len[i]) bulk_g2s(dst + (lane + 32u * i) * G.rrs, G.w + src[i], len[i], &S.raw_full[buf]);
            armed = lr + 1;
        }
        // every issued copy has landed before the CTA can exit
        if (lane == 0)
            for (uint32_t lr = (armed > kTRaw ? armed - kTRaw : 0); lr < armed; lr++)
                tg_drain(&S.raw_full[lr % kTRaw], (lr / kTRaw) & 1u);
        __syncwarp();
    } else if (warp == kTWarpX) {
        // ------------------------------------------------ staged inputs
        if (lane == 0) {
            const uint32_t xb = 128 * NP;                               // bytes of one half-slab
            uint32_t armed = 0;
            for (uint32_t i = 0; i < sl1 - sl0; i++) {
                const uint32_t si = i % NS, t = i / NS;
                if (t > 0 && !tg_wait(S, &S.sempty[si], (t - 1) & 1u, a.err)) break;
                const uint64_t off = (uint64_t)(sl0 + i) * (kTSlab * NP);   // halves
                uint8_t* dst = xbase + si * 2 * xb;
                mbar_expect_tx(&S.xfull[si], 2 * xb);
                bulk_g2s(dst, a.xh + off, xb, &S.xfull[si]);
                bulk_g2s(dst + xb, a.xl + off, xb, &S.xfull[si]);
                armed = i + 1;
            }
            for (uint32_t i = (armed > NS ? armed - NS : 0); i < armed; i++) tg_drain(&S.xfull[i % NS], (i / NS) & 1u);
        }
        __syncwarp();
    } else if (warp == kTWarpMma) {
        // ------------------------------------------------ tensor-core issue
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(kTRows, NP);
            const bool lo = G.type != T_F16;                            // F16 weights are exact in hi
            uint32_t issued = 0;
            for (uint32_t i = 0; i < sl1 - sl0; i++) {
                const uint32_t si = i % NS, t = i / NS;
                if (!tg_wait(S, &S.afull[si], t & 1u, a.err) || !tg_wait(S, &S.xfull[si], t & 1u, a.err)) break;
                tc_fence_after();
                const uint32_t ah = smem_u32(abase + si * 2 * kTATile), al = ah + kTATile;
                const uint32_t xh = smem_u32(xbase + si * 2 * (128 * NP)), xl = xh + 128 * NP;
#pragma unroll
                for (uint32_t kk = 0; kk < kTSlab / 16; kk++) {
                    const uint64_t dah = umma_desc(ah + kk * 32 * kTRows, 16 * kTRows, 128);
                    const uint64_t dal = umma_desc(al + kk * 32 * kTRows, 16 * kTRows, 128);
                    const uint64_t dxh = umma_desc(xh + kk * 32 * NP, 16 * NP, 128);
                    const uint64_t dxl = umma_desc(xl + kk * 32 * NP, 16 * NP, 128);
                    umma_f16(tmem, dah, dxh, idesc, (i | kk) != 0);
                    umma_f16(tmem, dah, dxl, idesc, 1);
                    if (lo) umma_f16(tmem, dal, dxh, idesc, 1);
                }
                umma_commit(&S.sempty[si]);
                issued = i + 1;
            }
            umma_commit(&S.accf);
            if (issued < sl1 - sl0) tg_drain(&S.accf, 0);               // aborted: let issued MMAs finish
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ dequant, then epilogue
        const uint32_t r = tid & (kTRows - 1), c = tid >> 7;           // row, 32-element run of the slab
        const bool valid = row0 + r < G.rows;
        uint32_t rng = 0;
        for (uint32_t i = 0; i < sl1 - sl0; i++) {
            const uint32_t s = sl0 + i, si = i % NS, t = i / NS;
            const uint32_t lr = s / spr - ur0, buf = lr % kTRaw, first = s % spr == 0;
            if (first && !tg_wait_warp(S, &S.raw_full[buf], (lr / kTRaw) & 1u, a.err)) break;
            if (t > 0 && !tg_wait_warp(S, &S.sempty[si], (t - 1) & 1u, a.err)) break;
            uint8_t* ahi = abase + si * 2 * kTATile + c * 4 * (16 * kTRows) + 16 * r;
            uint8_t* alo = ahi + kTATile;
            if (!valid) {
#pragma unroll
                for (int sl = 0; sl < 4; sl++) {
                    *reinterpret_cast<uint4*>(ahi + sl * (16 * kTRows)) = make_uint4(0, 0, 0, 0);
                    *reinterpret_cast<uint4*>(alo + sl * (16 * kTRows)) = make_uint4(0, 0, 0, 0);
                }
            } else {
                const uint64_t o = (uint64_t)(row0 + r) * G.row_bytes + (uint64_t)(s / spr) * G.ub;
                const uint8_t* p = rbase + buf * a.raw_bytes + r * G.rrs + (uint32_t)(o & 15u);
                const uint32_t j = (s % spr) * 2 + c;                  // run within the raw unit
                if (G.type == T_F16) {
                    const uint8_t* b = p + 64 * j;
#pragma unroll
                    for (int sl = 0; sl < 4; sl++) {
                        *reinterpret_cast<uint4*>(ahi + sl * (16 * kTRows)) = *reinterpret_cast<const uint4*>(b + 16 * sl);
                        *reinterpret_cast<uint4*>(alo + sl * (16 * kTRows)) = make_uint4(0, 0, 0, 0);
                    }
                } else {
                    float w[32];
                    switch (G.type) {
                    case T_Q4_K: dq_q4k(p, j, w); break;
                    case T_Q6_K: dq_q6k(p, j, w); break;
                    case T_Q8_0: dq_q80(p, j, w); break;
                    default: dq_q40(p, j, w); break;
                    }
                    float m = 0.f;
#pragma unroll
                    for (int e = 0; e < 32; e++) m = fmaxf(m, fabsf(w[e]));
                    if (!(m <= 65504.f)) rng = 1;                      // overflow (or NaN) in fp16
                    tstore(ahi, alo, w);
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                tg_arrive(&S.afull[si]);
                if ((s + 1) % spr == 0) tg_arrive(&S.raw_empty[buf]);
            }
        }
        if (rng && a.err) atomicOr(a.err, kTErrRange);
        // epilogue: warp w reads lanes 32 (w % 4) .. +31 (its rows), column
        // chunks of 16 starting at chunk w / 4, step 2
        const bool ok = tg_wait_warp(S, &S.accf, 0, a.err);
        tc_fence_after();
        if (ok) {
            const uint32_t q = warp & 3u;
            const uint32_t row = row0 + 32 * q + lane;
            float* part = G.part + (uint64_t)ks * a.B * G.rows;
            for (uint32_t cc = warp >> 2; 16 * cc < NP; cc += 2) {
                uint32_t v[16];
                tmem_ld16(tmem + ((32u * q) << 16) + 16 * cc, v);
                if (row < G.rows) {
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        const uint32_t b = 16 * cc + e;
                        if (b < a.B) part[(uint64_t)b * G.rows + row] = __uint_as_float(v[e]) * 5.9604644775390625e-08f;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTWarpMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(a.tcols) : "memory");
    }
}

// ---------------------------------------------------------------- host side

bool tgemm_type(uint32_t t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0 || t == T_Q4_0 || t == T_F16; }

static uint32_t tg_ru(uint32_t type) { return (type == T_Q4_K || type == T_Q6_K) ? 256u : 64u; }
static uint32_t tg_ub(uint32_t type) {
    switch (type) {
    case T_Q4_K: return 144;
    case T_Q6_K: return 210;
    case T_Q8_0: return 68;     // two 32-element blocks
    case T_Q4_0: return 36;
    default: return 128;        // F16
    }
}

size_t tgemm_smem(const TGemmArgs& a) { return (size_t)a.stages * tg_stage_bytes(a.NP) + (size_t)kTRaw * a.raw_bytes; }

bool tgemm_init() {
    return LM_CUDA(cudaFuncSetAttribute(tgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTSmemMax));
}

// Fill the launch geometry of `a` (segments, B, K set by the caller). False (no
// error set) when a segment's format or shape has no tensor-core path.
bool tgemm_plan(TGemmArgs& a, uint32_t sms) {
    if (a.B == 0 || a.B > 64 || a.nseg == 0 || a.nseg > 3 || a.K % kTSlab != 0 || sms == 0) return false;
    a.NP = (a.B + 15) & ~15u;
    bool kq = false;
    uint32_t rbs = 0, raw = 0;
    for (uint32_t i = 0; i < a.nseg; i++) {
        TSeg& S = a.seg[i];
        if (!tgemm_type(S.type) || S.rows == 0) return false;
        if (reinterpret_cast<uintptr_t>(S.w) % 16 != 0) return false;
        if (S.row_bytes != type_bytes(S.type, a.K)) return false;
        kq = kq || S.type == T_Q4_K || S.type == T_Q6_K;
        S.ru = tg_ru(S.type);
        S.ub = tg_ub(S.type);
        uint32_t rrs = (S.ub + 15 + 4 + 15) & ~15u;        // alignment delta + one word of over-read
        if ((rrs / 16) % 2 == 0) rrs += 16;                // odd count of 16-byte units: rows over all banks
        S.rrs = rrs;
        raw = raw > kTRows * rrs ? raw : kTRows * rrs;
        S.rb0 = rbs;
        rbs += (S.rows + kTRows - 1) / kTRows;
    }
    a.ue = a.K % 256 == 0 ? 256u : 64u;
    if (kq && a.ue != 256) return false;
    a.raw_bytes = raw;
    a.stages = 0;
    for (uint32_t ns = kTMaxStages; ns >= 2; ns--)
        if ((size_t)ns * tg_stage_bytes(a.NP) + (size_t)kTRaw * raw <= kTSmemMax) { a.stages = ns; break; }
    if (a.stages == 0) return false;
    a.tcols = 32;
    while (a.tcols < a.NP) a.tcols *= 2;
    // K split: the fewest units per CTA among the splits whose waves x units
    // per CTA is smallest (one CTA per SM)
    const uint32_t units = a.K / a.ue;
    uint32_t best = 0, best_cost = 0xFFFFFFFFu;
    for (uint32_t ups = 1; ups <= units; ups++) {
        const uint32_t ks = (units + ups - 1) / ups;
        if (ups > 1 && (units + ups - 2) / (ups - 1) == ks) continue;   // same split as a smaller ups
        const uint32_t waves = (rbs * ks + sms - 1) / sms;
        const uint32_t cost = waves * ups;
        if (cost <= best_cost) { best_cost = cost; best = ups; }
    }
    a.ups = best;
    a.ksplit = (units + best - 1) / best;
    a.rblocks = rbs;
    return true;
}

bool launch_tgemm(const TGemmArgs& a, cudaStream_t st) {
    tgemm_kernel<<<dim3(a.rblocks, a.ksplit), kTThreads, tgemm_smem(a), st>>>(a);
    return LM_CUDA(cudaGetLastError());
}

}  // namespace lm
