// k_tgemm.cu -- tensor-core (tcgen05) dequant GEMM for a batch of input vectors.
//
// y[b][r] = sum_k W[r][k] x[b][k] for up to 64 vectors at once: the matrix
// products of batched decode (model.c:66-176 and gpt2.c's forward, once per
// sequence) and of the batch columns of the GEMV entry points. The weights stay
// in their GGUF block layout in HBM. A tile is 128 rows of one matrix x one K
// range; one persistent CTA per SM walks its tiles with five roles:
//
//   raw warp       bulk copies (TMA, cp.async.bulk.tensor) of each row's
//                  bytes of the current unit -- one 256-element super-block for
//                  K-quants, eight 32-element blocks or 64 elements otherwise --
//                  into a ring of raw buffers
//   x warp         bulk copies of the staged inputs of each 64-element slab
//                  (and of the super-block's sums for TG_KMIN tiles)
//   16 dequant     two groups of 8 decode alternate slabs (128 rows x 64
//   warps          elements) from the raw units into the A operand in tensor
//                  memory (below)
//   3 MMA warps    one allocates tensor memory; one thread per warp issues
//                  tcgen05.mma kind::f16 (M = 128, N = batch padded to 16,
//                  K = 16, f32 accumulators in tensor memory) of one chain --
//                  A_hi x_hi, A_hi x_lo, A_lo x_hi -- each into its own
//                  accumulator so their MMAs overlap in the tensor pipe;
//                  tcgen05.commit frees each stage and hands each finished tile
//                  (two accumulator sets, used by alternate tiles) to the epilogue
//   4 epilogue     read the accumulators (tcgen05.ld), add the chains and
//   warps          store raw sums to part[ksplit][B][rows] in the units that
//                  bfinish_kernel (k_bgemm.cu) scales and finishes
//
// The A operand (fp16 hi + lo, 22 significant bits), per format:
//   TG_PLAIN  each weight as gguf.c:409-503 and 561-590 decode it: Q8_0, Q4_0,
//             Q5_0 (q - z) * d and Q6_K (d sc)(q - 32) from exact fp16 pair
//             arithmetic (hi the rounded product, lo the remainder); Q4_1 and
//             F16 from the f32 weight
//   TG_KMIN   (Q4_K, Q5_K, gguf.c:504-560: w = d sc_j q - dmin m_j) A = d (sc_j q),
//             the integer sc_j q from one exact fp16 fused multiply-add; the
//             -dmin m_j terms enter through two more K = 16 MMAs per
//             super-block (chain 2): A = -32 dmin m_j (hi, lo) from shared
//             memory against the staged 32-element sums of x * 2^-5 (hi, lo)
// The products are exact and accumulate in f32, so the sums differ from the
// reference's f32 dot products only by rounding order (and, for K-quants, by
// the reference's rounding of each weight to f32).
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
//
// Launched with programmatic dependent launch: the set-up, the tensor-memory
// allocation, the raw warp's weight copies and the decode of the first units
// may run while the kernel that stages x is still finishing; the x warp waits
// for it (griddepcontrol.wait) before its first copy, and the epilogue before
// it writes partial sums that the previous finish may still be reading.
#include "internal.h"
#include "mma_gemv.cuh"
#include "pdl.cuh"
#include "quant.cuh"

#include <cuda_fp16.h>
#include <cudaTypedefs.h>

namespace lm {

constexpr uint32_t kTRows = 128;                 // MMA M: matrix rows per CTA
constexpr uint32_t kTSlab = 64;                  // K elements per stage
// Tensor memory (512 columns): two accumulator sets (used by alternate tiles)
// of three independent f32 accumulators (one per MMA chain), 64 columns each,
// so the MMAs of a K step do not wait on one another; then kTNA stages of the
// A slab, 32 columns hi and 32 lo (fp16 pairs: column c holds K elements 2c
// and 2c + 1).
constexpr uint32_t kTAccW = 64;                  // columns per accumulator (NP <= 64)
// Build-time pipeline shape (-D overrides): accumulator sets, A stages and
// dequant groups. The defaults measured fastest on llama_1b batch 64; one set
// with four A stages, or one dequant group, were within a few percent.
#ifndef LM_TG_SETS
#define LM_TG_SETS 2
#endif
#ifndef LM_TG_NA
#define LM_TG_NA 2
#endif
constexpr uint32_t kTSetCols = 3 * kTAccW;
constexpr uint32_t kTSets = LM_TG_SETS;          // accumulator sets (alternate tiles)
constexpr uint32_t kTACol0 = kTSets * kTSetCols; // first A-stage column
constexpr uint32_t kTACols = 64;
constexpr uint32_t kTNA = LM_TG_NA;              // A stages in tensor memory
constexpr uint32_t kTCols = 512;
static_assert(kTACol0 + kTNA * kTACols <= kTCols, "tensor memory: accumulators and A stages exceed 512 columns");
#ifndef LM_TG_GROUPS
#define LM_TG_GROUPS 2
#endif
constexpr uint32_t kTGroupWarps = 8;            // one dequant group: a slab's 128 rows x 2 runs
constexpr uint32_t kTGroups = LM_TG_GROUPS;     // groups decode slabs i with i % kTGroups == group
constexpr uint32_t kTDeqWarps = kTGroups * kTGroupWarps;
constexpr uint32_t kTEpiWarps = 4;              // tensor-memory lanes 0-127
constexpr uint32_t kTIssuers = 3;               // one issuing thread per accumulator chain
constexpr uint32_t kTWarpEpi = kTDeqWarps, kTWarpMma = kTWarpEpi + kTEpiWarps, kTWarpRaw = kTWarpMma + kTIssuers,
                   kTWarpX = kTWarpRaw + 1;
constexpr uint32_t kTThreads = (kTWarpX + 1) * 32;
constexpr uint32_t kTAlign = 1024;              // dynamic shared memory aligned up to this
constexpr uint32_t kTSlack = 64;                // after the raw buffers: the decoders' word reads
                                                // may run up to 8 bytes past a row's last byte
constexpr uint32_t kTRaw = 4;                    // raw buffers
constexpr uint32_t kTMinBytes = 2 * 2 * 16 * 128;    // two K = 16 A tiles of 128 rows (fp16)
constexpr uint32_t kTMaxStages = 4;              // x stages in shared memory
constexpr uint64_t kTWaitNs = 2000000000ull;     // 2 s
constexpr size_t kTSmemMax = 226 * 1024;

constexpr uint32_t kTErrWait = 1u;               // *err bits
constexpr uint32_t kTErrRange = 2u;              // a weight outside the fp16 range

struct TShared {
    uint64_t raw_full[kTRaw], raw_empty[kTRaw];
    uint64_t xfull[kTMaxStages], xempty[kTMaxStages];   // x slab landed / read by its MMAs
    uint64_t afull[kTNA], aempty[kTNA];                  // A slab in tensor memory / read by its MMAs
    uint64_t accf[kTSets], acce[kTSets];   // accumulator full (MMA -> epilogue) / empty
    uint64_t mdone;                     // every MMA of the CTA finished
    uint32_t tmem;
    uint32_t abort;
};

// ---------------------------------------------------------------- primitives

__device__ __forceinline__ uint64_t tg_time() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
// One test of the phase; a thread whose phase is not complete yet is suspended
// in hardware (up to kTSuspendNs, resuming when the phase completes) instead of
// spinning, so waiting roles leave the issue slots to the dequant warps.
constexpr uint32_t kTSuspendNs = 1000000;
__device__ __forceinline__ bool tg_try(uint32_t adr, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n" : "=r"(done) : "r"(adr), "r"(parity), "n"(kTSuspendNs) : "memory");
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
// A 16-bit field of the weights in global memory (2-byte aligned).
__device__ __forceinline__ uint32_t ldg_u16(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned short*>(p)); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// TMA tiled load of a 2-D box (x in elements of the map, y in rows) into
// shared memory, completing on `bar`. No multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}
// 16-byte asynchronous copy (both addresses 16-byte aligned); the executing
// thread's copies are tracked by tg_cpa_arrive.
__device__ __forceinline__ void tg_cpa16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// One arrival on `bar` once every cp.async this thread issued has landed.
__device__ __forceinline__ void tg_cpa_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

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

// 16 consecutive f32 columns of this warp's 32 tensor-memory lanes, not yet
// waited for: the registers are valid after tmem_wait_ld.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr) : "memory");
}
// Every tcgen05.ld of this thread has completed; `r` (the registers they
// wrote) is tied in so no use is scheduled above the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t* r) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :: "memory");
}

// This warp's 32 tensor-memory lanes, 16 consecutive columns, from registers.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
                   "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
// D (+)= A B with A (128 x 16 fp16) in tensor memory and B in shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
                 ::"r"(d), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
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

// fp16 pair arithmetic on raw bits, round to nearest, subnormals kept.
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hadd2u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// Two bytes of `word` (PRMT selector sel: 0x4140 bytes 0 and 1, 0x4342 bytes 2
// and 3) as the fp16 pair 1024 + byte: 0x64 above a byte is 2^10 with the byte
// as the low mantissa bits.
__device__ __forceinline__ uint32_t h1024(uint32_t word, uint32_t sel) { return __byte_perm(word, 0x64u, sel); }
__device__ __forceinline__ uint32_t h2pair(float v) {
    const __half h = __float2half_rn(v);
    const uint32_t b = __half_as_ushort(h);
    return b | (b << 16);
}
constexpr uint32_t kHNeg = 0x80008000u;          // sign bits of an fp16 pair
// Exact fp16 hi + lo of integers t*s (t, s fp16 pairs whose exact products have
// at most 22 significant bits): hi the rounded product, lo the remainder.
__device__ __forceinline__ void hilo(uint32_t t, uint32_t s, uint32_t& hi, uint32_t& lo) {
    hi = hmul2u(t, s);
    lo = hfma2u(t, s, hi ^ kHNeg);
}

// This warp's 32 tensor-memory lanes, 8 consecutive columns, from registers.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

// ---------------------------------------------------------------- decoders
// Each yields the 32 weights of run j of a unit -- 32 consecutive K elements,
// bit-exact with gguf.c -- as fp16 hi and lo pairs: h[i] and l[i] hold
// elements 2i (low half) and 2i + 1 (high half), the order of a row's A
// operand in tensor memory. p is the row's first byte of the unit in shared
// memory. Returns false when a weight of the run may leave the fp16 range
// (checked once per run from its scales).

// 2^23 + b for a byte b < 256 as f32 bits: the byte placed into the mantissa.
__device__ __forceinline__ float magic_byte(uint32_t word, uint32_t sel) {
    return __uint_as_float(__byte_perm(word, 0x4B000000u, sel));
}

// Eight weights to four hi pairs and four lo pairs.
__device__ __forceinline__ void st8(uint32_t* h, uint32_t* l, const float* w) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const __half2 hh = __floats2half2_rn(w[2 * q], w[2 * q + 1]);
        const float2 hf = __half22float2(hh);
        const __half2 ll = __floats2half2_rn(__fsub_rn(w[2 * q], hf.x), __fsub_rn(w[2 * q + 1], hf.y));
        h[q] = *reinterpret_cast<const uint32_t*>(&hh);
        l[q] = *reinterpret_cast<const uint32_t*>(&ll);
    }
}

// 6-bit scale of sub-block j of a K-quant super-block (gguf.c:391-399) from
// its first 16 bytes (d, dmin, scale bytes 0-11).
__device__ __forceinline__ uint32_t k4_scale(const uint4& hd, uint32_t j) {
    const uint32_t sh8 = 8u * (j & 3u);
    return j < 4 ? (hd.y >> sh8) & 63u : ((hd.w >> sh8) & 15u) | (((hd.y >> (sh8 + 6)) & 3u) << 4);
}
// The min terms of a K-quant super-block (gguf.c:391-399, the eight 6-bit
// mins m0..m7): -32 dmin m_j as exact fp16 hi + lo pairs (m0, m1) .. (m6, m7),
// the A rows of the two min MMAs (the staged sums are x * 2^-5 per 32 elements).
__device__ __forceinline__ bool k4_mins(const uint8_t* p, uint32_t* mh, uint32_t* ml) {
    const uint4 hd = *reinterpret_cast<const uint4*>(p);
    const uint32_t lo = hd.z & 0x3F3F3F3Fu;                                        // m0 .. m3
    const uint32_t hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);  // m4 .. m7
    const uint32_t n1024 = 0xE400E400u;                                            // -1024, -1024
    const float dmin = f16_bits(hd.x >> 16);
    const uint32_t dm2 = h2pair(-32.0f * dmin);
    hilo(hadd2u(h1024(lo, 0x4140u), n1024), dm2, mh[0], ml[0]);
    hilo(hadd2u(h1024(lo, 0x4342u), n1024), dm2, mh[1], ml[1]);
    hilo(hadd2u(h1024(hi, 0x4140u), n1024), dm2, mh[2], ml[2]);
    hilo(hadd2u(h1024(hi, 0x4342u), n1024), dm2, mh[3], ml[3]);
    return fabsf(dmin) * 2016.0f <= 65504.0f;
}

// Q4_K (gguf.c:504-529), TG_KMIN: run j = sub-block j; its quants are the low
// (j even) or high (j odd) nibbles of qs[32 (j/2) + l]. The integer sc_j * q
// comes from 1024 + q (low nibbles) or 1024 + 16q (high nibbles, not shifted
// down) by one exact fp16 fused multiply-add -- (1024 + q) sc - 1024 sc or
// (1024 + 16q) sc/16 - 64 sc -- and A = d (sc_j q) as its exact fp16 hi + lo.
__device__ __forceinline__ bool dqf_q4k(const uint8_t* p, uint32_t j, uint32_t* h, uint32_t* l) {
    const uint4 hd = *reinterpret_cast<const uint4*>(p);
    const float sc = u2f(k4_scale(hd, j));
    const bool odd = (j & 1u) != 0;
    const uint32_t s2 = h2pair(odd ? sc * 0.0625f : sc), c2 = h2pair(odd ? -64.0f * sc : -1024.0f * sc);
    const uint32_t dh = hd.x & 0xFFFFu, d2 = dh | (dh << 16);
    const uint32_t mask = odd ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
    const uint8_t* qp = p + 16 + 32 * (j >> 1);
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const uint4 q = *reinterpret_cast<const uint4*>(qp + 16 * half);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t n = qw[e] & mask;
            const int i = 8 * half + 2 * e;
            hilo(hfma2u(h1024(n, 0x4140u), s2, c2), d2, h[i], l[i]);
            hilo(hfma2u(h1024(n, 0x4342u), s2, c2), d2, h[i + 1], l[i + 1]);
        }
    }
    return fabsf(f16_bits(dh)) * 945.0f <= 65504.0f;
}

// Q5_K (gguf.c:530-560), TG_KMIN: Q4_K plus a high-bit plane: run j's quants
// are nibble j % 2 of qs[32 (j/2) + l] with bit j of qh[l] as bit 4;
// A = d (sc_j q) as exact fp16 hi + lo.
__device__ __forceinline__ bool dqf_q5k(const uint8_t* p, uint32_t j, uint32_t* h, uint32_t* l) {
    const uint4 hd = *reinterpret_cast<const uint4*>(p);
    const float sc = u2f(k4_scale(hd, j));
    const uint32_t s2 = h2pair(sc), c2 = h2pair(-1024.0f * sc);
    const uint32_t dh = hd.x & 0xFFFFu, d2 = dh | (dh << 16);
    const uint8_t* qp = p + 48 + 32 * (j >> 1);
    const uint8_t* hp = p + 16;
    const uint32_t sh = (j & 1u) * 4u;
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const uint4 q = *reinterpret_cast<const uint4*>(qp + 16 * half);
        const uint4 hq = *reinterpret_cast<const uint4*>(hp + 16 * half);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        const uint32_t hw[4] = {hq.x, hq.y, hq.z, hq.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t n = ((qw[e] >> sh) & 0x0F0F0F0Fu) | (((hw[e] >> j) & 0x01010101u) << 4);
            const int i = 8 * half + 2 * e;
            hilo(hfma2u(h1024(n, 0x4140u), s2, c2), d2, h[i], l[i]);
            hilo(hfma2u(h1024(n, 0x4342u), s2, c2), d2, h[i + 1], l[i + 1]);
        }
    }
    return fabsf(f16_bits(dh)) * 1953.0f <= 65504.0f;
}

// Q6_K (gguf.c:561-590): run j covers elements 128H + 32c + l (H = j/4, c = j%4,
// l < 32): low 4 bits from nibble c/2 of ql[64H + 32(c%2) + l], high 2 bits
// from bits 2c of qh[32H + l], scale sc[8H + 2c + l/16]; weight (d sc)(q - 32)
// with d sc exact in f32 and split into fp16 hi + lo, q - 32 exact in fp16
// ((1024 + q) - 1056): hi = (q-32) ds_hi rounded, lo = (q-32) ds_lo plus the
// exact remainder of hi, rounded once (22 significant bits in all).
__device__ __forceinline__ bool dqf_q6k(const uint8_t* p, uint32_t j, uint32_t* h, uint32_t* l) {
    const uint32_t H = j >> 2, c = j & 3u;
    uint32_t ql[8], qh[8];
    sm_words<8>(p + 64 * H + 32 * (c & 1u), ql);
    sm_words<8>(p + 128 + 32 * H, qh);
    const uint32_t sw = lds_u32(p + 192 + 8 * H + 2 * c);
    const float d = f16_bits(lds_u16(p + 208));
    const float ds0 = __fmul_rn(d, (float)(int)(int8_t)(uint8_t)(sw & 0xFFu));
    const float ds1 = __fmul_rn(d, (float)(int)(int8_t)(uint8_t)((sw >> 8) & 0xFFu));
    const uint32_t h0 = h2pair(ds0), h1 = h2pair(ds1);
    const uint32_t l0 = h2pair(ds0 - __half2float(__ushort_as_half((unsigned short)(h0 & 0xFFFFu))));
    const uint32_t l1 = h2pair(ds1 - __half2float(__ushort_as_half((unsigned short)(h1 & 0xFFFFu))));
    const uint32_t ns = (c >> 1) * 4u, hs = 2u * c;
    const uint32_t n1056 = 0xE420E420u;                                            // -1056, -1056
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t dh = i < 4 ? h0 : h1, dl = i < 4 ? l0 : l1;
        const uint32_t q6 = ((ql[i] >> ns) & 0x0F0F0F0Fu) | (((qh[i] >> hs) & 0x03030303u) << 4);
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const uint32_t t = hadd2u(h1024(q6, k ? 0x4342u : 0x4140u), n1056);
            const uint32_t hi = hmul2u(t, dh);
            h[2 * i + k] = hi;
            l[2 * i + k] = hfma2u(t, dl, hfma2u(t, dh, hi ^ kHNeg));
        }
    }
    return fmaxf(fabsf(ds0), fabsf(ds1)) * 32.0f <= 65504.0f;
}

// Q8_0 (gguf.c:489-503), TG_PLAIN: run j = block j of the unit, weight q * d:
// q from (1024 + (q ^ 0x80)) - 1152, then hi = q * d rounded and lo = the
// remainder, the same fp16 pair as rounding the exact f32 weight.
__device__ __forceinline__ bool dq_q80(const uint8_t* p, uint32_t j, uint32_t* h, uint32_t* l) {
    const uint8_t* b = p + 34 * j;
    const uint32_t dh = lds_u16(b);
    const uint32_t d2 = dh | (dh << 16);
    uint32_t q[8];
    sm_words<8>(b + 2, q);
    const uint32_t n1152 = 0xE480E480u;                                            // -1152, -1152
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t u = q[i] ^ 0x80808080u;
        hilo(hadd2u(h1024(u, 0x4140u), n1152), d2, h[2 * i], l[2 * i]);
        hilo(hadd2u(h1024(u, 0x4342u), n1152), d2, h[2 * i + 1], l[2 * i + 1]);
    }
    return fabsf(f16_bits(dh)) * 128.0f <= 65504.0f;
}

// Q4_0 (gguf.c:427-444), TG_PLAIN: run j = block j; element l < 16 is the low
// nibble of qs[l], element l + 16 its high nibble; weight (q - 8) * d as hi + lo.
__device__ __forceinline__ bool dq_q40(const uint8_t* p, uint32_t j, uint32_t* h, uint32_t* l) {
    const uint8_t* b = p + 18 * j;
    const uint32_t dh = lds_u16(b);
    const uint32_t d2 = dh | (dh << 16);
    uint32_t q[4];
    sm_words<4>(b + 2, q);
    const uint32_t n1032 = 0xE408E408u;                                            // -1032, -1032
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t n = (q[i & 3] >> (i < 4 ? 0u : 4u)) & 0x0F0F0F0Fu;       // elements 16.. are the high nibbles
        hilo(hadd2u(h1024(n, 0x4140u), n1032), d2, h[2 * i], l[2 * i]);
        hilo(hadd2u(h1024(n, 0x4342u), n1032), d2, h[2 * i + 1], l[2 * i + 1]);
    }
    return fabsf(f16_bits(dh)) * 8.0f <= 65504.0f;
}

// Q4_1 (gguf.c:445-462), TG_PLAIN: run j = block j; element l < 16 is the low
// nibble of qs[l], element l + 16 its high nibble; weight q * d + m (q * d is
// exact, so a fused multiply-add rounds as the reference's multiply-then-add),
// split into hi + lo.
__device__ __forceinline__ bool dq_q41(const uint8_t* p, uint32_t j, uint32_t* h, uint32_t* l) {
    const uint8_t* b = p + 20 * j;
    const uint32_t dm = lds_u32(b);
    const float d = f16_bits(dm & 0xFFFFu), m = f16_bits(dm >> 16);
    uint32_t q[4];
    sm_words<4>(b + 4, q);
#pragma unroll
    for (int sl = 0; sl < 4; sl++) {
        float w[8];
        const uint32_t sh = sl < 2 ? 0u : 4u;
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const uint32_t n = (q[(2 * sl + e) & 3] >> sh) & 0x0F0F0F0Fu;
#pragma unroll
            for (int k = 0; k < 4; k++) w[4 * e + k] = __fmaf_rn(magic_byte(n, 0x7440u | (uint32_t)k) - 8388608.0f, d, m);
        }
        st8(h + 4 * sl, l + 4 * sl, w);
    }
    return fabsf(d) * 15.0f + fabsf(m) <= 65504.0f;
}

// Q5_0 (gguf.c:463-488), TG_PLAIN: run j = block j; element l < 16 takes the
// low nibble of qs[l] and bit l of qh, element l + 16 the high nibble and bit
// l + 16; weight (q - 16) * d as hi + lo.
__device__ __forceinline__ bool dq_q50(const uint8_t* p, uint32_t j, uint32_t* h, uint32_t* l) {
    const uint8_t* b = p + 22 * j;
    const uint32_t dh = lds_u16(b);
    const uint32_t d2 = dh | (dh << 16);
    const uint32_t qh = lds_u32(b + 2);
    uint32_t q[4];
    sm_words<4>(b + 6, q);
    const uint32_t n1040 = 0xE410E410u;                                            // -1040, -1040
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t i0 = 4 * (i & 3);                                          // first qs byte of these 4
        const uint32_t n = (q[i & 3] >> (i < 4 ? 0u : 4u)) & 0x0F0F0F0Fu;
        const uint32_t hb = qh >> (i0 + (i < 4 ? 0u : 16u));                      // bits of elements i0 .. i0+3
        const uint32_t q5 = n | (((hb & 1u) | ((hb & 2u) << 7) | ((hb & 4u) << 14) | ((hb & 8u) << 21)) << 4);
        hilo(hadd2u(h1024(q5, 0x4140u), n1040), d2, h[2 * i], l[2 * i]);
        hilo(hadd2u(h1024(q5, 0x4342u), n1040), d2, h[2 * i + 1], l[2 * i + 1]);
    }
    return fabsf(f16_bits(dh)) * 16.0f <= 65504.0f;
}

// F16 rows: the weights are their own hi halves; lo is zero.
__device__ __forceinline__ bool dq_f16(const uint8_t* p, uint32_t j, uint32_t* h, uint32_t* l) {
    const uint8_t* b = p + 64 * j;
#pragma unroll
    for (int sl = 0; sl < 4; sl++) {
        const uint4 v = *reinterpret_cast<const uint4*>(b + 16 * sl);
        h[4 * sl] = v.x;
        h[4 * sl + 1] = v.y;
        h[4 * sl + 2] = v.z;
        h[4 * sl + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 16; i++) l[i] = 0;
    return true;
}

// ---------------------------------------------------------------- kernel
//
// Persistent: one CTA per SM walks the tiles (128 rows of one segment x one K
// range) t = blockIdx.x, + gridDim.x, ...; every role walks the same tile and
// slab sequence, so the shared-memory rings (raw units, A/x stages) and the
// two tensor-memory accumulators run across tile boundaries without a pause.

// One x stage: x hi + lo of a slab, then (kmin) the super-block's sums.
__host__ __device__ __forceinline__ uint32_t tg_stage_bytes(uint32_t np, uint32_t kmin) {
    return 2 * (128 * np) + (kmin ? 32 * np : 0u);
}

struct TTile {
    uint32_t seg, row0, ks, sl0, sl1;   // segment, first row, K split, slabs [sl0, sl1)
};
__device__ __forceinline__ TTile tg_tile(const TGemmArgs& a, uint32_t t) {
    const uint32_t rb = t / a.ksplit, ks = t - rb * a.ksplit;
    uint32_t s = 0;
#pragma unroll
    for (uint32_t i = 1; i < 3; i++)
        if (i < a.nseg && rb >= a.seg[i].rb0) s = i;
    const uint32_t units = a.K / a.ue, spu = a.ue / kTSlab;
    const uint32_t u0 = ks * a.ups, u1 = min(units, u0 + a.ups);
    return TTile{s, (rb - a.seg[s].rb0) * kTRows, ks, u0 * spu, u1 * spu};
}

__global__ void __launch_bounds__(kTThreads, 1) tgemm_kernel(const __grid_constant__ TGemmArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ TShared S;
    pdl_trigger();
    const uint32_t NS = a.stages, NP = a.NP;
    const uint32_t ntiles = a.rblocks * a.ksplit;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;

    uint8_t* const sbase = smem + ((kTAlign - (smem_u32(smem) & (kTAlign - 1))) & (kTAlign - 1));
    const uint32_t xsb = tg_stage_bytes(NP, a.kmin);
    uint8_t* const xbase = sbase;                                     // NS x (x hi, x lo[, sums])
    uint8_t* const rbase = xbase + NS * xsb;                          // kTRaw raw buffers
    // TG_KMIN: per A stage the two K = 16 A tiles of the min MMAs (kTMinBytes)
    uint8_t* const mbase = rbase + kTRaw * a.raw_bytes + kTSlack;

    if (tid == 0) {
        for (uint32_t i = 0; i < kTRaw; i++) {
            mbar_init(&S.raw_full[i], a.tma ? 1u : 32u);              // TMA: one expect-tx; cp.async: every raw lane
            mbar_init(&S.raw_empty[i], kTDeqWarps);
        }
        for (uint32_t i = 0; i < NS; i++) {
            mbar_init(&S.xfull[i], 1);
            mbar_init(&S.xempty[i], kTIssuers);                    // one commit per issuing thread
        }
        for (uint32_t i = 0; i < kTNA; i++) {
            mbar_init(&S.afull[i], kTGroupWarps);
            mbar_init(&S.aempty[i], kTIssuers);
        }
        for (uint32_t i = 0; i < kTSets; i++) { mbar_init(&S.accf[i], kTIssuers); mbar_init(&S.acce[i], kTEpiWarps); }
        mbar_init(&S.mdone, kTIssuers);
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
        uint32_t lr = 0;                                               // raw units issued
        bool ok = true;
        for (uint32_t t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
            const TTile T = tg_tile(a, t);
            const TSeg& G = a.seg[T.seg];
            const uint32_t spr = G.ru / kTSlab;
            for (uint32_t ur = T.sl0 / spr; ur < T.sl1 / spr; ur++) {
                const uint32_t buf = lr % kTRaw, ph = lr / kTRaw;
                if (ph > 0 && !tg_wait_warp(S, &S.raw_empty[buf], (ph - 1) & 1u, a.err)) { ok = false; break; }
                uint8_t* dst = rbase + buf * a.raw_bytes;
                if (a.tma) {
                    // one box: 128 rows x rrs bytes from the 16-byte boundary at or below the unit
                    if (lane == 0) {
                        mbar_expect_tx(&S.raw_full[buf], kTRows * G.rrs);
                        const uint64_t o = (uint64_t)ur * G.ub;
                        tma_load_2d(dst, &a.tmap[T.seg], (int32_t)((o & ~uint64_t(15)) >> 1), (int32_t)T.row0, &S.raw_full[buf]);
                    }
                    __syncwarp();
                } else {
                    // row strides that are not a multiple of 16 bytes: the 16-byte chunks
                    // covering each row's unit, lanes 0-15 on even rows, 16-31 on odd rows
                    const uint32_t ch = lane & 15u;
                    for (uint32_t r = lane >> 4; r < kTRows && T.row0 + r < G.rows; r += 2) {
                        const uint64_t o = (uint64_t)(T.row0 + r) * G.pitch + (uint64_t)ur * G.ub;
                        const uint64_t a16 = o & ~uint64_t(15);
                        const uint32_t nch = (uint32_t)((((o + G.ub + 15) & ~uint64_t(15)) - a16) >> 4);
                        if (ch < nch) tg_cpa16(dst + r * G.rrs + 16 * ch, G.w + a16 + 16 * ch);
                    }
                    tg_cpa_arrive(&S.raw_full[buf]);
                }
                lr++;
            }
        }
        // every issued copy has landed before the CTA can exit
        if (lane == 0)
            for (uint32_t u = (lr > kTRaw ? lr - kTRaw : 0); u < lr; u++) tg_drain(&S.raw_full[u % kTRaw], (u / kTRaw) & 1u);
        __syncwarp();
    } else if (warp == kTWarpX) {
        // ------------------------------------------------ staged inputs
        if (lane == 0) {
            pdl_wait();                                                 // x comes from the staging kernel
            const uint32_t xb = 128 * NP;                               // bytes of one half-slab
            const uint16_t* xsum = a.xh + (uint64_t)a.K * NP;           // the 32-element sums (K-quant min terms)
            uint32_t i = 0;                                             // slabs issued
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
                const TTile T = tg_tile(a, t);
                const bool sums = a.seg[T.seg].mode == TG_KMIN;
                for (uint32_t s = T.sl0; s < T.sl1; s++) {
                    const uint32_t si = i % NS, ph = i / NS;
                    if (ph > 0 && !tg_wait(S, &S.xempty[si], (ph - 1) & 1u, a.err)) { ok = false; break; }
                    const uint64_t off = (uint64_t)s * (kTSlab * NP);   // halves
                    uint8_t* dst = xbase + si * xsb;
                    const bool sb = sums && s % (256 / kTSlab) == 0;     // first slab of a super-block
                    mbar_expect_tx(&S.xfull[si], 2 * xb + (sb ? 32 * NP : 0u));
                    bulk_g2s(dst, a.xh + off, xb, &S.xfull[si]);
                    bulk_g2s(dst + xb, a.xl + off, xb, &S.xfull[si]);
                    if (sb) bulk_g2s(dst + 2 * xb, xsum + (uint64_t)(s / (256 / kTSlab)) * 16 * NP, 32 * NP, &S.xfull[si]);
                    i++;
                }
            }
            for (uint32_t u = (i > NS ? i - NS : 0); u < i; u++) tg_drain(&S.xfull[u % NS], (u / NS) & 1u);
        }
        __syncwarp();
    } else if (warp >= kTWarpMma && warp < kTWarpMma + kTIssuers) {
        // ------------------------------------------------ tensor-core issue: chain ch accumulates
        // A_hi x_hi (0), A_hi x_lo (1) or A_lo x_hi (2) -- chain 2 also the min
        // terms of TG_KMIN tiles; MMAs from several threads overlap in the
        // tensor pipe where one thread's would wait on each other
        const uint32_t ch = warp - kTWarpMma;
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(kTRows, NP);
            uint32_t i = 0, tl = 0;                                     // slabs, tiles consumed
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < ntiles; t += gridDim.x, tl++) {
                const TTile T = tg_tile(a, t);
                const TSeg& G = a.seg[T.seg];
                const bool work = ch != 2 || G.type != T_F16;           // F16 weights are exact in hi
                const bool kmin = ch == 2 && G.mode == TG_KMIN;
                const uint32_t ab = tl % kTSets, aph = tl / kTSets;
                if (aph > 0 && !tg_wait(S, &S.acce[ab], (aph - 1) & 1u, a.err)) break;
                tc_fence_after();
                const uint32_t d = tmem + ab * kTSetCols + ch * kTAccW;      // this chain's accumulator
                for (uint32_t s = T.sl0; s < T.sl1; s++, i++) {
                    const uint32_t si = i % NS, ai = i % kTNA;
                    if (!tg_wait(S, &S.afull[ai], (i / kTNA) & 1u, a.err) || !tg_wait(S, &S.xfull[si], (i / NS) & 1u, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xs = smem_u32(xbase + si * xsb);
                    if (work) {
                        const uint32_t at = tmem + kTACol0 + ai * kTACols + (ch == 2 ? kTACols / 2 : 0u);   // A hi or lo
                        const uint32_t xt = xs + (ch == 1 ? 128 * NP : 0u);                            // x hi or lo
#pragma unroll
                        for (uint32_t kk = 0; kk < kTSlab / 16; kk++)
                            umma_f16_ts(d, at + 8 * kk, umma_desc(xt + kk * 32 * NP, 16 * NP, 128), idesc,
                                        (s != T.sl0 || kk != 0) ? 1u : 0u);
                    }
                    if (kmin && s % (256 / kTSlab) == 0) {
                        // first slab of a super-block: sum_j -32 dmin m_j (S_hi_j + S_lo_j)
                        // with A = [m_hi, m_hi] then [m_lo, 0] from shared memory and
                        // B = the staged sums [S_hi, S_lo] after x hi and lo
                        const uint32_t mb = smem_u32(mbase + ai * kTMinBytes);
                        const uint64_t bd = umma_desc(xs + 256 * NP, 16 * NP, 128);
                        umma_f16(d, umma_desc(mb, 16 * kTRows, 128), bd, idesc, 1u);
                        umma_f16(d, umma_desc(mb + kTMinBytes / 2, 16 * kTRows, 128), bd, idesc, 1u);
                    }
                    umma_commit(&S.aempty[ai]);
                    umma_commit(&S.xempty[si]);
                }
                if (ok) umma_commit(&S.accf[ab]);
            }
            // every issued MMA has finished before the tensor memory is freed
            umma_commit(&S.mdone);
            tg_drain(&S.mdone, 0);
        }
        __syncwarp();
    } else if (warp >= kTWarpEpi) {
        // ------------------------------------------------ epilogue
        pdl_wait();                                                     // earlier kernels are done with part[]
        const uint32_t q = warp & 3u;                                   // tensor-memory lanes 32q..32q+31
        uint32_t tl = 0;
        for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x, tl++) {
            const TTile T = tg_tile(a, t);
            const TSeg& G = a.seg[T.seg];
            const uint32_t ab = tl % kTSets;
            if (!tg_wait_warp(S, &S.accf[ab], (tl / kTSets) & 1u, a.err)) break;
            tc_fence_after();
            const uint32_t row = T.row0 + 32 * q + lane;
            const bool lo = G.type != T_F16;
            float* part = G.part + (uint64_t)T.ks * a.B * G.rows;
            const uint32_t tb = tmem + ((32u * q) << 16) + ab * kTSetCols;
            for (uint32_t cc = 0; 16 * cc < NP; cc++) {
                // one load in flight at a time keeps the live registers to 32
                uint32_t u[16];
                float v[16];
                tmem_ld16(tb + 16 * cc, u);
                tmem_wait_ld(u);
#pragma unroll
                for (int e = 0; e < 16; e++) v[e] = __uint_as_float(u[e]);
                tmem_ld16(tb + kTAccW + 16 * cc, u);
                tmem_wait_ld(u);
#pragma unroll
                for (int e = 0; e < 16; e++) v[e] += __uint_as_float(u[e]);
                if (lo) {
                    tmem_ld16(tb + 2 * kTAccW + 16 * cc, u);
                    tmem_wait_ld(u);
#pragma unroll
                    for (int e = 0; e < 16; e++) v[e] += __uint_as_float(u[e]);
                }
                if (row < G.rows) {
                    float* dst = part + (uint64_t)(16 * cc) * G.rows + row;
                    const uint32_t nb = min(16u, a.B - min(a.B, 16 * cc));   // sequences of this chunk
#pragma unroll
                    for (int e = 0; e < 16; e++)
                        if ((uint32_t)e < nb) dst[(uint64_t)e * G.rows] = v[e] * 5.9604644775390625e-08f;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) tg_arrive(&S.acce[ab]);
        }
    } else {
        // ------------------------------------------------ dequant
        const uint32_t grp = warp / kTGroupWarps;                      // decodes the slabs i with i % kTGroups == grp
        const uint32_t r = tid & (kTRows - 1), c = (tid >> 7) & 1u;    // row, 32-element run of the slab
        uint32_t i = 0, lr = 0;                                         // slabs, raw units consumed
        bool ok = true, inrange = true;
        for (uint32_t t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
            const TTile T = tg_tile(a, t);
            const TSeg& G = a.seg[T.seg];
            const uint32_t spr = G.ru / kTSlab;
            const bool valid = T.row0 + r < G.rows;
            uint32_t cur = 0;
            for (uint32_t s = T.sl0; s < T.sl1; s++, i++) {
                const uint32_t ai = i % kTNA, aph = i / kTNA;
                if (s % spr == 0) {
                    cur = lr++;
                    if (!tg_wait_warp(S, &S.raw_full[cur % kTRaw], (cur / kTRaw) & 1u, a.err)) { ok = false; break; }
                }
                const bool mine = i % kTGroups == grp;
                if (!mine) {
                    if ((s + 1) % spr == 0) {
                        __syncwarp();
                        if (lane == 0) tg_arrive(&S.raw_empty[cur % kTRaw]);
                    }
                    continue;
                }
                uint32_t h[16], l[16], mh[4], ml[4];
                const bool mins = G.mode == TG_KMIN && c == 0 && s % spr == 0;   // this warp writes the mins
                if (!valid) {
#pragma unroll
                    for (int e = 0; e < 16; e++) h[e] = l[e] = 0;
#pragma unroll
                    for (int e = 0; e < 4; e++) mh[e] = ml[e] = 0;
                } else {
                    const uint64_t o = (uint64_t)(T.row0 + r) * G.pitch + (uint64_t)(s / spr) * G.ub;
                    const uint8_t* p = rbase + (cur % kTRaw) * a.raw_bytes + r * G.rrs + (uint32_t)(o & 15u);
                    const uint32_t j = (s % spr) * 2 + c;              // run within the raw unit
                    bool fine;
                    switch (G.type) {
                    case T_Q4_K: fine = dqf_q4k(p, j, h, l); break;
                    case T_Q5_K: fine = dqf_q5k(p, j, h, l); break;
                    case T_Q6_K: fine = dqf_q6k(p, j, h, l); break;
                    case T_Q8_0: fine = dq_q80(p, j, h, l); break;
                    case T_Q4_0: fine = dq_q40(p, j, h, l); break;
                    case T_Q4_1: fine = dq_q41(p, j, h, l); break;
                    case T_Q5_0: fine = dq_q50(p, j, h, l); break;
                    default: fine = dq_f16(p, j, h, l); break;
                    }
                    if (mins) fine = k4_mins(p, mh, ml) && fine;
                    inrange = inrange && fine;
                }
                // the A stage is free once the MMAs of slab i - kTNA have read it
                if (aph > 0 && !tg_wait_warp(S, &S.aempty[ai], (aph - 1) & 1u, a.err)) { ok = false; break; }
                tc_fence_after();
                // this warp's rows are tensor-memory lanes 32 (warp % 4) .. +31; run c
                // is K columns 16c .. 16c + 15 of the stage's hi and lo halves
                const uint32_t ta = tmem + ((32u * (warp & 3u)) << 16) + kTACol0 + ai * kTACols + 16 * c;
                tmem_st16(ta, h);
                tmem_st16(ta + kTACols / 2, l);
                if (mins) {
                    // row r of the min MMAs' A tiles (K-major core matrices: K
                    // elements 8g .. 8g + 7 of row r at 2048 g + 16 r): [m_hi, m_hi], [m_lo, 0]
                    uint8_t* mb = mbase + ai * kTMinBytes + 16 * r;
                    const uint4 vh4 = make_uint4(mh[0], mh[1], mh[2], mh[3]);
                    *reinterpret_cast<uint4*>(mb) = vh4;
                    *reinterpret_cast<uint4*>(mb + 16 * kTRows) = vh4;
                    *reinterpret_cast<uint4*>(mb + kTMinBytes / 2) = make_uint4(ml[0], ml[1], ml[2], ml[3]);
                    *reinterpret_cast<uint4*>(mb + kTMinBytes / 2 + 16 * kTRows) = make_uint4(0u, 0u, 0u, 0u);
                    fence_async_smem();                                // visible to the tensor core's reads
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    tg_arrive(&S.afull[ai]);
                    if ((s + 1) % spr == 0) tg_arrive(&S.raw_empty[cur % kTRaw]);
                }
            }
        }
        if (!inrange && a.err) atomicOr(a.err, kTErrRange);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTWarpMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(a.tcols) : "memory");
    }
}

// ---------------------------------------------------------------- host side

bool tgemm_type(uint32_t t) {
    return t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_Q8_0 || t == T_Q4_0 || t == T_Q4_1 || t == T_Q5_0 || t == T_F16;
}

// Elements per raw unit: a K-quant super-block; eight 32-element blocks when K
// allows (a 16-byte multiple of bytes: one TMA box per unit); F16 64 elements.
static uint32_t tg_ru(uint32_t type, uint32_t K) {
    if (type == T_Q4_K || type == T_Q5_K || type == T_Q6_K) return 256;
    if (type == T_F16) return 64;
    return K % 256 == 0 ? 256u : 64u;
}
static uint32_t tg_ub(uint32_t type, uint32_t ru) {
    switch (type) {
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_Q8_0: return ru / 32 * 34;
    case T_Q4_0: return ru / 32 * 18;
    case T_Q4_1: return ru / 32 * 20;
    case T_Q5_0: return ru / 32 * 22;
    default: return ru * 2;     // F16
    }
}

// cuTensorMapEncodeTiled from the driver, looked up once.
static PFN_cuTensorMapEncodeTiled_v12000 tg_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// 2-D map of a segment's rows as uint16 elements: box = rrs bytes x 128 rows,
// no swizzle; rows past the end read as zeros.
static bool tg_encode(CUtensorMap* m, const TSeg& S) {
    PFN_cuTensorMapEncodeTiled_v12000 fn = tg_encoder();
    if (!fn) return false;
    cuuint64_t dims[2] = {S.pitch / 2, S.rows};
    cuuint64_t strides[1] = {S.pitch};
    cuuint32_t box[2] = {S.rrs / 2, kTRows};
    cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t*>(S.w), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// At least kTSmemMin: two CTAs never share an SM (each allocates 512
// tensor-memory columns; a second one would wait for the first to finish).
constexpr size_t kTSmemMin = 120 * 1024;
static size_t tg_smem_for(const TGemmArgs& a, uint32_t stages) {
    return kTAlign + (size_t)stages * tg_stage_bytes(a.NP, a.kmin) + (size_t)kTRaw * a.raw_bytes + kTSlack +
           (a.kmin ? (size_t)kTNA * kTMinBytes : 0);
}
size_t tgemm_smem(const TGemmArgs& a) {
    const size_t n = tg_smem_for(a, a.stages);
    return n > kTSmemMin ? n : kTSmemMin;
}

bool tgemm_init() {
    return LM_CUDA(cudaFuncSetAttribute(tgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTSmemMax));
}

// Fill the launch geometry of `a` (segments, B, K set by the caller). False (no
// error set) when a segment's format or shape has no tensor-core path.
bool tgemm_plan(TGemmArgs& a, uint32_t sms) {
    if (a.B == 0 || a.B > 64 || a.nseg == 0 || a.nseg > 3 || a.K % kTSlab != 0 || sms == 0) return false;
    a.NP = (a.B + 15) & ~15u;
    a.kmin = 0;
    bool kq = false;
    uint32_t rbs = 0, raw = 0;
    a.tma = 1;
    for (uint32_t i = 0; i < a.nseg; i++) {
        TSeg& S = a.seg[i];
        if (!tgemm_type(S.type) || S.rows == 0) return false;
        if (reinterpret_cast<uintptr_t>(S.w) % 16 != 0) return false;
        if (S.row_bytes != type_bytes(S.type, a.K)) return false;
        if (S.pitch == 0) S.pitch = S.row_bytes;
        if (S.pitch < S.row_bytes) return false;
        kq = kq || S.type == T_Q4_K || S.type == T_Q5_K || S.type == T_Q6_K;
        S.mode = S.type == T_Q4_K || S.type == T_Q5_K ? TG_KMIN : TG_PLAIN;
        a.kmin = a.kmin || S.mode == TG_KMIN;
        S.ru = tg_ru(S.type, a.K);
        S.ub = tg_ub(S.type, S.ru);
        if (S.pitch % 16 != 0) a.tma = 0;                 // TMA needs 16-byte row strides
        S.rb0 = rbs;
        rbs += (S.rows + kTRows - 1) / kTRows;
    }
    for (uint32_t i = 0; i < a.nseg; i++) {
        TSeg& S = a.seg[i];
        if (a.tma) {
            // the box starts at the 16-byte boundary at or below each unit (the
            // byte offset of a unit is even: at most 14 bytes of lead-in); an odd
            // count of 16-byte units per row spreads the decoders' loads of 32
            // rows over all shared-memory banks (the box then reads a few bytes
            // of the next unit, or zeros past the row's end)
            uint32_t rrs = S.ub % 16 == 0 ? S.ub : (S.ub + 14 + 15) & ~15u;
            if ((rrs / 16) % 2 == 0) rrs += 16;
            S.rrs = rrs;
        } else {
            uint32_t rrs = (S.ub + 15 + 4 + 15) & ~15u;    // alignment delta + one word of over-read
            if ((rrs / 16) % 2 == 0) rrs += 16;            // odd count of 16-byte units: rows over all banks
            S.rrs = rrs;
        }
        raw = raw > kTRows * S.rrs ? raw : kTRows * S.rrs;
    }
    if (a.tma)
        for (uint32_t i = 0; i < a.nseg; i++)
            if (!tg_encode(&a.tmap[i], a.seg[i])) a.tma = 0;
    if (!a.tma)                                           // cp.async copies: the padded row stride
        for (uint32_t i = 0; i < a.nseg; i++) {
            TSeg& S = a.seg[i];
            uint32_t rrs = (S.ub + 15 + 4 + 15) & ~15u;
            if ((rrs / 16) % 2 == 0) rrs += 16;
            S.rrs = rrs;
            raw = raw > kTRows * rrs ? raw : kTRows * rrs;
        }
    a.ue = a.K % 256 == 0 ? 256u : 64u;
    if (kq && a.ue != 256) return false;
    a.raw_bytes = raw;
    a.stages = 0;
    for (uint32_t ns = kTMaxStages; ns >= 2; ns--)
        if (tg_smem_for(a, ns) <= kTSmemMax) { a.stages = ns; break; }
    if (a.stages == 0) return false;
    a.tcols = kTCols;                                    // accumulators + A stages
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
    a.grid = rbs * a.ksplit < sms ? rbs * a.ksplit : sms;
    return true;
}

bool launch_tgemm(const TGemmArgs& a, cudaStream_t st) {
    return LM_CUDA(launch_k(tgemm_kernel, dim3(a.grid), dim3(kTThreads), tgemm_smem(a), st, a));
}

}  // namespace lm
