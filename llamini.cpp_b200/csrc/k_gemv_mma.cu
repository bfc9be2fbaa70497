// k_gemv_mma.cu -- dequant-GEMV on the tensor cores, weights streamed by TMA.
//
// Same contract as the CUDA-core kernel in k_gemv.cu (llamini.cpp linear(),
// model.c:66-176, with the fused prologues/epilogues), organised for B200:
//
//  * Weight tiles move HBM -> shared memory with one cp.async.bulk per tile (a
//    tile is 16 consecutive rows, contiguous in GGUF layout; a gated tile adds
//    the 16 matching rows of the up matrix), completion tracked by an mbarrier.
//    CTAs are persistent and keep a ring of kStages tiles in flight, so HBM
//    sees ~100 KB of outstanding reads per SM without spending registers. The
//    first copies are issued before the kernel waits for its predecessor (the
//    weights do not depend on it), overlapping the previous kernel's tail.
//  * Every block format is affine per group of 16 or 32 weights:
//      w = alpha * q - beta     (q a small unsigned integer, gguf.c:427-590)
//    so  sum_i w_i x_i = alpha * sum_i q_i x_i - beta * sum_i x_i.
//    sum_i q_i x_i for 16 rows is an mma.sync.m16n8k16: the integers enter the
//    A operand as exact fp16 subnormals q * 2^-24 (one AND / byte permute on
//    the packed bytes), x enters B as an fp16 hi/lo pair (22 significant bits)
//    after scaling the vector by a power of two into fp16's range; f32
//    accumulation. alpha, beta and the 16-element sums of x are applied in f32.
//  * B columns 2s, 2s+1 carry x for "slot" s (a group, scale group or block);
//    chaining four slots' MMAs into one accumulator leaves slot s's sums in the
//    lanes with tig == s, so all 32 lanes apply scales in parallel.
#include "internal.h"
#include "quant.cuh"
#include "pdl.cuh"
#include "mma_gemv.cuh"

#include <cuda_fp16.h>
#include <cstdlib>

namespace lm {

constexpr int kMWarps = 8;
constexpr int kMThreads = kMWarps * 32;
constexpr uint32_t kStages = 2;              // weight tiles in flight per CTA

// Elements and bytes per iteration of a format's compute (FQ* SB / SBB).
__host__ __device__ __forceinline__ uint32_t seg_sb(uint32_t t) {
    return (t == T_Q4_K || t == T_Q5_K || t == T_Q6_K) ? 256u : 128u;
}
__host__ __device__ __forceinline__ uint32_t seg_sbb_dev(uint32_t t) {
    switch (t) {
    case T_Q4_K: return FQ4K::SBB;
    case T_Q5_K: return FQ5K::SBB;
    case T_Q6_K: return FQ6K::SBB;
    case T_Q8_0: return FQ80::SBB;
    case T_Q4_1: return FQ41::SBB;
    case T_Q5_0: return FQ50::SBB;
    default: return FQ40::SBB;
    }
}
static uint32_t seg_sbb(uint32_t t) {
    switch (t) {
    case T_Q4_K: return FQ4K::SBB;
    case T_Q5_K: return FQ5K::SBB;
    case T_Q6_K: return FQ6K::SBB;
    case T_Q8_0: return FQ80::SBB;
    case T_Q4_1: return FQ41::SBB;
    case T_Q5_0: return FQ50::SBB;
    default: return FQ40::SBB;
    }
}

bool mma_type(uint32_t t) {
    return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0 || t == T_Q4_0 || t == T_Q4_1 || t == T_Q5_0 || t == T_Q5_K;
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

// ------------------------------------------------------------------ tensor parallelism
// The fused reduction (GemvTp, internal.h). Every wait is bounded (2 s).
constexpr uint64_t kTpFuseWaitNs = 2000000000ull;
__device__ __forceinline__ uint64_t g_time() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t ld_acq_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Before staging: wait for every rank's rows of slot `pull`, then xf = x +
// (sum over ranks in rank order) -- the separate allreduce's arithmetic. The
// CTA that finishes reading last writes the sum back to x (every other CTA has
// read x by then) and opens the slot's next use. False after a wait ran out.
__device__ bool tp_pull(const GemvArgs& a, float* xf) {
    __shared__ uint32_t s_st;
    const GemvTp& t = a.tp;
    const uint32_t tid = threadIdx.x, K = a.K, P = t.pull;
    if (tid == 0) {
        // a wait of this session that already ran out: the group is broken, fail at once
        uint32_t ok = (*reinterpret_cast<volatile uint32_t*>(a.err) & kErrWaitTimeout) ? 0u : 1u;
        const uint32_t target = (*reinterpret_cast<volatile uint32_t*>(t.gen + P) + 1u) * ((K + 15u) / 16u);
        const uint32_t* arr = t.arrive[t.rank] + P * 8u;
        const uint64_t t0 = g_time();
        for (uint32_t r = 0; r < t.world && ok; r++) {
            for (uint32_t i = 0;; i++) {
                if ((int32_t)(ld_acq_sys(arr + r) - target) >= 0) break;
                if ((i & 63u) == 63u && g_time() - t0 > kTpFuseWaitNs) {
                    atomicOr(a.err, kErrWaitTimeout);
                    ok = 0;
                    break;
                }
            }
        }
        s_st = ok;
    }
    __syncthreads();
    if (!s_st) return false;
    // the ranks' rows are in this GPU's memory (peers stored them over NVLink):
    // after the acquire, L2 loads (not L1, which may hold an earlier use's rows),
    // all of a thread's loads in flight at once
    const float* mine = t.slots[t.rank] + (uint64_t)P * 8u * kTpFusedFloats;
    for (uint32_t i = tid; i < K; i += kMThreads) {
        float v[8];
#pragma unroll
        for (uint32_t r = 0; r < 8; r++) v[r] = r < t.world ? __ldcg(mine + (uint64_t)r * kTpFusedFloats + i) : 0.f;
        float s = 0.f;
#pragma unroll
        for (uint32_t r = 0; r < 8; r++)
            if (r < t.world) s += v[r];
        xf[i] = __ldcg(a.x + i) + s;
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(t.ticket + P, 1u);
        s_st = old + 1u == gridDim.x ? 2u : 1u;
    }
    __syncthreads();
    if (s_st == 2u) {
        float* xw = const_cast<float*>(a.x);          // the residual stream
        for (uint32_t i = tid; i < K; i += kMThreads) xw[i] = xf[i];
        if (tid == 0) {
            t.ticket[P] = 0u;
            *reinterpret_cast<volatile uint32_t*>(t.gen + P) = *reinterpret_cast<volatile uint32_t*>(t.gen + P) + 1u;
        }
    }
    return true;
}

// ------------------------------------------------------------------ x staging
// Normalise (RMSNorm model.c:4-10 / LayerNorm gpt2.c:130-139), choose E with
// max|x| 2^E < 2^14, write the fp16 hi/lo split and the scaled 16-element sums.
// x is a.x, or sm.xf itself after tp_pull (each element is read and written by
// the same thread).
__device__ void stage_x(const GemvArgs& a, const float* x, const MmaSmem& sm, float* s_scale) {
    const uint32_t K = a.K, n4 = K / 4, tid = threadIdx.x;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4* xf4 = reinterpret_cast<float4*>(sm.xf);
    float s = 0.f, m = 0.f, f = 1.0f;
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
    const float mx = m * f;
    int e = 0;
    if (mx > 0.f && mx < INFINITY) frexpf(mx, &e);
    int E = 14 - e;
    E = E > 100 ? 100 : (E < -100 ? -100 : E);
    const float F = f * __int_as_float((E + 127) << 23);
    // each lane takes whole float4s; a run of 16 is 4 consecutive lanes
    const uint32_t n4r = (n4 + 31u) & ~31u;
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

// ------------------------------------------------------------------ tiles

// Tensor maps of the segments whose rows are padded in shared memory (one TMA
// copy per tile instead of one bulk copy per row); has = 0: bulk copies.
struct alignas(64) GemvMaps {
    CUtensorMap m[kMaxSegs][2];
    uint32_t has[kMaxSegs][2];
};

// Thread 0: start the copies of tile t into stage buffer `buf` (128-byte aligned).
__device__ __forceinline__ void issue_tile(const GemvArgs& a, const GemvMaps& maps, uint32_t t, uint8_t* buf,
                                           uint64_t* bar) {
    const TileRef tr = tile_of(a, t);
    const GemvSeg& G = a.seg[tr.seg];
    const bool glu = G.epi == EPI_GLU_SILU || G.epi == EPI_GLU_GELU;
    const bool t1 = maps.has[tr.seg][0] != 0, t2 = maps.has[tr.seg][1] != 0;
    const uint32_t n1 = tile_tx(G.row_bytes, tr.nrows, t1);
    const uint32_t n2 = glu ? tile_tx(G.row_bytes2, tr.nrows, t2) : 0u;
    mbar_expect_tx(bar, n1 + n2);
    if (t1) tma_tile(buf, &maps.m[tr.seg][0], (int32_t)tr.row0, bar);
    else copy_rows(buf, G.w + (uint64_t)tr.row0 * G.row_bytes, G.row_bytes, tr.nrows, bar);
    if (glu) {
        if (t2) tma_tile(buf + up_offset(G), &maps.m[tr.seg][1], (int32_t)tr.row0, bar);
        else copy_rows(buf + up_offset(G), G.w2 + (uint64_t)tr.row0 * G.row_bytes2, G.row_bytes2, tr.nrows, bar);
    }
}

// Thread 0: start the copies of the CTA's work item j (see gemv_mma_kernel).
// K-chunks of rows of a multiple of 16 bytes: one TMA box (cu = the chunk's
// units); otherwise (cu = 0) one bulk copy per row of the 16-byte aligned window
// around the row's chunk, into slots of rsu units.
__device__ __noinline__ void issue_item(const GemvArgs& a, const GemvMaps& maps, uint32_t j, uint32_t nch,
                                        uint32_t n_tiles, uint32_t ipc, uint32_t cu, uint32_t rsu, uint8_t* buf,
                                        uint64_t* bar) {
    const uint32_t t = blockIdx.x + (j / nch) * gridDim.x;
    if (t >= n_tiles) return;
    if (!ipc) {
        issue_tile(a, maps, t, buf, bar);
        return;
    }
    const TileRef tr = tile_of(a, t);
    if (cu) {
        mbar_expect_tx(bar, 256u * (cu + 1u));
        tma_box(buf, &maps.m[0][0], (int32_t)((j % nch) * cu), (int32_t)tr.row0, bar);
        return;
    }
    const GemvSeg& G = a.seg[0];
    const uint64_t cb = (uint64_t)ipc * seg_sbb_dev(G.type), c0 = (j % nch) * cb;
    const uint64_t len = G.row_bytes - c0 < cb ? G.row_bytes - c0 : cb;
    uint32_t tx = 0;
    for (uint32_t r = 0; r < tr.nrows; r++) {
        const uint64_t s0 = (uint64_t)(tr.row0 + r) * G.row_bytes + c0;
        tx += (uint32_t)(((s0 + len + 15) & ~uint64_t(15)) - (s0 & ~uint64_t(15)));
    }
    mbar_expect_tx(bar, tx);
    for (uint32_t r = 0; r < tr.nrows; r++) {
        const uint64_t s0 = (uint64_t)(tr.row0 + r) * G.row_bytes + c0;
        const uint64_t a0 = s0 & ~uint64_t(15);
        bulk_g2s(buf + (uint64_t)r * 16u * rsu, G.w + a0, (uint32_t)(((s0 + len + 15) & ~uint64_t(15)) - a0), bar);
    }
}

// ------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kMThreads)
gemv_mma_kernel(const __grid_constant__ GemvArgs a, uint32_t stage_bytes, const __grid_constant__ GemvMaps maps,
                uint32_t ipc, uint32_t cu, uint32_t rsu) {
    extern __shared__ __align__(128) uint8_t smem_dyn[];
    // tensor copies need 128-byte aligned destinations
    uint8_t* const smem_raw = smem_dyn + ((128u - (smem_u32(smem_dyn) & 127u)) & 127u);
    __shared__ float s_scale;
    __shared__ __align__(8) uint64_t bars[kStages];
    __shared__ int s_fail;
    pdl_trigger();
    const uint32_t K = a.K, tid = threadIdx.x;
    const GemvSeg& last = a.seg[a.nseg - 1];
    const uint32_t n_tiles = last.tile0 + (last.rows + 15) / 16;

    uint8_t* stages = smem_raw;                                   // kStages * stage_bytes
    MmaSmem sm;
    sm.xf = reinterpret_cast<float*>(smem_raw + kStages * stage_bytes);
    sm.xh = reinterpret_cast<uint32_t*>(sm.xf + K);
    sm.xl = sm.xh + K / 2;
    sm.sx = reinterpret_cast<float*>(sm.xl + K / 2);
    sm.red = sm.sx + K / 16;
    sm.part = sm.red + 2 * kMWarps;

    // Work items: a tile, or (ipc > 0: rows too long for two whole tiles in shared
    // memory) each of its nch K-chunks of ipc iterations in turn, chunk c copied
    // as one TMA box of cu units + 1 from unit c * cu of the 16 rows. The CTA's
    // item j is chunk j % nch of tile blockIdx.x + (j / nch) * gridDim.x.
    const uint32_t nit = ipc ? (K + seg_sb(a.seg[0].type) - 1) / seg_sb(a.seg[0].type) : 0u;
    const uint32_t nch = ipc ? (nit + ipc - 1) / ipc : 1u;
    // weights first: they do not depend on the previous kernel
    if (tid == 0) {
        s_fail = 0;
        for (uint32_t i = 0; i < kStages; i++) mbar_init(&bars[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        for (uint32_t i = 0; i < kStages; i++) issue_item(a, maps, i, nch, n_tiles, ipc, cu, rsu, stages + i * stage_bytes, &bars[i]);
    }
    pdl_wait();                                                   // x comes from the previous kernel
    const bool pulled = a.tp.pull != kTpNone;
    if (pulled && !tp_pull(a, sm.xf)) {
        // the error bit is set; the first tiles' copies land before the CTA leaves
        if (tid == 0)
            for (uint32_t i = 0; i < kStages; i++)
                if (blockIdx.x + (i / nch) * gridDim.x < n_tiles) mbar_wait(&bars[i], 0);
        return;
    }
    stage_x(a, pulled ? sm.xf : a.x, sm, &s_scale);               // ends with __syncthreads
    const bool push = a.tp.push != kTpNone;
    const uint64_t push_off = push ? ((uint64_t)a.tp.push * 8u + a.tp.rank) * kTpFusedFloats : 0ull;

    const uint32_t lane = tid & 31u, warp = tid >> 5;
    Lane L;
    L.g = lane >> 2;
    L.tig = lane & 3u;
    L.slot = L.g >> 1;
    L.xpart = (L.g & 1u) ? sm.xl : sm.xh;

    uint32_t i = 0, tiles_done = 0;                // items consumed, tiles finished
    for (uint32_t t = blockIdx.x; t < n_tiles; t += gridDim.x, tiles_done++) {
        const TileRef tr = tile_of(a, t);
        const GemvSeg& G = a.seg[tr.seg];
        const bool glu = G.epi == EPI_GLU_SILU || G.epi == EPI_GLU_GELU;
        // a gated tile: warps 0..3 take the gate rows, 4..7 the up rows
        const uint32_t half = kMWarps / 2;
        const bool up = glu && warp >= half;
        const uint32_t first = glu ? warp % half : warp, step = glu ? half : kMWarps;
        float acc[2] = {0.f, 0.f};
        for (uint32_t c = 0; c < nch; c++, i++) {
            const uint32_t st = i % kStages, parity = (i / kStages) & 1u;
            uint8_t* buf = stages + st * stage_bytes;
            if (!mbar_wait(&bars[st], parity)) {
                atomicOr(a.err, kErrWaitTimeout);
                s_fail = 1;
            }
            __syncthreads();
            if (s_fail) return;                   // a copy never landed: the flag is set, stop
            if (ipc) {
                const uint64_t rb = 16u * rsu;
                const uint32_t it0 = c * ipc, it1 = min(it0 + ipc, nit);
                uint32_t mis = 0, mis8 = 0;
                if (!cu) {                        // per-row windows: where each row's chunk starts in its slot
                    const uint64_t c0 = (uint64_t)it0 * seg_sbb_dev(G.type);
                    mis = (uint32_t)(((uint64_t)(tr.row0 + L.g) * G.row_bytes + c0) & 15u);
                    mis8 = (uint32_t)(((uint64_t)(tr.row0 + L.g + 8) * G.row_bytes + c0) & 15u);
                }
                switch (G.type) {
                case T_Q4_K: chunk_rows<FQ4K>(buf, rb, mis, mis8, K, L, first, step, it0, it1, sm, acc); break;
                case T_Q6_K: chunk_rows<FQ6K>(buf, rb, mis, mis8, K, L, first, step, it0, it1, sm, acc); break;
                case T_Q8_0: chunk_rows<FQ80>(buf, rb, mis, mis8, K, L, first, step, it0, it1, sm, acc); break;
                case T_Q4_1: chunk_rows<FQ41>(buf, rb, mis, mis8, K, L, first, step, it0, it1, sm, acc); break;
                case T_Q5_K: chunk_rows<FQ5K>(buf, rb, mis, mis8, K, L, first, step, it0, it1, sm, acc); break;
                case T_Q5_0: chunk_rows<FQ50>(buf, rb, mis, mis8, K, L, first, step, it0, it1, sm, acc); break;
                default:     chunk_rows<FQ40>(buf, rb, mis, mis8, K, L, first, step, it0, it1, sm, acc); break;
                }
            } else {
                const uint8_t* base = up ? buf + up_offset(G) : buf;
                const uint64_t rb = smem_rs(up ? G.row_bytes2 : G.row_bytes);
                switch (G.type) {
                case T_Q4_K: tile_rows<FQ4K>(base, rb, K, L, first, step, sm, acc); break;
                case T_Q6_K: tile_rows<FQ6K>(base, rb, K, L, first, step, sm, acc); break;
                case T_Q8_0: tile_rows<FQ80>(base, rb, K, L, first, step, sm, acc); break;
                case T_Q4_1: tile_rows<FQ41>(base, rb, K, L, first, step, sm, acc); break;
                case T_Q5_K: tile_rows<FQ5K>(base, rb, K, L, first, step, sm, acc); break;
                case T_Q5_0: tile_rows<FQ50>(base, rb, K, L, first, step, sm, acc); break;
                default:     tile_rows<FQ40>(base, rb, K, L, first, step, sm, acc); break;
                }
            }
            if (c + 1 == nch) {
                // the lanes of a quad hold different slots' sums: combine them
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 1);
                    acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 2);
                }
                if (L.tig == 0) {
                    sm.part[warp * 16 + L.g] = acc[0];
                    sm.part[warp * 16 + L.g + 8] = acc[1];
                }
            }
            __syncthreads();                      // stage buffer consumed (last chunk: partials ready)
            if (tid == 0) issue_item(a, maps, i + kStages, nch, n_tiles, ipc, cu, rsu, buf, &bars[st]);
        }
        // epilogue: thread r < 16 finishes row row0 + r
        unsigned long long key = 0ull;
        if (tid < 16) {
            const uint32_t r = tid, row = tr.row0 + r;
            float v = 0.f, u = 0.f;
#pragma unroll
            for (uint32_t w = 0; w < kMWarps; w++) {
                if (glu && w >= half) u += sm.part[w * 16 + r];
                else v += sm.part[w * 16 + r];
            }
            v *= s_scale;
            u *= s_scale;
            if (r < tr.nrows) {
                switch (G.epi) {
                case EPI_STORE:
                    if (G.bias) v += G.bias[row];
                    if (push) {
                        // this rank's partial row into every rank's slot (peer memory)
                        for (uint32_t j = 0; j < a.tp.world; j++) a.tp.slots[j][push_off + row] = v;
                    } else {
                        G.out[row] = v;
                    }
                    break;
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
        __syncthreads();                          // part[] free for the next tile
    }
    if (push) {
        // this CTA's rows are stored: count its tiles into every rank's arrivals
        if (tid < 16) __threadfence_system();
        __syncthreads();
        if (tid < a.tp.world) {
            uint32_t* c = a.tp.arrive[tid] + a.tp.push * 8u + a.tp.rank;
            asm volatile("red.release.sys.global.add.u32 [%0], %1;\n" ::"l"(c), "r"(tiles_done) : "memory");
        }
    }
}

static size_t x_smem(uint32_t K) {
    // xf (4K bytes), xh, xl (2K bytes each), sx (K/4 bytes), then red and part
    return (size_t)K * 8 + (size_t)K / 16 * 4 + 2 * kMWarps * 4 + kMWarps * 16 * 4;
}

constexpr size_t kSmemLimit = 220 * 1024;     // dynamic shared memory per CTA (leaves room for static)
static int g_mma_regs = 128;

bool gemv_mma_init() {
    cudaFuncAttributes fa;
    if (!LM_CUDA(cudaFuncGetAttributes(&fa, gemv_mma_kernel))) return false;
    g_mma_regs = fa.numRegs > 0 ? fa.numRegs : 128;
    return LM_CUDA(cudaFuncSetAttribute(gemv_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit)) &&
           LM_CUDA(cudaFuncSetAttribute(gemv_mma_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
}

// The stage size and shared memory of `in` on the tensor-core kernel; false
// when some segment is not a tensor-core format (a gated pair sharing one
// format) or the tiles do not fit in shared memory.
// Rows too long for two whole tiles next to the staged input (K = 11008 at the
// 7B shape) move in K-chunks instead: *ipc_out iterations per chunk, *cu_out
// 16-byte units (even, so the padded stride cu + 1 keeps the rows an MMA reads
// in different banks); one segment, not gated, rows of a multiple of 16 bytes.
static bool mma_plan(const GemvArgs& in, uint64_t* stage_out, size_t* smem_out, uint32_t* ipc_out = nullptr,
                     uint32_t* cu_out = nullptr, uint32_t* rsu_out = nullptr) {
    if (ipc_out) *ipc_out = 0;
    if (cu_out) *cu_out = 0;
    if (rsu_out) *rsu_out = 0;
    if (in.K % 32 != 0) return false;
    if ((in.tp.push != kTpNone || in.tp.pull != kTpNone) &&
        (in.K > kTpFusedFloats || in.tp.world > 8 || (in.tp.pull != kTpNone && in.x == nullptr)))
        return false;
    uint64_t stage = 0;
    for (uint32_t i = 0; i < in.nseg; i++) {
        const GemvSeg& g = in.seg[i];
        const bool glu = g.epi == EPI_GLU_SILU || g.epi == EPI_GLU_GELU;
        if (!mma_type(g.type) || (glu && g.type2 != g.type)) return false;
        if (type_bytes(g.type, in.K) == 0) return false;
        // bulk copies need 16-byte aligned sources: the matrix base and every
        // tile start (row multiples of 16, so 16 * row_bytes suffices)
        if (reinterpret_cast<uintptr_t>(g.w) % 16 != 0 || (glu && reinterpret_cast<uintptr_t>(g.w2) % 16 != 0))
            return false;
        const uint64_t t1 = tile_bytes(g.row_bytes);
        const uint64_t t2 = glu ? tile_bytes(g.row_bytes2) : 0;
        stage = stage > t1 + t2 ? stage : t1 + t2;
    }
    // 16 bytes of slack past each stage: funnel-shifted word reads at the tile end
    stage = (stage + 16 + 127) & ~uint64_t(127);
    if (in.norm != NORM_NONE && (reinterpret_cast<uintptr_t>(in.norm_w) % 16 != 0 ||
                                 (in.norm == NORM_LAYER && reinterpret_cast<uintptr_t>(in.norm_b) % 16 != 0)))
        return false;
    if (reinterpret_cast<uintptr_t>(in.x) % 16 != 0) return false;
    size_t smem = kStages * stage + x_smem(in.K) + 128;          // + alignment slack
    if (smem > kSmemLimit) {
        const GemvSeg& g = in.seg[0];
        const bool glu = g.epi == EPI_GLU_SILU || g.epi == EPI_GLU_GELU;
        if (in.nseg != 1 || glu || g.row_bytes % 2 != 0) return false;
        const size_t xs = x_smem(in.K) + 128;
        if (xs >= kSmemLimit) return false;
        const size_t per_stage = (kSmemLimit - xs) / kStages;
        const uint32_t sbb = seg_sbb(g.type);
        const bool box = g.row_bytes % 16 == 0;                    // TMA box; else per-row windows
        uint32_t ipc = 0, cu = 0, rsu = 0;
        for (uint32_t k = 4000 / sbb; k >= 1 && ipc == 0; k--) {
            const uint32_t bytes = k * sbb;
            if (box && (bytes % 16 != 0 || (bytes / 16) % 2 != 0)) continue;
            // slot units: the chunk (+ one unit of padding), or its aligned window (+ padding), odd
            const uint32_t su = box ? bytes / 16 + 1 : ((bytes + 30 + 15) / 16 + 1) | 1u;
            if (su > 256 || (size_t)256 * su > per_stage) continue;
            ipc = k;
            cu = box ? bytes / 16 : 0;
            rsu = su;
        }
        if (ipc == 0) return false;
        stage = 256u * rsu;                                         // a multiple of 128
        smem = kStages * stage + xs;
        if (smem > kSmemLimit) return false;
        if (ipc_out) *ipc_out = ipc;
        if (cu_out) *cu_out = cu;
        if (rsu_out) *rsu_out = rsu;
    }
    *stage_out = stage;
    *smem_out = smem;
    return true;
}

bool gemv_mma_takes(const GemvArgs& a) {
    static const bool cuda_cores_only = getenv("LLAMINI_GEMV_CUDA_CORES") != nullptr;
    uint64_t stage;
    size_t smem;
    return !cuda_cores_only && mma_plan(a, &stage, &smem);
}

// Launch when mma_plan takes `in`; *handled = false otherwise, and the caller
// uses k_gemv.cu (which has no fused tensor-parallel reduction).
bool launch_gemv_mma(const GemvArgs& in, cudaStream_t st, bool* handled) {
    *handled = false;
    uint64_t stage = 0;
    size_t smem = 0;
    uint32_t ipc = 0, cu = 0, rsu = 0;
    if (!mma_plan(in, &stage, &smem, &ipc, &cu, &rsu)) return true;
    GemvArgs a = in;
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < a.nseg; i++) {
        a.seg[i].tile0 = tiles;
        tiles += (a.seg[i].rows + 15) / 16;
    }
    if (a.err == nullptr) a.err = dev_err_word();
    if (a.err == nullptr) return false;
    // resident CTAs per SM from registers, threads and shared memory (computed
    // here rather than queried: launches are also made during graph capture)
    uint32_t per_sm = 65536u / ((uint32_t)g_mma_regs * kMThreads);
    per_sm = per_sm < 2048u / kMThreads ? per_sm : 2048u / kMThreads;
    const uint32_t by_smem = (uint32_t)((228u * 1024u) / (smem + 1024u));
    per_sm = per_sm < by_smem ? per_sm : by_smem;
    if (per_sm < 1) per_sm = 1;
    uint32_t grid = (uint32_t)sm_count() * per_sm;
    if (grid > tiles) grid = tiles;
    // one TMA tensor copy per tile for padded rows (bulk copies per row if the
    // driver refuses a map)
    GemvMaps maps = {};
    if (ipc && cu) {
        // K-chunks: one box map of cu + 1 units (the driver may refuse it: then the CUDA-core kernel)
        if (!encode_box_map(&maps.m[0][0], a.seg[0].w, a.seg[0].row_bytes, a.seg[0].rows, cu + 1)) return true;
        maps.has[0][0] = 1;
    } else if (!ipc) {
        for (uint32_t i = 0; i < a.nseg; i++) {
            const GemvSeg& g = a.seg[i];
            const bool glu = g.epi == EPI_GLU_SILU || g.epi == EPI_GLU_GELU;
            if (padded_rows(g.row_bytes)) maps.has[i][0] = encode_tile_map(&maps.m[i][0], g.w, g.row_bytes, g.rows);
            if (glu && padded_rows(g.row_bytes2))
                maps.has[i][1] = encode_tile_map(&maps.m[i][1], g.w2, g.row_bytes2, g.rows);
        }
    }
    *handled = true;
    return LM_CUDA(launch_k(gemv_mma_kernel, dim3(grid), dim3(kMThreads), smem, st, a, (uint32_t)stage, maps, ipc, cu, rsu));
}

}  // namespace lm
