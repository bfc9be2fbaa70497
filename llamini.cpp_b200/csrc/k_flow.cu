// k_flow.cu -- batch-1 decode steps as one persistent dataflow kernel.
//
// One token step (generate.c:62-120) is a chain of dependent ops:
//
//   per layer: [norm + QKV] -> [attention] -> [O + residual] -> [norm + gate/up]
//              -> [down + residual]      then [final norm + lm_head + argmax]
//
// and at batch 1 each matrix is only 0.3-27 MB, so the step time is set by how
// fast one op hands its output to the next, not by HBM. This kernel keeps the
// task split of the earlier persistent kernel (16-row tiles, (head, split)
// attention tasks, per-op completion counters with release/acquire at GPU
// scope, a producer warp streaming every CTA's upcoming weight tiles into a
// shared-memory ring across op and step boundaries) and takes the input
// staging off the critical path:
//
//  * A GEMV's input travels as records (FlowRec, internal.h): per 16 elements
//    the fp16 high/low parts of x * 2^E already in mma.sync B-fragment order,
//    2^(24-E) and the group's sum. The op that produces the vector writes them
//    in its epilogue (a 16-row tile is exactly one group), so a consumer warp
//    loads its slice of K straight into registers: no shared-memory staging,
//    no block reductions, no barrier before the MMAs. A per-group exponent is
//    exact to apply (a power of two) and keeps 22 significant bits per element.
//  * RMSNorm (model.c:4-10) is applied after the dot product: the producer
//    folds the norm weight into the records and writes the sum of squares of
//    its 16 raw values; the epilogue scales the row sums by 1/rms. The merge of
//    attention splits (the O projection's input) is done by the consumer warps
//    in registers.
//  * Roles per CTA: 8 consumer warps (MMAs over their super-blocks of K, and
//    the attention tasks), one epilogue warp (sums the warps' partials, applies
//    norm, bias, residual, activation, argmax, writes outputs and the next
//    records, signals the op), one producer warp (weight copies). The epilogue
//    of tile i overlaps the MMAs of tile i + 1 through two partial buffers and
//    named barriers.
//
// Every wait is bounded (2 s of %globaltimer). When one runs out the CTA sets
// the step state's error bit and a global abort flag; every role then skips
// its remaining waits and work but still takes its named-barrier steps, so the
// CTA reaches its exit, where copies still in flight are waited for (bounded).
#include "internal.h"
#include "quant.cuh"
#include "rows.cuh"
#include "mma_gemv.cuh"
#include "attn_core.cuh"

#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <vector>

namespace lm {
#ifdef LLAMINI_FLOW_TIMELINE
// Profiling build only (flow_timeline.py): %globaltimer stamps per (CTA, op,
// point) of the last step of a launch, into g_tl[cta][op][8]: 0 the op's inputs
// are ready (consumer thread 0), 1 its fragments are staged, 2 its first weight
// tile is in shared memory, 3 the consumers' last MMAs are done, 4 the epilogue
// warp has the last tile's partials, 5 just before the op's release, 6 just
// after it, 7 the producer issues the op's first tile.
__device__ unsigned long long* g_tl = nullptr;
#define FLOW_TL(j, n, op, slot)                                                            \
    do {                                                                                 \
        if (g_tl != nullptr && (j) + 1 == (n)) {                                         \
            unsigned long long t_;                                                       \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                       \
            g_tl[((unsigned long long)blockIdx.x * 128 + (op)) * 8 + (slot)] = t_;       \
        }                                                                                \
    } while (0)
#else
#define FLOW_TL(j, n, op, slot) \
    do {                        \
    } while (0)
#endif
namespace {

constexpr int kCW = 8;                              // consumer warps
constexpr uint32_t kCT = kCW * 32;                  // consumer threads
constexpr uint32_t kEpiWarp = kCW, kProdWarp = kCW + 1;
constexpr uint32_t kFT = kCT + 64;                  // + epilogue warp + producer warp
constexpr uint32_t kPairT = kCT + 32;               // consumers + epilogue warp (named barriers 2..5)
constexpr uint32_t kQ = 16;                         // queued weight tiles per CTA
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr size_t kFlowSmem = 220 * 1024;
// named barriers: 1 consumers; 2, 3 tile partials ready (buffer 0, 1); 4, 5 buffer free
constexpr uint32_t kBarCons = 1, kBarDone = 2, kBarFree = 4;

struct FlowShared {
    FlowOp cop;                          // the consumers' current op
    FlowOp eop;                          // the epilogue warp's current op
    uint32_t tasks[kFlowMaxTasks];
    uint32_t ops_kind[kFlowMaxOps];
    uint64_t bar[kQ];
    uint64_t vend[kQ];
    uint32_t off[kQ];
    float part[2][kCW][2][16];           // per buffer, warp, (main | up) and row
    uint32_t consumed, issued, abort, epoch;
    uint32_t pos;                        // the current step's position (read once per step)
    // Producer gate: a GPU-scope release waits for every bulk copy the SM has
    // in flight (about a microsecond while the weight stream runs), so from the
    // start of an op's last tile in this CTA until that op's release the
    // producer issues nothing past tile gate_until. gate_set counts gates
    // requested (consumer thread 0), gate_clr releases done.
    uint32_t gate_set, gate_clr, gate_until;
};

__device__ __forceinline__ void bar_sync(uint32_t id, uint32_t n) {
    asm volatile("bar.sync %0, %1;\n" :: "r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t id, uint32_t n) {
    asm volatile("bar.arrive %0, %1;\n" :: "r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void cbar() { bar_sync(kBarCons, kCT); }
__device__ __forceinline__ bool cbar_or(bool v) {
    uint32_t r;
    asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n"
                 " selp.u32 %0, 1, 0, q;\n}\n"
                 : "=r"(r) : "r"((uint32_t)v), "n"(kCT) : "memory");
    return r != 0;
}
__device__ __forceinline__ uint32_t ld_acq(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t vload(const uint32_t* p) { return *reinterpret_cast<const volatile uint32_t*>(p); }
__device__ __forceinline__ void vstore(uint32_t* p, uint32_t v) { *reinterpret_cast<volatile uint32_t*>(p) = v; }
__device__ __forceinline__ void signal(uint32_t* ctr, uint32_t n) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" :: "l"(ctr), "r"(n) : "memory");
}

__device__ void fail(const FlowArgs& a, FlowShared& S) {
    atomicOr(&a.st->err, kErrWaitTimeout);
    atomicExch(&a.sync->abort, 1u);
    vstore(&S.abort, 1u);
}
// Inside wait loops: this CTA's flag or the global one (an L2 round trip, so
// only checked while waiting anyway); a global abort is remembered locally.
__device__ __forceinline__ bool aborted(const FlowArgs& a, FlowShared& S) {
    if (vload(&S.abort) != 0u) return true;
    if (vload(&a.sync->abort) == 0u) return false;
    vstore(&S.abort, 1u);
    return true;
}
// Outside wait loops: this CTA's flag only (shared memory). A CTA learns of
// another CTA's abort in its next wait.
__device__ __forceinline__ bool stopped(FlowShared& S) { return vload(&S.abort) != 0u; }
// The same answer for every lane of the warp (before warp-collective code).
__device__ __forceinline__ bool warp_stopped(FlowShared& S) { return __any_sync(0xffffffffu, stopped(S)); }
// Bounded wait until *ctr >= target (wrapping compare); false after an abort
// or once kWaitNs has passed.
__device__ bool dep_wait(const FlowArgs& a, FlowShared& S, const uint32_t* ctr, uint32_t target) {
    const uint64_t t0 = gtime();
    for (uint32_t i = 0;; i++) {
        if ((int32_t)(ld_acq(ctr) - target) >= 0) return true;
        if ((i & 63u) == 63u) {
            if (aborted(a, S)) { vstore(&S.abort, 1u); return false; }
            if (gtime() - t0 > kWaitNs) { fail(a, S); return false; }
        }
    }
}
__device__ __forceinline__ bool mbar_test(uint32_t adr, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n" : "=r"(done) : "r"(adr), "r"(parity) : "memory");
    return done != 0;
}
__device__ bool tile_wait(const FlowArgs& a, FlowShared& S, uint64_t* bar, uint32_t parity) {
    const uint32_t adr = smem_u32(bar);
    const uint64_t t0 = gtime();
    for (uint32_t i = 0;; i++) {
        if (mbar_test(adr, parity)) return true;
        if ((i & 15u) == 15u) {
            if (aborted(a, S)) return false;
            if (gtime() - t0 > kWaitNs) { fail(a, S); return false; }
        }
    }
}
// The wait target of op `o` (step E): its predecessor's completions so far.
__device__ __forceinline__ const uint32_t* wait_ctr(const FlowArgs& a, const FlowOp& op) {
    return op.wait == kFlowStepStart ? &a.sync->step_done : &a.done[op.wait];
}
__device__ __forceinline__ uint32_t wait_target(const FlowOp& op, uint32_t E) {
    return op.wait == kFlowStepStart ? E : (E + 1) * op.wait_n;
}

// ------------------------------------------------------------------ records

// E with max|x| * 2^E in [2^13, 2^14): 14 minus frexp's exponent of the group's
// largest magnitude, read from the float's exponent field (a zero or subnormal
// maximum gives the upper clamp, inf or NaN the lower one).
__device__ __forceinline__ int group_exp(float m) {
    const int e = (int)((__float_as_uint(m) >> 23) & 0xFFu) - 126;
    const int E = 14 - e;
    return E > 100 ? 100 : (E < -100 ? -100 : E);
}
__device__ __forceinline__ float pow2(int e) { return __int_as_float((e + 127) << 23); }
__device__ __forceinline__ uint32_t hbits(__half h) { return (uint32_t)__half_as_ushort(h); }

// Record of group G from 16 lanes (lane r < 16 holds element r; lanes 16..31
// pass 0): y the value, sq its raw square (summed into ss when norm).
__device__ void put_record16(const FlowRec& R, uint32_t G, float y, float sq, bool norm, uint32_t lane) {
    float m = fabsf(y), sy = y, s2 = sq;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        sy += __shfl_xor_sync(0xffffffffu, sy, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    const int E = group_exp(m);
    const float xs = y * pow2(E);
    const __half hh = __float2half_rn(xs);
    const __half hl = __float2half_rn(xs - __half2float(hh));
    const uint32_t hb = hbits(hh), lb = hbits(hl);
    // word w (of 8) pairs elements a and a + 2, a = 4 (w / 2) + w % 2
    const uint32_t w = lane & 7u, src = 4u * (w >> 1) + (w & 1u);
    const uint32_t h0 = __shfl_sync(0xffffffffu, hb, src), h2 = __shfl_sync(0xffffffffu, hb, src + 2);
    const uint32_t l0 = __shfl_sync(0xffffffffu, lb, src), l2 = __shfl_sync(0xffffffffu, lb, src + 2);
    if (lane < 16) R.w[(uint64_t)G * 16 + lane] = lane < 8 ? (h0 | (h2 << 16)) : (l0 | (l2 << 16));
    if (lane == 0) {
        R.fs[G] = make_float2(pow2(24 - E), sy);
        if (norm) R.ss[G] = s2;
    }
}

// The same record from one thread holding all 16 values (y) and their raw sum
// of squares.
__device__ void put_record1(const FlowRec& R, uint32_t G, const float* y, float sq, bool norm) {
    float m = 0.f, sy = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) { m = fmaxf(m, fabsf(y[i])); sy += y[i]; }
    const int E = group_exp(m);
    const float F = pow2(E);
    uint32_t hb[16], lb[16];
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const float xs = y[i] * F;
        const __half hh = __float2half_rn(xs);
        hb[i] = hbits(hh);
        lb[i] = hbits(__float2half_rn(xs - __half2float(hh)));
    }
    uint4* dst = reinterpret_cast<uint4*>(R.w + (uint64_t)G * 16);
#pragma unroll
    for (int q = 0; q < 2; q++) {          // q = 0: high words, 1: low words
        const uint32_t* b = q ? lb : hb;
        uint32_t wd[8];
#pragma unroll
        for (int w = 0; w < 8; w++) {
            const int s = 4 * (w >> 1) + (w & 1);
            wd[w] = b[s] | (b[s + 2] << 16);
        }
        dst[2 * q] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        dst[2 * q + 1] = make_uint4(wd[4], wd[5], wd[6], wd[7]);
    }
    R.fs[G] = make_float2(pow2(24 - E), sy);
    if (norm) R.ss[G] = sq;
}

// ------------------------------------------------------------------ input fragments
// For one 256-element super-block of K, a lane (g8 = lane / 4, tig = lane % 4,
// slot = g8 / 2, part = g8 % 2) supplies the B words (high part for even g8,
// low part for odd) of the four 16-element groups 4 slot + k, k = 0..3, of its
// slot, and after the MMA chains holds the products of slot tig, so it also
// needs 2^(24-E) and the sums of groups 4 tig + k. Both tile formats arrange
// their MMAs so that slot s covers elements 64s .. 64s + 63 (sb_q4k, sb_q6k).
struct XFrag {
    uint2 b[4];
    float2 fs[4];
};

// Encodes a lane's four merged values v of each group k into its fragment
// words and the group scales (quad reductions; see frag_attn).
__device__ __forceinline__ XFrag encode_frag(const float4* vk, uint32_t part, uint32_t tig) {
    XFrag X;
    float fk[4], sk[4];
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) {
        const float4 v = vk[k];
        float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
        float sy = (v.x + v.y) + (v.z + v.w);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        sy += __shfl_xor_sync(0xffffffffu, sy, 1);
        sy += __shfl_xor_sync(0xffffffffu, sy, 2);
        const int E = group_exp(m);
        const float F = pow2(E);
        const float x0 = v.x * F, x1 = v.y * F, x2 = v.z * F, x3 = v.w * F;
        const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
        const __half h2 = __float2half_rn(x2), h3 = __float2half_rn(x3);
        uint32_t p0, p1, p2, p3;
        if (part == 0) {
            p0 = hbits(h0); p1 = hbits(h1); p2 = hbits(h2); p3 = hbits(h3);
        } else {
            p0 = hbits(__float2half_rn(x0 - __half2float(h0)));
            p1 = hbits(__float2half_rn(x1 - __half2float(h1)));
            p2 = hbits(__float2half_rn(x2 - __half2float(h2)));
            p3 = hbits(__float2half_rn(x3 - __half2float(h3)));
        }
        X.b[k] = make_uint2(p0 | (p2 << 16), p1 | (p3 << 16));
        fk[k] = pow2(24 - E);
        sk[k] = sy;
    }
    // lane 8 tig has slot tig: its groups are the ones this lane scales
#pragma unroll
    for (uint32_t k = 0; k < 4; k++)
        X.fs[k] = make_float2(__shfl_sync(0xffffffffu, fk[k], 8 * tig), __shfl_sync(0xffffffffu, sk[k], 8 * tig));
    return X;
}

// Heads smaller than 64: each group merged on its own (merge_head4).
__device__ XFrag frag_attn_small(const FlowOp& op, uint32_t ns, uint32_t sb, uint32_t slot, uint32_t part,
                                 uint32_t tig) {
    const AttnArgs& at = op.at;
    const uint32_t hd = at.hd, stride = attn_part_stride(hd), NS = op.n_split;
    float4 v[4];
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) {
        const uint32_t e = 256u * sb + 64u * slot + 16u * k + 4u * tig, h = e / hd, d = e - h * hd;
        v[k] = merge_head4(at.part + (uint64_t)h * NS * stride, ns, stride, d);
    }
    return encode_frag(v, part, tig);
}

// Fragments from the attention partials: the lane merges its four elements of
// each of its four groups (the per-op attention kernel's merge, attn_core.cuh:
// weights exp(m_s - max m) in split order), the quad (4 lanes of one group)
// finds the group's exponent and sum. The four groups are 64 consecutive
// elements of one head (head sizes are multiples of 64), so the split weights
// are computed once and every load is issued before the first use.
__device__ XFrag frag_attn(const FlowOp& op, uint32_t ns, uint32_t sb, uint32_t slot, uint32_t part, uint32_t tig) {
    const AttnArgs& at = op.at;
    const uint32_t hd = at.hd, stride = attn_part_stride(hd), NS = op.n_split;
    const uint32_t e0 = 256u * sb + 64u * slot + 4u * tig, h = e0 / hd, d0 = e0 - h * hd;
    const float* src = at.part + (uint64_t)h * NS * stride;
    float4 acc[4];
#pragma unroll
    for (int k = 0; k < 4; k++) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    float M = -INFINITY, Ls = 0.f;
    if (hd % 64 != 0) {
        // heads of 16 or 32: the four groups may span heads; merge each group alone
        return frag_attn_small(op, ns, sb, slot, part, tig);
    }
    // the two lanes holding the same elements (high and low part, lane ^ 4)
    // weight alternate pairs of splits; with at most four splits one round of
    // loads brings every (m, l) and both of the lane's splits' values. The sums
    // are added in a fixed order (every CTA gets the same bits).
    if (ns <= 4) {
        float2 ml[4];
        float4 v0[4], v1[4];
        const uint32_t s0 = 2 * part, s1 = s0 + 1;
#pragma unroll
        for (uint32_t s = 0; s < 4; s++)
            ml[s] = s < ns ? __ldcg(reinterpret_cast<const float2*>(src + s * stride)) : make_float2(-INFINITY, 0.f);
#pragma unroll
        for (uint32_t k = 0; k < 4; k++) {
            v0[k] = s0 < ns ? __ldcg(reinterpret_cast<const float4*>(src + s0 * stride + 4 + d0 + 16 * k))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
            v1[k] = s1 < ns ? __ldcg(reinterpret_cast<const float4*>(src + s1 * stride + 4 + d0 + 16 * k))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (uint32_t s = 0; s < 4; s++) M = fmaxf(M, ml[s].x);
        const float2 m0 = part ? ml[2] : ml[0], m1 = part ? ml[3] : ml[1];
        const float w0 = s0 < ns ? expf(m0.x - M) : 0.f, w1 = s1 < ns ? expf(m1.x - M) : 0.f;
        Ls = fmaf(w1, m1.y, fmaf(w0, m0.y, 0.f));
#pragma unroll
        for (uint32_t k = 0; k < 4; k++) {
            acc[k].x = fmaf(v1[k].x, w1, v0[k].x * w0);
            acc[k].y = fmaf(v1[k].y, w1, v0[k].y * w0);
            acc[k].z = fmaf(v1[k].z, w1, v0[k].z * w0);
            acc[k].w = fmaf(v1[k].w, w1, v0[k].w * w0);
        }
    } else {
        for (uint32_t s = 0; s < ns; s++) M = fmaxf(M, __ldcg(src + s * stride));
        for (uint32_t s0 = 2 * part; s0 < ns; s0 += 4) {
            const uint32_t s1 = s0 + 1 < ns ? s0 + 1 : s0;
            const float2 m0 = __ldcg(reinterpret_cast<const float2*>(src + s0 * stride));
            const float2 m1 = __ldcg(reinterpret_cast<const float2*>(src + s1 * stride));
            float4 v0[4], v1[4];
#pragma unroll
            for (uint32_t k = 0; k < 4; k++) {
                v0[k] = __ldcg(reinterpret_cast<const float4*>(src + s0 * stride + 4 + d0 + 16 * k));
                v1[k] = __ldcg(reinterpret_cast<const float4*>(src + s1 * stride + 4 + d0 + 16 * k));
            }
            const float w0 = expf(m0.x - M), w1 = s1 != s0 ? expf(m1.x - M) : 0.f;
            Ls = fmaf(w1, m1.y, fmaf(w0, m0.y, Ls));
#pragma unroll
            for (uint32_t k = 0; k < 4; k++) {
                acc[k].x = fmaf(v1[k].x, w1, fmaf(v0[k].x, w0, acc[k].x));
                acc[k].y = fmaf(v1[k].y, w1, fmaf(v0[k].y, w0, acc[k].y));
                acc[k].z = fmaf(v1[k].z, w1, fmaf(v0[k].z, w0, acc[k].z));
                acc[k].w = fmaf(v1[k].w, w1, fmaf(v0[k].w, w0, acc[k].w));
            }
        }
    }
    // part 0 took splits 0, 1, 4, 5, ..., part 1 splits 2, 3, 6, 7, ...: add them
    // with the part-0 sum first on both lanes
    {
        const float o = __shfl_xor_sync(0xffffffffu, Ls, 4);
        Ls = part == 0 ? Ls + o : o + Ls;
    }
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) {
        float4 o;
        o.x = __shfl_xor_sync(0xffffffffu, acc[k].x, 4);
        o.y = __shfl_xor_sync(0xffffffffu, acc[k].y, 4);
        o.z = __shfl_xor_sync(0xffffffffu, acc[k].z, 4);
        o.w = __shfl_xor_sync(0xffffffffu, acc[k].w, 4);
        acc[k] = part == 0 ? make_float4(acc[k].x + o.x, acc[k].y + o.y, acc[k].z + o.z, acc[k].w + o.w)
                           : make_float4(o.x + acc[k].x, o.y + acc[k].y, o.z + acc[k].z, o.w + acc[k].w);
    }
    float4 vk[4];
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) vk[k] = make_float4(acc[k].x / Ls, acc[k].y / Ls, acc[k].z / Ls, acc[k].w / Ls);
    return encode_frag(vk, part, tig);
}

// Per-warp staging of the input fragments in shared memory (the attention
// staging area, idle during GEMV ops): for each of the warp's super-blocks, the
// 16 groups' 16 words and their (2^(24-E), sum) pairs, in record layout.
constexpr uint32_t kXsSbBytes = 16 * 64 + 16 * 8;
constexpr uint32_t kXsWarpBytes = kFlowMaxSb * kXsSbBytes;
__host__ __device__ __forceinline__ uint32_t xs_bytes() { return kCW * kXsWarpBytes; }

// The records of the warp's nsb (<= kFlowMaxSb) super-blocks warp, warp + 8, ...
// into its slots with cp.async (no registers), every copy in flight at once: one
// L2 round trip for all of them. Records are 16-byte aligned (256-word groups of
// words, 16-entry groups of scales) and so are the slots.
__device__ __forceinline__ void stage_recs(const FlowRec& R, uint32_t warp, uint32_t nsb, uint8_t* xs, uint32_t lane) {
    for (uint32_t s = 0; s < nsb; s++) {
        const uint32_t sb = warp + kCW * s;
        const uint8_t* w = reinterpret_cast<const uint8_t*>(R.w + (uint64_t)sb * 256);
        const uint8_t* f = reinterpret_cast<const uint8_t*>(R.fs + (uint64_t)sb * 16);
        uint8_t* d = xs + s * kXsSbBytes;
        cp_async16(d + 16 * lane, w + 16 * lane);
        cp_async16(d + 512 + 16 * lane, w + 512 + 16 * lane);
        if (lane < 8) cp_async16(d + 1024 + 16 * lane, f + 16 * lane);
    }
    cp_async_wait_all();
}
// Store a lane's fragment (computed in registers) into slot s of the slice.
__device__ __forceinline__ void stage_frag(const XFrag& X, uint8_t* xs, uint32_t slot, uint32_t part, uint32_t tig,
                                           uint32_t g8) {
    uint32_t* w = reinterpret_cast<uint32_t*>(xs);
#pragma unroll
    for (uint32_t k = 0; k < 4; k++)
        *reinterpret_cast<uint2*>(w + (4 * slot + k) * 16 + 8 * part + 2 * tig) = X.b[k];
    if (g8 == 0) {
        float2* fs = reinterpret_cast<float2*>(xs + 16 * 64);
#pragma unroll
        for (uint32_t k = 0; k < 4; k++) fs[4 * tig + k] = X.fs[k];
    }
}
// A lane's fragment of one staged super-block.
__device__ __forceinline__ XFrag load_frag(const uint8_t* xs, uint32_t slot, uint32_t part, uint32_t tig) {
    XFrag X;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(xs);
    const float2* fs = reinterpret_cast<const float2*>(xs + 16 * 64);
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) {
        X.b[k] = *reinterpret_cast<const uint2*>(w + (4 * slot + k) * 16 + 8 * part + 2 * tig);
        X.fs[k] = fs[4 * tig + k];
    }
    return X;
}

// ------------------------------------------------------------------ tile math
// Rows g8 and g8 + 8 of a 16-row tile, one super-block (bytes at rg, rg8 in
// shared memory). Every format is affine per group of weights (w = alpha q -
// beta); the integers enter the MMA as fp16 subnormals (q 2^-24), x as the
// record's fp16 pair, and alpha, beta and 2^(24-E) are applied in f32 after.

// Q4_K (gguf.c:504-529): in 64-element group j, byte b of qs[32j..32j+32) holds
// element 64j + b (low nibble) and 64j + 32 + b (high nibble). Lane tig takes
// bytes 4 tig..4 tig+3 of each 16-byte half, so one MMA covers 16 consecutive
// elements (one record group).
__device__ __forceinline__ void sb_q4k(const uint8_t* rg, const uint8_t* rg8, const XFrag& X, uint32_t slot,
                                       uint32_t tig, float& a0, float& a1) {
    const uint4 h = *reinterpret_cast<const uint4*>(rg), h8 = *reinterpret_cast<const uint4*>(rg8);
    float c[4][4];
#pragma unroll
    for (int k = 0; k < 4; k++) c[k][0] = c[k][1] = c[k][2] = c[k][3] = 0.f;
    constexpr uint32_t L4 = 0x000F000Fu, H4 = 0x00F000F0u;
#pragma unroll
    for (uint32_t j = 0; j < 4; j++) {
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(rg + 16 + 32 * j + 4 * tig);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(rg + 32 + 32 * j + 4 * tig);
        const uint32_t v0 = *reinterpret_cast<const uint32_t*>(rg8 + 16 + 32 * j + 4 * tig);
        const uint32_t v1 = *reinterpret_cast<const uint32_t*>(rg8 + 32 + 32 * j + 4 * tig);
        const uint32_t on = slot == j ? 0xFFFFFFFFu : 0u;
        const uint32_t w0s = w0 >> 8, w1s = w1 >> 8, v0s = v0 >> 8, v1s = v1 >> 8;
        mma16816(c[0], w0 & L4, v0 & L4, w0s & L4, v0s & L4, X.b[0].x & on, X.b[0].y & on);
        mma16816(c[1], w1 & L4, v1 & L4, w1s & L4, v1s & L4, X.b[1].x & on, X.b[1].y & on);
        mma16816(c[2], w0 & H4, v0 & H4, w0s & H4, v0s & H4, X.b[2].x & on, X.b[2].y & on);
        mma16816(c[3], w1 & H4, v1 & H4, w1s & H4, v1s & H4, X.b[3].x & on, X.b[3].y & on);
    }
    float sl, ml, sh, mh, tl, nl, th, nh;
    FQ4K::scales(h.y, h.z, h.w, tig, &sl, &ml, &sh, &mh);
    FQ4K::scales(h8.y, h8.z, h8.w, tig, &tl, &nl, &th, &nh);
    const float dg = h2f(h.x & 0xFFFFu), mg = h2f(h.x >> 16);
    const float dg8 = h2f(h8.x & 0xFFFFu), mg8 = h2f(h8.x >> 16);
    // sub-block 2 tig = groups k 0, 1; sub-block 2 tig + 1 = groups 2, 3 (16 q in place)
    const float pl = fmaf(X.fs[0].x, c[0][0] + c[0][1], X.fs[1].x * (c[1][0] + c[1][1]));
    const float pl8 = fmaf(X.fs[0].x, c[0][2] + c[0][3], X.fs[1].x * (c[1][2] + c[1][3]));
    const float ph = fmaf(X.fs[2].x, c[2][0] + c[2][1], X.fs[3].x * (c[3][0] + c[3][1]));
    const float ph8 = fmaf(X.fs[2].x, c[2][2] + c[2][3], X.fs[3].x * (c[3][2] + c[3][3]));
    const float sxl = X.fs[0].y + X.fs[1].y, sxh = X.fs[2].y + X.fs[3].y;
    a0 = fmaf(dg * sl, pl, fmaf(-mg * ml, sxl, a0));
    a0 = fmaf(dg * sh * 0.0625f, ph, fmaf(-mg * mh, sxh, a0));
    a1 = fmaf(dg8 * tl, pl8, fmaf(-mg8 * nl, sxl, a1));
    a1 = fmaf(dg8 * th * 0.0625f, ph8, fmaf(-mg8 * nh, sxh, a1));
}

// Q6_K (gguf.c:561-590): per 128-half H, byte l of ql[64H..], ql[64H+32..] and
// qh[32H..] give elements 128H + 32c + l (c = 0..3), each 16 of them (l / 16 =
// u) one scale group sc[8H + 2c + u] = record group 8H + 2c + u. The MMA of
// (H, u, c) covers that group and is slot 2H + c / 2, so the chain of (u, c %
// 2) over H and c / 2 visits every slot once; slot s's groups are then 4s + k
// with k = 2 (c % 2) + u, as for Q4_K.
__device__ __forceinline__ void sb_q6k(const uint8_t* bg, const uint8_t* bg8, const XFrag& X, uint32_t slot,
                                       uint32_t tig, float& a0, float& a1) {
    const float dg = h2f(lds_u16(bg + 208)), dg8 = h2f(lds_u16(bg8 + 208));
    float cc[4][4];
#pragma unroll
    for (int k = 0; k < 4; k++) cc[k][0] = cc[k][1] = cc[k][2] = cc[k][3] = 0.f;
#pragma unroll
    for (uint32_t H = 0; H < 2; H++) {
#pragma unroll
        for (uint32_t u = 0; u < 2; u++) {
            const uint32_t off = 16 * u + 4 * tig;
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
                const uint32_t k = 2 * (c & 1u) + u;
                const uint32_t on = slot == 2 * H + (c >> 1) ? 0xFFFFFFFFu : 0u;
                mma16816(cc[k], __byte_perm(wq[c], 0, 0x4240), __byte_perm(wm[c], 0, 0x4240),
                         __byte_perm(wq[c], 0, 0x4341), __byte_perm(wm[c], 0, 0x4341), X.b[k].x & on,
                         X.b[k].y & on);
            }
        }
    }
    // this lane: slot tig, group 4 tig + k, scale sc[4 tig + k]
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) {
        const uint32_t si = 192 + 4 * tig + k;
        const float ag = dg * (float)(int8_t)bg[si], ag8 = dg8 * (float)(int8_t)bg8[si];
        a0 = fmaf(ag * X.fs[k].x, cc[k][0] + cc[k][1], fmaf(-32.0f * ag, X.fs[k].y, a0));
        a1 = fmaf(ag8 * X.fs[k].x, cc[k][2] + cc[k][3], fmaf(-32.0f * ag8, X.fs[k].y, a1));
    }
}

__host__ __device__ __forceinline__ bool flow_glu(uint32_t epi) { return epi == EPI_GLU_SILU || epi == EPI_GLU_GELU; }
__host__ __device__ __forceinline__ uint32_t sb_bytes(uint32_t type) { return type == T_Q6_K ? 210u : 144u; }
// Ring bytes of a tile (sized for 16 rows; 16 bytes of slack for word reads).
__host__ __device__ __forceinline__ uint32_t ftile_alloc(const FlowSeg& G) {
    const uint32_t t1 = tile_bytes(G.row_bytes);
    const uint32_t body = flow_glu(G.epi) ? t1 + tile_bytes(G.row_bytes2) : t1;
    return (body + 16 + 127) & ~127u;
}

struct FTile {
    uint32_t seg, row0, nrows;
};
__device__ __forceinline__ FTile ftile_of(const FlowOp& op, uint32_t t) {
    uint32_t s = 0;
#pragma unroll
    for (uint32_t i = 1; i < 3; i++)
        if (i < op.nseg && t >= op.seg[i].tile0) s = i;
    const FlowSeg& G = op.seg[s];
    const uint32_t row0 = (t - G.tile0) * 16;
    return FTile{s, row0, min(16u, G.rows - row0)};
}

// ------------------------------------------------------------------ attention task

template <typename KV>
__device__ void attn_prefetch(const FlowOp& op, uint32_t task, uint32_t pos, float* stage, uint32_t tid) {
    const AttnArgs& at = op.at;
    const uint32_t h = task / op.n_split, split = task - h * op.n_split;
    const uint32_t g = h / (at.n_heads / at.n_kv);
    const SplitRange r = split_range(pos, op.n_split, split);
    if (split >= r.ns) return;
    const uint32_t hd = at.hd;
    const AttnSm sm = attn_carve(stage, hd, sizeof(KV) == 2);
    const KV* kc = reinterpret_cast<const KV*>(at.kc) + (uint64_t)g * at.max_seq * hd;
    const KV* vc = reinterpret_cast<const KV*>(at.vc) + (uint64_t)g * at.max_seq * hd;
    const uint32_t n = min(kAttnChunk, r.t1 - r.t0);
    const uint32_t nold = (r.t0 + n > pos) ? pos - r.t0 : n;
    attn_stage_async<KV>(sm, kc, vc, r.t0, nold, hd, tid, kCT);
}

// Task (head, split) of causal_mha (model.c:217-260) at the current position:
// RoPE of q and the new k, the cache write (one writer per kv head), the
// split's partial (m, l, o) for the O projection's merge.
template <typename KV>
__device__ void attn_task(const FlowOp& op, uint32_t task, uint32_t pos, float* stage, bool staged, uint32_t tid) {
    const AttnArgs& at = op.at;
    const uint32_t h = task / op.n_split, split = task - h * op.n_split;
    const uint32_t g = h / (at.n_heads / at.n_kv);
    const SplitRange r = split_range(pos, op.n_split, split);
    if (split >= r.ns) return;
    const uint32_t hd = at.hd, G = at.n_heads / at.n_kv;
    const AttnSm sm = attn_carve(stage, hd, sizeof(KV) == 2);
    const bool has_new = r.t0 <= pos && pos < r.t1;
    for (uint32_t i = tid; i < hd; i += kCT) {
        sm.qs[i] = __ldcg(at.qkv + (uint64_t)h * hd + i);
        if (has_new) {
            sm.kn[i] = __ldcg(at.qkv + (uint64_t)at.n_heads * hd + (uint64_t)g * hd + i);
            sm.vn[i] = __ldcg(at.qkv + (uint64_t)(at.n_heads + at.n_kv) * hd + (uint64_t)g * hd + i);
        }
    }
    cbar();
    rope_pairs(sm.qs, hd, pos, at.rope, at.theta, tid, kCT);
    if (has_new) rope_pairs(sm.kn, hd, pos, at.rope, at.theta, tid, kCT);
    cbar();
    KV* kc = reinterpret_cast<KV*>(at.kc) + (uint64_t)g * at.max_seq * hd;
    KV* vc = reinterpret_cast<KV*>(at.vc) + (uint64_t)g * at.max_seq * hd;
    if (has_new && h == g * G) {
        for (uint32_t i = tid; i < hd; i += kCT) {
            kv_put(kc + (uint64_t)pos * hd + i, sm.kn[i]);
            kv_put(vc + (uint64_t)pos * hd + i, sm.vn[i]);
        }
    }
    const float o = attn_chunks<KV>(sm, kc, vc, pos, r.t0, r.t1, hd, tid, kCT, staged, [] { cbar(); });
    const uint32_t stride = attn_part_stride(hd);
    float* dst = at.part + ((uint64_t)h * op.n_split + split) * stride;
    if (tid < hd) dst[4 + tid] = o;
    if (tid == 0) { dst[0] = sm.sc[kAttnChunk + 4]; dst[1] = sm.sc[kAttnChunk + 5]; }
}

// ------------------------------------------------------------------ step input

// Embedding row of `token` (tensor_get_row, tensor.c:24-30), scaled, into the
// residual stream, and its records (first layer's norm weight folded in). One
// warp; a lane encodes whole groups.
__device__ void embed_row(const FlowArgs& a, uint32_t token, uint32_t lane) {
    decode_row_part(a.tok, token, a.hidden, a.emb_scale, false, lane, 32);
    __syncwarp();
    const uint32_t ng = a.dim / 16;
    for (uint32_t G = lane; G < ng; G += 32) {
        float y[16];
        float sq = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const float hv = __ldcg(a.hidden + 16 * G + i);
            y[i] = hv * a.n1w0[16 * G + i];
            sq = fmaf(hv, hv, sq);
        }
        put_record1(a.in0, G, y, sq, true);
    }
}

// After the last lm_head tile of a step (one warp): the next token from the
// argmax (generate.c:143-156), the next position, the next input's records,
// then the next step is released.
__device__ void finish_step(const FlowArgs& a, uint32_t lane) {
    uint32_t nt = 0;
    if (lane == 0) {
        __threadfence();
        StepState* st = a.st;
        const unsigned long long k = atomicAdd(&st->argmax_key, 0ull);
        const uint32_t pos = vload(&st->pos);
        const uint32_t np = vload(&st->n_prompt);
        if (pos + 1 >= np && pos + 1 < a.max_tokens)
            a.tokens[pos + 1] = k ? 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull) : 0u;
        atomicExch(&st->argmax_key, 0ull);
        vstore(&st->pos, pos + 1);
        nt = pos + 1 < a.max_tokens ? vload(&a.tokens[pos + 1]) : 0u;
        if (nt >= a.tok.rows) nt = 0;                  // out-of-range ids read row 0
    }
    nt = __shfl_sync(0xffffffffu, nt, 0);
    embed_row(a, nt, lane);
    __syncwarp();
    if (lane == 0) {
        __threadfence();
        atomicAdd(&a.sync->step_done, 1u);
    }
}

// ------------------------------------------------------------------ roles

__device__ void producer(const FlowArgs& a, FlowShared& S, uint8_t* ring) {
    const uint32_t n_my = a.sched_len[blockIdx.x];
    const uint64_t R = a.ring_bytes;
    uint64_t head = 0;
    uint32_t seq = 0;
    for (uint32_t j = 0; j < a.n_steps; j++) {
        for (uint32_t i = 0; i < n_my; i++) {
            const uint32_t ent = S.tasks[i];
            if (S.ops_kind[ent >> 16] != FLOW_GEMV) continue;
            const FlowOp& op = a.ops[ent >> 16];
            const FTile tr = ftile_of(op, ent & 0xFFFFu);
            const FlowSeg& G = op.seg[tr.seg];
            const bool glu = flow_glu(G.epi);
            const uint32_t n1 = tile_tx(G.row_bytes, tr.nrows, G.map != nullptr);
            const uint32_t n2 = glu ? tile_tx(G.row_bytes2, tr.nrows, G.map2 != nullptr) : 0u;
            const uint32_t alloc = ftile_alloc(G);
            uint64_t off = head % R;
            if (off + alloc > R) { head += R - off; off = 0; }
            bool ok = false;
            const uint64_t t0 = gtime();
            for (uint32_t w = 0;; w++) {
                const uint32_t c = vload(&S.consumed);
                const uint64_t tail = c == 0 ? 0ull : S.vend[(c - 1) % kQ];
                const bool gated = vload(&S.gate_set) != vload(&S.gate_clr) &&
                                   (int32_t)(seq - vload(&S.gate_until)) > 0;
                if (seq - c < kQ && head + alloc - tail <= R && !gated) { ok = true; break; }
                __nanosleep(64);                  // leave the SM's issue slots to the other warps
                if ((w & 63u) == 63u && (aborted(a, S) || gtime() - t0 > kWaitNs)) break;
            }
            if (!ok || stopped(S)) {
                if (!stopped(S)) fail(a, S);
                vstore(&S.abort, 1u);
                return;
            }
            if (i == 0 || (S.tasks[i - 1] >> 16) != (ent >> 16)) FLOW_TL(j, a.n_steps, ent >> 16, 7);
            const uint32_t q = seq % kQ;
            S.off[q] = (uint32_t)off;
            S.vend[q] = head + alloc;
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            mbar_expect_tx(&S.bar[q], n1 + n2);
            if (G.map) tma_tile(ring + off, G.map, (int32_t)tr.row0, &S.bar[q]);
            else copy_rows(ring + off, G.w + (uint64_t)tr.row0 * G.row_bytes, G.row_bytes, tr.nrows, &S.bar[q]);
            if (glu) {
                uint8_t* up = ring + off + tile_bytes(G.row_bytes);
                if (G.map2) tma_tile(up, G.map2, (int32_t)tr.row0, &S.bar[q]);
                else copy_rows(up, G.w2 + (uint64_t)tr.row0 * G.row_bytes2, G.row_bytes2, tr.nrows, &S.bar[q]);
            }
            head += alloc;
            seq++;
            vstore(&S.issued, seq);
        }
    }
}

__device__ void consumer(const FlowArgs& a, FlowShared& S, uint8_t* ring, float* stage, uint32_t tid) {
    const uint32_t lane = tid & 31u, warp = tid >> 5;
    const uint32_t g8 = lane >> 2, tig = lane & 3u, slot = g8 >> 1, part = g8 & 1u;
    const uint32_t n_my = a.sched_len[blockIdx.x];
    const FlowOp& op = S.cop;
    uint32_t cseq = 0;
    uint32_t gset = 0;                   // gates requested (thread 0)
    uint8_t* xs = reinterpret_cast<uint8_t*>(stage) + warp * kXsWarpBytes;   // this warp's fragments
    uint32_t nsb = 0;
    for (uint32_t j = 0; j < a.n_steps; j++) {
        const uint32_t E = S.epoch + j;
        uint32_t run_op = 0xFFFFFFFFu, run_n = 0;
        for (uint32_t i = 0; i < n_my; i++) {
            const uint32_t ent = S.tasks[i], op_i = ent >> 16, task = ent & 0xFFFFu;
            const bool gemv = S.ops_kind[op_i] == FLOW_GEMV;
            bool prefetched = false;
            if (op_i != run_op) {
                cbar();                        // every consumer is done with the previous descriptor
                {
                    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.ops + op_i);
                    uint32_t* dst = reinterpret_cast<uint32_t*>(&S.cop);
                    for (uint32_t w = tid; w < (uint32_t)(sizeof(FlowOp) / 4); w += kCT) dst[w] = __ldg(src + w);
                }
                cbar();
                if (run_op == 0xFFFFFFFFu) {
                    // the step has started (acquire): its position, read here once (it
                    // changes only between steps), and the cache rows of earlier steps
                    bool ok = true;
                    if (tid == 0 && !stopped(S)) {
                        ok = dep_wait(a, S, &a.sync->step_done, E);
                        vstore(&S.pos, vload(&a.st->pos));
                    }
                    cbar_or(!ok);
                }
                if (!gemv) {
                    // cached K/V rows depend only on the step having started
                    if (!cbar_or(stopped(S))) {
                        if (op.at.kv_f16) attn_prefetch<__half>(op, task, vload(&S.pos), stage, tid);
                        else attn_prefetch<float>(op, task, vload(&S.pos), stage, tid);
                        prefetched = true;
                    }
                }
                bool ok = true;
                if (tid == 0 && !stopped(S)) ok = dep_wait(a, S, wait_ctr(a, op), wait_target(op, E));
                cbar_or(!ok);
                if (tid == 0) FLOW_TL(j, a.n_steps, op_i, 0);
                run_op = op_i;
                run_n = 0;
                if (gemv && !warp_stopped(S)) {
                    // this warp's super-blocks of K: warp, warp + 8, ...
                    const uint32_t nsbt = op.K / 256;
                    nsb = warp < nsbt ? (nsbt - warp + kCW - 1) / kCW : 0;
                    uint32_t ns = 1;
                    if (op.in_attn) ns = split_range(vload(&S.pos), op.n_split, 0).ns;
                    if (op.in_attn) {
                        for (uint32_t s = 0; s < nsb; s++)
                            stage_frag(frag_attn(op, ns, warp + kCW * s, slot, part, tig), xs + s * kXsSbBytes, slot,
                                       part, tig, g8);
                    } else {
                        stage_recs(op.in, warp, nsb, xs, lane);
                    }
                    if (tid == 0) FLOW_TL(j, a.n_steps, op_i, 1);
                    __syncwarp();
                }
            }
            if (gemv) {
                const uint32_t b = cseq & 1u;
                bar_sync(kBarFree + b, kPairT);          // partial buffer b was read
                const uint32_t q = cseq % kQ;
                bool ok = false;
                if (!stopped(S)) ok = tile_wait(a, S, &S.bar[q], (cseq / kQ) & 1u);
                ok = __all_sync(0xffffffffu, ok);
                if (tid == 0 && (i == 0 || (S.tasks[i - 1] >> 16) != op_i)) FLOW_TL(j, a.n_steps, op_i, 2);
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                if (ok) {
                    const FTile tr = ftile_of(op, task);
                    const FlowSeg& G = op.seg[tr.seg];
                    const uint8_t* buf = ring + S.off[q];
                    const bool glu = flow_glu(G.epi);
                    const uint64_t rs = smem_rs(G.row_bytes);
                    const uint8_t* up = buf + tile_bytes(G.row_bytes);
                    const uint64_t rs2 = smem_rs(G.row_bytes2);
                    const uint32_t sbb = sb_bytes(G.type);
                    const bool q6 = G.type == T_Q6_K;
                    for (uint32_t s = 0; s < nsb; s++) {
                        const XFrag X = load_frag(xs + s * kXsSbBytes, slot, part, tig);
                        const uint32_t off = (warp + kCW * s) * sbb;
                        const uint8_t* rg = buf + g8 * rs + off;
                        const uint8_t* rg8 = buf + (g8 + 8) * rs + off;
                        if (q6) sb_q6k(rg, rg8, X, slot, tig, acc[0], acc[1]);
                        else sb_q4k(rg, rg8, X, slot, tig, acc[0], acc[1]);
                        if (glu) {
                            const uint8_t* ug = up + g8 * rs2 + off;
                            const uint8_t* ug8 = up + (g8 + 8) * rs2 + off;
                            if (q6) sb_q6k(ug, ug8, X, slot, tig, acc[2], acc[3]);
                            else sb_q4k(ug, ug8, X, slot, tig, acc[2], acc[3]);
                        }
                    }
                }
                if (tid == 0) FLOW_TL(j, a.n_steps, op_i, 3);
                if (tid == 0 && (i + 1 == n_my || (S.tasks[i + 1] >> 16) != op_i)) {
                    // this CTA's last tile of the op is computed (by warp 0 at least):
                    // no new copies until the op's release
                    vstore(&S.gate_until, cseq);
                    vstore(&S.gate_set, ++gset);
                }
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 1);
                    acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 2);
                }
                if (tig == 0) {
                    S.part[b][warp][0][g8] = acc[0];
                    S.part[b][warp][0][g8 + 8] = acc[1];
                    S.part[b][warp][1][g8] = acc[2];
                    S.part[b][warp][1][g8 + 8] = acc[3];
                }
                bar_arrive(kBarDone + b, kPairT);        // partials of buffer b ready
                cseq++;
            } else {
                if (tid == 0 && (i + 1 == n_my || (S.tasks[i + 1] >> 16) != op_i)) {
                    vstore(&S.gate_until, cseq);          // the next GEMV tile may still come
                    vstore(&S.gate_set, ++gset);
                }
                if (!cbar_or(stopped(S))) {
                    if (op.at.kv_f16) attn_task<__half>(op, task, vload(&S.pos), stage, prefetched, tid);
                    else attn_task<float>(op, task, vload(&S.pos), stage, prefetched, tid);
                }
                run_n++;
                const bool last = i + 1 == n_my || (S.tasks[i + 1] >> 16) != op_i;
                if (last) {
                    cbar();                               // every thread's partials are written
                    if (tid == 0) FLOW_TL(j, a.n_steps, op_i, 5);
                    if (tid == 0 && !stopped(S)) signal(&a.done[op_i], run_n);
                    if (tid == 0) FLOW_TL(j, a.n_steps, op_i, 6);
                    if (tid == 0) atomicAdd(&S.gate_clr, 1u);
                }
            }
        }
    }
    // balance the epilogue warp's two extra "buffer free" arrivals
    bar_sync(kBarFree, kPairT);
    bar_sync(kBarFree + 1, kPairT);
}

__device__ void epilogue(const FlowArgs& a, FlowShared& S, uint32_t lane) {
    const uint32_t n_my = a.sched_len[blockIdx.x];
    const FlowOp& op = S.eop;
    bar_arrive(kBarFree, kPairT);                          // both partial buffers start free
    bar_arrive(kBarFree + 1, kPairT);
    uint32_t cseq = 0;
    for (uint32_t j = 0; j < a.n_steps; j++) {
        const uint32_t E = S.epoch + j;
        uint32_t run_op = 0xFFFFFFFFu, run_n = 0;
        float inv = 1.f;
        unsigned long long key = 0ull;
        for (uint32_t i = 0; i < n_my; i++) {
            const uint32_t ent = S.tasks[i], op_i = ent >> 16, task = ent & 0xFFFFu;
            if (S.ops_kind[op_i] != FLOW_GEMV) continue;
            if (op_i != run_op) {
                __syncwarp();
                {
                    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.ops + op_i);
                    uint32_t* dst = reinterpret_cast<uint32_t*>(&S.eop);
                    for (uint32_t w = lane; w < (uint32_t)(sizeof(FlowOp) / 4); w += 32) dst[w] = __ldg(src + w);
                }
                __syncwarp();
                // lane 0 waits; the warp barrier holds every lane until it returns and
                // orders its acquire before the other lanes' loads of the inputs
                if (lane == 0 && !stopped(S)) dep_wait(a, S, wait_ctr(a, op), wait_target(op, E));
                __syncwarp();
                inv = 1.f;
                if (op.in.ss != nullptr && !op.in_attn) {
                    // 1 / rms of the raw input (model.c:7-8), from the producers' group
                    // sums, added in a fixed order (every CTA gets the same bits)
                    const uint32_t ng = op.K / 16;
                    float s = 0.f;
                    // four loads in flight at a time (one L2 round trip for K <= 2048),
                    // added in group order
                    for (uint32_t g0 = lane; g0 < ng; g0 += 128) {
                        float sv[4];
#pragma unroll
                        for (uint32_t i = 0; i < 4; i++) sv[i] = g0 + 32 * i < ng ? __ldcg(op.in.ss + g0 + 32 * i) : 0.f;
#pragma unroll
                        for (uint32_t i = 0; i < 4; i++)
                            if (g0 + 32 * i < ng) s += sv[i];
                    }
                    s = wsum(s);
                    inv = 1.0f / sqrtf(s / (float)op.K + op.eps);
                }
                run_op = op_i;
                run_n = 0;
                key = 0ull;
            }
            const FTile tr = ftile_of(op, task);
            const FlowSeg& G = op.seg[tr.seg];
            const uint32_t row = tr.row0 + lane;
            const bool valid = lane < tr.nrows && !stopped(S);
            float bias = 0.f, res = 0.f, nw = 1.f;
            if (valid) {
                if (G.bias) bias = G.bias[row];
                if (G.epi == EPI_RESID) res = __ldcg(a.hidden + row);
                if (op.out_nw) nw = op.out_nw[row];
            }
            const uint32_t b = cseq & 1u;
            bar_sync(kBarDone + b, kPairT);
            if (lane == 0) FLOW_TL(j, a.n_steps, op_i, 4);
            float v = 0.f, u = 0.f;
            if (lane < 16) {
#pragma unroll
                for (int w = 0; w < kCW; w++) {
                    v += S.part[b][w][0][lane];
                    u += S.part[b][w][1][lane];
                }
            }
            bar_arrive(kBarFree + b, kPairT);
            if (lane == 0) vstore(&S.consumed, cseq + 1);      // the ring tile was read by every warp
            cseq++;
            v *= inv;
            u *= inv;
            float y = 0.f, sq = 0.f;
            if (valid) {
                switch (G.epi) {
                case EPI_STORE: v += bias; G.out[row] = v; y = v; break;
                case EPI_RESID: {                        // the residual add
                    v = res + (v + bias);
                    a.hidden[row] = v;
                    if (a.trace != nullptr && op.trace_off != 0xFFFFFFFFu) a.trace[op.trace_off + row] = v;
                    y = v * nw;
                    sq = v * v;
                    break;
                }
                case EPI_GLU_SILU: v = v / (1.0f + expf(-v)) * u; G.out[row] = v; y = v; break;   // model.c:22
                case EPI_GLU_GELU: v = m_gelu(v) * u; G.out[row] = v; y = v; break;
                default: break;
                }
                if (op.argmax) {
                    const unsigned long long k = m_key(v, row);
                    key = k > key ? k : key;
                }
            }
            const bool wab = warp_stopped(S);
            if (op.out.w != nullptr && !wab) put_record16(op.out, tr.row0 / 16, y, sq, op.out.ss != nullptr, lane);
            run_n++;
            const bool last = i + 1 == n_my || (S.tasks[i + 1] >> 16) != op_i;
            if (last && !wab) {
                // the warp barrier orders every lane's outputs before lane 0's
                // release (cumulative at GPU scope)
                __syncwarp();
                if (!op.argmax) {
                    if (lane == 0) FLOW_TL(j, a.n_steps, op_i, 5);
                    if (lane == 0) signal(&a.done[op_i], run_n);
                    if (lane == 0) FLOW_TL(j, a.n_steps, op_i, 6);
                } else {
                    // lm_head: fold the keys, then the CTA completing the op finishes the step
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
                        key = k2 > key ? k2 : key;
                    }
                    uint32_t fin = 0;
                    if (lane == 0) {
                        if (key != 0ull) atomicMax(&a.st->argmax_key, key);
                        __threadfence();
                        const uint32_t old = atomicAdd(&a.done[op_i], run_n);
                        fin = old + run_n == (E + 1) * op.ntasks ? 1u : 0u;
                    }
                    if (__shfl_sync(0xffffffffu, fin, 0)) finish_step(a, lane);
                }
            }
            if (last && lane == 0) atomicAdd(&S.gate_clr, 1u);    // the op is released: copies may go
        }
    }
}

__global__ void __launch_bounds__(kFT, 1) flow_kernel(const __grid_constant__ FlowArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ FlowShared S;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    // tensor copies need a 128-byte aligned destination
    uint8_t* ring = smem + ((128u - (smem_u32(smem) & 127u)) & 127u);
    float* stage = reinterpret_cast<float*>(ring + a.ring_bytes);
    if (tid == 0) {
        for (uint32_t q = 0; q < kQ; q++) mbar_init(&S.bar[q], 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        S.consumed = 0;
        S.gate_set = 0;
        S.gate_clr = 0;
        S.gate_until = 0;
        S.issued = 0;
        S.abort = vload(&a.sync->abort);
        S.epoch = ld_acq(&a.sync->epoch);
    }
    {
        const uint32_t* my = a.sched + (uint64_t)blockIdx.x * a.sched_stride;
        const uint32_t n_my = a.sched_len[blockIdx.x];
        for (uint32_t i = tid; i < n_my; i += kFT) S.tasks[i] = my[i];
        for (uint32_t o = tid; o < a.n_ops; o += kFT) S.ops_kind[o] = a.ops[o].kind;
    }
    __syncthreads();
    if (warp == kProdWarp) {
        if (lane == 0) producer(a, S, ring);
        __syncwarp();
    } else if (warp == kEpiWarp) {
        epilogue(a, S, lane);
    } else {
        consumer(a, S, ring, stage, tid);
    }
    __syncthreads();
    if (tid == 0) {
        // after an abort tiles may have been skipped unread: wait for every copy
        // that can still be in flight (the last kQ issued; older slots were
        // reissued only after their copy had landed)
        const uint32_t n = vload(&S.issued), c = n > kQ ? n - kQ : 0u;
        const uint64_t t0 = gtime();
        for (uint32_t q = c; q < n; q++) {
            const uint32_t adr = smem_u32(&S.bar[q % kQ]);
            while (!mbar_test(adr, (q / kQ) & 1u) && gtime() - t0 < kWaitNs) {
            }
        }
        __threadfence();
        const uint32_t old = atomicAdd(&a.sync->exit_ticket, 1u);
        if (old + 1 == gridDim.x) {
            a.sync->exit_ticket = 0;
            a.sync->epoch = S.epoch + a.n_steps;
            __threadfence();
        }
    }
}

// The first step's input (the token at the current position), before a launch.
__global__ void flow_embed_kernel(const __grid_constant__ FlowArgs a) {
    const uint32_t lane = threadIdx.x;
    uint32_t nt = 0;
    if (lane == 0) {
        const uint32_t pos = a.st->pos;
        nt = pos < a.max_tokens ? a.tokens[pos] : 0u;
        if (nt >= a.tok.rows) nt = 0;
    }
    nt = __shfl_sync(0xffffffffu, nt, 0);
    embed_row(a, nt, lane);
}

}  // namespace

bool flow_supported_type(uint32_t t) { return t == T_Q4_K || t == T_Q6_K; }

// Shared memory after the ring: the attention staging area, which the GEMV
// ops reuse for their input fragments.
static size_t stage_bytes(uint32_t hd) {
    const size_t at = attn_core_bytes(hd, false), x = xs_bytes();
    return ((at > x ? at : x) + 127) & ~size_t(127);
}

uint32_t flow_ring_bytes(uint32_t hd) {
    const size_t other = stage_bytes(hd) + 128;   // + alignment slack
    if (other + 4096 > kFlowSmem) return 0;
    return (uint32_t)((kFlowSmem - other) & ~size_t(127));
}

uint32_t flow_tile_alloc(const FlowSeg& G) { return ftile_alloc(G); }

// cuTensorMapEncodeTiled from the driver, looked up once.
static PFN_cuTensorMapEncodeTiled_v12000 flow_encoder() {
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

// Rank-3 view of a matrix's rows as uint16: {8 (one 16-byte unit), units per
// row, rows}, strides {16 bytes, row bytes}; box {8, units + 1, 16}.
bool encode_tile_map(CUtensorMap* m, const uint8_t* w, uint64_t rb, uint32_t rows) {
    return encode_box_map(m, w, rb, rows, (uint32_t)(rb / 16 + 1));
}

// The same view with a box of box_units units (a K-chunk of the rows plus one
// unit of padding); rows of a multiple of 16 bytes.
bool encode_box_map(CUtensorMap* m, const uint8_t* w, uint64_t rb, uint32_t rows, uint32_t box_units) {
    PFN_cuTensorMapEncodeTiled_v12000 fn = flow_encoder();
    if (!fn) return false;
    const uint64_t units = rb / 16;
    if (rb % 16 != 0 || box_units == 0 || box_units > 256 || reinterpret_cast<uintptr_t>(w) % 16 != 0) return false;
    cuuint64_t dims[3] = {8, units, rows};
    cuuint64_t strides[2] = {16, rb};
    cuuint32_t box[3] = {8, box_units, 16};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint8_t*>(w), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

uint32_t flow_maps_needed(const FlowOp* ops, uint32_t n_ops) {
    uint32_t n = 0;
    for (uint32_t o = 0; o < n_ops; o++) {
        if (ops[o].kind != FLOW_GEMV) continue;
        for (uint32_t i = 0; i < ops[o].nseg; i++) {
            const FlowSeg& G = ops[o].seg[i];
            n += padded_rows(G.row_bytes) ? 1u : 0u;
            n += flow_glu(G.epi) && padded_rows(G.row_bytes2) ? 1u : 0u;
        }
    }
    return n;
}

bool flow_encode_maps(FlowOp* ops, uint32_t n_ops, CUtensorMap* d_maps) {
    std::vector<CUtensorMap> host;
    struct Ref { uint32_t op, seg, which; };
    std::vector<Ref> refs;
    for (uint32_t o = 0; o < n_ops; o++) {
        if (ops[o].kind != FLOW_GEMV) continue;
        for (uint32_t i = 0; i < ops[o].nseg; i++) {
            const FlowSeg& G = ops[o].seg[i];
            for (uint32_t which = 0; which < 2; which++) {
                const uint64_t rb = which ? G.row_bytes2 : G.row_bytes;
                if ((which && !flow_glu(G.epi)) || !padded_rows(rb)) continue;
                CUtensorMap m;
                if (!encode_tile_map(&m, which ? G.w2 : G.w, rb, G.rows)) {
                    set_error("flow kernel: no tensor map for a %u-row matrix of %llu-byte rows", G.rows,
                              (unsigned long long)rb);
                    return false;
                }
                host.push_back(m);
                refs.push_back({o, i, which});
            }
        }
    }
    if (!host.empty() &&
        !LM_CUDA(cudaMemcpy(d_maps, host.data(), host.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice)))
        return false;
    for (size_t k = 0; k < refs.size(); k++) {
        FlowSeg& G = ops[refs[k].op].seg[refs[k].seg];
        (refs[k].which ? G.map2 : G.map) = d_maps + k;
    }
    return true;
}

bool flow_init() {
    return LM_CUDA(cudaFuncSetAttribute(flow_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFlowSmem));
}

bool launch_flow(const FlowArgs& a, cudaStream_t st) {
    const size_t smem = (size_t)a.ring_bytes + stage_bytes(a.hd) + 128;
    if (smem > kFlowSmem) { set_error("flow kernel: shared-memory plan does not fit"); return false; }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_cta);
    cfg.blockDim = dim3(kFT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;       // every CTA resident: CTAs wait on each other
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return LM_CUDA(cudaLaunchKernelEx(&cfg, flow_kernel, a));
}

bool launch_flow_embed(const FlowArgs& a, cudaStream_t st) {
    flow_embed_kernel<<<1, 32, 0, st>>>(a);
    return LM_CUDA(cudaGetLastError());
}

}  // namespace lm

#ifdef LLAMINI_FLOW_TIMELINE
// Profiling build only: enable = 1 clears and arms the stamp buffer (148 CTAs x
// 128 ops x 8 points), enable = 0 disarms it and copies it to host_out.
extern "C" int llamini_flow_timeline(int enable, void* host_out) {
    static unsigned long long* d = nullptr;
    const size_t n = 148ull * 128 * 8;
    if (enable) {
        if (!d && cudaMalloc(&d, n * 8) != cudaSuccess) return -1;
        if (cudaMemset(d, 0, n * 8) != cudaSuccess) return -1;
        return cudaMemcpyToSymbol(lm::g_tl, &d, sizeof(d)) == cudaSuccess ? 0 : -1;
    }
    if (!d || cudaDeviceSynchronize() != cudaSuccess) return -1;
    unsigned long long* z = nullptr;
    if (cudaMemcpyToSymbol(lm::g_tl, &z, sizeof(z)) != cudaSuccess) return -1;
    return cudaMemcpy(host_out, d, n * 8, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}
#endif
