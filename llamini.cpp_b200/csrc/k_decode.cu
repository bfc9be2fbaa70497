// k_decode.cu -- whole decode steps as one persistent kernel.
//
// The chain of launches of a token step (generate.c:62-120, gpt2.c:150-192)
// pays a launch hand-off per matrix, and at batch 1 each matrix is only a few
// microseconds of HBM traffic. Here one cooperative launch runs one or more
// steps: one CTA per SM, all resident, each working through a fixed list of
// tasks per step, in op order:
//
//   per layer: [norm + QKV tiles] [attention (head, split)] [O tiles + residual]
//              [norm + gate/up tiles + activation] [down tiles + residual]
//   then:      [final norm + lm_head tiles + argmax]  -> finisher
//
// A tile is 16 rows of one matrix (computed exactly like k_gemv_mma.cu). An op
// waits for its predecessor through a completion counter in global memory
// (acquire/release at GPU scope) instead of a kernel boundary, and the CTA's
// producer warp streams the weight tiles of its upcoming tasks into a byte
// ring in shared memory with cp.async.bulk -- weights never depend on the
// activations, so HBM reads run ahead across op and layer boundaries while the
// consumer warps wait for inputs. The CTA that completes the last lm_head tile
// is the step's finisher: it turns the argmax into the next token (generate.c:
// 143-156), advances the position and decodes the next token's embedding row,
// then releases the next step.
//
// Every wait is bounded (a dependency counter, a ring slot, a copy): when one
// runs out the CTA sets an error bit in the step state and a global abort flag
// that ends every other wait early, waits (bounded) for its own copies in
// flight and leaves. Counters only grow, so a step's targets are
// (steps before it + 1) x completions per step; they are zeroed when a session
// is (re)started.
#include "internal.h"
#include "quant.cuh"
#include "rows.cuh"
#include "mma_gemv.cuh"
#include "attn_core.cuh"

#include <cuda_fp16.h>

namespace lm {
namespace {

constexpr int kDWarps = 8;                          // consumer warps
constexpr uint32_t kDCons = kDWarps * 32;           // consumer threads (named barrier 1)
constexpr uint32_t kDThreads = kDCons + 32;         // + the producer warp
constexpr uint32_t kQ = 16;                         // queued weight tiles per CTA (one mbarrier each)
constexpr uint64_t kWaitNs = 2000000000ull;         // longest wait on a counter, ring slot or copy (2 s)
constexpr size_t kDecSmem = 218 * 1024;             // dynamic shared memory per CTA

struct DecShared {
    DecOp op;                // the consumers' current op (copied from global memory)
    uint32_t tasks[kDecMaxTasks];        // this CTA's task list
    uint32_t wait_ctr[kDecMaxOpsSmem];   // per op: counter index it waits on (kDecNoWait: step start)
    uint32_t wait_n[kDecMaxOpsSmem];     // per op: completions per step of that counter
    uint8_t kind[kDecMaxOpsSmem];        // per op: DEC_GEMV or DEC_ATTN
    uint64_t bar[kQ];
    uint64_t vend[kQ];       // producer only: virtual ring end of each queued tile
    uint32_t off[kQ];        // ring offset of each queued tile
    uint32_t consumed;       // tiles released by the consumers (volatile access)
    uint32_t abort;          // this CTA gave up (volatile access)
    uint32_t issued;         // tiles issued by the producer (volatile access)
    uint32_t epoch;          // steps finished before this launch
    uint32_t flag;
    uint32_t next_tok, next_pos;
    float scale;             // 2^(24-E) of the staged input
};

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kDCons) : "memory"); }
// Barrier among the consumer warps that also ORs a predicate across them, so
// every consumer thread takes the same branch after it.
__device__ __forceinline__ bool csync_or(bool v) {
    uint32_t r;
    asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n"
                 " selp.u32 %0, 1, 0, q;\n}\n"
                 : "=r"(r) : "r"((uint32_t)v), "n"(kDCons) : "memory");
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

// A bounded wait ran out: error bit for the host, abort for every CTA.
__device__ void fail(const DecArgs& a, DecShared& S) {
    atomicOr(&a.st->err, kErrWaitTimeout);
    atomicExch(&a.sync->abort, 1u);
    vstore(&S.abort, 1u);
}
__device__ __forceinline__ bool aborted(const DecArgs& a, DecShared& S) {
    return vload(&S.abort) != 0u || vload(&a.sync->abort) != 0u;
}

// Bounded wait until *ctr >= target (wrapping compare); false after an abort
// or once kWaitNs has passed.
__device__ bool dep_wait(const DecArgs& a, DecShared& S, const uint32_t* ctr, uint32_t target) {
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

// Bounded wait on a weight tile's mbarrier that also gives up after an abort.
__device__ bool tile_wait(const DecArgs& a, DecShared& S, uint64_t* bar, uint32_t parity) {
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

// ------------------------------------------------------------------ shared-memory plan

__host__ __device__ __forceinline__ uint32_t xs_floats(uint32_t kmax) { return 2 * kmax + kmax / 16; }
__host__ __device__ __forceinline__ uint32_t attn_floats(uint32_t hd) {
    return (uint32_t)((attn_core_bytes(hd, false) + 3) / 4);      // the f32 cache needs the most
}
__host__ __device__ __forceinline__ uint32_t stage_floats(uint32_t kmax, uint32_t hd) {
    const uint32_t a = xs_floats(kmax), b = attn_floats(hd);
    return ((a > b ? a : b) + 3) & ~3u;
}
constexpr uint32_t kTailFloats = 2 * kDWarps + kDWarps * 16;   // red + part

// Ring bytes of a tile (always sized for 16 rows so reads past a short last
// tile stay inside its own allocation; 16 bytes of slack for the word reads).
__host__ __device__ __forceinline__ uint32_t tile_alloc(const GemvSeg& G) {
    const bool glu = G.epi == EPI_GLU_SILU || G.epi == EPI_GLU_GELU;
    const uint32_t body = glu ? up_offset(G) + tile_bytes(G.row_bytes2) : tile_bytes(G.row_bytes);
    return (body + 16 + 127) & ~127u;
}

// ------------------------------------------------------------------ x staging
// As stage_x in k_gemv_mma.cu (same arithmetic, so the same bits), for the 256
// consumer threads and with L2 loads: the input was written by other CTAs
// during this launch, so L1 may hold stale lines of it.

__device__ void dsum_max(float& s, float& m, float* red, uint32_t tid) {
    s = wsum(s);
    m = wmax(m);
    csync();
    if ((tid & 31u) == 0) { red[tid >> 5] = s; red[kDWarps + (tid >> 5)] = m; }
    csync();
    float ts = 0.f, tm = 0.f;
#pragma unroll
    for (int i = 0; i < kDWarps; i++) { ts += red[i]; tm = fmaxf(tm, red[kDWarps + i]); }
    s = ts;
    m = tm;
}

__device__ void stage_x_dec(const DecArgs& da, const DecOp& op, const MmaSmem& sm, float* s_scale, uint32_t tid) {
    const GemvArgs& a = op.g;
    const uint32_t K = a.K, n4 = K / 4;
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    float4* xf4 = reinterpret_cast<float4*>(sm.xf);
    float s = 0.f, m = 0.f, f = 1.0f;
    if (op.x_merge) {
        // x = the attention output: merge each head's split partials (the same
        // merge as the per-op attention kernel's last CTA)
        const AttnArgs& at = op.at;
        const uint32_t NS = op.n_split, hd = at.hd, stride = attn_part_stride(hd);
        const uint32_t ns = split_range(vload(&da.st->pos), NS, 0).ns;
        for (uint32_t i = tid; i < n4; i += kDCons) {
            const uint32_t h = (4 * i) / hd, d = 4 * i - h * hd;
            const float4 v = merge_head4(at.part + (uint64_t)h * NS * stride, ns, stride, d);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            xf4[i] = v;
        }
        float ds = 0.f;
        dsum_max(ds, m, sm.red, tid);
    } else if (a.norm == NORM_RMS) {
        const float4* w4 = reinterpret_cast<const float4*>(a.norm_w);
#pragma unroll 4
        for (uint32_t i = tid; i < n4; i += kDCons) {
            const float4 v = __ldcg(x4 + i), w = w4[i];
            s = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, s))));
            const float4 o = make_float4(v.x * w.x, v.y * w.y, v.z * w.z, v.w * w.w);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
            xf4[i] = o;
        }
        dsum_max(s, m, sm.red, tid);
        f = 1.0f / sqrtf(s / (float)K + a.eps);    // model.c:7-8; applied to x*w below
    } else if (a.norm == NORM_LAYER) {
#pragma unroll 4
        for (uint32_t i = tid; i < n4; i += kDCons) {
            const float4 v = __ldcg(x4 + i);
            s += (v.x + v.y) + (v.z + v.w);
            xf4[i] = v;
        }
        dsum_max(s, m, sm.red, tid);
        const float mean = s / (float)K;          // two passes like gpt2.c:131-136
        float vs = 0.f;
        for (uint32_t i = tid; i < n4; i += kDCons) {
            const float4 v = xf4[i];
            const float c0 = v.x - mean, c1 = v.y - mean, c2 = v.z - mean, c3 = v.w - mean;
            vs = fmaf(c0, c0, fmaf(c1, c1, fmaf(c2, c2, fmaf(c3, c3, vs))));
        }
        float dummy = 0.f;
        dsum_max(vs, dummy, sm.red, tid);
        const float inv = 1.0f / sqrtf(vs / (float)K + a.eps);
        const float4* w4 = reinterpret_cast<const float4*>(a.norm_w);
        const float4* b4 = reinterpret_cast<const float4*>(a.norm_b);
        m = 0.f;
#pragma unroll 4
        for (uint32_t i = tid; i < n4; i += kDCons) {
            const float4 v = xf4[i], w = w4[i], b = b4[i];
            const float4 o = make_float4((v.x - mean) * inv * w.x + b.x, (v.y - mean) * inv * w.y + b.y,
                                         (v.z - mean) * inv * w.z + b.z, (v.w - mean) * inv * w.w + b.w);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
            xf4[i] = o;
        }
        float ds = 0.f;
        dsum_max(ds, m, sm.red, tid);
    } else {
#pragma unroll 4
        for (uint32_t i = tid; i < n4; i += kDCons) {
            const float4 v = __ldcg(x4 + i);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            xf4[i] = v;
        }
        float ds = 0.f;
        dsum_max(ds, m, sm.red, tid);
    }
    const float mx = m * f;
    int e = 0;
    if (mx > 0.f && mx < INFINITY) frexpf(mx, &e);
    int E = 14 - e;
    E = E > 100 ? 100 : (E < -100 ? -100 : E);
    const float F = f * __int_as_float((E + 127) << 23);
    const uint32_t n4r = (n4 + 31u) & ~31u;
    for (uint32_t i = tid; i < n4r; i += kDCons) {
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
    csync();
}

// ------------------------------------------------------------------ GEMV tile

// One 16-row tile whose weights are at `buf` in the ring; as the tile loop of
// gemv_mma_kernel. Releases the ring space before the epilogue.
__device__ void gemv_tile(const DecArgs& a, const DecOp& op, uint32_t t, const uint8_t* buf, const MmaSmem& sm,
                          DecShared& S, uint32_t tid, uint32_t cseq) {
    const GemvArgs& g = op.g;
    const uint32_t lane = tid & 31u, warp = tid >> 5;
    Lane L;
    L.g = lane >> 2;
    L.tig = lane & 3u;
    L.slot = L.g >> 1;
    L.xpart = (L.g & 1u) ? sm.xl : sm.xh;
    const TileRef tr = tile_of(g, t);
    const GemvSeg& G = g.seg[tr.seg];
    const bool glu = G.epi == EPI_GLU_SILU || G.epi == EPI_GLU_GELU;
    const uint32_t half = kDWarps / 2;
    const bool up = glu && warp >= half;
    const uint8_t* base = up ? buf + up_offset(G) : buf;
    const uint64_t rb = smem_rs(up ? G.row_bytes2 : G.row_bytes);
    const uint32_t first = glu ? warp % half : warp, step = glu ? half : kDWarps;
    // epilogue inputs from global memory, loaded before the MMA loop
    float res = 0.f, bias = 0.f;
    if (tid < 16 && tid < tr.nrows) {
        if (G.epi == EPI_RESID) res = __ldcg(G.out + tr.row0 + tid);
        if (G.bias) bias = G.bias[tr.row0 + tid];
    }
    float acc[2] = {0.f, 0.f};
    switch (G.type) {
    case T_Q4_K: tile_rows<FQ4K>(base, rb, g.K, L, first, step, sm, acc); break;
    case T_Q6_K: tile_rows<FQ6K>(base, rb, g.K, L, first, step, sm, acc); break;
    case T_Q8_0: tile_rows<FQ80>(base, rb, g.K, L, first, step, sm, acc); break;
    default:     tile_rows<FQ40>(base, rb, g.K, L, first, step, sm, acc); break;
    }
#pragma unroll
    for (int r = 0; r < 2; r++) {
        acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 1);
        acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 2);
    }
    if (L.tig == 0) {
        sm.part[warp * 16 + L.g] = acc[0];
        sm.part[warp * 16 + L.g + 8] = acc[1];
    }
    csync();                                   // ring tile consumed, partials ready
    if (tid == 0) vstore(&S.consumed, cseq + 1);
    unsigned long long key = 0ull;
    if (tid < 16) {
        const uint32_t r = tid, row = tr.row0 + r;
        float v = 0.f, u = 0.f;
#pragma unroll
        for (uint32_t w = 0; w < (uint32_t)kDWarps; w++) {
            if (glu && w >= half) u += sm.part[w * 16 + r];
            else v += sm.part[w * 16 + r];
        }
        v *= S.scale;
        u *= S.scale;
        if (r < tr.nrows) {
            switch (G.epi) {
            case EPI_STORE: if (G.bias) v += bias; G.out[row] = v; break;
            case EPI_RESID: {
                if (G.bias) v += bias;
                const float o = res + v;
                G.out[row] = o;
                if (a.trace != nullptr && op.trace_off != 0xFFFFFFFFu) a.trace[op.trace_off + row] = o;
                break;
            }
            case EPI_GLU_SILU: v = v / (1.0f + expf(-v)) * u; G.out[row] = v; break;   // model.c:22
            case EPI_GLU_GELU: v = m_gelu(v) * u; G.out[row] = v; break;
            case EPI_GELU: if (G.bias) v += bias; v = m_gelu(v); G.out[row] = v; break;
            }
            if (G.argmax) key = m_key(v, row);
        }
    }
    if (g.argmax_key != nullptr && warp == 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
            key = k2 > key ? k2 : key;
        }
        if (lane == 0 && key != 0ull) atomicMax(g.argmax_key, key);
    }
    csync();                                   // part[] free, outputs written
}

// ------------------------------------------------------------------ attention

struct AttnTask {
    uint32_t h, g, split;
    SplitRange r;
    uint32_t pos;
};
__device__ __forceinline__ AttnTask attn_task_of(const DecArgs& a, const DecOp& op, uint32_t task) {
    const AttnArgs& at = op.at;
    AttnTask t;
    t.h = task / op.n_split;
    t.split = task - t.h * op.n_split;
    t.g = t.h / (at.n_heads / at.n_kv);
    t.pos = vload(&a.st->pos);
    t.r = split_range(t.pos, op.n_split, t.split);
    return t;
}

// Issue the cached K/V rows of the task's first chunk. They were written in
// earlier steps, so this may run before the QKV op of this step is complete.
template <typename KV>
__device__ void attn_prefetch(const DecArgs& a, const DecOp& op, uint32_t task, float* stage, uint32_t tid) {
    const AttnArgs& at = op.at;
    const AttnTask t = attn_task_of(a, op, task);
    if (t.split >= t.r.ns) return;
    const uint32_t hd = at.hd;
    const AttnSm sm = attn_carve(stage, hd, sizeof(KV) == 2);
    const KV* kc = reinterpret_cast<const KV*>(at.kc) + (uint64_t)t.g * at.max_seq * hd;
    const KV* vc = reinterpret_cast<const KV*>(at.vc) + (uint64_t)t.g * at.max_seq * hd;
    const uint32_t n = min(kAttnChunk, t.r.t1 - t.r.t0);
    const uint32_t nold = (t.r.t0 + n > t.pos) ? t.pos - t.r.t0 : n;
    attn_stage_async<KV>(sm, kc, vc, t.r.t0, nold, hd, tid, kDCons);
}

// Task (head h, split) of causal_mha (model.c:217-260) at the current
// position; writes the split's partial (m, l, o). The O projection merges.
template <typename KV>
__device__ void attn_task(const DecArgs& a, const DecOp& op, uint32_t task, float* stage, bool staged, uint32_t tid) {
    const AttnArgs& at = op.at;
    const AttnTask t = attn_task_of(a, op, task);
    if (t.split >= t.r.ns) return;
    const uint32_t hd = at.hd, G = at.n_heads / at.n_kv;
    const AttnSm sm = attn_carve(stage, hd, sizeof(KV) == 2);
    const bool has_new = t.r.t0 <= t.pos && t.pos < t.r.t1;
    for (uint32_t i = tid; i < hd; i += kDCons) {
        sm.qs[i] = __ldcg(at.qkv + (uint64_t)t.h * hd + i);
        if (has_new) {
            sm.kn[i] = __ldcg(at.qkv + (uint64_t)at.n_heads * hd + (uint64_t)t.g * hd + i);
            sm.vn[i] = __ldcg(at.qkv + (uint64_t)(at.n_heads + at.n_kv) * hd + (uint64_t)t.g * hd + i);
        }
    }
    csync();
    rope_pairs(sm.qs, hd, t.pos, at.rope, at.theta, tid, kDCons);
    if (has_new) rope_pairs(sm.kn, hd, t.pos, at.rope, at.theta, tid, kDCons);
    csync();
    KV* kc = reinterpret_cast<KV*>(at.kc) + (uint64_t)t.g * at.max_seq * hd;
    KV* vc = reinterpret_cast<KV*>(at.vc) + (uint64_t)t.g * at.max_seq * hd;
    if (has_new && t.h == t.g * G) {              // one writer per kv head
        for (uint32_t i = tid; i < hd; i += kDCons) {
            kv_put(kc + (uint64_t)t.pos * hd + i, sm.kn[i]);
            kv_put(vc + (uint64_t)t.pos * hd + i, sm.vn[i]);
        }
    }
    const float o = attn_chunks<KV>(sm, kc, vc, t.pos, t.r.t0, t.r.t1, hd, tid, kDCons, staged, [] { csync(); });
    const uint32_t stride = attn_part_stride(hd);
    float* dst = at.part + ((uint64_t)t.h * op.n_split + t.split) * stride;
    if (tid < hd) dst[4 + tid] = o;
    if (tid == 0) { dst[0] = sm.sc[kAttnChunk + 4]; dst[1] = sm.sc[kAttnChunk + 5]; }
}

// ------------------------------------------------------------------ finisher

// After the last lm_head tile of a step: next token from the argmax
// (finish_kernel), next position, the next input's embedding row (embed_kernel),
// then release the next step.
__device__ void finish_step(const DecArgs& a, DecShared& S, uint32_t tid) {
    if (tid == 0) {
        __threadfence();
        StepState* st = a.st;
        const unsigned long long k = atomicAdd(&st->argmax_key, 0ull);
        const uint32_t pos = vload(&st->pos);
        const uint32_t np = vload(&st->n_prompt);
        if (pos + 1 >= np && pos + 1 < a.max_tokens)
            a.tokens[pos + 1] = k ? 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull) : 0u;
        atomicExch(&st->argmax_key, 0ull);
        vstore(&st->pos, pos + 1);
        uint32_t nt = pos + 1 < a.max_tokens ? vload(&a.tokens[pos + 1]) : 0u;
        if (nt >= a.tok.rows) nt = 0;                  // out-of-range ids read row 0
        S.next_tok = nt;
        S.next_pos = pos + 1;
    }
    csync();
    decode_row_part(a.tok, S.next_tok, a.hidden, a.emb_scale, false, tid, kDCons);
    if (a.pos.ptr != nullptr) {
        csync();
        const uint32_t p = S.next_pos < a.pos.rows ? S.next_pos : a.pos.rows - 1;
        decode_row_part(a.pos, p, a.hidden, 1.0f, true, tid, kDCons);
    }
    csync();
    if (tid == 0) {
        __threadfence();
        atomicAdd(&a.sync->step_done, 1u);
    }
}

// ------------------------------------------------------------------ roles

__device__ void producer(const DecArgs& a, DecShared& S, uint8_t* ring) {
    const uint32_t* my = S.tasks;
    const uint32_t n_my = a.sched_len[blockIdx.x];
    const uint64_t R = a.ring_bytes;
    uint64_t head = 0;
    uint32_t seq = 0;
    for (uint32_t j = 0; j < a.n_steps; j++) {
        for (uint32_t i = 0; i < n_my; i++) {
            const uint32_t ent = my[i];
            const DecOp& op = a.ops[ent >> 16];
            if (op.kind != DEC_GEMV) continue;
            const TileRef tr = tile_of(op.g, ent & 0xFFFFu);
            const GemvSeg& G = op.g.seg[tr.seg];
            const bool glu = G.epi == EPI_GLU_SILU || G.epi == EPI_GLU_GELU;
            const uint32_t n1 = rows_tx(G.row_bytes, tr.nrows);
            const uint32_t n2 = glu ? rows_tx(G.row_bytes2, tr.nrows) : 0u;
            const uint32_t alloc = tile_alloc(G);
            uint64_t off = head % R;
            if (off + alloc > R) { head += R - off; off = 0; }
            bool ok = false;
            const uint64_t t0 = gtime();
            for (uint32_t w = 0;; w++) {
                const uint32_t c = vload(&S.consumed);
                const uint64_t tail = c == 0 ? 0ull : S.vend[(c - 1) % kQ];
                if (seq - c < kQ && head + alloc - tail <= R) { ok = true; break; }
                if ((w & 63u) == 63u && (aborted(a, S) || gtime() - t0 > kWaitNs)) break;
            }
            if (!ok) {
                if (!aborted(a, S)) fail(a, S);
                vstore(&S.abort, 1u);
                return;
            }
            const uint32_t q = seq % kQ;
            S.off[q] = (uint32_t)off;
            S.vend[q] = head + alloc;
            // the consumers' reads of this ring space happened before they
            // released it; order them before the async-proxy writes
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            mbar_expect_tx(&S.bar[q], n1 + n2);
            copy_rows(ring + off, G.w + (uint64_t)tr.row0 * G.row_bytes, G.row_bytes, tr.nrows, &S.bar[q]);
            if (glu) copy_rows(ring + off + up_offset(G), G.w2 + (uint64_t)tr.row0 * G.row_bytes2, G.row_bytes2, tr.nrows,
                               &S.bar[q]);
            head += alloc;
            seq++;
            vstore(&S.issued, seq);
        }
    }
}

// Publish n more completions of op_i (release: this CTA's outputs first).
__device__ __forceinline__ void signal(uint32_t* ctr, uint32_t n) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" :: "l"(ctr), "r"(n) : "memory");
}

__device__ void consumer(const DecArgs& a, DecShared& S, uint8_t* ring, const MmaSmem& sm, float* stage,
                         uint32_t tid) {
    const uint32_t* my = S.tasks;
    const uint32_t n_my = a.sched_len[blockIdx.x];
    const DecOp& op = S.op;
    uint32_t cseq = 0;
    for (uint32_t j = 0; j < a.n_steps; j++) {
        const uint32_t E = S.epoch + j;
        uint32_t staged = 0xFFFFFFFFu, run_op = 0xFFFFFFFFu, run_n = 0;
        for (uint32_t i = 0; i < n_my; i++) {
            const uint32_t ent = my[i], op_i = ent >> 16, task = ent & 0xFFFFu;
            bool prefetched = false;
            if (op_i != run_op) {              // first task of this op here: wait for its input
                // the op's descriptor into shared memory (read-only, so this
                // runs while the input may still be on its way)
                {
                    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.ops + op_i);
                    uint32_t* dst = reinterpret_cast<uint32_t*>(&S.op);
                    csync();                   // every thread is done with the previous op
                    // warps 1..7 copy; warp 0 goes straight on to poll the input
                    for (uint32_t w = tid - 32; tid >= 32 && w < (uint32_t)(sizeof(DecOp) / 4); w += kDCons - 32)
                        dst[w] = __ldg(src + w);
                }
                if (S.kind[op_i] == DEC_ATTN) {
                    // the cached K/V rows do not depend on this op's input, only on
                    // the step having started (its position, the earlier steps' rows)
                    bool ok = true;
                    if (run_op == 0xFFFFFFFFu && tid == 0) ok = dep_wait(a, S, &a.sync->step_done, E);
                    if (csync_or(!ok)) return;     // also publishes the descriptor copy
                    if (op.at.kv_f16) attn_prefetch<__half>(a, op, task, stage, tid);
                    else attn_prefetch<float>(a, op, task, stage, tid);
                    prefetched = true;
                    staged = 0xFFFFFFFFu;
                }
                bool ok = true;
                if (tid == 0) {
                    const uint32_t w = S.wait_ctr[op_i];
                    if (w == kDecNoWait) ok = dep_wait(a, S, &a.sync->step_done, E);
                    else ok = dep_wait(a, S, &a.done[w], (E + 1) * S.wait_n[op_i]);
                }
                if (csync_or(!ok)) return;
                run_op = op_i;
                run_n = 0;
            }
            if (S.kind[op_i] == DEC_GEMV) {
                if (staged != op_i) {
                    stage_x_dec(a, op, sm, &S.scale, tid);
                    staged = op_i;
                }
                const uint32_t q = cseq % kQ;
                const bool ok = tile_wait(a, S, &S.bar[q], (cseq / kQ) & 1u);
                if (csync_or(!ok)) return;
                gemv_tile(a, op, task, ring + S.off[q], sm, S, tid, cseq);
                cseq++;
            } else {
                staged = 0xFFFFFFFFu;          // attention reuses the staging area
                if (op.at.kv_f16) attn_task<__half>(a, op, task, stage, prefetched, tid);
                else attn_task<float>(a, op, task, stage, prefetched, tid);
            }
            run_n++;
            const bool last = i + 1 == n_my || (my[i + 1] >> 16) != op_i;
            if (last) {                        // publish this CTA's tasks of the op at once
                if (op_i + 1 < a.n_ops) {
                    csync();                   // every thread's outputs are written
                    if (tid == 0) signal(&a.done[op_i], run_n);
                } else {                       // lm_head: the CTA that completes it finishes the step
                    csync();
                    if (tid == 0) {
                        __threadfence();
                        const uint32_t old = atomicAdd(&a.done[op_i], run_n);
                        S.flag = old + run_n == (E + 1) * op.ndone ? 1u : 0u;
                    }
                    csync();
                    if (S.flag) finish_step(a, S, tid);
                }
            }
        }
    }
}

__global__ void __launch_bounds__(kDThreads, 1) decode_kernel(const __grid_constant__ DecArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ DecShared S;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    uint8_t* ring = smem;
    float* stage = reinterpret_cast<float*>(smem + a.ring_bytes);
    MmaSmem sm;
    sm.xf = stage;
    sm.xh = reinterpret_cast<uint32_t*>(stage + a.kmax);
    sm.xl = sm.xh + a.kmax / 2;
    sm.sx = reinterpret_cast<float*>(sm.xl + a.kmax / 2);
    sm.red = stage + stage_floats(a.kmax, a.hd);
    sm.part = sm.red + 2 * kDWarps;
    if (tid == 0) {
        for (uint32_t q = 0; q < kQ; q++) mbar_init(&S.bar[q], 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        S.consumed = 0;
        S.issued = 0;
        S.flag = 0;
        S.abort = vload(&a.sync->abort);
        S.epoch = ld_acq(&a.sync->epoch);
    }
    {
        const uint32_t* my = a.sched + (uint64_t)blockIdx.x * a.sched_stride;
        const uint32_t n_my = a.sched_len[blockIdx.x];
        for (uint32_t i = tid; i < n_my; i += kDThreads) S.tasks[i] = my[i];
        for (uint32_t o = tid; o < a.n_ops; o += kDThreads) {
            const uint32_t w = a.ops[o].wait;
            S.wait_ctr[o] = w;
            S.wait_n[o] = w == kDecNoWait ? 0u : a.ops[w].ndone;
            S.kind[o] = (uint8_t)a.ops[o].kind;
        }
    }
    __syncthreads();
    if (warp == (uint32_t)kDWarps) {
        if (lane == 0) producer(a, S, ring);
        __syncwarp();
    } else {
        consumer(a, S, ring, sm, stage, tid);
    }
    __syncthreads();
    if (tid == 0) {
        // copies issued but never consumed (only after an abort): wait for them
        const uint32_t c = vload(&S.consumed), n = vload(&S.issued);
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

}  // namespace

bool decode_supported_type(uint32_t t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0 || t == T_Q4_0; }

uint32_t decode_ring_bytes(uint32_t kmax, uint32_t hd) {
    const size_t other = ((size_t)stage_floats(kmax, hd) + kTailFloats) * sizeof(float);
    if (other + 4096 > kDecSmem) return 0;
    return (uint32_t)((kDecSmem - other) & ~size_t(127));
}

size_t decode_smem(uint32_t ring, uint32_t kmax, uint32_t hd) {
    const size_t n = ring + ((size_t)stage_floats(kmax, hd) + kTailFloats) * sizeof(float);
    return n <= kDecSmem ? n : 0;
}

uint32_t decode_tile_alloc(const GemvSeg& G) { return tile_alloc(G); }
uint32_t decode_threads() { return kDThreads; }

bool decode_init() {
    return LM_CUDA(cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecSmem));
}

bool launch_decode(const DecArgs& a, cudaStream_t st) {
    const size_t smem = decode_smem(a.ring_bytes, a.kmax, a.hd);
    if (smem == 0) { set_error("decode kernel: shared-memory plan does not fit"); return false; }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_cta);
    cfg.blockDim = dim3(kDThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;       // every CTA resident: CTAs wait on each other
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return LM_CUDA(cudaLaunchKernelEx(&cfg, decode_kernel, a));
}

}  // namespace lm
