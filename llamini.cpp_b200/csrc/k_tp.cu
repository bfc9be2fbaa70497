// k_tp.cu -- tensor parallelism across the GPUs of one box: the allreduce after
// the o projection and after ffn_down (one process per GPU; LLaMA models with
// heads and FFN columns split over the ranks).
//
// Every rank exports one device buffer (cudaIpcGetMemHandle) and maps every
// peer's (cudaIpcOpenMemHandle), so all ranks' buffers are plain pointers over
// NVLink. Buffer layout: two slots of kTpSlotFloats floats (used by alternate
// allreduces), then kTpMaxRanks flags (u32), flag j written by rank j.
//
// Allreduce number n (every rank counts its own in device memory):
//   1. copy this rank's partial sums into its own slot n % 2;
//   2. fence (system scope), then store n into flag `rank` of every peer's
//      buffer with release semantics;
//   3. wait until every peer's flag in this rank's buffer reaches n (acquire,
//      bounded: an error bit and an early exit after kTpWaitNs);
//   4. out[i] += sum over ranks 0..world-1 of slot n % 2 [i], in rank order, so
//      every rank gets bit-identical results.
// A rank reuses slot n % 2 at allreduce n + 2 only after allreduce n + 1, which
// needs every peer's flag n + 1 -- set after that peer finished reading slot
// n % 2 -- so no copy overwrites data a peer still reads.
//
// The wide allreduce (a batch's or a prefill chunk's columns, up to
// kTpWideFloats floats) has slots, flags and counters of its own after these,
// and runs the same protocol per slice of kTpWideSlice floats: CTA c copies,
// flags, waits for and adds slice c only, so slices need no grid-wide barrier.
// The next allreduce's kernel starts after this one has finished on this rank
// (programmatic launch waits for it), so a peer's flag n + 1 for slice c again
// means that peer has read every rank's slice c of allreduce n.
#include "internal.h"
#include "pdl.cuh"

namespace lm {

constexpr uint64_t kTpWaitNs = 2000000000ull;   // 2 s

struct TpArgs {
    const float* part;                // this rank's partial sums
    float* out;                       // out[i] += the sum over ranks
    uint32_t n, rank, world;
    float* buf[kTpMaxRanks];          // every rank's buffer (this rank's included)
    uint32_t* gen;                    // allreduces this rank has finished
    uint32_t* err;
};

__device__ __forceinline__ uint32_t* tp_flags(float* buf) { return reinterpret_cast<uint32_t*>(buf + 2 * kTpSlotFloats); }
// wide slots: after the flags (16-byte aligned), then the wide flags [rank][slice]
__host__ __device__ __forceinline__ float* tp_wide(float* buf) { return buf + 2 * kTpSlotFloats + kTpMaxRanks; }
__device__ __forceinline__ uint32_t* tp_wflags(float* buf) {
    return reinterpret_cast<uint32_t*>(tp_wide(buf) + 2 * kTpWideFloats);
}
// fused slots [2][kTpMaxRanks][kTpFusedFloats] after the wide flags, then the
// arrival counters [2][kTpMaxRanks]
__host__ __device__ __forceinline__ float* tp_fslots(float* buf) {
    return tp_wide(buf) + 2 * kTpWideFloats + kTpMaxRanks * kTpWideCtas;
}
__host__ __device__ __forceinline__ uint32_t* tp_farrive(float* buf) {
    return reinterpret_cast<uint32_t*>(tp_fslots(buf) + 2 * kTpMaxRanks * kTpFusedFloats);
}
__device__ __forceinline__ uint64_t tp_time() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float ld_relaxed_sys(const float* p) {
    float v;
    asm volatile("ld.relaxed.sys.global.f32 %0, [%1];\n" : "=f"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(1024) tp_allreduce_kernel(const TpArgs a) {
    __shared__ uint32_t s_n, s_fail;
    pdl_trigger();
    pdl_wait();                                       // the partial sums come from the previous kernel
    const uint32_t tid = threadIdx.x;
    if (tid == 0) {
        s_n = *reinterpret_cast<volatile uint32_t*>(a.gen) + 1u;
        s_fail = 0;
    }
    __syncthreads();
    const uint32_t n = s_n;
    const uint32_t par = n & 1u;
    float* mine = a.buf[a.rank] + par * kTpSlotFloats;
    for (uint32_t i = tid; i < a.n; i += blockDim.x) mine[i] = a.part[i];
    __threadfence_system();                           // this thread's slot writes before any flag
    __syncthreads();
    if (tid < a.world && tid != a.rank) {
        st_release_sys(tp_flags(a.buf[tid]) + a.rank, n);
        const uint32_t* f = tp_flags(a.buf[a.rank]) + tid;
        const uint64_t t0 = tp_time();
        // a wait of this session that already ran out: the group is broken, fail at once
        if (*reinterpret_cast<volatile uint32_t*>(a.err) & kErrWaitTimeout) s_fail = 1;
        for (uint32_t i = 0; !s_fail; i++) {
            if ((int32_t)(ld_acquire_sys(f) - n) >= 0) break;
            if ((i & 63u) == 63u && tp_time() - t0 > kTpWaitNs) {
                atomicOr(a.err, kErrWaitTimeout);
                s_fail = 1;
                break;
            }
        }
    }
    __syncthreads();
    if (s_fail) return;
    for (uint32_t i = tid; i < a.n; i += blockDim.x) {
        float s = 0.f;
        for (uint32_t j = 0; j < a.world; j++)
            s += j == a.rank ? mine[i] : ld_relaxed_sys(a.buf[j] + par * kTpSlotFloats + i);
        a.out[i] += s;
    }
    __syncthreads();
    if (tid == 0) *reinterpret_cast<volatile uint32_t*>(a.gen) = n;
}

// grid ceil(n / kTpWideSlice), 256 threads: CTA c takes floats [c S, c S + S).
__global__ void __launch_bounds__(256) tp_allreduce_wide_kernel(const TpArgs a) {
    __shared__ uint32_t s_n, s_fail;
    pdl_trigger();
    pdl_wait();                                       // the partial sums come from the previous kernel
    const uint32_t tid = threadIdx.x, c = blockIdx.x;
    const uint32_t i0 = c * kTpWideSlice, i1 = min(a.n, i0 + kTpWideSlice);
    if (tid == 0) {
        s_n = *reinterpret_cast<volatile uint32_t*>(a.gen + c) + 1u;
        s_fail = 0;
    }
    __syncthreads();
    const uint32_t n = s_n, par = n & 1u;
    float* mine = tp_wide(a.buf[a.rank]) + par * kTpWideFloats;
    for (uint32_t i = i0 + tid; i < i1; i += blockDim.x) mine[i] = a.part[i];
    __threadfence_system();                           // this thread's slot writes before any flag
    __syncthreads();
    if (tid < a.world && tid != a.rank) {
        st_release_sys(tp_wflags(a.buf[tid]) + a.rank * kTpWideCtas + c, n);
        const uint32_t* f = tp_wflags(a.buf[a.rank]) + tid * kTpWideCtas + c;
        const uint64_t t0 = tp_time();
        if (*reinterpret_cast<volatile uint32_t*>(a.err) & kErrWaitTimeout) s_fail = 1;
        for (uint32_t i = 0; !s_fail; i++) {
            if ((int32_t)(ld_acquire_sys(f) - n) >= 0) break;
            if ((i & 63u) == 63u && tp_time() - t0 > kTpWaitNs) {
                atomicOr(a.err, kErrWaitTimeout);
                s_fail = 1;
                break;
            }
        }
    }
    __syncthreads();
    if (s_fail) return;
    // L2 loads (peer slots over NVLink), every rank's value in flight at once
    for (uint32_t i = i0 + tid; i < i1; i += blockDim.x) {
        float v[kTpMaxRanks];
#pragma unroll
        for (uint32_t j = 0; j < kTpMaxRanks; j++)
            v[j] = j < a.world ? __ldcg(tp_wide(a.buf[j]) + par * kTpWideFloats + i) : 0.f;
        float s = 0.f;
#pragma unroll
        for (uint32_t j = 0; j < kTpMaxRanks; j++)
            if (j < a.world) s += v[j];
        a.out[i] += s;
    }
    __syncthreads();
    if (tid == 0) *reinterpret_cast<volatile uint32_t*>(a.gen + c) = n;
}

// ---------------------------------------------------------------- host side

namespace {
TpState g_tp;
}

TpState& tp() { return g_tp; }

size_t tp_buffer_bytes() {
    return (2 * kTpSlotFloats + kTpMaxRanks + 2 * kTpWideFloats) * sizeof(float) +
           (size_t)kTpMaxRanks * kTpWideCtas * sizeof(uint32_t) +
           (size_t)2 * kTpMaxRanks * kTpFusedFloats * sizeof(float) + 2 * kTpMaxRanks * sizeof(uint32_t);
}

// device counters after the buffer's: gen (1), wide gen (kTpWideCtas), fused
// gen (2), fused tickets (2)
constexpr uint32_t kTpCounterWords = 1 + kTpWideCtas + 4;

GemvTp tp_fused_args(uint32_t push, uint32_t pull) {
    GemvTp t;
    for (uint32_t j = 0; j < g_tp.world && j < kTpMaxRanks; j++) {
        t.slots[j] = tp_fslots(g_tp.peer[j]);
        t.arrive[j] = tp_farrive(g_tp.peer[j]);
    }
    t.gen = g_tp.gen + 1 + kTpWideCtas;
    t.ticket = t.gen + 2;
    t.rank = g_tp.rank;
    t.world = g_tp.world;
    t.push = push;
    t.pull = pull;
    return t;
}

bool tp_alloc_buffer() {
    if (g_tp.local) return true;
    void* p = nullptr;
    // cudaMalloc directly: the buffer is exported by IPC handle
    if (!LM_CUDA(cudaMalloc(&p, tp_buffer_bytes()))) return false;
    if (!LM_CUDA(cudaMemset(p, 0, tp_buffer_bytes()))) { cudaFree(p); return false; }
    uint32_t* gen = nullptr;
    if (!LM_CUDA(cudaMalloc((void**)&gen, 4 * kTpCounterWords)) || !LM_CUDA(cudaMemset(gen, 0, 4 * kTpCounterWords))) {
        cudaFree(p);
        return false;
    }
    g_tp.local = (float*)p;
    g_tp.gen = gen;
    g_tp.wgen = gen + 1;
    return true;
}

bool launch_tp_allreduce(const float* part, float* out, uint32_t n, uint32_t* err, cudaStream_t st) {
    if (g_tp.world < 2) { set_error("allreduce without a tensor-parallel group"); return false; }
    if (n > kTpSlotFloats) { set_error("allreduce of %u floats (at most %u)", n, kTpSlotFloats); return false; }
    TpArgs a;
    a.part = part;
    a.out = out;
    a.n = n;
    a.rank = g_tp.rank;
    a.world = g_tp.world;
    for (uint32_t j = 0; j < kTpMaxRanks; j++) a.buf[j] = j < g_tp.world ? g_tp.peer[j] : nullptr;
    a.gen = g_tp.gen;
    a.err = err;
    return LM_CUDA(launch_k(tp_allreduce_kernel, dim3(1), dim3(1024), 0, st, a));
}

bool launch_tp_allreduce_wide(const float* part, float* out, uint32_t n, uint32_t* err, cudaStream_t st) {
    if (g_tp.world < 2) { set_error("allreduce without a tensor-parallel group"); return false; }
    if (n == 0 || n > kTpWideFloats) { set_error("wide allreduce of %u floats (1..%u)", n, kTpWideFloats); return false; }
    TpArgs a;
    a.part = part;
    a.out = out;
    a.n = n;
    a.rank = g_tp.rank;
    a.world = g_tp.world;
    for (uint32_t j = 0; j < kTpMaxRanks; j++) a.buf[j] = j < g_tp.world ? g_tp.peer[j] : nullptr;
    a.gen = g_tp.wgen;
    a.err = err;
    return LM_CUDA(launch_k(tp_allreduce_wide_kernel, dim3((n + kTpWideSlice - 1) / kTpWideSlice), dim3(256), 0, st, a));
}

}  // namespace lm
