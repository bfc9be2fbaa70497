// k_gemv.cu -- fused dequant-GEMV kernels (the decode hot loop).
//
// Replaces llamini.cpp's linear() on lazy weights (model.c:145-176: decode 256
// rows into an f32 scratch, then model.c:66-73's dot per row) with one pass
// that streams each weight byte from HBM exactly once and decodes it in
// registers. A launch computes several groups of rows ("segments") that share
// one input vector, with the vector's normalisation (RMSNorm / LayerNorm,
// model.c:4-10 / gpt2.c:130-139) as a prologue and bias, residual add, gated
// activation (model.c:20-25) or GELU (gpt2.c:182) and the greedy argmax
// (generate.c:3-9) as epilogues.
//
// Work split: the input vector is staged (normalised) in shared memory by every
// CTA. A warp owns a tile of R rows; its lanes stride over the 32-element units
// of the row (quant.cuh), so each lane loads its x values once and reuses them
// for the R rows. Lane partial sums are combined with warp shuffles.
#include "internal.h"
#include "quant.cuh"
#include "pdl.cuh"

#include <cuda_fp16.h>
#include <cstdlib>

namespace lm {

constexpr int kRows = 2;          // rows per warp tile
constexpr int kWarps = 8;         // warps per CTA
constexpr int kThreads = kWarps * 32;

// ------------------------------------------------------------------ row dots

template <uint32_t T>
__device__ __forceinline__ void dot_rows_q(const uint8_t* w, uint64_t rb, int nr,
                                           const float* __restrict__ xs, uint32_t K,
                                           float* acc, uint32_t lane) {
    using F = Fmt<T>;
    const uint32_t units = K / F::BE * F::UPB;
    for (uint32_t u = lane; u < units; u += 32) {
        const uint32_t blk = u / F::UPB, v = u % F::UPB;
        float xv[32];
        const float* xb = xs + blk * F::BE;
#pragma unroll
        for (uint32_t i = 0; i < 32; i++) xv[i] = xb[F::elem(v, i)];
#pragma unroll
        for (int r = 0; r < kRows; r++) {
            if (r < nr) {
                float wv[32];
                F::decode(w + (uint64_t)r * rb + (uint64_t)blk * F::BB, v, wv);
                float s = 0.f;
#pragma unroll
                for (uint32_t i = 0; i < 32; i++) s = fmaf(wv[i], xv[i], s);
                acc[r] += s;
            }
        }
    }
}

// F32 / F16 rows (eager host tensors and GPT-2 style F16 matrices): units of 32
// consecutive elements, the last one possibly partial.
template <uint32_t T>
__device__ __forceinline__ void dot_rows_f(const uint8_t* w, uint64_t rb, int nr,
                                           const float* __restrict__ xs, uint32_t K,
                                           float* acc, uint32_t lane) {
    for (uint32_t k = lane; k < K; k += 32) {
        float xv = xs[k];
#pragma unroll
        for (int r = 0; r < kRows; r++) {
            if (r < nr) {
                const uint8_t* row = w + (uint64_t)r * rb;
                float wv;
                if (T == T_F32) wv = __ldg(reinterpret_cast<const float*>(row) + k);
                else wv = f16_bits(__ldg(reinterpret_cast<const unsigned short*>(row) + k));
                acc[r] = fmaf(wv, xv, acc[r]);
            }
        }
    }
}

__device__ __forceinline__ bool dot_rows(uint32_t type, const uint8_t* w, uint64_t rb, int nr,
                                         const float* xs, uint32_t K, float* acc, uint32_t lane) {
    switch (type) {
    case T_Q4_K: dot_rows_q<T_Q4_K>(w, rb, nr, xs, K, acc, lane); return true;
    case T_Q6_K: dot_rows_q<T_Q6_K>(w, rb, nr, xs, K, acc, lane); return true;
    case T_Q5_K: dot_rows_q<T_Q5_K>(w, rb, nr, xs, K, acc, lane); return true;
    case T_Q4_0: dot_rows_q<T_Q4_0>(w, rb, nr, xs, K, acc, lane); return true;
    case T_Q4_1: dot_rows_q<T_Q4_1>(w, rb, nr, xs, K, acc, lane); return true;
    case T_Q5_0: dot_rows_q<T_Q5_0>(w, rb, nr, xs, K, acc, lane); return true;
    case T_Q8_0: dot_rows_q<T_Q8_0>(w, rb, nr, xs, K, acc, lane); return true;
    case T_F32:  dot_rows_f<T_F32>(w, rb, nr, xs, K, acc, lane); return true;
    case T_F16:  dot_rows_f<T_F16>(w, rb, nr, xs, K, acc, lane); return true;
    default: return false;
    }
}

// ------------------------------------------------------------------ helpers

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// tanh-approximated GELU (model.c:14-18, gpt2.c:144-148)
__device__ __forceinline__ float gelu_tanh(float x) {
    const float k0 = 0.79788456080286535587989211986876f;
    const float k1 = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(k0 * x * (1.0f + k1 * x * x)));
}
__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// Orderable key for the greedy argmax: larger value wins, and for equal values
// the smaller index wins (first strict maximum, generate.c:3-9). NaN never
// wins; a NaN in row 0 makes row 0 the answer, as the reference's comparisons
// against a NaN start value all fail.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    if (v != v) return idx == 0 ? ~0ull : 0ull;
    if (v == 0.0f) v = 0.0f;                      // -0 and +0 compare equal
    uint32_t b = __float_as_uint(v);
    uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

// Block-wide sum of one value per thread (blockDim.x a multiple of 32).
__device__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const uint32_t w = threadIdx.x >> 5, l = threadIdx.x & 31u;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    const uint32_t nw = blockDim.x >> 5;
    for (uint32_t i = 0; i < nw; i++) t += red[i];
    return t;
}

// ------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kThreads)
gemv_fused_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ float xs[];                 // K floats, then reduction scratch
    float* red = xs + ((a.K + 3u) & ~3u);
    const uint32_t K = a.K;
    pdl_trigger();
    pdl_wait();                                   // x comes from the previous kernel

    // Prologue: stage (and normalise) the input vector.
    if (a.norm == NORM_NONE) {
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) xs[i] = a.x[i];
    } else if (a.norm == NORM_RMS) {
        float ss = 0.f;
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) {
            float v = a.x[i];
            xs[i] = v;
            ss = fmaf(v, v, ss);
        }
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / (float)K + a.eps);
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) xs[i] = xs[i] * inv * a.norm_w[i];
    } else {
        float s = 0.f;
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) {
            float v = a.x[i];
            xs[i] = v;
            s += v;
        }
        const float mean = block_sum(s, red) / (float)K;
        float vs = 0.f;
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) {
            float c = xs[i] - mean;
            vs = fmaf(c, c, vs);
        }
        const float var = block_sum(vs, red) / (float)K;
        const float inv = 1.0f / sqrtf(var + a.eps);
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x)
            xs[i] = (xs[i] - mean) * inv * a.norm_w[i] + a.norm_b[i];
    }
    __syncthreads();
    if (a.x_out != nullptr && blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) a.x_out[i] = xs[i];

    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const GemvSeg& last = a.seg[a.nseg - 1];
    const uint32_t n_tiles = last.tile0 + (last.rows + kRows - 1) / kRows;
    unsigned long long best = 0ull;

    for (uint32_t t = blockIdx.x * kWarps + warp; t < n_tiles; t += gridDim.x * kWarps) {
        uint32_t s = 0;
#pragma unroll
        for (uint32_t i = 1; i < kMaxSegs; i++)
            if (i < a.nseg && t >= a.seg[i].tile0) s = i;
        const GemvSeg& g = a.seg[s];
        const uint32_t row0 = (t - g.tile0) * kRows;
        const int nr = (int)min((uint32_t)kRows, g.rows - row0);

        float acc[kRows], acc2[kRows];
#pragma unroll
        for (int r = 0; r < kRows; r++) { acc[r] = 0.f; acc2[r] = 0.f; }
        dot_rows(g.type, g.w + (uint64_t)row0 * g.row_bytes, g.row_bytes, nr, xs, K, acc, lane);
        const bool glu = g.epi == EPI_GLU_SILU || g.epi == EPI_GLU_GELU;
        if (glu) dot_rows(g.type2, g.w2 + (uint64_t)row0 * g.row_bytes2, g.row_bytes2, nr, xs, K, acc2, lane);
#pragma unroll
        for (int r = 0; r < kRows; r++) {
            acc[r] = warp_sum(acc[r]);
            if (glu) acc2[r] = warp_sum(acc2[r]);
        }
        // Lane r finishes row row0 + r.
#pragma unroll
        for (int r = 0; r < kRows; r++) {
            if ((int)lane == r && r < nr) {
                const uint32_t row = row0 + r;
                float v = acc[r];
                switch (g.epi) {
                case EPI_STORE:
                    if (g.bias) v += g.bias[row];
                    g.out[row] = v;
                    break;
                case EPI_RESID:
                    if (g.bias) v += g.bias[row];
                    g.out[row] += v;
                    break;
                case EPI_GLU_SILU:
                    v = silu(v) * acc2[r];
                    g.out[row] = v;
                    break;
                case EPI_GLU_GELU:
                    v = gelu_tanh(v) * acc2[r];
                    g.out[row] = v;
                    break;
                case EPI_GELU:
                    if (g.bias) v += g.bias[row];
                    v = gelu_tanh(v);
                    g.out[row] = v;
                    break;
                }
                if (g.argmax) {
                    unsigned long long k = argmax_key(v, row);
                    best = k > best ? k : best;
                }
            }
        }
    }

    if (a.argmax_key != nullptr) {
        // warp max, then one atomic per warp
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0 && best != 0ull) atomicMax(a.argmax_key, best);
    }
}

static size_t gemv_smem(uint32_t K) { return (((size_t)K + 3) & ~size_t(3)) * sizeof(float) + 64 * sizeof(float); }

bool gemv_init() {
    return LM_CUDA(cudaFuncSetAttribute(gemv_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)) &&
           LM_CUDA(cudaFuncSetAttribute(gemv_fused_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
}

bool launch_gemv(const GemvArgs& in, cudaStream_t st) {
    GemvArgs a = in;
    if (a.nseg == 0 || a.nseg > (uint32_t)kMaxSegs) { set_error("gemv: bad segment count %u", a.nseg); return false; }
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < a.nseg; i++) {
        const GemvSeg& g = a.seg[i];
        const bool glu = g.epi == EPI_GLU_SILU || g.epi == EPI_GLU_GELU;
        if (reinterpret_cast<uintptr_t>(g.w) % type_align(g.type) != 0 || g.row_bytes % type_align(g.type) != 0 ||
            (glu && (reinterpret_cast<uintptr_t>(g.w2) % type_align(g.type2) != 0 ||
                     g.row_bytes2 % type_align(g.type2) != 0))) {
            set_error("gemv: weights of type %u must be %u-byte aligned", g.type, type_align(g.type));
            return false;
        }
        a.seg[i].tile0 = tiles;
        tiles += (a.seg[i].rows + kRows - 1) / kRows;
    }
    static const bool cuda_cores_only = getenv("LLAMINI_GEMV_CUDA_CORES") != nullptr;
    if (!cuda_cores_only) {
        bool handled = false;
        if (!launch_gemv_mma(in, st, &handled)) return false;
        if (handled) return true;
    }
    if (in.tp.push != kTpNone || in.tp.pull != kTpNone) {
        set_error("gemv: the fused tensor-parallel reduction runs on the tensor-core GEMV only");
        return false;
    }
    size_t smem = gemv_smem(a.K);
    if (smem > 200 * 1024) { set_error("gemv: K=%u too large", a.K); return false; }
    uint32_t want = (tiles + kWarps - 1) / kWarps;
    uint32_t cap = (uint32_t)sm_count() * 4;
    uint32_t grid = want < cap ? want : cap;
    if (grid == 0) grid = 1;
    return LM_CUDA(launch_k(gemv_fused_kernel, dim3(grid), dim3(kThreads), smem, st, a));
}

// Multi-column plain GEMV: one fused launch per column (correct, not tuned for
// batch > 1; the batched path is a separate kernel family).
bool launch_gemv_plain(uint32_t type, const uint8_t* w, uint32_t rows, uint32_t cols,
                       const float* x, uint32_t batch, float* y, cudaStream_t st) {
    uint64_t rb = type_bytes(type, cols);
    if (rb == 0) { set_error("gemv: unsupported type %u or cols %u", type, cols); return false; }
    for (uint32_t b = 0; b < batch; b++) {
        GemvArgs a;
        a.x = x + (uint64_t)b * cols;
        a.K = cols;
        a.nseg = 1;
        a.seg[0].w = w;
        a.seg[0].row_bytes = rb;
        a.seg[0].type = type;
        a.seg[0].rows = rows;
        a.seg[0].epi = EPI_STORE;
        a.seg[0].out = y + (uint64_t)b * rows;
        if (!launch_gemv(a, st)) return false;
    }
    return true;
}

}  // namespace lm
