// k_ops.cu -- the small kernels of the token loop and of the host-pointer ops.
//
//  * embed:   token (and GPT-2 position) embedding row, decoded from the raw
//             table on the device (tensor.c:24-30, generate.c:83-85,
//             gpt2.c:163-164); also clears the step's argmax key.
//  * finish:  turns the argmax key into the next token, appends it while
//             generating (generate.c:150-153), optionally adds -log p of the
//             teacher-forced next token (generate.c:178-191), advances pos.
//  * per-op:  rms_norm, layer norm, rope, gated activation, bias/vec ops,
//             argmax, matmul and f32 attention used by the model.h/tensor.h/
//             generate.h host-pointer entry points.
#include "internal.h"
#include "quant.cuh"
#include "rows.cuh"
#include "pdl.cuh"

#include <cuda_fp16.h>

namespace lm {

// ------------------------------------------------------------------ dequant

template <uint32_t T>
__global__ void dequant_q_kernel(const uint8_t* __restrict__ raw, uint64_t n_units, float* __restrict__ out) {
    using F = Fmt<T>;
    for (uint64_t u = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; u < n_units;
         u += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t blk = u / F::UPB;
        const uint32_t v = (uint32_t)(u % F::UPB);
        float y[32];
        F::decode(raw + blk * F::BB, v, y);
        float* o = out + blk * F::BE;
#pragma unroll
        for (uint32_t i = 0; i < 32; i++) o[F::elem(v, i)] = y[i];
    }
}

__global__ void dequant_f_kernel(const uint8_t* __restrict__ raw, uint64_t n, uint32_t type, float* __restrict__ out) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        if (type == T_F32) out[i] = reinterpret_cast<const float*>(raw)[i];
        else out[i] = f16_bits(reinterpret_cast<const unsigned short*>(raw)[i]);
    }
}

static uint32_t grid_for(uint64_t n, uint32_t threads) {
    uint64_t g = (n + threads - 1) / threads;
    uint64_t cap = (uint64_t)sm_count() * 16;
    if (g > cap) g = cap;
    return g == 0 ? 1 : (uint32_t)g;
}

bool launch_dequant(uint32_t type, const uint8_t* raw, uint64_t n, float* out, cudaStream_t st) {
    TypeInfo ti;
    if (!type_info(type, &ti) || n % ti.block_elems != 0) { set_error("dequant: bad type %u / count", type); return false; }
    if (n == 0) return true;
    if (reinterpret_cast<uintptr_t>(raw) % type_align(type) != 0) {
        set_error("dequant: blocks of type %u must be %u-byte aligned", type, type_align(type));
        return false;
    }
    if (type == T_F32 || type == T_F16) {
        dequant_f_kernel<<<grid_for(n, 256), 256, 0, st>>>(raw, n, type, out);
        return LM_CUDA(cudaGetLastError());
    }
    const uint64_t units = n / 32;
    const uint32_t g = grid_for(units, 128);
    switch (type) {
    case T_Q4_0: dequant_q_kernel<T_Q4_0><<<g, 128, 0, st>>>(raw, units, out); break;
    case T_Q4_1: dequant_q_kernel<T_Q4_1><<<g, 128, 0, st>>>(raw, units, out); break;
    case T_Q5_0: dequant_q_kernel<T_Q5_0><<<g, 128, 0, st>>>(raw, units, out); break;
    case T_Q8_0: dequant_q_kernel<T_Q8_0><<<g, 128, 0, st>>>(raw, units, out); break;
    case T_Q4_K: dequant_q_kernel<T_Q4_K><<<g, 128, 0, st>>>(raw, units, out); break;
    case T_Q5_K: dequant_q_kernel<T_Q5_K><<<g, 128, 0, st>>>(raw, units, out); break;
    case T_Q6_K: dequant_q_kernel<T_Q6_K><<<g, 128, 0, st>>>(raw, units, out); break;
    default: set_error("dequant: unsupported type %u", type); return false;
    }
    return LM_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------ embed / finish

// Decode row `row` of a table (rows of `cols` elements) into out, scaled.
__device__ void decode_row(const DevMat& m, uint32_t row, float* out, float scale, bool add) {
    decode_row_part(m, row, out, scale, add, threadIdx.x, blockDim.x);
}

__global__ void embed_kernel(const EmbedArgs a) {
    pdl_trigger();
    pdl_wait();
    const uint32_t pos = a.st->pos;
    uint32_t tok = a.tokens[pos];
    if (tok >= a.tok.rows) tok = 0;            // out-of-range ids read row 0
    if (threadIdx.x == 0) a.st->argmax_key = 0ull;
    // gemma multiplies after the lookup (generate.c:84-85); 1.0 is exact
    decode_row(a.tok, tok, a.hidden, a.scale, false);
    if (a.pos.ptr != nullptr) {
        __syncthreads();
        uint32_t p = pos < a.pos.rows ? pos : a.pos.rows - 1;
        decode_row(a.pos, p, a.hidden, 1.0f, true);
    }
}

bool launch_embed(const EmbedArgs& a, cudaStream_t st) {
    return LM_CUDA(launch_k(embed_kernel, dim3(1), dim3(256), 0, st, a));
}

__global__ void finish_kernel(const FinishArgs a) {
    __shared__ float red[32];
    __shared__ float bmax;
    pdl_trigger();
    pdl_wait();
    StepState* s = a.st;
    const uint32_t pos = s->pos;
    if (a.nll && pos + 1 < a.max_tokens) {
        // -log softmax(logits)[target], max-subtracted like generate.c:184-188
        float m = -INFINITY;
        for (uint32_t i = threadIdx.x; i < a.vocab; i += blockDim.x) m = fmaxf(m, a.logits[i]);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = m;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = red[0];
            for (uint32_t i = 1; i < (blockDim.x >> 5); i++) t = fmaxf(t, red[i]);
            bmax = t;
        }
        __syncthreads();
        const float mx = bmax;
        float e = 0.f;
        for (uint32_t i = threadIdx.x; i < a.vocab; i += blockDim.x) e += expf(a.logits[i] - mx);
        for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
        __syncthreads();
        if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = e;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = 0.f;
            for (uint32_t i = 0; i < (blockDim.x >> 5); i++) t += red[i];
            const uint32_t tgt = a.tokens[pos + 1];
            const float lp = (a.logits[tgt < a.vocab ? tgt : 0] - mx) - logf(t);
            s->nll += -(double)lp;
            s->nll_count += 1;
        }
    }
    if (threadIdx.x == 0) {
        const unsigned long long k = s->argmax_key;
        const uint32_t tok = 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
        if (pos + 1 >= s->n_prompt && pos + 1 < a.max_tokens) a.tokens[pos + 1] = k ? tok : 0u;
        s->argmax_key = 0ull;
        s->pos = pos + 1;
    }
}

bool launch_finish(const FinishArgs& a, cudaStream_t st) {
    return LM_CUDA(launch_k(finish_kernel, dim3(1), dim3(1024), 0, st, a));
}

// ------------------------------------------------------------------ host-pointer ops

__device__ float blk_sum(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (uint32_t i = 0; i < (blockDim.x >> 5); i++) t += red[i];
    return t;
}

__global__ void rms_norm_kernel(float* out, const float* x, const float* w, uint32_t dim, float eps) {
    __shared__ float red[32];
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = blk_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)dim + eps);     // model.c:7-8
    for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x) out[i] = x[i] * inv * w[i];
}

__global__ void layer_norm_kernel(float* out, const float* x, const float* w, const float* b, uint32_t dim, float eps) {
    __shared__ float red[32];
    float s = 0.f;
    for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x) s += x[i];
    const float mean = blk_sum(s, red) / (float)dim;
    float v = 0.f;
    for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x) { float c = x[i] - mean; v = fmaf(c, c, v); }
    const float var = blk_sum(v, red) / (float)dim;
    const float inv = 1.0f / sqrtf(var + eps);
    for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x) out[i] = (x[i] - mean) * inv * w[i] + b[i];
}

__global__ void rope_kernel(float* v, uint32_t pos, uint32_t dim, uint32_t hd, float base, uint32_t neox) {
    const uint32_t half = hd / 2;
    for (uint32_t p = blockIdx.x * blockDim.x + threadIdx.x; p < dim / 2; p += gridDim.x * blockDim.x) {
        uint32_t i0, i1, e;
        if (neox) {
            const uint32_t h = p / half, j = p % half;
            i0 = h * hd + j; i1 = i0 + half; e = 2 * j;
            if (i1 >= dim) continue;                 // partial last head: left as is
        } else {
            i0 = 2 * p; i1 = i0 + 1; e = i0 % hd;
        }
        const float th = powf(base, -(float)e / (float)hd);
        const float ang = (float)pos * th;
        const float c = cosf(ang), s = sinf(ang);
        const float a = v[i0], b = v[i1];
        v[i0] = a * c - b * s;
        v[i1] = a * s + b * c;
    }
}

__device__ __forceinline__ float gelu_f(float x) {
    const float k0 = 0.79788456080286535587989211986876f;
    const float k1 = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(k0 * x * (1.0f + k1 * x * x)));
}

__global__ void glu_kernel(float* out, const float* g, const float* u, uint32_t n, uint32_t gelu) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float x = g[i];
        const float a = gelu ? gelu_f(x) : x / (1.0f + expf(-x));
        out[i] = a * u[i];
    }
}

__global__ void gelu_kernel(float* x, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] = gelu_f(x[i]);
}

__global__ void add_kernel(float* out, const float* a, const float* b, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = a[i] + b[i];
}

__global__ void scale_kernel(float* out, const float* a, float s, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = a[i] * s;
}

__global__ void copy_kernel(float* dst, const float* src, uint32_t n) {
    pdl_trigger();
    pdl_wait();
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) dst[i] = src[i];
}

// First strict maximum (generate.c:3-9). The reference starts from x[0] and
// only moves on a strict '>', so NaNs never win, -0 ties +0, and a NaN in x[0]
// makes the answer 0. Each thread keeps its best (value, lowest index) and a
// tree reduction merges them with the same rule.
__global__ void argmax_kernel(const float* x, uint32_t n, uint32_t* out) {
    __shared__ float bv[1024];
    __shared__ uint32_t bi[1024];
    float best = -INFINITY;
    uint32_t idx = 0xFFFFFFFFu;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        if (v > best || (v == best && i < idx)) { best = v; idx = i; }
    }
    bv[threadIdx.x] = best;
    bi[threadIdx.x] = idx;
    __syncthreads();
    for (uint32_t s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float v2 = bv[threadIdx.x + s], v1 = bv[threadIdx.x];
            const uint32_t i2 = bi[threadIdx.x + s], i1 = bi[threadIdx.x];
            if (v2 > v1 || (v2 == v1 && i2 < i1)) { bv[threadIdx.x] = v2; bi[threadIdx.x] = i2; }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const float x0 = x[0];
        *out = (x0 != x0 || bi[0] == 0xFFFFFFFFu) ? 0u : bi[0];
    }
}

// C[m,n] = A[m,k] B[k,n] (tensor.c:32-45); one thread per output.
__global__ void matmul_kernel(const float* A, const float* B, float* C, uint32_t m, uint32_t k, uint32_t n) {
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= m * n) return;
    const uint32_t i = idx / n, j = idx % n;
    float s = 0.f;
    for (uint32_t l = 0; l < k; l++) s = fmaf(A[(uint64_t)i * k + l], B[(uint64_t)l * n + j], s);
    C[idx] = s;
}

// f32 attention over a [pos+1][kv_dim] cache already holding position pos
// (model.c:234-259). Block per query head; three passes like the reference.
__global__ void mha_f32_kernel(const float* q, const float* kc, const float* vc, float* out,
                               uint32_t pos, uint32_t n_heads, uint32_t n_kv, uint32_t hd) {
    extern __shared__ float sc[];
    __shared__ float red[32];
    const uint32_t h = blockIdx.x, g = h / (n_heads / n_kv), kvd = n_kv * hd;
    const float* qh = q + (uint64_t)h * hd;
    const float rs = sqrtf((float)hd);
    for (uint32_t t = threadIdx.x; t <= pos; t += blockDim.x) {
        const float* kt = kc + (uint64_t)t * kvd + (uint64_t)g * hd;
        float s = 0.f;
        for (uint32_t d = 0; d < hd; d++) s = fmaf(qh[d], kt[d], s);
        sc[t] = s / rs;
    }
    __syncthreads();
    float m = -1e30f;
    for (uint32_t t = threadIdx.x; t <= pos; t += blockDim.x) m = fmaxf(m, sc[t]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float mx = red[0];
    for (uint32_t i = 1; i < (blockDim.x >> 5); i++) mx = fmaxf(mx, red[i]);
    __syncthreads();
    float l = 0.f;
    for (uint32_t t = threadIdx.x; t <= pos; t += blockDim.x) { float e = expf(sc[t] - mx); sc[t] = e; l += e; }
    l = blk_sum(l, red);
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.f;
        for (uint32_t t = 0; t <= pos; t++) o = fmaf(sc[t] / l, vc[(uint64_t)t * kvd + (uint64_t)g * hd + d], o);
        out[(uint64_t)h * hd + d] = o;
    }
}

static bool done(void) { return LM_CUDA(cudaGetLastError()); }
static uint32_t g1(uint32_t n) { uint32_t g = (n + 255) / 256; return g == 0 ? 1 : (g > 1024 ? 1024 : g); }

bool launch_rms_norm(float* out, const float* x, const float* w, uint32_t dim, float eps, cudaStream_t st) {
    rms_norm_kernel<<<1, 1024, 0, st>>>(out, x, w, dim, eps); return done();
}
bool launch_layer_norm(float* out, const float* x, const float* w, const float* b, uint32_t dim, float eps, cudaStream_t st) {
    layer_norm_kernel<<<1, 1024, 0, st>>>(out, x, w, b, dim, eps); return done();
}
bool launch_rope(float* v, uint32_t pos, uint32_t dim, uint32_t hd, float base, uint32_t neox, cudaStream_t st) {
    rope_kernel<<<g1(dim / 2), 256, 0, st>>>(v, pos, dim, hd, base, neox); return done();
}
bool launch_glu(float* out, const float* g, const float* u, uint32_t n, uint32_t gelu, cudaStream_t st) {
    glu_kernel<<<g1(n), 256, 0, st>>>(out, g, u, n, gelu); return done();
}
bool launch_gelu_inplace(float* x, uint32_t n, cudaStream_t st) {
    gelu_kernel<<<g1(n), 256, 0, st>>>(x, n); return done();
}
bool launch_add(float* out, const float* a, const float* b, uint32_t n, cudaStream_t st) {
    add_kernel<<<g1(n), 256, 0, st>>>(out, a, b, n); return done();
}
bool launch_scale(float* out, const float* a, float s, uint32_t n, cudaStream_t st) {
    scale_kernel<<<g1(n), 256, 0, st>>>(out, a, s, n); return done();
}
bool launch_copy_f32(float* dst, const float* src, uint32_t n, cudaStream_t st) {
    return LM_CUDA(launch_k(copy_kernel, dim3(g1(n)), dim3(256), 0, st, dst, src, n));
}
bool launch_argmax(const float* x, uint32_t n, uint32_t* out, cudaStream_t st) {
    argmax_kernel<<<1, 1024, 0, st>>>(x, n, out); return done();
}
bool launch_matmul(const float* A, const float* B, float* C, uint32_t m, uint32_t k, uint32_t n, cudaStream_t st) {
    uint32_t t = m * n;
    matmul_kernel<<<(t + 255) / 256 ? (t + 255) / 256 : 1, 256, 0, st>>>(A, B, C, m, k, n); return done();
}
bool launch_mha_f32(const float* q, float* kc, float* vc, float* out, uint32_t pos,
                    uint32_t n_heads, uint32_t n_kv, uint32_t hd, cudaStream_t st) {
    size_t smem = (size_t)(pos + 1) * sizeof(float);
    if (smem > 200 * 1024) { set_error("causal_mha: position %u too large", pos); return false; }
    mha_f32_kernel<<<n_heads, 256, smem, st>>>(q, kc, vc, out, pos, n_heads, n_kv, hd);
    return done();
}

bool gemv_init();
bool gemv_mma_init();
bool attn_init();
bool decode_init();
bool bgemm_init();
bool prefill_init();

// Per-kernel attributes, set once when the device is selected (never during a
// graph capture).
bool kernels_init() {
    // one shared-memory carveout for every kernel of the step, so consecutive
    // kernels never wait for an SM to reconfigure its L1 / shared split
    const int carve = cudaFuncAttributePreferredSharedMemoryCarveout;
    return gemv_init() && gemv_mma_init() && attn_init() && decode_init() && flow_init() && bgemm_init() && tgemm_init() && prefill_init() &&
           LM_CUDA(cudaFuncSetAttribute(embed_kernel, (cudaFuncAttribute)carve, 100)) &&
           LM_CUDA(cudaFuncSetAttribute(finish_kernel, (cudaFuncAttribute)carve, 100)) &&
           LM_CUDA(cudaFuncSetAttribute(copy_kernel, (cudaFuncAttribute)carve, 100)) &&
           LM_CUDA(cudaFuncSetAttribute(mha_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
}

}  // namespace lm
