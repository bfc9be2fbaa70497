// ops.cpp -- host-pointer entry points: the per-op functions of model.h,
// tensor.h and generate.h, the KV-cache handle of kv_cache.h, and the raw-block
// decode / GEMV calls of llamini_b200.h.
//
// These keep the reference's host-pointer contracts, so each call copies its
// operands to the GPU, runs one kernel and copies the result back. They are
// correct but not the fast path; the token loop (session.cpp) keeps everything
// resident on the device.
#include "internal.h"
#include "llamini_b200.h"
#include "generate.h"

#include <cstdlib>
#include <cstring>
#include <vector>
#include <algorithm>

namespace {

// Grow-only device scratch slots for the host-pointer ops.
struct Scratch {
    void* p = nullptr;
    size_t cap = 0;
    void* get(size_t n) {
        if (n <= cap) return p;
        lm::dev_free(p);
        p = lm::dev_alloc(n);
        cap = p ? n : 0;
        return p;
    }
};
Scratch g_s[11];

bool h2d(void* d, const void* h, size_t n) {
    return n == 0 || LM_CUDA(cudaMemcpyAsync(d, h, n, cudaMemcpyHostToDevice, lm::stream()));
}
bool d2h(void* h, const void* d, size_t n) {
    if (n && !LM_CUDA(cudaMemcpyAsync(h, d, n, cudaMemcpyDeviceToHost, lm::stream()))) return false;
    return LM_CUDA(cudaStreamSynchronize(lm::stream()));
}
float* fbuf(int slot, size_t n) { return (float*)g_s[slot].get(n * sizeof(float)); }

// y[b] = W x[b] for b < batch through the batched dequant-GEMM (per-sequence
// staging, split-K partials, finish); scratch in slots 6..9. *handled is false
// when the format or shape has no batched path (the caller loops columns).
// The tcgen05 GEMM (k_tgemm.cu): staging in its layout, the GEMM, the same
// finish; its error word (slot 10) is read back after the call.
bool gemv_batch_tc(uint32_t type, const uint8_t* w, uint32_t rows, uint32_t cols, const float* x, uint32_t batch,
                   float* y, bool* handled) {
    lm::TGemmArgs g;
    g.B = batch;
    g.K = cols;
    g.nseg = 1;
    g.seg[0].w = w;
    g.seg[0].row_bytes = lm::type_bytes(type, cols);
    g.seg[0].type = type;
    g.seg[0].rows = rows;
    if (g.seg[0].row_bytes == 0 || !lm::tgemm_plan(g, (uint32_t)lm::sm_count())) return true;
    *handled = true;
    uint16_t* xh = (uint16_t*)g_s[6].get(lm::tg_xh_halves(cols, g.NP) * 2);
    uint16_t* xl = (uint16_t*)g_s[7].get((size_t)g.NP * cols * 2);
    float* osc = fbuf(8, batch);
    float* part = fbuf(9, (size_t)g.ksplit * batch * rows);
    uint32_t* err = (uint32_t*)g_s[10].get(4);
    if (!xh || !xl || !osc || !part || !err) return false;
    if (!LM_CUDA(cudaMemsetAsync(err, 0, 4, lm::stream()))) return false;
    lm::BStageArgs st;
    st.x = x;
    st.ldx = cols;
    st.K = cols;
    st.B = batch;
    st.xh = xh;
    st.xl = xl;
    st.oscale = osc;
    st.np = g.NP;
    g.xh = xh;
    g.xl = xl;
    g.err = err;
    g.seg[0].part = part;
    lm::BFinishArgs f;
    f.part = part;
    f.ksplit = g.ksplit;
    f.B = batch;
    f.rows = rows;
    f.oscale = osc;
    f.epi = lm::EPI_STORE;
    f.out = y;
    f.ldo = rows;
    if (!lm::launch_bstage(st, lm::stream()) || !lm::launch_tgemm(g, lm::stream()) ||
        !lm::launch_bfinish(f, lm::stream()))
        return false;
    uint32_t e = 0;
    if (!d2h(&e, err, 4)) return false;
    if (e) {
        lm::set_error("tensor-core GEMM: %s", (e & 1u) ? "a pipeline wait ran out" : "a weight outside the fp16 range");
        return false;
    }
    return true;
}

bool gemv_batch(uint32_t type, const uint8_t* w, uint32_t rows, uint32_t cols, const float* x, uint32_t batch,
                float* y, bool* handled) {
    *handled = false;
    if (lm::batch_tc()) return gemv_batch_tc(type, w, rows, cols, x, batch, y, handled);
    lm::BGemmArgs g;
    g.B = batch;
    g.K = cols;
    g.nseg = 1;
    g.seg[0].w = w;
    g.seg[0].row_bytes = lm::type_bytes(type, cols);
    g.seg[0].type = type;
    g.seg[0].rows = rows;
    if (g.seg[0].row_bytes == 0 || !lm::bgemm_plan(g, 2u * (uint32_t)lm::sm_count())) return true;
    *handled = true;
    uint16_t* xh = (uint16_t*)g_s[6].get((size_t)batch * cols * 2);
    uint16_t* xl = (uint16_t*)g_s[7].get((size_t)batch * cols * 2);
    float* sx = fbuf(8, (size_t)batch * (cols / 16) + batch);
    float* part = fbuf(9, (size_t)g.ksplit * batch * rows);
    if (!xh || !xl || !sx || !part) return false;
    lm::BStageArgs st;
    st.x = x;
    st.ldx = cols;
    st.K = cols;
    st.B = batch;
    st.xh = xh;
    st.xl = xl;
    st.sx = sx;
    st.oscale = sx + (size_t)batch * (cols / 16);
    g.xh = xh;
    g.xl = xl;
    g.sx = sx;
    g.seg[0].part = part;
    lm::BFinishArgs f;
    f.part = part;
    f.ksplit = g.ksplit;
    f.B = batch;
    f.rows = rows;
    f.oscale = st.oscale;
    f.epi = lm::EPI_STORE;
    f.out = y;
    f.ldo = rows;
    return lm::launch_bstage(st, lm::stream()) && lm::launch_bgemm(g, lm::stream()) && lm::launch_bfinish(f, lm::stream());
}

bool gemv_any(uint32_t type, const uint8_t* w, uint32_t rows, uint32_t cols, const float* x, uint32_t batch, float* y) {
    if (batch > 1 && batch <= 64 && cols % 32 == 0) {
        bool handled = false;
        const bool ok = gemv_batch(type, w, rows, cols, x, batch, y, &handled);
        if (handled) return ok;
    }
    return lm::launch_gemv_plain(type, w, rows, cols, x, batch, y, lm::stream());
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- raw blocks

int llamini_dequant_device(u32 type, const void* d_blocks, u64 n, f32* d_out) {
    if (!lm::ensure_device()) return -1;
    return lm::launch_dequant(type, (const uint8_t*)d_blocks, n, d_out, lm::stream()) ? 0 : -1;
}

int llamini_dequant_host(u32 type, const void* blocks, u64 n, f32* out) {
    if (!lm::ensure_device()) return -1;
    const uint64_t nb = lm::type_bytes(type, n);
    if (nb == 0 && n != 0) { lm::set_error("dequant: unsupported type %u or count %llu", type, (unsigned long long)n); return -1; }
    if (n == 0) return 0;
    uint8_t* d_raw = (uint8_t*)g_s[0].get(nb + 16);
    float* d_out = fbuf(1, n);
    if (!d_raw || !d_out) return -1;
    if (!h2d(d_raw, blocks, nb)) return -1;
    if (!lm::launch_dequant(type, d_raw, n, d_out, lm::stream())) return -1;
    return d2h(out, d_out, n * sizeof(float)) ? 0 : -1;
}

int llamini_gemv_device(u32 type, const void* d_w, u32 rows, u32 cols, const f32* d_x, u32 batch, f32* d_y) {
    if (!lm::ensure_device()) return -1;
    return gemv_any(type, (const uint8_t*)d_w, rows, cols, d_x, batch, d_y) ? 0 : -1;
}

int llamini_gemv_host(u32 type, const void* w, u32 rows, u32 cols, const f32* x, u32 batch, f32* y) {
    if (!lm::ensure_device()) return -1;
    const uint64_t rb = lm::type_bytes(type, cols);
    if (rb == 0) { lm::set_error("gemv: unsupported type %u or cols %u", type, cols); return -1; }
    uint8_t* dw = (uint8_t*)g_s[0].get(rb * rows + 16);
    float* dx = fbuf(1, (size_t)batch * cols);
    float* dy = fbuf(2, (size_t)batch * rows);
    if (!dw || !dx || !dy) return -1;
    if (!h2d(dw, w, rb * rows) || !h2d(dx, x, (size_t)batch * cols * 4)) return -1;
    if (!gemv_any(type, dw, rows, cols, dx, batch, dy)) return -1;
    return d2h(y, dy, (size_t)batch * rows * 4) ? 0 : -1;
}

// ---------------------------------------------------------------- model.h ops

void rms_norm(f32* out, const f32* x, const f32* w, u32 dim, f32 eps) {
    if (!lm::ensure_device()) return;
    float* dx = fbuf(0, dim); float* dw = fbuf(1, dim); float* dout = fbuf(2, dim);
    if (!dx || !dw || !dout) return;
    if (h2d(dx, x, dim * 4) && h2d(dw, w, dim * 4) && lm::launch_rms_norm(dout, dx, dw, dim, eps, lm::stream()))
        d2h(out, dout, dim * 4);
}

void ffn_glu(f32* out, const f32* gate, const f32* up, u32 dim, FfnAct act) {
    if (!lm::ensure_device()) return;
    float* dg = fbuf(0, dim); float* du = fbuf(1, dim); float* dout = fbuf(2, dim);
    if (!dg || !du || !dout) return;
    if (h2d(dg, gate, dim * 4) && h2d(du, up, dim * 4) &&
        lm::launch_glu(dout, dg, du, dim, act == ACT_GELU, lm::stream()))
        d2h(out, dout, dim * 4);
}

void rope(f32* vec, u32 pos, u32 dim, u32 head_dim, f32 freq_base, RopeType type) {
    if (!lm::ensure_device()) return;
    float* dv = fbuf(0, dim);
    if (!dv) return;
    if (h2d(dv, vec, dim * 4) && lm::launch_rope(dv, pos, dim, head_dim, freq_base, type == ROPE_NEOX, lm::stream()))
        d2h(vec, dv, dim * 4);
}

void add_bias(f32* out, const f32* bias, u32 dim) {
    if (!lm::ensure_device()) return;
    float* da = fbuf(0, dim); float* db = fbuf(1, dim);
    if (!da || !db) return;
    if (h2d(da, out, dim * 4) && h2d(db, bias, dim * 4) && lm::launch_add(da, da, db, dim, lm::stream()))
        d2h(out, da, dim * 4);
}

void linear(f32* out, const f32* x, const Tensor* w, u32 in_dim, u32 out_dim) {
    if (!lm::ensure_device()) return;
    float* dx = fbuf(1, in_dim);
    float* dy = fbuf(2, out_dim);
    if (!dx || !dy || !h2d(dx, x, in_dim * 4)) return;
    if (w->data) {                                    // eager f32 (model.c:181-214)
        float* dw = fbuf(0, (size_t)in_dim * out_dim);
        if (!dw || !h2d(dw, w->data, (size_t)in_dim * out_dim * 4)) return;
        if (!lm::launch_gemv_plain(GGML_TYPE_F32, (const uint8_t*)dw, out_dim, in_dim, dx, 1, dy, lm::stream())) return;
        d2h(out, dy, out_dim * 4);
        return;
    }
    // lazy (model.c:159-176): stream the quantized bytes already in GPU memory
    const lm::DevMat* m = lm::find_gguf_tensor(w->src_info);
    lm::DevMat tmp;
    if (!m || m->cols != in_dim) {
        if (!lm::upload_gguf_tensor(w->src_gf, w->src_info, &tmp, out_dim, in_dim)) {
            memset(out, 0, (size_t)out_dim * sizeof(f32));  // like a failed row decode (model.c:164-172)
            return;
        }
        m = &tmp;
    }
    if (lm::launch_gemv_plain(m->type, m->ptr, out_dim, in_dim, dx, 1, dy, lm::stream()))
        d2h(out, dy, out_dim * 4);
}

void causal_mha(const f32* q, const f32* k, const f32* v, KVCache* cache,
                f32* out, u32 pos, u32 n_heads, u32 n_heads_kv, u32 head_dim) {
    const u32 kvd = n_heads_kv * head_dim;
    // store this position's key/value in the caller's host cache (model.c:222-224)
    memcpy(cache->key + (u64)pos * kvd, k, kvd * sizeof(f32));
    memcpy(cache->val + (u64)pos * kvd, v, kvd * sizeof(f32));
    cache->cur_seq = pos + 1;
    if (!lm::ensure_device()) return;
    const size_t n = (size_t)(pos + 1) * kvd;
    float* dk = fbuf(0, n); float* dv = fbuf(1, n);
    float* dq = fbuf(2, (size_t)n_heads * head_dim); float* dout = fbuf(3, (size_t)n_heads * head_dim);
    if (!dk || !dv || !dq || !dout) return;
    if (h2d(dk, cache->key, n * 4) && h2d(dv, cache->val, n * 4) && h2d(dq, q, (size_t)n_heads * head_dim * 4) &&
        lm::launch_mha_f32(dq, dk, dv, dout, pos, n_heads, n_heads_kv, head_dim, lm::stream()))
        d2h(out, dout, (size_t)n_heads * head_dim * 4);
}

// ---------------------------------------------------------------- tensor.h

Tensor* tensor_create(u32 ndim, u32* shape) {
    Tensor* t = (Tensor*)malloc(sizeof(Tensor));
    if (!t) return nullptr;
    memset(t, 0, sizeof(Tensor));
    t->ndim = ndim;
    t->size = 1;
    for (u32 i = 0; i < ndim && i < 4; i++) { t->dims[i] = shape[i]; t->size *= shape[i]; }
    t->data = (f32*)calloc(t->size, sizeof(f32));
    return t;
}

void tensor_free(Tensor* t) {
    if (!t) return;
    lm::forget_sources(t);
    free(t->data);
    free(t);
}

void matmul(Tensor* A, Tensor* B, Tensor* C) {
    if (!lm::ensure_device()) return;
    const u32 m = A->dims[0], k = A->dims[1], n = B->dims[1];
    float* da = fbuf(0, (size_t)m * k); float* db = fbuf(1, (size_t)k * n); float* dc = fbuf(2, (size_t)m * n);
    if (!da || !db || !dc) return;
    if (h2d(da, A->data, (size_t)m * k * 4) && h2d(db, B->data, (size_t)k * n * 4) &&
        lm::launch_matmul(da, db, dc, m, k, n, lm::stream()))
        d2h(C->data, dc, (size_t)m * n * 4);
}

void vec_add(f32* out, const f32* a, const f32* b, u32 n) {
    if (!lm::ensure_device()) return;
    float* da = fbuf(0, n); float* db = fbuf(1, n);
    if (!da || !db) return;
    if (h2d(da, a, n * 4) && h2d(db, b, n * 4) && lm::launch_add(da, da, db, n, lm::stream())) d2h(out, da, n * 4);
}

void vec_scale(f32* out, const f32* a, f32 s, u32 n) {
    if (!lm::ensure_device()) return;
    float* da = fbuf(0, n);
    if (!da) return;
    if (h2d(da, a, n * 4) && lm::launch_scale(da, da, s, n, lm::stream())) d2h(out, da, n * 4);
}

void tensor_get_row(const Tensor* t, u32 row, u32 row_len, f32* out) {
    if (t->data) {                                   // eager: a copy (tensor.c:25-28)
        memcpy(out, t->data + (u64)row * row_len, row_len * sizeof(f32));
        return;
    }
    // lazy: one-row decode; the result is ignored on failure like tensor.c:29
    gguf_dequantize_rows(t->src_gf, t->src_info, row, row + 1, row_len, out);
}

// ---------------------------------------------------------------- kv_cache.h

void kv_cache_init(KVCache* cache, u32 dim, u32 max_seq) {
    cache->dim = dim;
    cache->max_seq = max_seq;
    cache->cur_seq = 0;
    cache->key = (f32*)calloc((size_t)dim * max_seq, sizeof(f32));
    cache->val = (f32*)calloc((size_t)dim * max_seq, sizeof(f32));
}

void kv_cache_reset(KVCache* cache) {
    cache->cur_seq = 0;
    memset(cache->key, 0, (size_t)cache->dim * cache->max_seq * sizeof(f32));
    memset(cache->val, 0, (size_t)cache->dim * cache->max_seq * sizeof(f32));
}

// ---------------------------------------------------------------- generate.h sampling

u32 greedy_sample(const f32* logits, u32 vocab_size) {
    if (vocab_size == 0) return 0;
    if (!lm::ensure_device()) return 0;
    float* d = fbuf(0, vocab_size);
    uint32_t* r = (uint32_t*)fbuf(1, 1);
    uint32_t res = 0;
    if (d && r && h2d(d, logits, (size_t)vocab_size * 4) && lm::launch_argmax(d, vocab_size, r, lm::stream()))
        d2h(&res, r, 4);
    return res;
}

u32 sample_token(const f32* logits, u32 vocab_size, f32 temp, f32 top_p) {
    if (temp <= 0.0f) return greedy_sample(logits, vocab_size);
    // Temperature softmax + nucleus draw (generate.c:25-60). The draw consumes
    // the C library's rand() exactly like the reference, so it runs on the host.
    struct P { float p; u32 id; };
    std::vector<P> c(vocab_size);
    float mx = logits[0];
    for (u32 i = 1; i < vocab_size; i++) if (logits[i] > mx) mx = logits[i];
    float sum = 0.0f;
    for (u32 i = 0; i < vocab_size; i++) {
        float p = expf((logits[i] - mx) / temp);
        c[i] = {p, i};
        sum += p;
    }
    std::stable_sort(c.begin(), c.end(), [](const P& a, const P& b) { return a.p > b.p; });
    float cum = 0.0f;
    u32 keep = 0;
    while (keep < vocab_size) {
        cum += c[keep].p;
        keep++;
        if (cum >= top_p * sum) break;
    }
    float r = ((float)rand() / ((float)RAND_MAX + 1.0f)) * cum;
    float acc = 0.0f;
    u32 pick = c[0].id;
    for (u32 i = 0; i < keep; i++) {
        acc += c[i].p;
        if (r < acc) { pick = c[i].id; break; }
    }
    return pick;
}

}  // extern "C"
