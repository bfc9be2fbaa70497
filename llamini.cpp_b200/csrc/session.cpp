// session.cpp -- the device-resident token loop.
//
// A session binds one model to one array of per-layer KV caches. It owns the
// fp16 device cache, the activation buffers, a token buffer and a StepState
// block in GPU memory, and two CUDA graphs: one step and a run of kStepsPerGraph
// steps. A step (generate.c:62-120 for LLaMA, gpt2.c:150-192 for GPT-2) is
//
//   embed -> per layer: [norm+QKV GEMV] -> attention -> [O GEMV + residual]
//                       -> [norm+gate/up GEMV + activation] -> [down GEMV + residual]
//         -> [norm + lm_head GEMV + argmax] -> finish
//
// and reads its position and input token from device memory, so consecutive
// steps need no host involvement: the argmax of step p becomes the input of
// step p+1 on the device (generate.c:143-156 without the round trip).
#include "internal.h"
#include "llamini_b200.h"
#include "generate.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cmath>
#include <ctime>
#include <unordered_map>
#include <vector>

// Buffers and weight copies of chunked prefill (session.cpp, prefill section).
struct Prefill {
    float *hidden = nullptr, *qkv = nullptr, *attn = nullptr, *ffn_h = nullptr, *osc = nullptr;
    float* tp_part = nullptr;            // tensor parallel: the chunk's o / down partial sums
    float *part = nullptr, *part2 = nullptr, *part3 = nullptr;
    // teacher-forced scoring (built on first use): lm_head partials, the
    // chunk's logits [C][vocab], and per position the next token's log-prob
    float *hpart = nullptr, *logits = nullptr, *lp = nullptr;
    int head_state = 0;                  // 0 not built, 1 ready, -1 not available
    uint16_t *xh = nullptr, *xl = nullptr;
    uint32_t* err = nullptr;
    std::unordered_map<const uint8_t*, std::pair<const uint8_t*, uint64_t>> pitched;
};

struct llamini_session {
    int kind = 0;                         // 0 LLaMA family, 1 GPT-2
    const void* model = nullptr;
    KVCache* caches = nullptr;
    u32 cache_max_seq = 0, cache_dim = 0;
    const GGUFFile* gf = nullptr;         // file whose device tensors we use (may be null)

    // shape
    u32 n_layers = 0, dim = 0, n_heads = 0, n_kv = 0, hd = 0, ffn = 0, vocab = 0, max_seq = 0;
    u32 qd = 0, kvd = 0, n_split = 1, max_pos = 0;
    f32 eps = 0, rope_base = 0, emb_scale = 1;
    const float* theta = nullptr;        // RoPE frequencies (device, hd/2)
    u32 rope_mode = 0;                    // 0 none, 1 NORM, 2 NEOX
    u32 act_gelu = 0;
    u32 kv_f16 = 0;                       // cache element type (f32 unless asked)

    // weights (device)
    struct Layer {
        lm::DevMat q, k, v, o, gate, up, down;    // LLaMA (for GPT-2: q = fused qkv, o = out)
        const float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr;
        const float *bq = nullptr, *bk = nullptr, *bv = nullptr, *bo = nullptr, *bup = nullptr, *bdown = nullptr;
    };
    std::vector<Layer> layers;
    lm::DevMat tok, pos_tab, head;
    const float *fnw = nullptr, *fnb = nullptr;
    u64 weight_bytes = 0;

    // buffers (device)
    std::vector<void*> owned;
    float *hidden = nullptr, *qkv = nullptr, *attn = nullptr, *ffn_h = nullptr, *logits = nullptr;
    float* probs = nullptr;               // the device sampler's scratch (vocab floats)
    float *part = nullptr, *trace = nullptr;
    float* tp_part = nullptr;           // tensor parallel: this rank's o / down partial sums
    u32 tp_world = 1;                   // ranks the weights are split over
    int tp_fuse = 0;                    // 0 not decided, 1 reductions fused into the GEMVs, -1 separate
    bool tp_fuse_now = false;           // the step being enqueued uses the fused reductions
    struct Prefill* pf = nullptr;       // prompt chunks on the tensor-core GEMM (built on first use)
    int pf_state = 0;                   // 0 not tried, 1 built, -1 not available for this model
    u32 *counters = nullptr, *tokens = nullptr;
    void *kc = nullptr, *vc = nullptr;
    lm::StepState* st = nullptr;
    lm::StepState* st_host = nullptr;     // pinned staging for StepState writes/reads

    // graphs
    cudaGraphExec_t g_one = nullptr, g_many = nullptr, g_trace = nullptr, g_nll = nullptr;
    bool trace_on = false;

    // persistent decode kernel (k_decode.cu): op table, schedule and counters
    bool dec_on = false;
    lm::DecArgs dec;
    u32* dec_counters = nullptr;          // DecSync | done[n_ops] | tickets[n_layers][n_heads]
    size_t dec_counter_bytes = 0;

    // dataflow decode kernel (k_flow.cu): op table, schedule, counters, records
    bool flow_on = false;
    lm::FlowArgs flow;
    u32* flow_counters = nullptr;         // DecSync | done[n_ops]
    size_t flow_counter_bytes = 0;

    // host mirror of the device position / prompt length
    u32 pos = 0, n_prompt = 0;
};

namespace lm {
namespace {

constexpr u32 kStepsPerGraph = 8;
constexpr u32 kDecStepsPerLaunch = 64;    // decode-kernel steps per launch
std::vector<llamini_session*> g_sessions;

void* own(llamini_session* s, size_t bytes) {
    void* p = dev_alloc(bytes);
    if (p) s->owned.push_back(p);
    return p;
}

// Device copy of an f32 host vector (norm weights, biases).
const float* upload_f32(llamini_session* s, const f32* h, size_t n) {
    float* d = (float*)own(s, n * sizeof(float));
    if (!d) return nullptr;
    if (!LM_CUDA(cudaMemcpy(d, h, n * sizeof(float), cudaMemcpyHostToDevice))) return nullptr;
    return d;
}

// Device matrix for a weight tensor of shape rows x cols: the uploaded GGUF
// bytes when the tensor is lazy or was loaded from a GGUF file, otherwise its
// eager f32 host data.
bool weight(llamini_session* s, const Tensor* t, u32 rows, u32 cols, DevMat* out) {
    if (!t) { set_error("missing weight tensor"); return false; }
    if ((u64)t->size != (u64)rows * cols) { set_error("weight shape mismatch: %u elements, expected %ux%u", t->size, rows, cols); return false; }
    GGUFFile* gf = nullptr;
    const GGUFTensorInfo* info = nullptr;
    if (!t->data) { gf = t->src_gf; info = t->src_info; }
    else source_of(t, &gf, &info);
    if (info) {
        const DevMat* m = find_gguf_tensor(info);
        if (m && m->rows == rows && m->cols == cols) { *out = *m; }
        else if (!upload_gguf_tensor(gf, info, out, rows, cols)) return false;
        s->gf = gf;
        s->weight_bytes += out->row_bytes * rows;
        return true;
    }
    const float* d = upload_f32(s, t->data, (size_t)rows * cols);
    if (!d) return false;
    out->ptr = (const uint8_t*)d;
    out->type = GGML_TYPE_F32;
    out->rows = rows;
    out->cols = cols;
    out->row_bytes = (u64)cols * 4;
    s->weight_bytes += out->row_bytes * rows;
    return true;
}

void shard_rows(llamini_session* s, DevMat* m, u32 r0, u32 n);
bool shard_cols(llamini_session* s, DevMat* m, u32 c0, u32 c1);

// Tensor parallelism: rows [r0, r0 + nr) and columns [c0, c1) (on block
// boundaries) of a rows x cols weight, copied from the mapped GGUF file
// straight into a matrix of the session's own, so a rank uploads only its
// shard (gguf.c's mapping, model.c's tensor table). Eager f32 tensors take the
// whole-matrix path and are cut on the device.
bool weight_shard(llamini_session* s, const Tensor* t, u32 rows, u32 cols, u32 r0, u32 nr, u32 c0, u32 c1,
                  DevMat* out) {
    if (!t) { set_error("missing weight tensor"); return false; }
    if ((u64)t->size != (u64)rows * cols) { set_error("weight shape mismatch: %u elements, expected %ux%u", t->size, rows, cols); return false; }
    GGUFFile* gf = nullptr;
    const GGUFTensorInfo* info = nullptr;
    if (!t->data) { gf = t->src_gf; info = t->src_info; }
    else source_of(t, &gf, &info);
    if (!info) {
        if (!weight(s, t, rows, cols, out)) return false;
        if (nr != rows) shard_rows(s, out, r0, nr);
        return (c0 == 0 && c1 == cols) || shard_cols(s, out, c0, c1);
    }
    const uint32_t ty = info->ggml_type;
    const uint64_t rb = type_bytes(ty, cols), b0 = type_bytes(ty, c0), w = type_bytes(ty, c1 - c0);
    if (rb == 0 || w == 0 || (c0 && b0 == 0) || r0 + nr > rows || c1 > cols) {
        set_error("tensor parallel: rows %u+%u, columns %u..%u of tensor %s are not on block boundaries", r0, nr, c0, c1,
                  info->name);
        return false;
    }
    const uint64_t abs_off = gf->tensor_offset + info->offset;
    if (abs_off < info->offset || abs_off > gf->size || rb * rows > gf->size - abs_off) {
        set_error("tensor %s runs past the end of the file", info->name);
        return false;
    }
    uint8_t* d = (uint8_t*)own(s, w * nr + 16);       // 16 bytes of slack for word reads
    const uint8_t* src = (const uint8_t*)gf->data + abs_off + (uint64_t)r0 * rb + b0;
    if (!d || !LM_CUDA(cudaMemcpy2D(d, w, src, rb, w, nr, cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemset(d + w * nr, 0, 16)))
        return false;
    out->ptr = d;
    out->type = ty;
    out->rows = nr;
    out->cols = c1 - c0;
    out->row_bytes = w;
    s->gf = gf;
    s->weight_bytes += w * nr;
    return true;
}

const float* vec(llamini_session* s, const Tensor* t, u32 n) {
    if (!t || !t->data || t->size < n) { set_error("missing or short f32 tensor"); return nullptr; }
    s->weight_bytes += (u64)n * 4;
    return upload_f32(s, t->data, n);
}

// The shard of rank R of W: heads [R H/W, (R+1) H/W) and the matching kv heads
// (so the o-proj columns are the rank's heads), FFN columns [f0, f1) on
// 256-column super-block boundaries, split as evenly as the super-blocks allow
// (f0 = 256 floor(nsb R / W)). out = {head0, head1, kv0, kv1, f0, f1, ocol0,
// ocol1}; -1 with an error when the shapes do not split.
int tp_plan(u32 W, u32 R, u32 n_heads, u32 n_kv, u32 hd, u32 ffn, u32* out) {
    if (W == 0 || R >= W || n_heads == 0 || n_kv == 0 || n_heads % W != 0 || n_kv % W != 0 || ffn % 256 != 0 ||
        ffn / 256 < W) {
        set_error("tensor parallel over %u ranks: heads %u, kv heads %u, ffn %u do not split", W, n_heads, n_kv, ffn);
        return -1;
    }
    const u32 hw = n_heads / W, kw = n_kv / W, nsb = ffn / 256;
    out[0] = R * hw;
    out[1] = (R + 1) * hw;
    out[2] = R * kw;
    out[3] = (R + 1) * kw;
    out[4] = 256 * (u32)((uint64_t)nsb * R / W);
    out[5] = 256 * (u32)((uint64_t)nsb * (R + 1) / W);
    out[6] = R * hw * hd;
    out[7] = (R + 1) * hw * hd;
    return 0;
}

// Tensor parallelism: keep rows [r0, r0 + n) of m (a view, no copy).
void shard_rows(llamini_session* s, DevMat* m, u32 r0, u32 n) {
    s->weight_bytes -= m->row_bytes * (m->rows - n);
    m->ptr += (uint64_t)r0 * m->row_bytes;
    m->rows = n;
}
// Tensor parallelism: columns [c0, c1) of every row, copied into a matrix of
// their own (c0, c1 on block boundaries of m's format).
bool shard_cols(llamini_session* s, DevMat* m, u32 c0, u32 c1) {
    const uint64_t b0 = type_bytes(m->type, c0), w = type_bytes(m->type, c1 - c0);
    if ((c0 && b0 == 0) || w == 0) {
        set_error("tensor parallel: columns %u..%u of a type-%u matrix are not on block boundaries", c0, c1, m->type);
        return false;
    }
    uint8_t* d = (uint8_t*)own(s, w * m->rows + 16);
    if (!d || !LM_CUDA(cudaMemcpy2D(d, w, m->ptr + b0, m->row_bytes, w, m->rows, cudaMemcpyDeviceToDevice)) ||
        !LM_CUDA(cudaMemset(d + w * m->rows, 0, 16)))
        return false;
    s->weight_bytes -= (m->row_bytes - w) * m->rows;
    m->ptr = d;
    m->cols = c1 - c0;
    m->row_bytes = w;
    return true;
}

bool alloc_buffers(llamini_session* s) {
    const u32 L = s->n_layers;
    s->hidden = (float*)own(s, (size_t)s->dim * 4);
    s->qkv = (float*)own(s, (size_t)(s->qd + 2 * s->kvd) * 4);
    s->attn = (float*)own(s, (size_t)s->qd * 4);
    s->ffn_h = (float*)own(s, (size_t)s->ffn * 4);
    s->logits = (float*)own(s, (size_t)s->vocab * 4);
    s->probs = (float*)own(s, (size_t)s->vocab * 4);
    s->part = (float*)own(s, (size_t)s->n_heads * s->n_split * (s->hd + 4) * 4);
    s->trace = (float*)own(s, (size_t)L * s->dim * 4);
    s->counters = (u32*)own(s, (size_t)s->n_heads * 4);
    s->tokens = (u32*)own(s, ((size_t)s->max_seq + 1) * 4);
    const size_t kv_bytes = (size_t)L * s->n_kv * s->max_seq * s->hd * (s->kv_f16 ? 2 : 4);
    s->kc = own(s, kv_bytes);
    s->vc = own(s, kv_bytes);
    s->st = (StepState*)own(s, sizeof(StepState));
    if (s->tp_world > 1 && !(s->tp_part = (float*)own(s, (size_t)s->dim * 4))) return false;
    if (!s->hidden || !s->qkv || !s->attn || !s->ffn_h || !s->logits || !s->probs || !s->part || !s->trace ||
        !s->counters || !s->tokens || !s->kc || !s->vc || !s->st)
        return false;
    if (!LM_CUDA(cudaMallocHost((void**)&s->st_host, sizeof(StepState)))) return false;
    memset(s->st_host, 0, sizeof(StepState));
    return LM_CUDA(cudaMemset(s->counters, 0, (size_t)s->n_heads * 4)) &&
           LM_CUDA(cudaMemset(s->st, 0, sizeof(StepState))) &&
           LM_CUDA(cudaMemset(s->tokens, 0, ((size_t)s->max_seq + 1) * 4)) &&
           LM_CUDA(cudaMemset(s->kc, 0, kv_bytes)) && LM_CUDA(cudaMemset(s->vc, 0, kv_bytes));
}

// Position splits per query head of the per-op attention: about two (head,
// split) CTAs per SM (at the 7B shape, context ~1000: 3.27 ms/step against 3.39
// with one per SM and 3.52 with four); each split takes >= 64 positions, so short
// contexts use fewer. The dataflow kernel runs at most one task per CTA
// (flow_splits).
u32 choose_splits(u32 n_heads, u32 max_seq) {
    const u32 sms = (u32)sm_count();
    u32 s = n_heads ? 2 * sms / n_heads : 1;
    if (s < 1) s = 1;
    if (s > 32) s = 32;
    const u32 by_len = (max_seq + 63) / 64;
    if (s > by_len) s = by_len;
    return s ? s : 1;
}

// ---------------------------------------------------------------- the step

// ---- the arguments of each op of a step (shared by the per-op launches and
//      the persistent decode kernel)

EmbedArgs embed_args(llamini_session* s) {
    EmbedArgs e;
    e.st = s->st;
    e.tokens = s->tokens;
    e.tok = s->tok;
    e.pos = s->pos_tab;
    e.scale = s->emb_scale;
    e.hidden = s->hidden;
    e.dim = s->dim;
    return e;
}

// norm + QKV (LLaMA: three matrices; GPT-2: the fused qkv matrix)
GemvArgs qkv_args(llamini_session* s, u32 l) {
    const llamini_session::Layer& W = s->layers[l];
    const bool gpt2 = s->kind == 1;
    GemvArgs a;
    a.err = &s->st->err;
    a.x = s->hidden;
    a.K = s->dim;
    a.norm = gpt2 ? NORM_LAYER : NORM_RMS;
    a.norm_w = W.n1w;
    a.norm_b = W.n1b;
    a.eps = s->eps;
    if (gpt2) {
        a.nseg = 1;
        a.seg[0] = {W.q.ptr, nullptr, W.q.row_bytes, 0, W.q.type, 0, W.q.rows, EPI_STORE, s->qkv, W.bq, 0, 0};
    } else {
        a.nseg = 3;
        a.seg[0] = {W.q.ptr, nullptr, W.q.row_bytes, 0, W.q.type, 0, W.q.rows, EPI_STORE, s->qkv, W.bq, 0, 0};
        a.seg[1] = {W.k.ptr, nullptr, W.k.row_bytes, 0, W.k.type, 0, W.k.rows, EPI_STORE, s->qkv + s->qd, W.bk, 0, 0};
        a.seg[2] = {W.v.ptr, nullptr, W.v.row_bytes, 0, W.v.type, 0, W.v.rows, EPI_STORE, s->qkv + s->qd + s->kvd, W.bv, 0, 0};
    }
    if (s->tp_fuse_now && l > 0) a.tp = tp_fused_args(kTpNone, 1);   // the previous layer's down sums
    return a;
}

AttnArgs attn_args(llamini_session* s, u32 l) {
    AttnArgs at;
    at.st = s->st;
    at.qkv = s->qkv;
    const size_t per_layer = (size_t)s->n_kv * s->max_seq * s->hd * (s->kv_f16 ? 2 : 4);
    at.kc = (uint8_t*)s->kc + l * per_layer;
    at.vc = (uint8_t*)s->vc + l * per_layer;
    at.kv_f16 = s->kv_f16;
    at.out = s->attn;
    at.part = s->part;
    at.counter = s->counters;
    at.n_heads = s->n_heads;
    at.n_kv = s->n_kv;
    at.hd = s->hd;
    at.max_seq = s->max_seq;
    at.n_split = s->n_split;
    at.rope = s->rope_mode;
    at.theta = s->theta;
    return at;
}

// O projection + residual
GemvArgs o_args(llamini_session* s, u32 l) {
    const llamini_session::Layer& W = s->layers[l];
    GemvArgs o;
    o.err = &s->st->err;
    o.x = s->attn;
    o.K = s->qd;
    o.nseg = 1;
    o.seg[0] = {W.o.ptr, nullptr, W.o.row_bytes, 0, W.o.type, 0, W.o.rows, EPI_RESID, s->hidden, W.bo, 0, 0};
    if (s->tp_world > 1) {                            // partial sums; the allreduce adds them to hidden
        o.seg[0].epi = EPI_STORE;
        o.seg[0].out = s->tp_part;
        if (tp().rank != 0) o.seg[0].bias = nullptr;  // the bias enters the sum once
        if (s->tp_fuse_now) o.tp = tp_fused_args(0, kTpNone);
    }
    return o;
}

// norm + FFN up (gated for LLaMA, GELU for GPT-2)
GemvArgs ffn_args(llamini_session* s, u32 l) {
    const llamini_session::Layer& W = s->layers[l];
    const bool gpt2 = s->kind == 1;
    GemvArgs f;
    f.err = &s->st->err;
    f.x = s->hidden;
    f.K = s->dim;
    f.norm = gpt2 ? NORM_LAYER : NORM_RMS;
    f.norm_w = W.n2w;
    f.norm_b = W.n2b;
    f.eps = s->eps;
    f.nseg = 1;
    if (gpt2)
        f.seg[0] = {W.up.ptr, nullptr, W.up.row_bytes, 0, W.up.type, 0, W.up.rows, EPI_GELU, s->ffn_h, W.bup, 0, 0};
    else
        f.seg[0] = {W.gate.ptr, W.up.ptr, W.gate.row_bytes, W.up.row_bytes, W.gate.type, W.up.type, W.gate.rows,
                    s->act_gelu ? (u32)EPI_GLU_GELU : (u32)EPI_GLU_SILU, s->ffn_h, nullptr, 0, 0};
    if (s->tp_fuse_now) f.tp = tp_fused_args(kTpNone, 0);                // the o sums
    return f;
}

// down + residual
GemvArgs down_args(llamini_session* s, u32 l) {
    const llamini_session::Layer& W = s->layers[l];
    GemvArgs d;
    d.err = &s->st->err;
    d.x = s->ffn_h;
    d.K = s->ffn;
    d.nseg = 1;
    d.seg[0] = {W.down.ptr, nullptr, W.down.row_bytes, 0, W.down.type, 0, W.down.rows, EPI_RESID, s->hidden, W.bdown, 0, 0};
    if (s->tp_world > 1) {
        d.seg[0].epi = EPI_STORE;
        d.seg[0].out = s->tp_part;
        if (tp().rank != 0) d.seg[0].bias = nullptr;
        if (s->tp_fuse_now) d.tp = tp_fused_args(1, kTpNone);
    }
    return d;
}

// final norm + lm_head + argmax
GemvArgs head_args(llamini_session* s) {
    const bool gpt2 = s->kind == 1;
    GemvArgs h;
    h.err = &s->st->err;
    h.x = s->hidden;
    h.K = s->dim;
    h.norm = gpt2 ? NORM_LAYER : NORM_RMS;
    h.norm_w = s->fnw;
    h.norm_b = s->fnb;
    h.eps = s->eps;
    h.nseg = 1;
    h.seg[0] = {s->head.ptr, nullptr, s->head.row_bytes, 0, s->head.type, 0, s->head.rows, EPI_STORE, s->logits, nullptr, 0, 1};
    h.argmax_key = &s->st->argmax_key;
    if (s->tp_fuse_now) h.tp = tp_fused_args(kTpNone, 1);               // the last layer's down sums
    return h;
}

// Whether a tensor-parallel session's steps fuse the o / down reductions into
// the GEMVs: every GEMV of the step on the tensor-core kernel (the CUDA-core
// one has no fused path) and LLAMINI_TP_FUSED not 0; decided once.
bool tp_fused(llamini_session* s) {
    if (s->tp_world < 2) return false;
    if (s->tp_fuse) return s->tp_fuse > 0;
    s->tp_fuse = -1;
    const char* e = getenv("LLAMINI_TP_FUSED");
    if ((e && e[0] == '0') || s->dim > kTpFusedFloats) return false;
    s->tp_fuse_now = true;
    bool ok = gemv_mma_takes(head_args(s));
    for (u32 l = 0; ok && l < s->n_layers; l++)
        ok = gemv_mma_takes(qkv_args(s, l)) && gemv_mma_takes(o_args(s, l)) && gemv_mma_takes(ffn_args(s, l)) &&
             gemv_mma_takes(down_args(s, l));
    s->tp_fuse_now = false;
    s->tp_fuse = ok ? 1 : -1;
    return ok;
}

bool enqueue_step(llamini_session* s, cudaStream_t st, bool trace, bool nll) {
    // tensor parallel: the reductions fused into the GEMVs, except when the
    // residual stream is traced after every layer (it is complete only after
    // the next GEMV's pull there)
    s->tp_fuse_now = !trace && tp_fused(s);
    const bool sep = s->tp_world > 1 && !s->tp_fuse_now;
    bool ok = launch_embed(embed_args(s), st);
    for (u32 l = 0; ok && l < s->n_layers; l++) {
        ok = launch_gemv(qkv_args(s, l), st) && launch_attention(attn_args(s, l), st) && launch_gemv(o_args(s, l), st) &&
             (!sep || launch_tp_allreduce(s->tp_part, s->hidden, s->dim, &s->st->err, st)) &&
             launch_gemv(ffn_args(s, l), st) && launch_gemv(down_args(s, l), st) &&
             (!sep || launch_tp_allreduce(s->tp_part, s->hidden, s->dim, &s->st->err, st)) &&
             (!trace || launch_copy_f32(s->trace + (size_t)l * s->dim, s->hidden, s->dim, st));
    }
    ok = ok && launch_gemv(head_args(s), st);
    s->tp_fuse_now = false;
    if (!ok) return false;
    FinishArgs fa;
    fa.st = s->st;
    fa.tokens = s->tokens;
    fa.max_tokens = s->max_seq + 1;
    fa.logits = s->logits;
    fa.vocab = s->vocab;
    fa.nll = nll ? 1u : 0u;
    return launch_finish(fa, st);
}

bool capture(llamini_session* s, u32 steps, bool trace, bool nll, cudaGraphExec_t* out) {
    cudaStream_t st = stream();
    cudaGraph_t g = nullptr;
    if (!LM_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal))) return false;
    bool ok = true;
    for (u32 i = 0; i < steps && ok; i++) ok = enqueue_step(s, st, trace, nll);
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (!ok || !LM_CUDA(e)) { if (g) cudaGraphDestroy(g); return false; }
    ok = LM_CUDA(cudaGraphInstantiate(out, g, 0));
    cudaGraphDestroy(g);
    return ok;
}

void destroy(llamini_session* s) {
    if (!s) return;
    cudaStreamSynchronize(stream());
    cudaGraphExec_t gs[] = {s->g_one, s->g_many, s->g_trace, s->g_nll};
    for (auto g : gs) if (g) cudaGraphExecDestroy(g);
    for (void* p : s->owned) dev_free(p);
    if (s->st_host) cudaFreeHost(s->st_host);
    delete s->pf;
    delete s;
}

bool g_kv_f16 = false;

// Op table and per-CTA schedule of the persistent decode kernel, built when
// LLAMINI_DECODE_KERNEL=1 at session creation (the per-op graphs are the
// default while they are the faster path). Returns true with dec_on = false
// when the kernel is not asked for, or the model has a matrix format or shape
// it does not take.
bool build_decode(llamini_session* s) {
    s->dec_on = false;
    const char* env = getenv("LLAMINI_DECODE_KERNEL");
    if (!env || env[0] != '1') return true;
    if (s->tp_world > 1) return true;                 // the allreduces run as their own kernels
    if (s->hd > 256 || s->hd == 0 || s->hd % 4 != 0 || s->n_split > 32) return true;
    std::vector<DecOp> ops;
    u32 kmax = 0;
    bool ok = true;
    auto add_gemv = [&](GemvArgs g, u32 trace_off) {
        DecOp op;
        op.kind = DEC_GEMV;
        u32 tiles = 0;
        for (u32 i = 0; i < g.nseg; i++) {
            GemvSeg& G = g.seg[i];
            const bool glu = G.epi == EPI_GLU_SILU || G.epi == EPI_GLU_GELU;
            if (!decode_supported_type(G.type) || (glu && G.type2 != G.type)) ok = false;
            if (reinterpret_cast<uintptr_t>(G.w) % 16 != 0 || (glu && reinterpret_cast<uintptr_t>(G.w2) % 16 != 0))
                ok = false;
            G.tile0 = tiles;
            tiles += (G.rows + 15) / 16;
        }
        if (g.K % 32 != 0 || reinterpret_cast<uintptr_t>(g.x) % 16 != 0) ok = false;
        const u32 kr = (g.K + 127) & ~127u;
        kmax = kmax > kr ? kmax : kr;
        op.g = g;
        op.ntasks = op.ndone = tiles;
        op.trace_off = trace_off;
        op.wait = ops.empty() ? kDecNoWait : (u32)ops.size() - 1;
        ops.push_back(op);
    };
    const u32 L = s->n_layers;
    const size_t n_ops = (size_t)L * 5 + 1;
    const size_t counter_words = 4 + n_ops;
    s->dec_counters = (u32*)own(s, counter_words * 4);
    if (!s->dec_counters) return false;
    s->dec_counter_bytes = counter_words * 4;
    // attention splits: at most one (head, split) task per CTA
    u32 dns = (u32)sm_count() / s->n_heads;
    dns = dns < 1 ? 1u : (dns > s->n_split ? s->n_split : dns);
    for (u32 l = 0; l < L && ok; l++) {
        add_gemv(qkv_args(s, l), 0xFFFFFFFFu);
        // attention: one task per (head, split), each leaving a partial
        DecOp at;
        at.kind = DEC_ATTN;
        at.at = attn_args(s, l);
        at.at.counter = nullptr;
        at.at.n_split = dns;
        at.n_split = dns;
        at.ntasks = at.ndone = s->n_heads * dns;
        at.wait = (u32)ops.size() - 1;
        ops.push_back(at);
        // the O projection merges the partials while staging its input
        add_gemv(o_args(s, l), 0xFFFFFFFFu);
        ops.back().x_merge = 1;
        ops.back().at = at.at;
        ops.back().n_split = dns;
        add_gemv(ffn_args(s, l), 0xFFFFFFFFu);
        add_gemv(down_args(s, l), l * s->dim);
    }
    if (ok) add_gemv(head_args(s), 0xFFFFFFFFu);
    if (!ok || ops.size() != n_ops || n_ops >= kDecMaxOps) return true;
    // shared memory: the ring must hold at least two of the largest tiles
    const u32 ring = decode_ring_bytes(kmax, s->hd);
    u32 max_tile = 0;
    for (const DecOp& op : ops)
        if (op.kind == DEC_GEMV)
            for (u32 i = 0; i < op.g.nseg; i++) {
                const u32 t = decode_tile_alloc(op.g.seg[i]);
                max_tile = max_tile > t ? max_tile : t;
            }
    if (ring == 0 || 2 * (u64)max_tile > ring) return true;
    for (const DecOp& op : ops)
        if (op.ntasks > 0xFFFFu) return true;
    // schedule: the tasks of each op in turn, dealt round-robin over the CTAs
    // with the dealing position carried from op to op, so every CTA gets an
    // equal share of the step's tiles
    const u32 n_cta = (u32)sm_count();
    std::vector<std::vector<u32>> per(n_cta);
    u32 cursor = 0;
    for (u32 i = 0; i < (u32)ops.size(); i++)
        for (u32 t = 0; t < ops[i].ntasks; t++) {
            per[cursor].push_back((i << 16) | t);
            cursor = (cursor + 1) % n_cta;
        }
    u32 stride = 1;
    for (auto& v : per) stride = stride > v.size() ? stride : (u32)v.size();
    if (stride > kDecMaxTasks || ops.size() > kDecMaxOpsSmem) return true;
    std::vector<u32> sched((size_t)n_cta * stride, 0u), len(n_cta);
    for (u32 c = 0; c < n_cta; c++) {
        len[c] = (u32)per[c].size();
        for (size_t k = 0; k < per[c].size(); k++) sched[(size_t)c * stride + k] = per[c][k];
    }
    DecOp* d_ops = (DecOp*)own(s, ops.size() * sizeof(DecOp));
    u32* d_sched = (u32*)own(s, sched.size() * 4);
    u32* d_len = (u32*)own(s, len.size() * 4);
    if (!d_ops || !d_sched || !d_len) return false;
    if (!LM_CUDA(cudaMemcpy(d_ops, ops.data(), ops.size() * sizeof(DecOp), cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemcpy(d_sched, sched.data(), sched.size() * 4, cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemcpy(d_len, len.data(), len.size() * 4, cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemset(s->dec_counters, 0, s->dec_counter_bytes)))
        return false;
    DecArgs& a = s->dec;
    a.ops = d_ops;
    a.n_ops = (u32)ops.size();
    a.sched = d_sched;
    a.sched_len = d_len;
    a.sched_stride = stride;
    a.n_cta = n_cta;
    a.sync = reinterpret_cast<DecSync*>(s->dec_counters);
    a.done = s->dec_counters + 4;
    a.st = s->st;
    a.tokens = s->tokens;
    a.max_tokens = s->max_seq + 1;
    a.tok = s->tok;
    a.pos = s->pos_tab;
    a.emb_scale = s->emb_scale;
    a.hidden = s->hidden;
    a.trace = nullptr;
    a.n_steps = 1;
    a.ring_bytes = ring;
    a.kmax = kmax;
    a.hd = s->hd;
    s->dec_on = true;
    return true;
}



// Op table, records and per-CTA schedule of the dataflow decode kernel
// (k_flow.cu). Taken by LLaMA-family models (RMSNorm, no tensor parallelism)
// whose matrices are all Q4_K or Q6_K with every K a multiple of 256 up to
// 6144; returns true with flow_on = false for any other model, which keeps
// the per-op graphs. LLAMINI_DECODE_KERNEL=0 turns it off, =1 selects the
// earlier persistent kernel instead.
bool build_flow(llamini_session* s) {
    s->flow_on = false;
    const char* env = getenv("LLAMINI_DECODE_KERNEL");
    if (env && (env[0] == '0' || env[0] == '1')) return true;
    if (s->kind != 0 || s->tp_world > 1) return true;
    if (s->hd == 0 || s->hd % 16 != 0 || s->hd > 256 || s->n_split > 32) return true;
    const u32 kmax = 256 * 8 * kFlowMaxSb;
    auto k_ok = [&](u32 K) { return K % 256 == 0 && K <= kmax; };
    if (!k_ok(s->dim) || !k_ok(s->ffn) || !k_ok(s->qd) || s->dim % 16 != 0) return true;
    auto m_ok = [](const DevMat& m) {
        return flow_supported_type(m.type) && reinterpret_cast<uintptr_t>(m.ptr) % 16 == 0;
    };
    for (const auto& W : s->layers)
        if (!m_ok(W.q) || !m_ok(W.k) || !m_ok(W.v) || !m_ok(W.o) || !m_ok(W.gate) || !m_ok(W.up) ||
            !m_ok(W.down) || W.gate.type != W.up.type)
            return true;
    if (!m_ok(s->head) || s->tok.ptr == nullptr) return true;
    const u32 L = s->n_layers;
    // attention splits of the flow kernel: at most one (head, split) task per CTA
    // (the partials buffer is sized for the per-op count, which is at least this)
    u32 fns = (u32)sm_count() / s->n_heads;
    fns = fns < 1 ? 1u : (fns > s->n_split ? s->n_split : fns);
    // records: A = the residual stream for QKV and the lm_head, B = for gate/up, C = the FFN activation
    auto rec = [&](u32 n, bool ss, FlowRec* r) {
        r->w = (uint32_t*)own(s, (size_t)n * 4);
        r->fs = (float2*)own(s, (size_t)n / 16 * sizeof(float2));
        r->ss = ss ? (float*)own(s, (size_t)n / 16 * 4) : nullptr;
        return r->w && r->fs && (!ss || r->ss);
    };
    FlowRec ra, rb, rc;
    if (!rec(s->dim, true, &ra) || !rec(s->dim, true, &rb) || !rec(s->ffn, false, &rc)) return false;
    std::vector<FlowOp> ops;
    auto seg = [](const DevMat& m, u32 epi, float* out, const float* bias) {
        FlowSeg g;
        g.w = m.ptr;
        g.row_bytes = m.row_bytes;
        g.type = m.type;
        g.rows = m.rows;
        g.epi = epi;
        g.out = out;
        g.bias = bias;
        return g;
    };
    auto gemv = [&](u32 K, u32 wait) {
        FlowOp op;
        op.kind = FLOW_GEMV;
        op.K = K;
        op.wait = wait;
        op.eps = s->eps;
        return op;
    };
    auto finish_op = [&](FlowOp& op) {
        u32 tiles = 0;
        for (u32 i = 0; i < op.nseg; i++) {
            op.seg[i].tile0 = tiles;
            tiles += (op.seg[i].rows + 15) / 16;
        }
        if (op.kind == FLOW_GEMV) op.ntasks = tiles;
        op.wait_n = op.wait == kFlowStepStart ? 0u : ops[op.wait].ntasks;
        ops.push_back(op);
        return (u32)ops.size() - 1;
    };
    u32 prev = kFlowStepStart;
    for (u32 l = 0; l < L; l++) {
        const auto& W = s->layers[l];
        FlowOp q = gemv(s->dim, prev);
        q.nseg = 3;
        q.seg[0] = seg(W.q, EPI_STORE, s->qkv, W.bq);
        q.seg[1] = seg(W.k, EPI_STORE, s->qkv + s->qd, W.bk);
        q.seg[2] = seg(W.v, EPI_STORE, s->qkv + s->qd + s->kvd, W.bv);
        q.in = ra;
        const u32 qi = finish_op(q);
        FlowOp at;
        at.kind = FLOW_ATTN;
        at.at = attn_args(s, l);
        at.at.counter = nullptr;
        at.at.n_split = fns;
        at.n_split = fns;
        at.ntasks = s->n_heads * fns;
        at.wait = qi;
        const u32 ai = finish_op(at);
        FlowOp o = gemv(s->qd, ai);
        o.nseg = 1;
        o.seg[0] = seg(W.o, EPI_RESID, nullptr, W.bo);
        o.in_attn = 1;
        o.at = ops[ai].at;
        o.n_split = fns;
        o.out = rb;
        o.out_nw = W.n2w;
        const u32 oi = finish_op(o);
        FlowOp f = gemv(s->dim, oi);
        f.nseg = 1;
        f.seg[0] = seg(W.gate, s->act_gelu ? (u32)EPI_GLU_GELU : (u32)EPI_GLU_SILU, s->ffn_h, nullptr);
        f.seg[0].w2 = W.up.ptr;
        f.seg[0].row_bytes2 = W.up.row_bytes;
        f.in = rb;
        f.out = rc;
        const u32 fi = finish_op(f);
        FlowOp d = gemv(s->ffn, fi);
        d.nseg = 1;
        d.seg[0] = seg(W.down, EPI_RESID, nullptr, W.bdown);
        d.in = rc;
        d.out = ra;
        d.out_nw = l + 1 < L ? s->layers[l + 1].n1w : s->fnw;
        d.trace_off = l * s->dim;
        prev = finish_op(d);
    }
    FlowOp h = gemv(s->dim, prev);
    h.nseg = 1;
    h.seg[0] = seg(s->head, EPI_STORE, s->logits, nullptr);
    h.in = ra;
    h.argmax = 1;
    finish_op(h);
    if (ops.size() > kFlowMaxOps || ops.size() >= (1u << 16)) return true;
    for (const FlowOp& op : ops)
        if (op.ntasks > 0xFFFFu) return true;
    // shared memory: the ring must hold two of the largest tiles
    const u32 ring = flow_ring_bytes(s->hd);
    u32 max_tile = 0;
    for (const FlowOp& op : ops)
        for (u32 i = 0; op.kind == FLOW_GEMV && i < op.nseg; i++) {
            const u32 t = flow_tile_alloc(op.seg[i]);
            max_tile = max_tile > t ? max_tile : t;
        }
    if (ring == 0 || 2 * (u64)max_tile > ring) return true;
    // schedule: the tasks of each op in turn, dealt round-robin over the CTAs
    // with the dealing position carried from op to op
    const u32 n_cta = (u32)sm_count();
    std::vector<std::vector<u32>> per(n_cta);
    u32 cursor = 0;
    for (u32 i = 0; i < (u32)ops.size(); i++)
        for (u32 t = 0; t < ops[i].ntasks; t++) {
            per[cursor].push_back((i << 16) | t);
            cursor = (cursor + 1) % n_cta;
        }
    u32 stride = 1;
    for (auto& v : per) stride = stride > v.size() ? stride : (u32)v.size();
    if (stride > kFlowMaxTasks) return true;
    std::vector<u32> sched((size_t)n_cta * stride, 0u), len(n_cta);
    for (u32 c = 0; c < n_cta; c++) {
        len[c] = (u32)per[c].size();
        for (size_t k = 0; k < per[c].size(); k++) sched[(size_t)c * stride + k] = per[c][k];
    }
    // one tensor map per matrix whose tiles move through TMA tensor copies
    const u32 n_maps = flow_maps_needed(ops.data(), (u32)ops.size());
    if (n_maps) {
        CUtensorMap* d_maps = (CUtensorMap*)own(s, (size_t)n_maps * sizeof(CUtensorMap));
        if (!d_maps) return false;
        if (!flow_encode_maps(ops.data(), (u32)ops.size(), d_maps)) return true;   // keep the per-op graphs
    }
    const size_t counter_words = 4 + ops.size();
    s->flow_counters = (u32*)own(s, counter_words * 4);
    FlowOp* d_ops = (FlowOp*)own(s, ops.size() * sizeof(FlowOp));
    u32* d_sched = (u32*)own(s, sched.size() * 4);
    u32* d_len = (u32*)own(s, len.size() * 4);
    if (!s->flow_counters || !d_ops || !d_sched || !d_len) return false;
    s->flow_counter_bytes = counter_words * 4;
    if (!LM_CUDA(cudaMemcpy(d_ops, ops.data(), ops.size() * sizeof(FlowOp), cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemcpy(d_sched, sched.data(), sched.size() * 4, cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemcpy(d_len, len.data(), len.size() * 4, cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemset(s->flow_counters, 0, s->flow_counter_bytes)))
        return false;
    FlowArgs& a = s->flow;
    a.ops = d_ops;
    a.n_ops = (u32)ops.size();
    a.sched = d_sched;
    a.sched_len = d_len;
    a.sched_stride = stride;
    a.n_cta = n_cta;
    a.sync = reinterpret_cast<DecSync*>(s->flow_counters);
    a.done = s->flow_counters + 4;
    a.st = s->st;
    a.tokens = s->tokens;
    a.max_tokens = s->max_seq + 1;
    a.tok = s->tok;
    a.emb_scale = s->emb_scale;
    a.hidden = s->hidden;
    a.in0 = ra;
    a.n1w0 = s->layers[0].n1w;
    a.dim = s->dim;
    a.trace = nullptr;
    a.n_steps = 1;
    a.ring_bytes = ring;
    a.hd = s->hd;
    s->flow_on = true;
    return true;
}

// theta_j = base^(-2j/hd), evaluated exactly as model.c:38 / model.c:50 do
bool upload_theta(llamini_session* s) {
    std::vector<f32> th(s->hd / 2 ? s->hd / 2 : 1);
    for (u32 j = 0; j < s->hd / 2; j++) th[j] = powf(s->rope_base, -(f32)(2 * j) / (f32)s->hd);
    s->theta = upload_f32(s, th.data(), th.size());
    return s->theta != nullptr;
}

bool finish_build(llamini_session* s) {
    s->kv_f16 = g_kv_f16 ? 1u : 0u;
    s->n_split = choose_splits(s->n_heads, s->max_seq);
    if (!alloc_buffers(s)) return false;
    if (!capture(s, 1, false, false, &s->g_one)) return false;
    if (!capture(s, kStepsPerGraph, false, false, &s->g_many)) return false;
    if (!build_flow(s)) return false;
    return s->flow_on || build_decode(s);
}

llamini_session* find(const void* model, KVCache* caches) {
    for (auto* s : g_sessions)
        if (s->model == model && s->caches == caches && s->cache_max_seq == caches[0].max_seq &&
            s->cache_dim == caches[0].dim)
            return s;
    return nullptr;
}

void drop_where(bool (*pred)(const llamini_session*, const void*), const void* key) {
    for (auto it = g_sessions.begin(); it != g_sessions.end();) {
        if (pred(*it, key)) { destroy(*it); it = g_sessions.erase(it); }
        else ++it;
    }
}

// Shape and device weights of a LLaMA-family model (everything a step reads
// that does not depend on the caches).
bool bind_llama(llamini_session* s, LLaMAModel* m, u32 max_seq) {
    const LLaMAConfig& c = m->cfg;
    s->kind = 0;
    s->model = m;
    s->n_layers = c.n_layers; s->dim = c.dim; s->n_heads = c.n_heads; s->n_kv = c.n_heads_kv;
    s->hd = c.head_dim; s->ffn = c.ffn_dim; s->vocab = c.vocab_size;
    s->qd = c.n_heads * c.head_dim; s->kvd = c.n_heads_kv * c.head_dim;
    s->max_seq = max_seq;
    s->max_pos = max_seq;                             // generate.c:142
    s->eps = c.rms_eps; s->rope_base = c.rope_freq_base; s->emb_scale = c.embedding_scale;
    s->rope_mode = c.rope_type == ROPE_NEOX ? 2u : 1u;
    s->act_gelu = c.ffn_act == ACT_GELU;
    bool ok = s->n_kv > 0 && s->n_heads % s->n_kv == 0 && s->hd > 0;
    if (!ok) set_error("llama session: inconsistent heads (heads %u kv %u hd %u)", s->n_heads, s->n_kv, s->hd);
    // tensor parallelism: rank R of W keeps heads [R H/W, (R+1) H/W), the matching
    // kv heads, and FFN columns [f0, f1) on 256-column boundaries (uneven when the
    // super-blocks do not divide); embeddings, norms and lm_head stay whole
    const u32 W = tp().world, R = tp().rank;
    u32 f0 = 0, f1 = c.ffn_dim;
    if (ok && W > 1) {
        s->tp_world = W;
        u32 plan[8];
        if (tp_plan(W, R, s->n_heads, s->n_kv, s->hd, c.ffn_dim, plan) != 0) return false;
        s->n_heads /= W;
        s->n_kv /= W;
        s->qd /= W;
        s->kvd /= W;
        f0 = plan[4];
        f1 = plan[5];
        s->ffn = f1 - f0;
    }
    ok = ok && weight(s, m->embeddings, c.vocab_size, c.dim, &s->tok);
    ok = ok && weight(s, m->lm_head, c.vocab_size, c.dim, &s->head);
    s->fnw = ok ? vec(s, m->final_norm, c.dim) : nullptr;
    ok = ok && s->fnw;
    s->layers.resize(c.n_layers);
    for (u32 l = 0; ok && l < c.n_layers; l++) {
        const DecoderLayer& L = m->layers[l];
        auto& W = s->layers[l];
        const u32 QD = c.n_heads * c.head_dim, KVD = c.n_heads_kv * c.head_dim;   // whole-model widths
        if (s->tp_world > 1) {
            // this rank's shard only, straight from the mapped file
            ok = weight_shard(s, L.q_proj, QD, c.dim, R * s->qd, s->qd, 0, c.dim, &W.q) &&
                 weight_shard(s, L.k_proj, KVD, c.dim, R * s->kvd, s->kvd, 0, c.dim, &W.k) &&
                 weight_shard(s, L.v_proj, KVD, c.dim, R * s->kvd, s->kvd, 0, c.dim, &W.v) &&
                 weight_shard(s, L.o_proj, c.dim, QD, 0, c.dim, R * s->qd, (R + 1) * s->qd, &W.o) &&
                 weight_shard(s, L.gate_proj, c.ffn_dim, c.dim, f0, f1 - f0, 0, c.dim, &W.gate) &&
                 weight_shard(s, L.up_proj, c.ffn_dim, c.dim, f0, f1 - f0, 0, c.dim, &W.up) &&
                 weight_shard(s, L.down_proj, c.dim, c.ffn_dim, 0, c.dim, f0, f1, &W.down);
        } else {
            ok = weight(s, L.q_proj, QD, c.dim, &W.q) && weight(s, L.k_proj, KVD, c.dim, &W.k) &&
                 weight(s, L.v_proj, KVD, c.dim, &W.v) && weight(s, L.o_proj, c.dim, QD, &W.o) &&
                 weight(s, L.gate_proj, c.ffn_dim, c.dim, &W.gate) && weight(s, L.up_proj, c.ffn_dim, c.dim, &W.up) &&
                 weight(s, L.down_proj, c.dim, c.ffn_dim, &W.down);
        }
        if (ok) { W.n1w = vec(s, L.attn_norm, c.dim); W.n2w = vec(s, L.ffn_norm, c.dim); ok = W.n1w && W.n2w; }
        if (ok && c.qkv_bias) {
            W.bq = vec(s, L.q_bias, QD); W.bk = vec(s, L.k_bias, KVD); W.bv = vec(s, L.v_bias, KVD);
            ok = W.bq && W.bk && W.bv;
            if (ok && s->tp_world > 1) {                  // this rank's slice of each bias
                W.bq += R * s->qd;
                W.bk += R * s->kvd;
                W.bv += R * s->kvd;
            }
        }
    }
    // the tok table is read one row per step, not whole
    if (ok) s->weight_bytes -= s->tok.row_bytes * (s->tok.rows - 1);
    return ok && upload_theta(s);
}

bool bind_gpt2(llamini_session* s, GPT2Model* m, u32 max_seq) {
    const GPT2Config& c = m->cfg;
    s->kind = 1;
    s->model = m;
    s->n_layers = c.n_layers; s->dim = c.dim; s->n_heads = c.n_heads; s->n_kv = c.n_heads;
    s->hd = c.n_heads ? c.dim / c.n_heads : 0; s->ffn = c.ffn_dim; s->vocab = c.vocab_size;
    s->qd = c.dim; s->kvd = c.dim;
    s->max_seq = max_seq;
    s->max_pos = max_seq < c.n_ctx ? max_seq : c.n_ctx;   // gpt2.c:205
    s->eps = c.ln_eps; s->rope_mode = 0; s->emb_scale = 1.0f;
    bool ok = s->hd > 0;
    if (!ok) set_error("gpt2 session: no heads");
    ok = ok && weight(s, m->token_embd, c.vocab_size, c.dim, &s->tok);
    ok = ok && weight(s, m->pos_embd, c.n_ctx, c.dim, &s->pos_tab);
    ok = ok && weight(s, m->lm_head, c.vocab_size, c.dim, &s->head);
    if (ok) { s->fnw = vec(s, m->output_norm_w, c.dim); s->fnb = vec(s, m->output_norm_b, c.dim); ok = s->fnw && s->fnb; }
    s->layers.resize(c.n_layers);
    for (u32 l = 0; ok && l < c.n_layers; l++) {
        const GPT2Layer& L = m->layers[l];
        auto& W = s->layers[l];
        ok = weight(s, L.attn_qkv_w, 3 * c.dim, c.dim, &W.q) && weight(s, L.attn_out_w, c.dim, c.dim, &W.o) &&
             weight(s, L.ffn_up_w, c.ffn_dim, c.dim, &W.up) && weight(s, L.ffn_down_w, c.dim, c.ffn_dim, &W.down);
        if (ok) {
            W.n1w = vec(s, L.attn_norm_w, c.dim); W.n1b = vec(s, L.attn_norm_b, c.dim);
            W.n2w = vec(s, L.ffn_norm_w, c.dim); W.n2b = vec(s, L.ffn_norm_b, c.dim);
            W.bq = vec(s, L.attn_qkv_b, 3 * c.dim); W.bo = vec(s, L.attn_out_b, c.dim);
            W.bup = vec(s, L.ffn_up_b, c.ffn_dim); W.bdown = vec(s, L.ffn_down_b, c.dim);
            ok = W.n1w && W.n1b && W.n2w && W.n2b && W.bq && W.bo && W.bup && W.bdown;
        }
    }
    if (ok) {
        s->weight_bytes -= s->tok.row_bytes * (s->tok.rows - 1);
        s->weight_bytes -= s->pos_tab.row_bytes * (s->pos_tab.rows - 1);
    }
    return ok && upload_theta(s);
}

llamini_session* build_llama(LLaMAModel* m, KVCache* caches) {
    if (!ensure_device()) return nullptr;
    auto* s = new llamini_session();
    s->caches = caches;
    s->cache_max_seq = caches[0].max_seq;
    s->cache_dim = caches[0].dim;
    bool ok = bind_llama(s, m, caches[0].max_seq);
    if (ok && caches[0].dim != s->kvd * s->tp_world) {    // the caller's cache is whole-model width
        set_error("llama session: cache dim %u != kv dim %u", caches[0].dim, s->kvd * s->tp_world);
        ok = false;
    }
    ok = ok && finish_build(s);
    if (!ok) { destroy(s); return nullptr; }
    g_sessions.push_back(s);
    return s;
}

llamini_session* build_gpt2(GPT2Model* m, KVCache* caches) {
    if (!ensure_device()) return nullptr;
    auto* s = new llamini_session();
    s->caches = caches;
    s->cache_max_seq = caches[0].max_seq;
    s->cache_dim = caches[0].dim;
    bool ok = bind_gpt2(s, m, caches[0].max_seq);
    if (ok && caches[0].dim != m->cfg.dim) {
        set_error("gpt2 session: cache dim %u != model dim %u", caches[0].dim, m->cfg.dim);
        ok = false;
    }
    ok = ok && finish_build(s);
    if (!ok) { destroy(s); return nullptr; }
    g_sessions.push_back(s);
    return s;
}

// ---------------------------------------------------------------- running

bool write_state(llamini_session* s, u32 pos, u32 n_prompt, bool reset_nll) {
    cudaStream_t st = stream();
    if (!LM_CUDA(cudaStreamSynchronize(st))) return false;   // st_host is reused
    s->st_host->pos = pos;
    s->st_host->n_prompt = n_prompt;
    s->st_host->trace = 0;
    s->st_host->err = 0;
    s->st_host->argmax_key = 0;
    s->st_host->nll = 0.0;
    s->st_host->nll_count = 0;
    const size_t n = reset_nll ? sizeof(StepState) : offsetof(StepState, nll);
    if (!LM_CUDA(cudaMemcpyAsync(s->st, s->st_host, n, cudaMemcpyHostToDevice, st))) return false;
    if (s->dec_on && !LM_CUDA(cudaMemsetAsync(s->dec_counters, 0, s->dec_counter_bytes, st))) return false;
    if (s->flow_on && !LM_CUDA(cudaMemsetAsync(s->flow_counters, 0, s->flow_counter_bytes, st))) return false;
    s->pos = pos;
    s->n_prompt = n_prompt;
    return true;
}

bool run_steps(llamini_session* s, u32 n) {
    if ((u64)s->pos + n > s->max_pos) {
        set_error("position %u + %u steps passes the cache capacity %u", s->pos, n, s->max_pos);
        return false;
    }
    cudaStream_t st = stream();
    if (s->flow_on && n > 0) {
        // the kernel prepares the input of each following step itself; the
        // first step's input is prepared here
        FlowArgs a = s->flow;
        a.trace = s->trace_on ? s->trace : nullptr;
        if (!launch_flow_embed(a, st)) return false;
        for (u32 left = n; left > 0;) {
            a.n_steps = left < kDecStepsPerLaunch ? left : kDecStepsPerLaunch;
            if (!launch_flow(a, st)) return false;
            left -= a.n_steps;
        }
        s->pos += n;
        return true;
    }
    if (s->dec_on && n > 0) {
        // the kernel embeds the input of each following step itself; the first
        // step's input is embedded here
        if (!launch_embed(embed_args(s), st)) return false;
        DecArgs a = s->dec;
        a.trace = s->trace_on ? s->trace : nullptr;
        for (u32 left = n; left > 0;) {
            a.n_steps = left < kDecStepsPerLaunch ? left : kDecStepsPerLaunch;
            if (!launch_decode(a, st)) return false;
            left -= a.n_steps;
        }
        s->pos += n;
        return true;
    }
    if (s->trace_on) {
        if (!s->g_trace && !capture(s, 1, true, false, &s->g_trace)) return false;
        for (u32 i = 0; i < n; i++) if (!LM_CUDA(cudaGraphLaunch(s->g_trace, st))) return false;
        s->pos += n;
        return true;
    }
    u32 left = n;
    while (left >= kStepsPerGraph) {
        if (!LM_CUDA(cudaGraphLaunch(s->g_many, st))) return false;
        left -= kStepsPerGraph;
    }
    while (left--) if (!LM_CUDA(cudaGraphLaunch(s->g_one, st))) return false;
    s->pos += n;
    return true;
}

// Device-side error bits (bounded waits that ran out): read after a sync.
bool check_device_errors(llamini_session* s) {
    uint32_t e = 0;
    if (!LM_CUDA(cudaMemcpy(&e, &s->st->err, 4, cudaMemcpyDeviceToHost))) return false;
    if (e) {
        set_error("a kernel reported error bits 0x%x (a bounded wait ran out: a weight copy, or a tensor-parallel "
                  "peer that did not arrive; the bits stay set, so the session refuses later steps)", e);
        return false;
    }
    return true;
}

void set_cur_seq(llamini_session* s, u32 n) {
    for (u32 l = 0; l < s->n_layers; l++) s->caches[l].cur_seq = n;
}
void set_cur_seq(llamini_session* s) { set_cur_seq(s, s->pos); }

}  // namespace

void drop_sessions_for_model(const void* model) {
    drop_where([](const llamini_session* s, const void* k) { return s->model == k; }, model);
}
void drop_sessions_for_gguf(const GGUFFile* gf) {
    drop_where([](const llamini_session* s, const void* k) { return s->gf == k; }, gf);
}
void drop_all_sessions() {
    for (auto* s : g_sessions) destroy(s);
    g_sessions.clear();
}

namespace {
// Prompt positions [pos, pos + n) without logits: chunked prefill when the
// model allows it, else decode steps (defined with the batched code below).
bool run_prompt(llamini_session* s, u32 n);
int prefill_perplexity(llamini_session* s, u32 steps, double* nll);
}  // namespace

// Shared by forward_step and gpt2_forward_step.
static void forward_one(llamini_session* s, u32 pos, u32 token, f32* logits_out) {
    if (!s) { if (logits_out) memset(logits_out, 0, 4); return; }
    if (pos >= s->max_seq) { set_error("forward: position %u outside the cache (%u)", pos, s->max_seq); return; }
    cudaStream_t st = stream();
    if (!write_state(s, pos, 0xFFFFFFFFu, false)) return;
    if (!LM_CUDA(cudaMemcpyAsync(s->tokens + pos, &token, 4, cudaMemcpyHostToDevice, st))) return;
    const u32 saved = s->max_pos;
    s->max_pos = s->max_seq;
    bool ok = run_steps(s, 1);
    s->max_pos = saved;
    if (!ok) return;
    if (logits_out && !LM_CUDA(cudaMemcpyAsync(logits_out, s->logits, (size_t)s->vocab * 4, cudaMemcpyDeviceToHost, st))) return;
    if (!LM_CUDA(cudaStreamSynchronize(st)) || !check_device_errors(s)) return;
    set_cur_seq(s);
}

// generate.c:122-167 / gpt2.c:194-229.
static u32 generate(llamini_session* s, u32* input, u32 n_in, u32* out, u32 max_gen, u32 eos, f32 temp, f32 top_p) {
    memcpy(out, input, (size_t)n_in * sizeof(u32));
    if (!s) return n_in;
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    u32 total = n_in;
    cudaStream_t st = stream();
    if (temp > 0.0f) {
        // Sampled decoding (generate.c:122-167 with sample_token): the prompt as
        // in the greedy path, then per token one step, one draw from the host
        // rand() stream (generate.c:50; one per token, in the reference's order)
        // and the device sampler (k_sample.cu), whose pick is the next step's
        // input; only the token comes back to the host.
        const u32 first = n_in > 0 ? n_in : 1;
        if (!write_state(s, 0, first, true)) return total;
        if (!LM_CUDA(cudaMemcpyAsync(s->tokens, out, (size_t)first * 4, cudaMemcpyHostToDevice, st))) return total;
        u32 pre = n_in > 1 ? n_in - 1 : 0;
        if (pre > s->max_pos) pre = s->max_pos;
        if (pre && !run_prompt(s, pre)) return total;
        u32 tok = 0;
        while (s->pos < s->max_pos) {
            const f32 u = (f32)rand() / ((f32)RAND_MAX + 1.0f);
            const u32 p = s->pos;
            if (!run_steps(s, 1)) break;
            if (!launch_sample(s->logits, s->vocab, temp, top_p, u, s->probs, s->tokens + p + 1, st) ||
                !LM_CUDA(cudaMemcpyAsync(&tok, s->tokens + p + 1, 4, cudaMemcpyDeviceToHost, st)) ||
                !LM_CUDA(cudaStreamSynchronize(st)))
                break;
            out[total++] = tok;
            if (tok == eos || total - n_in >= max_gen) break;
        }
    } else {
        // Forward passes the reference runs without an early EOS: every prompt
        // position, then one per generated token, the last one producing the
        // max_gen-th token (at least one token is always generated).
        const u32 gen_target = max_gen > 0 ? max_gen : 1;
        u64 want = (n_in > 0 ? (u64)n_in - 1 : 0) + gen_target;
        if (want > s->max_pos) want = s->max_pos;
        const u32 first = n_in > 0 ? n_in : 1;
        if (!write_state(s, 0, first, true)) return total;
        if (!LM_CUDA(cudaMemcpyAsync(s->tokens, out, (size_t)first * 4, cudaMemcpyHostToDevice, st))) return total;
        const bool eos_possible = eos < s->vocab;
        u32 done = 0;
        // prefill positions produce no tokens; run them in one go
        u32 pre = n_in > 1 ? n_in - 1 : 0;
        if (pre > want) pre = (u32)want;
        if (pre && !run_prompt(s, pre)) return total;
        done = pre;
        std::vector<u32> buf;
        u32 last = done;                                   // positions run, as the reference counts them
        while (done < want) {
            u32 chunk = (u32)(want - done);
            if (eos_possible && chunk > 16) chunk = 16;
            if (!run_steps(s, chunk)) break;
            // tokens produced: positions done+1 .. done+chunk
            buf.resize(chunk);
            if (!LM_CUDA(cudaMemcpyAsync(buf.data(), s->tokens + done + 1, (size_t)chunk * 4, cudaMemcpyDeviceToHost, st)) ||
                !LM_CUDA(cudaStreamSynchronize(st)))
                break;
            bool stop = false;
            for (u32 i = 0; i < chunk; i++) {
                const u32 p = done + i;                       // step position
                if (p + 1 < n_in) continue;
                out[total++] = buf[i];
                last = p + 1;
                if (buf[i] == eos || total - n_in >= gen_target) { stop = true; break; }
            }
            done += chunk;
            if (!stop) last = done;
            if (stop) break;
        }
        check_device_errors(s);
        set_cur_seq(s, last);
    }
    clock_gettime(CLOCK_MONOTONIC, &t1);
    const u32 ng = total - n_in;
    const double el = (double)(t1.tv_sec - t0.tv_sec) + (double)(t1.tv_nsec - t0.tv_nsec) * 1e-9;
    if (ng > 0 && el > 0.0) fprintf(stderr, "[%u tokens in %.2fs, %.2f tok/s]\n", ng, el, ng / el);
    return total;
}

// generate.c:169-197 / gpt2.c:231-256.
static f32 perplexity(llamini_session* s, const u32* tokens, u32 n) {
    if (!s) return -1.0f;
    for (u32 l = 0; l < s->n_layers; l++) kv_cache_reset(&s->caches[l]);
    u32 steps = 0;
    while (steps + 1 < n && steps < s->max_pos) steps++;
    if (steps == 0) return -1.0f;
    cudaStream_t st = stream();
    if (steps >= 2) {
        // 64 positions at a time through the tensor-core GEMMs, when available;
        // the log-probs are summed here in position order, as the reference does
        double nll = 0.0;
        if (!write_state(s, 0, n, true)) return -1.0f;
        const u32 ncopy = n < s->max_seq + 1 ? n : s->max_seq + 1;
        if (!LM_CUDA(cudaMemcpyAsync(s->tokens, tokens, (size_t)ncopy * 4, cudaMemcpyHostToDevice, st))) return -1.0f;
        const int r = prefill_perplexity(s, steps, &nll);
        if (r < 0) return -1.0f;                     // failed: the error is set
        if (r > 0) {
            set_cur_seq(s);
            return expf((f32)(nll / steps));
        }
    }
    if (!s->g_nll && !capture(s, 1, false, true, &s->g_nll)) return -1.0f;
    if (!write_state(s, 0, n, true)) return -1.0f;
    const u32 ncopy = n < s->max_seq + 1 ? n : s->max_seq + 1;
    if (!LM_CUDA(cudaMemcpyAsync(s->tokens, tokens, (size_t)ncopy * 4, cudaMemcpyHostToDevice, st))) return -1.0f;
    for (u32 i = 0; i < steps; i++) if (!LM_CUDA(cudaGraphLaunch(s->g_nll, st))) return -1.0f;
    s->pos = steps;
    if (!LM_CUDA(cudaMemcpyAsync(s->st_host, s->st, sizeof(StepState), cudaMemcpyDeviceToHost, st)) ||
        !LM_CUDA(cudaStreamSynchronize(st)))
        return -1.0f;
    set_cur_seq(s);
    if (s->st_host->nll_count == 0) return -1.0f;
    return expf((f32)(s->st_host->nll / s->st_host->nll_count));
}

static llamini_session* llama_session(LLaMAModel* m, KVCache* c) {
    if (!m || !c) { set_error("null model or caches"); return nullptr; }
    llamini_session* s = find(m, c);
    return s ? s : build_llama(m, c);
}
static llamini_session* gpt2_session(GPT2Model* m, KVCache* c) {
    if (!m || !c) { set_error("null model or caches"); return nullptr; }
    llamini_session* s = find(m, c);
    return s ? s : build_gpt2(m, c);
}

}  // namespace lm

// ================================================================ batched decode
//
// Up to max_batch sequences in lockstep: every step runs position p of every
// sequence; a sequence reads its prompt until p passes it, then its own greedy
// tokens (the semantics of generate_autoregressive per sequence). Each weight
// matrix is read once per step for the whole batch (k_bgemm.cu); norms, RoPE,
// attention and the argmax are per sequence.

struct llamini_batch {
    llamini_session* w = nullptr;     // shape and device weights (no single-sequence buffers)
    u32 max_batch = 0, max_seq = 0, B = 0;
    u32 n_split = 1, kv_f16 = 0, kmax = 0;
    float *hidden = nullptr, *qkv = nullptr, *attn = nullptr, *ffn_h = nullptr, *logits = nullptr;
    float* probs = nullptr;               // the device sampler's scratch (vocab floats)
    float* tp_part = nullptr;             // tensor parallel: the batch's o / down partial sums
    float *sx = nullptr, *part = nullptr, *part2 = nullptr, *part3 = nullptr, *apart = nullptr;
    uint16_t *xh = nullptr, *xl = nullptr;
    u32 *counters = nullptr, *tokens = nullptr, *n_prompt = nullptr;
    u32* err = nullptr;               // tensor-core GEMM error bits
    bool tc = false;                  // matrices on the tcgen05 GEMM (else mma.sync)
    // copies of matrices whose row size is not a multiple of 16 bytes, rows
    // padded to one (the tensor-core GEMM loads rows by TMA): pointer, pitch
    std::unordered_map<const uint8_t*, std::pair<const uint8_t*, uint64_t>> pitched;   // PitchMap
    unsigned long long* keys = nullptr;
    void *kc = nullptr, *vc = nullptr;
    lm::StepState* st = nullptr;
    size_t part_floats = 0;
    u32 plan_B = 0;                   // B the graphs were captured for
    cudaGraphExec_t g_one = nullptr, g_many = nullptr;
    u32 pos = 0;
    std::vector<u32> lens;
};

namespace lm {
namespace {

constexpr u32 kBatchStepsPerGraph = 8;

size_t batch_cache_bytes_per_seq(const llamini_batch* b) {
    return (size_t)b->w->n_kv * b->max_seq * b->w->hd * (b->kv_f16 ? 2 : 4);
}

// GEMM plan of up to three matrices that share an input, on the tcgen05 GEMM
// (k_tgemm.cu) or the mma.sync one (k_bgemm.cu); both write raw sums
// part[ksplit][B][rows] that bfinish_kernel completes.
struct BPlan {
    bool tc = false;
    BGemmArgs m;
    TGemmArgs t;
    u32 ksplit() const { return tc ? t.ksplit : m.ksplit; }
    float* part(u32 i) const { return tc ? t.seg[i].part : m.seg[i].part; }
    u32 rows(u32 i) const { return tc ? t.seg[i].rows : m.seg[i].rows; }
};

bool launch_plan(const BPlan& p, cudaStream_t st) { return p.tc ? launch_tgemm(p.t, st) : launch_bgemm(p.m, st); }

using PitchMap = std::unordered_map<const uint8_t*, std::pair<const uint8_t*, uint64_t>>;

// A copy of m with rows padded to a multiple of 16 bytes, when its rows are
// not (the tensor-core GEMM loads rows by TMA); recorded in `map`.
bool make_pitched(llamini_session* s, PitchMap& map, const DevMat& m) {
    if (!m.ptr || !tgemm_type(m.type) || m.row_bytes % 16 == 0 || map.count(m.ptr)) return true;
    const uint64_t p = (m.row_bytes + 15) & ~uint64_t(15);
    uint8_t* d = (uint8_t*)own(s, p * m.rows + 16);
    if (!d || !LM_CUDA(cudaMemcpy2D(d, p, m.ptr, m.row_bytes, m.row_bytes, m.rows, cudaMemcpyDeviceToDevice)))
        return false;
    map[m.ptr] = {d, p};
    return true;
}
bool make_pitched_all(llamini_session* s, PitchMap& map) {
    bool ok = make_pitched(s, map, s->head);
    for (u32 l = 0; ok && l < s->n_layers; l++) {
        const auto& W = s->layers[l];
        ok = make_pitched(s, map, W.q) && make_pitched(s, map, W.k) && make_pitched(s, map, W.v) &&
             make_pitched(s, map, W.o) && make_pitched(s, map, W.gate) && make_pitched(s, map, W.up) &&
             make_pitched(s, map, W.down);
    }
    return ok;
}

// Tensor-core GEMM plan of up to three matrices sharing staged inputs xh/xl of
// B columns (false: a format or shape the kernel does not take).
bool plan_tc(const uint16_t* xh, const uint16_t* xl, u32 B, u32* err, const PitchMap& pitched,
             const DevMat* const* m, float* const* parts, u32 n, u32 K, TGemmArgs* out) {
    TGemmArgs g;
    g.xh = xh;
    g.xl = xl;
    g.B = B;
    g.K = K;
    g.nseg = n;
    g.err = err;
    for (u32 i = 0; i < n; i++) {
        if (m[i]->cols != K) return false;
        g.seg[i].w = m[i]->ptr;
        g.seg[i].row_bytes = m[i]->row_bytes;
        g.seg[i].type = m[i]->type;
        g.seg[i].rows = m[i]->rows;
        g.seg[i].part = parts[i];
        const auto it = pitched.find(m[i]->ptr);
        if (it != pitched.end()) {
            g.seg[i].w = it->second.first;
            g.seg[i].pitch = it->second.second;
        }
    }
    if (!tgemm_plan(g, (u32)sm_count())) return false;
    *out = g;
    return true;
}

// False when a format or shape has no batched kernel; segment i writes its
// raw sums to parts[i].
bool batch_gemm(const llamini_batch* b, const DevMat* const* m, float* const* parts, u32 n, u32 K, BPlan* out) {
    BPlan p;
    p.tc = b->tc;
    for (u32 i = 0; i < n; i++)
        if (m[i]->cols != K) return false;
    if (p.tc) {
        if (!plan_tc(b->xh, b->xl, b->B, b->err, b->pitched, m, parts, n, K, &p.t)) return false;
    } else {
        BGemmArgs& g = p.m;
        g.xh = b->xh;
        g.xl = b->xl;
        g.sx = b->sx;
        g.B = b->B;
        g.K = K;
        g.nseg = n;
        for (u32 i = 0; i < n; i++) {
            g.seg[i].w = m[i]->ptr;
            g.seg[i].row_bytes = m[i]->row_bytes;
            g.seg[i].type = m[i]->type;
            g.seg[i].rows = m[i]->rows;
            g.seg[i].part = parts[i];
        }
        if (!bgemm_plan(g, 2u * (u32)sm_count())) return false;
    }
    *out = p;
    return true;
}
bool batch_gemm(const llamini_batch* b, const DevMat& m, u32 K, float* part, BPlan* out) {
    const DevMat* mm[1] = {&m};
    float* pp[1] = {part};
    return batch_gemm(b, mm, pp, 1, K, out);
}

bool batch_stage(llamini_batch* b, const float* x, u32 K, u32 norm, const float* w, const float* bias, cudaStream_t st) {
    BStageArgs a;
    a.x = x;
    a.ldx = K;
    a.K = K;
    a.B = b->B;
    a.norm = norm;
    a.norm_w = w;
    a.norm_b = bias;
    a.eps = b->w->eps;
    a.xh = b->xh;
    a.xl = b->xl;
    a.sx = b->sx;
    a.oscale = b->sx + (size_t)b->max_batch * (b->kmax / 16);
    a.np = b->tc ? (b->B + 15) & ~15u : 0u;
    return launch_bstage(a, st);
}

bool batch_finish(llamini_batch* b, const BPlan& g, u32 seg, const float* part2_src, uint32_t epi,
                  const float* bias, float* out, u32 ldo, unsigned long long* keys, cudaStream_t st) {
    BFinishArgs f;
    f.part = g.part(seg);
    f.part2 = part2_src;
    f.ksplit = g.ksplit();
    f.B = b->B;
    f.rows = g.rows(seg);
    f.oscale = b->sx + (size_t)b->max_batch * (b->kmax / 16);
    f.bias = bias;
    f.epi = epi;
    f.out = out;
    f.ldo = ldo;
    f.keys = keys;
    return launch_bfinish(f, st);
}

bool batch_linear(llamini_batch* b, const DevMat& m, u32 K, float* part, const float* part2_src, uint32_t epi,
                  const float* bias, float* out, u32 ldo, unsigned long long* keys, cudaStream_t st) {
    BPlan g;
    if (!batch_gemm(b, m, K, part, &g)) {
        set_error("batched decode: matrix format %u (%u x %u) has no batched kernel", m.type, m.rows, m.cols);
        return false;
    }
    if (!launch_plan(g, st)) return false;
    BFinishArgs f;
    f.part = part;
    f.part2 = part2_src;
    f.ksplit = g.ksplit();
    f.B = b->B;
    f.rows = m.rows;
    f.oscale = b->sx + (size_t)b->max_batch * (b->kmax / 16);
    f.bias = bias;
    f.epi = epi;
    f.out = out;
    f.ldo = ldo;
    f.keys = keys;
    return launch_bfinish(f, st);
}

bool batch_enqueue_step(llamini_batch* b, cudaStream_t st) {
    llamini_session* s = b->w;
    const bool gpt2 = s->kind == 1;
    const u32 qkvd = s->qd + 2 * s->kvd;
    BEmbedArgs e;
    e.st = b->st;
    e.tokens = b->tokens;
    e.tok_stride = b->max_seq + 1;
    e.tok = s->tok;
    e.pos = s->pos_tab;
    e.scale = s->emb_scale;
    e.hidden = b->hidden;
    e.dim = s->dim;
    if (!launch_bembed(e, b->B, st)) return false;
    const size_t per_seq = batch_cache_bytes_per_seq(b);
    for (u32 l = 0; l < s->n_layers; l++) {
        const llamini_session::Layer& W = s->layers[l];
        if (!batch_stage(b, b->hidden, s->dim, gpt2 ? NORM_LAYER : NORM_RMS, W.n1w, W.n1b, st)) return false;
        if (gpt2) {
            if (!batch_linear(b, W.q, s->dim, b->part, nullptr, EPI_STORE, W.bq, b->qkv, qkvd, nullptr, st)) return false;
        } else {
            // q, k and v share their input: one launch, three partial buffers
            const DevMat* mm[3] = {&W.q, &W.k, &W.v};
            float* pp[3] = {b->part, b->part2, b->part3};
            BPlan g;
            if (!batch_gemm(b, mm, pp, 3, s->dim, &g)) {
                set_error("batched decode: q/k/v formats have no batched kernel");
                return false;
            }
            if (!launch_plan(g, st) ||
                !batch_finish(b, g, 0, nullptr, EPI_STORE, W.bq, b->qkv, qkvd, nullptr, st) ||
                !batch_finish(b, g, 1, nullptr, EPI_STORE, W.bk, b->qkv + s->qd, qkvd, nullptr, st) ||
                !batch_finish(b, g, 2, nullptr, EPI_STORE, W.bv, b->qkv + s->qd + s->kvd, qkvd, nullptr, st))
                return false;
        }
        AttnArgs at;
        at.st = b->st;
        at.qkv = b->qkv;
        at.kc = (uint8_t*)b->kc + (size_t)l * b->max_batch * per_seq;
        at.vc = (uint8_t*)b->vc + (size_t)l * b->max_batch * per_seq;
        at.kv_f16 = b->kv_f16;
        at.out = b->attn;
        at.part = b->apart;
        at.counter = b->counters;
        at.n_heads = s->n_heads;
        at.n_kv = s->n_kv;
        at.hd = s->hd;
        at.max_seq = b->max_seq;
        at.n_split = b->n_split;
        at.rope = s->rope_mode;
        at.theta = s->theta;
        AttnBatch ab;
        ab.qkv_stride = qkvd;
        ab.cache_stride = per_seq;
        ab.out_stride = s->qd;
        ab.part_stride = (uint64_t)s->n_heads * b->n_split * (s->hd + 4);
        if (!launch_attention_batch(at, ab, b->B, st)) return false;
        if (!batch_stage(b, b->attn, s->qd, NORM_NONE, nullptr, nullptr, st) ||
            !batch_linear(b, W.o, s->qd, b->part, nullptr, EPI_RESID, W.bo, b->hidden, s->dim, nullptr, st))
            return false;
        if (!batch_stage(b, b->hidden, s->dim, gpt2 ? NORM_LAYER : NORM_RMS, W.n2w, W.n2b, st)) return false;
        if (gpt2) {
            if (!batch_linear(b, W.up, s->dim, b->part, nullptr, EPI_GELU, W.bup, b->ffn_h, s->ffn, nullptr, st))
                return false;
        } else {
            // gate and up in one launch; the finish combines act(gate) * up (model.c:14-25)
            const DevMat* mm[2] = {&W.gate, &W.up};
            float* pp[2] = {b->part, b->part2};
            BPlan g;
            if (!batch_gemm(b, mm, pp, 2, s->dim, &g)) {
                set_error("batched decode: gate/up formats have no batched kernel");
                return false;
            }
            if (!launch_plan(g, st) ||
                !batch_finish(b, g, 0, b->part2, s->act_gelu ? (u32)EPI_GLU_GELU : (u32)EPI_GLU_SILU, nullptr,
                              b->ffn_h, s->ffn, nullptr, st))
                return false;
        }
        if (!batch_stage(b, b->ffn_h, s->ffn, NORM_NONE, nullptr, nullptr, st) ||
            !batch_linear(b, W.down, s->ffn, b->part, nullptr, EPI_RESID, W.bdown, b->hidden, s->dim, nullptr, st))
            return false;
    }
    if (!batch_stage(b, b->hidden, s->dim, gpt2 ? NORM_LAYER : NORM_RMS, s->fnw, s->fnb, st) ||
        !batch_linear(b, s->head, s->dim, b->part, nullptr, EPI_STORE, nullptr, b->logits, s->vocab, b->keys, st))
        return false;
    BTokenArgs t;
    t.st = b->st;
    t.tokens = b->tokens;
    t.tok_stride = b->max_seq + 1;
    t.n_prompt = b->n_prompt;
    t.keys = b->keys;
    t.B = b->B;
    t.max_tokens = b->max_seq + 1;
    return launch_btoken(t, st);
}

// The step on the tensor-core GEMM: q, k and v finish in one launch, and the
// inputs are staged in the tensor-core layout.
bool batch_enqueue_step_tc(llamini_batch* b, cudaStream_t st) {
    llamini_session* s = b->w;
    const bool gpt2 = s->kind == 1;
    const u32 qkvd = s->qd + 2 * s->kvd;
    const u32 L = s->n_layers;
    float* osc = b->sx + (size_t)b->max_batch * (b->kmax / 16);
    BEmbedArgs e;
    e.st = b->st;
    e.tokens = b->tokens;
    e.tok_stride = b->max_seq + 1;
    e.tok = s->tok;
    e.pos = s->pos_tab;
    e.scale = s->emb_scale;
    e.hidden = b->hidden;
    e.dim = s->dim;
    if (!launch_bembed(e, b->B, st)) return false;
    const u32 norm = gpt2 ? NORM_LAYER : NORM_RMS;
    auto stage_args = [&](u32 K, u32 nm, const float* w, const float* bias) {
        BStageArgs a;
        a.K = K;
        a.B = b->B;
        a.norm = nm;
        a.norm_w = w;
        a.norm_b = bias;
        a.eps = s->eps;
        a.xh = b->xh;
        a.xl = b->xl;
        a.sx = b->sx;
        a.oscale = osc;
        a.np = (b->B + 15) & ~15u;
        return a;
    };
    auto fin_args = [&](const BPlan& g, u32 seg, const float* part2, u32 epi, const float* bias, float* out, u32 ldo) {
        BFinishArgs f;
        f.part = g.part(seg);
        f.part2 = part2;
        f.ksplit = g.ksplit();
        f.B = b->B;
        f.rows = g.rows(seg);
        f.oscale = osc;
        f.bias = bias;
        f.epi = epi;
        f.out = out;
        f.ldo = ldo;
        return f;
    };
    auto gemm = [&](const DevMat* const* mm, float* const* pp, u32 n, u32 K, BPlan* g) -> bool {
        if (!batch_gemm(b, mm, pp, n, K, g)) {
            set_error("batched decode: matrix format %u (%u x %u) has no batched kernel", mm[0]->type, mm[0]->rows, mm[0]->cols);
            return false;
        }
        return launch_plan(*g, st);
    };
    // finish (grid over rows x sequences), then stage the finished rows for the
    // next matrix (one 1024-thread CTA per sequence)
    auto finstage = [&](const BFinishArgs& f, u32 nm, const float* w, const float* bias) {
        if (!launch_bfinish(f, st)) return false;
        BStageArgs a = stage_args(f.rows, nm, w, bias);
        a.x = f.out;
        a.ldx = f.ldo;
        return launch_bstage(a, st);
    };
    {
        BStageArgs a = stage_args(s->dim, norm, s->layers[0].n1w, s->layers[0].n1b);
        a.x = b->hidden;
        a.ldx = s->dim;
        if (!launch_bstage(a, st)) return false;
    }
    const size_t per_seq = batch_cache_bytes_per_seq(b);
    for (u32 l = 0; l < L; l++) {
        const llamini_session::Layer& W = s->layers[l];
        BPlan g;
        if (gpt2) {
            const DevMat* mm[1] = {&W.q};
            float* pp[1] = {b->part};
            if (!gemm(mm, pp, 1, s->dim, &g) || !launch_bfinish(fin_args(g, 0, nullptr, EPI_STORE, W.bq, b->qkv, qkvd), st))
                return false;
        } else {
            const DevMat* mm[3] = {&W.q, &W.k, &W.v};
            float* pp[3] = {b->part, b->part2, b->part3};
            if (!gemm(mm, pp, 3, s->dim, &g)) return false;
            BFinishArgs f = fin_args(g, 0, nullptr, EPI_STORE, W.bq, b->qkv, qkvd);
            f.part_b = g.part(1);
            f.part_c = g.part(2);
            f.rows_b = g.rows(1);
            f.rows_c = g.rows(2);
            f.bias_b = W.bk;
            f.bias_c = W.bv;
            if (!launch_bfinish(f, st)) return false;
        }
        AttnArgs at;
        at.st = b->st;
        at.qkv = b->qkv;
        at.kc = (uint8_t*)b->kc + (size_t)l * b->max_batch * per_seq;
        at.vc = (uint8_t*)b->vc + (size_t)l * b->max_batch * per_seq;
        at.kv_f16 = b->kv_f16;
        at.out = b->attn;
        at.part = b->apart;
        at.counter = b->counters;
        at.n_heads = s->n_heads;
        at.n_kv = s->n_kv;
        at.hd = s->hd;
        at.max_seq = b->max_seq;
        at.n_split = b->n_split;
        at.rope = s->rope_mode;
        at.theta = s->theta;
        AttnBatch ab;
        ab.qkv_stride = qkvd;
        ab.cache_stride = per_seq;
        ab.out_stride = s->qd;
        ab.part_stride = (uint64_t)s->n_heads * b->n_split * (s->hd + 4);
        if (!launch_attention_batch(at, ab, b->B, st)) return false;
        {
            BStageArgs a = stage_args(s->qd, NORM_NONE, nullptr, nullptr);
            a.x = b->attn;
            a.ldx = s->qd;
            if (!launch_bstage(a, st)) return false;
        }
        // the residual add, then the next matrix's staging; in a tensor-parallel
        // group the ranks' partial sums first go through the wide allreduce
        auto resid = [&](const BPlan& gg, const float* bias, const float* nw, const float* nb) {
            if (s->tp_world == 1) return finstage(fin_args(gg, 0, nullptr, EPI_RESID, bias, b->hidden, s->dim), norm, nw, nb);
            if (!launch_bfinish(fin_args(gg, 0, nullptr, EPI_STORE, tp().rank == 0 ? bias : nullptr, b->tp_part, s->dim), st) ||
                !launch_tp_allreduce_wide(b->tp_part, b->hidden, b->B * s->dim, b->err, st))
                return false;
            BStageArgs a = stage_args(s->dim, norm, nw, nb);
            a.x = b->hidden;
            a.ldx = s->dim;
            return launch_bstage(a, st);
        };
        {
            const DevMat* mm[1] = {&W.o};
            float* pp[1] = {b->part};
            if (!gemm(mm, pp, 1, s->qd, &g) || !resid(g, W.bo, W.n2w, W.n2b)) return false;
        }
        if (gpt2) {
            const DevMat* mm[1] = {&W.up};
            float* pp[1] = {b->part};
            if (!gemm(mm, pp, 1, s->dim, &g) ||
                !finstage(fin_args(g, 0, nullptr, EPI_GELU, W.bup, b->ffn_h, s->ffn), NORM_NONE, nullptr, nullptr))
                return false;
        } else {
            const DevMat* mm[2] = {&W.gate, &W.up};
            float* pp[2] = {b->part, b->part2};
            const u32 epi = s->act_gelu ? (u32)EPI_GLU_GELU : (u32)EPI_GLU_SILU;
            if (!gemm(mm, pp, 2, s->dim, &g) ||
                !finstage(fin_args(g, 0, g.part(1), epi, nullptr, b->ffn_h, s->ffn), NORM_NONE, nullptr, nullptr))
                return false;
        }
        {
            const DevMat* mm[1] = {&W.down};
            float* pp[1] = {b->part};
            const float* nw = l + 1 < L ? s->layers[l + 1].n1w : s->fnw;
            const float* nb = l + 1 < L ? s->layers[l + 1].n1b : s->fnb;
            if (!gemm(mm, pp, 1, s->ffn, &g) || !resid(g, W.bdown, nw, nb)) return false;
        }
    }
    {
        const DevMat* mm[1] = {&s->head};
        float* pp[1] = {b->part};
        BPlan g;
        BFinishArgs f;
        if (!gemm(mm, pp, 1, s->dim, &g)) return false;
        f = fin_args(g, 0, nullptr, EPI_STORE, nullptr, b->logits, s->vocab);
        f.keys = b->keys;
        if (!launch_bfinish(f, st)) return false;
    }
    BTokenArgs t;
    t.st = b->st;
    t.tokens = b->tokens;
    t.tok_stride = b->max_seq + 1;
    t.n_prompt = b->n_prompt;
    t.keys = b->keys;
    t.B = b->B;
    t.max_tokens = b->max_seq + 1;
    return launch_btoken(t, st);
}

bool batch_capture(llamini_batch* b, u32 steps, cudaGraphExec_t* out) {
    cudaStream_t st = stream();
    cudaGraph_t g = nullptr;
    if (!LM_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal))) return false;
    bool ok = true;
    for (u32 i = 0; i < steps && ok; i++) ok = b->tc ? batch_enqueue_step_tc(b, st) : batch_enqueue_step(b, st);
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (!ok || !LM_CUDA(e)) { if (g) cudaGraphDestroy(g); return false; }
    ok = LM_CUDA(cudaGraphInstantiate(out, g, 0));
    cudaGraphDestroy(g);
    return ok;
}

void batch_destroy(llamini_batch* b) {
    if (!b) return;
    cudaStreamSynchronize(stream());
    if (b->g_one) cudaGraphExecDestroy(b->g_one);
    if (b->g_many) cudaGraphExecDestroy(b->g_many);
    destroy(b->w);
    delete b;
}

// Buffers for max_batch sequences; the GEMM plans (and so the partial-sum
// buffer) are sized for the largest batch.
bool batch_alloc(llamini_batch* b) {
    llamini_session* s = b->w;
    const u32 MB = b->max_batch;
    b->kmax = s->dim;
    if (s->qd > b->kmax) b->kmax = s->qd;
    if (s->ffn > b->kmax) b->kmax = s->ffn;
    b->kmax = (b->kmax + 255) & ~255u;
    b->kv_f16 = g_kv_f16 ? 1u : 0u;
    b->tc = batch_tc();
    b->err = (u32*)own(s, 4);
    if (!b->err || !LM_CUDA(cudaMemset(b->err, 0, 4))) return false;
    const u32 hb = s->n_heads * MB;
    u32 ns = (u32)(2 * sm_count()) / (hb ? hb : 1);
    if (ns < 1) ns = 1;
    if (ns > 32) ns = 32;
    const u32 by_len = (b->max_seq + 63) / 64;
    if (ns > by_len) ns = by_len;
    b->n_split = ns ? ns : 1;
    // partial sums: the largest plan over the step's matrices at the full batch
    b->B = MB;
    size_t pmax = 0;
    auto need = [&](const DevMat* const* mm, u32 n, u32 K) -> bool {
        float* none[3] = {nullptr, nullptr, nullptr};
        BPlan g;
        if (!batch_gemm(b, mm, none, n, K, &g)) {
            set_error("batched decode: matrix format %u (%u x %u) has no batched kernel", mm[0]->type, mm[0]->rows,
                      mm[0]->cols);
            return false;
        }
        for (u32 i = 0; i < n; i++) {
            const size_t m = (size_t)g.ksplit() * MB * mm[i]->rows;
            pmax = pmax > m ? pmax : m;
        }
        return true;
    };
    auto need1 = [&](const DevMat& m, u32 K) -> bool {
        const DevMat* mm[1] = {&m};
        return need(mm, 1, K);
    };
    auto plan_all = [&]() -> bool {
        bool ok = need1(s->head, s->dim);
        for (u32 l = 0; ok && l < s->n_layers; l++) {
            const auto& W = s->layers[l];
            ok = need1(W.o, s->qd) && need1(W.down, s->ffn);
            if (ok && s->kind == 1) ok = need1(W.q, s->dim) && need1(W.up, s->dim);
            if (ok && s->kind == 0) {
                const DevMat* qkv[3] = {&W.q, &W.k, &W.v};
                const DevMat* gu[2] = {&W.gate, &W.up};
                ok = need(qkv, 3, s->dim) && need(gu, 2, s->dim);
            }
        }
        return ok;
    };
    // rows of a size that is not a multiple of 16 bytes (Q6_K at some widths):
    // copies with a 16-byte row pitch, so the tensor-core GEMM can load by TMA
    if (b->tc && !make_pitched_all(s, b->pitched)) return false;
    if (!plan_all()) {
        // a shape the tensor-core GEMM does not take: the whole batch on mma.sync
        if (!b->tc) return false;
        b->tc = false;
        pmax = 0;
        if (!plan_all()) return false;
    }
    b->part_floats = pmax;
    const size_t per_seq = batch_cache_bytes_per_seq(b);
    const size_t cache = (size_t)s->n_layers * MB * per_seq;
    b->hidden = (float*)own(s, (size_t)MB * s->dim * 4);
    b->qkv = (float*)own(s, (size_t)MB * (s->qd + 2 * s->kvd) * 4);
    b->attn = (float*)own(s, (size_t)MB * s->qd * 4);
    b->ffn_h = (float*)own(s, (size_t)MB * s->ffn * 4);
    b->logits = (float*)own(s, (size_t)MB * s->vocab * 4);
    const size_t xcols = ((size_t)MB + 15) & ~size_t(15);         // the tensor-core layout pads the batch to 16
    b->xh = (uint16_t*)own(s, tg_xh_halves(b->kmax, xcols) * 2);
    b->xl = (uint16_t*)own(s, xcols * b->kmax * 2);
    b->sx = (float*)own(s, ((size_t)MB * (b->kmax / 16) + MB) * 4);
    b->part = (float*)own(s, pmax * 4);
    b->part2 = (float*)own(s, pmax * 4);
    b->part3 = (float*)own(s, pmax * 4);
    b->apart = (float*)own(s, (size_t)MB * s->n_heads * b->n_split * (s->hd + 4) * 4);
    b->counters = (u32*)own(s, (size_t)MB * s->n_heads * 4);
    b->tokens = (u32*)own(s, (size_t)MB * (b->max_seq + 1) * 4);
    b->n_prompt = (u32*)own(s, (size_t)MB * 4);
    b->keys = (unsigned long long*)own(s, (size_t)MB * 8);
    b->kc = own(s, cache);
    b->vc = own(s, cache);
    b->st = (StepState*)own(s, sizeof(StepState));
    if (s->tp_world > 1 && !(b->tp_part = (float*)own(s, (size_t)MB * s->dim * 4))) return false;
    if (!b->hidden || !b->qkv || !b->attn || !b->ffn_h || !b->logits || !b->xh || !b->xl || !b->sx || !b->part ||
        !b->part2 || !b->part3 || !b->apart || !b->counters || !b->tokens || !b->n_prompt || !b->keys || !b->kc || !b->vc || !b->st)
        return false;
    return LM_CUDA(cudaMemset(b->counters, 0, (size_t)MB * s->n_heads * 4)) &&
           LM_CUDA(cudaMemset(b->keys, 0, (size_t)MB * 8)) && LM_CUDA(cudaMemset(b->st, 0, sizeof(StepState))) &&
           LM_CUDA(cudaMemset(b->tokens, 0, (size_t)MB * (b->max_seq + 1) * 4)) &&
           LM_CUDA(cudaMemset(b->kc, 0, cache)) && LM_CUDA(cudaMemset(b->vc, 0, cache));
}

template <class M, class Bind>
llamini_batch* batch_create(M* model, u32 max_batch, u32 max_seq, Bind bind) {
    if (!ensure_device()) return nullptr;
    if (max_batch == 0 || max_batch > 64) { set_error("batched decode: batch %u outside 1..64", max_batch); return nullptr; }
    if (max_seq == 0) { set_error("batched decode: max_seq 0"); return nullptr; }
    auto* b = new llamini_batch();
    b->w = new llamini_session();
    b->max_batch = max_batch;
    b->max_seq = max_seq;
    if (!bind(b->w, model, max_seq)) { batch_destroy(b); return nullptr; }
    // a tensor-parallel group: LLaMA-family models (the shards bind_llama cuts)
    // on the tensor-core GEMM, the batch's columns allreduced after o and down
    if (tp().world > 1 && (b->w->tp_world < 2 || (u64)max_batch * b->w->dim > kTpWideFloats)) {
        set_error("batched decode: a tensor-parallel group takes LLaMA-family batches of at most %u x dim floats",
                  kTpWideFloats);
        batch_destroy(b);
        return nullptr;
    }
    if (!batch_alloc(b)) { batch_destroy(b); return nullptr; }
    if (b->w->tp_world > 1 && !b->tc) {
        set_error("batched decode: a tensor-parallel group needs the tensor-core GEMM");
        batch_destroy(b);
        return nullptr;
    }
    b->B = 0;
    return b;
}

// After a synchronize: false (error set) when a tensor-core GEMM of the steps
// run so far reported a failure.
bool batch_ok(llamini_batch* b) {
    if (!b->tc) return true;
    u32 e = 0;
    if (!LM_CUDA(cudaMemcpy(&e, b->err, 4, cudaMemcpyDeviceToHost))) return false;
    if (e == 0) return true;
    set_error("batched decode: tensor-core GEMM: %s", (e & 1u) ? "a pipeline wait ran out" : "a weight outside the fp16 range");
    return false;
}

// ---------------------------------------------------------------- prefill
//
// Prompt positions in chunks of kPfChunk: per layer the staging, tensor-core
// GEMMs and finishes of batched decode with the chunk's positions as columns,
// RoPE and cache writes for the chunk (prope), causal attention over the cache
// (pattn). Used for the prompt positions whose logits the caller does not read
// (generate_autoregressive's prefill, session steps inside the prompt).

constexpr u32 kPfChunk = 64;
int g_prefill = -1;                   // llamini_set_prefill: -1 default (on unless LLAMINI_PREFILL=0)

bool prefill_enabled() {
    static const bool env_on = [] { const char* e = getenv("LLAMINI_PREFILL"); return !(e && e[0] == '0'); }();
    return g_prefill >= 0 ? g_prefill == 1 : env_on;
}

// Build the session's prefill buffers (false, no error: not available).
bool prefill_build(llamini_session* s) {
    if (s->pf_state) return s->pf_state > 0;
    s->pf_state = -1;
    if ((s->kind != 0 && s->kind != 1) || (s->tp_world > 1 && (s->kind != 0 || (u64)kPfChunk * s->dim > kTpWideFloats)))
        return false;
    Prefill* pf = new Prefill();
    s->pf = pf;
    if (!make_pitched_all(s, pf->pitched)) return false;
    u32 kmax = s->dim;
    if (s->qd > kmax) kmax = s->qd;
    if (s->ffn > kmax) kmax = s->ffn;
    // partial sums: the largest plan over the step's matrices with full chunks
    size_t pmax = 0;
    auto need = [&](const DevMat* const* mm, u32 n, u32 K) -> bool {
        float* none[3] = {nullptr, nullptr, nullptr};
        TGemmArgs g;
        if (!plan_tc(nullptr, nullptr, kPfChunk, nullptr, pf->pitched, mm, none, n, K, &g)) return false;
        for (u32 i = 0; i < n; i++) {
            const size_t m = (size_t)g.ksplit * kPfChunk * mm[i]->rows;
            pmax = pmax > m ? pmax : m;
        }
        return true;
    };
    bool ok = true;
    for (u32 l = 0; ok && l < s->n_layers; l++) {
        const auto& W = s->layers[l];
        const DevMat* o1[1] = {&W.o};
        const DevMat* d1[1] = {&W.down};
        ok = need(o1, 1, s->qd) && need(d1, 1, s->ffn);
        if (ok && s->kind == 1) {
            const DevMat* q1[1] = {&W.q};
            const DevMat* u1[1] = {&W.up};
            ok = need(q1, 1, s->dim) && need(u1, 1, s->dim);
        } else if (ok) {
            const DevMat* qkv[3] = {&W.q, &W.k, &W.v};
            const DevMat* gu[2] = {&W.gate, &W.up};
            ok = need(qkv, 3, s->dim) && need(gu, 2, s->dim);
        }
    }
    if (!ok) return false;                                  // a format or shape the GEMM does not take
    const u32 qkvd = s->qd + 2 * s->kvd, C = kPfChunk;
    pf->hidden = (float*)own(s, (size_t)C * s->dim * 4);
    pf->qkv = (float*)own(s, (size_t)C * qkvd * 4);
    pf->attn = (float*)own(s, (size_t)C * s->qd * 4);
    pf->ffn_h = (float*)own(s, (size_t)C * s->ffn * 4);
    pf->osc = (float*)own(s, (size_t)C * 4);
    pf->xh = (uint16_t*)own(s, tg_xh_halves(kmax, C) * 2);
    pf->xl = (uint16_t*)own(s, (size_t)C * kmax * 2);
    pf->part = (float*)own(s, pmax * 4);
    pf->part2 = (float*)own(s, pmax * 4);
    pf->part3 = (float*)own(s, pmax * 4);
    pf->err = (uint32_t*)own(s, 4);
    if (s->tp_world > 1 && !(pf->tp_part = (float*)own(s, (size_t)C * s->dim * 4))) return false;
    if (!pf->hidden || !pf->qkv || !pf->attn || !pf->ffn_h || !pf->osc || !pf->xh || !pf->xl || !pf->part ||
        !pf->part2 || !pf->part3 || !pf->err || !LM_CUDA(cudaMemset(pf->err, 0, 4)))
        return false;
    s->pf_state = 1;
    return true;
}

// The columns of a prefill chunk: cp consecutive positions of each of ns
// sequences (column i * cp + j is position p0 + j of sequence i), with where
// their tokens and cache rows live.
struct PfCols {
    const u32* tokens = nullptr;          // sequence i's tokens at tokens + i * tok_stride
    u32 tok_stride = 0;
    void *kc = nullptr, *vc = nullptr;    // layer 0 of sequence 0
    size_t layer_bytes = 0;               // from one layer's cache to the next
    size_t seq_bytes = 0;                 // from one sequence's cache to the next (same layer)
    u32 ns = 1, cp = 0, kv_f16 = 0, max_seq = 0;
};

// A single session's chunk of C positions.
PfCols session_cols(const llamini_session* s, u32 C) {
    PfCols c;
    c.tokens = s->tokens;
    c.kc = s->kc;
    c.vc = s->vc;
    c.layer_bytes = (size_t)s->n_kv * s->max_seq * s->hd * (s->kv_f16 ? 2 : 4);
    c.cp = C;
    c.kv_f16 = s->kv_f16;
    c.max_seq = s->max_seq;
    return c;
}

// The chunk's positions p0 .. p0 + cp - 1 of each of its sequences through
// every layer (their cache rows written); with `score` (one sequence), also
// the final norm, lm_head and the log-prob of each scored position's next
// token (positions up to `last`) into pf->lp.
bool prefill_chunk(llamini_session* s, const PfCols& cols, u32 p0, cudaStream_t st, bool score = false,
                   u32 last = 0) {
    Prefill* pf = s->pf;
    const bool gpt2 = s->kind == 1;
    const u32 qkvd = s->qd + 2 * s->kvd, L = s->n_layers;
    const u32 norm = gpt2 ? NORM_LAYER : NORM_RMS;
    const u32 C = cols.ns * cols.cp;
    const u32 np = (C + 15) & ~15u;
    const uint64_t seq_elems = cols.seq_bytes / (cols.kv_f16 ? 2 : 4);
    if (C == 0 || C > kPfChunk || (score && cols.ns != 1)) {
        set_error("prefill: a chunk of %u x %u columns", cols.ns, cols.cp);
        return false;
    }
    PEmbedArgs e;
    e.tokens = cols.tokens;
    e.p0 = p0;
    e.C = C;
    e.cp = cols.cp;
    e.tok_stride = cols.tok_stride;
    e.tok = s->tok;
    e.pos = s->pos_tab;
    e.scale = s->emb_scale;
    e.hidden = pf->hidden;
    e.dim = s->dim;
    if (!launch_pembed(e, st)) return false;
    auto stage = [&](const float* x, u32 K, u32 nm, const float* w, const float* bias) {
        BStageArgs a;
        a.x = x;
        a.ldx = K;
        a.K = K;
        a.B = C;
        a.norm = nm;
        a.norm_w = w;
        a.norm_b = bias;
        a.eps = s->eps;
        a.xh = pf->xh;
        a.xl = pf->xl;
        a.oscale = pf->osc;
        a.np = np;
        return launch_bstage(a, st);
    };
    auto gemm = [&](const DevMat* const* mm, float* const* pp, u32 n, u32 K, TGemmArgs* g) -> bool {
        if (!plan_tc(pf->xh, pf->xl, C, pf->err, pf->pitched, mm, pp, n, K, g)) {
            set_error("prefill: matrix format %u (%u x %u) has no tensor-core plan", mm[0]->type, mm[0]->rows, mm[0]->cols);
            return false;
        }
        return launch_tgemm(*g, st);
    };
    auto fin = [&](const TGemmArgs& g, u32 seg, const float* part2, u32 epi, const float* bias, float* out, u32 ldo) {
        BFinishArgs f;
        f.part = g.seg[seg].part;
        f.part2 = part2;
        f.ksplit = g.ksplit;
        f.B = C;
        f.rows = g.seg[seg].rows;
        f.oscale = pf->osc;
        f.bias = bias;
        f.epi = epi;
        f.out = out;
        f.ldo = ldo;
        return f;
    };
    for (u32 l = 0; l < L; l++) {
        const llamini_session::Layer& W = s->layers[l];
        TGemmArgs g;
        if (!stage(pf->hidden, s->dim, norm, W.n1w, W.n1b)) return false;
        if (gpt2) {
            const DevMat* mm[1] = {&W.q};
            float* pp[1] = {pf->part};
            if (!gemm(mm, pp, 1, s->dim, &g) || !launch_bfinish(fin(g, 0, nullptr, EPI_STORE, W.bq, pf->qkv, qkvd), st))
                return false;
        } else {
            const DevMat* mm[3] = {&W.q, &W.k, &W.v};
            float* pp[3] = {pf->part, pf->part2, pf->part3};
            if (!gemm(mm, pp, 3, s->dim, &g)) return false;
            BFinishArgs f = fin(g, 0, nullptr, EPI_STORE, W.bq, pf->qkv, qkvd);
            f.part_b = g.seg[1].part;
            f.part_c = g.seg[2].part;
            f.rows_b = g.seg[1].rows;
            f.rows_c = g.seg[2].rows;
            f.bias_b = W.bk;
            f.bias_c = W.bv;
            if (!launch_bfinish(f, st)) return false;
        }
        void* kc = (uint8_t*)cols.kc + l * cols.layer_bytes;
        void* vc = (uint8_t*)cols.vc + l * cols.layer_bytes;
        PRopeArgs r;
        r.qkv = pf->qkv;
        r.qkv_stride = qkvd;
        r.kc = kc;
        r.vc = vc;
        r.kv_f16 = cols.kv_f16;
        r.n_heads = s->n_heads;
        r.n_kv = s->n_kv;
        r.hd = s->hd;
        r.max_seq = cols.max_seq;
        r.p0 = p0;
        r.rope = s->rope_mode;
        r.cp = cols.cp;
        r.seq_elems = seq_elems;
        r.theta = s->theta;
        if (!launch_prope(r, C, st)) return false;
        PAttnArgs at;
        at.qkv = pf->qkv;
        at.qkv_stride = qkvd;
        at.kc = kc;
        at.vc = vc;
        at.kv_f16 = cols.kv_f16;
        at.out = pf->attn;
        at.out_stride = s->qd;
        at.n_heads = s->n_heads;
        at.n_kv = s->n_kv;
        at.hd = s->hd;
        at.max_seq = cols.max_seq;
        at.p0 = p0;
        at.C = C;
        at.cp = cols.cp;
        at.seq_elems = seq_elems;
        if (!launch_pattn(at, st)) return false;
        // the residual adds after o and down; in a tensor-parallel group the
        // ranks' partial sums are added by the wide allreduce (bias on rank 0)
        auto resid = [&](const TGemmArgs& gg, const float* bias) {
            if (s->tp_world == 1) return launch_bfinish(fin(gg, 0, nullptr, EPI_RESID, bias, pf->hidden, s->dim), st);
            return launch_bfinish(fin(gg, 0, nullptr, EPI_STORE, tp().rank == 0 ? bias : nullptr, pf->tp_part, s->dim), st) &&
                   launch_tp_allreduce_wide(pf->tp_part, pf->hidden, C * s->dim, pf->err, st);
        };
        {
            const DevMat* mm[1] = {&W.o};
            float* pp[1] = {pf->part};
            if (!stage(pf->attn, s->qd, NORM_NONE, nullptr, nullptr) || !gemm(mm, pp, 1, s->qd, &g) || !resid(g, W.bo))
                return false;
        }
        if (!stage(pf->hidden, s->dim, norm, W.n2w, W.n2b)) return false;
        if (gpt2) {
            const DevMat* mm[1] = {&W.up};
            float* pp[1] = {pf->part};
            if (!gemm(mm, pp, 1, s->dim, &g) || !launch_bfinish(fin(g, 0, nullptr, EPI_GELU, W.bup, pf->ffn_h, s->ffn), st))
                return false;
        } else {
            const DevMat* mm[2] = {&W.gate, &W.up};
            float* pp[2] = {pf->part, pf->part2};
            const u32 epi = s->act_gelu ? (u32)EPI_GLU_GELU : (u32)EPI_GLU_SILU;
            if (!gemm(mm, pp, 2, s->dim, &g) || !launch_bfinish(fin(g, 0, g.seg[1].part, epi, nullptr, pf->ffn_h, s->ffn), st))
                return false;
        }
        {
            const DevMat* mm[1] = {&W.down};
            float* pp[1] = {pf->part};
            if (!stage(pf->ffn_h, s->ffn, NORM_NONE, nullptr, nullptr) || !gemm(mm, pp, 1, s->ffn, &g) ||
                !resid(g, W.bdown))
                return false;
        }
    }
    if (score) {
        // final norm + lm_head (head_args' matrix) for every position, then the
        // next token's log-prob (generate.c:176-188, gpt2.c:240-250)
        TGemmArgs g;
        const DevMat* mm[1] = {&s->head};
        float* pp[1] = {pf->hpart};
        if (!stage(pf->hidden, s->dim, norm, s->fnw, s->fnb) || !gemm(mm, pp, 1, s->dim, &g) ||
            !launch_bfinish(fin(g, 0, nullptr, EPI_STORE, nullptr, pf->logits, s->vocab), st))
            return false;
        PNllArgs n;
        n.logits = pf->logits;
        n.vocab = s->vocab;
        n.ld = s->vocab;
        n.tokens = cols.tokens;
        n.p0 = p0;
        n.C = C;
        n.last = last;
        n.lp = pf->lp;
        if (!launch_pnll(n, st)) return false;
    }
    return true;
}

// Buffers of teacher-forced scoring (false, no error: the lm_head has no
// tensor-core plan, e.g. a K-quant head whose width is not a multiple of 256).
bool prefill_head_build(llamini_session* s) {
    Prefill* pf = s->pf;
    if (pf->head_state) return pf->head_state > 0;
    pf->head_state = -1;
    const DevMat* mm[1] = {&s->head};
    float* none[3] = {nullptr, nullptr, nullptr};
    TGemmArgs g;
    if (!plan_tc(nullptr, nullptr, kPfChunk, nullptr, pf->pitched, mm, none, 1, s->dim, &g)) return false;
    pf->hpart = (float*)own(s, (size_t)g.ksplit * kPfChunk * s->vocab * 4);
    pf->logits = (float*)own(s, (size_t)kPfChunk * s->vocab * 4);
    pf->lp = (float*)own(s, (size_t)(s->max_pos + 1) * 4);
    if (!pf->hpart || !pf->logits || !pf->lp) return false;
    pf->head_state = 1;
    return true;
}

// compute_perplexity's positions 0 .. steps - 1 in chunks (tokens on the device,
// state at position 0); *nll = the sum of -log p(next token) in position order.
// 1 done, 0 the chunked path is not available (nothing ran), -1 failed (error set).
int prefill_perplexity(llamini_session* s, u32 steps, double* nll) {
    if (s->trace_on || !prefill_enabled() || !prefill_build(s) || !prefill_head_build(s)) return 0;
    cudaStream_t st = stream();
    for (u32 done = 0; done < steps;) {
        const u32 C = steps - done < kPfChunk ? steps - done : kPfChunk;
        if (!prefill_chunk(s, session_cols(s, C), done, st, true, steps - 1)) return -1;
        done += C;
    }
    std::vector<float> lp(steps);
    uint32_t e = 0;
    if (!LM_CUDA(cudaMemcpyAsync(lp.data(), s->pf->lp, (size_t)steps * 4, cudaMemcpyDeviceToHost, st)) ||
        !LM_CUDA(cudaMemcpyAsync(&e, s->pf->err, 4, cudaMemcpyDeviceToHost, st)) || !LM_CUDA(cudaStreamSynchronize(st)))
        return -1;
    if (e) {
        set_error("prefill: tensor-core GEMM: %s", (e & 1u) ? "a pipeline wait ran out" : "a weight outside the fp16 range");
        return -1;
    }
    double sum = 0.0;
    for (u32 i = 0; i < steps; i++) sum += -(double)lp[i];
    *nll = sum;
    s->pos = steps;
    s->st_host->pos = s->pos;
    return LM_CUDA(cudaMemcpyAsync(&s->st->pos, &s->st_host->pos, 4, cudaMemcpyHostToDevice, st)) &&
                   LM_CUDA(cudaStreamSynchronize(st)) ? 1 : -1;
}

bool run_prompt(llamini_session* s, u32 n) {
    if (n < 2 || s->trace_on || !prefill_enabled() || !prefill_build(s)) return run_steps(s, n);
    if ((u64)s->pos + n > s->max_pos) {
        set_error("position %u + %u steps passes the cache capacity %u", s->pos, n, s->max_pos);
        return false;
    }
    cudaStream_t st = stream();
    for (u32 done = 0; done < n;) {
        const u32 C = n - done < kPfChunk ? n - done : kPfChunk;
        if (!prefill_chunk(s, session_cols(s, C), s->pos + done, st)) return false;
        done += C;
    }
    // the decode steps continue at the position after the prompt chunk
    if (!LM_CUDA(cudaStreamSynchronize(st))) return false;
    uint32_t e = 0;
    if (!LM_CUDA(cudaMemcpy(&e, s->pf->err, 4, cudaMemcpyDeviceToHost))) return false;
    if (e) {
        set_error("prefill: tensor-core GEMM: %s", (e & 1u) ? "a pipeline wait ran out" : "a weight outside the fp16 range");
        return false;
    }
    s->pos += n;
    s->st_host->pos = s->pos;
    return LM_CUDA(cudaMemcpyAsync(&s->st->pos, &s->st_host->pos, 4, cudaMemcpyHostToDevice, st)) &&
           LM_CUDA(cudaStreamSynchronize(st));
}

// Lockstep positions pos .. pos + n - 1 of a batch whose next token is still
// every sequence's prompt (no sequence writes a token there): prefill chunks
// of cp positions x ns sequences (64 columns; cp = 64 / B), written into the
// batch's caches. The next lockstep step starts at the position after them.
// (batch_run takes this path for batches of up to 32 sequences.)
bool batch_prefill(llamini_batch* b, u32 n) {
    llamini_session* s = b->w;
    cudaStream_t st = stream();
    const u32 B = b->B, cp = B >= kPfChunk ? 1u : kPfChunk / B, ns_max = kPfChunk / cp;
    const size_t per_seq = batch_cache_bytes_per_seq(b);
    const u32 stride = b->max_seq + 1;
    for (u32 done = 0; done < n;) {
        const u32 c = n - done < cp ? n - done : cp;
        for (u32 i0 = 0; i0 < B; i0 += ns_max) {
            PfCols pc;
            pc.tokens = b->tokens + (size_t)i0 * stride;
            pc.tok_stride = stride;
            pc.kc = (uint8_t*)b->kc + (size_t)i0 * per_seq;
            pc.vc = (uint8_t*)b->vc + (size_t)i0 * per_seq;
            pc.layer_bytes = (size_t)b->max_batch * per_seq;
            pc.seq_bytes = per_seq;
            pc.ns = B - i0 < ns_max ? B - i0 : ns_max;
            pc.cp = c;
            pc.kv_f16 = b->kv_f16;
            pc.max_seq = b->max_seq;
            if (!prefill_chunk(s, pc, b->pos + done, st)) return false;
        }
        done += c;
    }
    if (!LM_CUDA(cudaStreamSynchronize(st))) return false;
    uint32_t e = 0;
    if (!LM_CUDA(cudaMemcpy(&e, s->pf->err, 4, cudaMemcpyDeviceToHost))) return false;
    if (e) {
        set_error("prefill: tensor-core GEMM: %s", (e & 1u) ? "a pipeline wait ran out" : "a weight outside the fp16 range");
        return false;
    }
    b->pos += n;
    const u32 pos = b->pos;
    return LM_CUDA(cudaMemcpy(&b->st->pos, &pos, 4, cudaMemcpyHostToDevice));
}

bool batch_run(llamini_batch* b, u32 n) {
    if ((u64)b->pos + n > b->w->max_pos) {
        set_error("batched decode: position %u + %u steps passes the capacity %u", b->pos, n, b->w->max_pos);
        return false;
    }
    // positions before every sequence's last prompt token: prefill
    u32 common = 0xFFFFFFFFu;
    for (u32 L : b->lens) common = L < common ? L : common;
    u32 pre = b->pos + 1 < common ? common - 1 - b->pos : 0;
    if (pre > n) pre = n;
    // at most 32 sequences (two or more positions per sequence in a chunk):
    // with one position per sequence a chunk reads the weights as often as the
    // lockstep steps, and the lockstep's split attention is the faster one
    if (pre >= 2 && b->B <= kPfChunk / 2 && prefill_enabled() && prefill_build(b->w)) {
        if (!batch_prefill(b, pre)) return false;
        n -= pre;
        if (n == 0) return true;
    }
    cudaStream_t st = stream();
    if (b->plan_B != b->B) {
        if (b->g_one) { cudaGraphExecDestroy(b->g_one); b->g_one = nullptr; }
        if (b->g_many) { cudaGraphExecDestroy(b->g_many); b->g_many = nullptr; }
        if (!batch_capture(b, 1, &b->g_one) || !batch_capture(b, kBatchStepsPerGraph, &b->g_many)) return false;
        b->plan_B = b->B;
    }
    u32 left = n;
    while (left >= kBatchStepsPerGraph) {
        if (!LM_CUDA(cudaGraphLaunch(b->g_many, st))) return false;
        left -= kBatchStepsPerGraph;
    }
    while (left--) if (!LM_CUDA(cudaGraphLaunch(b->g_one, st))) return false;
    b->pos += n;
    return true;
}

}  // namespace
}  // namespace lm

extern "C" {

void forward_step(LLaMAModel* model, KVCache* caches, u32 pos, u32 token_id, f32* logits_out) {
    lm::forward_one(lm::llama_session(model, caches), pos, token_id, logits_out);
}

u32 generate_autoregressive(LLaMAModel* model, KVCache* caches, u32* input_tokens, u32 in_token_count,
                            u32* out_tokens, u32 max_gen_tokens, u32 eos_id, f32 temp, f32 top_p) {
    return lm::generate(lm::llama_session(model, caches), input_tokens, in_token_count, out_tokens,
                        max_gen_tokens, eos_id, temp, top_p);
}

f32 compute_perplexity(LLaMAModel* model, KVCache* caches, const u32* tokens, u32 n_tokens) {
    return lm::perplexity(lm::llama_session(model, caches), tokens, n_tokens);
}

void gpt2_forward_step(GPT2Model* model, KVCache* caches, u32 pos, u32 token_id, f32* logits_out) {
    lm::forward_one(lm::gpt2_session(model, caches), pos, token_id, logits_out);
}

u32 gpt2_generate(GPT2Model* model, KVCache* caches, u32* input_tokens, u32 in_token_count,
                  u32* out_tokens, u32 max_gen_tokens, u32 eos_id, f32 temp, f32 top_p) {
    return lm::generate(lm::gpt2_session(model, caches), input_tokens, in_token_count, out_tokens,
                        max_gen_tokens, eos_id, temp, top_p);
}

f32 gpt2_compute_perplexity(GPT2Model* model, KVCache* caches, const u32* tokens, u32 n_tokens) {
    return lm::perplexity(lm::gpt2_session(model, caches), tokens, n_tokens);
}

llamini_session* llamini_llama_session(LLaMAModel* model, KVCache* caches) { return lm::llama_session(model, caches); }
llamini_session* llamini_gpt2_session(GPT2Model* model, KVCache* caches) { return lm::gpt2_session(model, caches); }

int llamini_session_begin(llamini_session* s, const u32* prompt, u32 n_prompt) {
    if (!s || n_prompt == 0 || n_prompt > s->max_seq) { lm::set_error("session_begin: bad prompt"); return -1; }
    if (!lm::write_state(s, 0, n_prompt, true)) return -1;
    return LM_CUDA(cudaMemcpyAsync(s->tokens, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, lm::stream())) &&
                   LM_CUDA(cudaStreamSynchronize(lm::stream()))
               ? 0 : -1;
}

int llamini_session_step(llamini_session* s, u32 n_steps) {
    if (!s) return -1;
    // positions whose next token is still the prompt's produce no token: prefill
    u32 pre = s->pos + 1 < s->n_prompt ? s->n_prompt - 1 - s->pos : 0;
    if (pre > n_steps) pre = n_steps;
    if (pre && !lm::run_prompt(s, pre)) return -1;
    return lm::run_steps(s, n_steps - pre) ? 0 : -1;
}

int llamini_session_prefill(llamini_session* s) { return s ? s->pf_state : -2; }

int llamini_set_prefill(int enable) {
    if (enable < -1 || enable > 1) { lm::set_error("prefill setting %d outside -1..1", enable); return -1; }
    lm::g_prefill = enable;
    return 0;
}

int llamini_session_tokens(llamini_session* s, u32* out, u32 n) {
    if (!s) return -1;
    const u32 valid = s->pos + 1 > s->n_prompt ? s->pos + 1 : s->n_prompt;
    const u32 k = n < valid ? n : valid;
    if (!LM_CUDA(cudaMemcpyAsync(out, s->tokens, (size_t)k * 4, cudaMemcpyDeviceToHost, lm::stream())) ||
        !LM_CUDA(cudaStreamSynchronize(lm::stream())) || !lm::check_device_errors(s))
        return -1;
    lm::set_cur_seq(s);
    return (int)valid;
}

int llamini_session_logits(llamini_session* s, f32* out) {
    if (!s) return -1;
    return LM_CUDA(cudaMemcpyAsync(out, s->logits, (size_t)s->vocab * 4, cudaMemcpyDeviceToHost, lm::stream())) &&
                   LM_CUDA(cudaStreamSynchronize(lm::stream()))
               ? 0 : -1;
}

u32 llamini_session_pos(llamini_session* s) { return s ? s->pos : 0; }
int llamini_session_kernel(llamini_session* s) { return s ? (s->flow_on ? 2 : s->dec_on ? 1 : 0) : -1; }
u64 llamini_session_weight_bytes(llamini_session* s) { return s ? s->weight_bytes : 0; }
u64 llamini_session_kv_bytes_per_pos(llamini_session* s) {
    return s ? (u64)s->n_layers * 2 * s->n_kv * s->hd * (s->kv_f16 ? 2 : 4) : 0;
}

int llamini_set_kv_f16(int enable) {
    lm::g_kv_f16 = enable != 0;
    return 0;
}

int llamini_session_trace(llamini_session* s, int enable) {
    if (!s) return -1;
    s->trace_on = enable != 0;
    return 0;
}

int llamini_session_trace_read(llamini_session* s, f32* out) {
    if (!s) return -1;
    return LM_CUDA(cudaMemcpyAsync(out, s->trace, (size_t)s->n_layers * s->dim * 4, cudaMemcpyDeviceToHost, lm::stream())) &&
                   LM_CUDA(cudaStreamSynchronize(lm::stream()))
               ? 0 : -1;
}


// ---------------------------------------------------------------- batched decode

llamini_batch* llamini_llama_batch(LLaMAModel* model, u32 max_batch, u32 max_seq) {
    if (!model) { lm::set_error("batched decode: null model"); return nullptr; }
    return lm::batch_create(model, max_batch, max_seq, lm::bind_llama);
}

llamini_batch* llamini_gpt2_batch(GPT2Model* model, u32 max_batch, u32 max_seq) {
    if (!model) { lm::set_error("batched decode: null model"); return nullptr; }
    return lm::batch_create(model, max_batch, max_seq, lm::bind_gpt2);
}

int llamini_batch_begin(llamini_batch* b, u32 n_seq, const u32* prompts, const u32* prompt_lens) {
    if (!b || !prompts || !prompt_lens) { lm::set_error("batched decode: null argument"); return -1; }
    if (n_seq == 0 || n_seq > b->max_batch) {
        lm::set_error("batched decode: %u sequences, created for 1..%u", n_seq, b->max_batch);
        return -1;
    }
    cudaStream_t st = lm::stream();
    if (!LM_CUDA(cudaStreamSynchronize(st))) return -1;
    const u32 stride = b->max_seq + 1;
    std::vector<u32> toks((size_t)n_seq * stride, 0u), lens(n_seq);
    size_t off = 0;
    for (u32 i = 0; i < n_seq; i++) {
        const u32 L = prompt_lens[i];
        if (L == 0 || L > b->max_seq) { lm::set_error("batched decode: prompt %u has length %u", i, L); return -1; }
        memcpy(&toks[(size_t)i * stride], prompts + off, (size_t)L * 4);
        off += L;
        lens[i] = L;
    }
    b->B = n_seq;
    b->lens = lens;
    b->pos = 0;
    lm::StepState z;
    memset(&z, 0, sizeof(z));
    if (!LM_CUDA(cudaMemcpy(b->tokens, toks.data(), toks.size() * 4, cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemcpy(b->n_prompt, lens.data(), (size_t)n_seq * 4, cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemcpy(b->st, &z, sizeof(z), cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemset(b->keys, 0, (size_t)b->max_batch * 8)))
        return -1;
    return 0;
}

int llamini_batch_step(llamini_batch* b, u32 n_steps) {
    if (!b || b->B == 0) { lm::set_error("batched decode: no batch begun"); return -1; }
    return lm::batch_run(b, n_steps) ? 0 : -1;
}

int llamini_batch_tokens(llamini_batch* b, u32 seq, u32* out, u32 n) {
    if (!b || !out || seq >= b->B) { lm::set_error("batched decode: bad sequence index"); return -1; }
    if (!LM_CUDA(cudaStreamSynchronize(lm::stream())) || !lm::batch_ok(b)) return -1;
    const u32 have = b->pos + 1 > b->lens[seq] ? b->pos + 1 : b->lens[seq];
    const u32 k = n < have ? n : have;
    if (!LM_CUDA(cudaMemcpy(out, b->tokens + (size_t)seq * (b->max_seq + 1), (size_t)k * 4, cudaMemcpyDeviceToHost)))
        return -1;
    return (int)have;
}

int llamini_batch_logits(llamini_batch* b, u32 seq, f32* out) {
    if (!b || !out || seq >= b->B) { lm::set_error("batched decode: bad sequence index"); return -1; }
    if (!LM_CUDA(cudaStreamSynchronize(lm::stream())) || !lm::batch_ok(b)) return -1;
    return LM_CUDA(cudaMemcpy(out, b->logits + (size_t)seq * b->w->vocab, (size_t)b->w->vocab * 4,
                              cudaMemcpyDeviceToHost)) ? 0 : -1;
}

u32 llamini_batch_pos(llamini_batch* b) { return b ? b->pos : 0; }

u64 llamini_batch_weight_bytes(llamini_batch* b) { return b ? b->w->weight_bytes : 0; }

void llamini_batch_free(llamini_batch* b) { lm::batch_destroy(b); }

int llamini_batch_gemm_kind(llamini_batch* b) { return b ? (b->tc ? 1 : 0) : -1; }

// ---------------------------------------------------------------- tensor parallelism

int llamini_tp_handle(void* out) {
    if (!out) { lm::set_error("tp handle: null output"); return -1; }
    if (!lm::ensure_device() || !lm::tp_alloc_buffer()) return -1;
    cudaIpcMemHandle_t h;
    if (!LM_CUDA(cudaIpcGetMemHandle(&h, lm::tp().local))) return -1;
    static_assert(sizeof(h) == 64, "IPC handles are 64 bytes");
    memcpy(out, &h, sizeof(h));
    return 0;
}

int llamini_tp_join(u32 rank, u32 world, const void* handles) {
    lm::TpState& T = lm::tp();
    if (world == 0 || world > lm::kTpMaxRanks || rank >= world) {
        lm::set_error("tp join: rank %u of %u (at most %u ranks)", rank, world, lm::kTpMaxRanks);
        return -1;
    }
    if (world == 1) {
        T.rank = 0;
        T.world = 1;
        return 0;
    }
    if (!handles) { lm::set_error("tp join: null handles"); return -1; }
    if (T.world > 1) { lm::set_error("tp join: this process is already in a group of %u", T.world); return -1; }
    if (!lm::ensure_device() || !lm::tp_alloc_buffer()) return -1;
    float* peer[lm::kTpMaxRanks] = {};
    for (u32 j = 0; j < world; j++) {
        if (j == rank) { peer[j] = T.local; continue; }
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t*)handles + 64 * j, sizeof(h));
        void* p = nullptr;
        if (!LM_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess))) {
            for (u32 k = 0; k < j; k++)
                if (k != rank && peer[k]) cudaIpcCloseMemHandle(peer[k]);
            return -1;
        }
        peer[j] = (float*)p;
    }
    for (u32 j = 0; j < lm::kTpMaxRanks; j++) T.peer[j] = peer[j];
    T.rank = rank;
    T.world = world;
    return 0;
}

int llamini_tp_leave(void) {
    lm::TpState& T = lm::tp();
    if (T.world < 2) return 0;
    if (!LM_CUDA(cudaDeviceSynchronize())) return -1;
    for (u32 j = 0; j < T.world; j++)
        if (j != T.rank && T.peer[j]) cudaIpcCloseMemHandle(T.peer[j]);
    for (u32 j = 0; j < lm::kTpMaxRanks; j++) T.peer[j] = nullptr;
    T.rank = 0;
    T.world = 1;
    // flags and counters from zero for the next group
    return LM_CUDA(cudaMemset(T.local, 0, lm::tp_buffer_bytes())) &&
                   LM_CUDA(cudaMemset(T.gen, 0, 4 * (1 + lm::kTpWideCtas + 4))) && LM_CUDA(cudaDeviceSynchronize())
               ? 0 : -1;
}

int llamini_tp_plan(u32 world, u32 rank, u32 n_heads, u32 n_kv, u32 head_dim, u32 ffn, u32* out) {
    if (!out) { lm::set_error("tp_plan: null output"); return -1; }
    return lm::tp_plan(world, rank, n_heads, n_kv, head_dim, ffn, out);
}
int llamini_tp_rank(void) { return (int)lm::tp().rank; }
int llamini_tp_world(void) { return (int)lm::tp().world; }

int llamini_set_batch_gemm(int kind) {
    if (kind < -1 || kind > 1) { lm::set_error("batched GEMM kind %d outside -1..1", kind); return -1; }
    lm::g_batch_gemm = kind;
    return 0;
}

}  // extern "C"
