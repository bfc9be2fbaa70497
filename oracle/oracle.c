/*
 * oracle.c -- CPU restatement of llamini.cpp's token loop. TEST INFRASTRUCTURE.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this
 * library; the product path never does. Build: oracle/Makefile
 * (gcc -O2 -fopenmp -ffp-contract=off). Each function cites the reference lines
 * whose arithmetic it restates; the float operations are written in the same
 * order as the reference so that the block decoders are bit-identical.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ formats */

uint32_t orc_block_elems(uint32_t type) {
    switch (type) {
    case ORC_F32: case ORC_F16: return 1;
    case ORC_Q4_0: case ORC_Q4_1: case ORC_Q5_0: case ORC_Q8_0: return 32;
    case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K: return 256;
    default: return 0;
    }
}

uint32_t orc_block_bytes(uint32_t type) {
    switch (type) {
    case ORC_F32: return 4;
    case ORC_F16: return 2;
    case ORC_Q4_0: return 18;
    case ORC_Q4_1: return 20;
    case ORC_Q5_0: return 22;
    case ORC_Q8_0: return 34;
    case ORC_Q4_K: return 144;
    case ORC_Q5_K: return 176;
    case ORC_Q6_K: return 210;
    default: return 0;
    }
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* gguf.c:364-386: sign, 5-bit exponent, 10-bit mantissa; subnormals are
 * renormalised, exponent 31 maps to inf/nan. */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    int32_t e = (h >> 10) & 31;
    uint32_t m = h & 1023u;
    uint32_t bits;
    if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e == 0 && m == 0) {
        bits = sign;
    } else {
        if (e == 0) {              /* subnormal: shift until the hidden bit appears */
            e = 1;
            while ((m & 1024u) == 0) { m <<= 1; e--; }
            m &= 1023u;
        }
        bits = sign | ((uint32_t)(e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* gguf.c:391-399: six-bit (scale, min) of sub-block j from the 12-byte field. */
static void k4_scale_min(const uint8_t* s, int j, uint8_t* sc, uint8_t* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 15) | ((s[j - 4] >> 6) << 4));
        *mn = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* One block of each format -> out[0..block_elems). */
static void dec_q4_0(const uint8_t* b, float* y) {          /* gguf.c:427-444 */
    float d = orc_f16_to_f32(rd16(b));
    for (int i = 0; i < 16; i++) {
        y[i]      = ((float)(b[2 + i] & 15) - 8.0f) * d;
        y[i + 16] = ((float)(b[2 + i] >> 4) - 8.0f) * d;
    }
}

static void dec_q4_1(const uint8_t* b, float* y) {          /* gguf.c:445-462 */
    float d = orc_f16_to_f32(rd16(b));
    float m = orc_f16_to_f32(rd16(b + 2));
    for (int i = 0; i < 16; i++) {
        y[i]      = (float)(b[4 + i] & 15) * d + m;
        y[i + 16] = (float)(b[4 + i] >> 4) * d + m;
    }
}

static void dec_q5_0(const uint8_t* b, float* y) {          /* gguf.c:463-488 */
    float d = orc_f16_to_f32(rd16(b));
    uint32_t hb = rd32(b + 2);
    for (int i = 0; i < 16; i++) {
        int lo = (int)((b[6 + i] & 15) | (((hb >> i) & 1u) << 4)) - 16;
        int hi = (int)((b[6 + i] >> 4) | (((hb >> (i + 16)) & 1u) << 4)) - 16;
        y[i]      = (float)lo * d;
        y[i + 16] = (float)hi * d;
    }
}

static void dec_q8_0(const uint8_t* b, float* y) {          /* gguf.c:489-503 */
    float d = orc_f16_to_f32(rd16(b));
    for (int i = 0; i < 32; i++) y[i] = (float)(int8_t)b[2 + i] * d;
}

static void dec_q4_k(const uint8_t* b, float* y) {          /* gguf.c:504-529 */
    float d = orc_f16_to_f32(rd16(b));
    float dmin = orc_f16_to_f32(rd16(b + 2));
    const uint8_t* sc = b + 4;
    const uint8_t* qs = b + 16;
    for (int g = 0; g < 4; g++) {                /* 64-element groups */
        uint8_t s0, m0, s1, m1;
        k4_scale_min(sc, 2 * g, &s0, &m0);
        k4_scale_min(sc, 2 * g + 1, &s1, &m1);
        float d0 = d * s0, n0 = dmin * m0;
        float d1 = d * s1, n1 = dmin * m1;
        for (int l = 0; l < 32; l++) {
            y[64 * g + l]      = d0 * (float)(qs[32 * g + l] & 15) - n0;
            y[64 * g + 32 + l] = d1 * (float)(qs[32 * g + l] >> 4) - n1;
        }
    }
}

static void dec_q5_k(const uint8_t* b, float* y) {          /* gguf.c:530-560 */
    float d = orc_f16_to_f32(rd16(b));
    float dmin = orc_f16_to_f32(rd16(b + 2));
    const uint8_t* sc = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int g = 0; g < 4; g++) {
        uint8_t s0, m0, s1, m1;
        k4_scale_min(sc, 2 * g, &s0, &m0);
        k4_scale_min(sc, 2 * g + 1, &s1, &m1);
        float d0 = d * s0, n0 = dmin * m0;
        float d1 = d * s1, n1 = dmin * m1;
        for (int l = 0; l < 32; l++) {
            int lo = (qs[32 * g + l] & 15) + (((qh[l] >> (2 * g)) & 1) ? 16 : 0);
            int hi = (qs[32 * g + l] >> 4) + (((qh[l] >> (2 * g + 1)) & 1) ? 16 : 0);
            y[64 * g + l]      = d0 * (float)lo - n0;
            y[64 * g + 32 + l] = d1 * (float)hi - n1;
        }
    }
}

static void dec_q6_k(const uint8_t* b, float* y) {          /* gguf.c:561-590 */
    float d = orc_f16_to_f32(rd16(b + 208));
    for (int h = 0; h < 2; h++) {                /* two 128-element halves */
        const uint8_t* ql = b + 64 * h;
        const uint8_t* qh = b + 128 + 32 * h;
        const int8_t* sc = (const int8_t*)(b + 192 + 8 * h);
        float* o = y + 128 * h;
        for (int l = 0; l < 32; l++) {
            int s = l / 16;
            int v0 = (int)((ql[l] & 15)      | (((qh[l] >> 0) & 3) << 4)) - 32;
            int v1 = (int)((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int v2 = (int)((ql[l] >> 4)      | (((qh[l] >> 4) & 3) << 4)) - 32;
            int v3 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            o[l]      = d * (float)sc[s + 0] * (float)v0;
            o[l + 32] = d * (float)sc[s + 2] * (float)v1;
            o[l + 64] = d * (float)sc[s + 4] * (float)v2;
            o[l + 96] = d * (float)sc[s + 6] * (float)v3;
        }
    }
}

int orc_dequant(uint32_t type, const uint8_t* raw, uint64_t n, float* out) {
    uint32_t be = orc_block_elems(type), bb = orc_block_bytes(type);
    if (be == 0 || n % be != 0) return -1;
    uint64_t nb = n / be;
    switch (type) {
    case ORC_F32: memcpy(out, raw, n * 4); return 0;
    case ORC_F16:
        for (uint64_t i = 0; i < n; i++) out[i] = orc_f16_to_f32(rd16(raw + 2 * i));
        return 0;
    default: break;
    }
    for (uint64_t i = 0; i < nb; i++) {
        const uint8_t* b = raw + i * bb;
        float* y = out + i * be;
        switch (type) {
        case ORC_Q4_0: dec_q4_0(b, y); break;
        case ORC_Q4_1: dec_q4_1(b, y); break;
        case ORC_Q5_0: dec_q5_0(b, y); break;
        case ORC_Q8_0: dec_q8_0(b, y); break;
        case ORC_Q4_K: dec_q4_k(b, y); break;
        case ORC_Q5_K: dec_q5_k(b, y); break;
        case ORC_Q6_K: dec_q6_k(b, y); break;
        default: return -1;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ linear */

static uint64_t row_bytes(const OrcMat* w) {
    return (uint64_t)w->cols / orc_block_elems(w->type) * orc_block_bytes(w->type);
}

/* model.c:159-176 decodes rows into a scratch buffer and runs model.c:66-73's
 * dot on each; here each thread decodes one row at a time. */
void orc_linear(const OrcMat* w, const float* x, float* y) {
    const uint64_t rb = row_bytes(w);
    const uint32_t K = w->cols;
#pragma omp parallel
    {
        float* row = (float*)malloc((size_t)K * sizeof(float));
#pragma omp for schedule(static)
        for (int64_t r = 0; r < (int64_t)w->rows; r++) {
            if (orc_dequant(w->type, w->data + (uint64_t)r * rb, K, row) != 0) { y[r] = 0.0f; continue; }
            float acc = 0.0f;
            for (uint32_t i = 0; i < K; i++) acc += row[i] * x[i];
            y[r] = acc;
        }
        free(row);
    }
}

/* ------------------------------------------------------------------ ops */

void orc_rms_norm(float* out, const float* x, const float* w, uint32_t dim, float eps) {
    /* model.c:4-10 */
    float ss = 0.0f;
    for (uint32_t i = 0; i < dim; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / dim + eps);
    for (uint32_t i = 0; i < dim; i++) out[i] = x[i] * inv * w[i];
}

void orc_layer_norm(float* out, const float* x, const float* w, const float* b, uint32_t dim, float eps) {
    /* gpt2.c:130-139: two-pass mean / variance */
    float mean = 0.0f;
    for (uint32_t i = 0; i < dim; i++) mean += x[i];
    mean /= (float)dim;
    float var = 0.0f;
    for (uint32_t i = 0; i < dim; i++) { float c = x[i] - mean; var += c * c; }
    var /= (float)dim;
    float inv = 1.0f / sqrtf(var + eps);
    for (uint32_t i = 0; i < dim; i++) out[i] = (x[i] - mean) * inv * w[i] + b[i];
}

float orc_gelu(float x) {
    /* model.c:14-18 / gpt2.c:144-148: tanh approximation */
    const float k0 = 0.79788456080286535587989211986876f;
    const float k1 = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(k0 * x * (1.0f + k1 * x * x)));
}

void orc_ffn_glu(float* out, const float* gate, const float* up, uint32_t n, int act_gelu) {
    /* model.c:20-25 */
    for (uint32_t i = 0; i < n; i++) {
        float g = act_gelu ? orc_gelu(gate[i]) : gate[i] / (1.0f + expf(-gate[i]));
        out[i] = g * up[i];
    }
}

void orc_rope(float* v, uint32_t pos, uint32_t dim, uint32_t hd, float base, int neox) {
    /* model.c:31-58 */
    if (neox) {
        uint32_t half = hd / 2;
        for (uint32_t h0 = 0; h0 < dim; h0 += hd) {
            for (uint32_t j = 0; j < half; j++) {
                float th = powf(base, -(float)(2 * j) / (float)hd);
                float c = cosf(pos * th), s = sinf(pos * th);
                float a = v[h0 + j], b = v[h0 + j + half];
                v[h0 + j] = a * c - b * s;
                v[h0 + j + half] = a * s + b * c;
            }
        }
        return;
    }
    for (uint32_t i = 0; i < dim; i += 2) {
        float th = powf(base, -(float)(i % hd) / (float)hd);
        float c = cosf(pos * th), s = sinf(pos * th);
        float a = v[i], b = v[i + 1];
        v[i] = a * c - b * s;
        v[i + 1] = a * s + b * c;
    }
}

void orc_causal_mha(const float* q, const float* k, const float* v, float* kc, float* vc,
                    float* out, uint32_t pos, uint32_t nh, uint32_t nkv, uint32_t hd) {
    /* model.c:217-260: store k/v at pos, then a three-pass softmax per head */
    uint32_t kvd = nkv * hd, grp = nh / nkv;
    memcpy(kc + (uint64_t)pos * kvd, k, kvd * sizeof(float));
    memcpy(vc + (uint64_t)pos * kvd, v, kvd * sizeof(float));
    float* sc = (float*)malloc((size_t)(pos + 1) * sizeof(float));
    for (uint32_t h = 0; h < nh; h++) {
        uint32_t g = h / grp;
        const float* qh = q + (uint64_t)h * hd;
        float mx = -1e30f;
        for (uint32_t t = 0; t <= pos; t++) {
            const float* kt = kc + (uint64_t)t * kvd + (uint64_t)g * hd;
            float s = 0.0f;
            for (uint32_t d = 0; d < hd; d++) s += qh[d] * kt[d];
            s /= sqrtf((float)hd);
            sc[t] = s;
            if (s > mx) mx = s;
        }
        float sum = 0.0f;
        for (uint32_t t = 0; t <= pos; t++) { sc[t] = expf(sc[t] - mx); sum += sc[t]; }
        float* o = out + (uint64_t)h * hd;
        for (uint32_t d = 0; d < hd; d++) o[d] = 0.0f;
        for (uint32_t t = 0; t <= pos; t++) {
            float wgt = sc[t] / sum;
            const float* vt = vc + (uint64_t)t * kvd + (uint64_t)g * hd;
            for (uint32_t d = 0; d < hd; d++) o[d] += wgt * vt[d];
        }
    }
    free(sc);
}

uint32_t orc_greedy(const float* x, uint32_t n) {
    /* generate.c:3-9: first index of the strict maximum */
    uint32_t bi = 0;
    float bv = x[0];
    for (uint32_t i = 1; i < n; i++) if (x[i] > bv) { bv = x[i]; bi = i; }
    return bi;
}

/* ------------------------------------------------------------------ models */

struct OrcState {
    uint32_t n_layers, kv_dim, max_seq;
    float** kc;
    float** vc;
};

static OrcState* state_new(uint32_t n_layers, uint32_t kv_dim, uint32_t max_seq) {
    OrcState* s = (OrcState*)calloc(1, sizeof(OrcState));
    s->n_layers = n_layers; s->kv_dim = kv_dim; s->max_seq = max_seq;
    s->kc = (float**)calloc(n_layers, sizeof(float*));
    s->vc = (float**)calloc(n_layers, sizeof(float*));
    for (uint32_t l = 0; l < n_layers; l++) {
        s->kc[l] = (float*)calloc((size_t)kv_dim * max_seq, sizeof(float));
        s->vc[l] = (float*)calloc((size_t)kv_dim * max_seq, sizeof(float));
    }
    return s;
}

OrcState* orc_llama_state_new(const OrcLlama* m) {
    return state_new(m->n_layers, m->n_heads_kv * m->head_dim, m->max_seq);
}

OrcState* orc_gpt2_state_new(const OrcGpt2* m) {
    return state_new(m->n_layers, m->dim, m->max_seq);
}

void orc_state_free(OrcState* s) {
    if (!s) return;
    for (uint32_t l = 0; l < s->n_layers; l++) { free(s->kc[l]); free(s->vc[l]); }
    free(s->kc); free(s->vc); free(s);
}

static void embed_row(const OrcMat* e, uint32_t row, float* out) {
    /* tensor.c:24-30: one-row decode of the embedding table */
    orc_dequant(e->type, e->data + (uint64_t)row * row_bytes(e), e->cols, out);
}

void orc_llama_forward(const OrcLlama* m, OrcState* s, uint32_t pos, uint32_t token,
                       float* logits, float* trace) {
    /* generate.c:62-120 */
    const uint32_t dim = m->dim, ffn = m->ffn_dim, hd = m->head_dim;
    const uint32_t qd = m->n_heads * hd, kvd = m->n_heads_kv * hd;
    float* h  = (float*)malloc(dim * sizeof(float));
    float* xn = (float*)malloc(dim * sizeof(float));
    float* q  = (float*)malloc(qd * sizeof(float));
    float* k  = (float*)malloc(kvd * sizeof(float));
    float* v  = (float*)malloc(kvd * sizeof(float));
    float* ao = (float*)malloc(qd * sizeof(float));
    float* ap = (float*)malloc(dim * sizeof(float));
    float* g  = (float*)malloc(ffn * sizeof(float));
    float* u  = (float*)malloc(ffn * sizeof(float));
    float* fh = (float*)malloc(ffn * sizeof(float));
    float* fo = (float*)malloc(dim * sizeof(float));

    embed_row(&m->tok_embd, token, h);
    if (m->emb_scale != 1.0f) for (uint32_t i = 0; i < dim; i++) h[i] *= m->emb_scale;

    for (uint32_t l = 0; l < m->n_layers; l++) {
        const OrcLlamaLayer* L = &m->layers[l];
        orc_rms_norm(xn, h, L->attn_norm, dim, m->rms_eps);
        orc_linear(&L->q, xn, q);
        orc_linear(&L->k, xn, k);
        orc_linear(&L->v, xn, v);
        if (L->bq) {
            for (uint32_t i = 0; i < qd; i++) q[i] += L->bq[i];
            for (uint32_t i = 0; i < kvd; i++) k[i] += L->bk[i];
            for (uint32_t i = 0; i < kvd; i++) v[i] += L->bv[i];
        }
        orc_rope(q, pos, qd, hd, m->rope_base, m->rope_neox);
        orc_rope(k, pos, kvd, hd, m->rope_base, m->rope_neox);
        orc_causal_mha(q, k, v, s->kc[l], s->vc[l], ao, pos, m->n_heads, m->n_heads_kv, hd);
        orc_linear(&L->o, ao, ap);
        for (uint32_t i = 0; i < dim; i++) h[i] += ap[i];
        orc_rms_norm(xn, h, L->ffn_norm, dim, m->rms_eps);
        orc_linear(&L->gate, xn, g);
        orc_linear(&L->up, xn, u);
        orc_ffn_glu(fh, g, u, ffn, m->act_gelu);
        orc_linear(&L->down, fh, fo);
        for (uint32_t i = 0; i < dim; i++) h[i] += fo[i];
        if (trace) memcpy(trace + (uint64_t)l * dim, h, dim * sizeof(float));
    }
    orc_rms_norm(xn, h, m->final_norm, dim, m->rms_eps);
    orc_linear(&m->lm_head, xn, logits);

    free(h); free(xn); free(q); free(k); free(v); free(ao); free(ap);
    free(g); free(u); free(fh); free(fo);
}

uint32_t orc_llama_generate(const OrcLlama* m, OrcState* s, const uint32_t* prompt, uint32_t n_prompt,
                            uint32_t* out, uint32_t max_gen, uint32_t eos) {
    /* generate.c:122-167 with temp = 0 */
    uint32_t total = n_prompt;
    memcpy(out, prompt, n_prompt * sizeof(uint32_t));
    float* logits = (float*)malloc((size_t)m->vocab * sizeof(float));
    for (uint32_t pos = 0; pos < m->max_seq;) {
        orc_llama_forward(m, s, pos, out[pos], logits, NULL);
        pos++;
        if (pos < n_prompt) continue;
        uint32_t t = orc_greedy(logits, m->vocab);
        out[total++] = t;
        if (t == eos || total - n_prompt >= max_gen) break;
    }
    free(logits);
    return total;
}

void orc_gpt2_forward(const OrcGpt2* m, OrcState* s, uint32_t pos, uint32_t token,
                      float* logits, float* trace) {
    /* gpt2.c:150-192 */
    const uint32_t dim = m->dim, ffn = m->ffn_dim, hd = dim / m->n_heads;
    float* h   = (float*)malloc(dim * sizeof(float));
    float* pe  = (float*)malloc(dim * sizeof(float));
    float* xn  = (float*)malloc(dim * sizeof(float));
    float* qkv = (float*)malloc(3 * dim * sizeof(float));
    float* ao  = (float*)malloc(dim * sizeof(float));
    float* ap  = (float*)malloc(dim * sizeof(float));
    float* fh  = (float*)malloc(ffn * sizeof(float));
    float* fo  = (float*)malloc(dim * sizeof(float));

    embed_row(&m->tok_embd, token, h);
    embed_row(&m->pos_embd, pos, pe);
    for (uint32_t i = 0; i < dim; i++) h[i] = h[i] + pe[i];

    for (uint32_t l = 0; l < m->n_layers; l++) {
        const OrcGpt2Layer* L = &m->layers[l];
        orc_layer_norm(xn, h, L->attn_norm_w, L->attn_norm_b, dim, m->ln_eps);
        orc_linear(&L->qkv, xn, qkv);
        for (uint32_t i = 0; i < 3 * dim; i++) qkv[i] += L->qkv_b[i];
        orc_causal_mha(qkv, qkv + dim, qkv + 2 * dim, s->kc[l], s->vc[l], ao, pos,
                       m->n_heads, m->n_heads, hd);
        orc_linear(&L->out, ao, ap);
        for (uint32_t i = 0; i < dim; i++) ap[i] += L->out_b[i];
        for (uint32_t i = 0; i < dim; i++) h[i] += ap[i];
        orc_layer_norm(xn, h, L->ffn_norm_w, L->ffn_norm_b, dim, m->ln_eps);
        orc_linear(&L->up, xn, fh);
        for (uint32_t i = 0; i < ffn; i++) fh[i] += L->up_b[i];
        for (uint32_t i = 0; i < ffn; i++) fh[i] = orc_gelu(fh[i]);
        orc_linear(&L->down, fh, fo);
        for (uint32_t i = 0; i < dim; i++) fo[i] += L->down_b[i];
        for (uint32_t i = 0; i < dim; i++) h[i] += fo[i];
        if (trace) memcpy(trace + (uint64_t)l * dim, h, dim * sizeof(float));
    }
    orc_layer_norm(xn, h, m->out_norm_w, m->out_norm_b, dim, m->ln_eps);
    orc_linear(&m->lm_head, xn, logits);

    free(h); free(pe); free(xn); free(qkv); free(ao); free(ap); free(fh); free(fo);
}

uint32_t orc_gpt2_generate(const OrcGpt2* m, OrcState* s, const uint32_t* prompt, uint32_t n_prompt,
                           uint32_t* out, uint32_t max_gen, uint32_t eos) {
    /* gpt2.c:194-229 with temp = 0; the position limit is min(max_seq, n_ctx) */
    uint32_t total = n_prompt;
    memcpy(out, prompt, n_prompt * sizeof(uint32_t));
    float* logits = (float*)malloc((size_t)m->vocab * sizeof(float));
    uint32_t lim = m->max_seq < m->n_ctx ? m->max_seq : m->n_ctx;
    for (uint32_t pos = 0; pos < lim;) {
        orc_gpt2_forward(m, s, pos, out[pos], logits, NULL);
        pos++;
        if (pos < n_prompt) continue;
        uint32_t t = orc_greedy(logits, m->vocab);
        out[total++] = t;
        if (t == eos || total - n_prompt >= max_gen) break;
    }
    free(logits);
    return total;
}
