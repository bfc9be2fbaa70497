/*
 * ref_driver.c -- flat C entry points over the llamini C API. TEST INFRASTRUCTURE.
 *
 * Written only against the reference's public headers (gguf.h, model.h,
 * generate.h, kv_cache.h, gpt2.h), so the same source builds two ways:
 *   - with the reference's own sources  -> oracle/_ref/libllamini_ref.so
 *     (the reference implementation, used as the authority for golden vectors
 *     and as the timed CPU baseline);
 *   - with include/ and libllamini_cuda.so -> oracle/_ref/libdriver_b200.so
 *     (proves the drop-in: unchanged caller code running on the GPU library).
 * Python reaches either through ctypes with plain pointers.
 */
#include "common.h"
#include "gguf.h"
#include "model.h"
#include "generate.h"
#include "kv_cache.h"
#include "gpt2.h"

static GGUFFile g_gf;
static int g_open = 0;
static int g_is_gpt2 = 0;
static LLaMAModel g_llama;
static GPT2Model g_gpt2;
static KVCache* g_caches = NULL;
static u32 g_n_layers = 0;

void drv_close(void) {
    if (!g_open) return;
    if (g_open == 2) {                 /* file only (drv_open_file) */
        gguf_close(&g_gf);
        g_open = 0;
        return;
    }
    for (u32 l = 0; l < g_n_layers; l++) { free(g_caches[l].key); free(g_caches[l].val); }
    free(g_caches);
    g_caches = NULL;
    if (g_is_gpt2) gpt2_model_free(&g_gpt2); else llama_model_free(&g_llama);
    gguf_close(&g_gf);
    g_open = 0;
}

/* Open a GGUF model the way main.c:400-481 does (arch dispatch, config, init,
 * load, one KV cache per layer). max_seq = 0 keeps the model's own context. */
int drv_open(const char* path, u32 max_seq) {
    drv_close();
    if (gguf_open(path, &g_gf) != 0) return -1;
    char* arch = gguf_get_str(&g_gf, "general.architecture");
    g_is_gpt2 = arch && strcmp(arch, "gpt2") == 0;
    free(arch);
    if (g_is_gpt2) {
        GPT2Config c = gpt2_config_from_gguf(&g_gf);
        if (gpt2_model_init(&g_gpt2, &c) != 0 || gpt2_load_weights(&g_gpt2, &g_gf) != 0) {
            gguf_close(&g_gf);
            return -1;
        }
        g_n_layers = c.n_layers;
        u32 ms = max_seq ? max_seq : c.n_ctx;
        g_caches = (KVCache*)calloc(g_n_layers, sizeof(KVCache));
        for (u32 l = 0; l < g_n_layers; l++) kv_cache_init(&g_caches[l], c.dim, ms);
    } else {
        LLaMAConfig d;
        memset(&d, 0, sizeof(d));
        d.dim = 2048; d.n_layers = 22; d.n_heads = 32; d.n_heads_kv = 4; d.ffn_dim = 5632;
        d.vocab_size = 32000; d.seq_len = 2048; d.rms_eps = 1e-5f; d.rope_freq_base = 10000.0f;
        LLaMAConfig c = llama_config_from_gguf(&g_gf, d, NULL);
        if (llama_model_init(&g_llama, &c) != 0 || llama_load_weights(&g_llama, &g_gf) != 0) {
            gguf_close(&g_gf);
            return -1;
        }
        g_n_layers = c.n_layers;
        u32 ms = max_seq ? max_seq : c.seq_len;
        g_caches = (KVCache*)calloc(g_n_layers, sizeof(KVCache));
        for (u32 l = 0; l < g_n_layers; l++) kv_cache_init(&g_caches[l], c.n_heads_kv * c.head_dim, ms);
    }
    g_open = 1;
    return 0;
}

/* Open a GGUF file without building a model, for drv_dequant_rows. */
int drv_open_file(const char* path) {
    drv_close();
    if (gguf_open(path, &g_gf) != 0) return -1;
    g_open = 2;
    return 0;
}

u32 drv_vocab(void) {
    if (!g_open) return 0;
    return g_is_gpt2 ? g_gpt2.cfg.vocab_size : g_llama.cfg.vocab_size;
}

void drv_reset(void) {
    for (u32 l = 0; l < g_n_layers; l++) kv_cache_reset(&g_caches[l]);
}

void drv_forward(u32 pos, u32 token, f32* logits) {
    if (g_is_gpt2) gpt2_forward_step(&g_gpt2, g_caches, pos, token, logits);
    else forward_step(&g_llama, g_caches, pos, token, logits);
}

/* Greedy run with the caches reset first (main.c:197-200). */
u32 drv_generate(u32* prompt, u32 n_prompt, u32* out, u32 max_gen, u32 eos) {
    drv_reset();
    if (g_is_gpt2) return gpt2_generate(&g_gpt2, g_caches, prompt, n_prompt, out, max_gen, eos, 0.0f, 0.0f);
    return generate_autoregressive(&g_llama, g_caches, prompt, n_prompt, out, max_gen, eos, 0.0f, 0.0f);
}

/* generate_autoregressive / gpt2_generate with sampling (temp > 0): srand(seed)
 * first, so the draws are rand()'s stream from that seed (generate.c:50). */
u32 drv_generate_sampled(u32* prompt, u32 n_prompt, u32* out, u32 max_gen, u32 eos, f32 temp, f32 top_p, u32 seed) {
    drv_reset();
    srand(seed);
    if (g_is_gpt2) return gpt2_generate(&g_gpt2, g_caches, prompt, n_prompt, out, max_gen, eos, temp, top_p);
    return generate_autoregressive(&g_llama, g_caches, prompt, n_prompt, out, max_gen, eos, temp, top_p);
}

f32 drv_perplexity(const u32* tokens, u32 n) {
    if (g_is_gpt2) return gpt2_compute_perplexity(&g_gpt2, g_caches, tokens, n);
    return compute_perplexity(&g_llama, g_caches, tokens, n);
}

/* Seconds spent in n_steps single-token forward passes at positions
 * pos0 .. pos0+n_steps-1 (each feeding the previous argmax), after the caller
 * has filled positions < pos0. Used for the CPU baseline timing. */
double drv_time_decode(u32 pos0, u32 first_token, u32 n_steps, u32* out_tokens) {
    u32 vocab = drv_vocab();
    f32* logits = (f32*)malloc((size_t)vocab * sizeof(f32));
    struct timespec a, b;
    u32 tok = first_token;
    clock_gettime(CLOCK_MONOTONIC, &a);
    for (u32 i = 0; i < n_steps; i++) {
        drv_forward(pos0 + i, tok, logits);
        tok = greedy_sample(logits, vocab);
        if (out_tokens) out_tokens[i] = tok;
    }
    clock_gettime(CLOCK_MONOTONIC, &b);
    free(logits);
    return (double)(b.tv_sec - a.tv_sec) + (double)(b.tv_nsec - a.tv_nsec) * 1e-9;
}

/* Dequantize rows of a named tensor of the open file (gguf.c:602-605). */
int drv_dequant_rows(const char* name, u32 row0, u32 row1, u32 row_len, f32* out) {
    const GGUFTensorInfo* ti = gguf_find_tensor(&g_gf, name);
    if (!ti) return -1;
    return gguf_dequantize_rows(&g_gf, ti, row0, row1, row_len, out);
}

/* Decode raw blocks of any type through a GGUF round trip is not possible
 * without a file, so raw-block goldens use a one-tensor GGUF written by the
 * fixture script and drv_dequant_rows above. */

/* The fake model of main.c:552-596 (dim 16, 1 layer, 4/2 heads, ffn 32,
 * vocab 8, weights from index patterns), generated greedily from the prompt
 * {1,3,4,2} with max 4 new tokens and eos 999. Returns the token count. */
u32 drv_fake_generate(u32* out8) {
    LLaMAConfig c;
    memset(&c, 0, sizeof(c));
    c.dim = 16; c.n_layers = 1; c.n_heads = 4; c.n_heads_kv = 2; c.head_dim = 4;
    c.ffn_dim = 32; c.vocab_size = 8; c.seq_len = 32; c.rms_eps = 1e-5f;
    c.rope_freq_base = 10000.0f; c.rope_type = ROPE_NORM; c.ffn_act = ACT_SILU;
    c.qkv_bias = 0; c.embedding_scale = 1.0f;
    LLaMAModel m;
    if (llama_model_init(&m, &c) != 0) return 0;
    /* The index patterns are evaluated in unsigned arithmetic exactly as in
     * main.c:568-578: (i % 7) - 3 wraps to ~4.29e9 when i % 7 < 3, so those
     * weights are huge. The golden tokens depend on that, so it is kept. */
    for (u32 i = 0; i < m.embeddings->size; i++) m.embeddings->data[i] = (f32)((i % 7) - 3) * 0.1f;
    for (u32 i = 0; i < m.final_norm->size; i++) m.final_norm->data[i] = 1.0f;
    for (u32 i = 0; i < m.lm_head->size; i++) m.lm_head->data[i] = (f32)((i % 5) - 2) * 0.1f;
    DecoderLayer* L = &m.layers[0];
    Tensor* pat[] = { L->q_proj, L->k_proj, L->v_proj, L->o_proj, L->gate_proj, L->up_proj, L->down_proj };
    for (u32 i = 0; i < L->attn_norm->size; i++) L->attn_norm->data[i] = 1.0f;
    for (u32 i = 0; i < L->ffn_norm->size; i++) L->ffn_norm->data[i] = 1.0f;
    for (u32 t = 0; t < 7; t++)
        for (u32 i = 0; i < pat[t]->size; i++) pat[t]->data[i] = (f32)((i % 5) - 2) * 0.05f;
    KVCache kc;
    kv_cache_init(&kc, c.n_heads_kv * c.head_dim, c.seq_len);
    u32 prompt[4] = {1, 3, 4, 2};
    u32 n = generate_autoregressive(&m, &kc, prompt, 4, out8, 4, 999, 0.0f, 0.0f);
    free(kc.key); free(kc.val);
    llama_model_free(&m);
    return n;
}

/* Per-op known-answer inputs of main.c:505-531. */
void drv_rms_norm(f32* out, const f32* x, const f32* w, u32 dim, f32 eps) { rms_norm(out, x, w, dim, eps); }
void drv_rope(f32* v, u32 pos, u32 dim, u32 hd, f32 base, int neox) {
    rope(v, pos, dim, hd, base, neox ? ROPE_NEOX : ROPE_NORM);
}
void drv_ffn_glu(f32* out, const f32* g, const f32* u, u32 n, int gelu) {
    ffn_glu(out, g, u, n, gelu ? ACT_GELU : ACT_SILU);
}
void drv_causal_mha(const f32* q, const f32* k, const f32* v, f32* kc, f32* vc, u32 max_seq,
                    f32* out, u32 pos, u32 nh, u32 nkv, u32 hd) {
    KVCache c;
    c.key = kc; c.val = vc; c.dim = nkv * hd; c.max_seq = max_seq; c.cur_seq = 0;
    causal_mha(q, k, v, &c, out, pos, nh, nkv, hd);
}
void drv_linear_f32(f32* out, const f32* x, const f32* w, u32 in_dim, u32 out_dim) {
    u32 shape[2] = { out_dim, in_dim };
    Tensor* t = tensor_create(2, shape);
    memcpy(t->data, w, (size_t)in_dim * out_dim * sizeof(f32));
    linear(out, x, t, in_dim, out_dim);
    tensor_free(t);
}
u32 drv_greedy(const f32* x, u32 n) { return greedy_sample(x, n); }
