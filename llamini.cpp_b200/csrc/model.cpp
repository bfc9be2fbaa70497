// model.cpp -- model configuration, construction and weight binding for the
// LLaMA family (llamini.cpp model.c:262-485) and GPT-2 (gpt2.c:1-127).
//
// Host bookkeeping with the reference's exact semantics (metadata keys,
// per-architecture quirks, lazy big matrices / eager norms and biases, tied
// lm_head). The difference: binding a weight also copies its GGUF bytes,
// unchanged, into GPU memory, where the token loop reads them.
#include "internal.h"
#include "llamini_b200.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cmath>

namespace {

char* copy_str(const char* s) {
    size_t n = strlen(s) + 1;
    char* d = (char*)malloc(n);
    if (d) memcpy(d, s, n);
    return d;
}

// Eager binding: decode the whole tensor into t->data (model.c:414-418).
int bind_eager(GGUFFile* gf, const char* name, Tensor* t) {
    const GGUFTensorInfo* info = gguf_find_tensor(gf, name);
    if (!info) return -1;
    return gguf_dequantize_tensor(gf, info, t->data, t->size);
}

// Lazy binding (model.c:429-437) plus the device copy of the quantized bytes.
int bind_lazy(GGUFFile* gf, const char* name, Tensor* t) {
    const GGUFTensorInfo* info = gguf_find_tensor(gf, name);
    if (!info || gguf_tensor_count(info) != t->size) return -1;
    lm::DevMat m;
    if (!lm::upload_gguf_tensor(gf, info, &m, t->dims[0], t->dims[1])) return -1;
    free(t->data);
    t->data = nullptr;
    t->src_gf = gf;
    t->src_info = info;
    return 0;
}

// GPT-2 keeps eager f32 host copies (gpt2.c:85-89); the matrices are also
// uploaded in their storage type and remembered as the tensor's source.
int bind_eager_with_source(GGUFFile* gf, const char* name, Tensor* t) {
    if (bind_eager(gf, name, t) != 0) return -1;
    const GGUFTensorInfo* info = gguf_find_tensor(gf, name);
    lm::DevMat m;
    if (!lm::upload_gguf_tensor(gf, info, &m, t->dims[0], t->dims[1])) return -1;
    lm::remember_source(t, gf, info);
    return 0;
}

Tensor* make2(u32 a, u32 b) {
    u32 s[2] = {a, b};
    return tensor_create(2, s);
}

}  // namespace

extern "C" {

LLaMAConfig llama_config_from_gguf(GGUFFile* gf, LLaMAConfig defaults, char** arch_out) {
    LLaMAConfig c = defaults;
    c.rope_type = ROPE_NORM;
    c.ffn_act = ACT_SILU;
    c.qkv_bias = 0;
    c.embedding_scale = 1.0f;

    char* arch = gguf_get_str(gf, "general.architecture");
    if (!arch) arch = copy_str("llama");            // files without the key are llama
    if (arch_out) *arch_out = copy_str(arch);

    // quirks not carried by the metadata (model.c:293-299)
    if (strcmp(arch, "qwen2") == 0) {
        c.rope_type = ROPE_NEOX;
        c.qkv_bias = 1;
    } else if (strcmp(arch, "gemma") == 0) {
        c.rope_type = ROPE_NEOX;
        c.ffn_act = ACT_GELU;
    }

    char key[64];
    auto k = [&](const char* suffix) { snprintf(key, sizeof(key), "%s.%s", arch, suffix); return key; };
    c.dim = gguf_get_u32(gf, k("embedding_length"), c.dim);
    c.n_layers = gguf_get_u32(gf, k("block_count"), c.n_layers);
    c.n_heads = gguf_get_u32(gf, k("attention.head_count"), c.n_heads);
    c.n_heads_kv = gguf_get_u32(gf, k("attention.head_count_kv"), c.n_heads);
    c.ffn_dim = gguf_get_u32(gf, k("feed_forward_length"), c.ffn_dim);
    c.rms_eps = gguf_get_f32(gf, k("attention.layer_norm_rms_epsilon"), c.rms_eps);
    c.rope_freq_base = gguf_get_f32(gf, k("rope.freq_base"), c.rope_freq_base);
    const u32 derived = c.n_heads > 0 ? c.dim / c.n_heads : 0;
    c.head_dim = gguf_get_u32(gf, k("attention.key_length"), derived);
    if (strcmp(arch, "gemma") == 0) c.embedding_scale = sqrtf((f32)c.dim);
    const u32 ctx = gguf_get_u32(gf, k("context_length"), c.seq_len);
    c.seq_len = ctx < MAX_SEQ_LEN ? ctx : MAX_SEQ_LEN;
    const u64 nv = gguf_meta_array_len(gf, "tokenizer.ggml.tokens", nullptr);
    if (nv > 0) c.vocab_size = (u32)nv;
    free(arch);
    return c;
}

int llama_model_init(LLaMAModel* model, LLaMAConfig* cfg) {
    memset(model, 0, sizeof(LLaMAModel));
    model->cfg = *cfg;
    model->layers = (DecoderLayer*)calloc(cfg->n_layers, sizeof(DecoderLayer));
    if (!model->layers) return -1;
    const u32 dim = cfg->dim, ffn = cfg->ffn_dim, hd = cfg->head_dim;
    const u32 kvd = cfg->n_heads_kv * hd, qd = cfg->n_heads * hd;
    model->embeddings = make2(cfg->vocab_size, dim);
    model->final_norm = make2(1, dim);
    model->lm_head = make2(cfg->vocab_size, dim);
    for (u32 l = 0; l < cfg->n_layers; l++) {
        DecoderLayer* L = &model->layers[l];
        L->attn_norm = make2(1, dim);
        L->q_proj = make2(qd, dim);
        L->k_proj = make2(kvd, dim);
        L->v_proj = make2(kvd, dim);
        L->o_proj = make2(dim, qd);
        L->ffn_norm = make2(1, dim);
        L->gate_proj = make2(ffn, dim);
        L->up_proj = make2(ffn, dim);
        L->down_proj = make2(dim, ffn);
        if (cfg->qkv_bias) {
            L->q_bias = make2(1, qd);
            L->k_bias = make2(1, kvd);
            L->v_bias = make2(1, kvd);
        }
    }
    return 0;
}

void llama_model_free(LLaMAModel* model) {
    if (!model) return;
    lm::drop_sessions_for_model(model);
    tensor_free(model->embeddings);
    tensor_free(model->final_norm);
    if (model->lm_head != model->embeddings) tensor_free(model->lm_head);   // tied (model.c:385-388)
    if (model->layers) {
        for (u32 l = 0; l < model->cfg.n_layers; l++) {
            DecoderLayer* L = &model->layers[l];
            Tensor* all[] = {L->attn_norm, L->q_proj, L->k_proj, L->v_proj, L->q_bias, L->k_bias,
                             L->v_bias, L->o_proj, L->ffn_norm, L->gate_proj, L->up_proj, L->down_proj};
            for (Tensor* t : all) tensor_free(t);
        }
        free(model->layers);
    }
    memset(model, 0, sizeof(LLaMAModel));
}

int llama_load_weights(LLaMAModel* model, GGUFFile* gf) {
    lm::drop_sessions_for_model(model);
    if (bind_lazy(gf, "token_embd.weight", model->embeddings) != 0) return -1;
    if (bind_eager(gf, "output_norm.weight", model->final_norm) != 0) return -1;
    if (gguf_find_tensor(gf, "output.weight")) {
        if (bind_lazy(gf, "output.weight", model->lm_head) != 0) return -1;
    } else {                                          // tied embeddings (model.c:447-452)
        tensor_free(model->lm_head);
        model->lm_head = model->embeddings;
    }
    char n[64];
    for (u32 l = 0; l < model->cfg.n_layers; l++) {
        DecoderLayer* L = &model->layers[l];
#define LM_BIND(fn, suffix, t) \
        snprintf(n, sizeof(n), "blk.%u." suffix, l); if (fn(gf, n, t) != 0) return -1;
        LM_BIND(bind_eager, "attn_norm.weight", L->attn_norm)
        LM_BIND(bind_lazy, "attn_q.weight", L->q_proj)
        LM_BIND(bind_lazy, "attn_k.weight", L->k_proj)
        LM_BIND(bind_lazy, "attn_v.weight", L->v_proj)
        if (model->cfg.qkv_bias) {
            LM_BIND(bind_eager, "attn_q.bias", L->q_bias)
            LM_BIND(bind_eager, "attn_k.bias", L->k_bias)
            LM_BIND(bind_eager, "attn_v.bias", L->v_bias)
        }
        LM_BIND(bind_lazy, "attn_output.weight", L->o_proj)
        LM_BIND(bind_eager, "ffn_norm.weight", L->ffn_norm)
        LM_BIND(bind_lazy, "ffn_gate.weight", L->gate_proj)
        LM_BIND(bind_lazy, "ffn_up.weight", L->up_proj)
        LM_BIND(bind_lazy, "ffn_down.weight", L->down_proj)
#undef LM_BIND
    }
    return 0;
}

// ---------------------------------------------------------------- GPT-2

GPT2Config gpt2_config_from_gguf(GGUFFile* gf) {
    GPT2Config c;
    c.dim = gguf_get_u32(gf, "gpt2.embedding_length", 768);
    c.n_layers = gguf_get_u32(gf, "gpt2.block_count", 12);
    c.n_heads = gguf_get_u32(gf, "gpt2.attention.head_count", 12);
    c.ffn_dim = gguf_get_u32(gf, "gpt2.feed_forward_length", c.dim * 4);
    const u32 ctx = gguf_get_u32(gf, "gpt2.context_length", 1024);
    c.n_ctx = ctx < MAX_SEQ_LEN ? ctx : MAX_SEQ_LEN;
    c.ln_eps = 1e-5f;                                 // no GGUF key for it (gpt2.c:13)
    const u64 nv = gguf_meta_array_len(gf, "tokenizer.ggml.tokens", nullptr);
    c.vocab_size = nv > 0 ? (u32)nv : 50257;
    return c;
}

int gpt2_model_init(GPT2Model* model, GPT2Config* cfg) {
    memset(model, 0, sizeof(GPT2Model));
    model->cfg = *cfg;
    model->layers = (GPT2Layer*)calloc(cfg->n_layers, sizeof(GPT2Layer));
    if (!model->layers) return -1;
    const u32 d = cfg->dim, f = cfg->ffn_dim;
    model->token_embd = make2(cfg->vocab_size, d);
    model->pos_embd = make2(cfg->n_ctx, d);
    model->output_norm_w = make2(1, d);
    model->output_norm_b = make2(1, d);
    model->lm_head = make2(cfg->vocab_size, d);
    for (u32 l = 0; l < cfg->n_layers; l++) {
        GPT2Layer* L = &model->layers[l];
        L->attn_norm_w = make2(1, d);
        L->attn_norm_b = make2(1, d);
        L->attn_qkv_w = make2(3 * d, d);
        L->attn_qkv_b = make2(1, 3 * d);
        L->attn_out_w = make2(d, d);
        L->attn_out_b = make2(1, d);
        L->ffn_norm_w = make2(1, d);
        L->ffn_norm_b = make2(1, d);
        L->ffn_up_w = make2(f, d);
        L->ffn_up_b = make2(1, f);
        L->ffn_down_w = make2(d, f);
        L->ffn_down_b = make2(1, d);
    }
    return 0;
}

void gpt2_model_free(GPT2Model* model) {
    if (!model) return;
    lm::drop_sessions_for_model(model);
    tensor_free(model->token_embd);
    tensor_free(model->pos_embd);
    tensor_free(model->output_norm_w);
    tensor_free(model->output_norm_b);
    tensor_free(model->lm_head);
    if (model->layers) {
        for (u32 l = 0; l < model->cfg.n_layers; l++) {
            GPT2Layer* L = &model->layers[l];
            Tensor* all[] = {L->attn_norm_w, L->attn_norm_b, L->attn_qkv_w, L->attn_qkv_b, L->attn_out_w,
                             L->attn_out_b, L->ffn_norm_w, L->ffn_norm_b, L->ffn_up_w, L->ffn_up_b,
                             L->ffn_down_w, L->ffn_down_b};
            for (Tensor* t : all) tensor_free(t);
        }
        free(model->layers);
    }
    memset(model, 0, sizeof(GPT2Model));
}

int gpt2_load_weights(GPT2Model* model, GGUFFile* gf) {
    lm::drop_sessions_for_model(model);
    if (bind_eager_with_source(gf, "token_embd.weight", model->token_embd) != 0) return -1;
    if (bind_eager_with_source(gf, "position_embd.weight", model->pos_embd) != 0) return -1;
    if (bind_eager(gf, "output_norm.weight", model->output_norm_w) != 0) return -1;
    if (bind_eager(gf, "output_norm.bias", model->output_norm_b) != 0) return -1;
    if (bind_eager_with_source(gf, "output.weight", model->lm_head) != 0) return -1;
    char n[64];
    for (u32 l = 0; l < model->cfg.n_layers; l++) {
        GPT2Layer* L = &model->layers[l];
#define LM_BIND(fn, suffix, t) \
        snprintf(n, sizeof(n), "blk.%u." suffix, l); if (fn(gf, n, t) != 0) return -1;
        LM_BIND(bind_eager, "attn_norm.weight", L->attn_norm_w)
        LM_BIND(bind_eager, "attn_norm.bias", L->attn_norm_b)
        LM_BIND(bind_eager_with_source, "attn_qkv.weight", L->attn_qkv_w)
        LM_BIND(bind_eager, "attn_qkv.bias", L->attn_qkv_b)
        LM_BIND(bind_eager_with_source, "attn_output.weight", L->attn_out_w)
        LM_BIND(bind_eager, "attn_output.bias", L->attn_out_b)
        LM_BIND(bind_eager, "ffn_norm.weight", L->ffn_norm_w)
        LM_BIND(bind_eager, "ffn_norm.bias", L->ffn_norm_b)
        LM_BIND(bind_eager_with_source, "ffn_up.weight", L->ffn_up_w)
        LM_BIND(bind_eager, "ffn_up.bias", L->ffn_up_b)
        LM_BIND(bind_eager_with_source, "ffn_down.weight", L->ffn_down_w)
        LM_BIND(bind_eager, "ffn_down.bias", L->ffn_down_b)
#undef LM_BIND
    }
    return 0;
}

}  // extern "C"
