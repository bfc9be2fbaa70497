/*
 * gpt2.h -- GPT-2 model path (llamini.cpp gpt2.h:1-70).
 *
 * Same structs and signatures as the reference: fused QKV with bias, learned
 * position embeddings, LayerNorm with bias, ungated tanh-GELU MLP, untied
 * lm_head. gpt2_load_weights keeps the reference's eager f32 host tensors and
 * additionally uploads each weight to GPU memory in its GGUF storage type, which
 * is what gpt2_forward_step / gpt2_generate run on.
 */
#ifndef GPT2_H
#define GPT2_H

#include "common.h"
#include "tensor.h"
#include "kv_cache.h"
#include "gguf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* gpt2.h:18-21 */
typedef struct {
    u32 dim, n_layers, n_heads, ffn_dim, vocab_size, n_ctx;
    f32 ln_eps;
} GPT2Config;

/* gpt2.h:23-30 */
typedef struct {
    Tensor *attn_norm_w, *attn_norm_b;
    Tensor *attn_qkv_w, *attn_qkv_b;
    Tensor *attn_out_w, *attn_out_b;
    Tensor *ffn_norm_w, *ffn_norm_b;
    Tensor *ffn_up_w, *ffn_up_b;
    Tensor *ffn_down_w, *ffn_down_b;
} GPT2Layer;

/* gpt2.h:32-40 */
typedef struct {
    GPT2Config cfg;
    Tensor* token_embd;
    Tensor* pos_embd;
    Tensor* output_norm_w;
    Tensor* output_norm_b;
    Tensor* lm_head;
    GPT2Layer* layers;
} GPT2Model;

/* gpt2.h:46, gpt2.c:5-18 */
GPT2Config gpt2_config_from_gguf(GGUFFile* gf);

/* gpt2.h:48-50, gpt2.c:20-127 */
int gpt2_model_init(GPT2Model* model, GPT2Config* cfg);
void gpt2_model_free(GPT2Model* model);
int gpt2_load_weights(GPT2Model* model, GGUFFile* gf);

/* One token through the GPT-2 stack; vocab_size logits to host logits_out
 * (gpt2.h:56, gpt2.c:150-192). */
void gpt2_forward_step(GPT2Model* model, KVCache* caches, u32 pos, u32 token_id, f32* logits_out);

/* Prefill then sample, stopping like generate_autoregressive; the position
 * limit is min(cache capacity, n_ctx) (gpt2.h:63, gpt2.c:194-229). */
u32 gpt2_generate(GPT2Model* model, KVCache* caches, u32* input_tokens, u32 in_token_count,
    u32* out_tokens, u32 max_gen_tokens, u32 eos_id, f32 temp, f32 top_p);

/* gpt2.h:68, gpt2.c:231-256 */
f32 gpt2_compute_perplexity(GPT2Model* model, KVCache* caches, const u32* tokens, u32 n_tokens);

#ifdef __cplusplus
}
#endif

#endif
