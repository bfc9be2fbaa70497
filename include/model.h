/*
 * model.h -- LLaMA-family model, its config and the per-op entry points
 * (llamini.cpp model.h:1-134).
 *
 * Structs, enums and signatures match the reference exactly. The per-op
 * functions take host pointers like the reference; here each runs as a GPU
 * kernel with the operands copied in and out (correct, but not the fast path:
 * forward_step / generate_autoregressive keep everything on the device).
 */
#ifndef MODEL_H
#define MODEL_H

#include "common.h"
#include "tensor.h"
#include "kv_cache.h"
#include "gguf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* RoPE pairing (model.h:14): NORM rotates (i, i+1); NEOX rotates (j, j+head_dim/2). */
typedef enum { ROPE_NORM, ROPE_NEOX } RopeType;

/* Gate activation of the gated FFN (model.h:18). */
typedef enum { ACT_SILU, ACT_GELU } FfnAct;

/* model.h:24-40 */
typedef struct {
    u32 dim;
    u32 n_layers;
    u32 n_heads;
    u32 n_heads_kv;
    u32 head_dim;
    u32 ffn_dim;
    u32 vocab_size;
    u32 seq_len;
    f32 rms_eps;
    f32 rope_freq_base;
    RopeType rope_type;
    FfnAct ffn_act;
    int qkv_bias;
    f32 embedding_scale;
} LLaMAConfig;

/* model.h:46-59; shapes are (out_dim, in_dim). Bias tensors are NULL unless
 * cfg.qkv_bias is set. */
typedef struct {
    Tensor* attn_norm;
    Tensor* q_proj;
    Tensor* k_proj;
    Tensor* v_proj;
    Tensor* q_bias;
    Tensor* k_bias;
    Tensor* v_bias;
    Tensor* o_proj;
    Tensor* ffn_norm;
    Tensor* gate_proj;
    Tensor* up_proj;
    Tensor* down_proj;
} DecoderLayer;

/* model.h:62-68 */
typedef struct {
    LLaMAConfig cfg;
    Tensor* embeddings;
    DecoderLayer* layers;
    Tensor* final_norm;
    Tensor* lm_head;
} LLaMAModel;

/* out = x / sqrt(mean(x^2) + eps) * w (model.h:73, model.c:4-10). */
void rms_norm(f32* out, const f32* x, const f32* w, u32 dim, f32 eps);

/* out = act(gate) * up (model.h:78, model.c:20-25). */
void ffn_glu(f32* out, const f32* gate, const f32* up, u32 dim, FfnAct act);

/* In-place rotary embedding at position pos (model.h:82, model.c:31-58). */
void rope(f32* vec, u32 pos, u32 dim, u32 head_dim, f32 freq_base, RopeType type);

/* y[out_dim] = W[out_dim, in_dim] x[in_dim]; W eager f32 or lazy GGUF-quantized
 * (model.h:93, model.c:178-215). A lazy W whose bytes are already in GPU memory
 * is not re-uploaded. */
void linear(f32* out, const f32* x, const Tensor* w, u32 in_dim, u32 out_dim);

/* out += bias (model.h:98, model.c:27-29). */
void add_bias(f32* out, const f32* bias, u32 dim);

/* One token of grouped-query causal attention at position pos over the host
 * cache: stores k/v at pos, sets cur_seq = pos+1, attends positions 0..pos
 * (model.h:105, model.c:217-260). */
void causal_mha(const f32* q, const f32* k, const f32* v, KVCache* cache,
                f32* out, u32 pos, u32 n_heads, u32 n_heads_kv, u32 head_dim);

/* model.h:110-111, model.c:331-408 */
int llama_model_init(LLaMAModel* model, LLaMAConfig* cfg);
void llama_model_free(LLaMAModel* model);

/* Read hyperparameters from <arch>.* metadata with per-architecture quirks
 * (model.h:125, model.c:279-329). */
LLaMAConfig llama_config_from_gguf(GGUFFile* gf, LLaMAConfig defaults, char** arch_out);

/* Bind every weight (big matrices lazy, norms/biases eager) and upload the
 * quantized bytes to GPU memory unchanged. 0 or -1 (model.h:132, model.c:439-485). */
int llama_load_weights(LLaMAModel* model, GGUFFile* gf);

#ifdef __cplusplus
}
#endif

#endif
