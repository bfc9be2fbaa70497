/*
 * oracle.h -- CPU restatement of llamini.cpp's token loop. TEST INFRASTRUCTURE.
 *
 * This is the checker, not the product: only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load it. Every function restates one piece of the
 * reference's algorithm (cited file:line) in plain C, compiled with
 * -ffp-contract=off so the block decoders round exactly like the reference.
 *
 * Parity is pinned two ways: the decoders and ops are compared against the
 * reference's own code compiled from its sources into oracle/_ref/ (see
 * oracle/Makefile), and against the committed fixtures in tests/golden/ that
 * were produced by that build.
 */
#ifndef LLAMINI_ORACLE_H
#define LLAMINI_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (gguf.h:29-37 of the reference). */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q5_0 = 6,
    ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q5_K = 13, ORC_Q6_K = 14
};

/* Elements per block and bytes per block of a type; 0 if unsupported. */
uint32_t orc_block_elems(uint32_t type);
uint32_t orc_block_bytes(uint32_t type);

/* Half -> float, including subnormals/inf/nan (gguf.c:364-386). */
float orc_f16_to_f32(uint16_t h);

/* Decode n elements (a multiple of the block size) of raw blocks
 * (gguf.c:409-594). Returns 0, or -1 for a bad type or a misaligned n. */
int orc_dequant(uint32_t type, const uint8_t* raw, uint64_t n, float* out);

/* A weight matrix in its GGUF storage: rows x cols elements, raw bytes. */
typedef struct {
    uint32_t type;
    uint32_t rows;
    uint32_t cols;
    const uint8_t* data;
} OrcMat;

/* y[r] = sum_k W[r][k] x[k]: decode rows then an f32 dot per row
 * (model.c:66-73, model.c:159-176). Rows run in parallel (OpenMP); each dot
 * is a plain sequential sum, so the result does not depend on the thread count. */
void orc_linear(const OrcMat* w, const float* x, float* y);

/* Ops (model.c:4-58, model.c:217-260, gpt2.c:130-148). */
void orc_rms_norm(float* out, const float* x, const float* w, uint32_t dim, float eps);
void orc_layer_norm(float* out, const float* x, const float* w, const float* b, uint32_t dim, float eps);
float orc_gelu(float x);
void orc_ffn_glu(float* out, const float* gate, const float* up, uint32_t n, int act_gelu);
void orc_rope(float* vec, uint32_t pos, uint32_t dim, uint32_t head_dim, float base, int neox);
/* kcache/vcache: [max_seq][n_kv*head_dim] f32, written at pos. */
void orc_causal_mha(const float* q, const float* k, const float* v, float* kcache, float* vcache,
                    float* out, uint32_t pos, uint32_t n_heads, uint32_t n_kv, uint32_t head_dim);
uint32_t orc_greedy(const float* logits, uint32_t n);

/* ---- LLaMA-family forward pass (generate.c:62-120) ---- */
typedef struct {
    OrcMat q, k, v, o, gate, up, down;
    const float* attn_norm;
    const float* ffn_norm;
    const float* bq;      /* NULL unless qkv bias */
    const float* bk;
    const float* bv;
} OrcLlamaLayer;

typedef struct {
    uint32_t dim, n_layers, n_heads, n_heads_kv, head_dim, ffn_dim, vocab, max_seq;
    float rms_eps, rope_base, emb_scale;
    int rope_neox, act_gelu;
    OrcMat tok_embd;
    OrcMat lm_head;
    const float* final_norm;
    const OrcLlamaLayer* layers;
} OrcLlama;

typedef struct OrcState OrcState;

OrcState* orc_llama_state_new(const OrcLlama* m);
void orc_state_free(OrcState* s);

/* One token at position pos. logits: vocab floats. trace (optional):
 * n_layers x dim residual stream after each layer. */
void orc_llama_forward(const OrcLlama* m, OrcState* s, uint32_t pos, uint32_t token,
                       float* logits, float* trace);

/* Greedy generate_autoregressive (generate.c:122-167) with temp = 0. Returns the
 * total token count written to out (prompt + generated). */
uint32_t orc_llama_generate(const OrcLlama* m, OrcState* s, const uint32_t* prompt, uint32_t n_prompt,
                            uint32_t* out, uint32_t max_gen, uint32_t eos);

/* ---- GPT-2 forward pass (gpt2.c:150-192) ---- */
typedef struct {
    const float *attn_norm_w, *attn_norm_b;
    OrcMat qkv; const float* qkv_b;
    OrcMat out; const float* out_b;
    const float *ffn_norm_w, *ffn_norm_b;
    OrcMat up; const float* up_b;
    OrcMat down; const float* down_b;
} OrcGpt2Layer;

typedef struct {
    uint32_t dim, n_layers, n_heads, ffn_dim, vocab, n_ctx, max_seq;
    float ln_eps;
    OrcMat tok_embd;   /* rows are decoded per lookup */
    OrcMat pos_embd;
    const float *out_norm_w, *out_norm_b;
    OrcMat lm_head;
    const OrcGpt2Layer* layers;
} OrcGpt2;

OrcState* orc_gpt2_state_new(const OrcGpt2* m);
void orc_gpt2_forward(const OrcGpt2* m, OrcState* s, uint32_t pos, uint32_t token,
                      float* logits, float* trace);
uint32_t orc_gpt2_generate(const OrcGpt2* m, OrcState* s, const uint32_t* prompt, uint32_t n_prompt,
                           uint32_t* out, uint32_t max_gen, uint32_t eos);

#ifdef __cplusplus
}
#endif

#endif
