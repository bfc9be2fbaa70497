/*
 * generate.h -- token loop of the LLaMA-family path (llamini.cpp generate.h:1-52).
 *
 * Same signatures and semantics as the reference. forward_step and
 * generate_autoregressive run the whole step on the GPU as a captured CUDA
 * graph; the argmax of greedy decoding happens on the device and only token ids
 * (and, for forward_step, the logits the caller asked for) cross to the host.
 */
#ifndef GENERATE_H
#define GENERATE_H

#include "common.h"
#include "tensor.h"
#include "kv_cache.h"
#include "model.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Index of the first strict maximum (generate.h:10, generate.c:3-9). */
u32 greedy_sample(const f32* logits, u32 vocab_size);

/* temp <= 0: greedy_sample. Otherwise temperature softmax + top-p nucleus draw
 * using rand() (generate.h:15, generate.c:25-60). */
u32 sample_token(const f32* logits, u32 vocab_size, f32 temp, f32 top_p);

/* One token through the full stack at position pos; writes vocab_size logits
 * to host logits_out (generate.h:24, generate.c:62-120). */
void forward_step(LLaMAModel* model, KVCache* caches, u32 pos, u32 token_id, f32* logits_out);

/* Prefill the prompt, then sample until eos_id, max_gen_tokens or the cache
 * capacity; returns prompt + generated count written to out_tokens
 * (generate.h:38, generate.c:122-167). */
u32 generate_autoregressive(LLaMAModel* model, KVCache* caches,
    u32* input_tokens, u32 in_token_count,
    u32* out_tokens, u32 max_gen_tokens, u32 eos_id, f32 temp, f32 top_p);

/* Teacher-forced perplexity over tokens[0..n_tokens) (generate.h:50, generate.c:169-197). */
f32 compute_perplexity(LLaMAModel* model, KVCache* caches, const u32* tokens, u32 n_tokens);

#ifdef __cplusplus
}
#endif

#endif
