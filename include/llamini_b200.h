/*
 * llamini_b200.h -- additive C entry points of the B200 library.
 *
 * Everything here is new: the reference (llamini.cpp) has no GPU, no batching
 * and no device-resident sessions, so none of these functions replaces a
 * reference symbol one-for-one. Each comment names the reference code whose
 * behaviour the function exposes or extends. All functions return 0 on success
 * and -1 on failure unless stated otherwise; the reason is kept in
 * llamini_last_error(). No function aborts the process.
 */
#ifndef LLAMINI_B200_H
#define LLAMINI_B200_H

#include "common.h"
#include "gguf.h"
#include "model.h"
#include "gpt2.h"
#include "kv_cache.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- runtime --------------------------------------------------------------- */

/* Sticky description of the last failure ("" if none). The reference reports
 * errors only through -1 returns and stderr (gguf.h comments, main.c:472-477). */
const char* llamini_last_error(void);
void llamini_clear_error(void);

/* Number of visible CUDA devices (0 without a GPU; never fails). */
int llamini_device_count(void);

/* Select the CUDA device used by every later call of this process. Must be
 * called before the first model is loaded. Default: device 0, or the value of
 * the LLAMINI_DEVICE environment variable. */
int llamini_set_device(int device);

/* The library's CUDA stream (a cudaStream_t) on the current device, created on
 * first use; NULL without a device. Timing code records events on it. */
void* llamini_stream(void);

/* Release every device resource the library holds (weights, KV caches, graphs). */
void llamini_release(void);

/* ---- block decoders and GEMV on raw blocks (the gguf.c:409-594 and
 *      model.c:66-176 hot loops, exposed without a GGUF file) ------------------ */

/* Bytes taken by n_elems elements of ggml `type` (0 if the type is unsupported
 * or n_elems is not a multiple of its block size). */
u64 llamini_type_bytes(u32 type, u64 n_elems);

/* Decode n_elems elements of raw `type` blocks from host memory into host f32
 * out, on the GPU. Bit-identical to gguf.c:409-594. */
int llamini_dequant_host(u32 type, const void* blocks, u64 n_elems, f32* out);

/* One sample_token draw (generate.c:25-60) by the device sampler that the
 * sampled generate path uses: logits in host memory (vocab floats), temp > 0,
 * top_p, and u = rand() / (RAND_MAX + 1) as the reference computes it (the
 * caller draws it, so the host rand() stream is consumed in the reference's
 * order). Returns the token id, or 0xFFFFFFFF on error. */
u32 llamini_sample_host(const f32* logits, u32 vocab, f32 temp, f32 top_p, f32 u);

/* Same decode between device buffers, enqueued on llamini_stream(). */
int llamini_dequant_device(u32 type, const void* d_blocks, u64 n_elems, f32* d_out);

/* y[b][r] = sum_k W[r][k] * x[b][k] for b < batch, W given as raw `type` rows of
 * `cols` elements (cols a multiple of the block size). Host buffers; x is
 * batch x cols f32, y is batch x rows f32 (model.c:66-73 per column). */
int llamini_gemv_host(u32 type, const void* w, u32 rows, u32 cols,
                      const f32* x, u32 batch, f32* y);

/* Device-pointer form of llamini_gemv_host, enqueued on llamini_stream(). */
int llamini_gemv_device(u32 type, const void* d_w, u32 rows, u32 cols,
                        const f32* d_x, u32 batch, f32* d_y);

/* Decode attention for one query position over caller-owned DEVICE buffers,
 * with no device allocation. No counterpart in the reference: it computes what
 * causal_mha (model.c:217-260) computes after the cache already holds position
 * pos (the reference stores k/v first, model.c:222-224). d_q and d_out are
 * n_heads x head_dim f32; d_key/d_val are f32 caches laid out like KVCache
 * (row p = position p, n_heads_kv x head_dim) holding rows 0..pos. The work is
 * enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream) of the
 * calling thread's current device.
 * For callers that may not allocate on their path (an engine whose page pool
 * already holds nearly all of HBM, a loop that cannot take cudaFree's implicit
 * device synchronisation): split partials and completion counters live in a
 * fixed 1 MiB (+1 KiB) array in the library's device memory. Limits: n_heads
 * <= 256, head_dim <= 256; larger requests fail with -1 and a message. The
 * counters start at zero and every call returns them to zero. The first call
 * on a device does the set-up (scratch address, kernel attribute) and should
 * come before any stream capture; it is kept for the life of the process, so
 * it does not survive a cudaDeviceReset of that device by the application.
 * Calls that overlap in time on one device (two streams, or unordered host
 * threads) share the scratch and race. */
int llamini_causal_mha_noalloc(const f32* d_q, const f32* d_key, const f32* d_val, f32* d_out,
                               u32 pos, u32 n_heads, u32 n_heads_kv, u32 head_dim, void* stream);

/* ---- device-resident decoding sessions (generate.c:122-167 without host
 *      round trips) --------------------------------------------------------- */

typedef struct llamini_session llamini_session;

/* Session for a loaded LLaMA-family model and its per-layer caches. The session
 * owns the device KV cache, the step graph and the token buffer; it is created
 * on first use by forward_step/generate_autoregressive as well, and this call
 * returns that same session. NULL on failure. */
llamini_session* llamini_llama_session(LLaMAModel* model, KVCache* caches);

/* Same for a GPT-2 model (gpt2.c:150-229). */
llamini_session* llamini_gpt2_session(GPT2Model* model, KVCache* caches);

/* Reset the session to position 0 with the given prompt (n_prompt >= 1). */
int llamini_session_begin(llamini_session* s, const u32* prompt, u32 n_prompt);

/* Enqueue n_steps forward passes without waiting. Step at position p embeds
 * token[p]; when p+1 >= n_prompt it also stores the greedy token as token[p+1].
 * Fails if the run would pass the cache capacity. */
int llamini_session_step(llamini_session* s, u32 n_steps);

/* Wait for queued steps, then copy token[0..n) to host out. Returns the number
 * of valid tokens (prompt + generated), or -1. */
int llamini_session_tokens(llamini_session* s, u32* out, u32 n);

/* Wait, then copy the logits of the most recent step (vocab_size floats). */
int llamini_session_logits(llamini_session* s, f32* out);

/* Current position (number of tokens already run through the stack). */
u32 llamini_session_pos(llamini_session* s);

/* How the session runs its steps: 2 = the dataflow decode kernel (one
 * cooperative launch for up to 64 steps; the default for LLaMA-family models
 * whose matrices are all Q4_K / Q6_K with K a multiple of 256 up to 6144),
 * 1 = the earlier persistent decode kernel (LLAMINI_DECODE_KERNEL=1 at session
 * creation, every matrix Q4_K, Q6_K, Q8_0 or Q4_0), 0 = one graph of per-op
 * kernels per step (every other model, or LLAMINI_DECODE_KERNEL=0); -1 = NULL. */
int llamini_session_kernel(llamini_session* s);

/* Algorithmic bytes one step reads: every weight matrix once, norms, biases and
 * one embedding row (the quantized sizes of gguf.c's block formats). */
u64 llamini_session_weight_bytes(llamini_session* s);

/* KV-cache bytes per cached position (all layers, K and V). */
u64 llamini_session_kv_bytes_per_pos(llamini_session* s);

/* Element type of the device KV cache of sessions created from now on:
 * 0 = f32 (default; the reference keeps an f32 cache, model.c:222-224, and the
 * f32 cache holds the 1e-3 parity bar), 1 = fp16 (half the cache traffic; on
 * the synthetic models its rounding moves logits by ~2e-3 relative L2). */
int llamini_set_kv_f16(int enable);

/* ---- batched decode (no counterpart in the reference, which decodes one
 *      sequence at a time: generate.c:122-167 run for each sequence) ---------- */

typedef struct llamini_batch llamini_batch;

/* A batch of up to max_batch (<= 64) independent sequences of at most max_seq
 * positions over a loaded model. Every weight matrix is read once per step for
 * the whole batch; the device KV cache holds max_batch x max_seq positions. The
 * matrices may be any of gguf.c's block formats or F16 with rows of a multiple
 * of 64 elements (256 for K-quants); NULL and a message otherwise.
 * Free it with llamini_batch_free before the model and its GGUF file. */
llamini_batch* llamini_llama_batch(LLaMAModel* model, u32 max_batch, u32 max_seq);
llamini_batch* llamini_gpt2_batch(GPT2Model* model, u32 max_batch, u32 max_seq);

/* Start n_seq sequences at position 0: prompts holds the n_seq prompts back to
 * back, prompt_lens their lengths (each >= 1). */
int llamini_batch_begin(llamini_batch* b, u32 n_seq, const u32* prompts, const u32* prompt_lens);

/* Enqueue n_steps positions of every sequence. At position p sequence s embeds
 * token[s][p]; once p + 1 is past its prompt its greedy token becomes
 * token[s][p + 1] -- per sequence exactly generate_autoregressive with temp 0
 * and no EOS (an EOS is for the caller to cut at). */
int llamini_batch_step(llamini_batch* b, u32 n_steps);

/* Wait, copy token[seq][0..n) to out; returns the number of valid tokens. */
int llamini_batch_tokens(llamini_batch* b, u32 seq, u32* out, u32 n);

/* Wait, copy the logits of sequence seq at the most recent step. */
int llamini_batch_logits(llamini_batch* b, u32 seq, f32* out);

u32 llamini_batch_pos(llamini_batch* b);
u64 llamini_batch_weight_bytes(llamini_batch* b);
void llamini_batch_free(llamini_batch* b);

/* Prompt positions whose logits nobody reads (generate_autoregressive's
 * prefill, llamini_session_step inside the prompt) run in chunks of 64
 * positions through the tcgen05 GEMM, with causal attention over the cache, when
 * every matrix takes the tensor-core path (one at a time otherwise): 1 = on (the
 * default), 0 = one position at a time, -1 = the default again
 * (LLAMINI_PREFILL=0 in the environment turns it off). The last prompt position
 * always runs through the decode step, which produces the logits. */
int llamini_set_prefill(int enable);

/* Whether this session's prompts have run through chunked prefill: 1 = yes (its
 * buffers are built), -1 = not available for this model (a format or shape the
 * tensor-core GEMM does not take, or a tensor-parallel group), 0 = not tried
 * yet; -2 = NULL. */
int llamini_session_prefill(llamini_session* s);

/* ---- tensor parallelism (no counterpart in the reference): LLaMA models split
 *      over the GPUs of one box, one process per GPU --------------------------- */

/* This process's 64-byte device-memory handle (a cudaIpcMemHandle_t) for the
 * allreduce buffer the other ranks read; pass every rank's to llamini_tp_join. */
int llamini_tp_handle(void* out64);

/* Join a group of `world` ranks as `rank`; handles = world handles of 64 bytes
 * in rank order. LLaMA sessions created afterwards hold this rank's shard:
 * heads [rank*H/world, (rank+1)*H/world) of q and o (o split by its columns),
 * the matching kv heads, and FFN columns split on 256-column boundaries (gate/up
 * rows, down columns); embeddings, norms and lm_head are whole, so every rank
 * computes the same logits. After the o projection and after ffn_down the
 * ranks' partial sums are added over NVLink (bounded waits; a rank that does not
 * arrive within 2 s sets the session's error). world = 1 leaves the group setting
 * at one rank. Prompt chunks (prefill) and batched sessions (LLaMA family, on
 * the tensor-core GEMM, at most 524288 / dim sequences) add their columns'
 * partial sums the same way, slice by slice. */
int llamini_tp_join(u32 rank, u32 world, const void* handles);
/* Leave the group (after the device has finished every step of the group's
 * sessions): unmaps the peers' buffers and clears this rank's buffer and
 * counters, so the process can join another group. Every rank of the group
 * leaves, and the ranks pass a host barrier before any of them joins again.
 * Sessions built in the group must not step afterwards. Returns 0 (also when
 * not in a group), -1 on a CUDA error. */
int llamini_tp_leave(void);
/* The shard a LLaMA session of rank `rank` in a group of `world` holds (the
 * plan llamini_tp_join's sessions use; no device needed): out[0..8) = {first
 * head, end head, first kv head, end kv head, first FFN column, end FFN column,
 * first o-proj column, end o-proj column}. FFN columns split on 256-column
 * super-block boundaries as evenly as they allow (first = 256 * floor(n_sb *
 * rank / world)). Returns 0, or -1 when the shapes do not split. */
int llamini_tp_plan(u32 world, u32 rank, u32 n_heads, u32 n_kv, u32 head_dim, u32 ffn, u32* out);
int llamini_tp_rank(void);
int llamini_tp_world(void);

/* Which GEMM a batch runs its matrices on: 1 = the tcgen05 tensor-core GEMM
 * (weights dequantised once per step into fp16 hi + lo, f32 accumulation in
 * tensor memory), 0 = the mma.sync GEMM; -1 = NULL. */
int llamini_batch_gemm_kind(llamini_batch* b);

/* GEMM for batched products (batches and the batch columns of llamini_gemv_*)
 * created or called from now on: 1 = tcgen05 (the default), 0 = mma.sync,
 * -1 = the default again (LLAMINI_BATCH_GEMM=mma in the environment selects
 * mma.sync). Shapes the tcgen05 GEMM does not take use mma.sync either way. */
int llamini_set_batch_gemm(int kind);

/* Per-layer residual stream of the most recent step: n_layers x dim floats,
 * captured when `enable` was set before the step ran. For parity tests. */
int llamini_session_trace(llamini_session* s, int enable);
int llamini_session_trace_read(llamini_session* s, f32* out);

#ifdef __cplusplus
}
#endif

#endif
