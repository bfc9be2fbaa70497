/*
 * kv_cache.h -- per-layer attention cache handle (llamini.cpp kv_cache.h:1-17).
 *
 * The struct and the two functions keep the reference's contract: key/val are
 * host buffers calloc'd by kv_cache_init that the caller releases with plain
 * free(). The GPU keeps its own fp16 copy of the cache (one per caches array,
 * created on the first forward pass that uses it); the host arrays are only
 * written by the host-pointer op causal_mha, and cur_seq is kept current by
 * every forward pass.
 */
#ifndef KV_CACHE_H
#define KV_CACHE_H

#include "common.h"
#include "tensor.h"

#ifdef __cplusplus
extern "C" {
#endif

/* kv_cache.h:7-13 */
typedef struct {
    f32* key;
    f32* val;
    u32 dim;
    u32 max_seq;
    u32 cur_seq;
} KVCache;

/* kv_cache.h:15 / kv_cache.c:3-9 */
void kv_cache_init(KVCache* cache, u32 dim, u32 max_seq);
/* kv_cache.h:16 / kv_cache.c:11-15 */
void kv_cache_reset(KVCache* cache);

#ifdef __cplusplus
}
#endif

#endif
