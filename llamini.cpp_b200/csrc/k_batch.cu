// k_batch.cu -- per-sequence embedding and token update of batched decode.
//
// Batched decode runs every sequence of the batch at the same position. Step
// at position p: sequence b embeds tokens[b][p] (tensor_get_row, tensor.c:24-30;
// GPT-2 adds the learned position row, gpt2.c:155-160), and afterwards its
// greedy token (generate.c:3-9, from the lm_head finish's argmax key) becomes
// tokens[b][p + 1] once p + 1 is past its prompt (generate.c:143-156).
#include "internal.h"
#include "pdl.cuh"
#include "rows.cuh"

namespace lm {

// grid B, 256 threads
__global__ void bembed_kernel(const BEmbedArgs a) {
    pdl_trigger();
    pdl_wait();                                    // the position and tokens come from the previous step
    const uint32_t b = blockIdx.x;
    const uint32_t pos = a.st->pos;
    uint32_t t = a.tokens[(uint64_t)b * a.tok_stride + pos];
    if (t >= a.tok.rows) t = 0;                    // out-of-range ids read row 0
    float* h = a.hidden + (uint64_t)b * a.dim;
    decode_row_part(a.tok, t, h, a.scale, false, threadIdx.x, blockDim.x);
    if (a.pos.ptr != nullptr) {
        __syncthreads();
        const uint32_t p = pos < a.pos.rows ? pos : a.pos.rows - 1;
        decode_row_part(a.pos, p, h, 1.0f, true, threadIdx.x, blockDim.x);
    }
}

// one CTA; thread b handles sequence b
__global__ void btoken_kernel(const BTokenArgs a) {
    pdl_trigger();
    pdl_wait();                                    // the argmax keys come from the lm_head finish
    const uint32_t pos = a.st->pos;
    for (uint32_t b = threadIdx.x; b < a.B; b += blockDim.x) {
        const unsigned long long k = a.keys[b];
        if (pos + 1 >= a.n_prompt[b] && pos + 1 < a.max_tokens)
            a.tokens[(uint64_t)b * a.tok_stride + pos + 1] = k ? 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull) : 0u;
        a.keys[b] = 0ull;
    }
    __syncthreads();
    if (threadIdx.x == 0) a.st->pos = pos + 1;
}

bool launch_bembed(const BEmbedArgs& a, uint32_t B, cudaStream_t st) {
    return LM_CUDA(launch_k(bembed_kernel, dim3(B), dim3(256), 0, st, a));
}
bool launch_btoken(const BTokenArgs& a, cudaStream_t st) {
    return LM_CUDA(launch_k(btoken_kernel, dim3(1), dim3(256), 0, st, a));
}

}  // namespace lm
