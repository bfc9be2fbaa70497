// rows.cuh -- decode one row of a GGUF table on the device (embedding lookups).
#pragma once

#include "internal.h"
#include "quant.cuh"

namespace lm {

// Decode row `row` of a table (rows of `cols` elements) into out, scaled
// (tensor_get_row, tensor.c:24-30); threads tid = 0..nth-1 share the work.
static __device__ __noinline__ void decode_row_part(const DevMat& m, uint32_t row, float* out, float scale, bool add,
                                                    uint32_t tid, uint32_t nth) {
    const uint8_t* r = m.ptr + (uint64_t)row * m.row_bytes;
    if (m.type == T_F32 || m.type == T_F16) {
        for (uint32_t i = tid; i < m.cols; i += nth) {
            float v = m.type == T_F32 ? reinterpret_cast<const float*>(r)[i]
                                      : f16_bits(reinterpret_cast<const unsigned short*>(r)[i]);
            v = v * scale;
            out[i] = add ? out[i] + v : v;
        }
        return;
    }
    const uint32_t units = m.cols / 32;
    for (uint32_t u = tid; u < units; u += nth) {
        float y[32];
        uint32_t blk = 0, v = 0, base = 0;
#define LM_DEC(T)                                                    \
        case T: {                                                    \
            blk = u / Fmt<T>::UPB; v = u % Fmt<T>::UPB;              \
            Fmt<T>::decode(r + (uint64_t)blk * Fmt<T>::BB, v, y);    \
            base = blk * Fmt<T>::BE;                                 \
            for (uint32_t i = 0; i < 32; i++) {                      \
                float t = y[i] * scale;                              \
                float* o = out + base + Fmt<T>::elem(v, i);          \
                *o = add ? *o + t : t;                               \
            }                                                        \
            break;                                                   \
        }
        switch (m.type) {
            LM_DEC(T_Q4_0) LM_DEC(T_Q4_1) LM_DEC(T_Q5_0) LM_DEC(T_Q8_0)
            LM_DEC(T_Q4_K) LM_DEC(T_Q5_K) LM_DEC(T_Q6_K)
            default: break;
        }
#undef LM_DEC
    }
}

}  // namespace lm
