/*
 * tensor.h -- the reference's Tensor handle (llamini.cpp tensor.h:1-36).
 *
 * A Tensor is either eager (data holds `size` host floats) or lazy (data is
 * NULL and src_gf/src_info name the GGUF tensor its rows come from). The layout
 * is caller-visible and identical to the reference. In this library a lazy
 * tensor's bytes also live in GPU memory once its model has been loaded; the
 * struct itself does not change.
 */
#ifndef TENSOR_H
#define TENSOR_H

#include "common.h"
#include "gguf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* tensor.h:16-23 */
typedef struct {
    u32 dims[4];
    u32 ndim;
    u32 size;
    f32* data;
    GGUFFile* src_gf;               /* non-NULL iff lazy */
    const GGUFTensorInfo* src_info; /* borrowed from src_gf->tensors */
} Tensor;

/* calloc'd eager tensor of the given shape (tensor.h:25, tensor.c:3-14). */
Tensor* tensor_create(u32 ndim, u32* shape);
/* Free data (NULL for lazy) and the handle (tensor.h:26, tensor.c:16-21). */
void tensor_free(Tensor* t);
/* C[m,n] = A[m,k] * B[k,n] on eager tensors, computed on the GPU
 * (tensor.h:27, tensor.c:32-45). */
void matmul(Tensor* A, Tensor* B, Tensor* C);
/* out = a + b and out = a * s over n floats, on the GPU (tensor.h:28-29, tensor.c:47-53). */
void vec_add(f32* out, const f32* a, const f32* b, u32 n);
void vec_scale(f32* out, const f32* a, f32 s, u32 n);

/* Copy logical row `row` (row_len elements) to host `out`: a memcpy for an
 * eager tensor, a one-row GPU dequant for a lazy one (tensor.h:35, tensor.c:24-30). */
void tensor_get_row(const Tensor* t, u32 row, u32 row_len, f32* out);

#ifdef __cplusplus
}
#endif

#endif
