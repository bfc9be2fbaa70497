/*
 * gguf.h -- GGUF file access and block dequantization (llamini.cpp gguf.h:1-149).
 *
 * Same types, constants and function signatures as the reference header; the
 * implementation behind them is this library's own. Parsing and metadata access
 * run on the host (they are file handling, not the token loop). The two
 * dequantize entry points run the block decoders on the GPU and copy the f32
 * result back, bit-identical to the reference's CPU decoders.
 */
#ifndef GGUF_H
#define GGUF_H

#include "common.h"

#ifdef __cplusplus
extern "C" {
#endif

/* "GGUF" little-endian (gguf.h:7). */
#define GGUF_MAGIC 0x46554747

/* Metadata value type tags as stored on disk (gguf.h:10-24). */
typedef enum {
    GGUF_TYPE_UINT8   = 0,
    GGUF_TYPE_INT8    = 1,
    GGUF_TYPE_UINT16  = 2,
    GGUF_TYPE_INT16   = 3,
    GGUF_TYPE_UINT32  = 4,
    GGUF_TYPE_INT32   = 5,
    GGUF_TYPE_FLOAT32 = 6,
    GGUF_TYPE_BOOL    = 7,
    GGUF_TYPE_STRING  = 8,
    GGUF_TYPE_ARRAY   = 9,
    GGUF_TYPE_UINT64  = 10,
    GGUF_TYPE_INT64   = 11,
    GGUF_TYPE_FLOAT64 = 12,
} GGUFValueType;

/* GGML tensor element types that can be decoded (gguf.h:29-37). Any other
 * type id makes the dequantize calls fail with -1. */
#define GGML_TYPE_F32   0
#define GGML_TYPE_F16   1
#define GGML_TYPE_Q4_0  2
#define GGML_TYPE_Q4_1  3
#define GGML_TYPE_Q5_0  6
#define GGML_TYPE_Q8_0  8
#define GGML_TYPE_Q4_K  12
#define GGML_TYPE_Q5_K  13
#define GGML_TYPE_Q6_K  14

/* One metadata entry (gguf.h:44-50). Scalars and arrays are referenced by the
 * byte offset of their payload in the mapped file and decoded on request. */
typedef struct {
    char* key;          /* owned, NUL-terminated */
    u32   type;         /* GGUFValueType */
    u64   value_off;    /* file offset of the value payload */
    u32   arr_elem_type;/* element type when type == GGUF_TYPE_ARRAY */
    u64   arr_len;      /* element count when type == GGUF_TYPE_ARRAY */
} GGUFMeta;

/* One tensor-info entry (gguf.h:53-59). dims are in ggml order (fastest first). */
typedef struct {
    char* name;
    u32   n_dims;
    u64   dims[4];
    u32   ggml_type;
    u64   offset;       /* relative to the start of the tensor-data section */
} GGUFTensorInfo;

/* Fixed file header (gguf.h:62-67). */
typedef struct {
    u32 magic;
    u32 version;
    u64 n_tensors;
    u64 n_metadata;
} GGUFHeader;

/* An opened, memory-mapped GGUF file (gguf.h:70-82). */
typedef struct {
    int fd;
    void* data;
    size_t size;
    GGUFHeader hdr;
    u64 tensor_offset;      /* aligned start of the tensor-data section */

    GGUFMeta* kv;
    u64 n_kv;

    GGUFTensorInfo* tensors;
    u64 n_tensors;
} GGUFFile;

/* Open + fully parse (header, metadata table, tensor table, aligned data
 * start). Returns 0, or -1 with *gf zeroed and fd = -1 (gguf.h:87, gguf.c:117-231). */
int gguf_open(const char* path, GGUFFile* gf);
/* Unmap and free everything gguf_open allocated (gguf.h:88, gguf.c:233-237). */
void gguf_close(GGUFFile* gf);

/* Copy elem_cnt raw f32 values from `offset` bytes into the tensor-data section;
 * -1 if the range leaves the file (gguf.h:92, gguf.c:239-250). */
int gguf_read_f32(GGUFFile* gf, u64 offset, f32* out, u64 elem_cnt);

/* Scalar metadata getters; return def_val when the key is missing or of another
 * type (gguf.h:97-98, gguf.c:256-274). */
u32 gguf_get_u32(GGUFFile* gf, const char* key, u32 def_val);
f32 gguf_get_f32(GGUFFile* gf, const char* key, f32 def_val);

/* malloc'd copy of a scalar STRING value, or NULL (gguf.h:104, gguf.c:276-286). */
char* gguf_get_str(GGUFFile* gf, const char* key);

/* Length of an ARRAY value (0 if absent), element type via *elem_type_out
 * (gguf.h:109, gguf.c:288-293). */
u64 gguf_meta_array_len(GGUFFile* gf, const char* key, u32* elem_type_out);

/* Array decoders; caller frees (gguf.h:115-124, gguf.c:295-338). */
char** gguf_get_string_array(GGUFFile* gf, const char* key, u64* count_out);
f32* gguf_get_f32_array(GGUFFile* gf, const char* key, u64* count_out);
i32* gguf_get_i32_array(GGUFFile* gf, const char* key, u64* count_out);

/* Tensor lookup by exact name; NULL if absent (gguf.h:128, gguf.c:344-348). */
const GGUFTensorInfo* gguf_find_tensor(GGUFFile* gf, const char* name);

/* Product of the tensor's dims (gguf.h:131, gguf.c:350-354). */
u64 gguf_tensor_count(const GGUFTensorInfo* info);

/* Decode the whole tensor to f32 into `out` (out_count must equal the element
 * count). 0 on success, -1 on a size mismatch, an out-of-file range, an
 * unsupported type, or no usable CUDA device (gguf.h:139, gguf.c:596-600). */
int gguf_dequantize_tensor(GGUFFile* gf, const GGUFTensorInfo* info, f32* out, u64 out_count);

/* Decode rows [row0,row1) of a tensor viewed as rows of row_len elements.
 * The element range must be block aligned, else -1 (gguf.h:147, gguf.c:602-605). */
int gguf_dequantize_rows(GGUFFile* gf, const GGUFTensorInfo* info, u32 row0, u32 row1, u32 row_len, f32* out);

#ifdef __cplusplus
}
#endif

#endif
