// gguf.cpp -- GGUF v2/v3 reader behind gguf.h (llamini.cpp gguf.c:1-354).
//
// Host-side file handling: mmap, header / metadata / tensor-info parsing with
// the same fail-closed limits as the reference (gguf.c:16-19, 139-207), and the
// metadata accessors. The two dequantize entry points validate the requested
// range exactly like gguf.c:409-416 and the per-type checks of gguf.c:417-590,
// then decode on the GPU (k_ops.cu, quant.cuh) and copy the f32 result back.
#include "internal.h"
#include "llamini_b200.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdlib>
#include <cstring>

namespace {

// Limits on file-controlled counts (same values as gguf.c:16-19).
constexpr uint64_t kMaxKv = 1u << 16;
constexpr uint64_t kMaxTensors = 1u << 20;
constexpr uint64_t kMaxArray = 1ull << 26;
constexpr uint64_t kMaxStr = 1u << 20;

// Bounds-checked reader: once a read would leave the file every later read is
// refused, so one check at the end of a record is enough.
struct Reader {
    const uint8_t* base;
    uint64_t size, pos;
    bool ok;

    bool take(void* dst, uint64_t n) {
        if (!ok || pos > size || n > size - pos) { ok = false; return false; }
        if (dst) memcpy(dst, base + pos, n);
        pos += n;
        return true;
    }
    uint32_t u32() { uint32_t v = 0; take(&v, 4); return v; }
    uint64_t u64() { uint64_t v = 0; take(&v, 8); return v; }
    char* str() {
        uint64_t n = u64();
        if (!ok || n > kMaxStr) { ok = false; return nullptr; }
        char* s = (char*)malloc(n + 1);
        if (!s) { ok = false; return nullptr; }
        if (!take(s, n)) { free(s); return nullptr; }
        s[n] = '\0';
        return s;
    }
    void skip_str() { uint64_t n = u64(); take(nullptr, n); }
};

uint64_t scalar_size(uint32_t t) {
    switch (t) {
    case GGUF_TYPE_UINT8: case GGUF_TYPE_INT8: case GGUF_TYPE_BOOL: return 1;
    case GGUF_TYPE_UINT16: case GGUF_TYPE_INT16: return 2;
    case GGUF_TYPE_UINT32: case GGUF_TYPE_INT32: case GGUF_TYPE_FLOAT32: return 4;
    case GGUF_TYPE_UINT64: case GGUF_TYPE_INT64: case GGUF_TYPE_FLOAT64: return 8;
    default: return 0;
    }
}

void release_tables(GGUFFile* gf) {
    if (gf->kv) {
        for (u64 i = 0; i < gf->n_kv; i++) free(gf->kv[i].key);
        free(gf->kv);
        gf->kv = nullptr;
    }
    if (gf->tensors) {
        for (u64 i = 0; i < gf->n_tensors; i++) free(gf->tensors[i].name);
        free(gf->tensors);
        gf->tensors = nullptr;
    }
}

bool file_bytes(const GGUFFile* gf, uint64_t off, void* dst, uint64_t n) {
    if (off > gf->size || n > gf->size - off) return false;
    memcpy(dst, (const uint8_t*)gf->data + off, n);
    return true;
}

const GGUFMeta* meta(const GGUFFile* gf, const char* key) {
    for (u64 i = 0; i < gf->n_kv; i++)
        if (gf->kv[i].key && strcmp(gf->kv[i].key, key) == 0) return &gf->kv[i];
    return nullptr;
}

bool parse(GGUFFile* gf) {
    Reader r{(const uint8_t*)gf->data, gf->size, 0, true};
    gf->hdr.magic = r.u32();
    gf->hdr.version = r.u32();
    gf->hdr.n_tensors = r.u64();
    gf->hdr.n_metadata = r.u64();
    if (!r.ok || gf->hdr.magic != GGUF_MAGIC) return false;
    if (gf->hdr.version != 2 && gf->hdr.version != 3) return false;   // v1 used 32-bit counts
    if (gf->hdr.n_metadata > kMaxKv || gf->hdr.n_tensors > kMaxTensors) return false;
    // Each entry needs a minimum number of bytes, so the counts are bounded by
    // what is left of the file (gguf.c:144-150).
    const uint64_t left = gf->size - r.pos;
    if (gf->hdr.n_metadata > left / 12 || gf->hdr.n_tensors > left / 24) return false;

    gf->n_kv = gf->hdr.n_metadata;
    gf->kv = (GGUFMeta*)calloc(gf->n_kv ? gf->n_kv : 1, sizeof(GGUFMeta));
    if (!gf->kv) return false;
    for (u64 i = 0; i < gf->n_kv; i++) {
        GGUFMeta* m = &gf->kv[i];
        m->key = r.str();
        m->type = r.u32();
        if (!r.ok) return false;
        if (m->type == GGUF_TYPE_ARRAY) {
            m->arr_elem_type = r.u32();
            m->arr_len = r.u64();
            m->value_off = r.pos;
            if (!r.ok || m->arr_len > kMaxArray) return false;
            const uint64_t rem = r.pos > r.size ? 0 : r.size - r.pos;
            if (m->arr_elem_type == GGUF_TYPE_STRING) {
                if (m->arr_len > rem / 8) return false;          // >= 8 bytes per string
                for (u64 j = 0; j < m->arr_len && r.ok; j++) r.skip_str();
            } else {
                const uint64_t es = scalar_size(m->arr_elem_type);
                if (es == 0 || m->arr_len > rem / es) return false;  // divide, never multiply
                r.take(nullptr, es * m->arr_len);
            }
        } else {
            m->value_off = r.pos;
            if (m->type == GGUF_TYPE_STRING) r.skip_str();
            else {
                const uint64_t es = scalar_size(m->type);
                if (es == 0) return false;
                r.take(nullptr, es);
            }
        }
        if (!r.ok) return false;
    }

    gf->n_tensors = gf->hdr.n_tensors;
    gf->tensors = (GGUFTensorInfo*)calloc(gf->n_tensors ? gf->n_tensors : 1, sizeof(GGUFTensorInfo));
    if (!gf->tensors) return false;
    const uint64_t cap = gf->size * 8;      // nothing is stored in under a bit per element
    for (u64 i = 0; i < gf->n_tensors; i++) {
        GGUFTensorInfo* t = &gf->tensors[i];
        t->name = r.str();
        t->n_dims = r.u32();
        if (!r.ok || t->n_dims == 0 || t->n_dims > 4) return false;
        uint64_t count = 1;
        for (u32 d = 0; d < t->n_dims; d++) {
            t->dims[d] = r.u64();
            if (!r.ok || t->dims[d] == 0 || t->dims[d] > cap) return false;
            count *= t->dims[d];
            if (count > cap) return false;
        }
        for (u32 d = t->n_dims; d < 4; d++) t->dims[d] = 1;
        t->ggml_type = r.u32();
        t->offset = r.u64();
        if (!r.ok || t->offset > gf->size) return false;
    }

    uint32_t align = gguf_get_u32(gf, "general.alignment", 32);
    if (align == 0) align = 32;
    gf->tensor_offset = (r.pos + align - 1) / align * align;
    return true;
}

// Element-range validation of gguf.c:409-416 plus the per-type checks; on
// success *raw / *nbytes describe the blocks covering [e0, e1).
bool check_range(const GGUFFile* gf, const GGUFTensorInfo* info, u64 e0, u64 e1,
                 const uint8_t** raw, uint64_t* nbytes) {
    const u64 n = gguf_tensor_count(info);
    if (e1 > n || e0 > e1) return false;
    const u64 abs_off = gf->tensor_offset + info->offset;
    if (abs_off < info->offset) return false;
    lm::TypeInfo ti;
    if (!lm::type_info(info->ggml_type, &ti)) return false;
    if (ti.block_elems == 1) {
        if (abs_off > gf->size || e1 * ti.block_bytes > gf->size - abs_off) return false;
        *raw = (const uint8_t*)gf->data + abs_off + e0 * ti.block_bytes;
        *nbytes = (e1 - e0) * ti.block_bytes;
        return true;
    }
    if (e0 % ti.block_elems || e1 % ti.block_elems || n % ti.block_elems) return false;
    if (abs_off > gf->size || n / ti.block_elems * ti.block_bytes > gf->size - abs_off) return false;
    *raw = (const uint8_t*)gf->data + abs_off + e0 / ti.block_elems * ti.block_bytes;
    *nbytes = (e1 - e0) / ti.block_elems * ti.block_bytes;
    return true;
}

int decode_range(GGUFFile* gf, const GGUFTensorInfo* info, u64 e0, u64 e1, f32* out) {
    const uint8_t* raw = nullptr;
    uint64_t nbytes = 0;
    if (!check_range(gf, info, e0, e1, &raw, &nbytes)) return -1;
    if (e1 == e0) return 0;
    if (info->ggml_type == GGML_TYPE_F32) {          // a plain copy (gguf.c:417-420)
        memcpy(out, raw, nbytes);
        return 0;
    }
    return llamini_dequant_host(info->ggml_type, raw, e1 - e0, out);
}

}  // namespace

extern "C" {

int gguf_open(const char* path, GGUFFile* gf) {
    memset(gf, 0, sizeof(GGUFFile));
    gf->fd = open(path, O_RDONLY);
    if (gf->fd < 0) return -1;
    struct stat st;
    if (fstat(gf->fd, &st) != 0 || st.st_size < 0) { close(gf->fd); return -1; }
    gf->size = (size_t)st.st_size;
    gf->data = mmap(nullptr, gf->size, PROT_READ, MAP_PRIVATE, gf->fd, 0);
    if (gf->data == MAP_FAILED) { close(gf->fd); return -1; }
    posix_fadvise(gf->fd, 0, (off_t)gf->size, POSIX_FADV_SEQUENTIAL);
    if (!parse(gf)) {
        release_tables(gf);
        munmap(gf->data, gf->size);
        close(gf->fd);
        memset(gf, 0, sizeof(GGUFFile));
        gf->fd = -1;
        return -1;
    }
    posix_madvise(gf->data, gf->size, POSIX_MADV_RANDOM);
    return 0;
}

void gguf_close(GGUFFile* gf) {
    lm::drop_gguf(gf);
    release_tables(gf);
    if (gf->data) munmap(gf->data, gf->size);
    if (gf->fd >= 0) close(gf->fd);
}

int gguf_read_f32(GGUFFile* gf, u64 offset, f32* out, u64 elem_cnt) {
    const u64 need = elem_cnt * sizeof(f32);
    if (gf->tensor_offset > gf->size) return -1;
    u64 avail = gf->size - gf->tensor_offset;
    if (offset > avail) return -1;
    avail -= offset;
    if (need > avail) return -1;
    memcpy(out, (const uint8_t*)gf->data + gf->tensor_offset + offset, need);
    return 0;
}

u32 gguf_get_u32(GGUFFile* gf, const char* key, u32 def_val) {
    const GGUFMeta* m = meta(gf, key);
    if (!m) return def_val;
    switch (m->type) {
    case GGUF_TYPE_UINT32: case GGUF_TYPE_INT32: { u32 v; return file_bytes(gf, m->value_off, &v, 4) ? v : def_val; }
    case GGUF_TYPE_UINT16: case GGUF_TYPE_INT16: { u16 v; return file_bytes(gf, m->value_off, &v, 2) ? v : def_val; }
    case GGUF_TYPE_UINT8: case GGUF_TYPE_INT8: { u8 v; return file_bytes(gf, m->value_off, &v, 1) ? v : def_val; }
    case GGUF_TYPE_UINT64: case GGUF_TYPE_INT64: { u64 v; return file_bytes(gf, m->value_off, &v, 8) ? (u32)v : def_val; }
    default: return def_val;
    }
}

f32 gguf_get_f32(GGUFFile* gf, const char* key, f32 def_val) {
    const GGUFMeta* m = meta(gf, key);
    if (!m) return def_val;
    if (m->type == GGUF_TYPE_FLOAT32) { f32 v; return file_bytes(gf, m->value_off, &v, 4) ? v : def_val; }
    if (m->type == GGUF_TYPE_FLOAT64) { double v; return file_bytes(gf, m->value_off, &v, 8) ? (f32)v : def_val; }
    return def_val;
}

char* gguf_get_str(GGUFFile* gf, const char* key) {
    const GGUFMeta* m = meta(gf, key);
    if (!m || m->type != GGUF_TYPE_STRING) return nullptr;
    u64 n;
    if (!file_bytes(gf, m->value_off, &n, 8) || n > kMaxStr) return nullptr;
    char* s = (char*)malloc(n + 1);
    if (!s) return nullptr;
    if (!file_bytes(gf, m->value_off + 8, s, n)) { free(s); return nullptr; }
    s[n] = '\0';
    return s;
}

u64 gguf_meta_array_len(GGUFFile* gf, const char* key, u32* elem_type_out) {
    const GGUFMeta* m = meta(gf, key);
    if (!m || m->type != GGUF_TYPE_ARRAY) return 0;
    if (elem_type_out) *elem_type_out = m->arr_elem_type;
    return m->arr_len;
}

char** gguf_get_string_array(GGUFFile* gf, const char* key, u64* count_out) {
    if (count_out) *count_out = 0;
    const GGUFMeta* m = meta(gf, key);
    if (!m || m->type != GGUF_TYPE_ARRAY || m->arr_elem_type != GGUF_TYPE_STRING) return nullptr;
    if (m->arr_len > kMaxArray) return nullptr;
    char** a = (char**)calloc(m->arr_len ? m->arr_len : 1, sizeof(char*));
    if (!a) return nullptr;
    Reader r{(const uint8_t*)gf->data, gf->size, m->value_off, true};
    for (u64 i = 0; i < m->arr_len; i++) {
        a[i] = r.str();
        if (!r.ok) {
            for (u64 j = 0; j <= i; j++) free(a[j]);
            free(a);
            return nullptr;
        }
    }
    if (count_out) *count_out = m->arr_len;
    return a;
}

static void* scalar_array(GGUFFile* gf, const char* key, u32 want, u64* count_out) {
    if (count_out) *count_out = 0;
    const GGUFMeta* m = meta(gf, key);
    if (!m || m->type != GGUF_TYPE_ARRAY || m->arr_elem_type != want) return nullptr;
    if (m->arr_len > kMaxArray) return nullptr;
    void* a = malloc((m->arr_len ? m->arr_len : 1) * 4);
    if (!a) return nullptr;
    if (!file_bytes(gf, m->value_off, a, m->arr_len * 4)) { free(a); return nullptr; }
    if (count_out) *count_out = m->arr_len;
    return a;
}

f32* gguf_get_f32_array(GGUFFile* gf, const char* key, u64* count_out) {
    return (f32*)scalar_array(gf, key, GGUF_TYPE_FLOAT32, count_out);
}

i32* gguf_get_i32_array(GGUFFile* gf, const char* key, u64* count_out) {
    return (i32*)scalar_array(gf, key, GGUF_TYPE_INT32, count_out);
}

const GGUFTensorInfo* gguf_find_tensor(GGUFFile* gf, const char* name) {
    for (u64 i = 0; i < gf->n_tensors; i++)
        if (gf->tensors[i].name && strcmp(gf->tensors[i].name, name) == 0) return &gf->tensors[i];
    return nullptr;
}

u64 gguf_tensor_count(const GGUFTensorInfo* info) {
    u64 n = 1;
    for (u32 d = 0; d < info->n_dims; d++) n *= info->dims[d];
    return n;
}

int gguf_dequantize_tensor(GGUFFile* gf, const GGUFTensorInfo* info, f32* out, u64 out_count) {
    const u64 n = gguf_tensor_count(info);
    if (n != out_count) return -1;
    return decode_range(gf, info, 0, n, out);
}

int gguf_dequantize_rows(GGUFFile* gf, const GGUFTensorInfo* info, u32 row0, u32 row1, u32 row_len, f32* out) {
    if (row1 < row0) return -1;
    return decode_range(gf, info, (u64)row0 * row_len, (u64)row1 * row_len, out);
}

}  // extern "C"
