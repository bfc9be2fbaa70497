// runtime.cpp -- process-wide state of libllamini_cuda.so: error reporting,
// device/stream selection, device allocation and the registry of GGUF tensors
// that have been copied to GPU memory.
#include "internal.h"
#include "llamini_b200.h"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

namespace lm {

// ---------------------------------------------------------------- errors
static char g_err[512] = "";

void set_error(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (strcmp(buf, g_err) != 0) fprintf(stderr, "[llamini-b200] %s\n", buf);
    memcpy(g_err, buf, sizeof(g_err));
}

bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    set_error("CUDA error %s (%d) in %s", cudaGetErrorString(e), (int)e, what);
    return false;
}

// ---------------------------------------------------------------- device
static int g_device = -1;          // selected device, -1 = not yet initialised
static int g_requested = -1;
static bool g_failed = false;
static cudaStream_t g_stream = nullptr;
static int g_sms = 148;

bool ensure_device() {
    if (g_device >= 0) return true;
    if (g_failed) { set_error("no usable CUDA device"); return false; }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        g_failed = true;
        set_error("no usable CUDA device (this library has no CPU path)");
        return false;
    }
    int dev = g_requested;
    if (dev < 0) {
        const char* e = getenv("LLAMINI_DEVICE");
        dev = e ? atoi(e) : 0;
    }
    if (dev < 0 || dev >= n) { set_error("device %d out of range (%d devices)", dev, n); g_failed = true; return false; }
    if (!LM_CUDA(cudaSetDevice(dev))) { g_failed = true; return false; }
    cudaDeviceProp p;
    if (!LM_CUDA(cudaGetDeviceProperties(&p, dev))) { g_failed = true; return false; }
    if (p.major < 10) {
        set_error("device %d is sm_%d%d; this library is built for sm_100a only", dev, p.major, p.minor);
        g_failed = true;
        return false;
    }
    g_sms = p.multiProcessorCount;
    if (!LM_CUDA(cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking))) { g_failed = true; return false; }
    if (!kernels_init()) { g_failed = true; return false; }
    g_device = dev;
    return true;
}

cudaStream_t stream() { return g_stream; }

// Programmatic dependent launch between the step's kernels; LLAMINI_PDL=0
// turns it off (every launch then waits for its predecessor to finish).
// Batched products run on the tcgen05 GEMM (k_tgemm.cu) unless
// LLAMINI_BATCH_GEMM=mma selects the mma.sync kernel (k_bgemm.cu).
int g_batch_gemm = -1;

bool batch_tc() {
    static const bool on = [] { const char* e = getenv("LLAMINI_BATCH_GEMM"); return !(e && strcmp(e, "mma") == 0); }();
    return g_batch_gemm >= 0 ? g_batch_gemm == 1 : on;
}

bool pdl_enabled() {
    static const bool on = [] { const char* e = getenv("LLAMINI_PDL"); return !(e && e[0] == '0'); }();
    return on;
}
int sm_count() { return g_sms; }

static uint32_t* g_err_word = nullptr;
uint32_t* dev_err_word() {
    if (!g_err_word && ensure_device()) {
        if (LM_CUDA(cudaMalloc(&g_err_word, 16))) LM_CUDA(cudaMemset(g_err_word, 0, 16));
    }
    return g_err_word;
}

void* dev_alloc(size_t bytes) {
    if (!ensure_device()) return nullptr;
    void* p = nullptr;
    if (bytes == 0) bytes = 16;
    if (!LM_CUDA(cudaMalloc(&p, bytes))) return nullptr;
    return p;
}

void dev_free(void* p) {
    if (p && g_device >= 0) cudaFree(p);
}

// ---------------------------------------------------------------- formats
bool type_info(uint32_t type, TypeInfo* ti) {
    switch (type) {
    case GGML_TYPE_F32:  *ti = {1, 4}; return true;
    case GGML_TYPE_F16:  *ti = {1, 2}; return true;
    case GGML_TYPE_Q4_0: *ti = {32, 18}; return true;
    case GGML_TYPE_Q4_1: *ti = {32, 20}; return true;
    case GGML_TYPE_Q5_0: *ti = {32, 22}; return true;
    case GGML_TYPE_Q8_0: *ti = {32, 34}; return true;
    case GGML_TYPE_Q4_K: *ti = {256, 144}; return true;
    case GGML_TYPE_Q5_K: *ti = {256, 176}; return true;
    case GGML_TYPE_Q6_K: *ti = {256, 210}; return true;
    default: return false;
    }
}

uint64_t type_bytes(uint32_t type, uint64_t n) {
    TypeInfo ti;
    if (!type_info(type, &ti) || n % ti.block_elems != 0) return 0;
    return n / ti.block_elems * ti.block_bytes;
}

uint32_t type_align(uint32_t type) {
    switch (type) {
    case GGML_TYPE_Q4_K: case GGML_TYPE_Q5_K: return 16;
    case GGML_TYPE_F32: return 4;
    case GGML_TYPE_F16: return 2;
    default: return 1;
    }
}

// ---------------------------------------------------------------- weight registry
struct GgufUpload {
    GGUFFile* gf;
    DevMat mat;
    void* alloc;
};
static std::unordered_map<const GGUFTensorInfo*, GgufUpload> g_uploads;

struct Source { GGUFFile* gf; const GGUFTensorInfo* info; };
static std::unordered_map<const Tensor*, Source> g_sources;

bool upload_gguf_tensor(GGUFFile* gf, const GGUFTensorInfo* info, DevMat* out, uint32_t rows, uint32_t cols) {
    auto it = g_uploads.find(info);
    if (it != g_uploads.end() && it->second.gf == gf && it->second.mat.rows == rows && it->second.mat.cols == cols) {
        *out = it->second.mat;
        return true;
    }
    if (it != g_uploads.end()) { dev_free(it->second.alloc); g_uploads.erase(it); }
    if (!ensure_device()) return false;
    const uint64_t n = gguf_tensor_count(info);
    if ((uint64_t)rows * cols != n) { set_error("tensor %s: %llu elements, expected %ux%u", info->name, (unsigned long long)n, rows, cols); return false; }
    const uint64_t rb = type_bytes(info->ggml_type, cols);
    if (rb == 0) { set_error("tensor %s: type %u cannot be used with rows of %u", info->name, info->ggml_type, cols); return false; }
    const uint64_t bytes = rb * rows;
    const uint64_t abs_off = gf->tensor_offset + info->offset;
    if (abs_off < info->offset || abs_off > gf->size || bytes > gf->size - abs_off) {
        set_error("tensor %s runs past the end of the file", info->name);
        return false;
    }
    // 16 bytes of slack: the decoders read whole aligned words around a block.
    void* d = dev_alloc(bytes + 16);
    if (!d) return false;
    const uint8_t* src = (const uint8_t*)gf->data + abs_off;
    if (!LM_CUDA(cudaMemcpy(d, src, bytes, cudaMemcpyHostToDevice)) ||
        !LM_CUDA(cudaMemset((uint8_t*)d + bytes, 0, 16))) {
        dev_free(d);
        return false;
    }
    GgufUpload u;
    u.gf = gf;
    u.alloc = d;
    u.mat.ptr = (const uint8_t*)d;
    u.mat.type = info->ggml_type;
    u.mat.rows = rows;
    u.mat.cols = cols;
    u.mat.row_bytes = rb;
    g_uploads[info] = u;
    *out = u.mat;
    return true;
}

const DevMat* find_gguf_tensor(const GGUFTensorInfo* info) {
    auto it = g_uploads.find(info);
    return it == g_uploads.end() ? nullptr : &it->second.mat;
}

void drop_gguf(GGUFFile* gf) {
    drop_sessions_for_gguf(gf);
    for (auto it = g_uploads.begin(); it != g_uploads.end();) {
        if (it->second.gf == gf) { dev_free(it->second.alloc); it = g_uploads.erase(it); }
        else ++it;
    }
    for (auto it = g_sources.begin(); it != g_sources.end();) {
        if (it->second.gf == gf) it = g_sources.erase(it);
        else ++it;
    }
}

void remember_source(const Tensor* t, GGUFFile* gf, const GGUFTensorInfo* info) { g_sources[t] = {gf, info}; }

bool source_of(const Tensor* t, GGUFFile** gf, const GGUFTensorInfo** info) {
    auto it = g_sources.find(t);
    if (it == g_sources.end()) return false;
    *gf = it->second.gf;
    *info = it->second.info;
    return true;
}

void forget_sources(const Tensor* t) { g_sources.erase(t); }

static void release_all() {
    drop_all_sessions();
    for (auto& kv : g_uploads) dev_free(kv.second.alloc);
    g_uploads.clear();
    g_sources.clear();
}

}  // namespace lm

// ---------------------------------------------------------------- C ABI
extern "C" {

const char* llamini_last_error(void) { return lm::g_err; }
void llamini_clear_error(void) { lm::g_err[0] = '\0'; }

int llamini_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}

int llamini_set_device(int device) {
    if (lm::g_device >= 0 && device != lm::g_device) {
        lm::set_error("llamini_set_device(%d): device %d already in use", device, lm::g_device);
        return -1;
    }
    lm::g_requested = device;
    return lm::ensure_device() ? 0 : -1;
}

void* llamini_stream(void) {
    if (!lm::ensure_device()) return nullptr;
    return (void*)lm::g_stream;
}

void llamini_release(void) { lm::release_all(); }

u64 llamini_type_bytes(u32 type, u64 n_elems) { return lm::type_bytes(type, n_elems); }

}  // extern "C"
