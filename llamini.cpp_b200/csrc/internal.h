// internal.h -- declarations shared by the host and device translation units of
// libllamini_cuda.so. Not installed; the public C ABI is include/*.h.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

#include "common.h"

#include <cuda.h>
#include "gguf.h"
#include "tensor.h"
#include "kv_cache.h"
#include "model.h"
#include "gpt2.h"

namespace lm {

// ---------------------------------------------------------------- errors
// Every failure is recorded here (sticky until llamini_clear_error) and echoed
// to stderr once; no call aborts the process.
void set_error(const char* fmt, ...);
bool cuda_ok(cudaError_t e, const char* what);
#define LM_CUDA(call) ::lm::cuda_ok((call), #call)

// ---------------------------------------------------------------- device
// Selects/initialises the CUDA device on first use. False (with an error set)
// when no device is usable; every GPU entry point checks this first.
bool ensure_device();
cudaStream_t stream();
int sm_count();

// Device allocations go through these so that failures are reported uniformly.
void* dev_alloc(size_t bytes);
void dev_free(void* p);

// ---------------------------------------------------------------- formats
struct TypeInfo { uint32_t block_elems, block_bytes; };
bool type_info(uint32_t type, TypeInfo* ti);
uint64_t type_bytes(uint32_t type, uint64_t n_elems);   // 0 if unsupported/misaligned
// Byte alignment the decoders need for a tensor of this type (16 for the
// K-quants read with 128-bit loads, the element size for F32/F16, else 1).
uint32_t type_align(uint32_t type);

// A weight matrix in GPU memory: the GGUF bytes of `rows` rows of `cols`
// elements each, stored unchanged (row r starts at ptr + r*row_bytes).
struct DevMat {
    const uint8_t* ptr = nullptr;
    uint32_t type = 0, rows = 0, cols = 0;
    uint64_t row_bytes = 0;
};

// ---------------------------------------------------------------- kernels (launchers)
// All launchers enqueue on `st` and return false (error set) on a launch failure.
bool kernels_init();
bool launch_dequant(uint32_t type, const uint8_t* d_raw, uint64_t n_elems, float* d_out, cudaStream_t st);

enum Epi : uint32_t {
    EPI_STORE = 0,      // out[r] = acc (+ bias[r])
    EPI_RESID = 1,      // out[r] += acc (+ bias[r])        (out is the residual stream)
    EPI_GLU_SILU = 2,   // out[r] = silu(acc_gate) * acc_up  (two matrices)
    EPI_GLU_GELU = 3,   // out[r] = gelu(acc_gate) * acc_up
    EPI_GELU = 4,       // out[r] = gelu(acc + bias[r])
};

enum Norm : uint32_t { NORM_NONE = 0, NORM_RMS = 1, NORM_LAYER = 2 };

// One group of output rows of a fused GEMV launch.
struct GemvSeg {
    const uint8_t* w = nullptr;    // matrix (gate matrix for GLU)
    const uint8_t* w2 = nullptr;   // up matrix for GLU
    uint64_t row_bytes = 0, row_bytes2 = 0;
    uint32_t type = 0, type2 = 0;
    uint32_t rows = 0;
    uint32_t epi = EPI_STORE;
    float* out = nullptr;
    const float* bias = nullptr;
    uint32_t tile0 = 0;            // first tile of this segment (filled by the launcher)
    uint32_t argmax = 0;           // 1: fold rows into the step's argmax key
};

constexpr int kMaxSegs = 4;

// Tensor parallelism with the reduction fused into the tensor-core GEMVs
// (k_gemv_mma.cu): a GEMV whose output is a partial sum (o, ffn_down of a
// rank's shard) stores its rows straight into fused slot `push` of every rank's
// buffer (peer memory over NVLink) and signals each rank's arrival counter; the
// next GEMV reading the residual stream waits for every rank's arrivals of slot
// `pull`, adds the ranks' rows (rank order) to its input and, in the CTA that
// finishes last, writes the sum back. kTpNone: no such step.
constexpr uint32_t kTpNone = 0xFFFFFFFFu;
constexpr uint32_t kTpFusedFloats = 16384;    // rows of a fused slot (dim <= 16384)
struct GemvTp {
    float* slots[8] = {};          // every rank's fused slots [2][8 ranks][kTpFusedFloats]
    uint32_t* arrive[8] = {};      // every rank's arrival counters [2][8 ranks]
    uint32_t* gen = nullptr;       // this rank's finished pulls of each slot [2] (device)
    uint32_t* ticket = nullptr;    // CTAs done reading, per slot [2] (device)
    uint32_t rank = 0, world = 1;
    uint32_t push = kTpNone, pull = kTpNone;
};

struct GemvArgs {
    const float* x = nullptr;      // input vector (normalised first when norm != NONE)
    uint32_t K = 0;
    uint32_t norm = NORM_NONE;
    const float* norm_w = nullptr;
    const float* norm_b = nullptr;
    float eps = 0.f;
    uint32_t nseg = 0;
    GemvSeg seg[kMaxSegs];
    unsigned long long* argmax_key = nullptr;
    float* x_out = nullptr;        // optional: store the normalised x (block 0 writes it)
    uint32_t* err = nullptr;       // error bits (a bounded wait that ran out sets kErrWaitTimeout)
    GemvTp tp;                     // fused tensor-parallel reduction (tensor-core GEMV only)
};

bool launch_gemv(const GemvArgs& a, cudaStream_t st);
// Tensor-core variant (k_gemv_mma.cu); *handled is false when some segment's
// format has no tensor-core path, and launch_gemv then uses the CUDA-core kernel.
bool launch_gemv_mma(const GemvArgs& a, cudaStream_t st, bool* handled);
// Whether launch_gemv runs `a` on the tensor-core kernel.
bool gemv_mma_takes(const GemvArgs& a);

// Plain multi-column GEMV used by llamini_gemv_* (no fusion).
bool launch_gemv_plain(uint32_t type, const uint8_t* w, uint32_t rows, uint32_t cols,
                       const float* x, uint32_t batch, float* y, cudaStream_t st);

// Error bits written by kernels into a device word the host checks.
constexpr uint32_t kErrWaitTimeout = 1u;   // a bounded wait on a copy gave up
uint32_t* dev_err_word();                  // library-wide word for launches outside a session

// Per-step device state shared by the kernels of one session.
struct StepState {
    uint32_t pos;          // position of the current step
    uint32_t n_prompt;     // tokens [0, n_prompt) are given; later ones are generated
    uint32_t trace;        // 1: copy the residual stream after each layer
    uint32_t err;          // error bits set by kernels (kErrWaitTimeout, ...)
    unsigned long long argmax_key;
    double nll;            // perplexity accumulator
    uint32_t nll_count;
};

struct EmbedArgs {
    StepState* st;
    const uint32_t* tokens;
    DevMat tok;            // token embedding table
    DevMat pos;            // learned position table (GPT-2) or ptr == nullptr
    float scale;           // embedding scale (1 unless gemma)
    float* hidden;
    uint32_t dim;
};
bool launch_embed(const EmbedArgs& a, cudaStream_t st);

struct AttnArgs {
    StepState* st;
    const float* qkv;      // q [n_heads*hd] | k [n_kv*hd] | v [n_kv*hd]
    void* kc;              // this layer's cache: [n_kv][max_seq][hd], f32 or fp16
    void* vc;
    uint32_t kv_f16;       // 1: fp16 elements, 0: f32 elements
    float* out;            // [n_heads*hd]
    float* part;           // [n_heads][n_split][hd + 4] partial results (m, l, -, -, o[hd])
    uint32_t* counter;     // [n_heads] completion counters (return to 0 after use)
    uint32_t n_heads, n_kv, hd, max_seq, n_split;
    uint32_t rope;         // 0 none, 1 NORM, 2 NEOX
    const float* theta;    // [hd/2] rotation frequencies base^(-2j/hd), computed on the host
};
bool launch_attention(const AttnArgs& a, cudaStream_t st);
// Per-sequence strides of batched decode attention (elements / bytes).
struct AttnBatch {
    uint64_t qkv_stride;   // floats between sequences' q|k|v rows
    uint64_t cache_stride; // bytes between sequences' caches of one layer
    uint64_t out_stride;   // floats between output rows
    uint64_t part_stride;  // floats between sequences' split partials
};
bool launch_attention_batch(const AttnArgs& a, const AttnBatch& bt, uint32_t B, cudaStream_t st);

struct FinishArgs {
    StepState* st;
    uint32_t* tokens;
    uint32_t max_tokens;
    const float* logits;   // for the perplexity accumulator (may be null)
    uint32_t vocab;
    uint32_t nll;          // 1: accumulate -log p(tokens[pos+1])
};
bool launch_finish(const FinishArgs& a, cudaStream_t st);

// ---------------------------------------------------------------- persistent decode step
// One launch runs whole token steps: every CTA (one per SM) works through a
// fixed list of tasks -- 16-row tiles of the step's matrices and (head, split)
// pieces of attention -- while its producer warp streams the weight tiles of
// its upcoming tasks into shared memory. Ops wait for their predecessor through
// per-op completion counters instead of kernel boundaries (k_decode.cu).
enum DecKind : uint32_t { DEC_GEMV = 0, DEC_ATTN = 1 };
constexpr uint32_t kDecNoWait = 0xFFFFFFFFu;   // waits for the previous step's finish

struct DecOp {
    uint32_t kind = DEC_GEMV;
    uint32_t ntasks = 0;         // tasks in the schedule
    uint32_t ndone = 0;          // completions signalled per step (tiles; heads for attention)
    uint32_t wait = kDecNoWait;  // op whose completion this op needs
    uint32_t trace_off = 0xFFFFFFFFu;   // residual-add ops that end a layer: offset in the trace buffer
    uint32_t n_split = 1;        // attention (and x_merge): position splits per head
    uint32_t x_merge = 0;        // DEC_GEMV: the input is the merge of `at`'s split partials
    GemvArgs g;                  // DEC_GEMV (segment tile0 filled)
    AttnArgs at = {};            // DEC_ATTN, and the partials an x_merge op reads
};

struct DecSync {
    uint32_t epoch;              // steps finished by earlier launches
    uint32_t exit_ticket;        // CTAs done with the current launch
    uint32_t step_done;          // steps finished so far (set by each step's finisher)
    uint32_t abort;              // set by a CTA whose bounded wait ran out
};

struct DecArgs {
    const DecOp* ops = nullptr;
    uint32_t n_ops = 0;
    const uint32_t* sched = nullptr;      // CTA c: sched_len[c] entries at sched + c * sched_stride
    const uint32_t* sched_len = nullptr;  // entry = (op << 16) | task
    uint32_t sched_stride = 0;
    uint32_t n_cta = 0;
    DecSync* sync = nullptr;
    uint32_t* done = nullptr;             // [n_ops] completions (monotonic)
    StepState* st = nullptr;
    uint32_t* tokens = nullptr;
    uint32_t max_tokens = 0;
    DevMat tok, pos;                      // embedding tables for the next step's input
    float emb_scale = 1.f;
    float* hidden = nullptr;
    float* trace = nullptr;               // per-layer residual stream, or null
    uint32_t n_steps = 1;
    uint32_t ring_bytes = 0;              // weight ring in shared memory
    uint32_t kmax = 0;                    // largest GEMV input length (multiple of 128)
    uint32_t hd = 0;                      // attention head size (for the shared-memory plan)
};
constexpr uint32_t kDecMaxOps = 1u << 16;
constexpr uint32_t kDecMaxOpsSmem = 256;      // ops of one step (per-op tables live in shared memory)
constexpr uint32_t kDecMaxTasks = 512;        // tasks of one CTA per step (its list lives in shared memory)
bool decode_init();
bool decode_supported_type(uint32_t type);
// Shared memory for a ring of `ring` bytes, inputs up to kmax and head size hd;
// 0 when it does not fit.
size_t decode_smem(uint32_t ring, uint32_t kmax, uint32_t hd);
uint32_t decode_ring_bytes(uint32_t kmax, uint32_t hd);
uint32_t decode_tile_alloc(const GemvSeg& G);    // ring bytes of one tile of G
bool launch_decode(const DecArgs& a, cudaStream_t st);

// ---------------------------------------------------------------- dataflow decode kernel
// Batch-1 decode steps as one persistent kernel (k_flow.cu) whose GEMV inputs
// travel between ops as records: per 16 consecutive elements x_i, the fp16
// high and low parts of x_i * 2^E (E chosen from the group's largest |x_i|),
// already in the order of an mma.sync B fragment, plus 2^(24-E) and the sum
// of the 16 values. The op that produces a vector writes its records in its
// epilogue (a 16-row tile is one group); the consumers copy their slice of K.
// An RMS-normalised input carries the norm weight folded in and, per group,
// the sum of squares of the raw vector; the consumer applies 1/rms to its dot
// products. The O projection's input is merged from the attention partials by
// the consumers themselves.
enum FlowKind : uint32_t { FLOW_GEMV = 0, FLOW_ATTN = 1 };
constexpr uint32_t kFlowStepStart = 0xFFFFFFFFu;   // the op waits for the step's input embedding

struct FlowRec {
    uint32_t* w = nullptr;     // [groups][16]: words 0..7 fp16 high pairs, 8..15 low pairs
    float2* fs = nullptr;      // [groups]: {2^(24-E), sum of the group's values}
    float* ss = nullptr;       // [groups]: sum of squares of the raw values (normalised inputs), or null
};

struct FlowSeg {
    const uint8_t* w = nullptr;     // matrix (gate for GLU)
    const uint8_t* w2 = nullptr;    // up matrix for GLU
    uint64_t row_bytes = 0, row_bytes2 = 0;
    uint32_t type = 0, rows = 0, epi = EPI_STORE, tile0 = 0;
    float* out = nullptr;            // f32 rows (EPI_RESID: unused, the residual stream takes the sum)
    const float* bias = nullptr;
    // rows of an even number of 16-byte units reach shared memory through one
    // TMA tensor copy per tile whose box is one unit wider than the row (the
    // padded stride keeps the 8 rows an MMA reads in different banks); other
    // rows move as one contiguous bulk copy. Set by flow_encode_maps.
    const CUtensorMap* map = nullptr;
    const CUtensorMap* map2 = nullptr;
};

struct FlowOp {
    uint32_t kind = FLOW_GEMV;
    uint32_t ntasks = 0;            // tiles, or (head, split) tasks; each completes once per step
    uint32_t wait = kFlowStepStart; // op whose completion this op needs
    uint32_t wait_n = 0;            // completions per step of that op
    // GEMV
    uint32_t K = 0, nseg = 0;
    uint32_t in_attn = 0;           // input = merge of at's split partials (else the records `in`)
    FlowRec in;                     // in.ss != null: RMSNorm of the input (eps below)
    float eps = 0.f;
    FlowSeg seg[3];
    FlowRec out;                    // records of the output for the next GEMV (out.w null: none)
    const float* out_nw = nullptr;  // norm weight folded into the output records (null: none)
    uint32_t trace_off = 0xFFFFFFFFu;   // residual-add ops that end a layer: offset in the trace
    uint32_t argmax = 0;            // the lm_head: argmax key and step finish
    // attention (kind FLOW_ATTN, and the partials an in_attn op merges)
    uint32_t n_split = 1;
    AttnArgs at = {};
};

struct FlowArgs {
    const FlowOp* ops = nullptr;
    uint32_t n_ops = 0;
    const uint32_t* sched = nullptr;      // CTA c: sched_len[c] entries at sched + c * sched_stride
    const uint32_t* sched_len = nullptr;  // entry = (op << 16) | task
    uint32_t sched_stride = 0;
    uint32_t n_cta = 0;
    DecSync* sync = nullptr;              // step_done counts finished steps (input embedded)
    uint32_t* done = nullptr;             // [n_ops] completions (monotonic)
    StepState* st = nullptr;
    uint32_t* tokens = nullptr;
    uint32_t max_tokens = 0;
    DevMat tok;                           // token embedding table
    float emb_scale = 1.f;
    float* hidden = nullptr;              // the residual stream
    FlowRec in0;                          // records of the first layer's input
    const float* n1w0 = nullptr;          // the first layer's attention norm weight
    uint32_t dim = 0;
    float* trace = nullptr;               // per-layer residual stream, or null
    uint32_t n_steps = 1;
    uint32_t ring_bytes = 0;
    uint32_t hd = 0;
};
constexpr uint32_t kFlowMaxOps = 256;         // ops of one step
constexpr uint32_t kFlowMaxTasks = 512;       // tasks of one CTA per step
constexpr uint32_t kFlowMaxSb = 3;            // 256-element super-blocks of K per consumer warp (K <= 6144)
bool flow_init();
bool flow_supported_type(uint32_t type);
uint32_t flow_ring_bytes(uint32_t hd);
uint32_t flow_tile_alloc(const FlowSeg& G);
// Tensor maps for every padded-row matrix of `ops` (written into `maps`, a
// device array of n_maps entries, and referenced from the segments); false
// with an error set when the driver refuses one.
uint32_t flow_maps_needed(const FlowOp* ops, uint32_t n_ops);
bool flow_encode_maps(FlowOp* ops, uint32_t n_ops, CUtensorMap* d_maps);
// Tensor map of a matrix's 16-row tiles at the padded shared-memory stride
// (rows of an even number of 16-byte units, at most 255 units); false when the
// driver refuses it.
bool encode_tile_map(CUtensorMap* m, const uint8_t* w, uint64_t row_bytes, uint32_t rows);
// The same view with a box of box_units 16-byte units per row (rows of a
// multiple of 16 bytes); false when the driver refuses it.
bool encode_box_map(CUtensorMap* m, const uint8_t* w, uint64_t row_bytes, uint32_t rows, uint32_t box_units);
bool launch_flow(const FlowArgs& a, cudaStream_t st);
bool launch_flow_embed(const FlowArgs& a, cudaStream_t st);

// sample_token (generate.c:25-60) on the device (k_sample.cu): one draw from
// the logits at d_logits with u = rand() / (RAND_MAX + 1) drawn by the caller;
// the token id is written to *d_tok. d_scratch holds vocab floats.
bool launch_sample(const float* d_logits, uint32_t vocab, float temp, float top_p, float u, float* d_scratch,
                   uint32_t* d_tok, cudaStream_t st);

// ---------------------------------------------------------------- batched GEMM
// Up to 64 input vectors per weight pass (k_bgemm.cu): staging per sequence,
// split-K dequant GEMM into raw partials, per-(sequence, row) finish.
struct BStageArgs {
    const float* x = nullptr;      // [B][ldx]
    uint32_t ldx = 0, K = 0, B = 0;
    uint32_t norm = NORM_NONE;
    const float* norm_w = nullptr;
    const float* norm_b = nullptr;
    float eps = 0.f;
    uint16_t* xh = nullptr;        // [B][K] fp16 bits of x * 2^E_b, high part
    uint16_t* xl = nullptr;        // low part
    float* sx = nullptr;           // [B][K/16] 16-element sums * 2^(E_b - 24)
    float* oscale = nullptr;       // [B] 2^(24 - E_b)
    // nonzero: xh/xl in the tensor-core GEMM's layout [K/8][np/8][8][8] for
    // np (the batch padded to 16) columns, no 16-element sums; when K % 256
    // == 0 also the 32-element sums after the inputs in xh (tg_xh_halves)
    uint32_t np = 0;
};
struct BSeg {
    const uint8_t* w = nullptr;
    uint64_t row_bytes = 0;
    uint32_t type = 0, rows = 0;
    uint32_t rb0 = 0;              // first row block (filled by bgemm_plan)
    float* part = nullptr;         // [ksplit][B][rows] raw sums
    uint32_t ub = 0, wrs = 0;      // bytes per K unit, shared-memory row stride (filled by bgemm_plan)
};
struct BGemmArgs {
    const uint16_t* xh = nullptr;
    const uint16_t* xl = nullptr;
    const float* sx = nullptr;
    uint32_t B = 0, K = 0;
    uint32_t nseg = 0;
    BSeg seg[3];
    // filled by bgemm_plan: unit elements, units per split, K split, row blocks,
    // largest weight row stride, input row stride (halves), padded batch, byte
    // offset of the low halves from the high halves in a buffer
    uint32_t ue = 0, ups = 0, ksplit = 0, rblocks = 0, wrs = 0, xs = 0, bpad = 0, xlo = 0;
};
struct BFinishArgs {
    const float* part = nullptr;   // [ksplit][B][rows]
    const float* part2 = nullptr;  // up-matrix sums for EPI_GLU_*
    uint32_t ksplit = 1, B = 0, rows = 0;
    const float* oscale = nullptr;
    const float* bias = nullptr;
    uint32_t epi = EPI_STORE;
    float* out = nullptr;          // out[b * ldo + r]
    uint32_t ldo = 0;
    unsigned long long* keys = nullptr;   // [B] argmax keys (or null)
    // up to two more segments whose rows follow in the output row (q, k and v
    // of one launch; EPI_STORE only): their partial sums, rows and biases
    const float* part_b = nullptr;
    const float* part_c = nullptr;
    const float* bias_b = nullptr;
    const float* bias_c = nullptr;
    uint32_t rows_b = 0, rows_c = 0;
};
struct BEmbedArgs {
    const StepState* st;           // pos (shared by the batch)
    const uint32_t* tokens;        // [B][tok_stride]
    uint32_t tok_stride;
    DevMat tok, pos;               // token table, learned positions (or ptr == nullptr)
    float scale;
    float* hidden;                 // [B][dim]
    uint32_t dim;
};
struct BTokenArgs {
    StepState* st;
    uint32_t* tokens;
    uint32_t tok_stride;
    const uint32_t* n_prompt;      // [B]
    unsigned long long* keys;      // [B] argmax keys of the step (reset here)
    uint32_t B, max_tokens;
};
bool launch_bembed(const BEmbedArgs& a, uint32_t B, cudaStream_t st);
bool launch_btoken(const BTokenArgs& a, cudaStream_t st);
bool bgemm_init();
bool bgemm_type(uint32_t type);
bool bgemm_plan(BGemmArgs& a, uint32_t target_ctas);
bool launch_bgemm(const BGemmArgs& a, cudaStream_t st);
bool launch_bstage(const BStageArgs& a, cudaStream_t st);

// Tensor-core (tcgen05) dequant GEMM for a batch of vectors (k_tgemm.cu):
// same partial sums as bgemm_kernel, inputs staged with BStageArgs::np.
// A operand kinds of a segment: TG_PLAIN the weights as fp16 hi + lo;
// TG_KMIN (Q4_K, Q5_K) d*sc*q as fp16 hi + lo, with the -dmin*m terms added by
// extra MMAs against the staged 32-element sums of the inputs.
constexpr uint32_t TG_PLAIN = 0, TG_KMIN = 1;
struct TSeg {
    const uint8_t* w = nullptr;
    uint64_t row_bytes = 0;
    uint64_t pitch = 0;            // bytes between rows (0: row_bytes)
    uint32_t type = 0, rows = 0;
    float* part = nullptr;         // [ksplit][B][rows] raw sums
    // filled by tgemm_plan: first row block, elements per raw unit, bytes of
    // one row's raw unit, raw-buffer row stride (= the TMA box width), and the
    // A operand kind (TG_PLAIN, TG_KMIN)
    uint32_t rb0 = 0, ru = 0, ub = 0, rrs = 0, mode = 0;
};
// Halves of an xh buffer staged for the tensor-core GEMM: the inputs, then
// (K % 256 == 0) per super-block 16 x np halves of 32-element sums.
inline size_t tg_xh_halves(size_t K, size_t np) { return np * (K + K / 16); }
struct alignas(64) TGemmArgs {
    // filled by tgemm_plan: per segment a 2-D TMA map of the rows as uint16
    // (used when `tma`; otherwise 16-byte cp.async copies)
    CUtensorMap tmap[3];
    const uint16_t* xh = nullptr;  // staged inputs, [K/8][NP/8][8][8] halves (then the sums)
    const uint16_t* xl = nullptr;
    uint32_t B = 0, K = 0;
    uint32_t nseg = 0;
    TSeg seg[3];
    uint32_t* err = nullptr;       // error bits (wait ran out, weight beyond fp16), or null
    // filled by tgemm_plan: padded batch, K split unit, units per CTA, K split,
    // row blocks, raw buffer bytes, A/x stages, tensor-memory columns, CTAs
    uint32_t NP = 0, ue = 0, ups = 0, ksplit = 0, rblocks = 0, raw_bytes = 0, stages = 0, tcols = 0, grid = 0;
    uint32_t tma = 0;
    uint32_t kmin = 0;             // some segment is TG_KMIN
};
// ---------------------------------------------------------------- tensor parallelism
// One process per GPU; LLaMA sessions hold this rank's shard of the heads and
// FFN columns, and sum the o-projection and ffn_down outputs across ranks
// with tp_allreduce_kernel (k_tp.cu) over peer memory.
constexpr uint32_t kTpMaxRanks = 8;
constexpr uint32_t kTpSlotFloats = 16384;
// The wide allreduce (batches and prefill chunks: one vector per column):
// slices of kTpWideSlice floats, one CTA each, at most kTpWideCtas of them.
constexpr uint32_t kTpWideCtas = 256;
constexpr uint32_t kTpWideSlice = 2048;
constexpr uint32_t kTpWideFloats = kTpWideCtas * kTpWideSlice;   // 64 columns of 8192
struct TpState {
    uint32_t rank = 0, world = 1;
    float* local = nullptr;                  // this rank's exported buffer
    float* peer[kTpMaxRanks] = {};           // every rank's buffer, mapped here (this rank's included)
    uint32_t* gen = nullptr;                 // allreduces this rank has finished (device)
    uint32_t* wgen = nullptr;                // wide allreduces finished, per slice (device, kTpWideCtas)
};
TpState& tp();
size_t tp_buffer_bytes();
bool tp_alloc_buffer();
// out[i] += sum over ranks of part[i] (rank order), i < n; part is this rank's.
bool launch_tp_allreduce(const float* part, float* out, uint32_t n, uint32_t* err, cudaStream_t st);
// out[i] += the sum over ranks of part[i], i < n <= kTpWideFloats, slice by slice.
bool launch_tp_allreduce_wide(const float* part, float* out, uint32_t n, uint32_t* err, cudaStream_t st);
// The group's fused-reduction pointers (push / pull slots kTpNone).
GemvTp tp_fused_args(uint32_t push, uint32_t pull);

// ---------------------------------------------------------------- prefill (k_prefill.cu)
// A chunk's columns are ns sequences x cp positions: column b is position
// p0 + b % cp of sequence b / cp (one sequence: cp = C, strides 0).
struct PEmbedArgs {
    const uint32_t* tokens;        // token of sequence i, position p at tokens[i * tok_stride + p]
    uint32_t p0, C, cp, tok_stride;
    DevMat tok, pos;               // token table, learned positions (or ptr == nullptr)
    float scale;
    float* hidden;                 // [C][dim]
    uint32_t dim;
};
struct PRopeArgs {
    float* qkv;                    // [C][qkv_stride]: q | k | v of each position
    uint32_t qkv_stride;
    void* kc;                      // this layer's cache [n_kv][max_seq][hd] of sequence 0
    void* vc;
    uint32_t kv_f16, n_heads, n_kv, hd, max_seq, p0, rope, cp;
    uint64_t seq_elems;            // cache elements from one sequence's layer to the next's
    const float* theta;
};
struct PAttnArgs {
    const float* qkv;
    uint32_t qkv_stride;
    const void* kc;
    const void* vc;
    uint32_t kv_f16;
    float* out;                    // [C][out_stride]
    uint32_t out_stride;
    uint32_t n_heads, n_kv, hd, max_seq, p0, C, cp;
    uint64_t seq_elems;
};
// Teacher-forced scoring of a chunk (compute_perplexity, generate.c:169-197):
// lp[p] = log softmax(logits of position p)[tokens[p + 1]] for p0 <= p <= last.
struct PNllArgs {
    const float* logits;           // [C][ld], position p0 + b at row b
    uint32_t vocab, ld;
    const uint32_t* tokens;        // device token ids
    uint32_t p0, C, last;
    float* lp;
};
bool prefill_init();
bool launch_pnll(const PNllArgs& a, cudaStream_t st);
bool launch_pembed(const PEmbedArgs& a, cudaStream_t st);
bool launch_prope(const PRopeArgs& a, uint32_t C, cudaStream_t st);
bool launch_pattn(const PAttnArgs& a, cudaStream_t st);

bool tgemm_init();
bool batch_tc();   // tcgen05 GEMM for batched products (default) or mma.sync
extern int g_batch_gemm;   // llamini_set_batch_gemm: -1 default, 0 mma.sync, 1 tcgen05
bool tgemm_type(uint32_t type);
bool tgemm_plan(TGemmArgs& a, uint32_t sms);
bool launch_tgemm(const TGemmArgs& a, cudaStream_t st);
bool launch_bfinish(const BFinishArgs& a, cudaStream_t st);

// Host-pointer op kernels (model.h per-op exports), device buffers in/out.
bool launch_rms_norm(float* out, const float* x, const float* w, uint32_t dim, float eps, cudaStream_t st);
bool launch_layer_norm(float* out, const float* x, const float* w, const float* b, uint32_t dim, float eps, cudaStream_t st);
bool launch_rope(float* v, uint32_t pos, uint32_t dim, uint32_t hd, float base, uint32_t neox, cudaStream_t st);
bool launch_glu(float* out, const float* g, const float* u, uint32_t n, uint32_t gelu, cudaStream_t st);
bool launch_gelu_inplace(float* x, uint32_t n, cudaStream_t st);
bool launch_add(float* out, const float* a, const float* b, uint32_t n, cudaStream_t st);
bool launch_scale(float* out, const float* a, float s, uint32_t n, cudaStream_t st);
bool launch_argmax(const float* x, uint32_t n, uint32_t* out, cudaStream_t st);
bool launch_matmul(const float* A, const float* B, float* C, uint32_t m, uint32_t k, uint32_t n, cudaStream_t st);
bool launch_mha_f32(const float* q, float* kc, float* vc, float* out, uint32_t pos,
                    uint32_t n_heads, uint32_t n_kv, uint32_t hd, cudaStream_t st);
bool launch_copy_f32(float* dst, const float* src, uint32_t n, cudaStream_t st);

// ---------------------------------------------------------------- weight registry
// Device copies of GGUF tensors, keyed by the GGUFTensorInfo they came from.
// Filled by llama_load_weights / gpt2_load_weights (or on demand), dropped by
// gguf_close.
bool upload_gguf_tensor(GGUFFile* gf, const GGUFTensorInfo* info, DevMat* out,
                        uint32_t rows, uint32_t cols);
const DevMat* find_gguf_tensor(const GGUFTensorInfo* info);
void drop_gguf(GGUFFile* gf);

// GPT-2's loader keeps eager f32 host tensors (gpt2.c:91-127); the GGUF tensor
// each one came from is remembered so the GPU can stream the quantized bytes.
void remember_source(const Tensor* t, GGUFFile* gf, const GGUFTensorInfo* info);
bool source_of(const Tensor* t, GGUFFile** gf, const GGUFTensorInfo** info);
void forget_sources(const Tensor* t);

// Sessions (session.cu)
void drop_sessions_for_model(const void* model);
void drop_sessions_for_gguf(const GGUFFile* gf);
void drop_all_sessions();

}  // namespace lm
