// jv_internal.h — shared declarations of the B200 Jevstral runtime (host C++ and CUDA).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "../../include/jv.h"

namespace jv {

// ------------------------------------------------------------------ errors

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define JV_CUDA(call)                                                                          \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            throw ::jv::Error(e_ == cudaErrorMemoryAllocation ? JV_ERR_OOM : JV_ERR_DEVICE,    \
                              std::string(#call) + ": " + cudaGetErrorString(e_));            \
    } while (0)

// ------------------------------------------------------------- GGML types

// ggml_type numbering (reference src/Jevstral/Gguf/GgmlType.cs:9-44).
enum GgmlType : int {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q8_1 = 9,
    T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 30,
    // Not a GGML type: the affine layout (qx.cpp) that every other block format is converted to
    // on load: per 16 weights, v = (a * q) + c with int8 q and fp32 a, c.
    T_QX = 64
};

// Tile geometry of a quantized matrix in HBM. The GGUF blocks of 128 consecutive rows ×
// 64 consecutive columns are gathered into one contiguous "chunk", split into planes so
// that every plane starts 16-byte aligned. The bits are the file's bits: re-tiled, never
// re-quantized. Chunks are stored [row tile][k step], so one k step of one row tile is a
// single bulk copy, and a GEMV CTA streams its row tile front to back.
//   Q8_0: qs  int8 [128][64]   | d fp16 [128][2]                                  = 8704 B
//   Q4_0: qs  u8   [128][2][16] | d fp16 [128][2]                                 = 4608 B
//   Q5_1: qs  u8   [128][2][16] | qh u32 [128][2] | d fp16 [128][2] | m fp16 [128][2] = 6144 B
//   QX:   q   int8 [128][64]    | a fp32 [128][4]  | c fp32 [128][4] (per 16 columns) = 12288 B
constexpr int TILE_ROWS = 128;
constexpr int TILE_K = 64;

__host__ __device__ constexpr int chunk_bytes(int type) {
    return type == T_Q8_0 ? 8704 : type == T_Q4_0 ? 4608 : type == T_Q5_1 ? 6144 : type == T_QX ? 12288 : 0;
}
__host__ __device__ constexpr int qs_bytes(int type) { return type == T_Q8_0 || type == T_QX ? 8192 : 4096; }

// qx.cpp: the GGUF formats with an affine form, and their conversion to row-major T_QX rows
// (per 64 columns: 64 int8 q, 4 fp32 a, 4 fp32 c) for the device re-tiling.
bool qx_expressible(int type);
int64_t qx_row_bytes(int cols);
void qx_convert_rows(int type, const uint8_t* src, int64_t src_row_bytes, int rows, int cols, uint8_t* dst);

struct QWeight {
    int type = 0;
    int rows = 0, cols = 0;      // output features (N), input features (K)
    int tiles = 0, ksteps = 0;   // rows / 128, cols / 64
    uint8_t* data = nullptr;     // [tiles][ksteps][chunk]
    size_t bytes() const { return (size_t)tiles * ksteps * chunk_bytes(type); }
};

// ----------------------------------------------------------- activations

// GEMM operands are fp16: the K-slab layout [K/64][Tpad][64] with the 128-byte swizzle
// already applied (16-byte chunk c of row t is stored at chunk c ^ (t & 7)). A row tile of
// BN tokens of one K slab is then one contiguous bulk copy that lands in shared memory in
// exactly the UMMA K-major SWIZZLE_128B layout.
__host__ __device__ inline size_t kslab_offset(int t, int k, int tpad) {
    int kb = k >> 6, kk = k & 63;
    int c = (kk >> 3) ^ (t & 7);
    return ((size_t)kb * tpad + t) * 64 + c * 8 + (kk & 7);
}

// ----------------------------------------------------------------- KV pages

// A KV page holds page_slots consecutive cache slots (a multiple of 8) of every (layer, kv
// head): the plane of (layer, head, K = 0 | V = 1) starts at kv_plane_offset bytes into the
// page. A plane is two halves (dims 0-63, then 64-127) of page_slots rows x 128 bytes, and
// inside a row the 16-byte chunk of dims 8c..8c+7 sits at chunk position c ^ (row & 7): the
// same 128-byte swizzle as the K-slab, so a run of rows whose first row is a multiple of 8
// away from its tile row copies straight into a tensor-core operand tile.
__host__ __device__ inline int64_t kv_plane_offset(int layer, int kv_heads, int head, int kv, int page_slots) {
    return (int64_t)((layer * kv_heads + head) * 2 + kv) * page_slots * 256;
}
// Byte offset inside a plane of the 16-byte chunk holding dims 8c..8c+7 (c < 16) of row `row`.
__host__ __device__ inline int kv_chunk_offset(int row, int c, int page_slots) {
    return (c >> 3) * page_slots * 128 + row * 128 + (((c & 7) ^ (row & 7)) << 4);
}
// Byte offset inside a plane of dim d of row `row`.
__host__ __device__ inline int kv_elem_offset(int row, int d, int page_slots) {
    return kv_chunk_offset(row, d >> 3, page_slots) + (d & 7) * 2;
}

// ------------------------------------------------------------ GEMM plans

// EPI_SWIGLU: the fused gate/up matrix (each 128-row tile = 64 gate rows then the 64 matching
// up rows) -> silu(gate) * up written as the fp16 K-slab operand of the down projection.
// EPI_PARTIAL (K split in two): each half writes its fp32 partial to ws[split] and nothing
// else; the consumer (the next RMSNorm) adds h += ws[0] + ws[1] as it reads h.
enum Epilogue : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_PARTIAL = 3 };


struct GemmArgs {
    const QWeight* w;
    const __half* x;   // K-slab fp16 activations, tpad rows
    int T, tpad, bn;   // tokens, padded tokens (multiple of bn), token tile
    float* y;          // [T][ldy]
    int ldy;
    int epilogue;
    int* err;          // device error word (JV_ERR_DEVICE_TIMEOUT on a bounded-wait timeout)
    __half* xs_out = nullptr;  // EPI_SWIGLU: K-slab [ff/64][tpad][64] of the activation
    int splits = 1;    // K splits (gemm_splits_for); > 1 needs ws and counters
    float* ws = nullptr;       // [splits][T][ldy] fp32 partials
    int* counters = nullptr;   // [tiles][tpad/bn], zero between launches
};
int gemm_splits_for(const QWeight& w);

// Token tiles for a GEMM over T tokens: balanced tiles of at most 256 (the MMA's N limit),
// multiples of 32, halved for products that would leave SMs idle. Depends on T and the matrix
// only, never on which tokens they are; the K order of the MMA chain does not depend on it,
// so a token's result is independent of its batch.
int gemm_tpad_for(int T);
int gemm_bn_for(int T, int units_per_tile, int sm_count);

// ------------------------------------------------------------ kernel API

void launch_repack(const uint8_t* raw, int type, int rows, int cols, int64_t raw_row_bytes, uint8_t* dst,
                   int dst_tiles, int ksteps, int row_in_tile_base, int tile_offset, int interleave,
                   cudaStream_t s);
void launch_embed(const QWeight& table, const int32_t* ids, int T, float* h, int hidden, int* err, cudaStream_t s);
// fp16 operands: a value that rounds to infinity in fp16 (|v| >= 65520) or is not a number.
// Kernels that pack fp16 record it in the context's error word (JV_ERR_NUMERIC and the site).
enum NumericSite : int { NS_RMSNORM = 65, NS_ROPE_KV = 66, NS_SWIGLU = 67, NS_DEC_INPUT = 68, NS_DEC_KV = 69, NS_KV_RESTORE = 70 };
#ifdef __CUDACC__
__device__ __forceinline__ bool f16_out_of_range(float v) { return !(fabsf(v) < 65520.f); }
__device__ __forceinline__ void report_numeric(int* err, int site) {
    if (!err) return;
    atomicCAS(err, 0, JV_ERR_NUMERIC);  // a timeout, if any, keeps priority
    atomicCAS(err + 1, 0, site);
}
#endif

// Bounds-checked builds (-DJV_BOUNDS_CHECK, libjv_checked.so): the index sites below test what
// they are about to use and, when it is out of range, record JV_ERR_RANGE with the site in the
// error word and use a safe stand-in instead (page 0, or the access skipped), so a bad index is
// reported rather than read or written. Normal builds compile the checks away.
enum BoundsSite : int {
    BS_ROPE_PAGE = 80, BS_ATTN_PAGE = 81, BS_ATTN_STAGED = 82, BS_MMA_ATTN_PAGE = 83, BS_DECODE_PAGE = 84,
    BS_GEMM_UNIT = 85, BS_SNAPSHOT_PAGE = 86
};
#ifdef __CUDACC__
__device__ __forceinline__ void report_oob(int* err, int site) {
    if (!err) return;
    atomicCAS(err, 0, JV_ERR_RANGE);
    atomicCAS(err + 1, 0, site);
}
// The physical KV page of `slot`. A context's page table on the device is preceded by two words:
// its entry count and the pool's page count (ctx_upload_pages), which a checked build tests.
__device__ __forceinline__ int kv_page(const int32_t* table, int slot, int page_slots, int* err, int site) {
#ifdef JV_BOUNDS_CHECK
    const int e = slot / page_slots;
    if (slot < 0 || e >= table[-2]) {
        report_oob(err, site);
        return 0;
    }
    const int p = table[e];
    if (p < 0 || p >= table[-1]) {
        report_oob(err, site);
        return 0;
    }
    return p;
#else
    (void)err;
    (void)site;
    return table[slot / page_slots];
#endif
}
#ifdef JV_BOUNDS_CHECK
#define JV_CHECK(cond, err, site) ((cond) ? true : (::jv::report_oob((err), (site)), false))
#else
#define JV_CHECK(cond, err, site) true
#endif
#endif

void launch_rmsnorm(const float* h, const float* w, int T, int n, float eps, __half* xs, int tpad, float* out32,
                    int* err, cudaStream_t s);
// Prefill RMSNorm into the fp16 K-slab, first folding a pending split-K residual into h
// (h += resid[0] + resid[1] when resid != nullptr, resid = [2][T][n]).
void launch_rmsnorm_resid(float* h, const float* resid, const float* w, int T, int n, float eps, __half* xs, int tpad,
                          int* err, cudaStream_t s);
// h += resid[0] + resid[1] (resid = [2][T][n]).
void launch_resid_add(float* h, const float* resid, int64_t count, cudaStream_t s);
void launch_rmsnorm_rows(const float* h, const int32_t* rows, int n_rows, const float* w, int n, float eps,
                         float* out32, __half* xs, int tpad, int* err, cudaStream_t s);
void launch_gemm(const GemmArgs& a, cudaStream_t s);
void launch_gemm_reference(const GemmArgs& a, cudaStream_t s);
void launch_gemv(const QWeight& w, const float* x, float* partial, int splits, cudaStream_t s);
void launch_gemv_reduce(const float* partial, int splits, int n, float* y, int epilogue, cudaStream_t s);
int gemv_splits_for(const QWeight& w, int sm_count);

struct RopeArgs {
    const float* qkv;       // [T][qdim + 2 kvdim]
    const int32_t* pos;     // [T]
    const int32_t* slot;    // [T]
    const float2* table;    // [max_pos][half] (cos*mscale, sin*mscale)
    int T, heads, kv_heads, head_dim, layer;
    float temperature_scale;
    int orig_ctx;
    __half* q16;            // [T][qdim] (prefill) or null
    float* q32;             // [T][qdim] (decode / capture) or null
    __half* kv_pool;        // page pool
    const int32_t* page_table;
    int64_t page_bytes;     // bytes per page
    int page_slots;         // slots per page
    float* k32;             // optional capture of rotated keys [T][kvdim]
    int* err = nullptr;     // error word (JV_ERR_NUMERIC when a value leaves the fp16 range)
};
void launch_rope_kv(const RopeArgs& a, cudaStream_t s);
#ifdef __CUDACC__
// The llama-4 query temperature at a position (Rope.cs / MinistralModel.cs:676-682): 1 below the
// original context, 1 + scale * ln(1 + floor(pos / orig)) past it.
__device__ __forceinline__ float rope_temperature(int pos, int orig_ctx, float temperature_scale) {
    float temp = 1.0f;
    if (orig_ctx > 0 && temperature_scale != 0.f) {
        float interval = floorf(__fdiv_rn((float)pos, (float)orig_ctx));
        if (interval != 0.f) temp = __fadd_rn(1.0f, __fmul_rn(temperature_scale, logf(__fadd_rn(1.0f, interval))));
    }
    return temp;
}
#endif
void launch_rope_table(float2* table, const float* freqs, int half, int pos0, int npos, float mscale, cudaStream_t s);

constexpr int ATT_ITEM_TOKENS = 32;  // tokens per prefill attention item (x 4 query heads = 128 rows)
// One query item: consecutive tokens of one segment, one KV head. The tokens see logical keys
// L < shared (slot base + L, the shared region) and then their own segment (slot segment + L -
// shared), in that order; base is 0 except in a batch of independent trees, where each tree's
// shared region starts at its own slot.
struct AttnItem {
    int32_t t0, ntok, kv_head, slot0, shared, segment, nblocks, base;
};
struct AttnArgs {
    const __half* q16;          // [T][heads*hd]
    const AttnItem* items;
    int n_items;
    const __half* kv_pool;
    const int32_t* page_table;
    int64_t page_bytes;
    int page_slots;
    int layer, heads, kv_heads;
    float scale;
    __half* ctx16;              // K-slab [qdim/64][tpad][64]
    int tpad;
    float* ctx32;               // optional [T][qdim]
    int max_keys = 0;           // largest visible-key count of any item (sizes the key table)
    int* err = nullptr;         // device error word (tensor-core kernel's bounded waits)
};
void launch_attention(const AttnArgs& a, cudaStream_t s);
void launch_attention_tc(const AttnArgs& a, cudaStream_t s);
// One bounded wait that nothing completes: gives up after bound_cycles and reports site 33.
void launch_wait_check(int* err, long long bound_cycles, cudaStream_t s);

struct DecodeAttnArgs {
    const float* q32;           // [heads*hd]
    const __half* kv_pool;
    const int32_t* page_table;
    int64_t page_bytes;
    int page_slots;
    int layer, heads, kv_heads, n_keys;  // n_keys = visible logical keys
    int shared, segment;                 // logical key L < shared is slot L, else segment + L - shared
    float scale;
    float* partial;             // workspace
    int splits;
    float* ctx32;               // [heads*hd]
    int* err = nullptr;         // error word (bounds-checked builds)
};
void launch_decode_attention(const DecodeAttnArgs& a, cudaStream_t s);

// ------------------------------------------------------- single-token step

// The per-step values of a decode step, read by the decode kernels from device memory so
// that a step's launches are the same for every token (and can be replayed as a graph).
// Causal step: visible logical keys [0, n_keys) with key L at slot L below `shared`, else at
// slot segment + L - shared.
struct DecodeStep {
    int32_t token, slot, pos, shared, segment, n_keys, index, pad;
};

enum DecMode : int { DEC_STORE = 0, DEC_ADD = 1, DEC_SWIGLU = 2, DEC_QKV = 3, DEC_HEAD = 4 };

struct DecGemvArgs {
    const uint8_t* w = nullptr;  // re-tiled matrix
    int ksteps = 0, rows = 0;
    const float* in = nullptr;   // x (fp32, n_in = 64 * ksteps)
    int n_in = 0;
    const float* norm_w = nullptr;  // RMSNorm gain (modes with a norm)
    float eps = 0.f;
    float* y = nullptr;          // STORE/ADD: [rows]; SWIGLU: [rows / 2]; HEAD: logits [rows]
    float* partial = nullptr;    // [splits][rows]
    int* counters = nullptr;     // [tiles + 1], zero between launches
    int* err = nullptr;          // device error word
    // DEC_QKV
    const DecodeStep* step = nullptr;
    const float2* rope_table = nullptr;
    int heads = 0, kv_heads = 0, layer = 0, orig_ctx = 0;
    float temperature_scale = 0.f;
    float* q32 = nullptr;
    __half* kv_pool = nullptr;
    const int32_t* page_table = nullptr;
    int64_t page_bytes = 0;
    int page_slots = 0;
    // DEC_HEAD
    float* cand_v = nullptr;     // [tiles]
    int* cand_i = nullptr;       // [tiles]
    int32_t* argmax_out = nullptr;
    int advance = 0;             // advance *step to the next token after the argmax
    int32_t* tokens_out = nullptr;  // [steps], written at step->index when advancing
    DecodeStep* step_rw = nullptr;
    // L2 prefetch of bytes a later kernel of the step reads (pf_bytes a multiple of 16, split
    // evenly over the CTAs; nothing waits for it)
    const uint8_t* pf = nullptr;
    int64_t pf_bytes = 0;
};
void launch_dec_gemv(int mode, bool norm, int type, const DecGemvArgs& a, int splits, cudaStream_t s);
int dec_splits_for(const QWeight& w, int sm_count);

struct DecAttnArgs {
    const float* q32;
    const __half* kv_pool;
    const int32_t* page_table;
    int64_t page_bytes;
    int page_slots;
    int layer, heads, kv_heads;
    float scale;
    const DecodeStep* step;
    float* partial;   // [heads][splits][DEC_ATTN_PSTRIDE]
    int* counters;    // [kv_heads], zero between launches
    float* ctx32;     // [heads * 128]
    const uint8_t* pf = nullptr;  // L2 prefetch of a later kernel's weights (as in DecGemvArgs)
    int* err = nullptr;           // error word (bounds-checked builds)
    int64_t pf_bytes = 0;
};
constexpr int DEC_ATTN_KEYS = 64;      // logical keys per attention split
constexpr int DEC_ATTN_PSTRIDE = 132;  // floats per (head, split) partial, 16-byte multiple
void launch_dec_attn(const DecAttnArgs& a, int splits, cudaStream_t s);

void launch_swiglu(const float* gu, int T, int ff, __half* xs, int tpad, float* out32, int* err, cudaStream_t s);
void launch_add(float* h, const float* x, int64_t n, cudaStream_t s);
void launch_head_rows(const QWeight& table, const float* normed, int n_out, const int32_t* rows, int n_rows,
                      float* out, int* err, cudaStream_t s);
void launch_argmax(const float* x, int n, int32_t* out, cudaStream_t s);
void launch_kslab_to_f32(const __half* xs, int T, int K, int tpad, float* out, cudaStream_t s);
// KV pages <-> the reference's flat fp32 snapshot layout (keys of every layer/head, then values).
// Elements [base, base + count) of the flat snapshot (count = 0: to the end), to or from a
// buffer holding exactly those elements.
void launch_kv_export(const __half* pool, const int32_t* page_table, int64_t page_bytes, int page_slots, int layers,
                      int kv_heads, int len, float* out, cudaStream_t s, int64_t base = 0, int64_t count = 0,
                      int* err = nullptr);
void launch_kv_import(__half* pool, const int32_t* page_table, int64_t page_bytes, int page_slots, int layers,
                      int kv_heads, int len, const float* in, int* err, cudaStream_t s, int64_t base = 0,
                      int64_t count = 0);
int64_t launches_total();

void note_launch(int n = 1);
// JV_DEBUG_SYNC (diagnostics): every programmatic-dependent launch is followed by a
// synchronisation of its stream (outside stream capture), and a failure names that kernel and
// the one launched before it. Launches then no longer overlap.
bool debug_sync_enabled();
void debug_after_launch(cudaStream_t s, const void* kernel);

#ifdef __CUDACC__
// Programmatic dependent launch. A kernel launched with launch_pdl may start while the
// previous kernel in the stream is finishing: it calls pdl_launch_dependents() to let the
// kernel after it do the same, and pdl_wait() before it touches anything the previous
// kernel writes (every read of a previous output, and every write, comes after pdl_wait).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

template <class... KArgs, class... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    JV_CUDA(cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...));
    if (debug_sync_enabled()) debug_after_launch(s, (const void*)kernel);
}
#endif

// The calling thread's jv_last_error() message; returns code.
int api_error(int code, const std::string& msg);
// A re-tiled quantized matrix described by the QuantMatMul C ABI; throws on bad arguments.
QWeight qweight_view(int type, const void* tiled, int rows, int cols);

}  // namespace jv
