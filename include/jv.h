/*
 * jv.h — C ABI of the B200 Jevstral forward pass.
 *
 * The .NET host keeps its public API (JevstralDecider, VerdictScorer, SystemPromptCache,
 * the `jev` CLI) and replaces the body of MinistralModel and KvCache with P/Invoke calls
 * into this library. Every entry point below names the reference member it replaces
 * (paths inside theolivenbaum/llm-shield). Signatures hold plain pointers and sizes only.
 *
 * Threading: a jv_model (weights on one GPU) may be shared by several jv_ctx; a jv_ctx
 * (one KV cache, one CUDA stream, activation buffers) is single-threaded, like a
 * MinistralModel instance (src/Jevstral/Model/MinistralModel.cs:21-22).
 *
 * Errors: every int-returning call returns a JV_* status. jv_last_error() gives the
 * calling thread's last message. The C# binding maps codes back to the exception types
 * the reference throws (src/Jevstral/Model/MinistralModel.cs:202,207,306;
 * src/Jevstral/Numerics/QuantMatMul.cs:300-302; src/Jevstral/Model/KvCache.cs:96-97,118-120;
 * src/Jevstral/Gguf/GgufFile.cs:156-172).
 */
#ifndef JV_H
#define JV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum jv_status {
    JV_OK = 0,
    JV_ERR_ARG = 1,            /* ArgumentException / ArgumentNullException          */
    JV_ERR_RANGE = 2,          /* ArgumentOutOfRangeException                        */
    JV_ERR_FORMAT = 3,         /* InvalidDataException / KeyNotFoundException         */
    JV_ERR_IO = 4,             /* IOException / FileNotFoundException                 */
    JV_ERR_UNSUPPORTED = 5,    /* NotSupportedException                              */
    JV_ERR_CANCELLED = 6,      /* OperationCanceledException                         */
    JV_ERR_DEVICE = 7,         /* a CUDA call failed                                 */
    JV_ERR_DEVICE_TIMEOUT = 8, /* a bounded device-side wait gave up                 */
    JV_ERR_OOM = 9,            /* device memory exhausted                            */
    JV_ERR_NUMERIC = 10        /* an activation left the fp16 range of the device path
                                  (|x| >= 65520 or not a number): ArithmeticException.
                                  The reference's fp32 path has no such limit.        */
};

typedef struct jv_model jv_model;       /* weights resident on one device            */
typedef struct jv_ctx jv_ctx;           /* MinistralModel instance: KV cache + stream */
typedef struct jv_snapshot jv_snapshot; /* refcounted KV pages of a prefix            */

/* ModelConfig (src/Jevstral/Model/ModelConfig.cs:11-56), plus the resolved RoPE magnitude
 * scale (Rope.MagnitudeScale, src/Jevstral/Model/Rope.cs:28) and the weight type. */
typedef struct jv_config {
    int32_t layers, hidden, heads, kv_heads, head_dim, ff, vocab, rope_dim;
    int32_t context_length, rope_orig_ctx, yarn_active, weight_type;
    float eps, rope_base, rope_scale, rope_mscale, temperature_scale;
} jv_config;

/* TokenLayout (src/Jevstral/Model/MinistralModel.cs:703-718): token t is written to KV slot
 * slot[t], rotated as position[t], and sees slots [0, shared[t]) and [segment[t], slot[t]].
 * outputs[] are the token indices whose logits are returned; end is one past the highest
 * slot written; sparse is carried for fidelity (it only picks a CPU loop in the reference). */
typedef struct jv_layout {
    const int32_t* slot;
    const int32_t* position;
    const int32_t* shared;
    const int32_t* segment;
    const int32_t* outputs;
    int32_t n_outputs;
    int32_t end;
    int32_t sparse;
} jv_layout;

/* IActivationSink.Observe (src/Jevstral/Model/MinistralModel.cs:787-790). Called
 * synchronously with host fp32 data named as the reference names them: "embeddings",
 * "blk.{l}.attn_norm|q_rope|k_rope|v|attn_weighted|attn_out|post_attn|ffn_norm|ffn_out|output",
 * "final_norm", "logits". */
typedef void (*jv_activation_sink)(void* user, const char* name, const float* values, int32_t rows,
                                   int32_t cols);

/* ---- library / device -------------------------------------------------------------- */

const char* jv_last_error(void);
int jv_device_count(int32_t* count);
/* Counts this library's kernel launches on the calling process (all contexts). */
int64_t jv_kernel_launches(void);
/* How this copy of the library was built (no counterpart in the reference): bit 0 set in the
 * bounds-checked build (libjv_checked.so), whose kernels test every KV page-table lookup and
 * GEMM work unit and fail the call with JV_ERR_RANGE, naming the site, instead of touching
 * memory out of range. The check stands in for a memory checker; it is slower and not for
 * serving. */
#define JV_FEATURE_BOUNDS_CHECK 1
int32_t jv_build_features(void);

/* ---- model (weights) ----------------------------------------------------------------- */

/* new MinistralModel(ggufPath) weight binding (MinistralModel.cs:56-123), GgufFile parsing
 * (src/Jevstral/Gguf/GgufFile.cs:76-172) and ModelConfig.FromGguf (ModelConfig.cs:62-112).
 * Copies the quantized blocks of every matrix to `device` once, re-tiled but bit-identical.
 * kv_pool_mb sizes the device KV page pool (0 = default). */
int jv_model_open(const char* gguf_path, int32_t device, int32_t kv_pool_mb, jv_model** out);
void jv_model_close(jv_model* model);
/* MinistralModel.Config (MinistralModel.cs:48). */
int jv_model_config(const jv_model* model, jv_config* out);

/* ---- context (MinistralModel instance state) ---------------------------------------- */

/* The KvCache + logits buffer a MinistralModel owns (MinistralModel.cs:100-101). */
int jv_ctx_create(jv_model* model, int32_t initial_capacity, jv_ctx** out);
void jv_ctx_destroy(jv_ctx* ctx);
/* Activation capture (the IActivationSink argument of ForwardAsync, MinistralModel.cs:155). */
int jv_ctx_set_sink(jv_ctx* ctx, jv_activation_sink sink, void* user);
/* ParallelOptions.CancellationToken: when *flag becomes non-zero the forward stops between
 * layers and returns JV_ERR_CANCELLED (KernelTests.cs:206-218). NULL clears it. */
int jv_ctx_set_cancel(jv_ctx* ctx, const volatile int32_t* flag);
/* The cudaStream_t every kernel of this context runs on (for event timing). */
void* jv_ctx_stream(jv_ctx* ctx);

/* Per-kernel-class timing with CUDA events on the context's stream (no counterpart in the
 * reference, which times with a Stopwatch around whole calls, src/Jevstral.Cli/Benchmark.cs:549-623).
 * While enabled every launch of the class is bracketed by events; totals accumulate until
 * reset. kind: 0 tensor-core GEMM, 1 GEMV, 2 attention, 3 everything else. flops/bytes are
 * the algorithmic work of the timed launches. */
enum jv_profile_kind { JV_PROF_GEMM = 0, JV_PROF_GEMV = 1, JV_PROF_ATTENTION = 2, JV_PROF_OTHER = 3 };
int jv_ctx_profile(jv_ctx* ctx, int32_t enable);
int jv_ctx_profile_read(jv_ctx* ctx, int32_t kind, double* total_ms, int64_t* launches, double* flops, double* bytes);
int jv_ctx_profile_reset(jv_ctx* ctx);

/* Check of the device-timeout path (no counterpart in the reference, which has no device
 * waits): runs one kernel whose bounded wait nothing completes. The wait gives up after
 * bound_cycles SM clock cycles (0 < bound_cycles <= 4e9; the tensor-core kernels use 4e9,
 * about 2 s), and the call returns JV_ERR_DEVICE_TIMEOUT with the wait named in
 * jv_last_error(). The context stays usable: its error word is cleared and later calls run
 * normally. Nothing faults or hangs. */
int jv_ctx_check_wait_timeout(jv_ctx* ctx, int64_t bound_cycles);

/* ---- forward passes ------------------------------------------------------------------- */

/* MinistralModel.ForwardAsync(tokens, options) (MinistralModel.cs:139) — appends tokens and
 * writes the full-vocabulary logits of the last position to logits[vocab]. With logits ==
 * NULL this is PrefillAsync (MinistralModel.cs:148): KV only, no LM head. */
int jv_forward(jv_ctx* ctx, const int32_t* tokens, int32_t n, float* logits);

/* MinistralModel.ForwardSelectedAsync (MinistralModel.cs:165-172): appends tokens; out[n_rows]
 * = logits of vocab rows `rows` at the last position. */
int jv_forward_selected(jv_ctx* ctx, const int32_t* tokens, int32_t n, const int32_t* rows,
                        int32_t n_rows, float* out);

/* MinistralModel.ForwardTreeAsync (MinistralModel.cs:198-219); ForwardBranchesAsync
 * (MinistralModel.cs:187) when n_trunk == 0. branch_tokens holds the branches back to back
 * (branch_lengths[b] tokens each). out[n_branches][n_rows] = logits of `rows` at each
 * branch's last token. The branch tokens stay in the KV cache, as in the reference. */
int jv_forward_tree(jv_ctx* ctx, const int32_t* trunk, int32_t n_trunk, const int32_t* branch_tokens,
                    const int32_t* branch_lengths, int32_t n_branches, const int32_t* rows,
                    int32_t n_rows, float* out);

/* Many independent ForwardTreeAsync decisions in one pass: the batch entry of the data-parallel
 * path (no single reference member; each decision is what MinistralModel.cs:198-219 computes
 * for its trunk and branches on an empty cache). Decision d has trunk_lengths[d] trunk tokens
 * and branch_counts[d] branches; `tokens` holds each decision's trunk and then its branches,
 * decision after decision, and branch_lengths every branch in that order. A decision sees only
 * its own tokens (not the cache's contents, not the other decisions). out[sum of branch_counts]
 * [n_rows] = logits of `rows` at each branch's last token, in branch order; each row is
 * bit-identical to that decision run alone by jv_forward_tree on an empty cache. The cache is
 * left as it was (its length is restored after the pass). */
int jv_decide_batch(jv_ctx* ctx, int32_t n_decisions, const int32_t* tokens, const int32_t* trunk_lengths,
                    const int32_t* branch_counts, const int32_t* branch_lengths, const int32_t* rows,
                    int32_t n_rows, float* out);

/* The private ForwardAsync(tokens, capture, options, computeLogits, layout, selectedRows,
 * selectedOut) every public overload funnels into (MinistralModel.cs:301-435).
 * layout == NULL means a causal append at the cache end. With rows != NULL, out receives
 * [n_outputs][n_rows] selected logits; with rows == NULL and full_vocab != 0, out receives
 * [n_outputs][vocab] (ForwardTreeLogitsAsync / ForwardRowsAsync, MinistralModel.cs:227-294);
 * with compute_logits != 0, logits receives the last position's full vocabulary. */
int jv_forward_layout(jv_ctx* ctx, const int32_t* tokens, int32_t n, const jv_layout* layout,
                      const int32_t* rows, int32_t n_rows, int32_t full_vocab, float* out,
                      int32_t compute_logits, float* logits);

/* The benchmark's decode loop (src/Jevstral.Cli/Benchmark.cs:411-422): `steps` single-token
 * forwards with the full LM head, each feeding back the argmax
 * (Kernels.ArgMax, src/Jevstral/Numerics/Kernels.cs:146) of the previous one, starting from
 * first_token. Writes the chosen tokens to out_tokens[steps]. */
int jv_decode_greedy(jv_ctx* ctx, int32_t first_token, int32_t steps, int32_t* out_tokens);

/* ---- QuantMatMul on device buffers (src/Jevstral/Numerics/QuantMatMul.cs) -------------
 * A quantized matrix lives on the device in this library's re-tiled layout (the GGUF blocks
 * of 128 rows x 64 columns gathered into one contiguous chunk; bits unchanged). All pointers
 * below are device pointers; stream is a cudaStream_t (NULL = the legacy default stream).
 * type is the GGML type id: 8 Q8_0, 7 Q5_1, 2 Q4_0. rows % 128 == 0, cols % 64 == 0. */

/* Bytes of the re-tiled layout (WeightMatrix, src/Jevstral/Numerics/WeightMatrix.cs:16-66). */
int64_t jv_qweight_bytes(int32_t type, int32_t rows, int32_t cols);
/* Re-tile `rows` GGUF rows (GgmlTypeInfo.RowBytes(type, cols) bytes each, back to back) into
 * `tiled` (jv_qweight_bytes bytes). */
int jv_qweight_pack(int32_t type, const void* gguf_rows, int32_t rows, int32_t cols, void* tiled, void* stream);
/* QuantMatMul.ForwardAsync for one token (QuantMatMul.cs:127-129 -> RunRowsFloat :140-176):
 * y[rows] = W x[cols] with W decoded to fp32 exactly as Dequantizer does and fp32 FMA. Uses a
 * split-K partial buffer that it allocates on the device on first use (and keeps). */
int jv_qmatvec(int32_t type, const void* tiled, int32_t rows, int32_t cols, const float* x, float* y, void* stream);
/* jv_qmatvec without any device allocation. No counterpart in the reference: it is for
 * callers that must not allocate device memory on the call path (a host that has planned
 * all of HBM up front, or one running under a memory cap owned by another component). The
 * split-K partials live in a fixed 1 MiB device array (JV_QMATVEC_SCRATCH_FLOATS_MAX = 262144
 * floats) built into the library; a call needs splits x rows floats (splits as jv_qmatvec
 * picks them) and fails with JV_ERR_RANGE above that. All calls on a device share the array:
 * nothing in it has to start at zero, but calls that overlap in time on one device race, so
 * serialize them. The first call on each device does a one-time set-up (a symbol-address
 * lookup with that device current); make it before any stream capture begins. */
#define JV_QMATVEC_SCRATCH_FLOATS_MAX 262144
int jv_qmatvec_noalloc(int32_t type, const void* tiled, int32_t rows, int32_t cols, const float* x, float* y,
                       void* stream);

/* ---- KV cache (src/Jevstral/Model/KvCache.cs) ----------------------------------------- */

int32_t jv_kv_length(jv_ctx* ctx);                             /* KvCache.Length   :23     */
int32_t jv_kv_capacity(jv_ctx* ctx);                           /* KvCache.Capacity :21     */
int jv_kv_reset(jv_ctx* ctx);                                  /* KvCache.Reset    :43     */
int jv_kv_truncate(jv_ctx* ctx, int32_t length);               /* KvCache.Truncate :46     */
int jv_kv_ensure_capacity(jv_ctx* ctx, int32_t required);      /* EnsureCapacity   :48-70  */
int64_t jv_kv_bytes_per_position(jv_ctx* ctx);                 /* BytesPerPosition :139    */
/* KvCache.Snapshot (:94-112): the reference's flat fp32 layout (keys for every layer and
 * head, then values), so SystemPromptCache files (SystemPromptCache.cs:110-164) stay valid.
 * n_floats must equal jv_kv_snapshot_floats(length). */
int64_t jv_kv_snapshot_floats(jv_ctx* ctx, int32_t length);
int jv_kv_snapshot(jv_ctx* ctx, int32_t length, float* out, int64_t n_floats);
/* KvCache.Restore (:115-136). */
int jv_kv_restore(jv_ctx* ctx, const float* snapshot, int64_t n_floats, int32_t length);

/* SystemPromptCache.Save (src/Jevstral/SystemPromptCache.cs:110-127) straight from the device
 * pages: writes the reference's "SHKV" file for the first n_tokens cached positions — uint32
 * magic 0x53484B56, int32 version 1, the fingerprint string as .NET's BinaryWriter writes it
 * (7-bit-encoded UTF-8 byte count, then the bytes), int32 token count, the tokens, int64 float
 * count, then the KvCache.Snapshot floats (:94-112) — streamed one (K|V, layer) slice at a time
 * through pinned memory, so the whole state never sits in host memory. The fingerprint is the
 * host's (ComputeFingerprint, :91-106); n_tokens must not exceed the cached length. */
int jv_kv_save_shkv(jv_ctx* ctx, const char* path, const char* fingerprint, const int32_t* tokens, int32_t n_tokens);
/* SystemPromptCache.TryLoad + RestoreInto (SystemPromptCache.cs:65-74,133-164) into the device
 * pages: reads an SHKV file, checks its magic, version, that its fingerprint equals `fingerprint`
 * and that its float count fits its token count on this model, then streams the floats into the
 * pages (the cache then holds exactly that prefix) and writes the tokens to tokens_out
 * (max_tokens entries) and their count to *n_tokens. TryLoad's miss (null) is JV_ERR_IO for a file
 * that cannot be opened and JV_ERR_FORMAT for one that is not a valid snapshot of this model and
 * prefix; both leave the cache as it was. */
int jv_kv_load_shkv(jv_ctx* ctx, const char* path, const char* fingerprint, int32_t* tokens_out, int32_t max_tokens,
                    int32_t* n_tokens);

/* Zero-copy prefix reuse (the question-snapshot LRU and system-prompt cache of
 * JevstralDecider.cs:131-137,262-280 without the memcpy): jv_kv_share pins the pages that
 * hold the first `length` positions; jv_kv_adopt makes a context's cache exactly that prefix
 * (copy-on-write for the one partially filled page). Contexts must share the jv_model. */
int jv_kv_share(jv_ctx* ctx, int32_t length, jv_snapshot** out);
int jv_kv_adopt(jv_ctx* ctx, const jv_snapshot* snapshot);
int32_t jv_snapshot_length(const jv_snapshot* snapshot);
void jv_snapshot_release(jv_snapshot* snapshot);

#ifdef __cplusplus
}
#endif

#endif /* JV_H */
