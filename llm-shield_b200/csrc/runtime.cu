// runtime.cu — the host side of the B200 Jevstral forward pass behind include/jv.h.
//
// jv_model  = the weight-holding half of MinistralModel (reference
//             src/Jevstral/Model/MinistralModel.cs:59-123): GGUF parse, ModelConfig, RoPE
//             frequencies, quantized matrices re-tiled into HBM, the KV page pool.
// jv_ctx    = the per-request half: KvCache (src/Jevstral/Model/KvCache.cs) as a page table
//             into the pool, one CUDA stream, activation buffers, the logits buffer.
// forward() = the private ForwardAsync (MinistralModel.cs:301-435) as a fixed sequence of
//             kernel launches on the context's stream.
#include <algorithm>
#include <cstddef>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "gguf.h"
#include "jv_internal.h"

using namespace jv;

// The structs of the ABI as the C# binding mirrors them (LayoutKind.Sequential, default packing):
// a change here is a breaking change of the binding.
static_assert(sizeof(jv_config) == 68, "jv_config: 12 int32 then 5 float");
static_assert(offsetof(jv_config, weight_type) == 44 && offsetof(jv_config, eps) == 48, "jv_config field offsets");
static_assert(offsetof(jv_config, temperature_scale) == 64, "jv_config field offsets");
static_assert(sizeof(jv_layout) == 56, "jv_layout: 5 pointers then 3 int32 (+4 padding)");
static_assert(offsetof(jv_layout, outputs) == 32 && offsetof(jv_layout, n_outputs) == 40, "jv_layout field offsets");
static_assert(offsetof(jv_layout, end) == 44 && offsetof(jv_layout, sparse) == 48, "jv_layout field offsets");

namespace {

thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

template <class F>
int guarded(F&& f) {
    try {
        f();
        return JV_OK;
    } catch (const Error& e) {
        return set_error(e.code, e.what());
    } catch (const std::bad_alloc&) {
        return set_error(JV_ERR_OOM, "host memory exhausted");
    } catch (const std::exception& e) {
        return set_error(JV_ERR_ARG, e.what());
    }
}

template <class T>
T* dalloc(size_t n) {
    if (n == 0) n = 1;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, n * sizeof(T));
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw Error(e == cudaErrorMemoryAllocation ? JV_ERR_OOM : JV_ERR_DEVICE,
                    "cudaMalloc of " + std::to_string(n * sizeof(T)) + " bytes: " + cudaGetErrorString(e));
    }
    return (T*)p;
}

// A device buffer that grows to the largest request (activations are re-used call to call).
template <class T>
struct DevVec {
    T* p = nullptr;
    size_t cap = 0;
    T* get(size_t n) {
        if (n > cap) {
            if (p) cudaFree(p);
            p = nullptr;
            cap = 0;
            p = dalloc<T>(n);
            // Zeroed and finished before the buffer is handed out: the contexts' streams are
            // non-blocking, so a memset left pending on the legacy stream could land after (and
            // wipe) what the first call's kernels write into the new buffer.
            JV_CUDA(cudaMemsetAsync(p, 0, n * sizeof(T), cudaStreamLegacy));
            JV_CUDA(cudaStreamSynchronize(cudaStreamLegacy));
            cap = n;
        }
        return p;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
};

template <class T>
struct HostVec {  // pinned
    T* p = nullptr;
    size_t cap = 0;
    T* get(size_t n) {
        if (n > cap) {
            if (p) cudaFreeHost(p);
            p = nullptr;
            cap = 0;
            JV_CUDA(cudaMallocHost((void**)&p, std::max<size_t>(n, 1) * sizeof(T)));
            cap = n;
        }
        return p;
    }
    void release() {
        if (p) cudaFreeHost(p);
        p = nullptr;
        cap = 0;
    }
};

struct LayerW {
    QWeight qkv, o, gu, down;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
};

}  // namespace

struct jv_model {
    int device = 0;
    int sm_count = 148;
    jv_config cfg{};
    std::vector<float> freqs;
    float mscale = 1.f;
    QWeight embd, head;  // head == embd when the LM head is tied (no output.weight)
    bool tied = true;
    bool has_qx = false;  // some matrix was converted to the affine layout (no fused decode kernels)
    float* out_norm = nullptr;
    std::vector<LayerW> layers;
    float2* rope_table = nullptr;
    int rope_positions = 0;
    // KV page pool: page p holds 64 slots of every layer and KV head, K and V.
    __half* pool = nullptr;
    int n_pages = 0;
    int page_slots = 64;
    int64_t page_bytes = 0;
    std::vector<int> refcount;
    std::vector<int> free_pages;
    std::mutex mu;
    std::vector<void*> allocations;

    int alloc_page() {
        std::lock_guard<std::mutex> g(mu);
        if (free_pages.empty())
            throw Error(JV_ERR_OOM, "KV page pool exhausted (" + std::to_string(n_pages) + " pages of " +
                                        std::to_string(page_slots) + " slots); open the model with a larger kv_pool_mb");
        int p = free_pages.back();
        free_pages.pop_back();
        refcount[p] = 1;
        return p;
    }
    void retain(int p) {
        std::lock_guard<std::mutex> g(mu);
        refcount[p]++;
    }
    void release(int p) {
        std::lock_guard<std::mutex> g(mu);
        if (--refcount[p] == 0) free_pages.push_back(p);
    }
    int refs(int p) {
        std::lock_guard<std::mutex> g(mu);
        return refcount[p];
    }
};

struct jv_snapshot {
    jv_model* model;
    std::vector<int> pages;
    int length;
};

struct jv_ctx {
    jv_model* m = nullptr;
    cudaStream_t stream = nullptr;
    int length = 0;     // KvCache.Length
    int capacity = 0;   // KvCache.Capacity (doubling, as the reference reports it)
    std::vector<int> pages;  // logical page -> physical page
    DevVec<int32_t> d_pages;
    bool pages_dirty = true;
    jv_activation_sink sink = nullptr;
    void* sink_user = nullptr;
    const volatile int32_t* cancel = nullptr;
    // device activations
    DevVec<float> h, qkv32, gu32, tmp32, q32, ctx32, x32, act32, k32, partial, out32, logits, cap32;
    DevVec<__half> xs, xs_ff, ctx16, q16;
    DevVec<int32_t> in_i32, out_i32;
    DevVec<float> gemm_ws;   // split-K partials
    DevVec<int> gemm_ctr;    // split-K arrival counters (the last CTA of a tile resets its own)
    DevVec<AttnItem> items;
    // single-token steps: arrival counters (zero between launches), head candidates, and the
    // device-resident step of the greedy loop
    DevVec<int> dec_ctr, dec_cand_i;
    DevVec<float> dec_cand_v, dec_attn;
    DevVec<DecodeStep> dec_step;
    DevVec<int32_t> dec_tokens;
    // jv_decode_greedy replays one captured step; the capture is valid while every buffer it
    // names (and the attention split count) is unchanged
    cudaGraphExec_t dec_graph = nullptr;
    std::vector<const void*> dec_graph_sig;
    int* d_err = nullptr;
    HostVec<int32_t> h_in;
    HostVec<float> h_out;
    HostVec<float> h_cap;
    HostVec<int32_t> h_err;
    // jv_ctx_profile: events around GEMM / GEMV / attention launches
    struct Pending {
        cudaEvent_t a, b;
        int kind;
        double flops, bytes;
    };
    bool prof = false;
    std::vector<Pending> pending;
    std::vector<cudaEvent_t> spare_events;
    double prof_ms[4] = {0, 0, 0, 0}, prof_flops[4] = {0, 0, 0, 0}, prof_bytes[4] = {0, 0, 0, 0};
    int64_t prof_launches[4] = {0, 0, 0, 0};

    cudaEvent_t take_event() {
        if (!spare_events.empty()) {
            cudaEvent_t e = spare_events.back();
            spare_events.pop_back();
            return e;
        }
        cudaEvent_t e;
        JV_CUDA(cudaEventCreate(&e));
        return e;
    }
    // Called after the stream is synchronized.
    void resolve_profile() {
        for (auto& p : pending) {
            float ms = 0.f;
            JV_CUDA(cudaEventElapsedTime(&ms, p.a, p.b));
            prof_ms[p.kind] += ms;
            prof_flops[p.kind] += p.flops;
            prof_bytes[p.kind] += p.bytes;
            prof_launches[p.kind] += 1;
            spare_events.push_back(p.a);
            spare_events.push_back(p.b);
        }
        pending.clear();
    }
};

namespace {
// Brackets the launches issued in its lifetime with events when profiling is on.
struct ProfScope {
    jv_ctx* x;
    jv_ctx::Pending p;
    ProfScope(jv_ctx* ctx, int kind, double flops, double bytes) : x(ctx) {
        if (!x->prof) return;
        p.a = x->take_event();
        p.b = x->take_event();
        p.kind = kind;
        p.flops = flops;
        p.bytes = bytes;
        JV_CUDA(cudaEventRecord(p.a, x->stream));
    }
    ~ProfScope() {
        if (!x->prof) return;
        if (cudaEventRecord(p.b, x->stream) == cudaSuccess) x->pending.push_back(p);
    }
};

double weight_bytes(const QWeight& w) { return (double)w.bytes(); }
}  // namespace

namespace {

void set_device(const jv_model* m) { JV_CUDA(cudaSetDevice(m->device)); }

// ------------------------------------------------------------ model load

bool native_type(int t) { return t == T_Q8_0 || t == T_Q4_0 || t == T_Q5_1; }

// The device layout of a matrix assembled from GGUF tensors of `types`: their own when they are
// one of the three formats the kernels decode directly, else the affine layout T_QX, which takes
// every other block format (and mixes of them, as the K-quant files do per tensor).
int pick_type(std::initializer_list<int> types, const std::string& what) {
    const int first = *types.begin();
    bool same = true, affine = true;
    for (int t : types) {
        same &= t == first;
        affine &= qx_expressible(t);
    }
    if (same && native_type(first)) return first;
    if (affine) return T_QX;
    throw Error(JV_ERR_UNSUPPORTED, what + ": weight type " + std::to_string(first) +
                                        " is not on the B200 path (Q8_0, Q5_1, Q4_0, and Q4_1, Q5_0, Q8_1, Q2_K-Q6_K "
                                        "through the affine layout, are)");
}

QWeight alloc_qweight(jv_model* m, int type, int rows, int cols) {
    if (!native_type(type) && type != T_QX)
        throw Error(JV_ERR_UNSUPPORTED, "weight type " + std::to_string(type) +
                                            " is not on the B200 path (Q8_0, Q5_1 and Q4_0 are)");
    if (type == T_QX) m->has_qx = true;
    if (rows % TILE_ROWS != 0 || cols % TILE_K != 0)
        throw Error(JV_ERR_UNSUPPORTED, "matrix " + std::to_string(rows) + "x" + std::to_string(cols) +
                                            " does not tile into 128 rows x 64 columns");
    QWeight w;
    w.type = type;
    w.rows = rows;
    w.cols = cols;
    w.tiles = rows / TILE_ROWS;
    w.ksteps = cols / TILE_K;
    w.data = dalloc<uint8_t>(w.bytes());
    m->allocations.push_back(w.data);
    return w;
}

struct Loader {
    jv_model* m;
    Gguf& g;
    cudaStream_t s;
    uint8_t* staging = nullptr;
    size_t staging_cap = 0;

    const GgufTensor& need(const std::string& name) {
        const GgufTensor* t = g.tensor(name);
        if (!t) throw Error(JV_ERR_FORMAT, g.path() + " is missing tensor '" + name + "'.");
        return *t;
    }
    void matrix_shape(const GgufTensor& t, int& rows, int& cols) {
        if (t.shape.size() != 2)
            throw Error(JV_ERR_FORMAT, "'" + t.name + "' has " + std::to_string(t.shape.size()) + " dimensions; a weight matrix needs 2.");
        rows = (int)t.shape[1];
        cols = (int)t.shape[0];
    }
    // Upload a GGUF matrix's raw rows and re-tile them into w. For the affine layout the rows
    // are converted on the host first (qx.cpp), then re-tiled the same way.
    void upload(const GgufTensor& t, QWeight& w, int tile_offset, int interleave, int rit_base) {
        int rows, cols;
        matrix_shape(t, rows, cols);
        if (t.type != w.type && w.type != T_QX)
            throw Error(JV_ERR_UNSUPPORTED, "'" + t.name + "' is " + std::to_string(t.type) +
                                                " but the fused matrix it belongs to is " + std::to_string(w.type));
        if (cols != w.cols) throw Error(JV_ERR_FORMAT, "'" + t.name + "' width disagrees with its fused matrix");
        int64_t rb = Gguf::row_bytes(t.type, cols);
        const uint8_t* src = g.data(t);
        std::vector<uint8_t> converted;
        if (w.type == T_QX) {
            converted.resize((size_t)qx_row_bytes(cols) * rows);
            qx_convert_rows(t.type, src, rb, rows, cols, converted.data());
            src = converted.data();
            rb = qx_row_bytes(cols);
        }
        size_t bytes = (size_t)rb * rows;
        if (bytes > staging_cap) {
            if (staging) cudaFree(staging);
            staging = nullptr;
            staging = dalloc<uint8_t>(bytes);
            staging_cap = bytes;
        }
        JV_CUDA(cudaMemcpyAsync(staging, src, bytes, cudaMemcpyHostToDevice, s));
        launch_repack(staging, w.type, rows, cols, rb, w.data, w.tiles, w.ksteps, rit_base, tile_offset, interleave, s);
        JV_CUDA(cudaStreamSynchronize(s));
    }
    float* vector(const std::string& name, int n) {
        const GgufTensor& t = need(name);
        int64_t elems = 1;
        for (auto d : t.shape) elems *= d;
        if (elems != n) throw Error(JV_ERR_FORMAT, "'" + name + "' has " + std::to_string(elems) + " elements; expected " + std::to_string(n));
        std::vector<float> v((size_t)n);
        const uint8_t* p = g.data(t);
        for (int i = 0; i < n; i++) {
            if (t.type == T_F32) {
                std::memcpy(&v[i], p + 4 * i, 4);
            } else if (t.type == T_F16) {
                __half_raw hr;
                std::memcpy(&hr.x, p + 2 * i, 2);
                v[i] = __half2float(__half(hr));
            } else if (t.type == T_BF16) {
                uint32_t bits = (uint32_t)(p[2 * i] | (p[2 * i + 1] << 8)) << 16;
                std::memcpy(&v[i], &bits, 4);
            } else {
                throw Error(JV_ERR_UNSUPPORTED, "'" + name + "' must be F32, F16 or BF16");
            }
        }
        float* d = dalloc<float>(n);
        m->allocations.push_back(d);
        JV_CUDA(cudaMemcpy(d, v.data(), sizeof(float) * n, cudaMemcpyHostToDevice));
        return d;
    }
    ~Loader() {
        if (staging) cudaFree(staging);
    }
};

// ModelConfig.FromGguf (reference src/Jevstral/Model/ModelConfig.cs:62-112), same keys and defaults.
void read_config(const Gguf& g, jv_model* m) {
    std::string a = g.str("general.architecture", "");
    if (a.empty()) throw Error(JV_ERR_FORMAT, g.path() + " has no general.architecture.");
    if (a != "mistral3" && a != "ministral3" && a != "llama")
        throw Error(JV_ERR_UNSUPPORTED, g.path() + " is architecture '" + a +
                                            "'; this runtime implements the Ministral-3 backbone (GGUF architecture \"mistral3\").");
    jv_config& c = m->cfg;
    c.heads = (int)g.req_num(a + ".attention.head_count");
    c.hidden = (int)g.req_num(a + ".embedding_length");
    c.head_dim = (int)g.num(a + ".attention.key_length", c.hidden / std::max(1, c.heads));
    c.layers = (int)g.req_num(a + ".block_count");
    c.kv_heads = (int)g.num(a + ".attention.head_count_kv", c.heads);
    c.ff = (int)g.req_num(a + ".feed_forward_length");
    int64_t tokens = g.array_len("tokenizer.ggml.tokens", -1);
    c.vocab = tokens >= 0 ? (int)tokens : (int)g.req_num(a + ".vocab_size");
    c.eps = (float)g.num(a + ".attention.layer_norm_rms_epsilon", 1e-5);
    c.context_length = (int)g.num(a + ".context_length", 32768);
    c.rope_base = (float)g.num(a + ".rope.freq_base", 10000.0);
    c.rope_dim = (int)g.num(a + ".rope.dimension_count", c.head_dim);
    c.rope_scale = (float)g.num(a + ".rope.scaling.factor", 1.0);
    std::string rtype = g.str(a + ".rope.scaling.type", "");
    c.rope_orig_ctx = (int)g.num(a + ".rope.scaling.original_context_length", 0);
    float beta_fast = (float)g.num(a + ".rope.scaling.yarn_beta_fast", g.num(a + ".rope.scaling.beta_fast", 32.0));
    float beta_slow = (float)g.num(a + ".rope.scaling.yarn_beta_slow", g.num(a + ".rope.scaling.beta_slow", 1.0));
    float ext = (float)g.num(a + ".rope.scaling.yarn_ext_factor", 1.0);
    float yarn_m = (float)g.num(a + ".rope.scaling.mscale", 0.0);
    float yarn_m_all = (float)g.num(a + ".rope.scaling.yarn_log_multiplier", g.num(a + ".rope.scaling.mscale_all_dim", 0.0));
    float attn_factor = (float)g.num(a + ".rope.scaling.attn_factor", g.num(a + ".rope.scaling.yarn_attn_factor", 1.0));
    c.temperature_scale = (float)g.num(a + ".attention.temperature_scale", g.num(a + ".rope.scaling_beta", 0.0));
    if (c.kv_heads <= 0 || c.heads % c.kv_heads != 0)
        throw Error(JV_ERR_FORMAT, std::to_string(c.heads) + " attention heads do not divide into " +
                                       std::to_string(c.kv_heads) + " KV heads.");
    c.yarn_active = rtype == "yarn" && c.rope_orig_ctx > 0 && ext != 0.f && c.rope_scale > 1.f;

    // Rope(), reference src/Jevstral/Model/Rope.cs:33-106.
    int half = c.rope_dim / 2;
    m->freqs.assign(half, 0.f);
    float freq_scale = 1.f / c.rope_scale;
    if (!c.yarn_active) {
        for (int i = 0; i < half; i++) m->freqs[i] = freq_scale / std::pow(c.rope_base, 2.f * i / c.rope_dim);
        m->mscale = attn_factor;
    } else {
        float low, high;
        if (beta_fast == 0.f && beta_slow == 0.f) {
            low = std::numeric_limits<float>::max();
            high = c.rope_dim / 2.f - 1.f;
        } else {
            auto corr = [&](float rot) {
                return c.rope_dim * std::log(c.rope_orig_ctx / (rot * 2 * (float)M_PI)) / (2 * std::log(c.rope_base));
            };
            low = std::max(0.f, std::floor(corr(beta_fast)));
            high = std::min(c.rope_dim / 2.f - 1.f, std::ceil(corr(beta_slow)));
        }
        for (int i = 0; i < half; i++) {
            float extrap = 1.f / std::pow(c.rope_base, 2.f * i / c.rope_dim);
            float interp = freq_scale * extrap;
            float y = (i - low) / std::max(0.001f, high - low);
            float mix = (1.f - std::min(std::max(y, 0.f), 1.f)) * ext;
            m->freqs[i] = interp * (1.f - mix) + extrap * mix;
        }
        auto ms = [](float scale, float mm) { return scale <= 1.f ? 1.f : 0.1f * mm * std::log(scale) + 1.f; };
        float mm = yarn_m != 0.f ? yarn_m : 1.f;
        float ratio = yarn_m_all != 0.f ? ms(c.rope_scale, mm) / ms(c.rope_scale, yarn_m_all) : ms(c.rope_scale, 1.f);
        m->mscale = ratio * attn_factor;
    }
    c.rope_mscale = m->mscale;
}

void load_model(jv_model* m, const std::string& path, int kv_pool_mb) {
    Gguf g(path);
    read_config(g, m);
    jv_config& c = m->cfg;
    if (c.head_dim != 128) throw Error(JV_ERR_UNSUPPORTED, "the B200 attention kernels need head_dim 128");
    if (c.rope_dim != c.head_dim) throw Error(JV_ERR_UNSUPPORTED, "partial rotary embeddings are not supported");
    if (c.heads / c.kv_heads != 4) throw Error(JV_ERR_UNSUPPORTED, "the B200 attention kernels pack 4 query heads per KV head");
    if (c.ff % 64 != 0) throw Error(JV_ERR_UNSUPPORTED, "feed_forward_length must be a multiple of 64");

    cudaStream_t s;
    JV_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    struct StreamGuard { cudaStream_t s; ~StreamGuard() { cudaStreamDestroy(s); } } sg{s};
    Loader L{m, g, s};

    // Embedding table (tied LM head unless output.weight exists).
    {
        const GgufTensor& t = L.need("token_embd.weight");
        int rows, cols;
        L.matrix_shape(t, rows, cols);
        if (cols != c.hidden)
            throw Error(JV_ERR_FORMAT, "token_embd is " + std::to_string(cols) + " wide but the model's hidden size is " + std::to_string(c.hidden) + ".");
        m->embd = alloc_qweight(m, pick_type({t.type}, "token_embd"), rows, cols);
        L.upload(t, m->embd, 0, 0, 0);
        if (c.vocab > rows) c.vocab = rows;
    }
    if (const GgufTensor* t = g.tensor("output.weight")) {
        int rows, cols;
        L.matrix_shape(*t, rows, cols);
        m->head = alloc_qweight(m, pick_type({t->type}, "output"), rows, cols);
        L.upload(*t, m->head, 0, 0, 0);
        m->tied = false;
    } else {
        m->head = m->embd;
        m->tied = true;
    }
    m->out_norm = L.vector("output_norm.weight", c.hidden);

    int qdim = c.heads * c.head_dim, kvdim = c.kv_heads * c.head_dim;
    m->layers.resize(c.layers);
    for (int l = 0; l < c.layers; l++) {
        std::string p = "blk." + std::to_string(l) + ".";
        LayerW& W = m->layers[l];
        W.attn_norm = L.vector(p + "attn_norm.weight", c.hidden);
        W.ffn_norm = L.vector(p + "ffn_norm.weight", c.hidden);
        const GgufTensor& tq = L.need(p + "attn_q.weight");
        const GgufTensor& tk = L.need(p + "attn_k.weight");
        const GgufTensor& tv = L.need(p + "attn_v.weight");
        const GgufTensor& to = L.need(p + "attn_output.weight");
        const GgufTensor& tg = L.need(p + "ffn_gate.weight");
        const GgufTensor& tu = L.need(p + "ffn_up.weight");
        const GgufTensor& td = L.need(p + "ffn_down.weight");
        int r, k;
        L.matrix_shape(tq, r, k);
        if (r != qdim) throw Error(JV_ERR_FORMAT, "attn_q has " + std::to_string(r) + " rows; expected " + std::to_string(qdim) + ".");
        L.matrix_shape(tk, r, k);
        if (r != kvdim) throw Error(JV_ERR_FORMAT, "attn_k has " + std::to_string(r) + " rows; expected " + std::to_string(kvdim) + ".");
        L.matrix_shape(tg, r, k);
        if (r != c.ff) throw Error(JV_ERR_FORMAT, "ffn_gate has " + std::to_string(r) + " rows; expected " + std::to_string(c.ff) + ".");
        // [Wq; Wk; Wv] as one matrix: one GEMM writes q | k | v per token.
        W.qkv = alloc_qweight(m, pick_type({tq.type, tk.type, tv.type}, p + "attn_q/k/v"), qdim + 2 * kvdim, c.hidden);
        L.upload(tq, W.qkv, 0, 0, 0);
        L.upload(tk, W.qkv, qdim / TILE_ROWS, 0, 0);
        L.upload(tv, W.qkv, (qdim + kvdim) / TILE_ROWS, 0, 0);
        int orows, ocols;
        L.matrix_shape(to, orows, ocols);
        W.o = alloc_qweight(m, pick_type({to.type}, p + "attn_output"), orows, ocols);
        L.upload(to, W.o, 0, 0, 0);
        // gate and up interleaved in alternating 16-row groups of each 128-row tile.
        W.gu = alloc_qweight(m, pick_type({tg.type, tu.type}, p + "ffn_gate/up"), 2 * c.ff, c.hidden);
        L.upload(tg, W.gu, 0, 1, 0);
        L.upload(tu, W.gu, 0, 1, 16);
        int drows, dcols;
        L.matrix_shape(td, drows, dcols);
        W.down = alloc_qweight(m, pick_type({td.type}, p + "ffn_down"), drows, dcols);
        L.upload(td, W.down, 0, 0, 0);
        if (W.o.rows != c.hidden || W.o.cols != qdim || W.down.rows != c.hidden || W.down.cols != c.ff)
            throw Error(JV_ERR_FORMAT, "blk." + std::to_string(l) + " projection shapes disagree with the config");
    }
    // the file's own type of the first layer's query projection (the embedding's when there are none)
    c.weight_type = g.tensor(c.layers > 0 ? "blk.0.attn_q.weight" : "token_embd.weight")->type;

    // RoPE table for every position the context window allows.
    m->rope_positions = std::max(c.context_length, 32768);
    int half = c.rope_dim / 2;
    float* d_freqs = dalloc<float>(half);
    JV_CUDA(cudaMemcpy(d_freqs, m->freqs.data(), sizeof(float) * half, cudaMemcpyHostToDevice));
    m->rope_table = dalloc<float2>((size_t)m->rope_positions * half);
    m->allocations.push_back(m->rope_table);
    launch_rope_table(m->rope_table, d_freqs, half, 0, m->rope_positions, m->mscale, s);
    JV_CUDA(cudaStreamSynchronize(s));
    cudaFree(d_freqs);

    // KV page pool.
    m->page_bytes = (int64_t)c.layers * c.kv_heads * 2 * m->page_slots * c.head_dim * sizeof(__half);
    int64_t pool_bytes = (int64_t)(kv_pool_mb > 0 ? kv_pool_mb : 8192) << 20;
    m->n_pages = (int)std::max<int64_t>(4, pool_bytes / m->page_bytes);
    m->pool = dalloc<__half>((size_t)m->n_pages * m->page_bytes / sizeof(__half));
    m->allocations.push_back(m->pool);
    m->refcount.assign(m->n_pages, 0);
    for (int i = m->n_pages - 1; i >= 0; i--) m->free_pages.push_back(i);
    JV_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------ KV pages

void ctx_ensure_capacity(jv_ctx* x, int required) {
    // KvCache.EnsureCapacity (KvCache.cs:48-70): the reported capacity doubles; pages are
    // only taken from the pool for the slots actually needed.
    if (required > x->capacity) {
        int cap = std::max(1, x->capacity);
        while (cap < required) cap *= 2;
        x->capacity = cap;
    }
    int need_pages = (required + x->m->page_slots - 1) / x->m->page_slots;
    while ((int)x->pages.size() < need_pages) {
        x->pages.push_back(x->m->alloc_page());
        x->pages_dirty = true;
    }
}

// Copy-on-write for pages shared with a snapshot or another context that this pass writes.
void ctx_make_writable(jv_ctx* x, const std::vector<int>& written_pages) {
    for (int lp : written_pages) {
        int pp = x->pages[lp];
        if (x->m->refs(pp) > 1) {
            int np = x->m->alloc_page();
            JV_CUDA(cudaMemcpyAsync((char*)x->m->pool + (int64_t)np * x->m->page_bytes,
                                    (char*)x->m->pool + (int64_t)pp * x->m->page_bytes, x->m->page_bytes,
                                    cudaMemcpyDeviceToDevice, x->stream));
            x->m->release(pp);
            x->pages[lp] = np;
            x->pages_dirty = true;
        }
    }
}

// The device page table: two words (the entry count and the pool's page count, which the
// bounds-checked build tests every lookup against), then logical page -> physical page.
void ctx_upload_pages(jv_ctx* x) {
    if (!x->pages_dirty) return;
    std::vector<int32_t> h(2 + x->pages.size());
    h[0] = (int32_t)x->pages.size();
    h[1] = x->m->n_pages;
    std::copy(x->pages.begin(), x->pages.end(), h.begin() + 2);
    int32_t* d = x->d_pages.get(h.size());
    JV_CUDA(cudaMemcpyAsync(d, h.data(), sizeof(int32_t) * h.size(), cudaMemcpyHostToDevice, x->stream));
    JV_CUDA(cudaStreamSynchronize(x->stream));  // the host vector may change before the copy would run
    x->pages_dirty = false;
}
const int32_t* ctx_table(jv_ctx* x) { return x->d_pages.p + 2; }

void ctx_release_pages(jv_ctx* x) {
    for (int p : x->pages) x->m->release(p);
    x->pages.clear();
    x->pages_dirty = true;
}

// ------------------------------------------------------------ forward

struct HostLayout {
    std::vector<int32_t> slot, pos, shared, seg, outputs;
    std::vector<int32_t> base;  // first slot of each token's shared region; empty = 0 (TokenLayout's case)
    int end = 0;
};

void check_cancel(jv_ctx* x) {
    if (x->cancel && *x->cancel) throw Error(JV_ERR_CANCELLED, "The operation was canceled.");
}

// Sites of a device-side timeout (report_timeout in tc_common.cuh): kernel x 16 + role.
const char* timeout_site(int site) {
    switch (site) {
        case 1: return "tensor-core GEMM, weight producer";
        case 2: return "tensor-core GEMM, activation producer";
        case 3: return "tensor-core GEMM, producer teardown";
        case 4: return "tensor-core GEMM, MMA issuer";
        case 5: return "tensor-core GEMM, MMA teardown";
        case 6: return "tensor-core GEMM, decoders";
        case 7: return "tensor-core GEMM, epilogue";
        case 8: return "tensor-core GEMM, decoders draining the last tile";
        case 17: return "tensor-core attention, K loader";
        case 18: return "tensor-core attention, V loader";
        case 19: return "tensor-core attention, MMA issuer";
        case 20: return "tensor-core attention, softmax of query tile A";
        case 21: return "tensor-core attention, softmax of query tile B";
        case 33: return "the wait check, which nothing completes";
        case 49: return "decode matvec, weight-slice copy";
        default: return "a device kernel";
    }
}

const char* bounds_site(int site) {
    switch (site) {
        case BS_ROPE_PAGE: return "RoPE / K-V write: page table";
        case BS_ATTN_PAGE: return "tensor-core attention: page table";
        case BS_ATTN_STAGED: return "tensor-core attention: staged page entry";
        case BS_MMA_ATTN_PAGE: return "mma.sync attention: page table";
        case BS_DECODE_PAGE: return "single-token step: page table";
        case BS_GEMM_UNIT: return "GEMM work unit";
        case BS_SNAPSHOT_PAGE: return "snapshot export/import: page table";
        default: return "a token id or vocabulary row";
    }
}

const char* numeric_site(int site) {
    switch (site) {
        case NS_RMSNORM: return "an RMSNorm (the fp16 operand of the next projection)";
        case NS_ROPE_KV: return "the RoPE / K-V page write";
        case NS_SWIGLU: return "the SwiGLU activation (the fp16 operand of the down projection)";
        case NS_DEC_INPUT: return "the input of a single-token matvec";
        case NS_DEC_KV: return "the single-token K-V page write";
        case NS_KV_RESTORE: return "a KV snapshot restore";
        default: return "a device kernel";
    }
}

void sync_check(jv_ctx* x) {
    JV_CUDA(cudaMemcpyAsync(x->h_err.get(2), x->d_err, 2 * sizeof(int), cudaMemcpyDeviceToHost, x->stream));
    JV_CUDA(cudaStreamSynchronize(x->stream));
    const int e = x->h_err.p[0], site = x->h_err.p[1];
    if (e != 0) {
        JV_CUDA(cudaMemsetAsync(x->d_err, 0, 2 * sizeof(int), x->stream));
        if (x->gemm_ctr.p) JV_CUDA(cudaMemsetAsync(x->gemm_ctr.p, 0, x->gemm_ctr.cap * sizeof(int), x->stream));
        JV_CUDA(cudaStreamSynchronize(x->stream));
        if (e == JV_ERR_DEVICE_TIMEOUT)
            throw Error(JV_ERR_DEVICE_TIMEOUT, std::string("a device-side wait timed out (") + timeout_site(site) + ")");
        if (e == JV_ERR_NUMERIC)
            throw Error(JV_ERR_NUMERIC, std::string("an activation left the fp16 range the device path computes in "
                                                    "(|x| >= 65520, or not a number) at ") + numeric_site(site) +
                                            "; the reference's fp32 path has no such limit");
        throw Error(e, std::string("a kernel reported an out-of-range index (") + bounds_site(site) + ")");
    }
}

// IActivationSink.Observe for a device fp32 tensor [rows][cols] (row stride ld).
void observe(jv_ctx* x, const std::string& name, const float* d, int rows, int cols, int ld = -1) {
    if (!x->sink) return;
    if (ld < 0) ld = cols;
    size_t n = (size_t)rows * cols;
    float* hbuf = x->h_cap.get(n);
    JV_CUDA(cudaMemcpy2DAsync(hbuf, sizeof(float) * cols, d, sizeof(float) * ld, sizeof(float) * cols, rows,
                              cudaMemcpyDeviceToHost, x->stream));
    JV_CUDA(cudaStreamSynchronize(x->stream));
    x->sink(x->sink_user, name.c_str(), hbuf, rows, cols);
}
void observe_kslab(jv_ctx* x, const std::string& name, const __half* xs, int T, int K, int tpad) {
    if (!x->sink) return;
    float* tmp = x->cap32.get((size_t)T * K);
    launch_kslab_to_f32(xs, T, K, tpad, tmp, x->stream);
    observe(x, name, tmp, T, K);
}

// JV_ATTN_KERNEL=mma selects the mma.sync prefill attention (kernels_attn.cu) instead of the
// tcgen05 one (attn_tc.cu): the cross-check of the tensor-core kernel.
bool attention_on_mma_sync() {
    static const bool v = [] {
        const char* e = getenv("JV_ATTN_KERNEL");
        return e != nullptr && strcmp(e, "mma") == 0;
    }();
    return v;
}

void gemm(jv_ctx* x, const QWeight& w, const __half* xs, int T, int tpad, float* y, int ldy, int epi,
          __half* xs_out = nullptr) {
    static const bool use_ref = getenv("JV_GEMM_REFERENCE") != nullptr;
    if (epi == EPI_SWIGLU && use_ref) {  // the CUDA-core check product has no fused epilogue
        float* gu = x->gu32.get((size_t)T * w.rows);
        gemm(x, w, xs, T, tpad, gu, w.rows, EPI_STORE);
        launch_swiglu(gu, T, w.rows / 2, xs_out, tpad, nullptr, x->d_err, x->stream);
        return;
    }
    GemmArgs a;
    a.xs_out = xs_out;
    a.w = &w;
    a.x = xs;
    a.T = T;
    a.tpad = tpad;
    a.bn = gemm_bn_for(T, w.tiles * ((epi == EPI_SWIGLU) ? 1 : gemm_splits_for(w)), x->m->sm_count);
    a.y = y;
    a.ldy = ldy;
    a.epilogue = epi;
    a.err = x->d_err;
    a.splits = epi == EPI_SWIGLU ? 1 : gemm_splits_for(w);
    if (a.splits > 1) {
        a.ws = x->gemm_ws.get((size_t)a.splits * T * ldy);
        a.counters = x->gemm_ctr.get((size_t)w.tiles * (tpad / a.bn));
    }
    ProfScope ps(x, JV_PROF_GEMM, 2.0 * T * w.rows * w.cols,
                 weight_bytes(w) + 2.0 * T * w.cols + (epi == EPI_ADD ? 8.0 : 4.0) * T * w.rows);
    if (use_ref)
        launch_gemm_reference(a, x->stream);
    else
        launch_gemm(a, x->stream);
}

// h += W xs for the residual projections (O, down). With a two-way K split the halves are not
// combined here: each writes its partial and the returned buffer ([2][T][ldy]) is added into
// h by the next RMSNorm (launch_rmsnorm_resid), which reads h anyway. Returns nullptr when h
// was updated in place (no split, or the CUDA-core check product).
const float* gemm_resid(jv_ctx* x, const QWeight& w, const __half* xs, int T, int tpad, float* h, int ldy) {
    static const bool use_ref = getenv("JV_GEMM_REFERENCE") != nullptr;
    if (use_ref || gemm_splits_for(w) != 2) {
        gemm(x, w, xs, T, tpad, h, ldy, EPI_ADD);
        return nullptr;
    }
    GemmArgs a;
    a.w = &w;
    a.x = xs;
    a.T = T;
    a.tpad = tpad;
    a.bn = gemm_bn_for(T, w.tiles * 2, x->m->sm_count);
    a.y = h;
    a.ldy = ldy;
    a.epilogue = EPI_PARTIAL;
    a.err = x->d_err;
    a.splits = 2;
    a.ws = x->gemm_ws.get((size_t)2 * T * ldy);
    a.counters = x->gemm_ctr.get((size_t)w.tiles * (tpad / a.bn));
    ProfScope ps(x, JV_PROF_GEMM, 2.0 * T * w.rows * w.cols, weight_bytes(w) + 2.0 * T * w.cols + 8.0 * T * w.rows);
    launch_gemm(a, x->stream);
    return a.ws;
}

void gemv(jv_ctx* x, const QWeight& w, const float* v, float* y, int epi) {
    int splits = gemv_splits_for(w, x->m->sm_count);
    float* part = x->partial.get((size_t)splits * w.rows);
    ProfScope ps(x, JV_PROF_GEMV, 2.0 * w.rows * w.cols, weight_bytes(w) + 4.0 * w.cols + 4.0 * w.rows);
    launch_gemv(w, v, part, splits, x->stream);
    launch_gemv_reduce(part, splits, w.rows, y, epi, x->stream);
}

// One single-token step through every layer with the fused decode kernels: five launches per
// layer (see kernels_decode.cu), then optionally the LM head with its argmax. Everything the
// step varies by (token, slot, position, visible keys) is read from *d_step on the device.
// attn_splits bounds the visible keys (64 per split) for every step this sequence serves.
constexpr int DEC_ATTN_CTR = 4096;  // attention counters start here in dec_ctr
// JV_DECODE_PREFETCH=0 turns the decode step's L2 weight prefetch off (for measuring what it gives).
bool dec_prefetch_enabled() {
    static const bool v = [] {
        const char* e = getenv("JV_DECODE_PREFETCH");
        return !(e != nullptr && strcmp(e, "0") == 0);
    }();
    return v;
}

void decode_step(jv_ctx* x, DecodeStep* d_step, int attn_splits, bool head, bool advance, int32_t* tokens_out) {
    jv_model* m = x->m;
    const jv_config& c = m->cfg;
    cudaStream_t s = x->stream;
    const int hidden = c.hidden, qdim = c.heads * c.head_dim, ff = c.ff;
    if (c.head_dim != 128) throw Error(JV_ERR_UNSUPPORTED, "decode: head_dim must be 128");
    const int sms = m->sm_count;
    float* h = x->h.get(hidden);
    float* q32 = x->q32.get(qdim);
    float* ctx = x->ctx32.get(qdim);
    float* act = x->act32.get(ff);
    int* ctr = x->dec_ctr.get(DEC_ATTN_CTR + c.kv_heads);
    size_t need = 0;
    for (const LayerW& W : m->layers)
        for (const QWeight* w : {&W.qkv, &W.o, &W.gu, &W.down})
            need = std::max(need, (size_t)dec_splits_for(*w, sms) * w->rows);
    if (head) need = std::max(need, (size_t)dec_splits_for(m->head, sms) * m->head.rows);
    float* part = x->partial.get(std::max<size_t>(need, 1));
    float* apart = x->dec_attn.get((size_t)c.heads * attn_splits * DEC_ATTN_PSTRIDE);
    if (m->layers.size() && m->head.tiles + 1 > DEC_ATTN_CTR) throw Error(JV_ERR_UNSUPPORTED, "decode: vocabulary too large");

    launch_embed(m->embd, &d_step->token, 1, h, hidden, x->d_err, s);
    // Weight prefetch into L2, one matrix ahead (a Q4_0 layer is 65.5 MB, about half the 126 MB
    // L2): QKV fetches O; the attention the first half of gate/up and O the second; gate/up
    // fetches down; down fetches the next layer's QKV, or the head's first 32 MB after the last
    // layer. The first QKV of a step is read from HBM.
    auto pf_of = [](const QWeight& w, int64_t from, int64_t upto) {
        const int64_t b = (int64_t)w.bytes();
        from = std::min(from, b) & ~(int64_t)15;
        upto = std::min(upto, b) & ~(int64_t)15;
        return std::make_pair((const uint8_t*)w.data + from, std::max<int64_t>(0, upto - from));
    };
    const bool prefetch = dec_prefetch_enabled();
    for (int l = 0; l < c.layers; l++) {
        const LayerW& W = m->layers[l];
        const int64_t gu_half = ((int64_t)W.gu.bytes() / 2) & ~(int64_t)15;
        std::pair<const uint8_t*, int64_t> none{nullptr, 0};
        auto pf_qkv = prefetch ? pf_of(W.o, 0, INT64_MAX) : none;
        auto pf_attn = prefetch ? pf_of(W.gu, 0, gu_half) : none;
        auto pf_o = prefetch ? pf_of(W.gu, gu_half, INT64_MAX) : none;
        auto pf_gu = prefetch ? pf_of(W.down, 0, INT64_MAX) : none;
        auto pf_down = !prefetch ? none
                       : l + 1 < c.layers ? pf_of(m->layers[l + 1].qkv, 0, INT64_MAX)
                       : head ? pf_of(m->head, 0, 32ll << 20) : none;
        DecGemvArgs a;
        a.partial = part;
        a.counters = ctr;
        a.err = x->d_err;
        a.eps = c.eps;
        // 1. attn_norm + QKV + RoPE + K/V write
        a.w = W.qkv.data;
        a.ksteps = W.qkv.ksteps;
        a.rows = W.qkv.rows;
        a.in = h;
        a.n_in = hidden;
        a.norm_w = W.attn_norm;
        a.step = d_step;
        a.rope_table = m->rope_table;
        a.heads = c.heads;
        a.kv_heads = c.kv_heads;
        a.layer = l;
        a.orig_ctx = c.rope_orig_ctx;
        a.temperature_scale = c.temperature_scale;
        a.q32 = q32;
        a.kv_pool = m->pool;
        a.page_table = ctx_table(x);
        a.page_bytes = m->page_bytes;
        a.page_slots = m->page_slots;
        a.pf = pf_qkv.first;
        a.pf_bytes = pf_qkv.second;
        launch_dec_gemv(DEC_QKV, true, W.qkv.type, a, dec_splits_for(W.qkv, sms), s);
        a.pf = nullptr;
        a.pf_bytes = 0;
        // 2. attention
        DecAttnArgs da;
        da.q32 = q32;
        da.kv_pool = m->pool;
        da.page_table = ctx_table(x);
        da.page_bytes = m->page_bytes;
        da.page_slots = m->page_slots;
        da.layer = l;
        da.heads = c.heads;
        da.kv_heads = c.kv_heads;
        da.scale = 1.f / std::sqrt((float)c.head_dim);
        da.step = d_step;
        da.partial = apart;
        da.counters = ctr + DEC_ATTN_CTR;
        da.err = x->d_err;
        da.ctx32 = ctx;
        da.pf = pf_attn.first;
        da.pf_bytes = pf_attn.second;
        launch_dec_attn(da, attn_splits, s);
        // 3. O + residual
        DecGemvArgs o = a;
        o.w = W.o.data;
        o.ksteps = W.o.ksteps;
        o.rows = W.o.rows;
        o.in = ctx;
        o.n_in = qdim;
        o.norm_w = nullptr;
        o.y = h;
        o.pf = pf_o.first;
        o.pf_bytes = pf_o.second;
        launch_dec_gemv(DEC_ADD, false, W.o.type, o, dec_splits_for(W.o, sms), s);
        // 4. ffn_norm + gate/up + SwiGLU
        DecGemvArgs g = a;
        g.w = W.gu.data;
        g.ksteps = W.gu.ksteps;
        g.rows = W.gu.rows;
        g.in = h;
        g.n_in = hidden;
        g.norm_w = W.ffn_norm;
        g.y = act;
        g.pf = pf_gu.first;
        g.pf_bytes = pf_gu.second;
        launch_dec_gemv(DEC_SWIGLU, true, W.gu.type, g, dec_splits_for(W.gu, sms), s);
        // 5. down + residual
        DecGemvArgs d = a;
        d.w = W.down.data;
        d.ksteps = W.down.ksteps;
        d.rows = W.down.rows;
        d.in = act;
        d.n_in = ff;
        d.norm_w = nullptr;
        d.y = h;
        d.pf = pf_down.first;
        d.pf_bytes = pf_down.second;
        launch_dec_gemv(DEC_ADD, false, W.down.type, d, dec_splits_for(W.down, sms), s);
    }
    if (head) {
        DecGemvArgs a;
        a.err = x->d_err;
        a.partial = part;
        a.w = m->head.data;
        a.ksteps = m->head.ksteps;
        a.rows = m->head.rows;
        a.in = h;
        a.n_in = hidden;
        a.norm_w = m->out_norm;
        a.eps = c.eps;
        a.y = x->logits.get(m->head.rows);
        a.counters = ctr;
        a.cand_v = x->dec_cand_v.get(m->head.tiles);
        a.cand_i = x->dec_cand_i.get(m->head.tiles);
        a.argmax_out = x->out_i32.get(1);
        a.advance = advance ? 1 : 0;
        a.tokens_out = tokens_out;
        a.step_rw = d_step;
        launch_dec_gemv(DEC_HEAD, true, m->head.type, a, dec_splits_for(m->head, sms), s);
    }
}

// The private ForwardAsync (reference MinistralModel.cs:301-435).
//   L == nullptr: a causal append at the cache end.
//   rows != nullptr: selected vocab rows per output -> out[n_out][n_rows].
//   rows == nullptr && full_vocab: full vocabulary per output -> out[n_out][vocab].
//   compute_logits: full-vocabulary logits of the last position -> logits[vocab].
void forward(jv_ctx* x, const int32_t* tokens, int T, const HostLayout* L, const int32_t* rows, int n_rows,
             bool full_vocab, float* out, bool compute_logits, float* logits) {
    jv_model* m = x->m;
    const jv_config& c = m->cfg;
    set_device(m);
    if (T <= 0) throw Error(JV_ERR_ARG, "No tokens to forward.");
    for (int i = 0; i < T; i++)
        if ((unsigned)tokens[i] >= (unsigned)m->embd.rows)
            throw Error(JV_ERR_RANGE, "Token id " + std::to_string(tokens[i]) + " is outside the " +
                                          std::to_string(m->embd.rows) + "-entry embedding table.");
    for (int i = 0; i < n_rows && rows; i++)
        if ((unsigned)rows[i] >= (unsigned)m->head.rows)
            throw Error(JV_ERR_RANGE, "vocabulary row " + std::to_string(rows[i]) + " is out of range");

    const int start = x->length;
    HostLayout causal;
    if (!L) {
        causal.slot.resize(T);
        causal.pos.resize(T);
        causal.shared.assign(T, start);
        causal.seg.assign(T, start);
        for (int t = 0; t < T; t++) causal.slot[t] = causal.pos[t] = start + t;
        causal.outputs = {T - 1};
        causal.end = start + T;
        L = &causal;
    }
    const int end = L->end;
    int n_out = (int)L->outputs.size();
    for (int t = 0; t < T; t++) {
        if (L->slot[t] < 0 || L->slot[t] >= end || L->seg[t] < 0 || L->seg[t] > L->slot[t] || L->shared[t] < 0 ||
            L->shared[t] > end || L->pos[t] < 0)
            throw Error(JV_ERR_ARG, "layout entry " + std::to_string(t) + " is inconsistent");
        if (L->pos[t] >= m->rope_positions)
            throw Error(JV_ERR_RANGE, "position " + std::to_string(L->pos[t]) + " is beyond the model's context window");
    }
    for (int o : L->outputs)
        if (o < 0 || o >= T) throw Error(JV_ERR_ARG, "output index out of range");
    // Token t sees slots [base, shared) and then [segment, slot]: sh[t] shared keys from bs[t].
    std::vector<int> bs(T, 0), sh(T);
    for (int t = 0; t < T; t++) {
        if (!L->base.empty()) bs[t] = L->base[t];
        if (bs[t] < 0 || bs[t] > L->shared[t]) throw Error(JV_ERR_ARG, "layout entry " + std::to_string(t) + " is inconsistent");
        sh[t] = L->shared[t] - bs[t];
    }
    if (T == 1 && bs[0] != 0 && sh[0] != 0)
        throw Error(JV_ERR_UNSUPPORTED, "a single-token step must see its shared keys from slot 0");

    // KvCache.EnsureCapacity(end); copy-on-write for the pages this pass writes.
    ctx_ensure_capacity(x, end);
    {
        std::vector<int> wp;
        for (int t = 0; t < T; t++) wp.push_back(L->slot[t] / m->page_slots);
        std::sort(wp.begin(), wp.end());
        wp.erase(std::unique(wp.begin(), wp.end()), wp.end());
        ctx_make_writable(x, wp);
    }
    ctx_upload_pages(x);

    const int hidden = c.hidden, qdim = c.heads * c.head_dim, kvdim = c.kv_heads * c.head_dim, ff = c.ff;
    const int qkvn = qdim + 2 * kvdim;
    const bool decode = T == 1;
    const int tpad = gemm_tpad_for(T);
    const float scale = 1.f / std::sqrt((float)c.head_dim);

    // Attention work items: runs of consecutive tokens that share (shared, segment) and have
    // consecutive slots, cut into ATT_ITEM_TOKENS-token tiles, one item per tile (or pair of
    // tiles) and KV head; longest first. The tensor-core kernel can take two consecutive tiles of
    // a run per item (they share every K/V block); pairing halves the K/V traffic but doubles the
    // item's time, so a pass that fits one wave of single tiles pairs none, one that fits a wave
    // only when paired pairs its shortest tiles until it does, and a longer pass pairs them all.
    const bool attn_tc = !attention_on_mma_sync();
    std::vector<AttnItem> items;
    if (!decode) {
        struct Tile { int t0, n, lim; bool cont; };  // cont: full, and the run goes on in the next tile
        std::vector<Tile> tiles;
        auto same_run = [&](int a, int b) {
            return L->shared[b] == L->shared[a] && bs[b] == bs[a] && L->seg[b] == L->seg[a] && L->slot[b] == L->slot[a] + (b - a);
        };
        for (int t = 0; t < T;) {
            int n = 1;
            while (n < ATT_ITEM_TOKENS && t + n < T && same_run(t, t + n)) n++;
            const bool cont = n == ATT_ITEM_TOKENS && t + n < T && same_run(t, t + n);
            tiles.push_back({t, n, sh[t] + (L->slot[t] + n - 1 - L->seg[t] + 1), cont});
            t += n;
        }
        std::vector<char> paired(tiles.size(), 0);  // tile i takes tile i + 1 as its second tile
        if (attn_tc) {
            std::vector<int> cand;
            for (size_t i = 0; i + 1 < tiles.size(); i++)
                if (tiles[i].cont) cand.push_back((int)i++);
            const int64_t kvh = c.kv_heads, sms = m->sm_count;
            const int64_t n_single = (int64_t)tiles.size() * kvh, n_all = ((int64_t)tiles.size() - (int64_t)cand.size()) * kvh;
            if (n_all > sms) {
                for (int i : cand) paired[i] = 1;
            } else if (n_single > sms) {
                std::stable_sort(cand.begin(), cand.end(), [&](int a, int b) { return tiles[a + 1].lim < tiles[b + 1].lim; });
                int64_t n = n_single;
                for (int i : cand) {
                    if (n <= sms) break;
                    paired[i] = 1;
                    n -= kvh;
                }
            }
        }
        for (size_t i = 0; i < tiles.size(); i++) {
            const Tile& a = tiles[i];
            const bool two = paired[i] != 0;
            const int n = two ? a.n + tiles[i + 1].n : a.n;
            const int lim = two ? tiles[i + 1].lim : a.lim;
            for (int g = 0; g < c.kv_heads; g++) {
                AttnItem it;
                it.t0 = a.t0;
                it.ntok = n;
                it.kv_head = g;
                it.slot0 = L->slot[a.t0];
                it.shared = sh[a.t0];
                it.segment = L->seg[a.t0];
                it.nblocks = (lim + 63) / 64;
                it.base = bs[a.t0];
                items.push_back(it);
            }
            if (two) i++;
        }
        std::stable_sort(items.begin(), items.end(), [](const AttnItem& a, const AttnItem& b) { return a.nblocks > b.nblocks; });
    }
    int max_item_keys = 0;
    for (const AttnItem& it : items) max_item_keys = std::max(max_item_keys, it.nblocks * 64);
    // Algorithmic attention work: QK^T and PV over exactly the visible (query, key) pairs.
    double attn_flops = 0, attn_bytes = 2.0 * 2 * T * qdim;
    for (int t = 0; t < T; t++) attn_flops += 4.0 * c.heads * c.head_dim * (sh[t] + (L->slot[t] - L->seg[t] + 1));
    for (const AttnItem& it : items)
        attn_bytes += (double)(it.shared + (it.slot0 + it.ntok - 1 - it.segment + 1)) * c.head_dim * 2 * 2;

    // One H2D for every per-call input: tokens, slot, pos, outputs, rows, items.
    size_t n_items_words = items.size() * (sizeof(AttnItem) / 4);
    size_t items_off = 3 * (size_t)T + n_out + (size_t)std::max(0, n_rows);
    items_off = (items_off + 7) & ~(size_t)7;  // 32-byte alignment for the item structs
    size_t total_words = items_off + n_items_words;
    // A single token without an activation sink runs the fused decode kernels, which read
    // the step from device memory (appended to the same upload).
    const bool fused = decode && x->sink == nullptr && !m->has_qx;
    const size_t step_off = (total_words + 7) & ~(size_t)7;
    if (fused) total_words = step_off + sizeof(DecodeStep) / 4;
    int32_t* hin = x->h_in.get(total_words);
    int32_t* din = x->in_i32.get(total_words);
    std::memcpy(hin, tokens, sizeof(int32_t) * T);
    std::memcpy(hin + T, L->slot.data(), sizeof(int32_t) * T);
    std::memcpy(hin + 2 * T, L->pos.data(), sizeof(int32_t) * T);
    std::memcpy(hin + 3 * T, L->outputs.data(), sizeof(int32_t) * n_out);
    if (n_rows > 0 && rows) std::memcpy(hin + 3 * T + n_out, rows, sizeof(int32_t) * n_rows);
    if (!items.empty()) std::memcpy(hin + items_off, items.data(), items.size() * sizeof(AttnItem));
    int dec_keys = 0;
    if (fused) {
        DecodeStep st{};
        st.token = tokens[0];
        st.slot = L->slot[0];
        st.pos = L->pos[0];
        st.shared = sh[0];
        st.segment = L->seg[0];
        st.n_keys = dec_keys = sh[0] + (L->slot[0] - L->seg[0] + 1);
        std::memcpy(hin + step_off, &st, sizeof st);
    }
    JV_CUDA(cudaMemcpyAsync(din, hin, sizeof(int32_t) * total_words, cudaMemcpyHostToDevice, x->stream));
    const int32_t* d_tokens = din;
    const int32_t* d_slot = din + T;
    const int32_t* d_pos = din + 2 * T;
    const int32_t* d_outs = din + 3 * T;
    const int32_t* d_rows = din + 3 * T + n_out;
    const AttnItem* d_items = (const AttnItem*)(din + items_off);

    cudaStream_t s = x->stream;
    float* h = x->h.get((size_t)T * hidden);
    if (fused) {
        check_cancel(x);
        decode_step(x, (DecodeStep*)(din + step_off), (dec_keys + DEC_ATTN_KEYS - 1) / DEC_ATTN_KEYS, compute_logits,
                    false, nullptr);
    } else {
        launch_embed(m->embd, d_tokens, T, h, hidden, x->d_err, s);
        observe(x, "embeddings", h, T, hidden);
    }

    float* qkv32 = x->qkv32.get((size_t)T * qkvn);
    const bool capture = x->sink != nullptr;
    // split-K partials of the last O / down projection not yet added into h (see gemm_resid)
    const float* resid = nullptr;

    for (int l = 0; l < (fused ? 0 : c.layers); l++) {
        check_cancel(x);
        const LayerW& W = m->layers[l];
        std::string p = "blk." + std::to_string(l) + ".";
        RopeArgs ra;
        ra.qkv = qkv32;
        ra.pos = d_pos;
        ra.slot = d_slot;
        ra.table = m->rope_table;
        ra.T = T;
        ra.heads = c.heads;
        ra.kv_heads = c.kv_heads;
        ra.head_dim = c.head_dim;
        ra.layer = l;
        ra.temperature_scale = c.temperature_scale;
        ra.orig_ctx = c.rope_orig_ctx;
        ra.kv_pool = m->pool;
        ra.page_table = ctx_table(x);
        ra.page_bytes = m->page_bytes;
        ra.page_slots = m->page_slots;
        ra.k32 = capture ? x->k32.get((size_t)T * kvdim) : nullptr;
        ra.err = x->d_err;
        if (decode) {
            float* xn = x->x32.get(hidden);
            launch_rmsnorm(h, W.attn_norm, 1, hidden, c.eps, nullptr, 0, xn, x->d_err, s);
            observe(x, p + "attn_norm", xn, 1, hidden);
            gemv(x, W.qkv, xn, qkv32, EPI_STORE);
            ra.q16 = nullptr;
            ra.q32 = x->q32.get(qdim);
            launch_rope_kv(ra, s);
            observe(x, p + "q_rope", ra.q32, 1, qdim);
            if (capture) observe(x, p + "k_rope", ra.k32, 1, kvdim);
            observe(x, p + "v", qkv32 + qdim + kvdim, 1, kvdim, qkvn);
            DecodeAttnArgs da;
            da.q32 = ra.q32;
            da.kv_pool = m->pool;
            da.page_table = ctx_table(x);
            da.page_bytes = m->page_bytes;
            da.page_slots = m->page_slots;
            da.layer = l;
            da.heads = c.heads;
            da.kv_heads = c.kv_heads;
            da.shared = sh[0];
            da.segment = L->seg[0];
            da.n_keys = sh[0] + (L->slot[0] - L->seg[0] + 1);
            da.scale = scale;
            da.splits = (da.n_keys + 63) / 64;
            da.partial = x->tmp32.get((size_t)c.heads * da.splits * (2 + c.head_dim));
            da.ctx32 = x->ctx32.get(qdim);
            da.err = x->d_err;
            {
                ProfScope ps(x, JV_PROF_ATTENTION, 4.0 * c.heads * c.head_dim * da.n_keys,
                             (double)da.n_keys * c.kv_heads * c.head_dim * 2 * 2 + 8.0 * qdim);
                launch_decode_attention(da, s);
            }
            observe(x, p + "attn_weighted", da.ctx32, 1, qdim);
            if (capture) {
                float* ao = x->out32.get(hidden);
                gemv(x, W.o, da.ctx32, ao, EPI_STORE);
                observe(x, p + "attn_out", ao, 1, hidden);
                launch_add(h, ao, hidden, s);
            } else {
                gemv(x, W.o, da.ctx32, h, EPI_ADD);
            }
            observe(x, p + "post_attn", h, 1, hidden);
            launch_rmsnorm(h, W.ffn_norm, 1, hidden, c.eps, nullptr, 0, xn, x->d_err, s);
            observe(x, p + "ffn_norm", xn, 1, hidden);
            float* gu = x->gu32.get(2 * (size_t)ff);
            gemv(x, W.gu, xn, gu, EPI_STORE);
            float* act = x->act32.get(ff);
            launch_swiglu(gu, 1, ff, nullptr, 0, act, x->d_err, s);
            if (capture) {
                float* fo = x->out32.get(hidden);
                gemv(x, W.down, act, fo, EPI_STORE);
                observe(x, p + "ffn_out", fo, 1, hidden);
                launch_add(h, fo, hidden, s);
            } else {
                gemv(x, W.down, act, h, EPI_ADD);
            }
            observe(x, p + "output", h, 1, hidden);
            continue;
        }
        __half* xs = x->xs.get((size_t)tpad * hidden);
        if (capture)
            launch_rmsnorm(h, W.attn_norm, T, hidden, c.eps, xs, tpad, nullptr, x->d_err, s);
        else
            launch_rmsnorm_resid(h, resid, W.attn_norm, T, hidden, c.eps, xs, tpad, x->d_err, s);
        observe_kslab(x, p + "attn_norm", xs, T, hidden, tpad);
        ra.q16 = x->q16.get((size_t)T * qdim);
        ra.q32 = capture ? x->q32.get((size_t)T * qdim) : nullptr;
        gemm(x, W.qkv, xs, T, tpad, qkv32, qkvn, EPI_STORE);
        launch_rope_kv(ra, s);
        if (capture) {
            observe(x, p + "q_rope", ra.q32, T, qdim);
            observe(x, p + "k_rope", ra.k32, T, kvdim);
            observe(x, p + "v", qkv32 + qdim + kvdim, T, kvdim, qkvn);
        }
        AttnArgs aa;
        aa.q16 = ra.q16;
        aa.items = d_items;
        aa.n_items = (int)items.size();
        aa.kv_pool = m->pool;
        aa.page_table = ctx_table(x);
        aa.page_bytes = m->page_bytes;
        aa.page_slots = m->page_slots;
        aa.layer = l;
        aa.heads = c.heads;
        aa.kv_heads = c.kv_heads;
        aa.scale = scale;
        aa.ctx16 = x->ctx16.get((size_t)tpad * qdim);
        aa.tpad = tpad;
        aa.ctx32 = capture ? x->ctx32.get((size_t)T * qdim) : nullptr;
        aa.max_keys = max_item_keys;
        aa.err = x->d_err;
        {
            ProfScope ps(x, JV_PROF_ATTENTION, attn_flops, attn_bytes);
            if (attn_tc)
                launch_attention_tc(aa, s);
            else
                launch_attention(aa, s);
        }
        if (capture) observe(x, p + "attn_weighted", aa.ctx32, T, qdim);
        if (capture) {
            float* ao = x->out32.get((size_t)T * hidden);
            gemm(x, W.o, aa.ctx16, T, tpad, ao, hidden, EPI_STORE);
            observe(x, p + "attn_out", ao, T, hidden);
            launch_add(h, ao, (int64_t)T * hidden, s);
        } else {
            resid = gemm_resid(x, W.o, aa.ctx16, T, tpad, h, hidden);
        }
        observe(x, p + "post_attn", h, T, hidden);
        if (capture)
            launch_rmsnorm(h, W.ffn_norm, T, hidden, c.eps, xs, tpad, nullptr, x->d_err, s);
        else
            launch_rmsnorm_resid(h, resid, W.ffn_norm, T, hidden, c.eps, xs, tpad, x->d_err, s);
        resid = nullptr;
        observe_kslab(x, p + "ffn_norm", xs, T, hidden, tpad);
        __half* xf = x->xs_ff.get((size_t)tpad * ff);
        gemm(x, W.gu, xs, T, tpad, nullptr, 2 * ff, EPI_SWIGLU, xf);
        if (capture) {
            float* fo = x->out32.get((size_t)T * hidden);
            gemm(x, W.down, xf, T, tpad, fo, hidden, EPI_STORE);
            observe(x, p + "ffn_out", fo, T, hidden);
            launch_add(h, fo, (int64_t)T * hidden, s);
        } else {
            resid = gemm_resid(x, W.down, xf, T, tpad, h, hidden);
        }
        observe(x, p + "output", h, T, hidden);
    }
    if (resid) launch_resid_add(h, resid, (int64_t)T * hidden, s);  // the last layer's pending half sums
    check_cancel(x);
    // KvCache.Advance(max(0, end - Length)).
    x->length += std::max(0, end - x->length);

    // Heads (MinistralModel.cs:362-424).
    if (rows && out) {
        float* normed = x->x32.get((size_t)n_out * hidden);
        launch_rmsnorm_rows(h, d_outs, n_out, m->out_norm, hidden, c.eps, normed, nullptr, 0, x->d_err, s);
        float* d_res = x->out32.get((size_t)n_out * n_rows);
        launch_head_rows(m->head, normed, n_out, d_rows, n_rows, d_res, x->d_err, s);
        float* hres = x->h_out.get((size_t)n_out * n_rows);
        JV_CUDA(cudaMemcpyAsync(hres, d_res, sizeof(float) * n_out * n_rows, cudaMemcpyDeviceToHost, s));
        sync_check(x);
        std::memcpy(out, hres, sizeof(float) * n_out * n_rows);
    } else if (full_vocab && out) {
        int V = m->head.rows;
        float* d_res = x->logits.get((size_t)n_out * V);
        if (n_out >= 2) {
            int tp = gemm_tpad_for(n_out);
            __half* xo = x->xs.get((size_t)std::max(tp, tpad) * hidden);
            launch_rmsnorm_rows(h, d_outs, n_out, m->out_norm, hidden, c.eps, nullptr, xo, tp, x->d_err, s);
            gemm(x, m->head, xo, n_out, tp, d_res, V, EPI_STORE);
        } else {
            float* normed = x->x32.get(hidden);
            launch_rmsnorm_rows(h, d_outs, 1, m->out_norm, hidden, c.eps, normed, nullptr, 0, x->d_err, s);
            gemv(x, m->head, normed, d_res, EPI_STORE);
        }
        float* hres = x->h_out.get((size_t)n_out * V);
        JV_CUDA(cudaMemcpyAsync(hres, d_res, sizeof(float) * n_out * V, cudaMemcpyDeviceToHost, s));
        sync_check(x);
        std::memcpy(out, hres, sizeof(float) * n_out * V);
    }
    if (compute_logits) {
        int V = m->head.rows;
        float* normed = x->x32.get(hidden);
        float* d_logits = x->logits.get(V);
        int32_t last = T - 1;
        // the last row index lives in the output list for causal passes; for explicit
        // layouts use a one-word upload
        if (!fused) {  // the fused decode step already wrote the logits
            int32_t* d_last = x->out_i32.get(1);
            JV_CUDA(cudaMemcpyAsync(d_last, &last, sizeof(int32_t), cudaMemcpyHostToDevice, s));
            launch_rmsnorm_rows(h, d_last, 1, m->out_norm, hidden, c.eps, normed, nullptr, 0, x->d_err, s);
            observe(x, "final_norm", normed, 1, hidden);
            gemv(x, m->head, normed, d_logits, EPI_STORE);
        }
        observe(x, "logits", d_logits, 1, V);
        if (logits) {
            float* hres = x->h_out.get(V);
            JV_CUDA(cudaMemcpyAsync(hres, d_logits, sizeof(float) * V, cudaMemcpyDeviceToHost, s));
            sync_check(x);
            std::memcpy(logits, hres, sizeof(float) * V);
        }
    }
    sync_check(x);
    x->resolve_profile();
}

HostLayout layout_from(const jv_layout* l, int T) {
    HostLayout L;
    if (!l->slot || !l->position || !l->shared || !l->segment) throw Error(JV_ERR_ARG, "layout arrays must not be NULL");
    L.slot.assign(l->slot, l->slot + T);
    L.pos.assign(l->position, l->position + T);
    L.shared.assign(l->shared, l->shared + T);
    L.seg.assign(l->segment, l->segment + T);
    if (l->n_outputs > 0) {
        if (!l->outputs) throw Error(JV_ERR_ARG, "layout outputs must not be NULL");
        L.outputs.assign(l->outputs, l->outputs + l->n_outputs);
    } else {
        L.outputs = {T - 1};
    }
    L.end = l->end;
    return L;
}

// TokenLayout.Tree (reference MinistralModel.cs:720-745).
HostLayout layout_tree(int start, int trunk, const std::vector<int>& offsets, int tokens) {
    HostLayout L;
    L.slot.resize(tokens);
    L.pos.resize(tokens);
    L.shared.resize(tokens);
    L.seg.resize(tokens);
    int branch = -1;
    for (int t = 0; t < tokens; t++) {
        L.slot[t] = start + t;
        while (branch + 1 < (int)offsets.size() && t >= offsets[branch + 1]) branch++;
        if (t < trunk || branch < 0) {
            L.pos[t] = start + t;
            L.shared[t] = start;
            L.seg[t] = start;
        } else {
            L.pos[t] = start + trunk + (t - offsets[branch]);
            L.shared[t] = start + trunk;
            L.seg[t] = start + offsets[branch];
        }
    }
    L.outputs.resize(offsets.size());
    for (size_t b = 0; b < offsets.size(); b++) L.outputs[b] = (b + 1 < offsets.size() ? offsets[b + 1] : tokens) - 1;
    L.end = start + tokens;
    return L;
}

}  // namespace

namespace jv {
int api_error(int code, const std::string& msg) { return set_error(code, msg); }

QWeight qweight_view(int type, const void* tiled, int rows, int cols) {
    if (type != T_Q8_0 && type != T_Q4_0 && type != T_Q5_1)
        throw Error(JV_ERR_UNSUPPORTED, "weight type " + std::to_string(type) + " is not on the B200 path (Q8_0, Q5_1, Q4_0 are)");
    if (rows <= 0 || cols <= 0 || rows % TILE_ROWS != 0 || cols % TILE_K != 0)
        throw Error(JV_ERR_ARG, "a re-tiled matrix needs rows % 128 == 0 and cols % 64 == 0; got " + std::to_string(rows) +
                                    "x" + std::to_string(cols));
    QWeight w;
    w.type = type;
    w.rows = rows;
    w.cols = cols;
    w.tiles = rows / TILE_ROWS;
    w.ksteps = cols / TILE_K;
    w.data = (uint8_t*)tiled;
    return w;
}
}  // namespace jv

// =========================================================================== C ABI

extern "C" {

int32_t jv_build_features(void) {
#ifdef JV_BOUNDS_CHECK
    return JV_FEATURE_BOUNDS_CHECK;
#else
    return 0;
#endif
}
const char* jv_last_error(void) { return g_last_error.c_str(); }

int jv_device_count(int32_t* count) {
    return guarded([&] {
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        *count = n;
    });
}

int64_t jv_kernel_launches(void) { return launches_total(); }

int jv_model_open(const char* gguf_path, int32_t device, int32_t kv_pool_mb, jv_model** out) {
    if (!out) return set_error(JV_ERR_ARG, "out must not be NULL");
    *out = nullptr;
    if (!gguf_path) return set_error(JV_ERR_ARG, "gguf_path must not be NULL");
    jv_model* m = new jv_model();
    int rc = guarded([&] {
        int n = 0;
        JV_CUDA(cudaGetDeviceCount(&n));
        if (device < 0 || device >= n) throw Error(JV_ERR_ARG, "device " + std::to_string(device) + " does not exist");
        m->device = device;
        JV_CUDA(cudaSetDevice(device));
        cudaDeviceProp prop;
        JV_CUDA(cudaGetDeviceProperties(&prop, device));
        if (prop.major != 10)
            throw Error(JV_ERR_UNSUPPORTED, std::string("this library is built for sm_100a (B200); device is ") + prop.name);
        m->sm_count = prop.multiProcessorCount;
        load_model(m, gguf_path, kv_pool_mb);
    });
    if (rc != JV_OK) {
        cudaSetDevice(m->device);
        for (void* p : m->allocations) cudaFree(p);
        delete m;
        return rc;
    }
    *out = m;
    return JV_OK;
}

void jv_model_close(jv_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    cudaDeviceSynchronize();
    for (void* p : m->allocations) cudaFree(p);
    delete m;
}

int jv_model_config(const jv_model* m, jv_config* out) {
    if (!m || !out) return set_error(JV_ERR_ARG, "NULL argument");
    *out = m->cfg;
    return JV_OK;
}

int jv_ctx_create(jv_model* m, int32_t initial_capacity, jv_ctx** out) {
    if (!m || !out) return set_error(JV_ERR_ARG, "NULL argument");
    *out = nullptr;
    jv_ctx* x = new jv_ctx();
    x->m = m;
    int rc = guarded([&] {
        set_device(m);
        JV_CUDA(cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking));
        x->d_err = dalloc<int>(2);  // error code, then the site of a timeout
        JV_CUDA(cudaMemsetAsync(x->d_err, 0, 2 * sizeof(int), x->stream));
        JV_CUDA(cudaStreamSynchronize(x->stream));
        x->capacity = std::max(1, initial_capacity > 0 ? initial_capacity : 512);
        ctx_ensure_capacity(x, 1);
    });
    if (rc != JV_OK) {
        if (x->stream) cudaStreamDestroy(x->stream);
        delete x;
        return rc;
    }
    *out = x;
    return JV_OK;
}

void jv_ctx_destroy(jv_ctx* x) {
    if (!x) return;
    cudaSetDevice(x->m->device);
    cudaStreamSynchronize(x->stream);
    ctx_release_pages(x);
    for (auto* v : {&x->h, &x->qkv32, &x->gu32, &x->tmp32, &x->q32, &x->ctx32, &x->x32, &x->act32, &x->k32, &x->partial,
                    &x->out32, &x->logits, &x->cap32})
        v->release();
    if (x->dec_graph) cudaGraphExecDestroy(x->dec_graph);
    for (auto* v : {&x->dec_ctr, &x->dec_cand_i, &x->dec_tokens}) v->release();
    x->dec_cand_v.release();
    x->dec_attn.release();
    x->dec_step.release();
    x->xs.release();
    x->gemm_ws.release();
    x->gemm_ctr.release();
    x->xs_ff.release();
    x->ctx16.release();
    x->q16.release();
    x->in_i32.release();
    x->out_i32.release();
    x->items.release();
    x->d_pages.release();
    x->h_in.release();
    x->h_out.release();
    x->h_cap.release();
    x->h_err.release();
    if (x->d_err) cudaFree(x->d_err);
    for (auto& p : x->pending) {
        cudaEventDestroy(p.a);
        cudaEventDestroy(p.b);
    }
    for (auto e : x->spare_events) cudaEventDestroy(e);
    cudaStreamDestroy(x->stream);
    delete x;
}

int jv_ctx_set_sink(jv_ctx* x, jv_activation_sink sink, void* user) {
    if (!x) return set_error(JV_ERR_ARG, "NULL context");
    x->sink = sink;
    x->sink_user = user;
    return JV_OK;
}

int jv_ctx_set_cancel(jv_ctx* x, const volatile int32_t* flag) {
    if (!x) return set_error(JV_ERR_ARG, "NULL context");
    x->cancel = flag;
    return JV_OK;
}

void* jv_ctx_stream(jv_ctx* x) { return x ? (void*)x->stream : nullptr; }

int jv_ctx_profile(jv_ctx* x, int32_t enable) {
    if (!x) return set_error(JV_ERR_ARG, "NULL context");
    x->prof = enable != 0;
    return JV_OK;
}

int jv_ctx_profile_read(jv_ctx* x, int32_t kind, double* total_ms, int64_t* launches, double* flops, double* bytes) {
    if (!x || kind < 0 || kind > 3) return set_error(JV_ERR_ARG, "bad profile query");
    if (total_ms) *total_ms = x->prof_ms[kind];
    if (launches) *launches = x->prof_launches[kind];
    if (flops) *flops = x->prof_flops[kind];
    if (bytes) *bytes = x->prof_bytes[kind];
    return JV_OK;
}

int jv_ctx_profile_reset(jv_ctx* x) {
    if (!x) return set_error(JV_ERR_ARG, "NULL context");
    for (int k = 0; k < 4; k++) {
        x->prof_ms[k] = x->prof_flops[k] = x->prof_bytes[k] = 0;
        x->prof_launches[k] = 0;
    }
    return JV_OK;
}

int jv_ctx_check_wait_timeout(jv_ctx* x, int64_t bound_cycles) {
    if (!x) return set_error(JV_ERR_ARG, "NULL context");
    if (bound_cycles <= 0 || bound_cycles > 4000000000ll)
        return set_error(JV_ERR_RANGE, "bound_cycles must be in (0, 4e9]");
    return guarded([&] {
        set_device(x->m);
        launch_wait_check(x->d_err, (long long)bound_cycles, x->stream);
        sync_check(x);
    });
}

int jv_forward(jv_ctx* x, const int32_t* tokens, int32_t n, float* logits) {
    if (!x || (!tokens && n > 0)) return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] { forward(x, tokens, n, nullptr, nullptr, 0, false, nullptr, logits != nullptr, logits); });
}

int jv_forward_selected(jv_ctx* x, const int32_t* tokens, int32_t n, const int32_t* rows, int32_t n_rows, float* out) {
    if (!x || !rows || !out || (!tokens && n > 0)) return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] { forward(x, tokens, n, nullptr, rows, n_rows, false, out, false, nullptr); });
}

int jv_forward_tree(jv_ctx* x, const int32_t* trunk, int32_t n_trunk, const int32_t* branch_tokens,
                    const int32_t* branch_lengths, int32_t n_branches, const int32_t* rows, int32_t n_rows, float* out) {
    if (!x || !out || !branch_lengths || n_trunk < 0) return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] {
        if (n_branches <= 0) throw Error(JV_ERR_ARG, "No branches to forward.");
        std::vector<int> offsets(n_branches);
        int total = n_trunk;
        for (int b = 0; b < n_branches; b++) {
            if (branch_lengths[b] <= 0) throw Error(JV_ERR_ARG, "Branch " + std::to_string(b) + " is empty.");
            offsets[b] = total;
            total += branch_lengths[b];
        }
        std::vector<int32_t> tokens(total);
        if (n_trunk > 0) std::memcpy(tokens.data(), trunk, sizeof(int32_t) * n_trunk);
        std::memcpy(tokens.data() + n_trunk, branch_tokens, sizeof(int32_t) * (total - n_trunk));
        HostLayout L = layout_tree(x->length, n_trunk, offsets, total);
        forward(x, tokens.data(), total, &L, rows, n_rows, rows == nullptr, out, false, nullptr);
    });
}

int jv_decide_batch(jv_ctx* x, int32_t n_decisions, const int32_t* tokens, const int32_t* trunk_lengths,
                    const int32_t* branch_counts, const int32_t* branch_lengths, const int32_t* rows, int32_t n_rows,
                    float* out) {
    if (!x || !tokens || !trunk_lengths || !branch_counts || !branch_lengths || !rows || !out)
        return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] {
        if (n_decisions <= 0) throw Error(JV_ERR_ARG, "No decisions to forward.");
        // Decision d occupies slots [base_d, base_d + its tokens) after the cache's current end;
        // its trunk is causal from base_d with positions from 0, each branch sees the trunk and
        // itself (TokenLayout.Tree per decision, with the shared region starting at base_d).
        const int start = x->length;
        HostLayout L;
        int cursor = start, t = 0, br = 0;
        for (int d = 0; d < n_decisions; d++) {
            const int trunk = trunk_lengths[d], nb = branch_counts[d];
            if (trunk < 0) throw Error(JV_ERR_ARG, "Decision " + std::to_string(d) + " has a negative trunk length.");
            if (nb <= 0) throw Error(JV_ERR_ARG, "Decision " + std::to_string(d) + " has no branches.");
            const int base = cursor;
            for (int i = 0; i < trunk; i++, t++) {
                L.slot.push_back(cursor++);
                L.pos.push_back(i);
                L.base.push_back(base);
                L.shared.push_back(base);
                L.seg.push_back(base);
            }
            for (int b = 0; b < nb; b++, br++) {
                const int n = branch_lengths[br];
                if (n <= 0) throw Error(JV_ERR_ARG, "Branch " + std::to_string(b) + " of decision " + std::to_string(d) + " is empty.");
                const int seg = cursor;
                for (int i = 0; i < n; i++, t++) {
                    L.slot.push_back(cursor++);
                    L.pos.push_back(trunk + i);
                    L.base.push_back(base);
                    L.shared.push_back(base + trunk);
                    L.seg.push_back(seg);
                }
                L.outputs.push_back(t - 1);
            }
        }
        L.end = cursor;
        forward(x, tokens, t, &L, rows, n_rows, false, out, false, nullptr);
        x->length = start;  // the batch's slots are scratch: the cache is left as it was
    });
}

int jv_forward_layout(jv_ctx* x, const int32_t* tokens, int32_t n, const jv_layout* layout, const int32_t* rows,
                      int32_t n_rows, int32_t full_vocab, float* out, int32_t compute_logits, float* logits) {
    if (!x || (!tokens && n > 0)) return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] {
        if (n <= 0) throw Error(JV_ERR_ARG, "No tokens to forward.");
        if (layout) {
            HostLayout L = layout_from(layout, n);
            forward(x, tokens, n, &L, rows, n_rows, full_vocab != 0, out, compute_logits != 0, logits);
        } else {
            forward(x, tokens, n, nullptr, rows, n_rows, full_vocab != 0, out, compute_logits != 0, logits);
        }
    });
}

int jv_decode_greedy(jv_ctx* x, int32_t first_token, int32_t steps, int32_t* out_tokens) {
    if (!x || !out_tokens) return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] {
        if (steps <= 0) return;
        jv_model* m = x->m;
        set_device(m);
        if (x->sink || m->has_qx) {  // activation capture, or affine-layout weights (no fused decode
                                     // kernels): the step-by-step path
            int32_t tok = first_token;
            for (int i = 0; i < steps; i++) {
                forward(x, &tok, 1, nullptr, nullptr, 0, false, nullptr, true, nullptr);
                int32_t* d_next = x->out_i32.get(1);
                launch_argmax(x->logits.p, m->head.rows, d_next, x->stream);
                JV_CUDA(cudaMemcpyAsync(&out_tokens[i], d_next, sizeof(int32_t), cudaMemcpyDeviceToHost, x->stream));
                JV_CUDA(cudaStreamSynchronize(x->stream));
                tok = out_tokens[i];
            }
            return;
        }
        // Device-resident loop: the head kernel writes each argmax into the step record, which
        // the next step's embedding reads; the host only launches.
        if ((unsigned)first_token >= (unsigned)m->embd.rows)
            throw Error(JV_ERR_RANGE, "Token id " + std::to_string(first_token) + " is outside the " +
                                          std::to_string(m->embd.rows) + "-entry embedding table.");
        const int start = x->length, end = start + steps;
        if (end > m->rope_positions) throw Error(JV_ERR_RANGE, "position " + std::to_string(end - 1) + " is beyond the model's context window");
        ctx_ensure_capacity(x, end);
        std::vector<int> wp;
        for (int p = start / m->page_slots; p <= (end - 1) / m->page_slots; p++) wp.push_back(p);
        ctx_make_writable(x, wp);
        ctx_upload_pages(x);
        cudaStream_t s = x->stream;
        DecodeStep* d_step = x->dec_step.get(1);
        int32_t* d_toks = x->dec_tokens.get((size_t)steps);
        DecodeStep st{};
        st.token = first_token;
        st.slot = st.pos = st.shared = st.segment = start;
        st.n_keys = start + 1;
        int32_t* hst = x->h_in.get(sizeof(DecodeStep) / 4);
        std::memcpy(hst, &st, sizeof st);
        JV_CUDA(cudaMemcpyAsync(d_step, hst, sizeof st, cudaMemcpyHostToDevice, s));
        const int splits = (end + DEC_ATTN_KEYS - 1) / DEC_ATTN_KEYS;
        const int64_t l0 = launches_total();
        decode_step(x, d_step, splits, true, true, d_toks);
        const int64_t per_step = launches_total() - l0;
        if (steps > 1) {
            std::vector<const void*> sig = {x->h.p, x->q32.p, x->ctx32.p, x->act32.p, x->partial.p, x->dec_attn.p,
                                            x->dec_ctr.p, x->logits.p, x->dec_cand_v.p, x->dec_cand_i.p, x->out_i32.p,
                                            x->d_pages.p, d_step, d_toks, (const void*)(intptr_t)splits};
            if (!x->dec_graph || sig != x->dec_graph_sig) {
                if (x->dec_graph) cudaGraphExecDestroy(x->dec_graph);
                x->dec_graph = nullptr;
                cudaGraph_t g = nullptr;
                JV_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
                try {
                    decode_step(x, d_step, splits, true, true, d_toks);
                } catch (...) {
                    cudaStreamEndCapture(s, &g);
                    if (g) cudaGraphDestroy(g);
                    throw;
                }
                JV_CUDA(cudaStreamEndCapture(s, &g));
                note_launch(-(int)per_step);  // captured, not run
                cudaError_t e = cudaGraphInstantiate(&x->dec_graph, g, 0);
                cudaGraphDestroy(g);
                if (e != cudaSuccess) {
                    x->dec_graph = nullptr;
                    JV_CUDA(e);
                }
                x->dec_graph_sig = sig;
            }
            for (int i = 1; i < steps; i++) {
                if (x->cancel && *x->cancel) {
                    sync_check(x);
                    x->length = start + i;
                    throw Error(JV_ERR_CANCELLED, "The operation was canceled.");
                }
                JV_CUDA(cudaGraphLaunch(x->dec_graph, s));
                note_launch((int)per_step);
            }
        }
        float* hres = x->h_out.get((size_t)steps);
        JV_CUDA(cudaMemcpyAsync(hres, d_toks, sizeof(int32_t) * steps, cudaMemcpyDeviceToHost, s));
        sync_check(x);
        std::memcpy(out_tokens, hres, sizeof(int32_t) * steps);
        x->length = end;
    });
}

int32_t jv_kv_length(jv_ctx* x) { return x ? x->length : 0; }
int32_t jv_kv_capacity(jv_ctx* x) { return x ? x->capacity : 0; }
int jv_kv_reset(jv_ctx* x) {
    if (!x) return set_error(JV_ERR_ARG, "NULL context");
    x->length = 0;
    return JV_OK;
}
int jv_kv_truncate(jv_ctx* x, int32_t length) {
    if (!x) return set_error(JV_ERR_ARG, "NULL context");
    x->length = std::min(std::max(length, 0), x->length);
    return JV_OK;
}
int jv_kv_ensure_capacity(jv_ctx* x, int32_t required) {
    if (!x) return set_error(JV_ERR_ARG, "NULL context");
    return guarded([&] { set_device(x->m); ctx_ensure_capacity(x, required); });
}
int64_t jv_kv_bytes_per_position(jv_ctx* x) {
    if (!x) return 0;
    const jv_config& c = x->m->cfg;
    return (int64_t)c.layers * c.kv_heads * c.head_dim * (int64_t)sizeof(float) * 2;
}
int64_t jv_kv_snapshot_floats(jv_ctx* x, int32_t length) {
    if (!x) return 0;
    const jv_config& c = x->m->cfg;
    return (int64_t)c.layers * c.kv_heads * length * c.head_dim * 2;
}
int jv_kv_snapshot(jv_ctx* x, int32_t length, float* out, int64_t n_floats) {
    if (!x || !out) return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] {
        if (length > x->length || length < 0)
            throw Error(JV_ERR_RANGE, "Only " + std::to_string(x->length) + " positions are cached.");
        int64_t need = jv_kv_snapshot_floats(x, length);
        if (n_floats != need) throw Error(JV_ERR_ARG, "snapshot buffer holds " + std::to_string(n_floats) + " floats; needs " + std::to_string(need));
        set_device(x->m);
        ctx_upload_pages(x);
        float* d = x->cap32.get((size_t)need);
        const jv_config& c = x->m->cfg;
        launch_kv_export(x->m->pool, ctx_table(x), x->m->page_bytes, x->m->page_slots, c.layers, c.kv_heads, length, d, x->stream, 0, 0,
                         x->d_err);
        JV_CUDA(cudaMemcpyAsync(out, d, sizeof(float) * need, cudaMemcpyDeviceToHost, x->stream));
        JV_CUDA(cudaStreamSynchronize(x->stream));
    });
}
int jv_kv_restore(jv_ctx* x, const float* snap, int64_t n_floats, int32_t length) {
    if (!x || !snap) return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] {
        int64_t need = jv_kv_snapshot_floats(x, length);
        if (n_floats != need)
            throw Error(JV_ERR_ARG, "Snapshot holds " + std::to_string(n_floats) + " floats; " + std::to_string(length) +
                                        " positions need " + std::to_string(need) + ".");
        set_device(x->m);
        ctx_ensure_capacity(x, std::max(1, length));
        std::vector<int> wp;
        for (int p = 0; p * x->m->page_slots < length; p++) wp.push_back(p);
        ctx_make_writable(x, wp);
        ctx_upload_pages(x);
        float* d = x->cap32.get((size_t)std::max<int64_t>(1, need));
        JV_CUDA(cudaMemcpyAsync(d, snap, sizeof(float) * need, cudaMemcpyHostToDevice, x->stream));
        const jv_config& c = x->m->cfg;
        launch_kv_import(x->m->pool, ctx_table(x), x->m->page_bytes, x->m->page_slots, c.layers, c.kv_heads, length, d, x->d_err, x->stream);
        JV_CUDA(cudaStreamSynchronize(x->stream));
        x->length = length;
    });
}

// ---- SHKV persistence straight from / into the device pages (SystemPromptCache.Save / TryLoad)

namespace {

constexpr uint32_t SHKV_MAGIC = 0x53484B56u;  // "SHKV", SystemPromptCache.cs:25
constexpr int32_t SHKV_VERSION = 1;           // SystemPromptCache.cs:26

// BinaryWriter.Write(string): the UTF-8 byte count as a 7-bit encoded integer, then the bytes.
void shkv_put_string(std::string& out, const std::string& v) {
    uint32_t n = (uint32_t)v.size();
    while (n >= 0x80) {
        out.push_back((char)(n | 0x80));
        n >>= 7;
    }
    out.push_back((char)n);
    out += v;
}
void shkv_put32(std::string& out, uint32_t v) { out.append((const char*)&v, 4); }
void shkv_put64(std::string& out, int64_t v) { out.append((const char*)&v, 8); }

struct File {
    std::FILE* f = nullptr;
    ~File() {
        if (f) std::fclose(f);
    }
};

}  // namespace

int jv_kv_save_shkv(jv_ctx* x, const char* path, const char* fingerprint, const int32_t* tokens, int32_t n_tokens) {
    if (!x || !path || !fingerprint || (!tokens && n_tokens > 0)) return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] {
        if (n_tokens < 0 || n_tokens > x->length)
            throw Error(JV_ERR_RANGE, "Only " + std::to_string(x->length) + " positions are cached.");
        set_device(x->m);
        ctx_upload_pages(x);
        const jv_config& c = x->m->cfg;
        const int64_t total = jv_kv_snapshot_floats(x, n_tokens);
        std::string head;
        shkv_put32(head, SHKV_MAGIC);
        shkv_put32(head, (uint32_t)SHKV_VERSION);
        shkv_put_string(head, fingerprint);
        shkv_put32(head, (uint32_t)n_tokens);
        for (int i = 0; i < n_tokens; i++) shkv_put32(head, (uint32_t)tokens[i]);
        shkv_put64(head, total);
        File f;
        f.f = std::fopen(path, "wb");
        if (!f.f) throw Error(JV_ERR_IO, std::string("cannot create ") + path);
        if (std::fwrite(head.data(), 1, head.size(), f.f) != head.size()) throw Error(JV_ERR_IO, std::string("write failed: ") + path);
        // one (K|V, layer) slice of the flat layout at a time: gather from the pages on the
        // device, one copy to pinned memory, one write
        const int64_t slice = (int64_t)c.kv_heads * n_tokens * 128;
        float* d = x->cap32.get((size_t)std::max<int64_t>(1, slice));
        float* h = x->h_cap.get((size_t)std::max<int64_t>(1, slice));
        for (int64_t base = 0; base < total; base += slice) {
            launch_kv_export(x->m->pool, ctx_table(x), x->m->page_bytes, x->m->page_slots, c.layers, c.kv_heads, n_tokens, d,
                             x->stream, base, slice, x->d_err);
            JV_CUDA(cudaMemcpyAsync(h, d, sizeof(float) * slice, cudaMemcpyDeviceToHost, x->stream));
            JV_CUDA(cudaStreamSynchronize(x->stream));
            if (std::fwrite(h, sizeof(float), (size_t)slice, f.f) != (size_t)slice)
                throw Error(JV_ERR_IO, std::string("write failed: ") + path);
        }
        if (std::fflush(f.f) != 0) throw Error(JV_ERR_IO, std::string("write failed: ") + path);
    });
}

int jv_kv_load_shkv(jv_ctx* x, const char* path, const char* fingerprint, int32_t* tokens_out, int32_t max_tokens,
                    int32_t* n_tokens) {
    if (!x || !path || !fingerprint || !n_tokens) return set_error(JV_ERR_ARG, "NULL argument");
    *n_tokens = 0;
    return guarded([&] {
        File f;
        f.f = std::fopen(path, "rb");
        if (!f.f) throw Error(JV_ERR_IO, std::string("cannot open ") + path);
        auto get = [&](void* dst, size_t n) {
            if (std::fread(dst, 1, n, f.f) != n) throw Error(JV_ERR_FORMAT, std::string(path) + " is truncated");
        };
        uint32_t magic = 0;
        int32_t version = 0;
        get(&magic, 4);
        get(&version, 4);
        if (magic != SHKV_MAGIC || version != SHKV_VERSION) throw Error(JV_ERR_FORMAT, std::string(path) + " is not an SHKV v1 file");
        uint32_t len = 0;
        for (int shift = 0;; shift += 7) {
            uint8_t b = 0;
            get(&b, 1);
            if (shift > 28) throw Error(JV_ERR_FORMAT, "bad fingerprint length");
            len |= (uint32_t)(b & 0x7F) << shift;
            if (!(b & 0x80)) break;
        }
        if (len > (1u << 20)) throw Error(JV_ERR_FORMAT, "bad fingerprint length");
        std::string fp(len, '\0');
        get(fp.data(), len);
        if (fp != fingerprint) throw Error(JV_ERR_FORMAT, "the snapshot was captured for a different model or prefix");
        int32_t count = 0;
        get(&count, 4);
        if (count < 0 || count > 1000000) throw Error(JV_ERR_FORMAT, "bad token count");
        std::vector<int32_t> toks((size_t)count);
        if (count) get(toks.data(), sizeof(int32_t) * (size_t)count);
        int64_t state = 0;
        get(&state, 8);
        if (state != jv_kv_snapshot_floats(x, count))
            throw Error(JV_ERR_FORMAT, "the snapshot holds " + std::to_string(state) + " floats; " + std::to_string(count) +
                                           " positions of this model need " + std::to_string(jv_kv_snapshot_floats(x, count)));
        const long here = std::ftell(f.f);
        std::fseek(f.f, 0, SEEK_END);
        const long end = std::ftell(f.f);
        if (here < 0 || end - here < (long)(state * 4)) throw Error(JV_ERR_FORMAT, std::string(path) + " is truncated");
        std::fseek(f.f, here, SEEK_SET);
        if (count > max_tokens || (!tokens_out && count > 0))
            throw Error(JV_ERR_RANGE, "the snapshot holds " + std::to_string(count) + " tokens; the buffer holds " +
                                          std::to_string(max_tokens));
        // the file is a valid snapshot of this model: now replace the cache with it
        set_device(x->m);
        const jv_config& c = x->m->cfg;
        ctx_ensure_capacity(x, std::max(1, count));
        std::vector<int> wp;
        for (int p = 0; p * x->m->page_slots < count; p++) wp.push_back(p);
        ctx_make_writable(x, wp);
        ctx_upload_pages(x);
        const int64_t slice = (int64_t)c.kv_heads * count * 128;
        float* d = x->cap32.get((size_t)std::max<int64_t>(1, slice));
        float* h = x->h_cap.get((size_t)std::max<int64_t>(1, slice));
        x->length = 0;  // the pages hold a partial copy until the last slice is in
        for (int64_t base = 0; base < state; base += slice) {
            if (std::fread(h, sizeof(float), (size_t)slice, f.f) != (size_t)slice)
                throw Error(JV_ERR_IO, std::string("read failed: ") + path);
            JV_CUDA(cudaMemcpyAsync(d, h, sizeof(float) * slice, cudaMemcpyHostToDevice, x->stream));
            launch_kv_import(x->m->pool, ctx_table(x), x->m->page_bytes, x->m->page_slots, c.layers, c.kv_heads, count, d,
                             x->d_err, x->stream, base, slice);
            JV_CUDA(cudaStreamSynchronize(x->stream));
        }
        sync_check(x);
        x->length = count;
        if (count) std::memcpy(tokens_out, toks.data(), sizeof(int32_t) * (size_t)count);
        *n_tokens = count;
    });
}

int jv_kv_share(jv_ctx* x, int32_t length, jv_snapshot** out) {
    if (!x || !out) return set_error(JV_ERR_ARG, "NULL argument");
    *out = nullptr;
    return guarded([&] {
        if (length > x->length || length < 0)
            throw Error(JV_ERR_RANGE, "Only " + std::to_string(x->length) + " positions are cached.");
        jv_snapshot* s = new jv_snapshot();
        s->model = x->m;
        s->length = length;
        int np = (length + x->m->page_slots - 1) / x->m->page_slots;
        for (int i = 0; i < np; i++) {
            s->pages.push_back(x->pages[i]);
            x->m->retain(x->pages[i]);
        }
        *out = s;
    });
}

int jv_kv_adopt(jv_ctx* x, const jv_snapshot* s) {
    if (!x || !s) return set_error(JV_ERR_ARG, "NULL argument");
    return guarded([&] {
        if (s->model != x->m) throw Error(JV_ERR_ARG, "the snapshot belongs to another model");
        set_device(x->m);
        JV_CUDA(cudaStreamSynchronize(x->stream));
        for (int p : s->pages) x->m->retain(p);
        ctx_release_pages(x);
        x->pages = s->pages;
        x->pages_dirty = true;
        x->length = s->length;
        if (x->capacity < s->length) ctx_ensure_capacity(x, s->length);
    });
}

int32_t jv_snapshot_length(const jv_snapshot* s) { return s ? s->length : 0; }

void jv_snapshot_release(jv_snapshot* s) {
    if (!s) return;
    for (int p : s->pages) s->model->release(p);
    delete s;
}

}  // extern "C"
