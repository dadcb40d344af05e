// jv_oracle.cpp — CPU restatement of the Jevstral Ministral-3 forward pass.
//
// TEST INFRASTRUCTURE ONLY. This file is the parity oracle for the B200 build: the
// tests, the smoke check and bench.py's CPU-baseline leg load it (through ctypes) to
// check or time the CUDA path. The product library never links, loads or calls it.
//
// It restates, op for op and in float32, the reference's managed CPU path
// (theolivenbaum/llm-shield, src/Jevstral/...). Each function names the reference
// lines it follows. The reference itself is C# (.NET 10) and cannot be built here, so
// this restatement is pinned instead by:
//   * the dequantizer golden vectors of tests/fixtures/quantization.json (bit-exact),
//   * the reference's NumPy model tools/reference_shieldstral.py run on the same
//     random weights (tests/golden/, at tolerance), and
//   * the kernel-definition tests of tests/Jevstral.Tests/*.cs restated in pytest.
//
// Build: oracle/Makefile (g++ -O3 -mavx2 -mfma -ffp-contract=off). Contraction is off
// because the reference keeps multiply and add separate wherever it writes them
// separately (Dequantizer Q5_1, RmsNorm, Rope.Apply, SwiGlu), and uses explicit FMA
// exactly where it asks for one (PanelGemm tiles, AttentionKernels).
#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <functional>
#include <limits>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <vector>

namespace orc {

// ------------------------------------------------------------------ errors

static thread_local std::string g_error;

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
// Codes mirror include/jv.h so tests can compare error behaviour across both sides.
enum { OK = 0, ERR_ARG = 1, ERR_RANGE = 2, ERR_FORMAT = 3, ERR_IO = 4, ERR_UNSUPPORTED = 5 };

// ------------------------------------------------------------- threading

static int g_threads = 0;
static int thread_count() {
    if (g_threads > 0) return g_threads;
    unsigned n = std::thread::hardware_concurrency();
    return n == 0 ? 1 : (int)n;
}

// Parallel.ForAsync(0, n, options, body) — the reference's only fan-out. Every
// index writes disjoint output, so the worker count never changes a result
// (KernelTests.MaxDegreeOfParallelismDoesNotChangeTheResult, KernelTests.cs:180-203).
static void parallel_for(int n, const std::function<void(int)>& body) {
    int workers = std::min(thread_count(), n);
    if (workers <= 1) {
        for (int i = 0; i < n; i++) body(i);
        return;
    }
    std::atomic<int> next{0};
    std::vector<std::thread> pool;
    pool.reserve(workers);
    for (int w = 0; w < workers; w++)
        pool.emplace_back([&] {
            for (int i; (i = next.fetch_add(1)) < n;) body(i);
        });
    for (auto& t : pool) t.join();
}

// ------------------------------------------------------------ GGML types

// ggml_type numbering, GgmlType.cs:9-44 (only what the hot path reads).
enum GgmlType : uint32_t {
    F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9,
    Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, BF16 = 30
};

// GgmlTypeInfo.BlockSize / TypeSize, GgmlType.cs:55-106.
static int block_size(uint32_t t) {
    switch (t) {
        case F32: case F16: case BF16: return 1;
        case Q4_0: case Q4_1: case Q5_0: case Q5_1: case Q8_0: case Q8_1: return 32;
        case Q2_K: case Q3_K: case Q4_K: case Q5_K: case Q6_K: return 256;
        default: throw Error(ERR_UNSUPPORTED, "GGML type " + std::to_string(t) + " is not on the hot path");
    }
}
static int type_size(uint32_t t) {
    switch (t) {
        case F32: return 4;
        case F16: case BF16: return 2;
        case Q4_0: return 2 + 16;
        case Q4_1: return 2 + 2 + 16;
        case Q5_0: return 2 + 4 + 16;
        case Q5_1: return 2 + 2 + 4 + 16;
        case Q8_0: return 2 + 32;
        case Q8_1: return 2 + 2 + 32;
        case Q2_K: return 84;
        case Q3_K: return 110;
        case Q4_K: return 144;
        case Q5_K: return 176;
        case Q6_K: return 210;
        default: throw Error(ERR_UNSUPPORTED, "GGML type " + std::to_string(t) + " is not on the hot path");
    }
}
// GgmlTypeInfo.RowBytes, GgmlType.cs:112-120.
static int64_t row_bytes(uint32_t t, int64_t elements) {
    int b = block_size(t);
    if (elements % b != 0)
        throw Error(ERR_ARG, "rows must be a multiple of " + std::to_string(b) + " elements; got " +
                                 std::to_string(elements));
    return elements / b * type_size(t);
}

// IEEE half -> float, exact (the C# `(float)Half` conversion).
static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: renormalise
            int e = -1;
            do { e++; man <<= 1; } while ((man & 0x400) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000 | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}
static inline uint16_t rd16(const uint8_t* p) { uint16_t v; std::memcpy(&v, p, 2); return v; }
static inline uint32_t rd32(const uint8_t* p) { uint32_t v; std::memcpy(&v, p, 4); return v; }

// Dequantizer.Dequantize, Dequantizer.cs:45-93, restricted to the hot-path types.
// Q4_0 :155-182   v = d * (nibble - 8); low nibbles are elements 0-15, high 16-31.
// Q5_1 :240-268   v = d * q5 + m, multiply then add (never fused).
// Q8_0 :270-305   v = d * q.
static void dequantize(uint32_t type, const uint8_t* src, float* dst, int64_t count) {
    int bs = block_size(type);
    if (count % bs != 0)
        throw Error(ERR_ARG, "decodes whole blocks of " + std::to_string(bs) + "; asked for " +
                                 std::to_string(count) + " elements");
    switch (type) {
        case F32: std::memcpy(dst, src, (size_t)count * 4); return;
        case F16:
            for (int64_t i = 0; i < count; i++) dst[i] = half_to_float(rd16(src + 2 * i));
            return;
        case BF16:
            for (int64_t i = 0; i < count; i++) {
                uint32_t bits = (uint32_t)rd16(src + 2 * i) << 16;
                std::memcpy(dst + i, &bits, 4);
            }
            return;
        case Q4_0:
            for (int64_t b = 0; b < count / 32; b++, src += 18, dst += 32) {
                float d = half_to_float(rd16(src));
                const uint8_t* qs = src + 2;
                for (int j = 0; j < 16; j++) {
                    dst[j] = d * (float)((qs[j] & 0x0F) - 8);
                    dst[16 + j] = d * (float)((qs[j] >> 4) - 8);
                }
            }
            return;
        case Q5_1:
            for (int64_t b = 0; b < count / 32; b++, src += 24, dst += 32) {
                float d = half_to_float(rd16(src));
                float m = half_to_float(rd16(src + 2));
                uint32_t qh = rd32(src + 4);
                const uint8_t* qs = src + 8;
                for (int j = 0; j < 16; j++) {
                    int lo = (qs[j] & 0x0F) | (int)(((qh >> j) & 1) << 4);
                    int hi = (qs[j] >> 4) | (int)(((qh >> (j + 16)) & 1) << 4);
                    float plo = d * (float)lo;
                    float phi = d * (float)hi;
                    dst[j] = plo + m;
                    dst[16 + j] = phi + m;
                }
            }
            return;
        case Q8_0:
            for (int64_t b = 0; b < count / 32; b++, src += 34, dst += 32) {
                float d = half_to_float(rd16(src));
                const int8_t* qs = (const int8_t*)(src + 2);
                for (int j = 0; j < 32; j++) dst[j] = d * (float)qs[j];
            }
            return;
        // Q4_1 :184-209  v = d * nibble + m.
        case Q4_1:
            for (int64_t b = 0; b < count / 32; b++, src += 20, dst += 32) {
                float d = half_to_float(rd16(src)), m = half_to_float(rd16(src + 2));
                const uint8_t* qs = src + 4;
                for (int j = 0; j < 16; j++) {
                    float lo = d * (float)(qs[j] & 0x0F), hi = d * (float)(qs[j] >> 4);
                    dst[j] = lo + m;
                    dst[16 + j] = hi + m;
                }
            }
            return;
        // Q5_0 :211-238  v = d * (q5 - 16).
        case Q5_0:
            for (int64_t b = 0; b < count / 32; b++, src += 22, dst += 32) {
                float d = half_to_float(rd16(src));
                uint32_t qh = rd32(src + 2);
                const uint8_t* qs = src + 6;
                for (int j = 0; j < 16; j++) {
                    int lo = (qs[j] & 0x0F) | (int)(((qh >> j) & 1) << 4);
                    int hi = (qs[j] >> 4) | (int)(((qh >> (j + 16)) & 1) << 4);
                    dst[j] = d * (float)(lo - 16);
                    dst[16 + j] = d * (float)(hi - 16);
                }
            }
            return;
        // Q8_1 :307-318  v = d * q (the stored block sum plays no part).
        case Q8_1:
            for (int64_t b = 0; b < count / 32; b++, src += 36, dst += 32) {
                float d = half_to_float(rd16(src));
                const int8_t* qs = (const int8_t*)(src + 4);
                for (int j = 0; j < 32; j++) dst[j] = d * (float)qs[j];
            }
            return;
        // Q2_K :323-344  per 16: dl = d * (sc & 15), ml = dmin * (sc >> 4); v = dl * q - ml.
        case Q2_K:
            for (int64_t b = 0; b < count / 256; b++, src += 84, dst += 256) {
                const uint8_t* scales = src;
                const uint8_t* qs = src + 16;
                float d = half_to_float(rd16(src + 80)), dmin = half_to_float(rd16(src + 82));
                int o = 0;
                for (int g = 0; g < 2; g++)
                    for (int s = 0; s < 4; s++)
                        for (int j = 0; j < 32; j++, o++) {
                            int sb = o >> 4;
                            float dl = d * (float)(scales[sb] & 0x0F), ml = dmin * (float)(scales[sb] >> 4);
                            int q = (qs[g * 32 + j] >> (2 * s)) & 3;
                            float p = dl * (float)q;
                            dst[o] = p - ml;
                        }
            }
            return;
        // Q3_K :346-376  6-bit signed scales per 16; v = d * sc * (ql - 4 * (1 - hbit)).
        case Q3_K:
            for (int64_t b = 0; b < count / 256; b++, src += 110, dst += 256) {
                const uint8_t* hmask = src;
                const uint8_t* qs = src + 32;
                const uint8_t* scales = src + 96;
                float d = half_to_float(rd16(src + 108));
                int sc[16];
                for (int k = 0; k < 16; k++) {
                    int low = scales[k & 7] >> (k < 8 ? 0 : 4);
                    int high = scales[8 + (k & 3)] >> (2 * (k >> 2));
                    sc[k] = (int)(int8_t)(((low & 0x0F) | ((high & 0x03) << 4)) - 32);
                }
                int o = 0;
                for (int g = 0; g < 2; g++)
                    for (int s = 0; s < 4; s++)
                        for (int j = 0; j < 32; j++, o++) {
                            int ql = (qs[g * 32 + j] >> (2 * s)) & 3;
                            int qh = ((hmask[j] >> (g * 4 + s)) & 1) ^ 1;
                            float t = d * (float)sc[o >> 4];
                            dst[o] = t * (float)(ql - (qh << 2));
                        }
            }
            return;
        // Q4_K :396-419 / Q5_K :421-448  per 32: dl = d * sc, ml = dmin * mn; v = dl * q - ml,
        // the 6-bit scale/min pairs unpacked as UnpackK4Scales (:385-394) does.
        case Q4_K:
        case Q5_K: {
            const bool five = type == Q5_K;
            const int bytes = five ? 176 : 144;
            for (int64_t b = 0; b < count / 256; b++, src += bytes, dst += 256) {
                float d = half_to_float(rd16(src)), dmin = half_to_float(rd16(src + 2));
                const uint8_t* p = src + 4;
                uint8_t sc[8], mn[8];
                for (int i = 0; i < 4; i++) {
                    sc[i] = p[i] & 0x3F;
                    mn[i] = p[4 + i] & 0x3F;
                    sc[4 + i] = (uint8_t)((p[8 + i] & 0x0F) | ((p[i] >> 2) & 0x30));
                    mn[4 + i] = (uint8_t)((p[8 + i] >> 4) | ((p[4 + i] >> 2) & 0x30));
                }
                const uint8_t* qh = src + 16;
                const uint8_t* qs = src + (five ? 48 : 16);
                int o = 0;
                for (int g = 0; g < 4; g++)
                    for (int s = 0; s < 2; s++) {
                        int sb = g * 2 + s;
                        float dl = d * (float)sc[sb], ml = dmin * (float)mn[sb];
                        for (int j = 0; j < 32; j++, o++) {
                            int q = (qs[g * 32 + j] >> (4 * s)) & 0x0F;
                            if (five) q |= ((qh[j] >> sb) & 1) << 4;
                            float t = dl * (float)q;
                            dst[o] = t - ml;
                        }
                    }
            }
            return;
        }
        // Q6_K :450-471  v = d * scales[o / 16] * (q6 - 32).
        case Q6_K:
            for (int64_t b = 0; b < count / 256; b++, src += 210, dst += 256) {
                const uint8_t* ql = src;
                const uint8_t* qh = src + 128;
                const int8_t* scales = (const int8_t*)(src + 192);
                float d = half_to_float(rd16(src + 208));
                int o = 0;
                for (int g = 0; g < 2; g++)
                    for (int s = 0; s < 2; s++)
                        for (int j = 0; j < 64; j++, o++) {
                            int lo = (ql[g * 64 + j] >> (4 * s)) & 0x0F;
                            int hi = (qh[g * 32 + (j & 31)] >> (2 * (s * 2 + (j >> 5)))) & 0x03;
                            float t = d * (float)scales[o >> 4];
                            dst[o] = t * (float)((lo | (hi << 4)) - 32);
                        }
            }
            return;
        default:
            throw Error(ERR_UNSUPPORTED, "no dequantizer for GGML type " + std::to_string(type));
    }
}

// ------------------------------------------------------- vector primitives

// Horizontal sum of a 16-lane vector the way a 512-bit register is folded: halves,
// then quarters, down to one lane. `System.Numerics.Vector.Sum` and the tail of every
// TensorPrimitives reduction fold this way; their exact order is not pinned by any
// reference test, so anything built on it is matched at tolerance only.
static float fold16(const float* v) {
    float a[16];
    std::memcpy(a, v, sizeof a);
    for (int w = 8; w >= 1; w /= 2)
        for (int i = 0; i < w; i++) a[i] = a[i] + a[i + w];
    return a[0];
}

// TensorPrimitives.Dot (System.Numerics.Tensors 10.0.0, not vendored): 16 lanes of
// fused multiply-add, folded at the end. Used by RunRowsFloat (QuantMatMul.cs:167), the
// verdict head (MinistralModel.cs:401) and the portable attention path (:527).
static float dot(const float* a, const float* b, int n) {
    float acc[16] = {0};
    int i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 16; l++) acc[l] = std::fmaf(a[i + l], b[i + l], acc[l]);
    float s = fold16(acc);
    for (; i < n; i++) s = std::fmaf(a[i], b[i], s);
    return s;
}

// TensorPrimitives.Sum, same caveat as dot().
static float sum(const float* x, int n) {
    float acc[16] = {0};
    int i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 16; l++) acc[l] += x[i + l];
    float s = fold16(acc);
    for (; i < n; i++) s += x[i];
    return s;
}

// Kernels.RmsNorm, Kernels.cs:25-60. Two 16-lane float accumulators of squares (even
// and odd 16-element slices), folded to float and widened to double for the final add;
// the scalar tail accumulates in double. scale = 1/sqrt((float)(sum/n) + eps), then
// y = (x * scale) * w.
static void rmsnorm(const float* x, const float* w, float eps, float* y, int n) {
    double s = 0;
    int i = 0;
    if (n >= 32) {
        float even[16] = {0}, odd[16] = {0};
        for (; i + 32 <= n; i += 32)
            for (int l = 0; l < 16; l++) {
                float a = x[i + l], b = x[i + 16 + l];
                float aa = a * a, bb = b * b;
                even[l] = even[l] + aa;
                odd[l] = odd[l] + bb;
            }
        s = (double)fold16(even) + (double)fold16(odd);
    }
    for (; i < n; i++) s += (double)x[i] * (double)x[i];
    float scale = 1.0f / std::sqrt((float)(s / n) + eps);
    for (int k = 0; k < n; k++) {
        float v = x[k] * scale;
        y[k] = v * w[k];
    }
}

// Kernels.Softmax, Kernels.cs:102-121: max-shift, exp, divide by the sum; a row whose
// max is not finite (all masked) becomes uniform.
static void softmax(float* x, int n) {
    if (n == 0) return;
    float mx = -std::numeric_limits<float>::infinity();
    bool nan = false;
    for (int i = 0; i < n; i++) {
        if (std::isnan(x[i])) nan = true;
        mx = std::max(mx, x[i]);
    }
    if (nan || !std::isfinite(mx)) {
        for (int i = 0; i < n; i++) x[i] = 1.0f / n;
        return;
    }
    for (int i = 0; i < n; i++) x[i] = std::exp(x[i] - mx);
    float s = sum(x, n);
    for (int i = 0; i < n; i++) x[i] = x[i] / s;
}

// Kernels.SwiGlu, Kernels.cs:82-89: up <- gate*up; dst <- sigmoid(gate); dst <- dst*up.
// dst may alias gate.
static void swiglu(const float* gate, float* up, float* dst, int n) {
    for (int i = 0; i < n; i++) up[i] = gate[i] * up[i];
    for (int i = 0; i < n; i++) dst[i] = 1.0f / (1.0f + std::exp(-gate[i]));
    for (int i = 0; i < n; i++) dst[i] = dst[i] * up[i];
}

// ------------------------------------------------------------ QuantMatMul

struct Matrix {  // WeightMatrix, WeightMatrix.cs:16-66
    uint32_t type = F32;
    const uint8_t* data = nullptr;
    int rows = 0, cols = 0;
    int64_t rowBytes = 0;
    bool empty() const { return data == nullptr; }
    const uint8_t* row(int r) const { return data + (int64_t)r * rowBytes; }
};

static const int kPanel = 64;     // PanelGemm.PanelWidth, PanelGemm.cs:36
static const int kKBlock = 2048;  // PanelGemm.KBlock, PanelGemm.cs:43

// PanelGemm.ForwardAsync/RunPanel/Pack/Tile*, PanelGemm.cs:76-318.
// y[t, r] = one fused multiply-add chain over k in ascending order, started from zero,
// continued through y across 2048-wide K blocks. That order is the whole contract: it
// makes a token's result independent of the batch around it (PanelGemmTests.cs:61-74).
// Here the 64-row panel is decoded per K block into [k][64] and tokens are streamed
// six at a time against it with 8-lane AVX2 FMA, which keeps exactly that per-element
// chain (each lane is its own output row).
// The same tile with 16-lane AVX-512 vectors (the reference's Tile512x6 width), used when the
// host has AVX-512F: six tokens against the whole 64-row panel per k, each lane still its own
// output row's FMA chain in ascending k, so the results are the AVX2 tile's bit for bit.
__attribute__((target("avx512f"))) static void panel_tile6_avx512(const float* packed, const float* xk, int64_t cols,
                                                                 int kc, bool acc, float* yr, int64_t rows) {
    __m512 c[6][4];
    for (int i = 0; i < 6; i++)
        for (int h = 0; h < 4; h++)
            c[i][h] = acc ? _mm512_loadu_ps(yr + i * rows + 16 * h) : _mm512_setzero_ps();
    const float* p = packed;
    for (int k = 0; k < kc; k++, p += kPanel) {
        __m512 b0 = _mm512_loadu_ps(p), b1 = _mm512_loadu_ps(p + 16), b2 = _mm512_loadu_ps(p + 32),
               b3 = _mm512_loadu_ps(p + 48);
        for (int i = 0; i < 6; i++) {
            __m512 a = _mm512_set1_ps(xk[i * cols + k]);
            c[i][0] = _mm512_fmadd_ps(a, b0, c[i][0]);
            c[i][1] = _mm512_fmadd_ps(a, b1, c[i][1]);
            c[i][2] = _mm512_fmadd_ps(a, b2, c[i][2]);
            c[i][3] = _mm512_fmadd_ps(a, b3, c[i][3]);
        }
    }
    for (int i = 0; i < 6; i++)
        for (int h = 0; h < 4; h++) _mm512_storeu_ps(yr + i * rows + 16 * h, c[i][h]);
}

// 0: the widest vectors the host has; 1: the AVX2 tile only (orc_set_isa).
static int g_isa = 0;
static bool use_avx512() {
    static const bool has = __builtin_cpu_supports("avx512f");
    return has && g_isa == 0;
}

static void panel_gemm(const Matrix& w, const float* x, int tokens, float* y) {
    int cols = w.cols, rows = w.rows;
    int panels = rows / kPanel;
    const bool wide = use_avx512();
    parallel_for(panels, [&](int panel) {
        int r0 = panel * kPanel;
        int kb = std::min(cols, kKBlock);
        std::vector<float> packed((size_t)kb * kPanel);
        std::vector<float> rowbuf((size_t)kb);
        for (int k0 = 0; k0 < cols; k0 += kKBlock) {
            int kc = std::min(kKBlock, cols - k0);
            int64_t off = row_bytes(w.type, k0);
            for (int j = 0; j < kPanel; j++) {
                dequantize(w.type, w.row(r0 + j) + off, rowbuf.data(), kc);
                for (int k = 0; k < kc; k++) packed[(size_t)k * kPanel + j] = rowbuf[k];
            }
            bool acc = k0 != 0;
            const float* xk = x + k0;
            float* yr = y + r0;
            int t = 0;
            if (wide)
                for (; t + 6 <= tokens; t += 6)
                    panel_tile6_avx512(packed.data(), xk + (int64_t)t * cols, cols, kc, acc, yr + (int64_t)t * rows, rows);
            for (; t + 6 <= tokens; t += 6) {
                for (int s = 0; s < kPanel; s += 16) {
                    __m256 c[6][2];
                    for (int i = 0; i < 6; i++)
                        for (int h = 0; h < 2; h++)
                            c[i][h] = acc ? _mm256_loadu_ps(yr + (int64_t)(t + i) * rows + s + 8 * h)
                                          : _mm256_setzero_ps();
                    const float* p = packed.data() + s;
                    for (int k = 0; k < kc; k++, p += kPanel) {
                        __m256 b0 = _mm256_loadu_ps(p), b1 = _mm256_loadu_ps(p + 8);
                        for (int i = 0; i < 6; i++) {
                            __m256 a = _mm256_set1_ps(xk[(int64_t)(t + i) * cols + k]);
                            c[i][0] = _mm256_fmadd_ps(a, b0, c[i][0]);
                            c[i][1] = _mm256_fmadd_ps(a, b1, c[i][1]);
                        }
                    }
                    for (int i = 0; i < 6; i++)
                        for (int h = 0; h < 2; h++)
                            _mm256_storeu_ps(yr + (int64_t)(t + i) * rows + s + 8 * h, c[i][h]);
                }
            }
            for (; t < tokens; t++) {
                __m256 c[8];
                for (int h = 0; h < 8; h++)
                    c[h] = acc ? _mm256_loadu_ps(yr + (int64_t)t * rows + 8 * h) : _mm256_setzero_ps();
                const float* p = packed.data();
                for (int k = 0; k < kc; k++, p += kPanel) {
                    __m256 a = _mm256_set1_ps(xk[(int64_t)t * cols + k]);
                    for (int h = 0; h < 8; h++) c[h] = _mm256_fmadd_ps(a, _mm256_loadu_ps(p + 8 * h), c[h]);
                }
                for (int h = 0; h < 8; h++) _mm256_storeu_ps(yr + (int64_t)t * rows + 8 * h, c[h]);
            }
        }
    });
}

// QuantMatMul.RunRowsFloat, QuantMatMul.cs:140-176: decode a row, then
// TensorPrimitives.Dot against every token (the Float strategy; QuantMatMul.cs:90-95
// would pick the int8 path under Auto on AVX-512 for Q8_0, which the oracle pins off).
static void rows_float(const Matrix& w, const float* x, int tokens, float* y) {
    int cols = w.cols, rows = w.rows;
    int chunks = (rows + 63) / 64;
    parallel_for(chunks, [&](int chunk) {
        std::vector<float> scratch((size_t)cols);
        int r1 = std::min(rows, chunk * 64 + 64);
        for (int r = chunk * 64; r < r1; r++) {
            dequantize(w.type, w.row(r), scratch.data(), cols);
            for (int t = 0; t < tokens; t++) y[(int64_t)t * rows + r] = dot(x + (int64_t)t * cols, scratch.data(), cols);
        }
    });
}

// QuantMatMul.ForwardAsync, QuantMatMul.cs:66-121: two or more tokens take the panel
// GEMM (PanelMinTokens = 2, :51) when the shape tiles into 64-row panels; otherwise the
// row-wise float path.
static void matmul(const Matrix& w, const float* x, int tokens, float* y) {
    bool panel = tokens >= 2 && w.rows % kPanel == 0 && w.cols % block_size(w.type) == 0 &&
                 (w.cols <= kKBlock || kKBlock % block_size(w.type) == 0);
    if (panel)
        panel_gemm(w, x, tokens, y);
    else
        rows_float(w, x, tokens, y);
}

// ------------------------------------------------------------------ GGUF

struct Tensor {
    std::string name;
    std::vector<int64_t> shape;
    uint32_t type;
    uint64_t offset;
};

// A GGUF v2/v3 reader (GgufFile.cs:76-172): header, metadata, tensor table, alignment,
// truncation check. Metadata values that the model reads are kept as double / string /
// string-array-length.
struct Gguf {
    std::string path;
    uint8_t* base = nullptr;
    size_t length = 0;
    uint32_t version = 0;
    uint64_t dataOffset = 0;
    std::map<std::string, double> nums;
    std::map<std::string, std::string> strs;
    std::map<std::string, int64_t> arrayLens;
    std::map<std::string, Tensor> tensors;

    ~Gguf() {
        if (base) munmap(base, length);
    }

    uint64_t cur = 0;
    void need(uint64_t n) {
        if (cur + n > length) throw Error(ERR_FORMAT, path + " ends inside its header");
    }
    uint32_t u32() { need(4); uint32_t v; std::memcpy(&v, base + cur, 4); cur += 4; return v; }
    uint64_t u64() { need(8); uint64_t v; std::memcpy(&v, base + cur, 8); cur += 8; return v; }
    std::string str() {
        uint64_t n = u64();
        need(n);
        std::string s((const char*)base + cur, n);
        cur += n;
        return s;
    }
    static int scalar_size(uint32_t t) {
        switch (t) {
            case 0: case 1: case 7: return 1;
            case 2: case 3: return 2;
            case 4: case 5: case 6: return 4;
            case 10: case 11: case 12: return 8;
            default: return -1;
        }
    }
    double scalar(uint32_t t) {
        int sz = scalar_size(t);
        need(sz);
        const uint8_t* p = base + cur;
        cur += sz;
        switch (t) {
            case 0: return (double)*(const uint8_t*)p;
            case 1: return (double)*(const int8_t*)p;
            case 2: { uint16_t v; std::memcpy(&v, p, 2); return v; }
            case 3: { int16_t v; std::memcpy(&v, p, 2); return v; }
            case 4: { uint32_t v; std::memcpy(&v, p, 4); return v; }
            case 5: { int32_t v; std::memcpy(&v, p, 4); return v; }
            case 6: { float v; std::memcpy(&v, p, 4); return v; }
            case 7: return (double)*p;
            case 10: { uint64_t v; std::memcpy(&v, p, 8); return (double)v; }
            case 11: { int64_t v; std::memcpy(&v, p, 8); return (double)v; }
            case 12: { double v; std::memcpy(&v, p, 8); return v; }
        }
        return 0;
    }
    void value(const std::string& key, uint32_t t) {
        if (t == 8) {
            strs[key] = str();
        } else if (t == 9) {
            uint32_t et = u32();
            uint64_t n = u64();
            arrayLens[key] = (int64_t)n;
            for (uint64_t i = 0; i < n; i++) {
                if (et == 8) { uint64_t len = u64(); need(len); cur += len; }
                else if (et == 9) throw Error(ERR_FORMAT, path + ": nested arrays are not supported");
                else { int sz = scalar_size(et); if (sz < 0) throw Error(ERR_FORMAT, path + ": bad array type"); need(sz); cur += sz; }
            }
        } else {
            if (scalar_size(t) < 0) throw Error(ERR_FORMAT, path + ": unknown metadata value type " + std::to_string(t));
            nums[key] = scalar(t);
        }
    }

    explicit Gguf(const std::string& p) : path(p) {
        int fd = ::open(p.c_str(), O_RDONLY);
        if (fd < 0) throw Error(ERR_IO, "GGUF not found: " + p);
        struct stat st;
        fstat(fd, &st);
        length = (size_t)st.st_size;
        if (length < 16) { ::close(fd); throw Error(ERR_FORMAT, p + " is not a GGUF file (too short)."); }
        void* m = mmap(nullptr, length, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (m == MAP_FAILED) throw Error(ERR_IO, "cannot map " + p);
        base = (uint8_t*)m;
        uint32_t magic = u32();
        if (magic != 0x46554747u) throw Error(ERR_FORMAT, p + " is not a GGUF file (bad magic).");
        version = u32();
        if (version < 2 || version > 3) throw Error(ERR_FORMAT, "GGUF version " + std::to_string(version) + " is not supported (expected 2 or 3).");
        uint64_t nt = u64(), nkv = u64();
        for (uint64_t i = 0; i < nkv; i++) {
            std::string key = str();
            uint32_t t = u32();
            value(key, t);
        }
        for (uint64_t i = 0; i < nt; i++) {
            Tensor t;
            t.name = str();
            uint32_t dims = u32();
            for (uint32_t d = 0; d < dims; d++) t.shape.push_back((int64_t)u64());
            t.type = u32();
            t.offset = u64();
            tensors[t.name] = t;
        }
        uint64_t align = nums.count("general.alignment") ? (uint64_t)nums["general.alignment"] : 32;
        dataOffset = cur + (align - cur % align) % align;
        // GgufFile.ThrowIfTruncated, GgufFile.cs:156-172
        uint64_t required = dataOffset;
        for (auto& kv : tensors) {
            const Tensor& t = kv.second;
            int64_t elems = 1;
            for (auto s : t.shape) elems *= s;
            int64_t bytes;
            try { bytes = row_bytes(t.type, elems); } catch (Error&) { continue; }
            required = std::max<uint64_t>(required, dataOffset + t.offset + (uint64_t)bytes);
        }
        if (length < required)
            throw Error(ERR_IO, p + " is incomplete: " + std::to_string(length) + " bytes on disk but its tensors need " +
                                    std::to_string(required) + ". Re-download it.");
    }

    double num(const std::string& k, double dflt) const {
        auto it = nums.find(k);
        return it == nums.end() ? dflt : it->second;
    }
    double req(const std::string& k) const {
        auto it = nums.find(k);
        if (it == nums.end()) throw Error(ERR_FORMAT, path + " is missing metadata '" + k + "'");
        return it->second;
    }
    const Tensor* find(const std::string& name) const {
        auto it = tensors.find(name);
        return it == tensors.end() ? nullptr : &it->second;
    }
    const uint8_t* ptr(const Tensor& t) const { return base + dataOffset + t.offset; }
};

// ------------------------------------------------------------- ModelConfig

// ModelConfig.FromGguf, ModelConfig.cs:62-112 (llama.cpp key names, same defaults).
struct Config {
    int layers, hidden, heads, kvHeads, headDim, ff, vocab, ctx;
    float eps, ropeBase;
    int ropeDim;
    float ropeScale;
    std::string ropeType;
    int ropeOrigCtx;
    float betaFast, betaSlow, extFactor, mscale, mscaleAllDim, attnFactor, tempScale;
    bool yarnActive() const { return ropeType == "yarn" && ropeOrigCtx > 0 && extFactor != 0.f && ropeScale > 1.f; }
    int group() const { return heads / kvHeads; }
    int qDim() const { return heads * headDim; }
    int kvDim() const { return kvHeads * headDim; }
};

static Config config_from(const Gguf& g) {
    auto it = g.strs.find("general.architecture");
    if (it == g.strs.end()) throw Error(ERR_FORMAT, g.path + " has no general.architecture.");
    std::string a = it->second;
    if (a != "mistral3" && a != "ministral3" && a != "llama")
        throw Error(ERR_UNSUPPORTED, g.path + " is architecture '" + a + "'; only the Ministral-3 backbone is implemented.");
    Config c;
    c.heads = (int)g.req(a + ".attention.head_count");
    c.hidden = (int)g.req(a + ".embedding_length");
    c.headDim = (int)g.num(a + ".attention.key_length", c.hidden / std::max(1, c.heads));
    c.layers = (int)g.req(a + ".block_count");
    c.kvHeads = (int)g.num(a + ".attention.head_count_kv", c.heads);
    c.ff = (int)g.req(a + ".feed_forward_length");
    auto tl = g.arrayLens.find("tokenizer.ggml.tokens");
    c.vocab = tl != g.arrayLens.end() ? (int)tl->second : (int)g.req(a + ".vocab_size");
    c.eps = (float)g.num(a + ".attention.layer_norm_rms_epsilon", 1e-5);
    c.ctx = (int)g.num(a + ".context_length", 32768);
    c.ropeBase = (float)g.num(a + ".rope.freq_base", 10000.0);
    c.ropeDim = (int)g.num(a + ".rope.dimension_count", c.headDim);
    c.ropeScale = (float)g.num(a + ".rope.scaling.factor", 1.0);
    auto rt = g.strs.find(a + ".rope.scaling.type");
    c.ropeType = rt == g.strs.end() ? "" : rt->second;
    c.ropeOrigCtx = (int)g.num(a + ".rope.scaling.original_context_length", 0);
    c.betaFast = (float)g.num(a + ".rope.scaling.yarn_beta_fast", g.num(a + ".rope.scaling.beta_fast", 32.0));
    c.betaSlow = (float)g.num(a + ".rope.scaling.yarn_beta_slow", g.num(a + ".rope.scaling.beta_slow", 1.0));
    c.extFactor = (float)g.num(a + ".rope.scaling.yarn_ext_factor", 1.0);
    c.mscale = (float)g.num(a + ".rope.scaling.mscale", 0.0);
    c.mscaleAllDim = (float)g.num(a + ".rope.scaling.yarn_log_multiplier", g.num(a + ".rope.scaling.mscale_all_dim", 0.0));
    c.attnFactor = (float)g.num(a + ".rope.scaling.attn_factor", g.num(a + ".rope.scaling.yarn_attn_factor", 1.0));
    c.tempScale = (float)g.num(a + ".attention.temperature_scale", g.num(a + ".rope.scaling_beta", 0.0));
    if (c.kvHeads <= 0 || c.heads % c.kvHeads != 0)
        throw Error(ERR_FORMAT, std::to_string(c.heads) + " attention heads do not divide into " + std::to_string(c.kvHeads) + " KV heads.");
    return c;
}

// ------------------------------------------------------------------ RoPE

// Rope(), Rope.cs:33-106: one frequency per rotated pair, YaRN ramp when active, and the
// single magnitude factor.
struct Rope {
    std::vector<float> freqs;
    float mscale = 1.f;
    explicit Rope(const Config& c) {
        int half = c.ropeDim / 2;
        freqs.resize(half);
        float freqScale = 1.f / c.ropeScale;
        if (!c.yarnActive()) {
            for (int i = 0; i < half; i++) freqs[i] = freqScale / std::pow(c.ropeBase, 2.f * i / c.ropeDim);
            mscale = c.attnFactor;
            return;
        }
        float low, high;
        if (c.betaFast == 0.f && c.betaSlow == 0.f) {
            low = std::numeric_limits<float>::max();
            high = c.ropeDim / 2.f - 1.f;
        } else {
            auto corr = [&](float rot) {
                return c.ropeDim * std::log(c.ropeOrigCtx / (rot * 2 * (float)M_PI)) / (2 * std::log(c.ropeBase));
            };
            low = std::max(0.f, std::floor(corr(c.betaFast)));
            high = std::min(c.ropeDim / 2.f - 1.f, std::ceil(corr(c.betaSlow)));
        }
        for (int i = 0; i < half; i++) {
            float extrap = 1.f / std::pow(c.ropeBase, 2.f * i / c.ropeDim);
            float interp = freqScale * extrap;
            float y = (i - low) / std::max(0.001f, high - low);
            float mix = (1.f - std::min(std::max(y, 0.f), 1.f)) * c.extFactor;
            freqs[i] = interp * (1.f - mix) + extrap * mix;
        }
        // ComputeMagnitudeScale, Rope.cs:78-88
        auto ms = [](float scale, float m) { return scale <= 1.f ? 1.f : 0.1f * m * std::log(scale) + 1.f; };
        float factor = c.ropeScale;
        float m = c.mscale != 0.f ? c.mscale : 1.f;
        float ratio = c.mscaleAllDim != 0.f ? ms(factor, m) / ms(factor, c.mscaleAllDim) : ms(factor, 1.f);
        mscale = ratio * c.attnFactor;
    }

    // Rope.Apply, Rope.cs:112-135: adjacent pairs (x[2i], x[2i+1]).
    void apply(float* data, int heads, int headDim, int position) const {
        int half = (int)freqs.size();
        std::vector<float> cs(half), sn(half);
        for (int i = 0; i < half; i++) {
            float theta = (float)position * freqs[i];
            cs[i] = std::cos(theta) * mscale;
            sn[i] = std::sin(theta) * mscale;
        }
        for (int h = 0; h < heads; h++) {
            float* x = data + (int64_t)h * headDim;
            for (int i = 0; i < half; i++) {
                float x0 = x[2 * i], x1 = x[2 * i + 1];
                float a = x0 * cs[i], b = x1 * sn[i];
                float c2 = x0 * sn[i], d = x1 * cs[i];
                x[2 * i] = a - b;
                x[2 * i + 1] = c2 + d;
            }
        }
    }
};

// --------------------------------------------------------------- KV cache

// KvCache, KvCache.cs:12-140: fp32 [layer][head][capacity][dim], doubling growth.
struct KvCache {
    int layers, heads, dim;
    int capacity, length = 0;
    std::vector<std::vector<float>> keys, values;
    KvCache(int l, int h, int d, int cap) : layers(l), heads(h), dim(d), capacity(std::max(1, cap)) {
        keys = alloc(capacity);
        values = alloc(capacity);
    }
    std::vector<std::vector<float>> alloc(int cap) {
        std::vector<std::vector<float>> a(layers);
        for (auto& v : a) v.assign((size_t)heads * cap * dim, 0.f);
        return a;
    }
    void reset() { length = 0; }
    void truncate(int len) { length = std::min(std::max(len, 0), length); }
    void ensure(int required) {
        if (required <= capacity) return;
        int cap = capacity;
        while (cap < required) cap *= 2;
        auto k = alloc(cap), v = alloc(cap);
        for (int l = 0; l < layers; l++)
            for (int h = 0; h < heads; h++) {
                std::memcpy(&k[l][(size_t)h * cap * dim], &keys[l][(size_t)h * capacity * dim], sizeof(float) * length * dim);
                std::memcpy(&v[l][(size_t)h * cap * dim], &values[l][(size_t)h * capacity * dim], sizeof(float) * length * dim);
            }
        keys.swap(k);
        values.swap(v);
        capacity = cap;
    }
    void advance(int n) { length += n; }
    float* key(int l, int h, int p) { return &keys[l][((size_t)h * capacity + p) * dim]; }
    float* value(int l, int h, int p) { return &values[l][((size_t)h * capacity + p) * dim]; }
    int64_t snapshot_floats(int len) const { return (int64_t)layers * heads * len * dim * 2; }
    // Snapshot/Restore, KvCache.cs:94-136: keys for every layer and head, then values.
    void snapshot(int len, float* out) {
        if (len > length) throw Error(ERR_RANGE, "Only " + std::to_string(length) + " positions are cached.");
        size_t cur = 0;
        for (int pass = 0; pass < 2; pass++)
            for (int l = 0; l < layers; l++)
                for (int h = 0; h < heads; h++) {
                    const float* src = pass == 0 ? key(l, h, 0) : value(l, h, 0);
                    std::memcpy(out + cur, src, sizeof(float) * (size_t)len * dim);
                    cur += (size_t)len * dim;
                }
    }
    void restore(const float* snap, int64_t n, int len) {
        if (n != snapshot_floats(len))
            throw Error(ERR_ARG, "Snapshot holds " + std::to_string(n) + " floats; " + std::to_string(len) +
                                     " positions need " + std::to_string(snapshot_floats(len)) + ".");
        ensure(len);
        size_t cur = 0;
        for (int pass = 0; pass < 2; pass++)
            for (int l = 0; l < layers; l++)
                for (int h = 0; h < heads; h++) {
                    float* dst = pass == 0 ? key(l, h, 0) : value(l, h, 0);
                    std::memcpy(dst, snap + cur, sizeof(float) * (size_t)len * dim);
                    cur += (size_t)len * dim;
                }
        length = len;
    }
};

// ------------------------------------------------------------ TokenLayout

// TokenLayout, MinistralModel.cs:703-780.
struct Layout {
    std::vector<int> slot, pos, shared, seg, outputs;
    bool sparse = false;
    int end = 0;
};

// TokenLayout.Tree, MinistralModel.cs:720-745.
static Layout layout_tree(int startPos, int trunk, const std::vector<int>& offsets, int tokens) {
    Layout L;
    L.slot.resize(tokens); L.pos.resize(tokens); L.shared.resize(tokens); L.seg.resize(tokens);
    int branch = -1;
    for (int t = 0; t < tokens; t++) {
        L.slot[t] = startPos + t;
        while (branch + 1 < (int)offsets.size() && t >= offsets[branch + 1]) branch++;
        if (t < trunk || branch < 0) {
            L.pos[t] = startPos + t; L.shared[t] = startPos; L.seg[t] = startPos;
        } else {
            L.pos[t] = startPos + trunk + (t - offsets[branch]);
            L.shared[t] = startPos + trunk;
            L.seg[t] = startPos + offsets[branch];
        }
    }
    L.outputs.resize(offsets.size());
    for (size_t b = 0; b < offsets.size(); b++)
        L.outputs[b] = (b + 1 < offsets.size() ? offsets[b + 1] : tokens) - 1;
    L.end = startPos + tokens;
    return L;
}

// TokenLayout.Rows, MinistralModel.cs:758-780.
static Layout layout_rows(int shared, const std::vector<int>& rowBase, const std::vector<int>& rowLength,
                          const std::vector<int>& rowTokens, bool sparse) {
    Layout L;
    int total = 0;
    for (int c : rowTokens) total += c;
    L.slot.resize(total); L.pos.resize(total); L.shared.resize(total); L.seg.resize(total);
    L.outputs.resize(rowTokens.size());
    int t = 0, end = shared;
    for (size_t r = 0; r < rowTokens.size(); r++) {
        for (int i = 0; i < rowTokens[r]; i++, t++) {
            L.slot[t] = rowBase[r] + rowLength[r] + i;
            L.pos[t] = shared + rowLength[r] + i;
            L.shared[t] = shared;
            L.seg[t] = rowBase[r];
            end = std::max(end, L.slot[t] + 1);
        }
        L.outputs[r] = t - 1;
    }
    L.sparse = sparse;
    L.end = end;
    return L;
}

// ------------------------------------------------------------------ model

typedef void (*Sink)(void* user, const char* name, const float* values, int rows, int cols);

struct Layer {
    std::vector<float> attnNorm, ffnNorm;
    Matrix q, k, v, o, gate, up, down;
};

struct Model {
    std::unique_ptr<Gguf> gguf;
    Config cfg;
    std::unique_ptr<Rope> rope;
    Matrix embd, lmHead;
    std::vector<float> outNorm;
    std::vector<Layer> layers;
    std::unique_ptr<KvCache> kv;
    std::vector<float> logits;

    Matrix matrix(const std::string& name, bool required = true) {
        const Tensor* t = gguf->find(name);
        if (!t) {
            if (required) throw Error(ERR_FORMAT, gguf->path + " is missing tensor '" + name + "'.");
            return Matrix{};
        }
        if (t->shape.size() != 2) throw Error(ERR_FORMAT, "'" + name + "' has " + std::to_string(t->shape.size()) + " dimensions; a weight matrix needs 2.");
        Matrix m;
        m.type = t->type;
        block_size(t->type);
        m.data = gguf->ptr(*t);
        m.rows = (int)t->shape[1];
        m.cols = (int)t->shape[0];
        m.rowBytes = row_bytes(m.type, m.cols);
        return m;
    }
    std::vector<float> vec(const std::string& name) {
        const Tensor* t = gguf->find(name);
        if (!t) throw Error(ERR_FORMAT, gguf->path + " is missing tensor '" + name + "'.");
        int64_t n = 1;
        for (auto s : t->shape) n *= s;
        std::vector<float> v((size_t)n);
        dequantize(t->type, gguf->ptr(*t), v.data(), n);
        return v;
    }

    // MinistralModel(GgufFile), MinistralModel.cs:59-123.
    Model(const std::string& path, int initialCapacity) {
        gguf.reset(new Gguf(path));
        cfg = config_from(*gguf);
        rope.reset(new Rope(cfg));
        embd = matrix("token_embd.weight");
        outNorm = vec("output_norm.weight");
        lmHead = matrix("output.weight", false);
        layers.resize(cfg.layers);
        for (int l = 0; l < cfg.layers; l++) {
            std::string p = "blk." + std::to_string(l) + ".";
            Layer& L = layers[l];
            L.attnNorm = vec(p + "attn_norm.weight");
            L.q = matrix(p + "attn_q.weight");
            L.k = matrix(p + "attn_k.weight");
            L.v = matrix(p + "attn_v.weight");
            L.o = matrix(p + "attn_output.weight");
            L.ffnNorm = vec(p + "ffn_norm.weight");
            L.gate = matrix(p + "ffn_gate.weight");
            L.up = matrix(p + "ffn_up.weight");
            L.down = matrix(p + "ffn_down.weight");
        }
        if (embd.cols != cfg.hidden) throw Error(ERR_FORMAT, "token_embd width disagrees with the hidden size.");
        if (layers[0].q.rows != cfg.qDim()) throw Error(ERR_FORMAT, "attn_q rows disagree with heads x head_dim.");
        if (layers[0].k.rows != cfg.kvDim()) throw Error(ERR_FORMAT, "attn_k rows disagree with kv_heads x head_dim.");
        if (layers[0].gate.rows != cfg.ff) throw Error(ERR_FORMAT, "ffn_gate rows disagree with the FFN size.");
        kv.reset(new KvCache(cfg.layers, cfg.kvHeads, cfg.headDim, initialCapacity));
        logits.assign(cfg.vocab, 0.f);
    }

    const Matrix& head() const { return lmHead.empty() ? embd : lmHead; }

    // QuantMatMul.GatherRows, QuantMatMul.cs:294-305.
    void gather(const int32_t* ids, int n, float* dst) {
        for (int i = 0; i < n; i++) {
            int id = ids[i];
            if ((unsigned)id >= (unsigned)embd.rows)
                throw Error(ERR_RANGE, "Token id " + std::to_string(id) + " is outside the " + std::to_string(embd.rows) + "-entry embedding table.");
            dequantize(embd.type, embd.row(id), dst + (int64_t)i * embd.cols, embd.cols);
        }
    }

    void norm_rows(const float* src, const std::vector<float>& w, float* dst, int rows, int width) {
        for (int t = 0; t < rows; t++) rmsnorm(src + (int64_t)t * width, w.data(), cfg.eps, dst + (int64_t)t * width, width);
    }

    // ApplyPositionScale, MinistralModel.cs:676-682.
    void position_scale(float* q, int n, int position) {
        if (cfg.ropeOrigCtx <= 0 || cfg.tempScale == 0.f) return;
        float interval = std::floor((float)position / cfg.ropeOrigCtx);
        if (interval == 0.f) return;
        float s = 1.f + cfg.tempScale * std::log(1.f + interval);
        for (int i = 0; i < n; i++) q[i] = q[i] * s;
    }

    // AttendHead, MinistralModel.cs:564-636, with AttentionKernels.Scores/WeightedSum
    // (AttentionKernels.cs:44-105): each score is a fused chain over d ascending, times
    // the scale; softmax over exactly the visible keys [0, shared) then [segment, slot];
    // the weighted sum is a fused chain over those keys in that order.
    void attend_head(int layer, int kvHead, int head, const float* q, float* ctx, int seq, int startPos,
                     const Layout* L, float scale) {
        const int hd = cfg.headDim;
        const float* keys = kv->key(layer, kvHead, 0);
        const float* vals = kv->value(layer, kvHead, 0);
        std::vector<float> row;
        for (int t = 0; t < seq; t++) {
            int shared = L ? L->shared[t] : startPos;
            int segment = L ? L->seg[t] : startPos;
            int slot = L ? L->slot[t] : startPos + t;
            int limit = shared + (slot - segment + 1);
            row.resize(std::max(limit, 1));
            const float* qv = q + (int64_t)t * cfg.qDim() + (int64_t)head * hd;
            for (int i = 0; i < limit; i++) {
                int p = i < shared ? i : segment + (i - shared);
                const float* k = keys + (int64_t)p * hd;
                float a = 0.f;
                for (int d = 0; d < hd; d++) a = std::fmaf(qv[d], k[d], a);
                row[i] = a * scale;
            }
            softmax(row.data(), limit);
            float* o = ctx + (int64_t)t * cfg.qDim() + (int64_t)head * hd;
            for (int d = 0; d < hd; d++) o[d] = 0.f;
            for (int i = 0; i < limit; i++) {
                int p = i < shared ? i : segment + (i - shared);
                const float* v = vals + (int64_t)p * hd;
                float w = row[i];
                for (int d = 0; d < hd; d++) o[d] = std::fmaf(w, v[d], o[d]);
            }
        }
    }

    // The portable per-key loop, MinistralModel.cs:504-547 (sparse layouts): Dot times
    // the scale, softmax, then AddScaled (multiply, then add; zero weights skipped).
    void attend_head_portable(int layer, int kvHead, int head, const float* q, float* ctx, int seq, int startPos,
                              const Layout* L, float scale) {
        const int hd = cfg.headDim;
        const float* keys = kv->key(layer, kvHead, 0);
        const float* vals = kv->value(layer, kvHead, 0);
        std::vector<float> row;
        for (int t = 0; t < seq; t++) {
            int self = L ? L->slot[t] : startPos + t;
            int shared = L ? L->shared[t] : startPos;
            int segment = L ? L->seg[t] : startPos;
            int limit = shared + (self - segment + 1);
            row.resize(std::max(limit, 1));
            const float* qv = q + (int64_t)t * cfg.qDim() + (int64_t)head * hd;
            for (int i = 0; i < limit; i++) {
                int p = i < shared ? i : segment + (i - shared);
                row[i] = dot(qv, keys + (int64_t)p * hd, hd) * scale;
            }
            softmax(row.data(), limit);
            float* o = ctx + (int64_t)t * cfg.qDim() + (int64_t)head * hd;
            for (int d = 0; d < hd; d++) o[d] = 0.f;
            for (int i = 0; i < limit; i++) {
                float w = row[i];
                int p = i < shared ? i : segment + (i - shared);
                if (w != 0.f) {
                    const float* v = vals + (int64_t)p * hd;
                    for (int d = 0; d < hd; d++) { float sv = v[d] * w; o[d] = o[d] + sv; }
                }
            }
        }
    }

    // AttentionAsync, MinistralModel.cs:446-557.
    void attention(int l, const float* input, float* out, int seq, int startPos, const Layout* L, Sink sink, void* user) {
        const Layer& layer = layers[l];
        int qDim = cfg.qDim(), kvDim = cfg.kvDim(), hd = cfg.headDim;
        float scale = 1.f / std::sqrt((float)hd);
        std::vector<float> q((size_t)seq * qDim), kvb((size_t)seq * kvDim), ctx((size_t)seq * qDim);
        matmul(layer.q, input, seq, q.data());
        for (int t = 0; t < seq; t++) {  // RotateQueries :638-647
            int position = L ? L->pos[t] : startPos + t;
            rope->apply(q.data() + (int64_t)t * qDim, cfg.heads, hd, position);
            position_scale(q.data() + (int64_t)t * qDim, qDim, position);
        }
        if (sink) sink(user, ("blk." + std::to_string(l) + ".q_rope").c_str(), q.data(), seq, qDim);
        matmul(layer.k, input, seq, kvb.data());
        for (int t = 0; t < seq; t++) {  // StoreKeys :649-660
            float* row = kvb.data() + (int64_t)t * kvDim;
            rope->apply(row, cfg.kvHeads, hd, L ? L->pos[t] : startPos + t);
            int slot = L ? L->slot[t] : startPos + t;
            for (int kh = 0; kh < cfg.kvHeads; kh++) std::memcpy(kv->key(l, kh, slot), row + kh * hd, sizeof(float) * hd);
        }
        if (sink) sink(user, ("blk." + std::to_string(l) + ".k_rope").c_str(), kvb.data(), seq, kvDim);
        matmul(layer.v, input, seq, kvb.data());
        for (int t = 0; t < seq; t++) {  // StoreValues :662-669
            int slot = L ? L->slot[t] : startPos + t;
            for (int kh = 0; kh < cfg.kvHeads; kh++)
                std::memcpy(kv->value(l, kh, slot), kvb.data() + (int64_t)t * kvDim + kh * hd, sizeof(float) * hd);
        }
        if (sink) sink(user, ("blk." + std::to_string(l) + ".v").c_str(), kvb.data(), seq, kvDim);
        bool fast = hd == 128 && !(L && L->sparse);
        int group = cfg.group();
        parallel_for(cfg.heads, [&](int head) {
            if (fast)
                attend_head(l, head / group, head, q.data(), ctx.data(), seq, startPos, L, scale);
            else
                attend_head_portable(l, head / group, head, q.data(), ctx.data(), seq, startPos, L, scale);
        });
        if (sink) sink(user, ("blk." + std::to_string(l) + ".attn_weighted").c_str(), ctx.data(), seq, qDim);
        matmul(layer.o, ctx.data(), seq, out);
    }

    // The private ForwardAsync, MinistralModel.cs:301-435.
    // selectedMode: 0 = none; 1 = selected rows per output (out = [nOut][nRows]);
    //               2 = full vocabulary per output (out = [nOut][vocab]).
    void forward(const int32_t* tokens, int seq, bool computeLogits, const Layout* L, const int32_t* rows, int nRows,
                 int selectedMode, int nOut, float* out, Sink sink, void* user) {
        if (seq <= 0) throw Error(ERR_ARG, "No tokens to forward.");
        int startPos = kv->length;
        int hidden = cfg.hidden, ff = cfg.ff;
        int end = L ? L->end : startPos + seq;
        kv->ensure(end);
        std::vector<float> h((size_t)seq * hidden), norm((size_t)seq * hidden), scratch((size_t)seq * hidden);
        std::vector<float> g((size_t)seq * ff), u((size_t)seq * ff);
        gather(tokens, seq, h.data());
        if (sink) sink(user, "embeddings", h.data(), seq, hidden);
        for (int l = 0; l < cfg.layers; l++) {
            const Layer& layer = layers[l];
            std::string p = "blk." + std::to_string(l) + ".";
            norm_rows(h.data(), layer.attnNorm, norm.data(), seq, hidden);
            if (sink) sink(user, (p + "attn_norm").c_str(), norm.data(), seq, hidden);
            attention(l, norm.data(), scratch.data(), seq, startPos, L, sink, user);
            if (sink) sink(user, (p + "attn_out").c_str(), scratch.data(), seq, hidden);
            for (size_t i = 0; i < h.size(); i++) h[i] = h[i] + scratch[i];
            if (sink) sink(user, (p + "post_attn").c_str(), h.data(), seq, hidden);
            norm_rows(h.data(), layer.ffnNorm, norm.data(), seq, hidden);
            if (sink) sink(user, (p + "ffn_norm").c_str(), norm.data(), seq, hidden);
            matmul(layer.gate, norm.data(), seq, g.data());
            matmul(layer.up, norm.data(), seq, u.data());
            swiglu(g.data(), u.data(), g.data(), seq * ff);
            matmul(layer.down, g.data(), seq, scratch.data());
            if (sink) sink(user, (p + "ffn_out").c_str(), scratch.data(), seq, hidden);
            for (size_t i = 0; i < h.size(); i++) h[i] = h[i] + scratch[i];
            if (sink) sink(user, (p + "output").c_str(), h.data(), seq, hidden);
        }
        kv->advance(std::max(0, end - kv->length));

        if (selectedMode == 2) {  // :362-385 full vocabulary per output, one batched product
            std::vector<float> rowsBuf((size_t)nOut * hidden);
            for (int b = 0; b < nOut; b++) {
                int o = L ? L->outputs[b] : seq - 1;
                rmsnorm(h.data() + (int64_t)o * hidden, outNorm.data(), cfg.eps, rowsBuf.data() + (int64_t)b * hidden, hidden);
            }
            matmul(head(), rowsBuf.data(), nOut, out);
        } else if (selectedMode == 1) {  // :386-410 verdict rows only
            const Matrix& table = head();
            std::vector<float> n((size_t)hidden), row((size_t)hidden);
            for (int b = 0; b < nOut; b++) {
                int last = L ? L->outputs[b] : seq - 1;
                rmsnorm(h.data() + (int64_t)last * hidden, outNorm.data(), cfg.eps, n.data(), hidden);
                for (int i = 0; i < nRows; i++) {
                    if ((unsigned)rows[i] >= (unsigned)table.rows)
                        throw Error(ERR_RANGE, "vocabulary row " + std::to_string(rows[i]) + " is out of range");
                    dequantize(table.type, table.row(rows[i]), row.data(), hidden);
                    out[(int64_t)b * nRows + i] = dot(n.data(), row.data(), hidden);
                }
            }
        }
        if (!computeLogits) return;
        std::vector<float> last((size_t)hidden);  // :411-424
        rmsnorm(h.data() + (int64_t)(seq - 1) * hidden, outNorm.data(), cfg.eps, last.data(), hidden);
        if (sink) sink(user, "final_norm", last.data(), 1, hidden);
        matmul(head(), last.data(), 1, logits.data());
        if (sink) sink(user, "logits", logits.data(), 1, cfg.vocab);
    }
};

static int fail(const Error& e) {
    g_error = e.what();
    return e.code;
}

}  // namespace orc

using namespace orc;

#define ORC_TRY(...)                                          \
    try {                                                     \
        __VA_ARGS__;                                               \
        return OK;                                            \
    } catch (const Error& e) {                                \
        return fail(e);                                       \
    } catch (const std::exception& e) {                       \
        g_error = e.what();                                   \
        return ERR_ARG;                                       \
    }

extern "C" {

struct orc_config {
    int32_t layers, hidden, heads, kv_heads, head_dim, ff, vocab, rope_dim;
    float eps, rope_base, rope_mscale, temperature_scale;
    int32_t rope_orig_ctx, yarn_active;
};

const char* orc_last_error(void) { return g_error.c_str(); }
void orc_set_threads(int n) { g_threads = n; }
void orc_set_isa(int isa) { g_isa = isa; }
int orc_isa(void) { return use_avx512() ? 512 : 256; }
int orc_threads(void) { return thread_count(); }

int orc_open(const char* path, int initial_capacity, void** out) {
    *out = nullptr;
    ORC_TRY(*out = new Model(path, initial_capacity));
}
void orc_close(void* m) { delete (Model*)m; }

int orc_config_get(void* m, orc_config* c) {
    Model* M = (Model*)m;
    const Config& k = M->cfg;
    c->layers = k.layers; c->hidden = k.hidden; c->heads = k.heads; c->kv_heads = k.kvHeads;
    c->head_dim = k.headDim; c->ff = k.ff; c->vocab = k.vocab; c->rope_dim = k.ropeDim;
    c->eps = k.eps; c->rope_base = k.ropeBase; c->rope_mscale = M->rope->mscale;
    c->temperature_scale = k.tempScale; c->rope_orig_ctx = k.ropeOrigCtx; c->yarn_active = k.yarnActive();
    return OK;
}
int orc_rope_freqs(void* m, float* out) {
    Model* M = (Model*)m;
    std::memcpy(out, M->rope->freqs.data(), sizeof(float) * M->rope->freqs.size());
    return (int)M->rope->freqs.size();
}

// MinistralModel.ForwardAsync / PrefillAsync (MinistralModel.cs:139-157): appends tokens;
// logits (vocab floats) of the last position when compute_logits.
int orc_forward(void* m, const int32_t* tokens, int32_t n, int32_t compute_logits, float* logits, Sink sink, void* user) {
    Model* M = (Model*)m;
    ORC_TRY({
        M->forward(tokens, n, compute_logits != 0, nullptr, nullptr, 0, 0, 0, nullptr, sink, user);
        if (compute_logits && logits) std::memcpy(logits, M->logits.data(), sizeof(float) * M->cfg.vocab);
    });
}

// MinistralModel.ForwardSelectedAsync, MinistralModel.cs:165-172.
int orc_forward_selected(void* m, const int32_t* tokens, int32_t n, const int32_t* rows, int32_t n_rows, float* out) {
    Model* M = (Model*)m;
    ORC_TRY(M->forward(tokens, n, false, nullptr, rows, n_rows, 1, 1, out, nullptr, nullptr));
}

// MinistralModel.ForwardTreeAsync (:198-219) / ForwardBranchesAsync (:187) when n_trunk == 0.
// branch_tokens holds the branches back to back; out is [n_branches][n_rows], or
// [n_branches][vocab] when rows is NULL (full vocabulary at each branch's last token).
int orc_forward_tree(void* m, const int32_t* trunk, int32_t n_trunk, const int32_t* branch_tokens,
                     const int32_t* branch_lengths, int32_t n_branches, const int32_t* rows, int32_t n_rows,
                     float* out, Sink sink, void* user) {
    Model* M = (Model*)m;
    ORC_TRY({
        if (n_branches <= 0) throw Error(ERR_ARG, "No branches to forward.");
        std::vector<int> offsets(n_branches);
        int total = n_trunk;
        for (int b = 0; b < n_branches; b++) {
            if (branch_lengths[b] <= 0) throw Error(ERR_ARG, "Branch " + std::to_string(b) + " is empty.");
            offsets[b] = total;
            total += branch_lengths[b];
        }
        std::vector<int32_t> tokens(total);
        for (int i = 0; i < n_trunk; i++) tokens[i] = trunk[i];
        for (int i = n_trunk; i < total; i++) tokens[i] = branch_tokens[i - n_trunk];
        Layout L = layout_tree(M->kv->length, n_trunk, offsets, total);
        M->forward(tokens.data(), total, false, &L, rows, n_rows, rows ? 1 : 2, n_branches, out, sink, user);
    });
}

// MinistralModel.ForwardRowsAsync (:282-294): independent rows after a shared prefix.
int orc_forward_rows(void* m, int32_t shared, const int32_t* row_base, const int32_t* row_length,
                     const int32_t* row_tokens, const int32_t* row_counts, int32_t n_rowsets, const int32_t* rows,
                     int32_t n_rows, float* out) {
    Model* M = (Model*)m;
    ORC_TRY({
        std::vector<int> base(row_base, row_base + n_rowsets), len(row_length, row_length + n_rowsets),
            counts(row_counts, row_counts + n_rowsets);
        int total = 0, mx = 0;
        for (int c : counts) {
            if (c <= 0) throw Error(ERR_ARG, "Every row needs at least one token.");
            total += c;
            mx = std::max(mx, c);
        }
        Layout L = layout_rows(shared, base, len, counts, mx < 16);
        M->forward(row_tokens, total, false, &L, rows, n_rows, rows ? 1 : 2, n_rowsets, out, nullptr, nullptr);
    });
}

int32_t orc_kv_length(void* m) { return ((Model*)m)->kv->length; }
int32_t orc_kv_capacity(void* m) { return ((Model*)m)->kv->capacity; }
void orc_kv_reset(void* m) { ((Model*)m)->kv->reset(); }
void orc_kv_truncate(void* m, int32_t len) { ((Model*)m)->kv->truncate(len); }
int64_t orc_kv_snapshot_floats(void* m, int32_t len) { return ((Model*)m)->kv->snapshot_floats(len); }
int orc_kv_snapshot(void* m, int32_t len, float* out) { ORC_TRY(((Model*)m)->kv->snapshot(len, out)); }
int orc_kv_restore(void* m, const float* snap, int64_t n, int32_t len) { ORC_TRY(((Model*)m)->kv->restore(snap, n, len)); }

// ---- kernel-level restatements, for the definition tests

int orc_dequantize(uint32_t type, const uint8_t* src, float* dst, int64_t count) { ORC_TRY(dequantize(type, src, dst, count)); }
int64_t orc_row_bytes(uint32_t type, int64_t elements) {
    try { return row_bytes(type, elements); } catch (const Error& e) { g_error = e.what(); return -1; }
}
int orc_matmul(uint32_t type, const uint8_t* w, int32_t rows, int32_t cols, const float* x, int32_t tokens, float* y) {
    ORC_TRY({
        Matrix m;
        m.type = type; m.data = w; m.rows = rows; m.cols = cols; m.rowBytes = row_bytes(type, cols);
        matmul(m, x, tokens, y);
    });
}
void orc_rmsnorm(const float* x, const float* w, int32_t n, float eps, float* y) { rmsnorm(x, w, eps, y, n); }
void orc_softmax(float* x, int32_t n) { softmax(x, n); }
void orc_swiglu(const float* gate, float* up, float* dst, int32_t n) { swiglu(gate, up, dst, n); }
float orc_dot(const float* a, const float* b, int32_t n) { return dot(a, b, n); }
}
