// kernels_elem.cu — the fused elementwise kernels: RMSNorm (writing the fp16 GEMM operand
// straight into the K-slab layout), the RoPE table, RoPE + temperature + KV page write,
// SwiGLU, residual add.
#include "jv_internal.h"

namespace jv {

// --------------------------------------------------------------- RMSNorm

// Kernels.RmsNorm (reference src/Jevstral/Numerics/Kernels.cs:25-60):
//   scale = 1 / sqrt((float)(sum(x^2) / n) + eps);  y = (x * scale) * w
// The sum of squares is accumulated in double (the reference widens its two float
// accumulators to double) over a fixed thread/lane assignment and a fixed tree, so it is
// deterministic. Output goes to the fp16 K-slab operand (xs, prefill) and/or fp32 (out32,
// decode path and capture).
constexpr int NORM_THREADS = 256;

__device__ __forceinline__ double block_sum_double(double v, double* red) {
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0;
    if (threadIdx.x == 0) {
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
        red[32] = s;
    }
    __syncthreads();
    return red[32];
}

__device__ __forceinline__ void rmsnorm_row(const float* __restrict__ x, const float* __restrict__ w, int n, float eps,
                                            int t, __half* __restrict__ xs, int tpad, float* __restrict__ out32, int* err) {
    __shared__ double red[33];
    double s = 0;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        float v = x[k];
        s += (double)v * (double)v;
    }
    s = block_sum_double(s, red);
    float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(s / n), eps)));
    bool bad = false;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        float y = __fmul_rn(__fmul_rn(x[k], scale), w[k]);
        if (xs) {
            bad |= f16_out_of_range(y);
            xs[kslab_offset(t, k, tpad)] = __float2half_rn(y);
        }
        if (out32) out32[k] = y;
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) report_numeric(err, NS_RMSNORM);
}

__global__ void __launch_bounds__(NORM_THREADS) k_rmsnorm(const float* __restrict__ h, const float* __restrict__ w,
                                                           int n, float eps, __half* __restrict__ xs, int tpad,
                                                           float* __restrict__ out32, int* err) {
    int t = blockIdx.x;
    rmsnorm_row(h + (int64_t)t * n, w, n, eps, t, xs, tpad, out32 ? out32 + (int64_t)t * n : nullptr, err);
}

void launch_rmsnorm(const float* h, const float* w, int T, int n, float eps, __half* xs, int tpad, float* out32,
                    int* err, cudaStream_t s) {
    k_rmsnorm<<<T, NORM_THREADS, 0, s>>>(h, w, n, eps, xs, tpad, out32, err);
    note_launch();
}

// The prefill RMSNorm: one row per CTA, each thread holding up to RN_VEC float4 of the row
// in registers (one load pass, one store pass). With `resid`, the row is first completed
// with the split-K partials of the projection that produced it: h = h + (p0 + p1), the same
// value the one-pass epilogue computes. Sum of squares in double, per thread then a fixed
// tree, as in rmsnorm_row.
constexpr int RN_VEC = 4;
__global__ void __launch_bounds__(NORM_THREADS) k_rmsnorm_resid(float* __restrict__ h, const float* __restrict__ resid,
                                                                 const float* __restrict__ w, int n, float eps,
                                                                 __half* __restrict__ xs, int tpad, int64_t plane,
                                                                 int* err) {
    __shared__ double red[33];
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, n4 = n >> 2;
    float4* hr = (float4*)(h + (int64_t)t * n);
    const float4* p0 = resid ? (const float4*)(resid + (int64_t)t * n) : nullptr;
    const float4* p1 = resid ? (const float4*)(resid + plane + (int64_t)t * n) : nullptr;
    float4 v[RN_VEC];
    double s = 0;
#pragma unroll
    for (int j = 0; j < RN_VEC; j++) {
        const int i = threadIdx.x + j * NORM_THREADS;
        if (i < n4) {
            v[j] = hr[i];
            if (resid) {
                const float4 a = p0[i], b = p1[i];
                v[j].x = __fadd_rn(v[j].x, __fadd_rn(a.x, b.x));
                v[j].y = __fadd_rn(v[j].y, __fadd_rn(a.y, b.y));
                v[j].z = __fadd_rn(v[j].z, __fadd_rn(a.z, b.z));
                v[j].w = __fadd_rn(v[j].w, __fadd_rn(a.w, b.w));
                hr[i] = v[j];
            }
            s += (double)v[j].x * v[j].x + (double)v[j].y * v[j].y + (double)v[j].z * v[j].z + (double)v[j].w * v[j].w;
        }
    }
    s = block_sum_double(s, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(s / n), eps)));
    const float4* w4 = (const float4*)w;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < RN_VEC; j++) {
        const int i = threadIdx.x + j * NORM_THREADS;
        if (i < n4) {
            const float4 g = w4[i];
            const float y0 = __fmul_rn(__fmul_rn(v[j].x, scale), g.x), y1 = __fmul_rn(__fmul_rn(v[j].y, scale), g.y);
            const float y2 = __fmul_rn(__fmul_rn(v[j].z, scale), g.z), y3 = __fmul_rn(__fmul_rn(v[j].w, scale), g.w);
            bad |= f16_out_of_range(y0) | f16_out_of_range(y1) | f16_out_of_range(y2) | f16_out_of_range(y3);
            __half2 lo = __floats2half2_rn(y0, y1);
            __half2 hi = __floats2half2_rn(y2, y3);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&lo);
            pk.y = *reinterpret_cast<uint32_t*>(&hi);
            *(uint2*)(xs + kslab_offset(t, 4 * i, tpad)) = pk;
        }
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) report_numeric(err, NS_RMSNORM);
}

void launch_rmsnorm_resid(float* h, const float* resid, const float* w, int T, int n, float eps, __half* xs, int tpad,
                          int* err, cudaStream_t s) {
    if (n % 4 != 0 || n > 4 * RN_VEC * NORM_THREADS) throw Error(JV_ERR_UNSUPPORTED, "rmsnorm: row width");
    launch_pdl(k_rmsnorm_resid, dim3(T), dim3(NORM_THREADS), 0, s, h, resid, w, n, eps, xs, tpad, (int64_t)T * n, err);
    note_launch();
}

__global__ void k_resid_add(float* __restrict__ h, const float* __restrict__ resid, int64_t count) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) h[i] = __fadd_rn(h[i], __fadd_rn(resid[i], resid[count + i]));
}

void launch_resid_add(float* h, const float* resid, int64_t count, cudaStream_t s) {
    k_resid_add<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(h, resid, count);
    note_launch();
}

// RMSNorm of selected rows (the output rows of a tree/rows pass, MinistralModel.cs:371-373,396).
__global__ void __launch_bounds__(NORM_THREADS) k_rmsnorm_rows(const float* __restrict__ h, const int32_t* __restrict__ rows,
                                                                const float* __restrict__ w, int n, float eps,
                                                                float* __restrict__ out32, __half* __restrict__ xs, int tpad,
                                                                int* err) {
    int b = blockIdx.x;
    rmsnorm_row(h + (int64_t)rows[b] * n, w, n, eps, b, xs, tpad, out32 ? out32 + (int64_t)b * n : nullptr, err);
}

void launch_rmsnorm_rows(const float* h, const int32_t* rows, int n_rows, const float* w, int n, float eps,
                         float* out32, __half* xs, int tpad, int* err, cudaStream_t s) {
    k_rmsnorm_rows<<<n_rows, NORM_THREADS, 0, s>>>(h, rows, w, n, eps, out32, xs, tpad, err);
    note_launch();
}

// ------------------------------------------------------------------ RoPE

// Rope.Apply's per-position table (reference src/Jevstral/Model/Rope.cs:112-135):
// theta = (float)position * freq[i] in fp32, then cos/sin correctly rounded to fp32 (via
// double precision), times the magnitude scale.
__global__ void k_rope_table(float2* __restrict__ table, const float* __restrict__ freqs, int half, int pos0, int npos,
                             float mscale) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)npos * half) return;
    int p = pos0 + (int)(i / half), f = (int)(i % half);
    float theta = __fmul_rn((float)p, freqs[f]);
    double sd, cd;
    sincos((double)theta, &sd, &cd);
    table[(int64_t)p * half + f] = make_float2(__fmul_rn((float)cd, mscale), __fmul_rn((float)sd, mscale));
}

void launch_rope_table(float2* table, const float* freqs, int half, int pos0, int npos, float mscale, cudaStream_t s) {
    int64_t n = (int64_t)npos * half;
    if (n <= 0) return;
    k_rope_table<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(table, freqs, half, pos0, npos, mscale);
    note_launch();
}

// RotateQueries / StoreKeys / StoreValues / ApplyPositionScale (MinistralModel.cs:638-682):
// adjacent-pair rotation at position[t] (x0*cos - x1*sin, x0*sin + x1*cos with separate
// roundings), the llama-4 temperature on q, then q to the attention operand and k, v to
// their KV page slots as fp16. One CTA per token; each thread takes 4 consecutive elements
// (two pairs) per step, every load of the token issued up front; the token's KV page is
// looked up once.
__device__ __forceinline__ void rope_pair2(const float4 x, const float4 cs, float temp, float* r) {
    r[0] = __fsub_rn(__fmul_rn(x.x, cs.x), __fmul_rn(x.y, cs.y));
    r[1] = __fadd_rn(__fmul_rn(x.x, cs.y), __fmul_rn(x.y, cs.x));
    r[2] = __fsub_rn(__fmul_rn(x.z, cs.z), __fmul_rn(x.w, cs.w));
    r[3] = __fadd_rn(__fmul_rn(x.z, cs.w), __fmul_rn(x.w, cs.z));
    if (temp != 1.0f)
        for (int e = 0; e < 4; e++) r[e] = __fmul_rn(r[e], temp);
}

__global__ void __launch_bounds__(256) k_rope_kv(RopeArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x;
    const int hd = a.head_dim, half = hd / 2;
    const int qdim = a.heads * hd, kvdim = a.kv_heads * hd;
    const int pos = a.pos[t], slot = a.slot[t];
    const float* row = a.qkv + (int64_t)t * (qdim + 2 * kvdim);
    const float4* tab4 = (const float4*)(a.table + (int64_t)pos * half);  // two (cos, sin) pairs each
    const float temp = rope_temperature(pos, a.orig_ctx, a.temperature_scale);
    // K plane of (layer, kv head 0) in this token's page; heads and V are fixed plane offsets,
    // the slot's row inside a plane is swizzled (kv_elem_offset)
    const int page = kv_page(a.page_table, slot, a.page_slots, a.err, BS_ROPE_PAGE), row_in_page = slot % a.page_slots;
    char* kv0 = (char*)a.kv_pool + (int64_t)page * a.page_bytes + kv_plane_offset(a.layer, a.kv_heads, 0, 0, a.page_slots);
    const int64_t head_stride = (int64_t)2 * a.page_slots * 256, v_off = (int64_t)a.page_slots * 256;
    const int nq4 = qdim / 4, nk4 = kvdim / 4;
    bool bad = false;
    for (int i = threadIdx.x; i < nq4 + 2 * nk4; i += blockDim.x) {
        const float4 x = *(const float4*)(row + 4 * i);
        if (i < nq4 + nk4) {
            const int e = 4 * i;  // q, then k
            const int d = e % hd;
            const float4 cs = tab4[d / 4];
            float r[4];
            rope_pair2(x, cs, i < nq4 ? temp : 1.0f, r);
            if (i >= nq4 || a.q16)
                bad |= f16_out_of_range(r[0]) | f16_out_of_range(r[1]) | f16_out_of_range(r[2]) | f16_out_of_range(r[3]);
            if (i < nq4) {
                if (a.q16) {
                    __half2 lo = __floats2half2_rn(r[0], r[1]), hi = __floats2half2_rn(r[2], r[3]);
                    uint2 pk;
                    pk.x = *reinterpret_cast<uint32_t*>(&lo);
                    pk.y = *reinterpret_cast<uint32_t*>(&hi);
                    *(uint2*)(a.q16 + (int64_t)t * qdim + e) = pk;
                }
                if (a.q32) *(float4*)(a.q32 + (int64_t)t * qdim + e) = make_float4(r[0], r[1], r[2], r[3]);
            } else {
                const int ke = e - qdim, head = ke / hd;
                __half2* dst = (__half2*)(kv0 + head * head_stride + kv_elem_offset(row_in_page, d, a.page_slots));
                dst[0] = __floats2half2_rn(r[0], r[1]);
                dst[1] = __floats2half2_rn(r[2], r[3]);
                if (a.k32) *(float4*)(a.k32 + (int64_t)t * kvdim + ke) = make_float4(r[0], r[1], r[2], r[3]);
            }
        } else {  // v: straight copy to its slot
            const int ve = 4 * i - qdim - kvdim, head = ve / hd, d = ve % hd;
            bad |= f16_out_of_range(x.x) | f16_out_of_range(x.y) | f16_out_of_range(x.z) | f16_out_of_range(x.w);
            __half2* dst = (__half2*)(kv0 + head * head_stride + v_off + kv_elem_offset(row_in_page, d, a.page_slots));
            dst[0] = __floats2half2_rn(x.x, x.y);
            dst[1] = __floats2half2_rn(x.z, x.w);
        }
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) report_numeric(a.err, NS_ROPE_KV);
}

void launch_rope_kv(const RopeArgs& a, cudaStream_t s) {
    if (a.head_dim % 4 != 0) throw Error(JV_ERR_UNSUPPORTED, "rope: head_dim must be a multiple of 4");
    launch_pdl(k_rope_kv, dim3(a.T), dim3(256), 0, s, a);
    note_launch();
}

// ---------------------------------------------------------------- SwiGLU

// Kernels.SwiGlu (Kernels.cs:82-89): up <- g*u; dst <- 1/(1+exp(-g)); dst <- dst*up.
// gu holds the fused gate/up product: feature j = 64i + w sits in row tile i, gate at
// column 128i + 32*(w/16) + w%16 and up 16 columns further.
__global__ void k_swiglu(const float* __restrict__ gu, int ff, __half* __restrict__ xs, int tpad, float* __restrict__ out32,
                         int* err) {
    int t = blockIdx.x;
    const float* row = gu + (int64_t)t * 2 * ff;
    bool bad = false;
    for (int j = threadIdx.x; j < ff; j += blockDim.x) {
        int w = j & 63;
        int col = (j >> 6) * 128 + (w >> 4) * 32 + (w & 15);
        float g = row[col], u = row[col + 16];
        float up = __fmul_rn(g, u);
        float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
        float y = __fmul_rn(sg, up);
        if (xs) {
            bad |= f16_out_of_range(y);
            xs[kslab_offset(t, j, tpad)] = __float2half_rn(y);
        }
        if (out32) out32[(int64_t)t * ff + j] = y;
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) report_numeric(err, NS_SWIGLU);
}

void launch_swiglu(const float* gu, int T, int ff, __half* xs, int tpad, float* out32, int* err, cudaStream_t s) {
    k_swiglu<<<T, 256, 0, s>>>(gu, ff, xs, tpad, out32, err);
    note_launch();
}

// ------------------------------------------------------------ residual add

// Kernels.Add (Kernels.cs:63): h += x.
__global__ void k_add(float* __restrict__ h, const float* __restrict__ x, int64_t n) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) h[i] = __fadd_rn(h[i], x[i]);
}

void launch_add(float* h, const float* x, int64_t n, cudaStream_t s) {
    k_add<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(h, x, n);
    note_launch();
}

// K-slab fp16 -> plain fp32 [T][K] (activation capture only).
__global__ void k_kslab_to_f32(const __half* __restrict__ xs, int T, int K, int tpad, float* __restrict__ out) {
    int t = blockIdx.x;
    for (int k = threadIdx.x; k < K; k += blockDim.x) out[(int64_t)t * K + k] = __half2float(xs[kslab_offset(t, k, tpad)]);
}

void launch_kslab_to_f32(const __half* xs, int T, int K, int tpad, float* out, cudaStream_t s) {
    k_kslab_to_f32<<<T, 256, 0, s>>>(xs, T, K, tpad, out);
    note_launch();
}

}  // namespace jv

namespace jv {

// KvCache.Snapshot / Restore layout (reference src/Jevstral/Model/KvCache.cs:94-136):
// [pass: K then V][layer][kv head][position < len][128] fp32.
__global__ void k_kv_export(const __half* __restrict__ pool, const int32_t* __restrict__ page_table, int64_t page_bytes,
                            int page_slots, int layers, int kv_heads, int len, float* __restrict__ out, int64_t base,
                            int64_t count, int* err) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < count; j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = base + j;
        int d = (int)(i % 128);
        int64_t r = i / 128;
        int p = (int)(r % len);
        r /= len;
        int h = (int)(r % kv_heads);
        r /= kv_heads;
        int l = (int)(r % layers);
        int kv = (int)(r / layers);
        int page = kv_page(page_table, p, page_slots, err, BS_SNAPSHOT_PAGE);
        const __half* src = (const __half*)((const char*)pool + (int64_t)page * page_bytes +
                                             kv_plane_offset(l, kv_heads, h, kv, page_slots) +
                                             kv_elem_offset(p % page_slots, d, page_slots));
        out[j] = __half2float(*src);
    }
}

__global__ void k_kv_import(__half* __restrict__ pool, const int32_t* __restrict__ page_table, int64_t page_bytes,
                            int page_slots, int layers, int kv_heads, int len, const float* __restrict__ in, int* err,
                            int64_t base, int64_t count) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < count; j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = base + j;
        int d = (int)(i % 128);
        int64_t r = i / 128;
        int p = (int)(r % len);
        r /= len;
        int h = (int)(r % kv_heads);
        r /= kv_heads;
        int l = (int)(r % layers);
        int kv = (int)(r / layers);
        int page = kv_page(page_table, p, page_slots, err, BS_SNAPSHOT_PAGE);
        __half* dst = (__half*)((char*)pool + (int64_t)page * page_bytes + kv_plane_offset(l, kv_heads, h, kv, page_slots) +
                                kv_elem_offset(p % page_slots, d, page_slots));
        const float v = in[j];
        if (f16_out_of_range(v)) report_numeric(err, NS_KV_RESTORE);
        *dst = __float2half_rn(v);
    }
}

void launch_kv_export(const __half* pool, const int32_t* page_table, int64_t page_bytes, int page_slots, int layers,
                      int kv_heads, int len, float* out, cudaStream_t s, int64_t base, int64_t count, int* err) {
    if (len <= 0) return;
    if (count <= 0) count = (int64_t)2 * layers * kv_heads * len * 128 - base;
    k_kv_export<<<1024, 256, 0, s>>>(pool, page_table, page_bytes, page_slots, layers, kv_heads, len, out, base, count,
                                     err);
    note_launch();
}
void launch_kv_import(__half* pool, const int32_t* page_table, int64_t page_bytes, int page_slots, int layers,
                      int kv_heads, int len, const float* in, int* err, cudaStream_t s, int64_t base, int64_t count) {
    if (len <= 0) return;
    if (count <= 0) count = (int64_t)2 * layers * kv_heads * len * 128 - base;
    k_kv_import<<<1024, 256, 0, s>>>(pool, page_table, page_bytes, page_slots, layers, kv_heads, len, in, err, base, count);
    note_launch();
}

}  // namespace jv
