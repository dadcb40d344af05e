// kernels_quant.cu — kernels that read quantized weights with CUDA cores: weight re-tiling,
// embedding gather, the decode dequant-GEMV, the verdict-row head and argmax.
//
// Dequantization here is bit-exact with the reference (src/Jevstral/Quantization/
// Dequantizer.cs:155-305): Q8_0 d*q, Q4_0 d*(n-8), Q5_1 d*q5 + m, each a single
// IEEE-rounded multiply (then add), written with __fmul_rn/__fadd_rn so nvcc cannot
// contract them into an FMA.
#include "jv_internal.h"

#include <atomic>
#include <cstdlib>
#include <string>

namespace jv {

static std::atomic<int64_t> g_launches{0};
void note_launch(int n) { g_launches += n; }
int64_t launches_total() { return g_launches.load(); }

bool debug_sync_enabled() {
    static const bool on = getenv("JV_DEBUG_SYNC") != nullptr;
    return on;
}
void debug_after_launch(cudaStream_t s, const void* kernel) {
    static thread_local std::string prev = "(none)";
    const char* name = nullptr;
    if (cudaFuncGetName(&name, kernel) != cudaSuccess || name == nullptr) {
        cudaGetLastError();
        name = "(unnamed kernel)";
    }
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &st) == cudaSuccess && st == cudaStreamCaptureStatusNone) {
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess)
            throw Error(JV_ERR_DEVICE, std::string("after ") + name + " (the programmatic-dependent launch before it: " + prev +
                                           "): " + cudaGetErrorString(e));
    }
    prev = name;
}

// ------------------------------------------------------------- re-tiling

// raw: `rows` GGUF rows of `cols` elements (raw_row_bytes each). Row j goes to
//   interleave == 0: tile tile_offset + j/128, row-in-tile j%128
//   interleave != 0: tile j/64; within the tile, 16-row groups alternate gate and up
//                    (gate rows at 32*(w/16) + w%16, up rows 16 further, w = j%64), so a
//                    warp's lanes l and l+16 hold the gate and up row of one FFN feature.
//                    row_in_tile_base is 0 for the gate matrix and 16 for the up matrix.
__global__ void k_repack(const uint8_t* __restrict__ raw, int type, int rows, int cols, int64_t raw_row_bytes,
                         uint8_t* __restrict__ dst, int ksteps, int row_in_tile_base, int tile_offset,
                         int interleave) {
    const int unit = type == T_QX ? 64 : 32;  // QX rows come in 96-byte units of 64 columns
    int blocks_per_row = cols / unit;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)rows * blocks_per_row) return;
    int j = (int)(idx / blocks_per_row), b = (int)(idx % blocks_per_row);
    int tile, rit;
    if (interleave) {
        tile = j / 64;
        int w = j % 64;
        rit = (w >> 4) * 32 + (w & 15) + row_in_tile_base;
    } else {
        tile = tile_offset + j / 128;
        rit = j % 128;
    }
    int ks = type == T_QX ? b : b >> 1, half = b & 1;
    uint8_t* chunk = dst + ((int64_t)tile * ksteps + ks) * chunk_bytes(type);
    const uint8_t* src = raw + (int64_t)j * raw_row_bytes;
    if (type == T_QX) {  // 64 q, 4 a, 4 c of one 64-column unit
        src += (int64_t)b * 96;
        for (int i = 0; i < 64; i++) chunk[rit * 64 + i] = src[i];
        for (int i = 0; i < 16; i++) chunk[8192 + rit * 16 + i] = src[64 + i];
        for (int i = 0; i < 16; i++) chunk[10240 + rit * 16 + i] = src[80 + i];
    } else if (type == T_Q8_0) {
        src += (int64_t)b * 34;
        for (int i = 0; i < 32; i++) chunk[rit * 64 + half * 32 + i] = src[2 + i];
        chunk[8192 + (rit * 2 + half) * 2] = src[0];
        chunk[8192 + (rit * 2 + half) * 2 + 1] = src[1];
    } else if (type == T_Q4_0) {
        src += (int64_t)b * 18;
        for (int i = 0; i < 16; i++) chunk[rit * 32 + half * 16 + i] = src[2 + i];
        chunk[4096 + (rit * 2 + half) * 2] = src[0];
        chunk[4096 + (rit * 2 + half) * 2 + 1] = src[1];
    } else {  // Q5_1: d m qh qs
        src += (int64_t)b * 24;
        for (int i = 0; i < 16; i++) chunk[rit * 32 + half * 16 + i] = src[8 + i];
        for (int i = 0; i < 4; i++) chunk[4096 + (rit * 2 + half) * 4 + i] = src[4 + i];
        chunk[5120 + (rit * 2 + half) * 2] = src[0];
        chunk[5120 + (rit * 2 + half) * 2 + 1] = src[1];
        chunk[5632 + (rit * 2 + half) * 2] = src[2];
        chunk[5632 + (rit * 2 + half) * 2 + 1] = src[3];
    }
}

void launch_repack(const uint8_t* raw, int type, int rows, int cols, int64_t raw_row_bytes, uint8_t* dst,
                   int dst_tiles, int ksteps, int row_in_tile_base, int tile_offset, int interleave,
                   cudaStream_t s) {
    (void)dst_tiles;
    int64_t n = (int64_t)rows * (cols / (type == T_QX ? 64 : 32));
    int threads = 256;
    int64_t grid = (n + threads - 1) / threads;
    k_repack<<<(unsigned)grid, threads, 0, s>>>(raw, type, rows, cols, raw_row_bytes, dst, ksteps, row_in_tile_base,
                                                tile_offset, interleave);
    note_launch();
}

// ---------------------------------------------------------- element decode

__device__ __forceinline__ float dq_element(const uint8_t* __restrict__ data, int type, int ksteps, int r, int k) {
    int tile = r >> 7, rit = r & 127, ks = k >> 6, kk = k & 63, half = kk >> 5, e = kk & 31;
    const uint8_t* chunk = data + ((int64_t)tile * ksteps + ks) * chunk_bytes(type);
    if (type == T_QX) {
        const float a = *(const float*)(chunk + 8192 + (rit * 4 + (kk >> 4)) * 4);
        const float c = *(const float*)(chunk + 10240 + (rit * 4 + (kk >> 4)) * 4);
        return __fadd_rn(__fmul_rn(a, (float)(int8_t)chunk[rit * 64 + kk]), c);
    }
    if (type == T_Q8_0) {
        float d = __half2float(*(const __half*)(chunk + 8192 + (rit * 2 + half) * 2));
        return __fmul_rn(d, (float)(int8_t)chunk[rit * 64 + kk]);
    }
    uint8_t byte = chunk[rit * 32 + half * 16 + (e & 15)];
    int nib = e < 16 ? (byte & 15) : (byte >> 4);
    if (type == T_Q4_0) {
        float d = __half2float(*(const __half*)(chunk + 4096 + (rit * 2 + half) * 2));
        return __fmul_rn(d, (float)(nib - 8));
    }
    uint32_t qh = *(const uint32_t*)(chunk + 4096 + (rit * 2 + half) * 4);
    int q = nib | (int)(((qh >> e) & 1u) << 4);
    float d = __half2float(*(const __half*)(chunk + 5120 + (rit * 2 + half) * 2));
    float m = __half2float(*(const __half*)(chunk + 5632 + (rit * 2 + half) * 2));
    return __fadd_rn(__fmul_rn(d, (float)q), m);
}

// QuantMatMul.GatherRows (reference src/Jevstral/Numerics/QuantMatMul.cs:294-305): decode the
// referenced rows of the embedding table. The host validates ids; an id out of range here
// only sets the error word.
__global__ void k_embed(const uint8_t* __restrict__ data, int type, int ksteps, int vocab, const int32_t* __restrict__ ids,
                        float* __restrict__ h, int hidden, int* err) {
    int t = blockIdx.x;
    int id = ids[t];
    if ((unsigned)id >= (unsigned)vocab) {
        if (threadIdx.x == 0 && blockIdx.y == 0) atomicExch(err, JV_ERR_RANGE);
        return;
    }
    for (int k = blockIdx.y * blockDim.x + threadIdx.x; k < hidden; k += gridDim.y * blockDim.x)
        h[(int64_t)t * hidden + k] = dq_element(data, type, ksteps, id, k);
}

void launch_embed(const QWeight& table, const int32_t* ids, int T, float* h, int hidden, int* err, cudaStream_t s) {
    // a single row gets one CTA per 256 elements; many rows, one CTA each
    dim3 grid(T, T < 16 ? (hidden + 255) / 256 : 1);
    k_embed<<<grid, 256, 0, s>>>(table.data, table.type, table.ksteps, table.rows, ids, h, hidden, err);
    note_launch();
}

// ----------------------------------------------------------------- GEMV

// The decode matvec (QuantMatMul.RunRowsFloat, QuantMatMul.cs:140-176): y = W x with the
// weights decoded to fp32 exactly as the reference decodes them and fp32 fused
// multiply-adds. HBM-bound: each CTA streams one 128-row tile over a contiguous range of
// k steps with 128-bit loads; thread i owns row i/2 and 32-element block i%2 of every
// chunk. Partial sums per k-range go to `partial[split][n]` and are added in split order
// by k_gemv_reduce, so the result never depends on scheduling.
constexpr int GEMV_THREADS = 256;
constexpr int GEMV_UNROLL = 4;

template <int TYPE>
__device__ __forceinline__ float gemv_chunk(const uint8_t* __restrict__ chunk, const float* __restrict__ xs, int rit,
                                           int half, float acc) {
    if (TYPE == T_QX) {
        const int4* q = (const int4*)(chunk + rit * 64 + half * 32);
        int4 qa = __ldg(q), qb = __ldg(q + 1);
        const float2 a = __ldg((const float2*)(chunk + 8192 + (rit * 4 + half * 2) * 4));
        const float2 c = __ldg((const float2*)(chunk + 10240 + (rit * 4 + half * 2) * 4));
        const int8_t* p0 = (const int8_t*)&qa;
        const int8_t* p1 = (const int8_t*)&qb;
#pragma unroll
        for (int i = 0; i < 16; i++) acc = fmaf(xs[i], __fadd_rn(__fmul_rn(a.x, (float)p0[i]), c.x), acc);
#pragma unroll
        for (int i = 0; i < 16; i++) acc = fmaf(xs[16 + i], __fadd_rn(__fmul_rn(a.y, (float)p1[i]), c.y), acc);
        return acc;
    } else if (TYPE == T_Q8_0) {
        const int4* q = (const int4*)(chunk + rit * 64 + half * 32);
        int4 a = __ldg(q), b = __ldg(q + 1);
        float d = __half2float(__ldg((const __half*)(chunk + 8192 + (rit * 2 + half) * 2)));
        const int8_t* qa = (const int8_t*)&a;
        const int8_t* qb = (const int8_t*)&b;
#pragma unroll
        for (int i = 0; i < 16; i++) acc = fmaf(xs[i], __fmul_rn(d, (float)qa[i]), acc);
#pragma unroll
        for (int i = 0; i < 16; i++) acc = fmaf(xs[16 + i], __fmul_rn(d, (float)qb[i]), acc);
        return acc;
    } else if (TYPE == T_Q4_0) {
        int4 a = __ldg((const int4*)(chunk + rit * 32 + half * 16));
        float d = __half2float(__ldg((const __half*)(chunk + 4096 + (rit * 2 + half) * 2)));
        const uint8_t* qa = (const uint8_t*)&a;
#pragma unroll
        for (int i = 0; i < 16; i++) acc = fmaf(xs[i], __fmul_rn(d, (float)((qa[i] & 15) - 8)), acc);
#pragma unroll
        for (int i = 0; i < 16; i++) acc = fmaf(xs[16 + i], __fmul_rn(d, (float)((qa[i] >> 4) - 8)), acc);
        return acc;
    } else {
        int4 a = __ldg((const int4*)(chunk + rit * 32 + half * 16));
        uint32_t qh = __ldg((const uint32_t*)(chunk + 4096 + (rit * 2 + half) * 4));
        float d = __half2float(__ldg((const __half*)(chunk + 5120 + (rit * 2 + half) * 2)));
        float m = __half2float(__ldg((const __half*)(chunk + 5632 + (rit * 2 + half) * 2)));
        const uint8_t* qa = (const uint8_t*)&a;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            int q = (qa[i] & 15) | (int)(((qh >> i) & 1u) << 4);
            acc = fmaf(xs[i], __fadd_rn(__fmul_rn(d, (float)q), m), acc);
        }
#pragma unroll
        for (int i = 0; i < 16; i++) {
            int q = (qa[i] >> 4) | (int)(((qh >> (i + 16)) & 1u) << 4);
            acc = fmaf(xs[16 + i], __fadd_rn(__fmul_rn(d, (float)q), m), acc);
        }
        return acc;
    }
}

template <int TYPE>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(const uint8_t* __restrict__ data, int ksteps, int n_rows,
                                                        const float* __restrict__ x, float* __restrict__ partial,
                                                        int splits) {
    extern __shared__ float xs_all[];
    int tile = blockIdx.x, split = blockIdx.y;
    int per = (ksteps + splits - 1) / splits;
    int ks0 = split * per, ks1 = min(ksteps, ks0 + per);
    int nk = max(0, ks1 - ks0);
    for (int i = threadIdx.x; i < nk * 64; i += blockDim.x) xs_all[i] = x[(int64_t)ks0 * 64 + i];
    __syncthreads();
    int rit = threadIdx.x >> 1, half = threadIdx.x & 1;
    const int cb = chunk_bytes(TYPE);
    const uint8_t* base = data + ((int64_t)tile * ksteps + ks0) * cb;
    float acc = 0.f;
    int ks = 0;
    for (; ks + GEMV_UNROLL <= nk; ks += GEMV_UNROLL) {
#pragma unroll
        for (int u = 0; u < GEMV_UNROLL; u++)
            acc = gemv_chunk<TYPE>(base + (int64_t)(ks + u) * cb, xs_all + (ks + u) * 64 + half * 32, rit, half, acc);
    }
    for (; ks < nk; ks++) acc = gemv_chunk<TYPE>(base + (int64_t)ks * cb, xs_all + ks * 64 + half * 32, rit, half, acc);
    float other = __shfl_xor_sync(0xffffffffu, acc, 1);
    if (half == 0) {
        float total = acc + other;
        int n = tile * 128 + rit;
        if (n < n_rows) partial[(int64_t)split * n_rows + n] = total;
    }
}

int gemv_splits_for(const QWeight& w, int sm_count) {
    int want = (3 * sm_count + w.tiles - 1) / w.tiles;  // about three CTAs per SM
    want = want < 1 ? 1 : want;
    int maxs = (w.ksteps + 3) / 4;                       // keep >= 4 k steps per CTA
    if (maxs < 1) maxs = 1;
    return want < maxs ? want : maxs;
}

void launch_gemv(const QWeight& w, const float* x, float* partial, int splits, cudaStream_t s) {
    dim3 grid(w.tiles, splits);
    int per = (w.ksteps + splits - 1) / splits;
    size_t smem = (size_t)per * 64 * sizeof(float);
    if (smem > 227 * 1024) throw Error(JV_ERR_UNSUPPORTED, "gemv: the activation slice does not fit in shared memory");
    if (w.type == T_Q8_0) {
        if (smem > 48 * 1024)
            JV_CUDA(cudaFuncSetAttribute(k_gemv<T_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_gemv<T_Q8_0><<<grid, GEMV_THREADS, smem, s>>>(w.data, w.ksteps, w.rows, x, partial, splits);
    } else if (w.type == T_Q4_0) {
        if (smem > 48 * 1024)
            JV_CUDA(cudaFuncSetAttribute(k_gemv<T_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_gemv<T_Q4_0><<<grid, GEMV_THREADS, smem, s>>>(w.data, w.ksteps, w.rows, x, partial, splits);
    } else if (w.type == T_QX) {
        if (smem > 48 * 1024)
            JV_CUDA(cudaFuncSetAttribute(k_gemv<T_QX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_gemv<T_QX><<<grid, GEMV_THREADS, smem, s>>>(w.data, w.ksteps, w.rows, x, partial, splits);
    } else {
        if (smem > 48 * 1024)
            JV_CUDA(cudaFuncSetAttribute(k_gemv<T_Q5_1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_gemv<T_Q5_1><<<grid, GEMV_THREADS, smem, s>>>(w.data, w.ksteps, w.rows, x, partial, splits);
    }
    note_launch();
}

__global__ void k_gemv_reduce(const float* __restrict__ partial, int splits, int n, float* __restrict__ y, int epilogue) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float s = 0.f;
    for (int p = 0; p < splits; p++) s += partial[(int64_t)p * n + i];
    if (epilogue == EPI_ADD)
        y[i] = y[i] + s;
    else
        y[i] = s;
}

void launch_gemv_reduce(const float* partial, int splits, int n, float* y, int epilogue, cudaStream_t s) {
    k_gemv_reduce<<<(n + 255) / 256, 256, 0, s>>>(partial, splits, n, y, epilogue);
    note_launch();
}

// ------------------------------------------------------------ verdict head

// The selected-rows head (MinistralModel.cs:386-410): for output b and vocab row r,
// logit = Dot(rmsnorm(h[out_b]), dequant(E[r])). One warp per (b, r) pair; lane l takes
// every 32nd element and the lanes are folded with a fixed shuffle tree.
__global__ void k_head_rows(const uint8_t* __restrict__ data, int type, int ksteps, int vocab,
                            const float* __restrict__ normed, int hidden, int n_out, const int32_t* __restrict__ rows,
                            int n_rows, float* __restrict__ out, int* err) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= n_out * n_rows) return;
    int b = warp / n_rows, i = warp % n_rows;
    int r = rows[i];
    if ((unsigned)r >= (unsigned)vocab) {
        if (lane == 0) atomicExch(err, JV_ERR_RANGE);
        return;
    }
    const float* nv = normed + (int64_t)b * hidden;
    float acc = 0.f;
    for (int k = lane; k < hidden; k += 32) acc = fmaf(nv[k], dq_element(data, type, ksteps, r, k), acc);
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[(int64_t)b * n_rows + i] = acc;
}

void launch_head_rows(const QWeight& table, const float* normed, int n_out, const int32_t* rows, int n_rows,
                      float* out, int* err, cudaStream_t s) {
    int warps = n_out * n_rows;
    int threads = 128;
    int grid = (warps * 32 + threads - 1) / threads;
    k_head_rows<<<grid, threads, 0, s>>>(table.data, table.type, table.ksteps, table.rows, normed, table.cols, n_out,
                                         rows, n_rows, out, err);
    note_launch();
}

// ------------------------------------------------------------------ argmax

// Kernels.ArgMax / TensorPrimitives.IndexOfMax (Kernels.cs:146): the first index of the
// largest value; a NaN wins at its first index.
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
    bool vn = v != v, bn = bv != bv;
    if (vn || bn) {
        if (vn && bn) return i < bi;
        return vn;
    }
    return v > bv || (v == bv && i < bi);
}

__global__ void k_argmax(const float* __restrict__ x, int n, int32_t* out) {
    __shared__ float sv[1024];
    __shared__ int si[1024];
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        if (am_better(x[i], i, bv, bi)) { bv = x[i]; bi = i; }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int w = blockDim.x / 2; w >= 1; w >>= 1) {
        if ((int)threadIdx.x < w && am_better(sv[threadIdx.x + w], si[threadIdx.x + w], sv[threadIdx.x], si[threadIdx.x])) {
            sv[threadIdx.x] = sv[threadIdx.x + w];
            si[threadIdx.x] = si[threadIdx.x + w];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) *out = si[0] == 0x7fffffff ? 0 : si[0];
}

void launch_argmax(const float* x, int n, int32_t* out, cudaStream_t s) {
    k_argmax<<<1, 1024, 0, s>>>(x, n, out);
    note_launch();
}

}  // namespace jv
