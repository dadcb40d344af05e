// decode_common.cuh — device helpers of the single-token kernels (kernels_decode.cu): the
// tensor-core dequant-matvec fragments, mbarrier / bulk-copy / cp.async wrappers, and small
// reductions.
#pragma once

#include "jv_internal.h"

namespace jv {
namespace {

constexpr int DG_THREADS = 256;  // 8 warps x 16 rows = one 128-row tile
constexpr int DG_UNROLL = 4;     // k steps whose raw words are loaded before any is used

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// Bytes of x picked by the byte_perm selector as the fp16 pair (1024 + b0, 1024 + b1), minus
// `bias` (exact: every operand is an integer below 2048).
__device__ __forceinline__ uint32_t int_pair(uint32_t x, uint32_t sel, __half2 bias) {
    uint32_t w = __byte_perm(x, 0x64646464u, sel);
    __half2 h = __hsub2(*reinterpret_cast<__half2*>(&w), bias);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Fifth bits of four elements (bits 0-3 of h) into bit 4 of each byte.
__device__ __forceinline__ uint32_t spread4(uint32_t h) {
    return ((h & 1u) << 4) | ((h & 2u) << 11) | ((h & 4u) << 18) | ((h & 8u) << 25);
}

// The raw words one lane needs for one k step: rows r (g) and r + 8 (h), blocks 0 and 1.
template <int TYPE>
struct Raw {
    uint32_t q[2][2][TYPE == T_Q8_0 ? 2 : 1];  // [row][block][word]
    uint32_t d[2];                             // fp16 d of blocks 0,1 per row
    uint32_t qh[2][2];                         // Q5_1: fifth bits per row and block
    uint32_t m[2];                             // Q5_1: fp16 m of blocks 0,1 per row
};

template <int TYPE>
__device__ __forceinline__ void load_raw(Raw<TYPE>& r, const uint8_t* __restrict__ chunk, int row, int kq) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int rr = row + 8 * h;
#pragma unroll
        for (int b = 0; b < 2; b++) {
            if (TYPE == T_Q8_0) {
                uint2 v = *(const uint2*)(chunk + rr * 64 + 32 * b + 8 * kq);
                r.q[h][b][0] = v.x;
                r.q[h][b][TYPE == T_Q8_0 ? 1 : 0] = v.y;
            } else {
                r.q[h][b][0] = *(const uint32_t*)(chunk + rr * 32 + 16 * b + 4 * kq);
            }
        }
        r.d[h] = *(const uint32_t*)(chunk + qs_bytes(TYPE) + (TYPE == T_Q5_1 ? 1024 : 0) + rr * 4);
        if (TYPE == T_Q5_1) {
            uint2 v = *(const uint2*)(chunk + 4096 + rr * 8);
            r.qh[h][0] = v.x;
            r.qh[h][1] = v.y;
            r.m[h] = *(const uint32_t*)(chunk + 5632 + rr * 4);
        }
    }
}

// A fragments of the two MMAs (sub = 0, 1) of block b: regs {row g k lo, row h k lo, row g
// k hi, row h k hi} as the m16n8k16 row-major A layout wants them.
template <int TYPE>
__device__ __forceinline__ void a_frags(const Raw<TYPE>& r, int b, int kq, uint32_t (&a)[2][4]) {
    if (TYPE == T_Q8_0) {
        const __half2 bias = __floats2half2_rn(1152.f, 1152.f);  // 1024 + 128: biased int8
#pragma unroll
        for (int h = 0; h < 2; h++) {
#pragma unroll
            for (int s = 0; s < 2; s++) {
                uint32_t x = r.q[h][b][s & (TYPE == T_Q8_0 ? 1 : 0)] ^ 0x80808080u;
                a[s][h] = int_pair(x, 0x4140u, bias);
                a[s][2 + h] = int_pair(x, 0x4342u, bias);
            }
        }
    } else {
        const __half2 bias = TYPE == T_Q4_0 ? __floats2half2_rn(1032.f, 1032.f) : __floats2half2_rn(1024.f, 1024.f);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint32_t q = r.q[h][b][0];
            uint32_t lo = q & 0x0F0F0F0Fu, hi = (q >> 4) & 0x0F0F0F0Fu;
            if (TYPE == T_Q5_1) {
                lo |= spread4((r.qh[h][b] >> (4 * kq)) & 0xFu);
                hi |= spread4((r.qh[h][b] >> (16 + 4 * kq)) & 0xFu);
            }
            a[0][h] = int_pair(lo, 0x4140u, bias);
            a[0][2 + h] = int_pair(lo, 0x4342u, bias);
            a[1][h] = int_pair(hi, 0x4140u, bias);
            a[1][2 + h] = int_pair(hi, 0x4342u, bias);
        }
    }
}

// First element (within a k step) of the four consecutive x values lane kq feeds to MMA
// (b, sub); the A side above holds the weights of exactly those elements.
template <int TYPE>
__device__ __forceinline__ int x_base(int b, int sub, int kq) {
    return TYPE == T_Q8_0 ? 32 * b + 8 * kq + 4 * sub : 32 * b + 16 * sub + 4 * kq;
}

__device__ __forceinline__ float half_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
__device__ __forceinline__ float half_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

__device__ __forceinline__ double block_sum_d(double v, double* red) {
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
        red[32] = s;
    }
    __syncthreads();
    return red[32];
}


__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void dg_mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void dg_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void dg_mbar_arrive_local(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void dg_bulk(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ bool dg_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}
// Bounded wait for phase `parity` of an mbarrier; false if it never completed within 4e9 SM
// clock cycles (about 2 s at the maximum clock). The SM's cycle counter only moves forward,
// unlike %globaltimer, which the driver may step.
__device__ __forceinline__ bool dg_wait(uint32_t bar, uint32_t parity) {
    if (dg_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!dg_try(bar, parity))
        if (clock64() - t0 > 4000000000ll) return false;
    return true;
}
// This CTA's share of an L2 prefetch of [pf, pf + bytes) (bytes a multiple of 16) split evenly
// over the grid's CTAs: pieces of at most 64 KB, issued by the calling thread; nothing waits for
// them. A later kernel of the step then finds its weights in L2 instead of HBM, while HBM keeps
// streaming across the boundaries between launches.
__device__ __forceinline__ void dg_prefetch_share(const uint8_t* pf, int64_t bytes) {
    if (!pf || bytes <= 0) return;
    const int64_t ncta = (int64_t)gridDim.x * gridDim.y;
    const int64_t cta = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
    const int64_t share = ((bytes + ncta - 1) / ncta + 15) & ~(int64_t)15;
    const int64_t b1 = min(bytes, (cta + 1) * share);
    for (int64_t o = cta * share; o < b1; o += 65536) {
        const uint32_t n = (uint32_t)min((int64_t)65536, b1 - o);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(pf + o), "r"(n) : "memory");
    }
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Kernels.ArgMax / IndexOfMax order: the larger value, the first index on ties, a NaN wins.
__device__ __forceinline__ bool dec_better(float v, int i, float bv, int bi) {
    bool vn = v != v, bn = bv != bv;
    if (vn || bn) {
        if (vn && bn) return i < bi;
        return vn;
    }
    return v > bv || (v == bv && i < bi);
}

// The (layer, head, K|V) plane of the page holding `slot` (rows inside it are swizzled: see
// kv_chunk_offset / kv_elem_offset).
__device__ __forceinline__ char* kv_plane(__half* pool, const int32_t* page_table, int64_t page_bytes, int page_slots,
                                          int layer, int kv_heads, int head, int kv, int slot, int* err) {
    return (char*)pool + (int64_t)kv_page(page_table, slot, page_slots, err, BS_DECODE_PAGE) * page_bytes +
           kv_plane_offset(layer, kv_heads, head, kv, page_slots);
}

}  // namespace
}  // namespace jv
