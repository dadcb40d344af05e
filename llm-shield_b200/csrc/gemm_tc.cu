// gemm_tc.cu — the prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Y[t, n] (+)= sum_k X[t, k] * W[n, k]: the reference's PanelGemm (src/Jevstral/Numerics/
// PanelGemm.cs:76-300), with W still in its GGUF quantization in HBM.
//
// Operands are swapped so the weights are the MMA's M side: a CTA owns 128 weight rows
// (TMEM lanes) and a tile of BN tokens (TMEM columns, BN <= 256), and walks K in steps of
// 64 in ascending order. Per k step:
//   * warp 0 (one lane) bulk-copies the raw quant chunk of its 128 rows (one contiguous
//     re-tiled chunk, see jv_internal.h) and the BN x 64 fp16 activation tile (one
//     contiguous run of the pre-swizzled K-slab layout) into shared memory, completing
//     on an mbarrier with a transaction count;
//   * warps 4-11 decode the chunk to fp16 (d*q, d*(n-8), d*q5+m in fp32, rounded once to
//     fp16) straight into the UMMA K-major SWIZZLE_128B layout;
//   * warp 1 (one lane) issues four tcgen05.mma kind::f16 (K = 16 each) into the fp32
//     TMEM accumulator and commits to the stage's "empty" mbarrier.
// After the last k step warps 4-7 read the accumulator with tcgen05.ld and store (or add
// into) Y; lanes are weight rows, so every store instruction writes 32 consecutive floats.
//
// Batch invariance: each output is one accumulation chain over K in a fixed order, with
// no split of K, and the tensor core computes an element from its own row and column
// only. A token's result therefore does not depend on BN, on its column in the tile or on
// the other tokens of the call (the property of PanelGemmTests.cs:61-74).
//
// Every mbarrier wait is bounded (about two seconds of %globaltimer); on expiry the thread
// sets the error word, the producer waits (bounded) for its copies in flight, the MMA lane
// still commits so the accumulator is quiescent, and the CTA frees its TMEM and returns.
// No cluster launch and no multicast: nothing here reads another GPU's memory.
#include "jv_internal.h"

namespace jv {

constexpr int GEMM_THREADS = 384;
constexpr int DEC_THREADS = 256;
constexpr uint64_t WAIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t s_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
// Bounded wait: false after ~2 s without the phase completing.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    uint64_t t0 = gtimer();
    while (!mbar_try(bar, parity))
        if (gtimer() - t0 > WAIT_NS) return false;
    return true;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(slot), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

// UMMA shared-memory matrix descriptor, K-major SWIZZLE_128B: start address >> 4 in bits
// 0-13, leading byte offset (unused by this layout) 16 B, stride byte offset 1024 B (one
// 8-row x 128-byte swizzle atom), descriptor version 1 (bits 46-47), layout 2 = SWIZZLE_128B
// (bits 61-63).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(16u >> 4) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A/B fp16 (bits 7-9, 10-12 = 0;
// 1 would be bf16), both K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_f16(int n, int m) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Bytes b0, b1 of x (picked by the byte_perm selector) as the fp16 pair (1024 + b0, 1024 + b1):
// a byte placed under the exponent of 1024 (0x64) is 1024 + b exactly.
__device__ __forceinline__ __half2 byte_pair(uint32_t x, uint32_t sel) {
    uint32_t w = __byte_perm(x, 0x64646464u, sel);
    return *reinterpret_cast<__half2*>(&w);
}
__device__ __forceinline__ uint32_t hu(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Decode one (row, 16-byte chunk) item: 8 consecutive weights of row r, k = 8c..8c+7, as
// packed fp16 pairs. Q8_0 and Q4_0: the integer is exact in fp16 and d * q is one
// correctly rounded fp16 multiply — the same value as the exact fp32 product rounded to
// fp16. Q5_1: d * q5 + m with one fp16 rounding (an fp16 FMA).
template <int TYPE>
__device__ __forceinline__ uint4 decode8(const uint8_t* __restrict__ raw, int r, int c) {
    uint4 o;
    if (TYPE == T_Q8_0) {
        uint2 q = *(const uint2*)(raw + r * 64 + c * 8);
        __half2 d2 = __half2half2(*(const __half*)(raw + 8192 + (r * 2 + (c >> 2)) * 2));
        uint32_t x0 = q.x ^ 0x80808080u, x1 = q.y ^ 0x80808080u;  // int8 -> biased byte b = q + 128
        const __half2 bias = __floats2half2_rn(1152.f, 1152.f);    // 1024 + 128
        o.x = hu(__hmul2(__hsub2(byte_pair(x0, 0x4140u), bias), d2));
        o.y = hu(__hmul2(__hsub2(byte_pair(x0, 0x4342u), bias), d2));
        o.z = hu(__hmul2(__hsub2(byte_pair(x1, 0x4140u), bias), d2));
        o.w = hu(__hmul2(__hsub2(byte_pair(x1, 0x4342u), bias), d2));
        return o;
    }
    int b = c >> 2, e0 = (c & 3) * 8;
    uint2 q = *(const uint2*)(raw + r * 32 + b * 16 + (e0 & 15));
    uint32_t x0, x1;
    if (e0 < 16) {
        x0 = q.x & 0x0F0F0F0Fu;
        x1 = q.y & 0x0F0F0F0Fu;
    } else {
        x0 = (q.x >> 4) & 0x0F0F0F0Fu;
        x1 = (q.y >> 4) & 0x0F0F0F0Fu;
    }
    if (TYPE == T_Q4_0) {
        __half2 d2 = __half2half2(*(const __half*)(raw + 4096 + (r * 2 + b) * 2));
        const __half2 bias = __floats2half2_rn(1032.f, 1032.f);  // 1024 + 8
        o.x = hu(__hmul2(__hsub2(byte_pair(x0, 0x4140u), bias), d2));
        o.y = hu(__hmul2(__hsub2(byte_pair(x0, 0x4342u), bias), d2));
        o.z = hu(__hmul2(__hsub2(byte_pair(x1, 0x4140u), bias), d2));
        o.w = hu(__hmul2(__hsub2(byte_pair(x1, 0x4342u), bias), d2));
        return o;
    }
    // Q5_1: fifth bit of element e from qh bit e, spread into bit 4 of each byte.
    uint32_t qh = *(const uint32_t*)(raw + 4096 + (r * 2 + b) * 4);
    __half2 d2 = __half2half2(*(const __half*)(raw + 5120 + (r * 2 + b) * 2));
    __half2 m2 = __half2half2(*(const __half*)(raw + 5632 + (r * 2 + b) * 2));
    uint32_t h0 = (qh >> e0) & 0xFu, h1 = (qh >> (e0 + 4)) & 0xFu;
    x0 |= ((h0 & 1u) << 4) | ((h0 & 2u) << 11) | ((h0 & 4u) << 18) | ((h0 & 8u) << 25);
    x1 |= ((h1 & 1u) << 4) | ((h1 & 2u) << 11) | ((h1 & 4u) << 18) | ((h1 & 8u) << 25);
    const __half2 bias = __floats2half2_rn(1024.f, 1024.f);
    o.x = hu(__hfma2(__hsub2(byte_pair(x0, 0x4140u), bias), d2, m2));
    o.y = hu(__hfma2(__hsub2(byte_pair(x0, 0x4342u), bias), d2, m2));
    o.z = hu(__hfma2(__hsub2(byte_pair(x1, 0x4140u), bias), d2, m2));
    o.w = hu(__hfma2(__hsub2(byte_pair(x1, 0x4342u), bias), d2, m2));
    return o;
}

struct TcParams {
    const uint8_t* w;
    const __half* x;
    float* y;
    int* err;
    __half* xs_out;   // EPI_SWIGLU destination (K-slab, tpad rows)
    float* ws;        // split-K partials [split][T][ldy] (splits > 1)
    int* counters;    // one arrival counter per (row tile, token tile); zero between launches
    int ksteps, T, tpad, bn, ldy, epilogue, stages, ncols, splits;
    int raw_off, b_off, bar_off;  // byte offsets inside the 1024-aligned dynamic smem
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }

template <int TYPE>
__global__ void __launch_bounds__(GEMM_THREADS, 1) k_gemm_tc(TcParams p) {
    extern __shared__ uint8_t gsm_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)gsm_raw + 1023) & ~(uintptr_t)1023);
    const int S = p.stages;
    const int cb = chunk_bytes(TYPE);
    uint8_t* As = sm;                       // S x 16 KB
    uint8_t* Bs = sm + p.b_off;             // S x bn*128
    uint8_t* Rs = sm + p.raw_off;           // S x chunk
    uint64_t* bars = (uint64_t*)(sm + p.bar_off);
    uint32_t* tslot = (uint32_t*)(bars + 3 * S + 1);
    volatile int* last_flag = (volatile int*)(tslot + 1);
    const uint32_t full0 = s_addr(bars), dec0 = s_addr(bars + S), empty0 = s_addr(bars + 2 * S), accf = s_addr(bars + 3 * S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, t0 = blockIdx.y * p.bn;
    // Split-K: this CTA's contiguous share of the k steps. The split is fixed by the weight
    // shape (host side), never by the token count, so it cannot break batch invariance.
    const int nks = p.ksteps / p.splits, kbase = blockIdx.z * nks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(dec0 + 8 * s, DEC_THREADS);
            mbar_init(empty0 + 8 * s, 1);
        }
        mbar_init(accf, 1);
        fence_barrier_init();
    }
    if (warp == 2) tmem_alloc(s_addr(tslot), p.ncols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            const uint8_t* wsrc = p.w + ((int64_t)tile * p.ksteps + kbase) * cb;
            const uint32_t bbytes = (uint32_t)p.bn * 128u;
            for (int ks = 0; ks < nks; ks++) {
                int s = ks % S;
                uint32_t ph = (uint32_t)(ks / S) & 1u;
                if (!mbar_wait(empty0 + 8 * s, ph ^ 1u)) { ok = false; break; }
                mbar_expect_tx(full0 + 8 * s, (uint32_t)cb + bbytes);
                bulk_g2s(s_addr(Rs + s * cb), wsrc + (int64_t)ks * cb, (uint32_t)cb, full0 + 8 * s);
                bulk_g2s(s_addr(Bs + (size_t)s * bbytes), p.x + ((int64_t)(kbase + ks) * p.tpad + t0) * 64, bbytes,
                         full0 + 8 * s);
                issued++;
            }
            if (!ok) atomicExch(p.err, JV_ERR_DEVICE_TIMEOUT);
            // Never leave with copies in flight into this CTA's shared memory.
            for (int i = issued - 1; i >= 0 && i >= issued - S; i--)
                if (!mbar_wait(full0 + 8 * (i % S), (uint32_t)(i / S) & 1u)) atomicExch(p.err, JV_ERR_DEVICE_TIMEOUT);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(p.bn, 128);
            const uint32_t bbytes = (uint32_t)p.bn * 128u;
            for (int ks = 0; ks < nks; ks++) {
                int s = ks % S;
                uint32_t ph = (uint32_t)(ks / S) & 1u;
                if (!mbar_wait(full0 + 8 * s, ph) || !mbar_wait(dec0 + 8 * s, ph)) {
                    atomicExch(p.err, JV_ERR_DEVICE_TIMEOUT);
                    break;
                }
                tc_fence_after();
                uint32_t a_base = s_addr(As + s * 16384), b_base = s_addr(Bs + (size_t)s * bbytes);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    umma(tmem, sdesc(a_base + 32 * j), sdesc(b_base + 32 * j), idesc, (ks > 0 || j > 0) ? 1u : 0u);
                umma_commit(empty0 + 8 * s);
            }
            umma_commit(accf);  // always: the epilogue and teardown wait for a quiescent accumulator
        }
    } else if (warp >= 4) {
        // Thread dt decodes chunk c = dt % 8 of rows r0 + 32*it (it = 0..3); the swizzled
        // position of that chunk is the same for all four rows.
        const int dt = threadIdx.x - 128;
        const int c = dt & 7, r0 = dt >> 3;
        const int a_off = r0 * 128 + ((c ^ (r0 & 7)) << 4);
        bool ok = true;
        for (int ks = 0; ks < nks; ks++) {
            int s = ks % S;
            uint32_t ph = (uint32_t)(ks / S) & 1u;
            if (!mbar_wait(full0 + 8 * s, ph)) { ok = false; break; }
            const uint8_t* raw = Rs + s * cb;
            uint8_t* A = As + s * 16384 + a_off;
            uint4 v[4];
#pragma unroll
            for (int it = 0; it < 4; it++) v[it] = decode8<TYPE>(raw, r0 + 32 * it, c);
#pragma unroll
            for (int it = 0; it < 4; it++) *(uint4*)(A + it * 32 * 128) = v[it];
            fence_proxy_async();
            mbar_arrive(dec0 + 8 * s);
        }
        if (!ok) atomicExch(p.err, JV_ERR_DEVICE_TIMEOUT);
        if (warp < 8) {
            // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 = weight rows of this tile.
            int q = warp & 3;
            bool ready = mbar_wait(accf, 0);
            tc_fence_after();
            const int n = tile * 128 + q * 32 + lane;
            const bool good = ready && ok;
            if (p.epilogue == EPI_SWIGLU) {
                // Kernels.SwiGlu (reference src/Jevstral/Numerics/Kernels.cs:82-89):
                // up <- g*u; s <- 1/(1+exp(-g)); y <- s*up. Up rows (lanes 64-127) go through
                // the stage memory, free now that every MMA has completed.
                float* ubuf = (float*)sm;  // [bn][64]
                if (good && q >= 2)
                    for (int col = 0; col < p.bn; col += 16) {
                        float v[16];
                        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col, v);
#pragma unroll
                        for (int j = 0; j < 16; j++) ubuf[(col + j) * 64 + (q - 2) * 32 + lane] = v[j];
                    }
                epi_bar();
                if (good && q < 2) {
                    const int jf = tile * 64 + q * 32 + lane;  // FFN feature
                    for (int col = 0; col < p.bn; col += 16) {
                        float g[16];
                        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col, g);
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            int t = t0 + col + j;
                            float u = ubuf[(col + j) * 64 + q * 32 + lane];
                            float up = __fmul_rn(g[j], u);
                            float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g[j])));
                            if (t < p.T) p.xs_out[kslab_offset(t, jf, p.tpad)] = __float2half_rn(__fmul_rn(sg, up));
                        }
                    }
                }
            } else if (p.splits == 1) {
                if (good) {
                    for (int col = 0; col < p.bn; col += 16) {
                        float v[16];
                        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col, v);
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            int t = t0 + col + j;
                            if (t < p.T) {
                                float* dst = p.y + (int64_t)t * p.ldy + n;
                                if (p.epilogue == EPI_ADD)
                                    *dst = __fadd_rn(*dst, v[j]);
                                else
                                    *dst = v[j];
                            }
                        }
                    }
                }
            } else {
                // Both K halves publish their partial; the CTA that arrives last adds the other
                // half to its own (still in TMEM): p0 + p1, which is the same value whichever
                // CTA that is (IEEE addition commutes).
                float* mine = p.ws + (int64_t)blockIdx.z * p.T * p.ldy;
                const float* other = p.ws + (int64_t)(1 - blockIdx.z) * p.T * p.ldy;
                if (good) {
                    for (int col = 0; col < p.bn; col += 16) {
                        float v[16];
                        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col, v);
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            int t = t0 + col + j;
                            if (t < p.T) mine[(int64_t)t * p.ldy + n] = v[j];
                        }
                    }
                }
                __threadfence();
                epi_bar();
                if (warp == 4 && lane == 0) {
                    int* ctr = p.counters + blockIdx.x * gridDim.y + blockIdx.y;
                    int old = atomicAdd(ctr, 1);
                    int last = old == p.splits - 1;
                    if (last) atomicExch(ctr, 0);
                    *last_flag = last;
                }
                epi_bar();
                if (*last_flag && good) {
                    __threadfence();
                    for (int col = 0; col < p.bn; col += 16) {
                        float v[16], o[16], yv[16];
                        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col, v);
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            int t = t0 + col + j;
                            o[j] = t < p.T ? __ldcg(other + (int64_t)t * p.ldy + n) : 0.f;
                            yv[j] = (t < p.T && p.epilogue == EPI_ADD) ? p.y[(int64_t)t * p.ldy + n] : 0.f;
                        }
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            int t = t0 + col + j;
                            if (t < p.T) {
                                float s = __fadd_rn(v[j], o[j]);
                                p.y[(int64_t)t * p.ldy + n] = p.epilogue == EPI_ADD ? __fadd_rn(yv[j], s) : s;
                            }
                        }
                    }
                }
            }
            if (!ready) atomicExch(p.err, JV_ERR_DEVICE_TIMEOUT);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, p.ncols);
    }
}

int gemm_bn_for(int T) {
    int tiles = (T + 255) / 256;
    int per = (T + tiles - 1) / tiles;
    int bn = (per + 15) / 16 * 16;
    return bn < 16 ? 16 : bn;
}
int gemm_tpad_for(int T) {
    int bn = gemm_bn_for(T);
    return (T + bn - 1) / bn * bn;
}

template <int TYPE>
static void launch_tc_typed(const GemmArgs& a, cudaStream_t s) {
    const QWeight& w = *a.w;
    TcParams p;
    p.w = w.data;
    p.x = a.x;
    p.y = a.y;
    p.err = a.err;
    p.ksteps = w.ksteps;
    p.T = a.T;
    p.tpad = a.tpad;
    p.bn = a.bn;
    p.ldy = a.ldy;
    p.epilogue = a.epilogue;
    p.splits = a.splits;
    p.xs_out = a.xs_out;
    p.ws = a.ws;
    p.counters = a.counters;
    int cb = chunk_bytes(TYPE);
    size_t per_stage = 16384 + (size_t)a.bn * 128 + cb;
    p.stages = (per_stage * 4 + 3072 <= 225 * 1024) ? 4 : 3;
    int nc = 32;
    while (nc < a.bn) nc <<= 1;
    p.ncols = nc;
    p.b_off = 16384 * p.stages;
    p.raw_off = p.b_off + a.bn * 128 * p.stages;
    p.bar_off = (p.raw_off + cb * p.stages + 15) & ~15;
    size_t smem = (size_t)p.bar_off + 8 * (3 * p.stages + 1) + 16 + 1024;
    static int configured = 0;
    if (configured < (int)smem) {
        JV_CUDA(cudaFuncSetAttribute(k_gemm_tc<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        configured = (int)smem;
    }
    dim3 grid(w.tiles, a.tpad / a.bn, a.splits);
    k_gemm_tc<TYPE><<<grid, GEMM_THREADS, smem, s>>>(p);
    note_launch();
}

int gemm_splits_for(const QWeight& w) {
    // Few row tiles and a long K (the 3072-row O and down projections): two K halves, so
    // the product fills the GPU. A property of the matrix, never of the token count.
    return (w.tiles <= 32 && w.ksteps >= 64 && w.ksteps % 2 == 0) ? 2 : 1;
}

void launch_gemm(const GemmArgs& a, cudaStream_t s) {
    if (a.bn % 16 != 0 || a.bn < 16 || a.bn > 256 || a.tpad % a.bn != 0)
        throw Error(JV_ERR_ARG, "gemm: token tile must be a multiple of 16 in [16, 256] dividing the padded rows");
    if (a.splits < 1 || a.splits > 2 || a.w->ksteps % a.splits != 0 || (a.splits > 1 && (!a.ws || !a.counters)))
        throw Error(JV_ERR_ARG, "gemm: bad split-K arguments");
    if (a.epilogue == EPI_SWIGLU && (a.splits != 1 || !a.xs_out))
        throw Error(JV_ERR_ARG, "gemm: the SwiGLU epilogue needs an unsplit product and an output slab");
    switch (a.w->type) {
        case T_Q8_0: launch_tc_typed<T_Q8_0>(a, s); break;
        case T_Q4_0: launch_tc_typed<T_Q4_0>(a, s); break;
        case T_Q5_1: launch_tc_typed<T_Q5_1>(a, s); break;
        default: throw Error(JV_ERR_UNSUPPORTED, "gemm: weight type not on the B200 path");
    }
}

// ------------------------------------------------------- reference GEMM

// A plain CUDA-core product over the *same* fp16 operands (weights decoded and rounded to
// fp16 exactly as the tensor-core producer does). Used only by the library's self-test
// entry point to check the tcgen05 kernel at full shapes; never on the forward path.
template <int TYPE>
__global__ void k_gemm_ref(const uint8_t* __restrict__ w, int ksteps, const __half* __restrict__ x, int T, int tpad,
                           float* __restrict__ y, int ldy, int epilogue) {
    int n = blockIdx.x * 128 + threadIdx.x;
    int t = blockIdx.y;
    int tile = n >> 7, r = n & 127;
    float acc = 0.f;
    for (int ks = 0; ks < ksteps; ks++) {
        const uint8_t* raw = w + ((int64_t)tile * ksteps + ks) * chunk_bytes(TYPE);
        for (int c = 0; c < 8; c++) {
            uint4 h = decode8<TYPE>(raw, r, c);
            const __half* hw = (const __half*)&h;
            for (int i = 0; i < 8; i++) {
                int k = ks * 64 + c * 8 + i;
                acc = fmaf(__half2float(x[kslab_offset(t, k, tpad)]), __half2float(hw[i]), acc);
            }
        }
    }
    float* dst = y + (int64_t)t * ldy + n;
    *dst = epilogue == EPI_ADD ? *dst + acc : acc;
}

void launch_gemm_reference(const GemmArgs& a, cudaStream_t s) {
    dim3 grid(a.w->tiles, a.T);
    switch (a.w->type) {
        case T_Q8_0: k_gemm_ref<T_Q8_0><<<grid, 128, 0, s>>>(a.w->data, a.w->ksteps, a.x, a.T, a.tpad, a.y, a.ldy, a.epilogue); break;
        case T_Q4_0: k_gemm_ref<T_Q4_0><<<grid, 128, 0, s>>>(a.w->data, a.w->ksteps, a.x, a.T, a.tpad, a.y, a.ldy, a.epilogue); break;
        default: k_gemm_ref<T_Q5_1><<<grid, 128, 0, s>>>(a.w->data, a.w->ksteps, a.x, a.T, a.tpad, a.y, a.ldy, a.epilogue); break;
    }
    note_launch();
}

}  // namespace jv
