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

// int8 / small unsigned byte -> exact fp32 via the 2^23 magic number: byte b placed in the
// mantissa of 2^23 gives 2^23 + b; subtracting the bias yields the integer exactly.
__device__ __forceinline__ float byte_f(uint32_t x, uint32_t sel) { return __uint_as_float(__byte_perm(x, 0x4B000000u, sel)); }

__device__ __forceinline__ uint32_t h2u(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *(uint32_t*)&h;
}

// Decode one (row, 16-byte chunk) item: 8 consecutive weights of row r, k = 8c..8c+7.
template <int TYPE>
__device__ __forceinline__ uint4 decode8(const uint8_t* __restrict__ raw, int r, int c) {
    float f[8];
    if (TYPE == T_Q8_0) {
        uint2 q = *(const uint2*)(raw + r * 64 + c * 8);
        float d = __half2float(*(const __half*)(raw + 8192 + (r * 2 + (c >> 2)) * 2));
        uint32_t x0 = q.x ^ 0x80808080u, x1 = q.y ^ 0x80808080u;
        const float bias = 8388736.0f;  // 2^23 + 128
#pragma unroll
        for (int i = 0; i < 4; i++) {
            f[i] = __fmul_rn(d, __fsub_rn(byte_f(x0, 0x7540u + i), bias));
            f[4 + i] = __fmul_rn(d, __fsub_rn(byte_f(x1, 0x7540u + i), bias));
        }
    } else {
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
            float d = __half2float(*(const __half*)(raw + 4096 + (r * 2 + b) * 2));
            const float bias = 8388616.0f;  // 2^23 + 8
#pragma unroll
            for (int i = 0; i < 4; i++) {
                f[i] = __fmul_rn(d, __fsub_rn(byte_f(x0, 0x7540u + i), bias));
                f[4 + i] = __fmul_rn(d, __fsub_rn(byte_f(x1, 0x7540u + i), bias));
            }
        } else {  // Q5_1
            uint32_t qh = *(const uint32_t*)(raw + 4096 + (r * 2 + b) * 4);
            float d = __half2float(*(const __half*)(raw + 5120 + (r * 2 + b) * 2));
            float m = __half2float(*(const __half*)(raw + 5632 + (r * 2 + b) * 2));
            uint32_t h0 = (qh >> e0) & 0xFu, h1 = (qh >> (e0 + 4)) & 0xFu;
            x0 |= ((h0 & 1u) << 4) | ((h0 & 2u) << 11) | ((h0 & 4u) << 18) | ((h0 & 8u) << 25);
            x1 |= ((h1 & 1u) << 4) | ((h1 & 2u) << 11) | ((h1 & 4u) << 18) | ((h1 & 8u) << 25);
            const float bias = 8388608.0f;  // 2^23
#pragma unroll
            for (int i = 0; i < 4; i++) {
                f[i] = __fadd_rn(__fmul_rn(d, __fsub_rn(byte_f(x0, 0x7540u + i), bias)), m);
                f[4 + i] = __fadd_rn(__fmul_rn(d, __fsub_rn(byte_f(x1, 0x7540u + i), bias)), m);
            }
        }
    }
    return make_uint4(h2u(f[0], f[1]), h2u(f[2], f[3]), h2u(f[4], f[5]), h2u(f[6], f[7]));
}

struct TcParams {
    const uint8_t* w;
    const __half* x;
    float* y;
    int* err;
    int ksteps, T, tpad, bn, ldy, epilogue, stages, ncols;
    int raw_off, b_off, bar_off;  // byte offsets inside the 1024-aligned dynamic smem
};

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
    const uint32_t full0 = s_addr(bars), dec0 = s_addr(bars + S), empty0 = s_addr(bars + 2 * S), accf = s_addr(bars + 3 * S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, t0 = blockIdx.y * p.bn;

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
            const uint8_t* wsrc = p.w + (int64_t)tile * p.ksteps * cb;
            const uint32_t bbytes = (uint32_t)p.bn * 128u;
            for (int ks = 0; ks < p.ksteps; ks++) {
                int s = ks % S;
                uint32_t ph = (uint32_t)(ks / S) & 1u;
                if (!mbar_wait(empty0 + 8 * s, ph ^ 1u)) { ok = false; break; }
                mbar_expect_tx(full0 + 8 * s, (uint32_t)cb + bbytes);
                bulk_g2s(s_addr(Rs + s * cb), wsrc + (int64_t)ks * cb, (uint32_t)cb, full0 + 8 * s);
                bulk_g2s(s_addr(Bs + (size_t)s * bbytes), p.x + ((int64_t)ks * p.tpad + t0) * 64, bbytes, full0 + 8 * s);
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
            for (int ks = 0; ks < p.ksteps; ks++) {
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
        const int dt = threadIdx.x - 128;
        bool ok = true;
        for (int ks = 0; ks < p.ksteps; ks++) {
            int s = ks % S;
            uint32_t ph = (uint32_t)(ks / S) & 1u;
            if (!mbar_wait(full0 + 8 * s, ph)) { ok = false; break; }
            const uint8_t* raw = Rs + s * cb;
            uint8_t* A = As + s * 16384;
#pragma unroll
            for (int it = 0; it < 4; it++) {
                int item = it * DEC_THREADS + dt;
                int r = item >> 3, c = item & 7;
                *(uint4*)(A + r * 128 + ((c ^ (r & 7)) << 4)) = decode8<TYPE>(raw, r, c);
            }
            fence_proxy_async();
            mbar_arrive(dec0 + 8 * s);
        }
        if (!ok) atomicExch(p.err, JV_ERR_DEVICE_TIMEOUT);
        if (warp < 8) {
            // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 = weight rows of this tile.
            int q = warp & 3;
            bool ready = mbar_wait(accf, 0);
            tc_fence_after();
            if (ready && ok) {
                int n = tile * 128 + q * 32 + lane;
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
            } else if (!ready) {
                atomicExch(p.err, JV_ERR_DEVICE_TIMEOUT);
            }
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
    int cb = chunk_bytes(TYPE);
    size_t per_stage = 16384 + (size_t)a.bn * 128 + cb;
    p.stages = (per_stage * 4 + 2048 <= 200 * 1024) ? 4 : 3;
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
    dim3 grid(w.tiles, a.tpad / a.bn);
    k_gemm_tc<TYPE><<<grid, GEMM_THREADS, smem, s>>>(p);
    note_launch();
}

void launch_gemm(const GemmArgs& a, cudaStream_t s) {
    if (a.bn % 16 != 0 || a.bn < 16 || a.bn > 256 || a.tpad % a.bn != 0)
        throw Error(JV_ERR_ARG, "gemm: token tile must be a multiple of 16 in [16, 256] dividing the padded rows");
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
