// gemm_tc.cu — the prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Y[t, n] (+)= sum_k X[t, k] * W[n, k]: the reference's PanelGemm (src/Jevstral/Numerics/
// PanelGemm.cs:76-300), with W still in its GGUF quantization in HBM.
//
// Operands are swapped so the weights are the MMA's M side: a work unit is 128 weight rows
// (TMEM lanes) x a tile of BN tokens (TMEM columns, BN <= 256) x a contiguous range of k
// steps of 64, walked in ascending order. The kernel is persistent: one CTA per SM takes
// units round-robin, and its warps run decoupled pipelines across unit boundaries:
//   * warp 0, lane 0 — bulk-copies each k step's raw quant chunk (one contiguous re-tiled
//     chunk of 128 rows x 64 columns, see jv_internal.h) into a deep ring, and the BN x 64
//     fp16 activation tile (one contiguous run of the pre-swizzled K-slab layout) into a
//     second ring, each completing on an mbarrier with a transaction count;
//   * warps 8-15 — decode a raw chunk to fp16 in registers, hand its ring slot back at
//     once, and store the values into a decoded-weight slot in the UMMA K-major
//     SWIZZLE_128B layout;
//   * warp 1, lane 0 — issues four tcgen05.mma kind::f16 (K = 16) per k step into one of
//     two fp32 TMEM accumulators and commits to free the activation and decoded slots;
//   * warps 4-7 — drain the other accumulator with tcgen05.ld while the next unit
//     accumulates: store, add into Y, fused SwiGLU, or the split-K combine.
// Raw chunks are freed by the decoders, not by the tensor core, so the weight stream runs
// many steps ahead; only the fp16 activation ring and the decoded slots follow the MMA.
//
// Batch invariance: each output is one accumulation chain over K in a fixed order; the
// only K split is fixed per weight matrix (gemm_splits_for), never by the token count; the
// tensor core computes an element from its own row and column only. A token's result
// therefore does not depend on BN, its column in the tile, or the other tokens of the call
// (the property of PanelGemmTests.cs:61-74).
//
// Every mbarrier wait is bounded (WAIT_CYCLES of the SM clock, about 2 s), with one verdict per
// warp. On expiry the warp sets the error word and its role stops; the others then time out in turn; the producer
// waits (bounded) for its copies in flight, the MMA lane drains its own MMAs, and the CTA
// frees its TMEM and returns. No cluster launch and no multicast: nothing here reads another
// GPU's memory.
#include "gemm_plan.h"
#include "tc_common.cuh"

namespace jv {

constexpr int GEMM_THREADS = 512;
constexpr int DEC_WARP0 = 8;
constexpr int DEC_WARPS_PER_GROUP = 4;  // two decoder groups, alternate k steps
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
// fp16. Q5_1: d * q5 + m with one fp16 rounding (an fp16 FMA). QX: (a * q) + c in fp32, then
// one rounding to fp16. The raw words an item needs are loaded first (item_load, from shared
// memory or straight from global memory), then decoded from registers (item_decode).
struct Item {
    uint2 q;         // the item's 8 quantized values (bytes or nibble pairs)
    uint32_t w0, w1, w2;  // Q8_0/Q4_0: d; Q5_1: d, m, qh; QX: a, c
};

template <int TYPE>
__device__ __forceinline__ Item item_load(const uint8_t* __restrict__ raw, int r, int c) {
    Item it;
    if (TYPE == T_Q8_0 || TYPE == T_QX) {
        it.q = *(const uint2*)(raw + r * 64 + c * 8);
        if (TYPE == T_Q8_0) {
            it.w0 = *(const uint16_t*)(raw + 8192 + (r * 2 + (c >> 2)) * 2);
        } else {
            it.w0 = *(const uint32_t*)(raw + 8192 + (r * 4 + (c >> 1)) * 4);
            it.w1 = *(const uint32_t*)(raw + 10240 + (r * 4 + (c >> 1)) * 4);
        }
        return it;
    }
    const int b = c >> 2, e0 = (c & 3) * 8;
    it.q = *(const uint2*)(raw + r * 32 + b * 16 + (e0 & 15));
    if (TYPE == T_Q4_0) {
        it.w0 = *(const uint16_t*)(raw + 4096 + (r * 2 + b) * 2);
    } else {
        it.w0 = *(const uint16_t*)(raw + 5120 + (r * 2 + b) * 2);
        it.w1 = *(const uint16_t*)(raw + 5632 + (r * 2 + b) * 2);
        it.w2 = *(const uint32_t*)(raw + 4096 + (r * 2 + b) * 4);
    }
    return it;
}

template <int TYPE>
__device__ __forceinline__ uint4 item_decode(const Item& it, int c) {
    uint4 o;
    if (TYPE == T_QX) {
        const float a = __uint_as_float(it.w0), cc = __uint_as_float(it.w1);
        const int8_t* qb = (const int8_t*)&it.q;
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; i++)
            w[i] = hu(__floats2half2_rn(__fadd_rn(__fmul_rn(a, (float)qb[2 * i]), cc),
                                        __fadd_rn(__fmul_rn(a, (float)qb[2 * i + 1]), cc)));
        o.x = w[0];
        o.y = w[1];
        o.z = w[2];
        o.w = w[3];
        return o;
    }
    const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)it.w0));
    if (TYPE == T_Q8_0) {
        uint32_t x0 = it.q.x ^ 0x80808080u, x1 = it.q.y ^ 0x80808080u;  // int8 -> biased byte b = q + 128
        const __half2 bias = __floats2half2_rn(1152.f, 1152.f);        // 1024 + 128
        o.x = hu(__hmul2(__hsub2(byte_pair(x0, 0x4140u), bias), d2));
        o.y = hu(__hmul2(__hsub2(byte_pair(x0, 0x4342u), bias), d2));
        o.z = hu(__hmul2(__hsub2(byte_pair(x1, 0x4140u), bias), d2));
        o.w = hu(__hmul2(__hsub2(byte_pair(x1, 0x4342u), bias), d2));
        return o;
    }
    const int e0 = (c & 3) * 8;
    uint32_t x0, x1;
    if (e0 < 16) {
        x0 = it.q.x & 0x0F0F0F0Fu;
        x1 = it.q.y & 0x0F0F0F0Fu;
    } else {
        x0 = (it.q.x >> 4) & 0x0F0F0F0Fu;
        x1 = (it.q.y >> 4) & 0x0F0F0F0Fu;
    }
    if (TYPE == T_Q4_0) {
        const __half2 bias = __floats2half2_rn(1032.f, 1032.f);  // 1024 + 8
        o.x = hu(__hmul2(__hsub2(byte_pair(x0, 0x4140u), bias), d2));
        o.y = hu(__hmul2(__hsub2(byte_pair(x0, 0x4342u), bias), d2));
        o.z = hu(__hmul2(__hsub2(byte_pair(x1, 0x4140u), bias), d2));
        o.w = hu(__hmul2(__hsub2(byte_pair(x1, 0x4342u), bias), d2));
        return o;
    }
    // Q5_1: fifth bit of element e from qh bit e, spread into bit 4 of each byte.
    const uint32_t qh = it.w2;
    const __half2 m2 = __half2half2(__ushort_as_half((unsigned short)it.w1));
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

template <int TYPE>
__device__ __forceinline__ uint4 decode8(const uint8_t* __restrict__ raw, int r, int c) {
    return item_decode<TYPE>(item_load<TYPE>(raw, r, c), c);
}

constexpr int RAW_PREFETCH = 24;  // raw chunks prefetched into L2 ahead of the shared-memory copies

struct TcParams {
    const uint8_t* w;
    const __half* x;
    float* y;
    int* err;
    __half* xs_out;   // EPI_SWIGLU destination (K-slab, tpad rows)
    float* ws;        // split-K partials [split][T][ldy] (splits > 1)
    int* counters;    // one arrival counter per (row tile, token tile); zero between launches
    int ksteps, T, tpad, bn, ldy, epilogue, ncols, splits;
    int tiles, ttiles, units;   // work units = tiles x ttiles x splits
    int nr, ns;                 // ring depths: raw chunks; stages (activation tile + decoded weights)
    int raw_off, b_off, bar_off;  // byte offsets inside the 1024-aligned dynamic smem (A at 0)
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }
// The four epilogue warps' joint verdict (named barrier 1 with an AND reduction), so that on a
// timeout all of them leave the unit loop together and none waits at epi_bar for the others.
__device__ __forceinline__ bool epi_all(bool p) {
    uint32_t r;
    asm volatile(
        "{\n.reg .pred q, o;\nsetp.ne.u32 q, %1, 0;\nbar.red.and.pred o, 1, 128, q;\nselp.u32 %0, 1, 0, o;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)p)
        : "memory");
    return r != 0;
}
// A bounded wait taken by a whole warp: every lane gets the same verdict, so on a timeout the
// warp leaves together and never reaches a .sync.aligned tcgen05 instruction or a __syncwarp
// with lanes missing.
__device__ __forceinline__ bool warp_wait_all(uint32_t bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// Position in a ring of n mbarrier-guarded slots: slot index and the parity of its current use.
struct Ring {
    int n, idx = 0;
    uint32_t phase = 0;
    __device__ explicit Ring(int slots) : n(slots) {}
    __device__ __forceinline__ void next() {
        if (++idx == n) { idx = 0; phase ^= 1u; }
    }
    __device__ __forceinline__ void prev() {
        if (--idx < 0) { idx = n - 1; phase ^= 1u; }
    }
};

// Work unit u -> (row tile, token tile, K split), token tiles and splits of one row tile
// adjacent so concurrently running CTAs share each weight chunk through L2.
__device__ __forceinline__ void unit_coords(int u, int splits, int ttiles, int& tile, int& tt, int& sp) {
    sp = u % splits;
    int r = u / splits;
    tt = r % ttiles;
    tile = r / ttiles;
}

// What drain_cols does with accumulator values: write them as they are (a K-split partial),
// store / add them into Y (after adding the other K half when `other` is given), or the
// SwiGLU of each gate/up pair into the fp16 K-slab of the down projection's input.
enum DrainKind : int { DR_RAW = 0, DR_STORE = 1, DR_ADD = 2, DR_SWIGLU = 3 };

// Start column of share s when the last unit's columns are split in thirds, in whole
// 16-column chunks: share 0 = [drain_share(0), drain_share(1)) for the epilogue warps, shares
// 1 and 2 for the two decoder groups; drain_share(3) = bn.
__device__ __forceinline__ int drain_share(int bn, int s) {
    const int nch = bn / 16;
    return s <= 0 ? 0 : s >= 3 ? bn : 16 * ((s * nch + 2) / 3);
}

// Drain accumulator columns [c0, c1) (multiples of 16) of TMEM lane quarter q: one 16-column
// tcgen05.ld in flight while the previous chunk is processed. Row n of the output, tokens
// t0 + column for columns below tn.
__device__ __forceinline__ void drain_cols(uint32_t tacc, int c0, int c1, int kind, int lane, int q, int n, int tile,
                                           int t0, int tn, int tpad, int ldy, float* __restrict__ y,
                                           const float* __restrict__ other, __half* __restrict__ xs_out, int* err) {
    if (c0 >= c1) return;
    bool bad = false;
    uint32_t cur[16], nxt[16];
    tmem_ld16_issue(tacc + (uint32_t)c0, cur);
    tmem_wait16(cur);
    for (int col = c0; col < c1; col += 16) {
        const bool more = col + 16 < c1;
        if (more) tmem_ld16_issue(tacc + (uint32_t)(col + 16), nxt);
        const int lim = min(16, tn - col);
        if (kind == DR_SWIGLU) {
            // Kernels.SwiGlu (reference src/Jevstral/Numerics/Kernels.cs:82-89):
            // up <- g*u; s <- 1/(1+exp(-g)); y <- s*up. Lanes 0-15 hold gate rows, lanes 16-31
            // the matching up rows: one shuffle pairs them, lane l < 16 writes columns 0-7 of
            // the chunk, lane l + 16 columns 8-15.
            const int jf = tile * 64 + q * 16 + (lane & 15);
            const bool hi = lane >= 16;
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; j++) o[j] = __shfl_xor_sync(0xffffffffu, __uint_as_float(cur[j]), 16);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int jj = hi ? j + 8 : j;
                const float mv = hi ? __uint_as_float(cur[j + 8]) : __uint_as_float(cur[j]);
                const float ov = hi ? o[j + 8] : o[j];
                const float gg = hi ? ov : mv;
                const float uu = hi ? mv : ov;
                const float up = __fmul_rn(gg, uu);
                const float sg = __frcp_rn(__fadd_rn(1.0f, __expf(-gg)));
                const float act = __fmul_rn(sg, up);
                if (jj < lim) {
                    bad |= f16_out_of_range(act);
                    xs_out[kslab_offset(t0 + col + jj, jf, tpad)] = __float2half_rn(act);
                }
            }
        } else {
            // Row pointers step by ldy per token.
            float* yp = y + (int64_t)(t0 + col) * ldy + n;
            if (other) {
                const float* op = other + (int64_t)(t0 + col) * ldy + n;
                float o[16], yv[16];
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    o[j] = j < lim ? __ldcg(op + (int64_t)j * ldy) : 0.f;
                    yv[j] = (kind == DR_ADD && j < lim) ? yp[(int64_t)j * ldy] : 0.f;
                }
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (j < lim) {
                        const float s = __fadd_rn(__uint_as_float(cur[j]), o[j]);
                        yp[(int64_t)j * ldy] = kind == DR_ADD ? __fadd_rn(yv[j], s) : s;
                    }
            } else if (kind == DR_ADD) {
                float yv[16];
#pragma unroll
                for (int j = 0; j < 16; j++) yv[j] = j < lim ? yp[(int64_t)j * ldy] : 0.f;
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (j < lim) yp[(int64_t)j * ldy] = __fadd_rn(yv[j], __uint_as_float(cur[j]));
            } else {
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (j < lim) yp[(int64_t)j * ldy] = __uint_as_float(cur[j]);
            }
        }
        if (more) {
            tmem_wait16(nxt);
#pragma unroll
            for (int j = 0; j < 16; j++) cur[j] = nxt[j];
        }
    }
    if (bad) report_numeric(err, NS_SWIGLU);
}

template <int TYPE, int EPI, bool CSPLIT>
__global__ void __launch_bounds__(GEMM_THREADS, 1) k_gemm_tc(TcParams p) {
    // Every parameter in a register or a restrict pointer: nothing below takes the address of
    // the parameter block, so no access is re-read after a store.
    const uint8_t* __restrict__ g_w = p.w;
    const __half* __restrict__ g_x = p.x;
    float* __restrict__ g_y = p.y;
    int* __restrict__ g_err = p.err;
    __half* __restrict__ g_xs_out = p.xs_out;
    float* g_ws = p.ws;
    int* __restrict__ g_ctr = p.counters;
    // The epilogue is a template parameter: each instantiation carries only its own drain code.
    // CSPLIT: a K-split store/add whose halves are combined through the counters (the
    // activation-capture path; the hot path splits only with EPI_PARTIAL).
    constexpr int epi = EPI;
    const int ksteps = p.ksteps, T = p.T, tpad = p.tpad, bn = p.bn, ldy = p.ldy, ncols = p.ncols;
    const int splits = p.splits, ttiles = p.ttiles, units = p.units, nr_ = p.nr, ns_ = p.ns;
    const int raw_off = p.raw_off, b_off = p.b_off, bar_off = p.bar_off;
    extern __shared__ uint8_t gsm_raw[];
    // 1024-aligned for the SWIZZLE_128B tiles; pointer arithmetic on the shared array keeps the
    // pointer in the shared state space (plain ld/st.shared rather than generic accesses)
    uint8_t* sm = gsm_raw + ((1024u - (s_addr(gsm_raw) & 1023u)) & 1023u);
    const int cb = chunk_bytes(TYPE);
    const int NR = nr_, NS = ns_;
    uint8_t* As = sm;               // NS x 16 KB decoded weights
    uint8_t* Bs = sm + b_off;     // NS x bn*128 activations
    uint8_t* Rs = sm + raw_off;   // NR x chunk raw quant blocks
    uint64_t* bars = (uint64_t*)(sm + bar_off);
    // raw ring: raw_full (copy landed), raw_empty (4 decoder warps read it)
    // stage ring: b_full (activation tile landed: the copy's transaction bytes alone), a_full
    //             (4 decoder warps wrote the fp16 weights), st_empty (the MMA that read both
    //             completed)
    const uint32_t raw_full = s_addr(bars), raw_empty = raw_full + 8 * NR;
    const uint32_t b_full = raw_empty + 8 * NR, a_full = b_full + 8 * NS, st_empty = a_full + 8 * NS;
    const uint32_t acc_full = st_empty + 8 * NS, acc_empty = acc_full + 16, drained = acc_empty + 16;
    uint32_t* tslot = (uint32_t*)(bars + 2 * NR + 3 * NS + 5);
    volatile int* last_flag = (volatile int*)(tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nks = ksteps / splits;      // k steps per unit
    const uint32_t bbytes = (uint32_t)bn * 128u;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NR; i++) { mbar_init(raw_full + 8 * i, 1); mbar_init(raw_empty + 8 * i, DEC_WARPS_PER_GROUP); }
        for (int i = 0; i < NS; i++) {
            mbar_init(b_full + 8 * i, 1);
            mbar_init(a_full + 8 * i, DEC_WARPS_PER_GROUP);
            mbar_init(st_empty + 8 * i, 1);
        }
        for (int i = 0; i < 2; i++) { mbar_init(acc_full + 8 * i, 1); mbar_init(acc_empty + 8 * i, 4); }
        mbar_init(drained, 1);
        fence_barrier_init();
    }
    if (warp == 2) tmem_alloc(s_addr(tslot), 2 * ncols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    // The weights do not depend on the previous kernel: their stream and decode start now;
    // the activation loads and every global write wait for it (pdl_wait in those roles).
    pdl_launch_dependents();

    if (warp == 0 || warp == 3) {
        if (lane == 0) {  // ----------------------------------------------- producers
            // Warp 0 streams the raw weight chunks (ring freed by the decoders), warp 3 the
            // activation tiles (stage ring, freed by the MMA): neither waits on the other.
            const bool weights = warp == 0;
            const int depth = weights ? NR : NS;
            const uint32_t full = weights ? raw_full : b_full, empty = weights ? raw_empty : st_empty;
            const uint32_t bytes = weights ? (uint32_t)cb : bbytes;
            uint8_t* ring = weights ? Rs : Bs;
            Ring r(depth);
            bool ok = true;
            int issued = 0;
            if (!weights) pdl_wait();
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                int tile, tt, sp;
                unit_coords(u, splits, ttiles, tile, tt, sp);
                const int kb = sp * nks, t0 = tt * bn;
                if (!JV_CHECK(tile < p.tiles && kb + nks <= ksteps && t0 + bn <= tpad, g_err, BS_GEMM_UNIT)) break;
                const uint8_t* src = weights ? g_w + ((int64_t)tile * ksteps + kb) * cb
                                             : (const uint8_t*)(g_x + ((int64_t)kb * tpad + t0) * 64);
                const int64_t step = weights ? (int64_t)cb : (int64_t)tpad * 128;
                // The raw ring holds only a few chunks, too few to cover HBM latency on its
                // own: run an L2 prefetch RAW_PREFETCH chunks ahead of the copies.
                if (weights)
                    for (int ks = 0; ks < RAW_PREFETCH && ks < nks; ks++) bulk_prefetch_l2(src + ks * step, bytes);
                for (int ks = 0; ks < nks; ks++) {
                    if (weights && ks + RAW_PREFETCH < nks) bulk_prefetch_l2(src + (ks + RAW_PREFETCH) * step, bytes);
                    if (!mbar_wait(empty + 8 * r.idx, r.phase ^ 1u)) { ok = false; break; }
                    mbar_expect_tx(full + 8 * r.idx, bytes);
                    bulk_g2s(s_addr(ring + (size_t)r.idx * bytes), src + ks * step, bytes, full + 8 * r.idx);
                    r.next();
                    issued++;
                }
            }
            if (!ok) report_timeout(g_err, weights ? 1 : 2);
            // Never leave with copies in flight into this CTA's shared memory: wait for the
            // last min(issued, ring) copies.
            for (int i = 0; i < issued && i < depth; i++) {
                r.prev();
                if (!mbar_wait(full + 8 * r.idx, r.phase)) report_timeout(g_err, 3);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // --------------------------------------------- MMA issue
            const uint32_t idesc = idesc_f16(bn, 128);
            Ring rs(NS);
            bool ok = true;
            int i = 0;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, i++) {
                const int ab = i & 1;
                if (!mbar_wait(acc_empty + 8 * ab, (uint32_t)((i >> 1) & 1) ^ 1u)) { ok = false; break; }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(ab * ncols);
                for (int ks = 0; ks < nks; ks++) {
                    if (!mbar_poll(a_full + 8 * rs.idx, rs.phase) || !mbar_poll(b_full + 8 * rs.idx, rs.phase)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint32_t a_base = s_addr(As + rs.idx * 16384), b_base = s_addr(Bs + (size_t)rs.idx * bbytes);
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        umma(acc, sdesc(a_base + 32 * j), sdesc(b_base + 32 * j), idesc, (ks > 0 || j > 0) ? 1u : 0u);
                    umma_commit(st_empty + 8 * rs.idx);
                    rs.next();
                }
                if (ok) umma_commit(acc_full + 8 * ab);
            }
            if (!ok) report_timeout(g_err, 4);
            // Wait until every MMA this lane issued has completed before teardown.
            umma_commit(drained);
            if (!mbar_wait(drained, 0)) report_timeout(g_err, 5);
        }
    } else if (warp >= DEC_WARP0) {  // --------------------------------------- decode
        // Two groups of four warps take alternate k steps (group g the steps k = g mod 2 of
        // the CTA's sequence), so two chunks are decoded at once and each wait/arrive covers
        // twice the work. Thread dt of a group decodes chunk c = dt % 8 of rows r0 + 16*it
        // (it = 0..7); the swizzled position of that chunk is the same for all eight rows.
        const int grp = (warp - DEC_WARP0) / DEC_WARPS_PER_GROUP;
        const int dt = threadIdx.x - (DEC_WARP0 + grp * DEC_WARPS_PER_GROUP) * 32;
        const int c = dt & 7, r0 = dt >> 3;
        const int a_off = r0 * 128 + ((c ^ (r0 & 7)) << 4);
        Ring rr(NR), rs(NS);
        if (grp) { rr.next(); rs.next(); }
        bool ok = true;
        int k = 0;  // position in the CTA's sequence of k steps
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            for (int ks = 0; ks < nks; ks++, k++) {
                if ((k & 1) != grp) continue;
                if (!warp_wait_all(raw_full + 8 * rr.idx, rr.phase)) { ok = false; break; }
                const uint8_t* raw = Rs + rr.idx * cb;
                uint4 v[8];
#pragma unroll
                for (int it = 0; it < 8; it++) v[it] = decode8<TYPE>(raw, r0 + 16 * it, c);
                __syncwarp();
                if (lane == 0) mbar_arrive(raw_empty + 8 * rr.idx);
                rr.next();
                rr.next();
                if (!warp_wait_all(st_empty + 8 * rs.idx, rs.phase ^ 1u)) { ok = false; break; }
                uint8_t* A = As + rs.idx * 16384 + a_off;
#pragma unroll
                for (int it = 0; it < 8; it++) *(uint4*)(A + it * 16 * 128) = v[it];
                fence_proxy_async();  // each writer's generic-proxy stores -> visible to the tensor core
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full + 8 * rs.idx);
                rs.next();
                rs.next();
            }
        }
        if (!ok) report_timeout(g_err, 6);
    } else if (warp >= 4) {  // ------------------------------------------------- epilogue
        // Warp w reads TMEM lanes 32*(w%4) .. +31 = weight rows of the unit's tile. The CTA's
        // last unit is drained by these warps and the (then idle) decoder warps together,
        // a third of the columns each (see drain_share).
        const int q = warp & 3;
        constexpr bool counter_split = CSPLIT;
        pdl_wait();
        int i = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, i++) {
            int tile, tt, sp;
            unit_coords(u, splits, ttiles, tile, tt, sp);
            const int t0 = tt * bn, ab = i & 1;
            const bool w = warp_wait_all(acc_full + 8 * ab, (uint32_t)((i >> 1) & 1));
            const bool ready = counter_split ? epi_all(w) : w;
            tc_fence_after();
            if (!ready) {
                if (lane == 0) report_timeout(g_err, 7);
                break;
            }
            const uint32_t tacc = tmem + (uint32_t)(ab * ncols) + ((uint32_t)(q * 32) << 16);
            const int n = tile * 128 + q * 32 + lane;
            const int tn = min(bn, T - t0);  // valid columns of this token tile
            float* mine = splits > 1 ? g_ws + (int64_t)sp * T * ldy : nullptr;
            if (counter_split) {
                // Both K halves publish their partial; the unit that finishes last adds the
                // other half to its own (still in TMEM): p0 + p1, the same value whichever
                // unit that is (IEEE addition commutes).
                drain_cols(tacc, 0, bn, DR_RAW, lane, q, n, tile, t0, tn, tpad, ldy, mine, nullptr, g_xs_out, g_err);
                __threadfence();
                epi_bar();
                if (warp == 4 && lane == 0) {
                    int* ctr = g_ctr + tile * ttiles + tt;
                    int old = atomicAdd(ctr, 1);
                    int is_last = old == splits - 1;
                    if (is_last) atomicExch(ctr, 0);
                    *last_flag = is_last;
                }
                epi_bar();
                const bool last = *last_flag != 0;
                epi_bar();  // the flag is re-used by the next unit
                if (last) {
                    __threadfence();
                    drain_cols(tacc, 0, bn, epi == EPI_ADD ? DR_ADD : DR_STORE, lane, q, n, tile, t0, tn, tpad, ldy, g_y,
                               g_ws + (int64_t)(1 - sp) * T * ldy, g_xs_out, g_err);
                }
            } else {
                const int cend = u + (int)gridDim.x >= units ? drain_share(bn, 1) : bn;  // last unit: share 0
                const int kind = epi == EPI_PARTIAL ? DR_RAW : epi == EPI_SWIGLU ? DR_SWIGLU : epi == EPI_ADD ? DR_ADD : DR_STORE;
                drain_cols(tacc, 0, cend, kind, lane, q, n, tile, t0, tn, tpad, ldy, epi == EPI_PARTIAL ? mine : g_y, nullptr,
                           g_xs_out, g_err);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + 8 * ab);
        }
    }
    // The decoder warps, done with the main loop, drain two thirds of the last unit's columns
    // (the epilogue warps drain the first third), so the tail after the last MMA is short.
    if (warp >= DEC_WARP0 && !CSPLIT && (int)blockIdx.x < units) {
        const int my_units = (units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
        const int il = my_units - 1, ul = (int)blockIdx.x + il * (int)gridDim.x;
        int tile, tt, sp;
        unit_coords(ul, splits, ttiles, tile, tt, sp);
        const int ab = il & 1, q = warp & 3, grp = (warp - DEC_WARP0) / DEC_WARPS_PER_GROUP;
        pdl_wait();
        // `drained` (one phase, committed after the CTA's last MMA) rather than the last unit's
        // acc_full: these warps never waited on the earlier units' phases, so with few k steps a
        // unit two back could still be open and a parity test of acc_full would pass early.
        const bool ready = warp_wait_all(drained, 0u);
        tc_fence_after();
        if (ready) {
            const int t0 = tt * bn;
            const uint32_t tacc = tmem + (uint32_t)(ab * ncols) + ((uint32_t)(q * 32) << 16);
            const int kind = epi == EPI_PARTIAL ? DR_RAW : epi == EPI_SWIGLU ? DR_SWIGLU : epi == EPI_ADD ? DR_ADD : DR_STORE;
            drain_cols(tacc, drain_share(bn, grp + 1), drain_share(bn, grp + 2), kind, lane, q, tile * 128 + q * 32 + lane, tile,
                       t0, min(bn, T - t0), tpad, ldy, epi == EPI_PARTIAL ? g_ws + (int64_t)sp * T * ldy : g_y, nullptr,
                       g_xs_out, g_err);
        } else {
            report_timeout(g_err, 8);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * ncols);
    }
}

// ------------------------------------------------------------------------------------------------
// k_gemm_tm: the same product with the decoded weights (the MMA's A operand) in tensor memory.
//
// In k_gemm_tc every k step moves ~113 KB through shared memory at N = 256 (raw chunk in and
// out, decoded weights in and out, the activation tile in and the tensor core's reads of both
// operands), which at ~128 B per clock is ~880 clocks against the 512 the four MMAs need; the
// tensor pipe idles half the time. Here:
//   * the decoder warps read each weight row straight from global memory (L2, kept ahead by a
//     bulk L2 prefetch) into registers — no raw chunk in shared memory;
//   * they write the decoded fp16 row into TMEM (tcgen05.st, one row per lane, fp16 pairs (2j,
//     2j + 1) in column j) and the MMA reads A from there (tcgen05.mma ... [d], [a], b_desc);
//   * shared memory holds only the activation ring (7 stages at N = 224).
// TMEM (512 columns): accumulator 0 in [0, bn), A stage 0 in [224, 256), accumulator 1 in
// [256, 256 + bn), A stage 1 in [480, 512); so bn <= 224. Decoder group g (warps 8 + 4g ..
// 11 + 4g, one TMEM lane quarter each) decodes the k steps g, g + 2, ... of the CTA's sequence
// into A stage g. Everything else (units, epilogues, bounded waits, batch invariance) is k_gemm_tc's.
constexpr int TM_MAX_BN = 224;
constexpr int TM_PREFETCH = 24;  // own k steps whose weight chunks a decoder group keeps in flight to L2

__device__ __forceinline__ uint32_t tm_a_col(int g) { return 224u + 256u * (uint32_t)g; }

// D (TMEM) (+)= A (TMEM, fp16 pairs two to a column) x B (shared-memory descriptor).
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "r"(tmem_a), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}
// 32 consecutive TMEM columns of this warp's 32 lanes, one row of 64 fp16 weights per lane.
__device__ __forceinline__ void tm_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,"
        "%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tm_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// The raw bytes of one weight row (64 weights = two 32-wide blocks) of one chunk, in registers.
template <int TYPE>
struct RowRaw {
    uint4 q[TYPE == T_Q8_0 ? 4 : 2];  // Q8_0: 64 int8; Q4_0 / Q5_1: two blocks of 16 nibble-pair bytes
    uint32_t d;                       // fp16 d of blocks 0 and 1
    uint32_t m;                       // Q5_1: fp16 m of blocks 0 and 1
    uint2 qh;                         // Q5_1: the fifth bits of blocks 0 and 1
};

template <int TYPE>
__device__ __forceinline__ void row_load(RowRaw<TYPE>& r, const uint8_t* __restrict__ chunk, int row) {
    if (TYPE == T_Q8_0) {
        const uint4* q = (const uint4*)(chunk + row * 64);
#pragma unroll
        for (int i = 0; i < 4; i++) r.q[i] = __ldg(q + i);
        r.d = __ldg((const uint32_t*)(chunk + 8192 + row * 4));
    } else {
        const uint4* q = (const uint4*)(chunk + row * 32);
        r.q[0] = __ldg(q);
        r.q[1] = __ldg(q + 1);
        if (TYPE == T_Q4_0) {
            r.d = __ldg((const uint32_t*)(chunk + 4096 + row * 4));
        } else {
            r.qh = __ldg((const uint2*)(chunk + 4096 + row * 8));
            r.d = __ldg((const uint32_t*)(chunk + 5120 + row * 4));
            r.m = __ldg((const uint32_t*)(chunk + 5632 + row * 4));
        }
    }
}

__device__ __forceinline__ uint32_t w_at(const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// The row's 64 weights decoded to fp16 with exactly decode8's arithmetic: column j of the
// result holds weights (2j, 2j + 1).
template <int TYPE>
__device__ __forceinline__ void row_decode(const RowRaw<TYPE>& r, uint32_t (&v)[32]) {
    const __half2 d0 = __half2half2(__ushort_as_half((unsigned short)(r.d & 0xFFFFu)));
    const __half2 d1 = __half2half2(__ushort_as_half((unsigned short)(r.d >> 16)));
    if constexpr (TYPE == T_Q8_0) {
        const __half2 bias = __floats2half2_rn(1152.f, 1152.f);  // 1024 + 128
#pragma unroll
        for (int i = 0; i < 16; i++) {  // word i = weights 4i .. 4i + 3
            const uint32_t x = w_at(r.q[i >> 2], i & 3) ^ 0x80808080u;
            const __half2 d = i < 8 ? d0 : d1;
            v[2 * i] = hu(__hmul2(__hsub2(byte_pair(x, 0x4140u), bias), d));
            v[2 * i + 1] = hu(__hmul2(__hsub2(byte_pair(x, 0x4342u), bias), d));
        }
    } else {
        // Q4_0 / Q5_1: block b's byte j holds weight j (low nibble) and j + 16 (high nibble).
#pragma unroll
        for (int b = 0; b < 2; b++) {
            const __half2 d = b ? d1 : d0;
            __half2 m2 = __float2half2_rn(0.f);
            uint32_t qh = 0;
            if (TYPE == T_Q5_1) {
                m2 = __half2half2(__ushort_as_half((unsigned short)(b ? (r.m >> 16) : (r.m & 0xFFFFu))));
                qh = b ? r.qh.y : r.qh.x;
            }
#pragma unroll
            for (int half = 0; half < 2; half++) {  // weights 16 * half .. 16 * half + 15 of the block
#pragma unroll
                for (int i = 0; i < 4; i++) {       // word i of the block: bytes 4i .. 4i + 3
                    uint32_t x = w_at(r.q[b], i);
                    x = half ? (x >> 4) & 0x0F0F0F0Fu : x & 0x0F0F0F0Fu;
                    const int e = 16 * half + 4 * i;  // first weight of these four within the block
                    const int col = 16 * b + e / 2;
                    if (TYPE == T_Q4_0) {
                        const __half2 bias = __floats2half2_rn(1032.f, 1032.f);  // 1024 + 8
                        v[col] = hu(__hmul2(__hsub2(byte_pair(x, 0x4140u), bias), d));
                        v[col + 1] = hu(__hmul2(__hsub2(byte_pair(x, 0x4342u), bias), d));
                    } else {
                        const uint32_t h4 = (qh >> e) & 0xFu;
                        x |= ((h4 & 1u) << 4) | ((h4 & 2u) << 11) | ((h4 & 4u) << 18) | ((h4 & 8u) << 25);
                        const __half2 bias = __floats2half2_rn(1024.f, 1024.f);
                        v[col] = hu(__hfma2(__hsub2(byte_pair(x, 0x4140u), bias), d, m2));
                        v[col + 1] = hu(__hfma2(__hsub2(byte_pair(x, 0x4342u), bias), d, m2));
                    }
                }
            }
        }
    }
}

template <int TYPE, int EPI, bool CSPLIT>
__global__ void __launch_bounds__(GEMM_THREADS, 1) k_gemm_tm(TcParams p) {
    const uint8_t* __restrict__ g_w = p.w;
    const __half* __restrict__ g_x = p.x;
    float* __restrict__ g_y = p.y;
    int* __restrict__ g_err = p.err;
    __half* __restrict__ g_xs_out = p.xs_out;
    float* g_ws = p.ws;
    int* __restrict__ g_ctr = p.counters;
    constexpr int epi = EPI;
    const int ksteps = p.ksteps, T = p.T, tpad = p.tpad, bn = p.bn, ldy = p.ldy;
    const int splits = p.splits, ttiles = p.ttiles, units = p.units, NB = p.ns;
    const int bar_off = p.bar_off;
    extern __shared__ uint8_t gsm_raw[];
    uint8_t* sm = gsm_raw + ((1024u - (s_addr(gsm_raw) & 1023u)) & 1023u);
    const int cb = chunk_bytes(TYPE);
    uint8_t* Bs = sm;  // NB x bn*128 activation tiles
    uint64_t* bars = (uint64_t*)(sm + bar_off);
    // b_full (activation tile landed), b_empty (the MMA that read it completed), a_full (four
    // decoder warps wrote the A stage), a_empty (the MMA that read the A stage completed)
    const uint32_t b_full = s_addr(bars), b_empty = b_full + 8 * NB;
    const uint32_t a_full = b_empty + 8 * NB, a_empty = a_full + 16;
    const uint32_t acc_full = a_empty + 16, acc_empty = acc_full + 16, drained = acc_empty + 16;
    uint32_t* tslot = (uint32_t*)(bars + 2 * NB + 9);
    volatile int* last_flag = (volatile int*)(tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nks = ksteps / splits;
    const uint32_t bbytes = (uint32_t)bn * 128u;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NB; i++) { mbar_init(b_full + 8 * i, 1); mbar_init(b_empty + 8 * i, 1); }
        for (int i = 0; i < 2; i++) {
            mbar_init(a_full + 8 * i, DEC_WARPS_PER_GROUP);
            mbar_init(a_empty + 8 * i, 1);
            mbar_init(acc_full + 8 * i, 1);
            mbar_init(acc_empty + 8 * i, 4);
        }
        mbar_init(drained, 1);
        fence_barrier_init();
    }
    if (warp == 2) tmem_alloc(s_addr(tslot), 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_launch_dependents();

    if (warp == 3) {
        if (lane == 0) {  // ------------------------------------------ activation producer
            Ring r(NB);
            bool ok = true;
            int issued = 0;
            pdl_wait();
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                int tile, tt, sp;
                unit_coords(u, splits, ttiles, tile, tt, sp);
                const int kb = sp * nks, t0 = tt * bn;
                const uint8_t* src = (const uint8_t*)(g_x + ((int64_t)kb * tpad + t0) * 64);
                for (int ks = 0; ks < nks; ks++) {
                    if (!mbar_wait(b_empty + 8 * r.idx, r.phase ^ 1u)) { ok = false; break; }
                    mbar_expect_tx(b_full + 8 * r.idx, bbytes);
                    bulk_g2s(s_addr(Bs + (size_t)r.idx * bbytes), src + (int64_t)ks * tpad * 128, bbytes, b_full + 8 * r.idx);
                    r.next();
                    issued++;
                }
            }
            if (!ok) report_timeout(g_err, 2);
            for (int i = 0; i < issued && i < NB; i++) {
                r.prev();
                if (!mbar_wait(b_full + 8 * r.idx, r.phase)) report_timeout(g_err, 3);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // --------------------------------------------- MMA issue
            const uint32_t idesc = idesc_f16(bn, 128);
            Ring rb(NB);
            bool ok = true;
            int i = 0, k = 0;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, i++) {
                const int ab = i & 1;
                if (!mbar_wait(acc_empty + 8 * ab, (uint32_t)((i >> 1) & 1) ^ 1u)) { ok = false; break; }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(ab * 256);
                for (int ks = 0; ks < nks; ks++, k++) {
                    const int sa = k & 1;
                    if (!mbar_poll(a_full + 8 * sa, (uint32_t)((k >> 1) & 1)) || !mbar_poll(b_full + 8 * rb.idx, rb.phase)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_t = tmem + tm_a_col(sa), b_base = s_addr(Bs + (size_t)rb.idx * bbytes);
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        umma_ts(acc, a_t + 8u * j, sdesc(b_base + 32 * j), idesc, (ks > 0 || j > 0) ? 1u : 0u);
                    umma_commit(b_empty + 8 * rb.idx);
                    umma_commit(a_empty + 8 * sa);
                    rb.next();
                }
                if (ok) umma_commit(acc_full + 8 * ab);
            }
            if (!ok) report_timeout(g_err, 4);
            umma_commit(drained);
            if (!mbar_wait(drained, 0)) report_timeout(g_err, 5);
        }
    } else if (warp >= DEC_WARP0) {  // --------------------------------------- decode
        // Group g decodes the CTA's k steps g, g + 2, ... into A stage g; warp quarter q owns
        // TMEM lanes (rows) 32q .. 32q + 31, one row per lane. Each own step's weight rows are
        // loaded into registers one own step ahead (and their chunks prefetched into L2
        // TM_PREFETCH own steps ahead), so the loads fly while the previous step is decoded.
        const int grp = (warp - DEC_WARP0) / DEC_WARPS_PER_GROUP, q = warp & 3;
        const int row = 32 * q + lane;
        const uint32_t a_dst = tmem + ((uint32_t)(32 * q) << 16) + tm_a_col(grp);
        const int my_units = (int)blockIdx.x < units ? (units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
        const int total = my_units * nks;  // k steps in the CTA's sequence
        auto chunk_of = [&](int k) -> const uint8_t* {
            const int i = k / nks, ks = k - i * nks;
            int tile, tt, sp;
            unit_coords((int)blockIdx.x + i * (int)gridDim.x, splits, ttiles, tile, tt, sp);
            return g_w + ((int64_t)tile * ksteps + sp * nks + ks) * cb;
        };
        if (q == 0 && lane == 0)
            for (int k = grp; k < total && k < grp + 2 * TM_PREFETCH; k += 2) bulk_prefetch_l2(chunk_of(k), (uint32_t)cb);
        RowRaw<TYPE> nxt;
        if (grp < total) row_load<TYPE>(nxt, chunk_of(grp), row);
        bool ok = true;
        int n = 0;
        for (int k = grp; k < total; k += 2, n++) {
            const RowRaw<TYPE> cur = nxt;
            if (k + 2 < total) row_load<TYPE>(nxt, chunk_of(k + 2), row);
            if (q == 0 && lane == 0 && k + 2 * TM_PREFETCH < total) bulk_prefetch_l2(chunk_of(k + 2 * TM_PREFETCH), (uint32_t)cb);
            uint32_t v[32];
            row_decode<TYPE>(cur, v);
            if (!warp_wait_all(a_empty + 8 * grp, (uint32_t)(n & 1) ^ 1u)) { ok = false; break; }
            tc_fence_after();
            tm_st32(a_dst, v);
            tm_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(a_full + 8 * grp);
        }
        if (!ok) report_timeout(g_err, 6);
    } else if (warp >= 4) {  // ------------------------------------------------- epilogue
        const int q = warp & 3;
        constexpr bool counter_split = CSPLIT;
        pdl_wait();
        int i = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, i++) {
            int tile, tt, sp;
            unit_coords(u, splits, ttiles, tile, tt, sp);
            const int t0 = tt * bn, ab = i & 1;
            const bool w = warp_wait_all(acc_full + 8 * ab, (uint32_t)((i >> 1) & 1));
            const bool ready = counter_split ? epi_all(w) : w;
            tc_fence_after();
            if (!ready) {
                if (lane == 0) report_timeout(g_err, 7);
                break;
            }
            const uint32_t tacc = tmem + (uint32_t)(ab * 256) + ((uint32_t)(q * 32) << 16);
            const int nrow = tile * 128 + q * 32 + lane;
            const int tn = min(bn, T - t0);
            float* mine = splits > 1 ? g_ws + (int64_t)sp * T * ldy : nullptr;
            if (counter_split) {
                drain_cols(tacc, 0, bn, DR_RAW, lane, q, nrow, tile, t0, tn, tpad, ldy, mine, nullptr, g_xs_out, g_err);
                __threadfence();
                epi_bar();
                if (warp == 4 && lane == 0) {
                    int* ctr = g_ctr + tile * ttiles + tt;
                    int old = atomicAdd(ctr, 1);
                    int is_last = old == splits - 1;
                    if (is_last) atomicExch(ctr, 0);
                    *last_flag = is_last;
                }
                epi_bar();
                const bool last = *last_flag != 0;
                epi_bar();
                if (last) {
                    __threadfence();
                    drain_cols(tacc, 0, bn, epi == EPI_ADD ? DR_ADD : DR_STORE, lane, q, nrow, tile, t0, tn, tpad, ldy, g_y,
                               g_ws + (int64_t)(1 - sp) * T * ldy, g_xs_out, g_err);
                }
            } else {
                const int cend = u + (int)gridDim.x >= units ? drain_share(bn, 1) : bn;
                const int kind = epi == EPI_PARTIAL ? DR_RAW : epi == EPI_SWIGLU ? DR_SWIGLU : epi == EPI_ADD ? DR_ADD : DR_STORE;
                drain_cols(tacc, 0, cend, kind, lane, q, nrow, tile, t0, tn, tpad, ldy, epi == EPI_PARTIAL ? mine : g_y, nullptr,
                           g_xs_out, g_err);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + 8 * ab);
        }
    }
    // The decoder warps, done with the main loop, drain two thirds of the last unit's columns.
    if (warp >= DEC_WARP0 && !CSPLIT && (int)blockIdx.x < units) {
        const int my_units = (units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
        const int il = my_units - 1, ul = (int)blockIdx.x + il * (int)gridDim.x;
        int tile, tt, sp;
        unit_coords(ul, splits, ttiles, tile, tt, sp);
        const int ab = il & 1, q = warp & 3, grp = (warp - DEC_WARP0) / DEC_WARPS_PER_GROUP;
        pdl_wait();
        // `drained` (one phase, committed after the CTA's last MMA) rather than the last unit's
        // acc_full: these warps never waited on the earlier units' phases, so with few k steps a
        // unit two back could still be open and a parity test of acc_full would pass early.
        const bool ready = warp_wait_all(drained, 0u);
        tc_fence_after();
        if (ready) {
            const int t0 = tt * bn;
            const uint32_t tacc = tmem + (uint32_t)(ab * 256) + ((uint32_t)(q * 32) << 16);
            const int kind = epi == EPI_PARTIAL ? DR_RAW : epi == EPI_SWIGLU ? DR_SWIGLU : epi == EPI_ADD ? DR_ADD : DR_STORE;
            drain_cols(tacc, drain_share(bn, grp + 1), drain_share(bn, grp + 2), kind, lane, q, tile * 128 + q * 32 + lane, tile,
                       t0, min(bn, T - t0), tpad, ldy, epi == EPI_PARTIAL ? g_ws + (int64_t)sp * T * ldy : g_y, nullptr,
                       g_xs_out, g_err);
        } else {
            report_timeout(g_err, 8);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// Token tiles of a pass of T tokens: ceil(T / max) balanced tiles, multiples of 16, max = 256 (the
// MMA's N limit) for k_gemm_tc and 224 for k_gemm_tm (the widest accumulator that leaves room for
// two A stages in TMEM). From 128 to max tokens a
// product with few row tiles (the 48-tile QKV, the split 24-tile projections) takes two tiles of
// T / 2 so that it still covers most SMs; one with many row tiles (gate/up, the head) keeps one
// tile of T, which halves its MMA instructions and still fills the SMs. tpad is a multiple of both.
enum GemmKernel : int { GK_1SM = 1, GK_TMEM = 2 };
static bool gemm_on_smem_a();
static int gemm_max_bn() { return gemm_on_smem_a() ? 256 : TM_MAX_BN; }
int gemm_tpad_for(int T) {
    const int mx = gemm_max_bn();
    if (T >= 128 && T <= mx) return 2 * (((T + 1) / 2 + 15) / 16 * 16);
    const int n = T > 0 ? (T + mx - 1) / mx : 1;
    const int bn = ((T + n - 1) / n + 15) / 16 * 16;
    return n * (bn < 16 ? 16 : bn);
}
// units_per_tile = row tiles x K splits of the product.
int gemm_bn_for(int T, int units_per_tile, int sm_count) {
    const int tpad = gemm_tpad_for(T);
    const int mx = gemm_max_bn();
    if (T >= 128 && T <= mx) return units_per_tile * 4 >= sm_count * 3 ? tpad : tpad / 2;
    const int n = T > 0 ? (T + mx - 1) / mx : 1;
    return tpad / n;
}

static int g_sm_count = 0;

// The prefill GEMM kernel: k_gemm_tc, or with JV_GEMM_KERNEL=tmem k_gemm_tm (decoded weights in
// TMEM, token tiles of at most 224). Both give the same bits (test_gemm_kernels_are_bit_identical).
static GemmKernel gemm_kernel_choice() {
    static const GemmKernel v = [] {
        const char* e = getenv("JV_GEMM_KERNEL");
        if (e != nullptr && strcmp(e, "tmem") == 0) return GK_TMEM;
        return GK_1SM;
    }();
    return v;
}
static bool gemm_on_smem_a() { return gemm_kernel_choice() != GK_TMEM; }

template <int TYPE, int EPI, bool CSPLIT>
static void launch_tc_typed(const GemmArgs& a, cudaStream_t s) {
    const QWeight& w = *a.w;
    TcParams p{};
    p.w = w.data;
    p.x = a.x;
    p.y = a.y;
    p.err = a.err;
    p.xs_out = a.xs_out;
    p.ws = a.ws;
    p.counters = a.counters;
    p.ksteps = w.ksteps;
    p.T = a.T;
    p.tpad = a.tpad;
    p.bn = a.bn;
    p.ldy = a.ldy;
    p.epilogue = a.epilogue;
    p.splits = a.splits;
    p.tiles = w.tiles;
    p.ttiles = a.tpad / a.bn;
    p.units = p.tiles * p.ttiles * p.splits;
    const int cb = chunk_bytes(TYPE);
    int nc = 32;
    while (nc < a.bn) nc <<= 1;
    p.ncols = nc;
    if (!gemm_on_smem_a()) {
        // k_gemm_tm: shared memory holds only the activation ring (up to 8 stages in ~222 KB).
        if (TYPE == T_QX) throw Error(JV_ERR_UNSUPPORTED, "gemm: the TMEM-operand kernel takes Q8_0, Q5_1 and Q4_0 only");
        if (a.bn > TM_MAX_BN) throw Error(JV_ERR_ARG, "gemm: token tile above 224 for the TMEM-operand kernel");
        const size_t budget = 222 * 1024, stage = (size_t)a.bn * 128;
        p.ns = (int)std::min<size_t>(8, budget / stage);
        p.nr = 0;
        p.b_off = 0;
        p.raw_off = 0;
        p.bar_off = (int)(stage * p.ns);
        // at least ~120 KB so that one CTA holds the SM (TMEM is allocated whole)
        size_t smem = std::max<size_t>((size_t)p.bar_off + 8 * (2 * p.ns + 9) + 16 + 1024, 120 * 1024);
        JV_CUDA(cudaFuncSetAttribute(k_gemm_tm<TYPE, EPI, CSPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        if (g_sm_count == 0) {
            int dev = 0;
            JV_CUDA(cudaGetDevice(&dev));
            JV_CUDA(cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev));
        }
        launch_pdl(k_gemm_tm<TYPE, EPI, CSPLIT>, dim3(std::min(p.units, g_sm_count)), dim3(GEMM_THREADS), smem, s, p);
        note_launch();
        return;
    }
    // Ring depths and offsets (gemm_plan.h: the raw ring is even, or at least NS + 2 slots, so
    // the decoder groups' parity waits are exact).
    GemmRingPlan plan;
    if (!gemm_ring_plan(a.bn, cb, &plan)) throw Error(JV_ERR_ARG, "gemm: shared memory budget exceeded");
    p.ns = plan.ns;
    p.nr = plan.nr;
    p.b_off = plan.b_off;
    p.raw_off = plan.raw_off;
    p.bar_off = plan.bar_off;
    const size_t smem = plan.smem;
    JV_CUDA(cudaFuncSetAttribute(k_gemm_tc<TYPE, EPI, CSPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (g_sm_count == 0) {
        int dev = 0;
        JV_CUDA(cudaGetDevice(&dev));
        JV_CUDA(cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev));
    }
    int grid = std::min(p.units, g_sm_count);
    launch_pdl(k_gemm_tc<TYPE, EPI, CSPLIT>, dim3(grid), dim3(GEMM_THREADS), smem, s, p);
    note_launch();
}

template <int TYPE>
static void launch_tc_epi(const GemmArgs& a, cudaStream_t s) {
    const bool cs = a.splits > 1;
    switch (a.epilogue) {
        case EPI_STORE: cs ? launch_tc_typed<TYPE, EPI_STORE, true>(a, s) : launch_tc_typed<TYPE, EPI_STORE, false>(a, s); break;
        case EPI_ADD: cs ? launch_tc_typed<TYPE, EPI_ADD, true>(a, s) : launch_tc_typed<TYPE, EPI_ADD, false>(a, s); break;
        case EPI_SWIGLU: launch_tc_typed<TYPE, EPI_SWIGLU, false>(a, s); break;
        case EPI_PARTIAL: launch_tc_typed<TYPE, EPI_PARTIAL, false>(a, s); break;
        default: throw Error(JV_ERR_ARG, "gemm: bad epilogue");
    }
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
        case T_Q8_0: launch_tc_epi<T_Q8_0>(a, s); break;
        case T_Q4_0: launch_tc_epi<T_Q4_0>(a, s); break;
        case T_Q5_1: launch_tc_epi<T_Q5_1>(a, s); break;
        case T_QX: launch_tc_epi<T_QX>(a, s); break;
        default: throw Error(JV_ERR_UNSUPPORTED, "gemm: weight type not on the B200 path");
    }
}

// ------------------------------------------------------- reference GEMM

// A plain CUDA-core product over the *same* fp16 operands (weights decoded and rounded to
// fp16 exactly as the tensor-core producer does). Selected only by the JV_GEMM_REFERENCE
// environment variable, to check the tcgen05 kernel at full shapes; never the default path.
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
        case T_QX: k_gemm_ref<T_QX><<<grid, 128, 0, s>>>(a.w->data, a.w->ksteps, a.x, a.T, a.tpad, a.y, a.ldy, a.epilogue); break;
        default: k_gemm_ref<T_Q5_1><<<grid, 128, 0, s>>>(a.w->data, a.w->ksteps, a.x, a.T, a.tpad, a.y, a.ldy, a.epilogue); break;
    }
    note_launch();
}

}  // namespace jv
