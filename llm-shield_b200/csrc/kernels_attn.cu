// kernels_attn.cu — tree-masked grouped-query attention over the paged fp16 KV cache.
//
// Semantics (reference src/Jevstral/Model/MinistralModel.cs:446-636 and
// src/Jevstral/Numerics/AttentionKernels.cs): token t of a pass sees the cache slots
// [0, shared) and [segment, slot], in that order, and nothing else — the trunk is causal,
// each branch sees the whole trunk plus its own earlier tokens and never a sibling.
//
// Keys are walked in *logical* order: logical index L < shared is slot base + L (base is 0 except
// in a batch of independent trees), L >= shared is slot segment + (L - shared). Blocks of 64 keys are cut on logical indices, so a token
// meets exactly the same key blocks, in the same order and at the same positions inside
// each block, whether it runs in a tree, alone after the trunk, or after a cached prefix.
// With a block that a row cannot see being an exact no-op (max unchanged, rescale factor
// exactly 1, probabilities exactly 0), a token's output is bit-identical across all three
// (the reference's DeciderTests.BranchesMatchRunningEachContinuationAlone property).
//
// Prefill kernel: one CTA = one KV head × up to 32 tokens of one segment; its 4 query
// heads ride in the M dimension (128 rows = 32 tokens × 4 heads, 8 warps), so every K/V byte
// read feeds all the heads that share it. K/V blocks of 64 keys stream through a 3-deep
// cp.async ring. fp16 operands, fp32 accumulation and online softmax.
#include "jv_internal.h"

namespace jv {

constexpr int ATT_THREADS = 256;  // 8 warps x 16 query rows
constexpr int ATT_KEYS = 64;      // keys per block
constexpr int ATT_ROWS = 128;     // query rows per CTA: ATT_ITEM_TOKENS tokens x 4 heads
constexpr int ATT_STAGES = 3;     // K/V blocks in flight: the one being used and two ahead
constexpr int ATT_HD = 128;
constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *(uint32_t*)&h;
}

// Row r of a [rows][128] fp16 tile: 16-byte chunk c lives at chunk c ^ (r & 7).
__device__ __forceinline__ int swz(int r, int c) { return r * ATT_HD + ((c ^ (r & 7)) << 3); }

// The (layer, head, K|V) plane of the page holding `slot`, and the slot's row in it.
__device__ __forceinline__ const char* kv_plane(const __half* pool, const int32_t* page_table, int64_t page_bytes,
                                                int page_slots, int layer, int kv_heads, int head, int kv, int slot,
                                                int& row, int* err) {
    row = slot % page_slots;
    return (const char*)pool + (int64_t)kv_page(page_table, slot, page_slots, err, BS_MMA_ATTN_PAGE) * page_bytes +
           kv_plane_offset(layer, kv_heads, head, kv, page_slots);
}

__global__ void __launch_bounds__(ATT_THREADS) k_attention(AttnArgs a) {
    extern __shared__ __align__(128) unsigned char att_smem[];
    __half* Qs = (__half*)att_smem;                 // [64][128]
    __half* Ks = Qs + ATT_ROWS * ATT_HD;                 // [stages][64][128]
    __half* Vs = Ks + ATT_STAGES * ATT_KEYS * ATT_HD;    // [stages][64][128]

    pdl_launch_dependents();
    pdl_wait();
    const AttnItem it = a.items[blockIdx.x];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int group = a.heads / a.kv_heads;  // 4 for Ministral-3 (asserted on the host)
    const int qdim = a.heads * ATT_HD;
    const int max_limit = it.shared + (it.slot0 + it.ntok - 1 - it.segment + 1);

    // Where every visible key lives, looked up once: (physical page << 8) | slot in page, so
    // that the block loads below issue their copies without a dependent page-table read.
    uint32_t* tab = (uint32_t*)(Vs + ATT_STAGES * ATT_KEYS * ATT_HD);
    for (int L0 = tid; L0 < max_limit; L0 += 4 * ATT_THREADS) {
        int slot[4], page[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int L = L0 + j * ATT_THREADS;
            slot[j] = L < it.shared ? it.base + L : it.segment + (L - it.shared);
            page[j] = L < max_limit ? kv_page(a.page_table, slot[j], a.page_slots, a.err, BS_MMA_ATTN_PAGE) : 0;
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int L = L0 + j * ATT_THREADS;
            if (L < max_limit) tab[L] = ((uint32_t)page[j] << 8) | (uint32_t)(slot[j] % a.page_slots);
        }
    }
    const int64_t head_off = (int64_t)((a.layer * a.kv_heads + it.kv_head) * 2) * a.page_slots * 256;
    const int64_t v_off = (int64_t)a.page_slots * 256;
    __syncthreads();

    // Q tile: row r = token (r / group) × head (r % group) of this KV head.
    for (int id = tid; id < ATT_ROWS * 16; id += ATT_THREADS) {
        int r = id >> 4, c = id & 15;
        int tl = r / group, j = r % group;
        const __half* src = a.q16;
        int bytes = 0;
        if (tl < it.ntok) {
            src = a.q16 + (int64_t)(it.t0 + tl) * qdim + (it.kv_head * group + j) * ATT_HD + c * 8;
            bytes = 16;
        }
        cp_async16(Qs + swz(r, c), src, bytes);
    }
    auto load_block = [&](int blk, int buf) {
        __half* kd = Ks + buf * ATT_KEYS * ATT_HD;
        __half* vd = Vs + buf * ATT_KEYS * ATT_HD;
        for (int id = tid; id < ATT_KEYS * 16; id += ATT_THREADS) {
            int r = id >> 4, c = id & 15;
            int L = blk * ATT_KEYS + r;
            const __half* ks = a.kv_pool;
            const __half* vs = a.kv_pool;
            int bytes = 0;
            if (L < max_limit) {
                const uint32_t e = tab[L];
                const char* plane = (const char*)a.kv_pool + (int64_t)(e >> 8) * a.page_bytes + head_off;
                const int off = kv_chunk_offset((int)(e & 255u), c, a.page_slots);
                ks = (const __half*)(plane + off);
                vs = (const __half*)(plane + v_off + off);
                bytes = 16;
            }
            cp_async16(kd + swz(r, c), ks, bytes);
            cp_async16(vd + swz(r, c), vs, bytes);
        }
    };
    // Blocks 0 and 1 in flight before the loop; each iteration issues block blk + 2 (an empty
    // group past the end), so waiting for all but the two newest groups means block blk landed.
    load_block(0, 0);
    cp_async_commit();
    if (it.nblocks > 1) load_block(1, 1);
    cp_async_commit();

    // Per-thread rows: r0 = 16*warp + g, r1 = r0 + 8.
    const int g = lane >> 2, q4 = lane & 3;
    const int rA = warp * 16 + g, rB = rA + 8;
    const int tlA = rA / group, tlB = rB / group;
    const int limA = tlA < it.ntok ? it.shared + (it.slot0 + tlA - it.segment + 1) : 1;
    const int limB = tlB < it.ntok ? it.shared + (it.slot0 + tlB - it.segment + 1) : 1;
    const float sl2 = a.scale * LOG2E;

    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
    uint32_t qa[8][4];

    for (int blk = 0; blk < it.nblocks; blk++) {
        const int buf = blk % ATT_STAGES;
        if (blk + 2 < it.nblocks) load_block(blk + 2, (blk + 2) % ATT_STAGES);
        cp_async_commit();
        cp_async_wait<2>();
        __syncthreads();
        if (blk == 0) {
#pragma unroll
            for (int kk = 0; kk < 8; kk++) {
                int r = warp * 16 + (lane & 15);
                int c = kk * 2 + (lane >> 4);
                ldsm_x4(qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], Qs + swz(r, c));
            }
        }
        const __half* kb = Ks + buf * ATT_KEYS * ATT_HD;
        const __half* vb = Vs + buf * ATT_KEYS * ATT_HD;

        // S = Q K^T for this warp's 16 rows x 64 keys.
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {
                uint32_t b0, b1, b2, b3;
                int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
                int c = kk * 2 + ((lane >> 3) & 1);
                ldsm_x4(b0, b1, b2, b3, kb + swz(key, c));
                mma16816(s[2 * np], qa[kk], b0, b1);
                mma16816(s[2 * np + 1], qa[kk], b2, b3);
            }
        }
        // Mask and online softmax (scores in log2 units: s * scale * log2 e).
        float bmA = -INFINITY, bmB = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            int L0 = blk * ATT_KEYS + nt * 8 + 2 * q4;
#pragma unroll
            for (int e = 0; e < 2; e++) {
                int L = L0 + e;
                s[nt][e] = L < limA ? s[nt][e] * sl2 : -INFINITY;
                s[nt][2 + e] = L < limB ? s[nt][2 + e] * sl2 : -INFINITY;
                bmA = fmaxf(bmA, s[nt][e]);
                bmB = fmaxf(bmB, s[nt][2 + e]);
            }
        }
        bmA = fmaxf(bmA, __shfl_xor_sync(0xffffffffu, bmA, 1));
        bmA = fmaxf(bmA, __shfl_xor_sync(0xffffffffu, bmA, 2));
        bmB = fmaxf(bmB, __shfl_xor_sync(0xffffffffu, bmB, 1));
        bmB = fmaxf(bmB, __shfl_xor_sync(0xffffffffu, bmB, 2));
        float nmA = fmaxf(mA, bmA), nmB = fmaxf(mB, bmB);
        float alA = nmA == -INFINITY ? 1.f : exp2f(mA - nmA);
        float alB = nmB == -INFINITY ? 1.f : exp2f(mB - nmB);
        float sumA = 0.f, sumB = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                float pa = s[nt][e] == -INFINITY ? 0.f : exp2f(s[nt][e] - nmA);
                float pb = s[nt][2 + e] == -INFINITY ? 0.f : exp2f(s[nt][2 + e] - nmB);
                s[nt][e] = pa;
                s[nt][2 + e] = pb;
                sumA += pa;
                sumB += pb;
            }
        }
        sumA += __shfl_xor_sync(0xffffffffu, sumA, 1);
        sumA += __shfl_xor_sync(0xffffffffu, sumA, 2);
        sumB += __shfl_xor_sync(0xffffffffu, sumB, 1);
        sumB += __shfl_xor_sync(0xffffffffu, sumB, 2);
        lA = lA * alA + sumA;
        lB = lB * alB + sumB;
        mA = nmA;
        mB = nmB;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            o[i][0] *= alA; o[i][1] *= alA;
            o[i][2] *= alB; o[i][3] *= alB;
        }
        // O += P V.
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t pa[4];
            pa[0] = pack_half2(s[2 * j][0], s[2 * j][1]);
            pa[1] = pack_half2(s[2 * j][2], s[2 * j][3]);
            pa[2] = pack_half2(s[2 * j + 1][0], s[2 * j + 1][1]);
            pa[3] = pack_half2(s[2 * j + 1][2], s[2 * j + 1][3]);
#pragma unroll
            for (int dp = 0; dp < 8; dp++) {
                uint32_t b0, b1, b2, b3;
                int key = j * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                int c = dp * 2 + (lane >> 4);
                ldsm_x4_t(b0, b1, b2, b3, vb + swz(key, c));
                mma16816(o[2 * dp], pa, b0, b1);
                mma16816(o[2 * dp + 1], pa, b2, b3);
            }
        }
        __syncthreads();
    }

    // Normalise and write the context rows: row -> (token, head), dims 8*nt + 2*q4 + {0,1}.
    float invA = 1.f / lA, invB = 1.f / lB;
#pragma unroll
    for (int half = 0; half < 2; half++) {
        int r = half ? rB : rA;
        int tl = r / group, j = r % group;
        if (tl >= it.ntok) continue;
        int t = it.t0 + tl;
        int head = it.kv_head * group + j;
        float inv = half ? invB : invA;
#pragma unroll
        for (int nt = 0; nt < 16; nt++) {
            int col = head * ATT_HD + nt * 8 + 2 * q4;
            float v0 = o[nt][2 * half] * inv, v1 = o[nt][2 * half + 1] * inv;
            if (a.ctx16) *(__half2*)(a.ctx16 + kslab_offset(t, col, a.tpad)) = __floats2half2_rn(v0, v1);
            if (a.ctx32) {
                a.ctx32[(int64_t)t * qdim + col] = v0;
                a.ctx32[(int64_t)t * qdim + col + 1] = v1;
            }
        }
    }
}

void launch_attention(const AttnArgs& a, cudaStream_t s) {
    if (a.n_items <= 0) return;
    if (a.page_slots > 256) throw Error(JV_ERR_UNSUPPORTED, "attention: pages of more than 256 slots");
    size_t smem = (size_t)(ATT_ROWS + 2 * ATT_STAGES * ATT_KEYS) * ATT_HD * sizeof(__half) + (size_t)a.max_keys * 4;
    if (smem > 227 * 1024) throw Error(JV_ERR_UNSUPPORTED, "attention: too many visible keys for one pass");
    static size_t configured = 0;
    if (smem > configured) {
        JV_CUDA(cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = smem;
    }
    launch_pdl(k_attention, dim3(a.n_items), dim3(ATT_THREADS), smem, s, a);
    note_launch();
}

// ------------------------------------------------------------ decode

// One query token (a decode step): split the visible keys [0, n_keys) over CTAs, each
// computing fp32 scores (a fused chain over d, times the scale), a local max-shifted
// softmax and the weighted value sum for the `group` heads of one KV head; a second kernel
// merges the splits in split order.
constexpr int DEC_KEYS = 64;

__global__ void k_decode_attention(DecodeAttnArgs a) {
    extern __shared__ float dsm[];
    const int group = a.heads / a.kv_heads;
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int k0 = split * DEC_KEYS, k1 = min(a.n_keys, k0 + DEC_KEYS);
    const int nk = k1 - k0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* qs = dsm;                      // [group][128]
    float* ps = qs + group * ATT_HD;      // [group][64]
    for (int i = threadIdx.x; i < group * ATT_HD; i += blockDim.x) qs[i] = a.q32[(int64_t)kvh * group * ATT_HD + i];
    __syncthreads();
    const int h = warp;  // one warp per query head of the group
    const float* q = qs + h * ATT_HD;
    float mx = -INFINITY;
    for (int i = lane; i < nk; i += 32) {
        int L = k0 + i;
        int slot = L < a.shared ? L : a.segment + (L - a.shared);
        int row;
        const char* k = kv_plane(a.kv_pool, a.page_table, a.page_bytes, a.page_slots, a.layer, a.kv_heads, kvh, 0, slot, row, a.err);
        float acc = 0.f;
        for (int d = 0; d < ATT_HD; d += 8) {
            int4 raw = *(const int4*)(k + kv_chunk_offset(row, d >> 3, a.page_slots));
            const __half2* kh = (const __half2*)&raw;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float2 kf = __half22float2(kh[e]);
                acc = fmaf(q[d + 2 * e], kf.x, acc);
                acc = fmaf(q[d + 2 * e + 1], kf.y, acc);
            }
        }
        float sc = acc * a.scale;
        ps[h * DEC_KEYS + i] = sc;
        mx = fmaxf(mx, sc);
    }
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __syncwarp();
    float l = 0.f;
    for (int i = lane; i < nk; i += 32) {
        float p = __expf(ps[h * DEC_KEYS + i] - mx);
        ps[h * DEC_KEYS + i] = p;
        l += p;
    }
    for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    __syncwarp();
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < nk; i++) {
        int L = k0 + i;
        int slot = L < a.shared ? L : a.segment + (L - a.shared);
        int row;
        const char* v = kv_plane(a.kv_pool, a.page_table, a.page_bytes, a.page_slots, a.layer, a.kv_heads, kvh, 1, slot, row, a.err);
        float p = ps[h * DEC_KEYS + i];
        uint2 raw = *(const uint2*)(v + kv_elem_offset(row, lane * 4, a.page_slots));
        const __half2* vh = (const __half2*)&raw;
        float2 v01 = __half22float2(vh[0]), v23 = __half22float2(vh[1]);
        acc[0] = fmaf(p, v01.x, acc[0]);
        acc[1] = fmaf(p, v01.y, acc[1]);
        acc[2] = fmaf(p, v23.x, acc[2]);
        acc[3] = fmaf(p, v23.y, acc[3]);
    }
    // partial layout: [head][split][2 + 128]
    int head = kvh * group + h;
    float* dst = a.partial + ((int64_t)head * a.splits + split) * (2 + ATT_HD);
    if (lane == 0) { dst[0] = mx; dst[1] = l; }
    for (int e = 0; e < 4; e++) dst[2 + lane * 4 + e] = acc[e];
}

__global__ void k_decode_combine(DecodeAttnArgs a) {
    int head = blockIdx.x, d = threadIdx.x;  // 128 threads
    const float* base = a.partial + (int64_t)head * a.splits * (2 + ATT_HD);
    float m = -INFINITY;
    for (int s = 0; s < a.splits; s++) m = fmaxf(m, base[(int64_t)s * (2 + ATT_HD)]);
    float l = 0.f, acc = 0.f;
    for (int s = 0; s < a.splits; s++) {
        const float* p = base + (int64_t)s * (2 + ATT_HD);
        float w = __expf(p[0] - m);
        l += w * p[1];
        acc += w * p[2 + d];
    }
    a.ctx32[(int64_t)head * ATT_HD + d] = acc / l;
}

void launch_decode_attention(const DecodeAttnArgs& a, cudaStream_t s) {
    int group = a.heads / a.kv_heads;
    dim3 grid(a.kv_heads, a.splits);
    size_t smem = (size_t)group * (ATT_HD + DEC_KEYS) * sizeof(float);
    k_decode_attention<<<grid, 32 * group, smem, s>>>(a);
    k_decode_combine<<<a.heads, ATT_HD, 0, s>>>(a);
    note_launch(2);
}

}  // namespace jv
