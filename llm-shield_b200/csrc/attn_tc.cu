// attn_tc.cu — tree-masked GQA prefill attention on the 5th-generation tensor cores.
//
// Semantics are those of k_attention (kernels_attn.cu; reference MinistralModel.cs:446-636):
// query row (token t, head h) sees logical keys L < limit(t), logical key L being cache slot L
// below `shared` and slot segment + (L - shared) above; keys are walked in logical order in
// blocks cut on logical indices, so a token's output is bit-identical whether it runs in a
// tree, alone after the trunk, or after a cached prefix.
//
// One CTA = one KV head x up to 32 tokens of one segment; the 4 query heads of the KV head ride
// in M (128 rows = TMEM lanes). Per block of 128 keys:
//   S  = Q K^T      tcgen05.mma kind::f16, M = 128, N = 128 keys, K = 128 dims -> TMEM (fp32)
//   P  = exp2(S * scale * log2 e - m)   softmax warps, one query row per thread, online max/sum,
//                                        O rescaled in TMEM when the row maximum moves
//   O += P V        M = 128, N = 128 dims, K = 128 keys; V read through an MN-major descriptor
// Warps 0-3 run the softmax and the output, warps 4-7 load Q and the K/V blocks (cp.async into
// a 2-deep ring, SWIZZLE_128B placement), warp 8 owns TMEM and issues the MMAs. S is double
// buffered, so the next block's Q K^T runs while this block's softmax does. Every wait is
// bounded (2 s of %globaltimer); on expiry the role records JV_ERR_DEVICE_TIMEOUT and stops.
#include "tc_common.cuh"

namespace jv {
namespace {

constexpr int AT_ROWS = 128;                 // 32 tokens x 4 query heads
constexpr int AT_KEYS = 128;                 // keys per block
constexpr int AT_THREADS = 288;              // 9 warps
constexpr int AT_TILE = 128 * 128 * 2;       // one [128][128] fp16 tile, two 16 KB halves
constexpr float AT_LOG2E = 1.4426950408889634f;

// Byte offset of 16-byte chunk c (0..15) of row r in a [128][128] fp16 tile stored as two
// SWIZZLE_128B halves (columns 0-63, then 64-127): row r at r * 128 B, chunk c & 7 at
// (c & 7) ^ (r & 7).
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
    return (uint32_t)((c >> 3) * 16384 + r * 128 + ((((c & 7) ^ (r & 7))) << 4));
}

// MN-major SWIZZLE_128B descriptor (the V operand of P V: N = dims contiguous): leading byte
// offset = distance between the two 64-dim halves, stride byte offset = 8 key rows.
__device__ __forceinline__ uint64_t sdesc_mn(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(16384u >> 4) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

__device__ __forceinline__ void cp16(uint32_t dst, const void* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// 32 consecutive TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,"
        "%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tld_wait(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                   "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}
__device__ __forceinline__ void tst32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,"
        "%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tst_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

// Bounded wait taken by a whole warp: every lane gets the same verdict, so the warp stays
// converged for the .sync.aligned tcgen05 instructions after it.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

__global__ void __launch_bounds__(AT_THREADS, 1) k_attn_tc(AttnArgs a) {
    extern __shared__ uint8_t at_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)at_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* Qs = sm;                       // [128 rows][128 dims]
    uint8_t* Ps = sm + AT_TILE;             // [128 rows][128 keys]
    uint8_t* KV = sm + 2 * AT_TILE;         // stage s: K tile at KV + s * 2 * AT_TILE, V tile after it
    uint32_t* tabs = (uint32_t*)(KV + 4 * AT_TILE);  // [2 stages][128 keys] (page << 8) | slot in page
    uint64_t* bars = (uint64_t*)(tabs + 2 * AT_KEYS);
    const uint32_t q_full = s_addr(bars), kv_full = q_full + 8, kv_empty = kv_full + 16, s_full = kv_empty + 16;
    const uint32_t s_empty = s_full + 16, p_full = s_empty + 16, o_done = p_full + 8;
    uint32_t* tslot = (uint32_t*)(bars + 11);
    volatile uint32_t* flags = tslot + 1;  // [2] loader stage verdicts

    pdl_launch_dependents();
    pdl_wait();
    const AttnItem it = a.items[blockIdx.x];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int group = a.heads / a.kv_heads;  // 4 (checked on the host)
    const int qdim = a.heads * 128;
    const int max_limit = it.shared + (it.slot0 + it.ntok - 1 - it.segment + 1);
    const int nb = (max_limit + AT_KEYS - 1) / AT_KEYS;

    if (tid == 0) {
        mbar_init(q_full, 128);
        for (int i = 0; i < 2; i++) {
            mbar_init(kv_full + 8 * i, 128);
            mbar_init(kv_empty + 8 * i, 1);
            mbar_init(s_full + 8 * i, 1);
            mbar_init(s_empty + 8 * i, 4);
        }
        mbar_init(p_full, 4);
        mbar_init(o_done, 1);
        fence_barrier_init();
    }
    if (warp == 8) tmem_alloc(s_addr(tslot), 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;  // O at columns 0-127, S buffers at 128-255 and 256-383
    int* err = a.err;

    if (warp >= 4 && warp < 8) {
        // ----------------------------------------------------------------- loaders
        const int lt = tid - 128;
        // Q: row r = token r / 4 x head r % 4 of this KV head
        for (int id = lt; id < AT_ROWS * 16; id += 128) {
            const int r = id >> 4, c = id & 15;
            const int tl = r / group, j = r % group;
            const bool ok = tl < it.ntok;
            const __half* src = ok ? a.q16 + (int64_t)(it.t0 + tl) * qdim + (it.kv_head * group + j) * 128 + c * 8 : a.q16;
            cp16(s_addr(Qs) + tile_off(r, c), src, ok ? 16 : 0);
        }
        cp_wait_all();
        fence_proxy_async();
        mbar_arrive(q_full);
        const int64_t head_off = (int64_t)((a.layer * a.kv_heads + it.kv_head) * 2) * a.page_slots * 256;
        const int64_t v_off = (int64_t)a.page_slots * 256;
        // where key lt of block b lives; the page-table read for block b + 1 is issued a block early
        auto lookup = [&](int b, int& page, int& sub) {
            const int L = b * AT_KEYS + lt;
            page = -1;
            sub = 0;
            if (L < max_limit) {
                const int slot = L < it.shared ? L : it.segment + (L - it.shared);
                page = __ldg(a.page_table + slot / a.page_slots);
                sub = slot % a.page_slots;
            }
        };
        int page, sub;
        lookup(0, page, sub);
        for (int b = 0; b < nb; b++) {
            const int s = b & 1;
            tabs[s * AT_KEYS + lt] = page < 0 ? 0xFFFFFFFFu : ((uint32_t)page << 8) | (uint32_t)sub;
            if (b + 1 < nb) lookup(b + 1, page, sub);
            // one thread waits for the stage; the named barrier hands its verdict (one flag per
            // stage, so a flag is rewritten only after every loader has read it) to the others
            if (lt == 0) flags[s] = mbar_wait(kv_empty + 8 * s, (uint32_t)((b >> 1) & 1) ^ 1u) ? 1u : 0u;
            asm volatile("bar.sync 1, 128;\n" ::: "memory");
            if (!flags[s]) {
                if (lt == 0) atomicExch(err, JV_ERR_DEVICE_TIMEOUT);
                break;
            }
            const uint32_t kd = s_addr(KV + s * 2 * AT_TILE), vd = kd + AT_TILE;
            const int c = lt & 15;
#pragma unroll 4
            for (int key = lt >> 4; key < AT_KEYS; key += 8) {
                const uint32_t e = tabs[s * AT_KEYS + key];
                const char* row = (const char*)a.kv_pool;
                int bytes = 0;
                if (e != 0xFFFFFFFFu) {
                    row = (const char*)a.kv_pool + (int64_t)(e >> 8) * a.page_bytes + (int64_t)(e & 255u) * 256 + head_off;
                    bytes = 16;
                }
                cp16(kd + tile_off(key, c), row + c * 16, bytes);
                cp16(vd + tile_off(key, c), row + v_off + c * 16, bytes);
            }
            cp_wait_all();
            fence_proxy_async();
            mbar_arrive(kv_full + 8 * s);
        }
        cp_wait_all();
    } else if (warp == 8) {
        if (lane == 0) {  // ------------------------------------------------------- MMA
            const uint32_t id_s = idesc_f16(AT_KEYS, AT_ROWS);
            const uint32_t id_pv = idesc_f16(128, AT_ROWS) | (1u << 16);  // B (V) MN-major
            bool ok = mbar_wait(q_full, 0);
            auto issue_s = [&](int b) -> bool {
                const int s = b & 1;
                if (!mbar_wait(kv_full + 8 * s, (uint32_t)((b >> 1) & 1))) return false;
                if (!mbar_wait(s_empty + 8 * s, (uint32_t)((b >> 1) & 1) ^ 1u)) return false;
                tc_fence_after();
                const uint32_t q = s_addr(Qs), k = s_addr(KV + s * 2 * AT_TILE);
                const uint32_t d = tmem + 128u + (uint32_t)(s * 128);
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t off = (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32);
                    umma(d, sdesc(q + off), sdesc(k + off), id_s, kk > 0 ? 1u : 0u);
                }
                umma_commit(s_full + 8 * s);
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int b = 0; b < nb && ok; b++) {
                if (b + 1 < nb && !issue_s(b + 1)) { ok = false; break; }
                if (!mbar_wait(p_full, (uint32_t)(b & 1))) { ok = false; break; }
                tc_fence_after();
                const uint32_t p = s_addr(Ps), v = s_addr(KV + (b & 1) * 2 * AT_TILE + AT_TILE);
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t off = (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32);
                    umma(tmem, sdesc(p + off), sdesc_mn(v + kk * 2048), id_pv, (b > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(kv_empty + 8 * (b & 1));
                umma_commit(o_done);  // last: its arrival implies the stage release before it
            }
            if (!ok) atomicExch(err, JV_ERR_DEVICE_TIMEOUT);
        }
    } else {
        // --------------------------------------------------- softmax and the output
        const int r = tid;  // query row = TMEM lane
        const int tl = r / group, j = r % group;
        const int lim = tl < it.ntok ? it.shared + (it.slot0 + tl - it.segment + 1) : 1;
        const float sl2 = a.scale * AT_LOG2E;
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        float m = -INFINITY, l = 0.f;  // running maximum (log2 units) and sum
        bool ok = true;
        for (int b = 0; b < nb; b++) {
            const int s = b & 1;
            if (!warp_wait(s_full + 8 * s, (uint32_t)((b >> 1) & 1))) { ok = false; break; }
            tc_fence_after();
            uint32_t v[128];
            {
                const uint32_t sb = tmem + lane_base + 128u + (uint32_t)(s * 128);
                uint32_t(&v0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[0]);
                uint32_t(&v1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[32]);
                uint32_t(&v2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[64]);
                uint32_t(&v3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[96]);
                tld32(sb, v0);
                tld32(sb + 32u, v1);
                tld32(sb + 64u, v2);
                tld32(sb + 96u, v3);
                tld_wait(v0);
                tld_wait(v1);
                tld_wait(v2);
                tld_wait(v3);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_empty + 8 * s);  // S buffer s may take block b + 2
            // keys at or past the row's limit are invisible
            const int vis = lim - b * AT_KEYS;
            if (vis < AT_KEYS) {
#pragma unroll
                for (int e = 0; e < 128; e++)
                    if (e >= vis) v[e] = __float_as_uint(-INFINITY);
            }
            float bm = -INFINITY;
#pragma unroll
            for (int e = 0; e < 128; e++) bm = fmaxf(bm, __uint_as_float(v[e]));
            const float mn = fmaxf(m, bm * sl2);  // finite: key 0 is visible to every row
            const float alpha = ex2(m - mn);      // 0 on the first block, where O is overwritten
            float rs = 0.f;
            uint32_t pk[64];
#pragma unroll
            for (int e = 0; e < 128; e += 2) {
                const float p0 = ex2(fmaf(__uint_as_float(v[e]), sl2, -mn));
                const float p1 = ex2(fmaf(__uint_as_float(v[e + 1]), sl2, -mn));
                rs += p0 + p1;
                __half2 hp = __floats2half2_rn(p0, p1);
                pk[e >> 1] = *reinterpret_cast<uint32_t*>(&hp);
            }
            l = l * alpha + rs;
            m = mn;
            // P may be overwritten and O rescaled once the previous block's P V has finished
            if (b > 0) {
                if (!warp_wait(o_done, (uint32_t)((b - 1) & 1))) { ok = false; break; }
                tc_fence_after();
            }
#pragma unroll
            for (int c = 0; c < 16; c++)
                *(uint4*)(Ps + tile_off(r, c)) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            // O *= alpha where the maximum moved (an exact no-op where alpha is 1)
            if (b > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                for (int h = 0; h < 4; h++) {
                    uint32_t o[32];
                    tld32(tmem + lane_base + (uint32_t)(h * 32), o);
                    tld_wait(o);
#pragma unroll
                    for (int e = 0; e < 32; e++) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                    tst32(tmem + lane_base + (uint32_t)(h * 32), o);
                }
                tst_wait();
            }
            fence_proxy_async();  // P stores -> visible to the tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (ok && !warp_wait(o_done, (uint32_t)((nb - 1) & 1))) ok = false;
        if (!ok) {
            atomicExch(err, JV_ERR_DEVICE_TIMEOUT);
        } else {
            tc_fence_after();
            const float inv = 1.f / l;
            const int t = it.t0 + tl, head = it.kv_head * group + j;
            for (int h = 0; h < 4; h++) {
                uint32_t o[32];
                tld32(tmem + lane_base + (uint32_t)(h * 32), o);
                tld_wait(o);
                if (tl < it.ntok) {
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const int col = head * 128 + h * 32 + c * 8;
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; e++) f[e] = __uint_as_float(o[8 * c + e]) * inv;
                        if (a.ctx16) {
                            __half2 q0 = __floats2half2_rn(f[0], f[1]), q1 = __floats2half2_rn(f[2], f[3]);
                            __half2 q2 = __floats2half2_rn(f[4], f[5]), q3 = __floats2half2_rn(f[6], f[7]);
                            *(uint4*)(a.ctx16 + kslab_offset(t, col, a.tpad)) =
                                make_uint4(*reinterpret_cast<uint32_t*>(&q0), *reinterpret_cast<uint32_t*>(&q1),
                                           *reinterpret_cast<uint32_t*>(&q2), *reinterpret_cast<uint32_t*>(&q3));
                        }
                        if (a.ctx32) {
                            float* dst = a.ctx32 + (int64_t)t * qdim + col;
                            *(float4*)dst = make_float4(f[0], f[1], f[2], f[3]);
                            *(float4*)(dst + 4) = make_float4(f[4], f[5], f[6], f[7]);
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace

constexpr size_t AT_SMEM = (size_t)6 * AT_TILE + 2 * AT_KEYS * 4 + 128 + 1024;

void launch_attention_tc(const AttnArgs& a, cudaStream_t s) {
    if (a.n_items <= 0) return;
    if (a.page_slots > 256) throw Error(JV_ERR_UNSUPPORTED, "attention: pages of more than 256 slots");
    if (a.heads != 4 * a.kv_heads) throw Error(JV_ERR_UNSUPPORTED, "attention: 4 query heads per KV head expected");
    static bool configured = false;
    if (!configured) {
        JV_CUDA(cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AT_SMEM));
        configured = true;
    }
    launch_pdl(k_attn_tc, dim3(a.n_items), dim3(AT_THREADS), AT_SMEM, s, a);
    note_launch();
}

}  // namespace jv
