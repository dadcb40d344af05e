// attn_tc.cu — tree-masked GQA prefill attention on the 5th-generation tensor cores.
//
// Semantics are those of k_attention (kernels_attn.cu; reference MinistralModel.cs:446-636):
// query row (token t, head h) sees logical keys L < limit(t), logical key L being cache slot
// base + L below `shared` and slot segment + (L - shared) above; keys are walked in logical order in
// blocks cut on logical indices, so a token's output is bit-identical whether it runs in a
// tree, alone after the trunk, or after a cached prefix.
//
// One CTA = one KV head x up to 64 consecutive tokens of one segment, as two query tiles X = A
// (tokens 0-31) and B (32-63); in a tile the 4 query heads of the KV head ride in M (128 rows =
// TMEM lanes). Both tiles share every K/V block. Per tile and block of 128 keys:
//   S  = Q K^T      tcgen05.mma kind::f16, M = 128, N = 128 keys, K = 128 dims -> TMEM (fp32)
//   P  = exp2(S * scale * log2 e - m)   one query row per softmax thread, online max/sum; the
//                                        reference maximum m moves only when a block exceeds it
//                                        by more than 2^8, and O is rescaled in TMEM then
//   O += P V        P from shared memory (K-major), V through an MN-major SWIZZLE_128B descriptor
// TMEM: O_A, O_B, S_A, S_B, 128 columns each. Warps 0-3 run tile A's softmax, warps 4-7 tile B's;
// a softmax hands its S columns back as soon as it has read them, so the next block's Q K^T runs
// while it computes the exponentials. The tiles take the single P buffer in turn (A(0), B(0),
// A(1), B(1), ..., then B alone). Warp 8 fills a 2-deep K ring and warp 9 a 2-deep V ring: KV
// pages store their rows in the operand swizzle (kv_chunk_offset), so each run of consecutive
// slots inside one page is two bulk copies (one per 64-dim half); a run whose first row sits at
// a different position modulo 8 in the page than in the tile (a branch segment starting off a
// multiple of 8) goes chunk by chunk through cp.async instead.
// Each tile has its own MMA issuer (lane 0 of warp 10 for A, of warp 11 for B; warp 10 also owns
// TMEM): a single thread issuing this loop's MMAs left the tensor core half idle. An issuer works
// through its own tile in order: S_X(b + 1) as soon as K(b + 1) is in place and the softmax has read
// S_X(b), then P V(b) once P_X(b) and V(b) are. Each tile releases a K stage
// through its own barrier (the two tiles' S MMAs are not ordered); a V stage is released by the
// last tile to use it, whose P V follows the other's through the P buffer. Every wait is bounded
// (WAIT_CYCLES of the SM clock); on expiry the role records JV_ERR_DEVICE_TIMEOUT and stops.
#include "tc_common.cuh"

namespace jv {
namespace {

constexpr int AT_ROWS = 128;                 // 32 tokens x 4 query heads per tile
constexpr int AT_KEYS = 128;                 // keys per block
constexpr int AT_THREADS = 384;              // 12 warps
constexpr int AT_TILE = 128 * 128 * 2;       // one [128][128] fp16 tile, two 16 KB halves
constexpr int AT_PAGES = 448;                // page-table entries staged in shared memory
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
__device__ __forceinline__ bool warp_wait_bounded(uint32_t bar, uint32_t parity, long long bound) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, bound));
}
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity) { return warp_wait_bounded(bar, parity, WAIT_CYCLES); }

__device__ __forceinline__ void mbar_add_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}

__global__ void __launch_bounds__(AT_THREADS, 1) k_attn_tc(AttnArgs a) {
    extern __shared__ uint8_t at_raw[];
    // 1024-aligned for the SWIZZLE_128B tiles; pointer arithmetic on the shared array keeps the
    // pointer in the shared state space (plain ld/st.shared rather than generic accesses)
    uint8_t* sm = at_raw + ((1024u - (s_addr(at_raw) & 1023u)) & 1023u);
    uint8_t* Qs = sm;                       // 2 tiles of [128 rows][128 dims]
    uint8_t* Ks = sm + 2 * AT_TILE;         // 2 stages of [128 keys][128 dims]
    uint8_t* Vs = sm + 4 * AT_TILE;         // 2 stages of [128 keys][128 dims]
    uint8_t* Ps = sm + 6 * AT_TILE;         // [128 rows][128 keys]: one tile's P at a time
    int32_t* pg = (int32_t*)(sm + 7 * AT_TILE);  // physical pages of the item's keys
    uint64_t* bars = (uint64_t*)(pg + AT_PAGES);
    // k_empty: per tile x and stage s at k_empty + 8 (2x + s); p_full, s_full, s_free, o_done per tile
    const uint32_t q_full = s_addr(bars), k_full = q_full + 8, k_empty = k_full + 16, v_full = k_empty + 32;
    const uint32_t v_empty = v_full + 16, s_full = v_empty + 16, s_free = s_full + 16, p_full = s_free + 16;
    const uint32_t o_done = p_full + 16;
    uint32_t* tslot = (uint32_t*)(bars + 20);

    // Items and the page table were uploaded before the pass: set-up reads them before waiting
    // for the previous kernel, which wrote Q and this pass's K/V.
    pdl_launch_dependents();
    const AttnItem it = a.items[blockIdx.x];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int group = a.heads / a.kv_heads;  // 4 (checked on the host)
    const int qdim = a.heads * 128;
    const int ps = a.page_slots;
    // per tile: tokens, visible keys of its last token, blocks
    const int ntA = min(it.ntok, 32), ntB = it.ntok - ntA;
    const int limA = it.shared + (it.slot0 + ntA - 1 - it.segment + 1);
    const int limB = ntB > 0 ? it.shared + (it.slot0 + it.ntok - 1 - it.segment + 1) : 0;
    const int nbA = (limA + AT_KEYS - 1) / AT_KEYS, nbB = (limB + AT_KEYS - 1) / AT_KEYS;
    const int max_limit = max(limA, limB), nb = max(nbA, nbB);
    // keys below `shared` (region A) are slots base.., the rest (region B) slots segment..
    const int nA = min(it.shared, max_limit), nBk = max_limit - nA;
    const int pA0 = it.base / ps;
    const int pagesA = nA > 0 ? (it.base + nA - 1) / ps - pA0 + 1 : 0;
    const int pB0 = nBk > 0 ? it.segment / ps : 0;
    const int pagesB = nBk > 0 ? (it.segment + nBk - 1) / ps - pB0 + 1 : 0;
    const bool staged = pagesA + pagesB <= AT_PAGES;  // else the loaders read the page table

    if (tid == 0) {
        mbar_init(q_full, 64);
        for (int i = 0; i < 2; i++) {
            mbar_init(k_full + 8 * i, 32);
            mbar_init(k_empty + 8 * i, 1);
            mbar_init(k_empty + 16 + 8 * i, 1);
            mbar_init(v_full + 8 * i, 32);
            mbar_init(v_empty + 8 * i, 1);
            mbar_init(s_full + 8 * i, 1);
            mbar_init(s_free + 8 * i, 4);
            mbar_init(p_full + 8 * i, 4);
            mbar_init(o_done + 8 * i, 1);
        }
        fence_barrier_init();
    }
    if (warp == 10) tmem_alloc(s_addr(tslot), 512);
    if (warp >= 8 && staged) {
        // stage the page-table entries of both key regions
        for (int i = tid - 256; i < pagesA + pagesB; i += 128)
            pg[i] = kv_page(a.page_table, (i < pagesA ? pA0 + i : pB0 + (i - pagesA)) * ps, ps, a.err, BS_ATTN_PAGE);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;  // O_A 0-127, O_B 128-255, S_A 256-383, S_B 384-511
    int* err = a.err;
    pdl_wait();

    if (warp >= 8) {
        // ------------------------------------------------- K / V rings, and Q first
        if (warp >= 10) {
            // Q row r of tile X = token 32 X + r / 4, head r % 4 of this KV head (4 query heads per
            // KV head, checked on the host). The two issuer warps load it before they issue: thread
            // t takes 16-byte chunk c = t % 16 of rows r = t / 16 + 4 h + 8 k, so its swizzle
            // (c ^ (r & 7)) is fixed per h and each step of k is one row group further.
            const int t = tid - 320, c = t & 15, rg = t >> 4;  // rg 0..3
            const __half* qsrc = a.q16 + (int64_t)it.t0 * qdim + (it.kv_head * 4 + (rg & 3)) * 128 + c * 8;
#pragma unroll
            for (int x = 0; x < 2; x++)
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int rr = rg + 4 * h;
                    const uint32_t dst0 = s_addr(Qs + x * AT_TILE) + (uint32_t)((c >> 3) * 16384 + rr * 128 + (((c & 7) ^ rr) << 4));
#pragma unroll
                    for (int k = 0; k < 16; k++) {
                        const int tl = 32 * x + (rr >> 2) + 2 * k;  // token of row rr + 8 k
                        const bool ok = tl < it.ntok;
                        cp16(dst0 + (uint32_t)(k * 1024), ok ? qsrc + (int64_t)tl * qdim : a.q16, ok ? 16 : 0);
                    }
                }
            cp_wait_all();
            fence_proxy_async();
            mbar_arrive(q_full);
        }
        if (warp == 8 || warp == 9) {
            const int kv = warp - 8;  // 0: K ring, 1: V ring
            const char* pool = (const char*)a.kv_pool + kv_plane_offset(a.layer, a.kv_heads, it.kv_head, kv, ps);
            const uint32_t full = kv ? v_full : k_full, empty = kv ? v_empty : k_empty;
            const uint32_t ring = s_addr(kv ? Vs : Ks);
            for (int b = 0; b < nb; b++) {
                const int s = b & 1;
                bool ok = true;
                if (lane == 0) {
                    if (kv) {
                        ok = mbar_wait(empty + 8 * s, (uint32_t)((b >> 1) & 1) ^ 1u);
                    } else {
                        // K(b - 2) must be done with by every tile that took it
                        for (int x = 0; x < 2 && ok; x++)
                            if (b >= 2 && b - 2 < (x ? nbB : nbA))
                                ok = mbar_wait(empty + 8 * (2 * x + s), (uint32_t)(((b - 2) >> 1) & 1));
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
                    if (lane == 0) report_timeout(err, 16 + 1 + kv);
                    break;
                }
                const uint32_t tile = ring + (uint32_t)(s * AT_TILE);
                const int L0 = b * AT_KEYS, nvalid = min(AT_KEYS, max_limit - L0);
                // runs of consecutive slots inside one page: region A, then region B
#pragma unroll 1
                for (int reg = 0; reg < 2; reg++) {
                    int La = reg == 0 ? L0 : max(L0, nA);
                    const int Lb = reg == 0 ? min(L0 + nvalid, nA) : L0 + nvalid;
                    while (La < Lb) {
                        const int slot = reg == 0 ? it.base + La : it.segment + (La - nA);
                        const int row = slot % ps;
                        const int n = min(Lb - La, ps - row);
                        const int gi = reg == 0 ? slot / ps - pA0 : pagesA + slot / ps - pB0;
                        const int page = !staged ? kv_page(a.page_table, slot, ps, err, BS_ATTN_PAGE)
                                         : JV_CHECK(gi >= 0 && gi < AT_PAGES, err, BS_ATTN_STAGED) ? pg[gi] : 0;
                        const char* plane = pool + (int64_t)page * a.page_bytes;
                        const int key0 = La - L0;
                        if (((key0 - row) & 7) == 0) {
                            if (lane == 0) {
                                mbar_add_tx(full + 8 * s, (uint32_t)(2 * n * 128));
                                bulk_g2s(tile + (uint32_t)(key0 * 128), plane + row * 128, (uint32_t)(n * 128), full + 8 * s);
                                bulk_g2s(tile + 16384u + (uint32_t)(key0 * 128), plane + ps * 128 + row * 128,
                                         (uint32_t)(n * 128), full + 8 * s);
                            }
                        } else {
                            for (int i = lane; i < n * 16; i += 32) {
                                const int r = i >> 4, c = i & 15;
                                cp16(tile + tile_off(key0 + r, c), plane + kv_chunk_offset(row + r, c, ps), 16);
                            }
                        }
                        La += n;
                    }
                }
                // rows past the last visible key: zeros, so 0-probability keys add exact zeros
                for (int i = lane; i < (AT_KEYS - nvalid) * 16; i += 32) {
                    const int r = nvalid + (i >> 4), c = i & 15;
                    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};\n" ::"r"(tile + tile_off(r, c)), "r"(0u) : "memory");
                }
                cp_wait_all();
                fence_proxy_async();
                mbar_arrive(full + 8 * s);
            }
            cp_wait_all();
        } else if (lane == 0) {
            // ------------------------------------------------------- MMA, one issuer per tile
            const int x = warp - 10;
            const int nbt = x ? nbB : nbA;
            const uint32_t id_s = idesc_f16(AT_KEYS, AT_ROWS);
            const uint32_t id_pv = idesc_f16(128, AT_ROWS) | (1u << 16);  // B (V) MN-major
            bool ok = nbt == 0 || mbar_wait(q_full, 0);
            tc_fence_after();
            const uint32_t q = s_addr(Qs + x * AT_TILE), o = tmem + (uint32_t)(x * 128), d = tmem + 256u + (uint32_t)(x * 128);
            // In order: S(0), then per block b: S(b + 1), P V(b). S(b + 1) needs only K(b + 1) and
            // the softmax's read of S(b), which comes before it waits for the P buffer, so the
            // order cannot stall; each wait tests one barrier, at most one phase behind the one
            // wanted (this thread consumed the phase before). Measured faster than an event loop
            // over all four barriers (704 vs 678 TFLOP/s on C5 trees).
            auto issue_s = [&](int b) -> bool {
                if (!mbar_poll(k_full + 8 * (b & 1), (uint32_t)((b >> 1) & 1))) return false;
                if (b > 0 && !mbar_poll(s_free + 8 * x, (uint32_t)((b - 1) & 1))) return false;
                tc_fence_after();
                const uint32_t k = s_addr(Ks + (b & 1) * AT_TILE);
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t off = (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32);
                    umma(d, sdesc(q + off), sdesc(k + off), id_s, kk > 0 ? 1u : 0u);
                }
                umma_commit(k_empty + 8 * (2 * x + (b & 1)));
                umma_commit(s_full + 8 * x);
                return true;
            };
            auto issue_pv = [&](int b) -> bool {
                if (!mbar_poll(p_full + 8 * x, (uint32_t)(b & 1))) return false;
                if (!mbar_poll(v_full + 8 * (b & 1), (uint32_t)((b >> 1) & 1))) return false;
                tc_fence_after();
                const uint32_t v = s_addr(Vs + (b & 1) * AT_TILE), p = s_addr(Ps);
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t off = (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32);
                    umma(o, sdesc(p + off), sdesc_mn(v + kk * 2048), id_pv, (b > 0 || kk > 0) ? 1u : 0u);
                }
                if (x == 1 || nbB == 0) umma_commit(v_empty + 8 * (b & 1));
                umma_commit(o_done + 8 * x);
                return true;
            };
            if (ok && nbt > 0) ok = issue_s(0);
            for (int b = 0; ok && b < nbt; b++) {
                if (b + 1 < nbt) ok = issue_s(b + 1);
                if (ok) ok = issue_pv(b);
            }
            if (!ok) report_timeout(err, x ? 16 + 6 : 16 + 3);
        }
    } else {
        // --------------------------------------------------- softmax and the output
        const int x = warp >> 2;  // tile
        const int r = tid & 127;  // query row = TMEM lane
        const int tl = 32 * x + r / group, j = r % group;
        const int nbt = x ? nbB : nbA;
        const int lim = tl < it.ntok ? it.shared + (it.slot0 + tl - it.segment + 1) : 1;
        const float sl2 = a.scale * AT_LOG2E;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t o_col = tmem + lane_base + (uint32_t)(x * 128);
        const uint32_t s_col = tmem + lane_base + 256u + (uint32_t)(x * 128);
        // m: the row's reference maximum (log2 units). It moves only when the block maximum
        // exceeds it by more than 8, so probabilities stay below 2^8 (fine in fp16) and O is
        // rescaled rarely; the sequence of m depends on the row's own scores in logical block
        // order only, so the bit-identity across tree / alone / cached holds.
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int b = 0; b < nbt; b++) {
            if (!warp_wait(s_full + 8 * x, (uint32_t)(b & 1))) { ok = false; break; }
            tc_fence_after();
            uint32_t v[128];
            {
                uint32_t(&v0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[0]);
                uint32_t(&v1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[32]);
                uint32_t(&v2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[64]);
                uint32_t(&v3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[96]);
                tld32(s_col, v0);
                tld32(s_col + 32u, v1);
                tld32(s_col + 64u, v2);
                tld32(s_col + 96u, v3);
                tld_wait(v0);
                tld_wait(v1);
                tld_wait(v2);
                tld_wait(v3);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free + 8 * x);  // S_X(b + 1) may overwrite S_X(b)
            // keys at or past the row's limit are invisible
            const int vis = lim - b * AT_KEYS;
            if (vis < AT_KEYS) {
#pragma unroll
                for (int e = 0; e < 128; e++)
                    if (e >= vis) v[e] = __float_as_uint(-INFINITY);
            }
            float bm = -INFINITY;
#pragma unroll
            for (int e = 0; e < 128; e += 2) bm = fmaxf(bm, fmaxf(__uint_as_float(v[e]), __uint_as_float(v[e + 1])));
            bm *= sl2;                                  // finite: key 0 is visible to every row
            const bool move = bm > m + 8.f;             // always on the first block (m = -inf)
            const float mn = move ? bm : m;
            const float alpha = move ? ex2(m - mn) : 1.f;  // 0 on the first block, where O is overwritten
            // probabilities as fp16 pairs (keys 2c, 2c + 1 in column c), packed in place, and their sum
            float rs = 0.f;
#pragma unroll
            for (int e = 0; e < 128; e += 2) {
                const float p0 = ex2(fmaf(__uint_as_float(v[e]), sl2, -mn));
                const float p1 = ex2(fmaf(__uint_as_float(v[e + 1]), sl2, -mn));
                rs += p0 + p1;
                __half2 hp = __floats2half2_rn(p0, p1);
                v[e >> 1] = *reinterpret_cast<uint32_t*>(&hp);
            }
            l = l * alpha + rs;
            m = mn;
            // The P buffer is free once the P V of its previous user has finished: tile B's block
            // b - 1 for A(b) (A's own for a lone tile), tile A's block b for B(b) while A takes
            // blocks, else B's own block b - 1. That P V completing implies every earlier one has,
            // P V_X(b - 1) included, so O_X may be rescaled too. Each of these barriers is at
            // most one phase behind the one awaited (this warp's previous wait covered the one
            // before it), so the parity test is exact.
            {
                int wt = -1, wb = 0;
                if (x == 0) {
                    if (b > 0) { wt = nbB > 0 ? 1 : 0; wb = b - 1; }
                } else if (b < nbA) {
                    wt = 0; wb = b;
                } else if (b > 0) {
                    wt = 1; wb = b - 1;
                }
                if (wt >= 0 && !warp_wait(o_done + 8 * wt, (uint32_t)(wb & 1))) { ok = false; break; }
            }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 16; c++)
                *(uint4*)(Ps + tile_off(r, c)) = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
            // O *= alpha for rows whose maximum moved
            if (b > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
                for (int h = 0; h < 2; h++) {
                    uint32_t o0[32], o1[32];
                    tld32(o_col + (uint32_t)(h * 64), o0);
                    tld32(o_col + (uint32_t)(h * 64 + 32), o1);
                    tld_wait(o0);
                    tld_wait(o1);
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        o0[e] = __float_as_uint(__uint_as_float(o0[e]) * alpha);
                        o1[e] = __float_as_uint(__uint_as_float(o1[e]) * alpha);
                    }
                    tst32(o_col + (uint32_t)(h * 64), o0);
                    tst32(o_col + (uint32_t)(h * 64 + 32), o1);
                }
            }
            tst_wait();
            fence_proxy_async();  // P stores -> visible to the tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full + 8 * x);
        }
        if (nbt > 0) {
            if (ok && !warp_wait(o_done + 8 * x, (uint32_t)((nbt - 1) & 1))) ok = false;
            if (!ok) {
                report_timeout(err, 16 + 4 + x);
            } else {
                tc_fence_after();
                const float inv = 1.f / l;
                const int t = it.t0 + tl, head = it.kv_head * group + j;
                for (int h = 0; h < 4; h++) {
                    uint32_t o[32];
                    tld32(o_col + (uint32_t)(h * 32), o);
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
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 10) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// One warp waits, with the bounded wait every tensor-core kernel uses, on an mbarrier that
// nothing arrives at; the wait gives up after `bound` cycles and reports site 33. This checks
// the device-timeout path (error word, site, host message, a context that stays usable)
// without faulting or hanging the GPU.
__global__ void k_wait_check(int* err, long long bound) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t b = s_addr(&bar);
    if (threadIdx.x == 0) {
        mbar_init(b, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (!warp_wait_bounded(b, 0u, bound) && threadIdx.x == 0) report_timeout(err, 33);
}

}  // namespace

constexpr size_t AT_SMEM = (size_t)7 * AT_TILE + AT_PAGES * 4 + 192 + 1024;

void launch_attention_tc(const AttnArgs& a, cudaStream_t s) {
    if (a.n_items <= 0) return;
    if (a.page_slots % 8 != 0 || a.page_slots > 256) throw Error(JV_ERR_UNSUPPORTED, "attention: page slots");
    if (a.heads != 4 * a.kv_heads) throw Error(JV_ERR_UNSUPPORTED, "attention: 4 query heads per KV head expected");
    static bool configured = false;
    if (!configured) {
        JV_CUDA(cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AT_SMEM));
        configured = true;
    }
    launch_pdl(k_attn_tc, dim3(a.n_items), dim3(AT_THREADS), AT_SMEM, s, a);
    note_launch();
}

void launch_wait_check(int* err, long long bound_cycles, cudaStream_t s) {
    k_wait_check<<<1, 32, 0, s>>>(err, bound_cycles);
    JV_CUDA(cudaGetLastError());
    note_launch();
}

}  // namespace jv
