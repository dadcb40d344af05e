// kernels_decode.cu — the single-token forward (a decode step), five fused kernels per layer:
//
//   1. attn_norm + QKV matvec + RoPE + temperature + K/V page write      (k_dec_gemv, DEC_QKV)
//   2. attention over the visible keys, split over keys, combined by the last CTA (k_dec_attn)
//   3. O matvec + residual add                                            (k_dec_gemv, DEC_ADD)
//   4. ffn_norm + gate/up matvec + SwiGLU                                  (k_dec_gemv, DEC_SWIGLU)
//   5. down matvec + residual add                                          (k_dec_gemv, DEC_ADD)
//
// and the LM head: final norm + full-vocabulary matvec + argmax (k_dec_gemv, DEC_HEAD).
//
// The matvec (reference QuantMatMul.RunRowsFloat, src/Jevstral/Numerics/QuantMatMul.cs:140-176)
// is HBM-bound, so its cost per weight byte must stay below the memory rate. Decoding every
// weight to fp32 and converting integers one by one does not: the conversions alone cap it
// near a third of HBM bandwidth. Here the quantized integers go straight into fp16 tensor-core
// fragments (mma.sync m16n8k16): q (Q8_0), q - 8 (Q4_0) and q5 (Q5_1) are small integers,
// exact in fp16. One MMA sums 16 products of a row with x; x is split into hi = fp16(x) and
// lo = fp16(x - hi) in the two B columns, so the products carry x to ~22 bits. Each 32-wide
// block's sum is then scaled by its fp32 d (and Q5_1 adds m times the block's sum of x):
//   y_r = sum_b d_rb * (sum_i q_rbi x_bi) [+ m_rb * sum_i x_bi],
// which is the reference's sum_i (d q_i [+ m]) x_i with the products regrouped per block.
//
// The dynamic values of a step (token, slot, position, visible keys) are read from a
// DecodeStep in device memory, so a step's launches do not change from one token to the
// next and can be replayed as a CUDA graph; DEC_HEAD can advance the step on the device.
#include "decode_common.cuh"

namespace jv {

namespace {

template <int TYPE, int MODE, bool NORM>
__global__ void __launch_bounds__(DG_THREADS) k_dec_gemv(DecGemvArgs a) {
    extern __shared__ __align__(128) uint8_t dg_smem[];
    __shared__ double red[33];
    __shared__ float s_out[128];
    __shared__ int s_last;
    __shared__ __align__(8) uint64_t s_bar;
    const int tile = blockIdx.x, split = blockIdx.y, splits = gridDim.y;
    const int ksteps = a.ksteps;
    const int per = (ksteps + splits - 1) / splits;
    const int ks0 = split * per, nk = max(0, min(ksteps, ks0 + per) - ks0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cb = chunk_bytes(TYPE);

    uint8_t* raw = dg_smem;                             // [per][chunk] this CTA's weights
    float* xs = (float*)(dg_smem + (size_t)per * cb);   // [per*64] this CTA's slice of x
    uint2* xf = (uint2*)(xs + per * 64);                // [per][2 blocks][2 subs][8 lanes]
    float* sx = (float*)(xf + per * 32);                // [per][2] block sums of x (Q5_1)

    // The weight slice is one contiguous run of chunks: stream it into shared memory first,
    // before waiting for the previous kernel (the weights do not depend on it).
    const uint32_t bar = smem_u32(&s_bar);
    const uint8_t* __restrict__ src = a.w + ((int64_t)tile * ksteps + ks0) * cb;
    if (threadIdx.x == 0) {
        dg_mbar_init(bar, 1);
        if (nk > 0) {
            dg_expect_tx(bar, (uint32_t)(nk * cb));
            for (int i = 0; i < nk; i++) dg_bulk(smem_u32(raw + (size_t)i * cb), src + (size_t)i * cb, (uint32_t)cb, bar);
        }
        dg_prefetch_share(a.pf, a.pf_bytes);
    }
    pdl_launch_dependents();
    pdl_wait();

    // ---- x: the CTA's K slice, RMS-normalised first when NORM (Kernels.RmsNorm, Kernels.cs:25-60)
    // Every load of a pass is issued before any is used (16-byte loads, fixed batches), so a
    // pass costs one memory round trip.
    float scale = 1.f;
    if (NORM) {
        const float4* in4 = (const float4*)a.in;
        const int n4 = a.n_in >> 2;
        double s = 0;
        for (int b0 = threadIdx.x; b0 < n4; b0 += 4 * DG_THREADS) {
            float4 v[4];
#pragma unroll
            for (int j = 0; j < 4; j++) v[j] = b0 + j * DG_THREADS < n4 ? in4[b0 + j * DG_THREADS] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 4; j++)
                s += (double)v[j].x * v[j].x + (double)v[j].y * v[j].y + (double)v[j].z * v[j].z + (double)v[j].w * v[j].w;
        }
        s = block_sum_d(s, red);
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(s / a.n_in), a.eps)));
    }
    {
        const float4* in4 = (const float4*)(a.in + ks0 * 64);
        const float4* w4 = NORM ? (const float4*)(a.norm_w + ks0 * 64) : nullptr;
        float4* xs4 = (float4*)xs;
        for (int i = threadIdx.x; i < nk * 16; i += DG_THREADS) {
            float4 v = in4[i];
            if (NORM) {
                const float4 w = w4[i];
                v.x = __fmul_rn(__fmul_rn(v.x, scale), w.x);
                v.y = __fmul_rn(__fmul_rn(v.y, scale), w.y);
                v.z = __fmul_rn(__fmul_rn(v.z, scale), w.z);
                v.w = __fmul_rn(__fmul_rn(v.w, scale), w.w);
            }
            xs4[i] = v;
        }
    }
    __syncthreads();
    // B fragments: column 0 = fp16(x), column 1 = fp16(x - column 0); lanes 0-3 / 4-7.
    bool bad = false;
    for (int e = threadIdx.x; e < nk * 32; e += DG_THREADS) {
        const int ks = e >> 5, rest = e & 31, b = rest >> 4, sub = (rest >> 3) & 1, l = rest & 7;
        const int kq = l & 3, n = l >> 2;
        const float* p = xs + ks * 64 + x_base<TYPE>(b, sub, kq);
        uint32_t w[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            bad |= f16_out_of_range(p[2 * j]) | f16_out_of_range(p[2 * j + 1]);
            __half h0 = __float2half_rn(p[2 * j]), h1 = __float2half_rn(p[2 * j + 1]);
            if (n == 1) {
                h0 = __float2half_rn(__fsub_rn(p[2 * j], __half2float(h0)));
                h1 = __float2half_rn(__fsub_rn(p[2 * j + 1], __half2float(h1)));
            }
            w[j] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        }
        xf[e] = make_uint2(w[0], w[1]);
    }
    if (TYPE == T_Q5_1)
        for (int e = threadIdx.x; e < nk * 2; e += DG_THREADS) {
            const float* p = xs + e * 32;
            float s = 0.f;
            for (int i = 0; i < 32; i++) s = __fadd_rn(s, p[i]);
            sx[e] = s;
        }
    if (__syncthreads_or(bad) && threadIdx.x == 0) report_numeric(a.err, NS_DEC_INPUT);
    // x staged for every warp, and one verdict on the copy for the whole CTA (the warps' mma.sync
    // below needs all lanes)
    if (!__syncthreads_and(nk == 0 || dg_wait(bar, 0))) {
        // the copy never landed: report, and do not leave while it may still be writing
        if (threadIdx.x == 0) {
            atomicExch(a.err, JV_ERR_DEVICE_TIMEOUT);
            atomicCAS(a.err + 1, 0, 49);
        }
        dg_wait(bar, 0);
        return;
    }

    // ---- main loop: warp w owns rows 16w + g and 16w + g + 8 of the tile
    const int g = lane >> 2, kq = lane & 3;
    const int row = 16 * warp + g;
    const uint8_t* base = raw;
    float acc[2] = {0.f, 0.f};
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < nk; k0 += DG_UNROLL) {
        Raw<TYPE> r[DG_UNROLL];
#pragma unroll
        for (int u = 0; u < DG_UNROLL; u++)
            if (k0 + u < nk) load_raw<TYPE>(r[u], base + (int64_t)(k0 + u) * cb, row, kq);
#pragma unroll
        for (int u = 0; u < DG_UNROLL; u++) {
            if (k0 + u >= nk) break;
            const int ks = k0 + u;
#pragma unroll
            for (int b = 0; b < 2; b++) {
                uint32_t af[2][4];
                a_frags<TYPE>(r[u], b, kq, af);
                uint2 b0 = lane < 8 ? xf[(ks * 2 + b) * 16 + lane] : make_uint2(0u, 0u);
                uint2 b1 = lane < 8 ? xf[(ks * 2 + b) * 16 + 8 + lane] : make_uint2(0u, 0u);
                float c[4];
                mma16816(c, af[0][0], af[0][1], af[0][2], af[0][3], b0.x, b0.y, zero);
                mma16816(c, af[1][0], af[1][1], af[1][2], af[1][3], b1.x, b1.y, c);
                // lanes with kq == 0 hold column 0 (x hi) and 1 (x lo) of rows g and g + 8
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const float s = __fadd_rn(c[2 * h], c[2 * h + 1]);
                    const float d = b ? half_hi(r[u].d[h]) : half_lo(r[u].d[h]);
                    acc[h] = fmaf(d, s, acc[h]);
                    if (TYPE == T_Q5_1) {
                        const float m = b ? half_hi(r[u].m[h]) : half_lo(r[u].m[h]);
                        acc[h] = fmaf(m, sx[ks * 2 + b], acc[h]);
                    }
                }
            }
        }
    }

    // ---- split-K: partials in order, summed by the last CTA of the tile
    const int n0 = tile * 128;
    if (splits == 1) {
        if (kq == 0) {
            s_out[row] = acc[0];
            s_out[row + 8] = acc[1];
        }
        __syncthreads();
    } else {
        if (kq == 0) {
            a.partial[(int64_t)split * a.rows + n0 + row] = acc[0];
            a.partial[(int64_t)split * a.rows + n0 + row + 8] = acc[1];
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const int prev = atomicAdd(a.counters + tile, 1);
            s_last = prev == splits - 1;
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (threadIdx.x < 128) {
            // in split order, eight loads in flight at a time
            float s = 0.f;
            for (int p0 = 0; p0 < splits; p0 += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; j++)
                    v[j] = p0 + j < splits ? __ldcg(a.partial + (int64_t)(p0 + j) * a.rows + n0 + threadIdx.x) : 0.f;
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (p0 + j < splits) s = __fadd_rn(s, v[j]);
            }
            s_out[threadIdx.x] = s;
        }
        if (threadIdx.x == 0) a.counters[tile] = 0;  // ready for the next launch
        __syncthreads();
    }

    // ---- epilogues
    const int t = threadIdx.x;
    if (MODE == DEC_STORE) {
        if (t < 128) a.y[n0 + t] = s_out[t];
    } else if (MODE == DEC_ADD) {
        if (t < 128) a.y[n0 + t] = __fadd_rn(a.y[n0 + t], s_out[t]);
    } else if (MODE == DEC_SWIGLU) {
        // Kernels.SwiGlu (Kernels.cs:82-89) on the 16-row gate/up interleave of the tile.
        if (t < 64) {
            const int gr = 32 * (t >> 4) + (t & 15);
            const float gg = s_out[gr], uu = s_out[gr + 16];
            const float up = __fmul_rn(gg, uu);
            const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gg)));
            a.y[tile * 64 + t] = __fmul_rn(sg, up);
        }
    } else if (MODE == DEC_QKV) {
        // One tile = one head of 128 (q heads, then k heads, then v heads). RotateQueries /
        // StoreKeys / StoreValues / ApplyPositionScale (MinistralModel.cs:638-682).
        const DecodeStep st = *a.step;
        const int hq = a.heads, hk = a.kv_heads;
        if (t < 64) {
            const float x0 = s_out[2 * t], x1 = s_out[2 * t + 1];
            if (tile < hq + hk) {
                const float2 cs = a.rope_table[(int64_t)st.pos * 64 + t];
                float r0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
                float r1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
                if (tile < hq) {
                    float temp = 1.0f;
                    if (a.orig_ctx > 0 && a.temperature_scale != 0.f) {
                        float interval = floorf(__fdiv_rn((float)st.pos, (float)a.orig_ctx));
                        if (interval != 0.f)
                            temp = __fadd_rn(1.0f, __fmul_rn(a.temperature_scale, logf(__fadd_rn(1.0f, interval))));
                    }
                    if (temp != 1.0f) { r0 = __fmul_rn(r0, temp); r1 = __fmul_rn(r1, temp); }
                    a.q32[tile * 128 + 2 * t] = r0;
                    a.q32[tile * 128 + 2 * t + 1] = r1;
                } else {
                    char* dst = kv_plane(a.kv_pool, a.page_table, a.page_bytes, a.page_slots, a.layer, hk, tile - hq, 0, st.slot, a.err);
                    if (f16_out_of_range(r0) || f16_out_of_range(r1)) report_numeric(a.err, NS_DEC_KV);
                    *(__half2*)(dst + kv_elem_offset(st.slot % a.page_slots, 2 * t, a.page_slots)) = __floats2half2_rn(r0, r1);
                }
            } else {
                char* dst = kv_plane(a.kv_pool, a.page_table, a.page_bytes, a.page_slots, a.layer, hk, tile - hq - hk, 1, st.slot, a.err);
                if (f16_out_of_range(x0) || f16_out_of_range(x1)) report_numeric(a.err, NS_DEC_KV);
                *(__half2*)(dst + kv_elem_offset(st.slot % a.page_slots, 2 * t, a.page_slots)) = __floats2half2_rn(x0, x1);
            }
        }
    } else if (MODE == DEC_HEAD) {
        // Logits of the tile's 128 vocabulary rows, then the first index of the maximum over
        // the whole vocabulary (Kernels.ArgMax, Kernels.cs:146) by the last CTA to finish.
        __shared__ float s_bv[128];
        __shared__ int s_bi[128];
        if (t < 128) {
            a.y[n0 + t] = s_out[t];
            s_bv[t] = s_out[t];
            s_bi[t] = n0 + t;
        }
        __syncthreads();
        for (int w = 64; w >= 1; w >>= 1) {
            if (t < w && dec_better(s_bv[t + w], s_bi[t + w], s_bv[t], s_bi[t])) {
                s_bv[t] = s_bv[t + w];
                s_bi[t] = s_bi[t + w];
            }
            __syncthreads();
        }
        if (t == 0) {
            a.cand_v[tile] = s_bv[0];
            a.cand_i[tile] = s_bi[0];
        }
        __threadfence();
        __syncthreads();
        if (t == 0) s_last = atomicAdd(a.counters + gridDim.x, 1) == (int)gridDim.x - 1;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = t; i < (int)gridDim.x; i += DG_THREADS) {
            const float v = __ldcg(a.cand_v + i);
            const int ix = __ldcg(a.cand_i + i);
            if (dec_better(v, ix, bv, bi)) { bv = v; bi = ix; }
        }
        __shared__ float u_bv[DG_THREADS];
        __shared__ int u_bi[DG_THREADS];
        u_bv[t] = bv;
        u_bi[t] = bi;
        __syncthreads();
        for (int w = DG_THREADS / 2; w >= 1; w >>= 1) {
            if (t < w && dec_better(u_bv[t + w], u_bi[t + w], u_bv[t], u_bi[t])) {
                u_bv[t] = u_bv[t + w];
                u_bi[t] = u_bi[t + w];
            }
            __syncthreads();
        }
        if (t == 0) {
            a.counters[gridDim.x] = 0;
            const int best = u_bi[0] == 0x7fffffff ? 0 : u_bi[0];
            if (a.argmax_out) *a.argmax_out = best;
            if (a.advance) {
                DecodeStep* st = a.step_rw;
                if (a.tokens_out) a.tokens_out[st->index] = best;
                st->token = best;
                st->index += 1;
                st->slot += 1;
                st->pos += 1;
                st->shared += 1;
                st->segment += 1;
                st->n_keys += 1;
            }
        }
    }
}

// ------------------------------------------------------------------ attention

// One query token against its visible keys (MinistralModel.AttendHead, MinistralModel.cs:564-636):
// CTA (kv head, split) takes logical keys [64 split, 64 split + 64) of the group's query heads
// (one warp each): scores as an fp32 FMA chain over d times the scale, a max-shifted softmax,
// the weighted value sum; the last CTA of the kv head merges the splits in split order.
// Logical key L is slot L below `shared`, else slot segment + L - shared.
constexpr int DA_KEYS = 64;
constexpr int DA_STRIDE = 136;  // halves per staged key row (272 B: conflict-free 16-byte reads)
constexpr int DA_PSTRIDE = DEC_ATTN_PSTRIDE;  // floats per split partial: m, l, pad, pad, acc[128]

__global__ void __launch_bounds__(256) k_dec_attn(DecAttnArgs a) {
    __shared__ __align__(16) __half ks[DA_KEYS * DA_STRIDE];
    __shared__ __align__(16) __half vs[DA_KEYS * 128];
    __shared__ __align__(16) float qs[8 * 128];
    __shared__ float ps[8 * DA_KEYS];
    __shared__ int s_last;
    __shared__ const char* krow[DA_KEYS];  // K and V planes of each key's page, and its row there
    __shared__ const char* vrow[DA_KEYS];
    __shared__ int krowi[DA_KEYS];
    if (threadIdx.x == 0) dg_prefetch_share(a.pf, a.pf_bytes);
    pdl_launch_dependents();
    pdl_wait();
    const DecodeStep st = *a.step;
    const int group = a.heads / a.kv_heads;
    const int kvh = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;
    const int k0 = split * DA_KEYS;
    const int nk = max(0, min(st.n_keys, k0 + DA_KEYS) - k0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nthreads = 32 * group;
    float* part = a.partial + ((int64_t)(kvh * group) * nsplit) * DA_PSTRIDE;

    if (nk > 0) {
        // rows of the split's keys first (one page-table lookup per key), then every 16-byte
        // piece of them in flight at once
        if ((int)threadIdx.x < nk) {
            const int L = k0 + threadIdx.x;
            const int slot = L < st.shared ? L : st.segment + (L - st.shared);
            __half* pool = const_cast<__half*>(a.kv_pool);
            krow[threadIdx.x] = kv_plane(pool, a.page_table, a.page_bytes, a.page_slots, a.layer, a.kv_heads, kvh, 0, slot, a.err);
            vrow[threadIdx.x] = kv_plane(pool, a.page_table, a.page_bytes, a.page_slots, a.layer, a.kv_heads, kvh, 1, slot, a.err);
            krowi[threadIdx.x] = slot % a.page_slots;
        }
        for (int i = threadIdx.x; i < group * 128; i += nthreads) qs[i] = a.q32[kvh * group * 128 + i];
        __syncthreads();
        for (int i = threadIdx.x; i < nk * 16; i += nthreads) {
            const int key = i >> 4, c = i & 15;
            const int off = kv_chunk_offset(krowi[key], c, a.page_slots);
            cp_async16(ks + key * DA_STRIDE + c * 8, krow[key] + off);
            cp_async16(vs + key * 128 + c * 8, vrow[key] + off);
        }
        cp_async_wait_all();
        __syncthreads();
        const int h = warp;
        const float* q = qs + h * 128;
        float mx = -INFINITY;
        for (int i = lane; i < nk; i += 32) {
            const __half* kr = ks + i * DA_STRIDE;
            float acc = 0.f;
#pragma unroll 4
            for (int d = 0; d < 128; d += 8) {
                int4 raw = *(const int4*)(kr + d);
                const __half2* kh = (const __half2*)&raw;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    float2 kf = __half22float2(kh[e]);
                    acc = fmaf(q[d + 2 * e], kf.x, acc);
                    acc = fmaf(q[d + 2 * e + 1], kf.y, acc);
                }
            }
            const float sc = acc * a.scale;
            ps[h * DA_KEYS + i] = sc;
            mx = fmaxf(mx, sc);
        }
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        __syncwarp();
        float l = 0.f;
        for (int i = lane; i < nk; i += 32) {
            const float p = __expf(ps[h * DA_KEYS + i] - mx);
            ps[h * DA_KEYS + i] = p;
            l += p;
        }
        for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        __syncwarp();
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < nk; i++) {
            const float p = ps[h * DA_KEYS + i];
            uint2 raw = *(const uint2*)(vs + i * 128 + lane * 4);
            const __half2* vh = (const __half2*)&raw;
            float2 v01 = __half22float2(vh[0]), v23 = __half22float2(vh[1]);
            acc[0] = fmaf(p, v01.x, acc[0]);
            acc[1] = fmaf(p, v01.y, acc[1]);
            acc[2] = fmaf(p, v23.x, acc[2]);
            acc[3] = fmaf(p, v23.y, acc[3]);
        }
        float* dst = part + ((int64_t)h * nsplit + split) * DA_PSTRIDE;
        if (lane == 0) { dst[0] = mx; dst[1] = l; }
        *(float4*)(dst + 4 + lane * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(a.counters + kvh, 1) == nsplit - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Merge the active splits in split order (k_decode_combine's arithmetic). Warp h merges
    // query head h: the maximum over splits with the lanes striding the splits, then each
    // lane's four dimensions with eight splits' loads in flight at a time.
    const int active = (st.n_keys + DA_KEYS - 1) / DA_KEYS;
    {
        const int h = warp;
        const float* hb = part + (int64_t)h * nsplit * DA_PSTRIDE;
        float m = -INFINITY;
        for (int sp = lane; sp < active; sp += 32) m = fmaxf(m, __ldcg(hb + (int64_t)sp * DA_PSTRIDE));
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int s0 = 0; s0 < active; s0 += 8) {
            float mv[8], lv[8];
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float* p = hb + (int64_t)(s0 + j) * DA_PSTRIDE;
                const bool ok = s0 + j < active;
                mv[j] = ok ? __ldcg(p) : 0.f;
                lv[j] = ok ? __ldcg(p + 1) : 0.f;
                v[j] = ok ? __ldcg((const float4*)(p + 4 + lane * 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (s0 + j >= active) break;
                const float w = __expf(mv[j] - m);
                l += w * lv[j];
                acc[0] += w * v[j].x;
                acc[1] += w * v[j].y;
                acc[2] += w * v[j].z;
                acc[3] += w * v[j].w;
            }
        }
        float* out = a.ctx32 + (kvh * group + h) * 128 + lane * 4;
#pragma unroll
        for (int e = 0; e < 4; e++) out[e] = acc[e] / l;
    }
    if (threadIdx.x == 0) a.counters[kvh] = 0;
}

template <int TYPE>
size_t dec_smem(int ksteps, int splits) {
    const int per = (ksteps + splits - 1) / splits;
    return (size_t)per * (chunk_bytes(TYPE) + 64 * 4 + 32 * 8 + 2 * 4);
}

template <int TYPE, int MODE, bool NORM>
void launch_dec_typed(const DecGemvArgs& a, int splits, cudaStream_t s) {
    const size_t smem = dec_smem<TYPE>(a.ksteps, splits);
    if (smem > 200 * 1024) throw Error(JV_ERR_UNSUPPORTED, "decode matvec: the K slice does not fit in shared memory");
    static size_t configured = 48 * 1024;
    if (smem > configured) {
        JV_CUDA(cudaFuncSetAttribute(k_dec_gemv<TYPE, MODE, NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = smem;
    }
    launch_pdl(k_dec_gemv<TYPE, MODE, NORM>, dim3(a.rows / 128, splits), dim3(DG_THREADS), smem, s, a);
}

template <int MODE, bool NORM>
void launch_dec_mode(int type, const DecGemvArgs& a, int splits, cudaStream_t s) {
    if (type == T_Q8_0)
        launch_dec_typed<T_Q8_0, MODE, NORM>(a, splits, s);
    else if (type == T_Q4_0)
        launch_dec_typed<T_Q4_0, MODE, NORM>(a, splits, s);
    else if (type == T_Q5_1)
        launch_dec_typed<T_Q5_1, MODE, NORM>(a, splits, s);
    else
        throw Error(JV_ERR_UNSUPPORTED, "decode matvec: unsupported weight type");
}

}  // namespace

int dec_splits_for(const QWeight& w, int sm_count) {
    // About four CTAs per SM and weight slices of at most 40 KB: the next kernel's CTAs then
    // find room to become resident and stage their own slices while this one runs (measured on
    // C4 against three CTAs / 64 KB: 1.47 vs 1.55 ms per step). Never fewer than 4 k steps.
    int splits = std::max(1, (4 * sm_count + w.tiles - 1) / w.tiles);
    splits = std::min(splits, std::max(1, (w.ksteps + 3) / 4));
    const int cb = chunk_bytes(w.type);
    const int max_per = std::max(1, (40 * 1024) / cb);
    splits = std::max(splits, (w.ksteps + max_per - 1) / max_per);
    return std::min(splits, w.ksteps);
}

void launch_dec_gemv(int mode, bool norm, int type, const DecGemvArgs& a, int splits, cudaStream_t s) {
    if (a.rows % 128 != 0) throw Error(JV_ERR_UNSUPPORTED, "decode matvec: rows must be a multiple of 128");
    switch (mode) {
        case DEC_STORE: norm ? launch_dec_mode<DEC_STORE, true>(type, a, splits, s) : launch_dec_mode<DEC_STORE, false>(type, a, splits, s); break;
        case DEC_ADD: launch_dec_mode<DEC_ADD, false>(type, a, splits, s); break;
        case DEC_SWIGLU: launch_dec_mode<DEC_SWIGLU, true>(type, a, splits, s); break;
        case DEC_QKV: launch_dec_mode<DEC_QKV, true>(type, a, splits, s); break;
        case DEC_HEAD: launch_dec_mode<DEC_HEAD, true>(type, a, splits, s); break;
        default: throw Error(JV_ERR_ARG, "decode matvec: bad mode");
    }
    note_launch();
}

void launch_dec_attn(const DecAttnArgs& a, int splits, cudaStream_t s) {
    const int group = a.heads / a.kv_heads;
    if (group < 1 || group > 8 || a.heads % a.kv_heads) throw Error(JV_ERR_UNSUPPORTED, "decode attention: group size");
    launch_pdl(k_dec_attn, dim3(a.kv_heads, splits), dim3(32 * group), 0, s, a);
    note_launch();
}

}  // namespace jv
