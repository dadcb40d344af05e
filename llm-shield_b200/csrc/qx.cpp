// qx.cpp — conversion of GGUF block formats to the affine layout T_QX the kernels decode.
//
// Every block format the reference decodes by an affine rule per group of weights
// (src/Jevstral/Quantization/Dequantizer.cs: Q4_0 :155, Q4_1 :184, Q5_0 :211, Q5_1 :240,
// Q8_0 :270, Q8_1 :307, Q2_K :323, Q3_K :346, Q4_K :396, Q5_K :421, Q6_K :450) can be written, for
// each 16 consecutive weights, as
//     v = (a * q) + c          (fp32, two roundings, never fused)
// with a small integer q and fp32 a, c taken from the block: a is the fp32 factor the reference
// multiplies q by (d, or its fp32 product d * scale), and c is what it adds after (m, or minus
// dmin * min). Where the reference only multiplies, c is -0.0, which leaves every product,
// including a negative zero, unchanged. So the decoded value equals the reference's bit for bit.
//
// Row-major T_QX ("raw" rows for the device re-tiling): for every 64 columns, 64 int8 q, then
// 4 fp32 a, then 4 fp32 c (one per 16 columns) = 96 bytes per 64 columns.
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "gguf.h"
#include "jv_internal.h"

namespace jv {
namespace {

float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16, exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { e++; man <<= 1; } while ((man & 0x400) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000 | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}
uint16_t rd16(const uint8_t* p) { uint16_t v; std::memcpy(&v, p, 2); return v; }
uint32_t rd32(const uint8_t* p) { uint32_t v; std::memcpy(&v, p, 4); return v; }

// One group of 16 weights in the affine form.
struct Group {
    float a, c;
    int8_t q[16];
};

// The groups of one GGUF block (32 or 256 weights) in order.
int block_groups(int type, const uint8_t* b, Group* g) {
    const float nz = -0.0f;
    switch (type) {
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: case T_Q8_1: {
            int q[32];
            float a = h2f(rd16(b)), c = nz;
            if (type == T_Q8_0 || type == T_Q8_1) {
                const int8_t* qs = (const int8_t*)(b + (type == T_Q8_0 ? 2 : 4));
                for (int j = 0; j < 32; j++) q[j] = qs[j];
            } else {
                const uint8_t* qs = b + (type == T_Q4_0 ? 2 : type == T_Q4_1 ? 4 : type == T_Q5_0 ? 6 : 8);
                uint32_t qh = type == T_Q5_0 ? rd32(b + 2) : type == T_Q5_1 ? rd32(b + 4) : 0;
                for (int j = 0; j < 16; j++) {
                    q[j] = qs[j] & 0x0F;
                    q[16 + j] = qs[j] >> 4;
                    if (type == T_Q5_0 || type == T_Q5_1) {
                        q[j] |= (int)((qh >> j) & 1) << 4;
                        q[16 + j] |= (int)((qh >> (j + 16)) & 1) << 4;
                    }
                }
                const int bias = type == T_Q4_0 ? 8 : type == T_Q5_0 ? 16 : 0;
                for (int j = 0; j < 32; j++) q[j] -= bias;
                if (type == T_Q4_1 || type == T_Q5_1) c = h2f(rd16(b + 2));
            }
            for (int h = 0; h < 2; h++) {
                g[h].a = a;
                g[h].c = c;
                for (int j = 0; j < 16; j++) g[h].q[j] = (int8_t)q[16 * h + j];
            }
            return 2;
        }
        case T_Q2_K: {
            const uint8_t* scales = b;
            const uint8_t* qs = b + 16;
            float d = h2f(rd16(b + 80)), dmin = h2f(rd16(b + 82));
            for (int o = 0; o < 256; o++) {
                int gi = o >> 4, gg = o >> 7, s = (o >> 5) & 3, j = o & 31;
                g[gi].a = d * (float)(scales[gi] & 0x0F);
                g[gi].c = -(dmin * (float)(scales[gi] >> 4));
                g[gi].q[o & 15] = (int8_t)((qs[gg * 32 + j] >> (2 * s)) & 3);
            }
            return 16;
        }
        case T_Q3_K: {
            const uint8_t* hmask = b;
            const uint8_t* qs = b + 32;
            const uint8_t* scales = b + 96;
            float d = h2f(rd16(b + 108));
            for (int k = 0; k < 16; k++) {
                int low = scales[k & 7] >> (k < 8 ? 0 : 4);
                int high = scales[8 + (k & 3)] >> (2 * (k >> 2));
                int sc = (int)(int8_t)(((low & 0x0F) | ((high & 0x03) << 4)) - 32);
                g[k].a = d * (float)sc;
                g[k].c = nz;
            }
            for (int o = 0; o < 256; o++) {
                int gg = o >> 7, s = (o >> 5) & 3, j = o & 31;
                int ql = (qs[gg * 32 + j] >> (2 * s)) & 3;
                int qh = ((hmask[j] >> (gg * 4 + s)) & 1) ^ 1;
                g[o >> 4].q[o & 15] = (int8_t)(ql - (qh << 2));
            }
            return 16;
        }
        case T_Q4_K: case T_Q5_K: {
            const bool five = type == T_Q5_K;
            float d = h2f(rd16(b)), dmin = h2f(rd16(b + 2));
            const uint8_t* p = b + 4;
            uint8_t sc[8], mn[8];
            for (int i = 0; i < 4; i++) {
                sc[i] = p[i] & 0x3F;
                mn[i] = p[4 + i] & 0x3F;
                sc[4 + i] = (uint8_t)((p[8 + i] & 0x0F) | ((p[i] >> 2) & 0x30));
                mn[4 + i] = (uint8_t)((p[8 + i] >> 4) | ((p[4 + i] >> 2) & 0x30));
            }
            const uint8_t* qh = b + 16;
            const uint8_t* qs = b + (five ? 48 : 16);
            for (int o = 0; o < 256; o++) {
                int sb = o >> 5, gg = sb >> 1, s = sb & 1, j = o & 31;
                int q = (qs[gg * 32 + j] >> (4 * s)) & 0x0F;
                if (five) q |= ((qh[j] >> sb) & 1) << 4;
                g[o >> 4].a = d * (float)sc[sb];
                g[o >> 4].c = -(dmin * (float)mn[sb]);
                g[o >> 4].q[o & 15] = (int8_t)q;
            }
            return 16;
        }
        case T_Q6_K: {
            const uint8_t* ql = b;
            const uint8_t* qh = b + 128;
            const int8_t* scales = (const int8_t*)(b + 192);
            float d = h2f(rd16(b + 208));
            for (int o = 0; o < 256; o++) {
                int gg = o >> 7, s = (o >> 6) & 1, j = o & 63;
                int lo = (ql[gg * 64 + j] >> (4 * s)) & 0x0F;
                int hi = (qh[gg * 32 + (j & 31)] >> (2 * (s * 2 + (j >> 5)))) & 0x03;
                g[o >> 4].a = d * (float)scales[o >> 4];
                g[o >> 4].c = nz;
                g[o >> 4].q[o & 15] = (int8_t)((lo | (hi << 4)) - 32);
            }
            return 16;
        }
        default:
            throw Error(JV_ERR_UNSUPPORTED, "GGML type " + std::to_string(type) + " has no affine form");
    }
}

}  // namespace

bool qx_expressible(int type) {
    switch (type) {
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: case T_Q8_1:
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return true;
        default: return false;
    }
}

int64_t qx_row_bytes(int cols) { return (int64_t)cols / 64 * 96; }

void qx_convert_rows(int type, const uint8_t* src, int64_t src_row_bytes, int rows, int cols, uint8_t* dst) {
    if (cols % 256 != 0 && (cols % 64 != 0 || Gguf::block_size(type) > 64))
        throw Error(JV_ERR_UNSUPPORTED, "a row of " + std::to_string(cols) + " weights does not convert to the affine layout");
    const int bs = Gguf::block_size(type), ts = Gguf::type_size(type);
    const int nt = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
    std::vector<std::thread> pool;
    for (int w = 0; w < nt; w++)
        pool.emplace_back([=] {
            std::vector<Group> groups((size_t)cols / 16);
            for (int r = w; r < rows; r += nt) {
                const uint8_t* row = src + (int64_t)r * src_row_bytes;
                int gi = 0;
                for (int b = 0; b < cols / bs; b++) gi += block_groups(type, row + (int64_t)b * ts, groups.data() + gi);
                uint8_t* out = dst + (int64_t)r * qx_row_bytes(cols);
                for (int k = 0; k < cols / 64; k++) {
                    uint8_t* u = out + (int64_t)k * 96;
                    for (int h = 0; h < 4; h++) {
                        const Group& gr = groups[(size_t)k * 4 + h];
                        std::memcpy(u + 16 * h, gr.q, 16);
                        std::memcpy(u + 64 + 4 * h, &gr.a, 4);
                        std::memcpy(u + 80 + 4 * h, &gr.c, 4);
                    }
                }
            }
        });
    for (auto& t : pool) t.join();
}

}  // namespace jv
