// gguf_synth.cpp — fills the tensor data of a random-init GGUF at the benchmark's sizes.
//
// Weights are N(0, std^2) from a counter-based generator (splitmix64 + Box-Muller), so a
// tensor's values depend only on (seed, tensor id, element index), never on the thread
// count. They are quantized with the rules of the `gguf` Python package's quantizers
// (gguf/quants.py 0.19.0, Q8_0/Q4_0/Q5_1 quantize_blocks), which the reference's converter
// uses (tools/convert_shieldstral_to_gguf.py:285-292): the same fp32 input gives the same
// bytes, checked by tests/test_synth.py against the package itself.
//
// Built twice: as libjvsynth.so (called in-process through ctypes) and, with -DJVS_MAIN, as the
// stand-alone `jvsynth` program, which fills a file whose header is already written. The
// benchmark's reference arm uses the program, so that process loads no library of this package.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// Element i of tensor `tid` under `seed`, as float32 N(0, std^2).
inline float normal_at(uint64_t seed, uint32_t tid, int64_t i, float stdev) {
    uint64_t key = splitmix64(seed ^ ((uint64_t)tid << 40)) ^ (uint64_t)(i >> 1);
    uint64_t h1 = splitmix64(key), h2 = splitmix64(h1);
    double u1 = ((double)(h1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);  // (0, 1]
    double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);          // [0, 1)
    double r = std::sqrt(-2.0 * std::log(u1));
    double z = (i & 1) ? r * std::sin(2.0 * M_PI * u2) : r * std::cos(2.0 * M_PI * u2);
    return (float)(z * (double)stdev);
}

// float32 -> IEEE half, round to nearest even (numpy's astype(np.float16)).
uint16_t f2h(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000;
    uint32_t e = (x >> 23) & 0xFF;
    uint32_t m = x & 0x7FFFFF;
    if (e == 0xFF) return (uint16_t)(sign | 0x7C00 | (m ? 0x200 : 0));
    int exp = (int)e - 127 + 15;
    if (exp >= 31) return (uint16_t)(sign | 0x7C00);
    if (exp <= 0) {
        if (exp < -10) return (uint16_t)sign;
        m |= 0x800000;
        int shift = 14 - exp;
        uint32_t half = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1), mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t half = ((uint32_t)exp << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFF;
    if (rem > 0x1000 || (rem == 0x1000 && (half & 1))) half++;
    return (uint16_t)(sign | half);
}

// Q8_0.quantize_blocks: d = max|x| / 127; q = round-half-away(x * (1/d)).
void q8_0(const float* x, uint8_t* out) {
    float amax = 0.f;
    for (int j = 0; j < 32; j++) amax = std::max(amax, std::fabs(x[j]));
    float d = amax / 127.0f;
    float id = d == 0.f ? 0.f : 1.0f / d;
    uint16_t dh = f2h(d);
    std::memcpy(out, &dh, 2);
    for (int j = 0; j < 32; j++) out[2 + j] = (uint8_t)(int8_t)std::round(x[j] * id);
}

// Q4_0.quantize_blocks: d = x[argmax|x|] / -8; q = min(15, trunc(x * (1/d) + 8.5)).
void q4_0(const float* x, uint8_t* out) {
    int imax = 0;
    float amax = -1.f;
    for (int j = 0; j < 32; j++)
        if (std::fabs(x[j]) > amax) { amax = std::fabs(x[j]); imax = j; }
    float mx = x[imax];
    float d = mx / -8.0f;
    float id = d == 0.f ? 0.f : 1.0f / d;
    uint8_t q[32];
    for (int j = 0; j < 32; j++) {
        float v = std::trunc(x[j] * id + 8.5f);
        int iv = (int)v;
        q[j] = (uint8_t)std::min(15, std::max(0, iv));
    }
    uint16_t dh = f2h(d);
    std::memcpy(out, &dh, 2);
    for (int j = 0; j < 16; j++) out[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
}

// Q5_1.quantize_blocks: d = (max - min) / 31, m = min; q = min(31, trunc((x - min) / d + 0.5)).
void q5_1(const float* x, uint8_t* out) {
    float mx = x[0], mn = x[0];
    for (int j = 1; j < 32; j++) { mx = std::max(mx, x[j]); mn = std::min(mn, x[j]); }
    float d = (mx - mn) / 31.0f;
    float id = d == 0.f ? 0.f : 1.0f / d;
    uint8_t q[32];
    for (int j = 0; j < 32; j++) {
        float v = std::trunc((x[j] - mn) * id + 0.5f);
        int iv = (int)v;
        q[j] = (uint8_t)std::min(31, std::max(0, iv));
    }
    uint16_t dh = f2h(d), mh = f2h(mn);
    std::memcpy(out, &dh, 2);
    std::memcpy(out + 2, &mh, 2);
    uint32_t qh = 0;
    for (int j = 0; j < 32; j++) qh |= (uint32_t)(q[j] >> 4) << j;
    std::memcpy(out + 4, &qh, 4);
    for (int j = 0; j < 16; j++) out[8 + j] = (uint8_t)((q[j] & 0x0F) | (uint8_t)(q[j + 16] << 4));
}

int block_bytes(int type) { return type == 8 ? 34 : type == 2 ? 18 : type == 7 ? 24 : type == 0 ? 128 : -1; }

// Formats written as random blocks (no quantizer: the bytes are drawn directly, with scales
// chosen so the decoded weights spread like N(0, 0.02^2) on average). GGML ids: Q4_1 3, Q5_0 6,
// Q2_K 10, Q3_K 11, Q4_K 12, Q5_K 13, Q6_K 14. Returns {weights per block, bytes per block}.
bool random_block_type(int type, int& bw, int& bb) {
    switch (type) {
        case 3: bw = 32; bb = 20; return true;
        case 6: bw = 32; bb = 22; return true;
        case 10: bw = 256; bb = 84; return true;
        case 11: bw = 256; bb = 110; return true;
        case 12: bw = 256; bb = 144; return true;
        case 13: bw = 256; bb = 176; return true;
        case 14: bw = 256; bb = 210; return true;
        default: return false;
    }
}

void random_block(int type, uint64_t key, uint8_t* out) {
    int bw, bb;
    random_block_type(type, bw, bb);
    uint64_t st = splitmix64(key);
    for (int i = 0; i < bb; i += 8) {
        st = splitmix64(st);
        for (int j = 0; j < 8 && i + j < bb; j++) out[i + j] = (uint8_t)(st >> (8 * j));
    }
    auto put16 = [&](int off, float v) {
        uint16_t h = f2h(v);
        std::memcpy(out + off, &h, 2);
    };
    switch (type) {
        case 3:  // Q4_1: d, m; v = d q + m, q in [0, 15]
            put16(0, 0.0043f);
            put16(2, -0.0043f * 7.5f);
            break;
        case 6:  // Q5_0: d; v = d (q - 16)
            put16(0, 0.0022f);
            break;
        case 10: {  // Q2_K: scale nibbles >= 1
            for (int i = 0; i < 16; i++) out[i] = (uint8_t)((out[i] & 0xF0) | (1 + (out[i] & 0x0F) % 15));
            put16(80, 0.0022f);
            put16(82, 0.0022f * 1.6f);
            break;
        }
        case 11:  // Q3_K: d (signed 6-bit scales in the packed bytes)
            put16(108, 0.0005f);
            break;
        case 12:  // Q4_K: d, dmin
            put16(0, 0.00014f);
            put16(2, 0.00014f * 7.5f);
            break;
        case 13:  // Q5_K
            put16(0, 0.00007f);
            put16(2, 0.00007f * 15.5f);
            break;
        case 14:  // Q6_K: scales in [1, 63], d last
            for (int i = 192; i < 208; i++) out[i] = (uint8_t)(1 + out[i] % 63);
            put16(208, 0.000034f);
            break;
    }
}

void quantize_row(int type, const float* x, int64_t cols, uint8_t* out) {
    if (type == 0) {
        std::memcpy(out, x, (size_t)cols * 4);
        return;
    }
    int bb = block_bytes(type);
    for (int64_t b = 0; b < cols / 32; b++) {
        const float* xb = x + b * 32;
        uint8_t* ob = out + b * bb;
        if (type == 8) q8_0(xb, ob);
        else if (type == 2) q4_0(xb, ob);
        else q5_1(xb, ob);
    }
}

}  // namespace

extern "C" {

// Quantize n floats (a multiple of 32) with the gguf package's rules. type: 8 Q8_0, 2 Q4_0,
// 7 Q5_1, 0 F32. Returns bytes written, -1 on a bad type or length.
int64_t jvs_quantize(const float* src, int type, int64_t n, uint8_t* dst) {
    if (block_bytes(type) < 0 || (type != 0 && n % 32 != 0)) return -1;
    quantize_row(type, src, n, dst);
    return type == 0 ? n * 4 : n / 32 * block_bytes(type);
}

void jvs_normal(uint64_t seed, uint32_t tid, float stdev, int64_t n, float* out) {
    for (int64_t i = 0; i < n; i++) out[i] = normal_at(seed, tid, i, stdev);
}

// Fill a rows x cols tensor (row-major GGUF blocks) at dst with quantized N(0, std^2)
// weights of tensor `tid`. Returns bytes written or -1.
int64_t jvs_fill(uint8_t* dst, int type, int64_t rows, int64_t cols, uint64_t seed, uint32_t tid, float stdev,
                 int threads) {
    int bw, bb;
    if (random_block_type(type, bw, bb)) {  // random blocks, one counter-based stream per block
        if (cols % bw != 0) return -1;
        const int64_t nb = cols / bw, rb = nb * bb;
        int nt = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
        nt = (int)std::min<int64_t>(nt, rows);
        std::vector<std::thread> pool;
        for (int w = 0; w < nt; w++)
            pool.emplace_back([=] {
                for (int64_t r = w; r < rows; r += nt)
                    for (int64_t b = 0; b < nb; b++)
                        random_block(type, splitmix64(seed ^ ((uint64_t)tid << 40)) ^ (uint64_t)(r * nb + b),
                                     dst + r * rb + b * bb);
            });
        for (auto& t : pool) t.join();
        return rows * rb;
    }
    if (block_bytes(type) < 0 || (type != 0 && cols % 32 != 0)) return -1;
    int64_t rb = type == 0 ? cols * 4 : cols / 32 * block_bytes(type);
    int nt = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
    nt = (int)std::min<int64_t>(nt, rows);
    std::vector<std::thread> pool;
    for (int w = 0; w < nt; w++)
        pool.emplace_back([=] {
            std::vector<float> row((size_t)cols);
            for (int64_t r = w; r < rows; r += nt) {
                for (int64_t k = 0; k < cols; k++) row[(size_t)k] = normal_at(seed, tid, r * cols + k, stdev);
                quantize_row(type, row.data(), cols, dst + r * rb);
            }
        });
    for (auto& t : pool) t.join();
    return rows * rb;
}
}

#ifdef JVS_MAIN
#include <cstdio>
#include <cstdlib>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

// jvsynth FILE TYPE SEED STD THREADS, then one line per matrix on stdin: "TID OFFSET ROWS COLS"
// (OFFSET = the tensor's absolute byte offset in FILE). Exit status 0 when every matrix was filled.
int main(int argc, char** argv) {
    if (argc != 6) {
        std::fprintf(stderr, "usage: jvsynth FILE TYPE SEED STD THREADS < 'TID OFFSET ROWS COLS' lines\n");
        return 2;
    }
    const int type = std::atoi(argv[2]);
    const uint64_t seed = std::strtoull(argv[3], nullptr, 10);
    const float stdev = std::strtof(argv[4], nullptr);
    const int threads = std::atoi(argv[5]);
    int fd = open(argv[1], O_RDWR);
    if (fd < 0) {
        std::perror(argv[1]);
        return 1;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        std::perror("fstat");
        return 1;
    }
    void* base = mmap(nullptr, (size_t)st.st_size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    if (base == MAP_FAILED) {
        std::perror("mmap");
        return 1;
    }
    unsigned tid;
    long long off, rows, cols;
    int rc = 0;
    while (std::scanf("%u %lld %lld %lld", &tid, &off, &rows, &cols) == 4) {
        int bw, bb;
        const int64_t rb = type == 0 ? cols * 4 : random_block_type(type, bw, bb) ? cols / bw * bb : cols / 32 * block_bytes(type);
        if (off < 0 || rows <= 0 || off + rows * rb > (long long)st.st_size) {
            std::fprintf(stderr, "jvsynth: tensor %u does not fit the file\n", tid);
            rc = 1;
            break;
        }
        if (jvs_fill((uint8_t*)base + off, type, rows, cols, seed, tid, stdev, threads) != rows * rb) {
            std::fprintf(stderr, "jvsynth: tensor %u: bad type or shape\n", tid);
            rc = 1;
            break;
        }
    }
    if (msync(base, (size_t)st.st_size, MS_SYNC) != 0) rc = 1;
    munmap(base, (size_t)st.st_size);
    close(fd);
    return rc;
}
#endif
