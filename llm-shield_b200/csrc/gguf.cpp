// gguf.cpp — GGUF v2/v3 parsing: header, metadata, tensor table, data alignment and the
// truncation check (reference src/Jevstral/Gguf/GgufFile.cs:76-172). The file is mapped
// read-only; weights are copied to the device by the model loader and the mapping is
// released when the model finishes loading.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "jv_internal.h"

namespace jv {

int Gguf::block_size(int type) {
    switch (type) {
        case T_F32: case T_F16: case T_BF16: return 1;
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: case T_Q8_1: return 32;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return 256;
        default: return -1;
    }
}
int Gguf::type_size(int type) {
    switch (type) {
        case T_F32: return 4;
        case T_F16: case T_BF16: return 2;
        case T_Q4_0: return 18;
        case T_Q4_1: return 20;
        case T_Q5_0: return 22;
        case T_Q5_1: return 24;
        case T_Q8_0: return 34;
        case T_Q8_1: return 36;
        case T_Q2_K: return 84;
        case T_Q3_K: return 110;
        case T_Q4_K: return 144;
        case T_Q5_K: return 176;
        case T_Q6_K: return 210;
        default: return -1;
    }
}
int64_t Gguf::row_bytes(int type, int64_t elements) {
    int b = block_size(type);
    if (b <= 0) throw Error(JV_ERR_UNSUPPORTED, "GGML type " + std::to_string(type) + " is not on the B200 path");
    if (elements % b != 0)
        throw Error(JV_ERR_FORMAT, "rows must be a multiple of " + std::to_string(b) + " elements; got " + std::to_string(elements));
    return elements / b * type_size(type);
}

void Gguf::need(uint64_t n) {
    if (cur_ + n > length_) throw Error(JV_ERR_FORMAT, path_ + " ends inside its header; re-download it.");
}
uint32_t Gguf::u32() { need(4); uint32_t v; std::memcpy(&v, base_ + cur_, 4); cur_ += 4; return v; }
uint64_t Gguf::u64() { need(8); uint64_t v; std::memcpy(&v, base_ + cur_, 8); cur_ += 8; return v; }
std::string Gguf::read_str() {
    uint64_t n = u64();
    need(n);
    std::string s((const char*)base_ + cur_, (size_t)n);
    cur_ += n;
    return s;
}

static int scalar_bytes(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;      // u8 i8 bool
        case 2: case 3: return 2;              // u16 i16
        case 4: case 5: case 6: return 4;      // u32 i32 f32
        case 10: case 11: case 12: return 8;   // u64 i64 f64
        default: return -1;
    }
}

void Gguf::skip_value(uint32_t t) {
    if (t == 8) { uint64_t n = u64(); need(n); cur_ += n; return; }
    int b = scalar_bytes(t);
    if (b < 0) throw Error(JV_ERR_FORMAT, path_ + ": unknown metadata value type " + std::to_string(t));
    need((uint64_t)b);
    cur_ += (uint64_t)b;
}

void Gguf::read_value(const std::string& key, uint32_t t) {
    if (t == 8) { strs_[key] = read_str(); return; }
    if (t == 9) {
        uint32_t et = u32();
        uint64_t n = u64();
        arrays_[key] = (int64_t)n;
        if (et == 9) throw Error(JV_ERR_FORMAT, path_ + ": nested metadata arrays are not supported");
        if (et != 8) {
            int b = scalar_bytes(et);
            if (b < 0) throw Error(JV_ERR_FORMAT, path_ + ": unknown array element type");
            need((uint64_t)b * n);
            cur_ += (uint64_t)b * n;
        } else {
            for (uint64_t i = 0; i < n; i++) skip_value(8);
        }
        return;
    }
    int b = scalar_bytes(t);
    if (b < 0) throw Error(JV_ERR_FORMAT, path_ + ": unknown metadata value type " + std::to_string(t));
    need((uint64_t)b);
    const uint8_t* p = base_ + cur_;
    double v = 0;
    switch (t) {
        case 0: v = *p; break;
        case 1: v = (int8_t)*p; break;
        case 2: { uint16_t x; std::memcpy(&x, p, 2); v = x; break; }
        case 3: { int16_t x; std::memcpy(&x, p, 2); v = x; break; }
        case 4: { uint32_t x; std::memcpy(&x, p, 4); v = x; break; }
        case 5: { int32_t x; std::memcpy(&x, p, 4); v = x; break; }
        case 6: { float x; std::memcpy(&x, p, 4); v = x; break; }
        case 7: v = *p ? 1 : 0; break;
        case 10: { uint64_t x; std::memcpy(&x, p, 8); v = (double)x; break; }
        case 11: { int64_t x; std::memcpy(&x, p, 8); v = (double)x; break; }
        case 12: { double x; std::memcpy(&x, p, 8); v = x; break; }
    }
    cur_ += (uint64_t)b;
    nums_[key] = v;
}

Gguf::Gguf(const std::string& path) : path_(path) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw Error(JV_ERR_IO, "GGUF not found: " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) { ::close(fd); throw Error(JV_ERR_IO, "cannot stat " + path); }
    length_ = (size_t)st.st_size;
    if (length_ < 24) { ::close(fd); throw Error(JV_ERR_FORMAT, path + " is not a GGUF file (too short)."); }
    void* m = mmap(nullptr, length_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) throw Error(JV_ERR_IO, "cannot map " + path);
    base_ = (uint8_t*)m;
    try {
        uint32_t magic = u32();
        if (magic != 0x46554747u) throw Error(JV_ERR_FORMAT, path + " is not a GGUF file (bad magic).");
        uint32_t version = u32();
        if (version < 2 || version > 3)
            throw Error(JV_ERR_UNSUPPORTED, "GGUF version " + std::to_string(version) + " is not supported (expected 2 or 3).");
        uint64_t n_tensors = u64(), n_kv = u64();
        for (uint64_t i = 0; i < n_kv; i++) {
            std::string key = read_str();
            uint32_t t = u32();
            read_value(key, t);
        }
        for (uint64_t i = 0; i < n_tensors; i++) {
            GgufTensor t;
            t.name = read_str();
            uint32_t dims = u32();
            if (dims > 4) throw Error(JV_ERR_FORMAT, path + ": tensor '" + t.name + "' has too many dimensions");
            for (uint32_t d = 0; d < dims; d++) t.shape.push_back((int64_t)u64());
            t.type = (int)u32();
            t.offset = u64();
            tensors_[t.name] = t;
        }
        uint64_t align = nums_.count("general.alignment") ? (uint64_t)nums_["general.alignment"] : 32;
        if (align == 0) align = 32;
        data_offset_ = cur_ + (align - cur_ % align) % align;
        uint64_t required = data_offset_;
        std::string last;
        for (auto& kv : tensors_) {
            const GgufTensor& t = kv.second;
            if (block_size(t.type) <= 0) continue;
            int64_t elems = 1;
            for (auto s : t.shape) elems *= s;
            if (elems % block_size(t.type) != 0) continue;
            uint64_t end = data_offset_ + t.offset + (uint64_t)(elems / block_size(t.type) * type_size(t.type));
            if (end > required) { required = end; last = t.name; }
        }
        if (length_ < required) {
            double missing = (double)(required - length_) / (1024.0 * 1024 * 1024);
            char buf[64];
            snprintf(buf, sizeof buf, "%.2f", missing);
            throw Error(JV_ERR_IO, path + " is incomplete: " + std::to_string(length_) + " bytes on disk but its " +
                                       std::to_string(tensors_.size()) + " tensors need " + std::to_string(required) +
                                       " (" + buf + " GiB missing; '" + last + "' is the last one). Re-download it.");
        }
    } catch (...) {
        munmap(base_, length_);
        base_ = nullptr;
        throw;
    }
}

Gguf::~Gguf() {
    if (base_) munmap(base_, length_);
}

double Gguf::num(const std::string& k, double dflt) const {
    auto it = nums_.find(k);
    return it == nums_.end() ? dflt : it->second;
}
double Gguf::req_num(const std::string& k) const {
    auto it = nums_.find(k);
    if (it == nums_.end()) throw Error(JV_ERR_FORMAT, path_ + " is missing metadata '" + k + "'.");
    return it->second;
}
std::string Gguf::str(const std::string& k, const std::string& dflt) const {
    auto it = strs_.find(k);
    return it == strs_.end() ? dflt : it->second;
}
int64_t Gguf::array_len(const std::string& k, int64_t dflt) const {
    auto it = arrays_.find(k);
    return it == arrays_.end() ? dflt : it->second;
}
const GgufTensor* Gguf::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

}  // namespace jv
