// gguf.h — a GGUF v2/v3 reader for the runtime (reference src/Jevstral/Gguf/GgufFile.cs).
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace jv {

struct GgufTensor {
    std::string name;
    std::vector<int64_t> shape;  // ne[0] is the fastest axis (elements per row)
    int type = 0;
    uint64_t offset = 0;         // relative to the data section
};

class Gguf {
public:
    explicit Gguf(const std::string& path);
    ~Gguf();
    Gguf(const Gguf&) = delete;
    Gguf& operator=(const Gguf&) = delete;

    const std::string& path() const { return path_; }
    bool has_num(const std::string& k) const { return nums_.count(k) != 0; }
    double num(const std::string& k, double dflt) const;
    double req_num(const std::string& k) const;
    std::string str(const std::string& k, const std::string& dflt) const;
    int64_t array_len(const std::string& k, int64_t dflt) const;
    const GgufTensor* tensor(const std::string& name) const;
    const uint8_t* data(const GgufTensor& t) const { return base_ + data_offset_ + t.offset; }

    static int block_size(int type);    // GgmlTypeInfo.BlockSize (GgmlType.cs:55-64)
    static int type_size(int type);     // GgmlTypeInfo.TypeSize  (GgmlType.cs:67-106)
    static int64_t row_bytes(int type, int64_t elements);  // GgmlTypeInfo.RowBytes (:112-120)

private:
    std::string path_;
    uint8_t* base_ = nullptr;
    size_t length_ = 0;
    uint64_t data_offset_ = 0;
    uint64_t cur_ = 0;
    std::map<std::string, double> nums_;
    std::map<std::string, std::string> strs_;
    std::map<std::string, int64_t> arrays_;
    std::map<std::string, GgufTensor> tensors_;

    void need(uint64_t n);
    uint32_t u32();
    uint64_t u64();
    std::string read_str();
    void skip_value(uint32_t type);
    void read_value(const std::string& key, uint32_t type);
};

}  // namespace jv
