// gguf.cuh — in-memory GGUF v3 file (host side of the model loader).
#pragma once
#include "common.cuh"
#include <map>
#include <cmath>

namespace vkb {

struct GgufValue {
    uint32_t type = 0;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
    std::vector<GgufValue> arr;
};

struct GgufTensor {
    std::string name;
    std::vector<int64_t> dims;  // PyTorch order, as stored
    uint32_t tag = 0;
    uint64_t offset = 0, nbytes = 0, n_elem = 0;
};

struct GgufFile {
    std::vector<uint8_t> bytes;
    std::map<std::string, GgufValue> meta;
    std::vector<GgufTensor> tensors;
    std::map<std::string, size_t> index;
    uint64_t data_base = 0;
    const uint8_t* data(const GgufTensor& t) const { return bytes.data() + data_base + t.offset; }
    // Looks up a tensor and (when dims is non-empty) checks its shape.
    const GgufTensor& tensor(const std::string& name, const std::vector<int64_t>& dims = {}) const;
    bool has(const std::string& name) const { return index.count(name) != 0; }
    uint32_t u32(const std::string& key) const;
    std::vector<float> f32(const std::string& name, const std::vector<int64_t>& dims = {}) const;
};

GgufFile* gguf_open(const std::string& path);
void gguf_parse(GgufFile& g);

}  // namespace vkb
