// gguf_reader.h -- minimal GGUF v2/v3 reader for the AR weights (host side).
//
// Reads the header, the KV pairs this library needs (integer and float32 scalars; strings and arrays
// are skipped), the tensor directory and the tensor bytes. Replaces the gguf_init_from_file / fread
// upload of the reference loader (src/gsv_ar.cpp:545-570).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace gsvcu {

struct GgufTensor {
    std::string name;
    std::vector<int64_t> dims;   // ne0 first (ne0 = innermost)
    uint32_t type = 0;           // ggml type id: 0 F32, 1 F16, 8 Q8_0
    uint64_t offset = 0;         // within the data section
    uint64_t nbytes = 0;
    const uint8_t* data = nullptr;
};

class GgufFile {
public:
    bool open(const std::string& path, std::string& err);
    const GgufTensor* tensor(const std::string& name) const;
    bool get_u32(const std::string& key, uint32_t& out) const;
    bool get_f32(const std::string& key, float& out) const;
    const std::vector<GgufTensor>& tensors() const { return tensors_; }

private:
    std::vector<uint8_t> buf_;
    std::vector<GgufTensor> tensors_;
    std::map<std::string, size_t> index_;
    std::map<std::string, uint64_t> u64_;   // integer scalars
    std::map<std::string, float> f32_;      // float32 scalars
};

}  // namespace gsvcu
