// Minimal GGUF (v2/v3) reader: metadata scalars and memory-mapped tensor data.
//
// Replaces the parts of src/model_loader.cpp:21-169 that the decoder needs:
// the mtd.text.* configuration keys (read_config, :116-128) and the raw bytes
// of token_embd / qwen3.blk.* / qwen3.output_norm tensors.  The file is mapped
// read-only; tensor pointers stay valid while the reader lives.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace mtb {

enum GgmlType : uint32_t { GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8 };

struct GgufTensor {
    std::string name;
    uint32_t type = 0;
    std::vector<int64_t> ne;  // ggml order: ne[0] is the contiguous axis
    uint64_t offset = 0;      // relative to the data section
    const uint8_t* data = nullptr;
    uint64_t nbytes = 0;
};

class GgufFile {
public:
    GgufFile() = default;
    ~GgufFile();
    GgufFile(const GgufFile&) = delete;
    GgufFile& operator=(const GgufFile&) = delete;

    // Returns false and sets error() on any malformed input.
    bool open(const std::string& path);
    const std::string& error() const { return error_; }

    const GgufTensor* tensor(const std::string& name) const;
    uint32_t get_u32(const std::string& key, uint32_t def) const;
    float get_f32(const std::string& key, float def) const;

private:
    std::string error_;
    void* map_ = nullptr;
    size_t map_size_ = 0;
    std::map<std::string, GgufTensor> tensors_;
    std::map<std::string, uint64_t> u_;  // integer-valued keys
    std::map<std::string, double> f_;    // float-valued keys
};

// Bytes of `n` elements of a type along ne[0] (q8_0: 34 bytes per 32).
uint64_t ggml_row_bytes(uint32_t type, int64_t n);

}  // namespace mtb
