// GGUF v2/v3 reader for the decode engine's upload path.
//
// Follows Local-LLM-Pure-Go/internal/engine/native/gguf/gguf.go:104-195
// (header, metadata, tensor infos), with two deliberate differences: the data
// section is aligned to general.alignment when the file sets it (the GGUF
// specification; gguf.go:187-192 always uses 32, which misplaces tensors of
// files written with another alignment), and every tensor's byte range is
// checked against the file size before it is read.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace b2 {

enum GgmlType : uint32_t {
    GGML_F32 = 0, GGML_F16 = 1, GGML_Q4_0 = 2, GGML_Q8_0 = 8, GGML_BF16 = 30,
};

struct GgufValue {
    uint32_t type = 0;
    bool is_array = false;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
    uint64_t arr_len = 0;
    std::vector<std::string> strs;  // kept only for small string arrays
};

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> dims;  // dims[0] = columns
    uint32_t type = 0;
    uint64_t offset = 0;         // relative to the data section
    uint64_t elements() const;
    uint64_t bytes() const;      // gguf.go:273-279
};

struct GgufFile {
    std::string path;
    uint32_t version = 0;
    std::map<std::string, GgufValue> meta;
    std::vector<GgufTensor> tensors;
    uint64_t data_offset = 0;
    uint64_t file_size = 0;

    const GgufTensor* find(const std::string& name) const;
    bool get_str(const std::string& k, std::string* out) const;
    bool get_u32(const std::string& k, uint32_t* out) const;   // gguf.go:209-226
    bool get_f32(const std::string& k, float* out) const;      // gguf.go:229-241
    int64_t array_len(const std::string& k) const;
};

uint64_t ggml_type_size(uint32_t t);   // gguf.go:422-457
uint64_t ggml_block_size(uint32_t t);  // gguf.go:460-473

// Returns 0 or a negative B2_ERR_* code with *err describing the failure.
int gguf_parse(const char* path, GgufFile* out, std::string* err);

}  // namespace b2
