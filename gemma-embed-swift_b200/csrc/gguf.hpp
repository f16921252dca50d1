// gguf.hpp -- read-only GGUF v2/v3 reader over a shared memory mapping.
//
// Behaviour of the reference reader (Sources/GemmaEmbed/GGUF/GGUFFile.swift:21-67,
// GGUFValue.swift:6-131, MappedFile.swift:17-50): header and version check, typed metadata,
// tensor directory with at most 4 dimensions, aligned data section (general.alignment,
// default 32), and a bounds check of every tensor against the file size.  Errors carry the
// same status classes as the reference's GemmaEmbedError cases.
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace ge {

enum GgmlType : uint32_t { GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8, GGML_BF16 = 30 };

struct GgufError {
    int code;
    std::string message;
};

struct GgufValue {
    uint32_t type = 0;        // GGUF metadata value type
    uint32_t elem = 0;        // element type of an array
    uint64_t count = 0;       // element count of an array
    const uint8_t* raw = nullptr;  // first byte of the value (of the first element for arrays)
};

struct GgufTensor {
    std::string name;
    std::vector<int64_t> shape;  // ne order: contiguous dimension first
    uint32_t type = 0;
    uint64_t offset = 0;
    const uint8_t* data = nullptr;

    int64_t elements() const;
    int64_t bytes() const;
    int64_t cols() const { return shape.empty() ? 1 : shape[0]; }
    int64_t rows() const { return elements() / cols(); }
};

class GgufFile {
public:
    GgufFile() = default;
    ~GgufFile();
    GgufFile(const GgufFile&) = delete;
    GgufFile& operator=(const GgufFile&) = delete;

    // Returns 0 or a status code with `err` filled in.
    int open(const std::string& path, GgufError& err);

    uint32_t version = 0;
    size_t size = 0;
    std::map<std::string, GgufValue> metadata;
    std::vector<GgufTensor> tensors;

    const GgufTensor* tensor(const std::string& name) const;
    bool get_int(const std::string& key, int64_t& out) const;
    bool get_float(const std::string& key, float& out) const;
    bool get_string(const std::string& key, std::string& out) const;
    // Integer array (int32/uint32 elements) and bool array accessors.
    bool get_int_array(const std::string& key, std::vector<int32_t>& out) const;
    bool get_bool_array(const std::string& key, std::vector<bool>& out) const;
    bool get_bool(const std::string& key, bool& out) const;
    bool get_float_array(const std::string& key, std::vector<float>& out) const;  // float32 elements
    // String array (tokenizer.ggml.tokens, tokenizer.ggml.merges).
    bool get_string_array(const std::string& key, std::vector<std::string>& out) const;
    // Element count of a string array.
    bool get_string_array_count(const std::string& key, int64_t& out) const;

private:
    uint8_t* base_ = nullptr;
    size_t mapped_ = 0;
    std::map<std::string, size_t> index_;
};

int64_t ggml_block_elems(uint32_t type);
int64_t ggml_block_bytes(uint32_t type);

}  // namespace ge
