// Read-only GGUF model file (format versions 2 and 3): the header, the
// metadata key/value table, the tensor directory, and the tensor data mapped
// from the file. Written from the published format: little-endian; magic
// "GGUF", u32 version, u64 tensor count, u64 metadata count; each key a
// string (u64 length + bytes), a u32 value type and the value (arrays: u32
// element type, u64 count, elements); each tensor a name, u32 dimension
// count, u64 extents (ne0 first), u32 ggml type and u64 offset into the data
// section, which starts at the next multiple of general.alignment (32 when
// absent) after the directory. The reference's loader for the same format is
// src/GGUF.cpp:81-145.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace q4k {

struct GgufValue {
    enum Kind { kInt, kUInt, kFloat, kBool, kString, kArray } kind = kInt;
    int64_t i = 0;
    uint64_t u = 0;
    double f = 0.0;
    std::string s;
    uint32_t array_type = 0;   // element type of an array
    uint64_t array_count = 0;  // elements of an array (their values are not kept)
    // integer value of an integer-typed entry; false for other kinds
    bool as_int(int64_t& out) const;
    bool as_float(double& out) const;
};

struct GgufTensor {
    std::string name;
    uint32_t type = 0;
    std::vector<int64_t> ne;  // extents, ne[0] innermost
    uint64_t offset = 0;      // into the data section
    uint64_t bytes = 0;       // 0 for types this library cannot size
};

class GgufFile {
public:
    // Maps and parses the file; throws Error(Q4K_EINVAL) on anything that is
    // not a well-formed GGUF file of version 2 or 3 (bad magic, truncation,
    // tensors past the end of the file or off the alignment).
    explicit GgufFile(const std::string& path);
    ~GgufFile();
    GgufFile(const GgufFile&) = delete;
    GgufFile& operator=(const GgufFile&) = delete;

    uint32_t version() const { return version_; }
    const std::map<std::string, GgufValue>& metadata() const { return meta_; }
    const GgufValue* find(const std::string& key) const;
    const std::vector<GgufTensor>& tensors() const { return tensors_; }
    const GgufTensor* tensor(const std::string& name) const;
    // First byte of a tensor's data in the mapping.
    const uint8_t* data(const GgufTensor& t) const { return base_ + data_start_ + t.offset; }

private:
    const uint8_t* base_ = nullptr;
    size_t size_ = 0;
    uint64_t data_start_ = 0;
    uint32_t version_ = 0;
    std::map<std::string, GgufValue> meta_;
    std::vector<GgufTensor> tensors_;
};

// Bytes of a tensor of ggml type `type` with ne0 x rows elements (0 when the
// type is not one this library reads).
uint64_t gguf_tensor_bytes(uint32_t type, int64_t ne0, int64_t rows);

}  // namespace q4k
