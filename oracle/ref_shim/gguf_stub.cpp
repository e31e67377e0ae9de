// In-memory stand-in for the reference's GGUF reader, written for this
// repository. It implements only the GGUF members that the reference's
// Weight constructor calls (src/Weight.cpp:53-61: get_tensor_info and
// read_tensor_data), serving synthetic tensors registered by the harness
// instead of a model file. Test infrastructure only.
#include "GGUF.hpp"

#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>

namespace refstub {
struct Entry {
    ggml_type type;
    std::array<int64_t, GGML_MAX_DIMS> dims;
    std::vector<std::byte> bytes;
};
std::mutex registry_mutex;
std::map<std::string, Entry> registry;

void put(const std::string& name, ggml_type type, int64_t ne0, int64_t ne1, const void* data, size_t bytes) {
    Entry e;
    e.type = type;
    e.dims = {ne0, ne1, 1, 1};
    e.bytes.resize(bytes);
    if (bytes) std::memcpy(e.bytes.data(), data, bytes);
    std::lock_guard<std::mutex> lock(registry_mutex);
    registry[name] = std::move(e);
}

void drop(const std::string& name) {
    std::lock_guard<std::mutex> lock(registry_mutex);
    registry.erase(name);
}
}  // namespace refstub

extern "C" void ggml_free(ggml_context*) {}
extern "C" void gguf_free(gguf_context*) {}

GGUF::GGUF(const std::filesystem::path& path, bool) : path_(path) {
    std::lock_guard<std::mutex> lock(refstub::registry_mutex);
    for (const auto& [name, e] : refstub::registry) {
        TensorInfo info{};
        info.name = name;
        info.dimensions = e.dims;
        info.type = e.type;
        info.bytes = e.bytes.size();
        info.file_offset = 0;
        tensors_.push_back(info);
    }
}

const GGUF::TensorInfo* GGUF::get_tensor_info(const std::string& name) const {
    for (const auto& t : tensors_)
        if (t.name == name) return &t;
    throw std::runtime_error("Tensor not found: " + name);
}

std::vector<std::byte> GGUF::read_tensor_data(const std::string& name) const {
    std::lock_guard<std::mutex> lock(refstub::registry_mutex);
    auto it = refstub::registry.find(name);
    if (it == refstub::registry.end()) throw std::runtime_error("Tensor data not found: " + name);
    return it->second.bytes;
}
