// Drop-in replacement for the reference's include/Weight.hpp (same public
// members and semantics: src/Weight.cpp:6-61), backed by the C ABI of
// q4k_b200.h. The device bytes are in this library's device layout
// (q4k_weight_device_bytes), so kernels::matmul can stream them with 16-byte
// bulk copies; `dimension` keeps the GGUF shape (dimension[0] = inputs per
// row, dimension[1] = rows) and may be narrowed by the caller, as the
// reference's tests do (MatmulTests.cpp:33).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#if __has_include(<ggml.h>)
#include <ggml.h>
#else
// GGML tensor type ids used by the hot path (values of the GGUF format).
enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_K = 12,
    GGML_TYPE_Q6_K = 14,
    GGML_TYPE_COUNT = 40,
};
#endif

struct DeviceBuffer {
    void* data{nullptr};
    std::size_t bytes{0};
    cudaStream_t stream{nullptr};

    // Stream-ordered allocation plus a synchronous upload (Weight.cpp:6-23).
    DeviceBuffer(const void* source, std::size_t bytes, cudaStream_t stream = nullptr);
    explicit DeviceBuffer(std::size_t bytes, cudaStream_t stream = nullptr);
    ~DeviceBuffer();

    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    DeviceBuffer(DeviceBuffer&& other) noexcept;
    DeviceBuffer& operator=(DeviceBuffer&& other) noexcept;
};

struct Weight {
    std::string name;
    ggml_type datatype;
    DeviceBuffer device_buffer{nullptr, 0};
    std::vector<std::int64_t> dimension;

    // From a tensor in GGUF file layout held in host memory.
    Weight(std::string tensor_name, ggml_type type, std::vector<std::int64_t> dims, const void* gguf_bytes);

    // Reference-compatible constructor (src/Weight.cpp:53-61): any model
    // object offering get_tensor_info(name) -> {type, dimensions} and
    // read_tensor_data(name) -> byte container, such as the reference's GGUF.
    template <class Model>
    Weight(const Model& model, const std::string& tensor_name)
        : Weight(tensor_name, static_cast<ggml_type>(model.get_tensor_info(tensor_name)->type),
                 std::vector<std::int64_t>(model.get_tensor_info(tensor_name)->dimensions.begin(),
                                           model.get_tensor_info(tensor_name)->dimensions.end()),
                 model.read_tensor_data(tensor_name).data()) {}
};
