// Drop-in replacement for the reference's include/Kernels.hpp: the same
// namespace, launch signatures, argument checks and exception types, with
// the work done by this library's sm_100a kernels through the C ABI of
// q4k_b200.h. Float activations are row-major device buffers; launches use
// the legacy default stream unless a stream parameter is given.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "Weight.hpp"

namespace kernels::detail {

inline constexpr unsigned threads = 256;

int get_sm_count();
void check_launch();

}  // namespace kernels::detail

namespace kernels {

class CudaStream {
public:
    CudaStream();
    ~CudaStream();
    CudaStream(const CudaStream&) = delete;
    CudaStream& operator=(const CudaStream&) = delete;
    CudaStream(CudaStream&& other) noexcept;
    CudaStream& operator=(CudaStream&& other) noexcept;

    cudaStream_t get() const;
    void synchronize() const;
    bool ready() const;

private:
    cudaStream_t stream_{nullptr};
};

void rms_norm(const float* input, const Weight& scale, float* output, size_t rows, size_t width, float epsilon);

void matmul(const float* input, const Weight& weight, float* output, size_t rows, cudaStream_t stream = nullptr);

void matmul(const float* input, const Weight& weight, float* output, size_t rows, const CudaStream& stream);

void rope(float* input, size_t tokens, size_t heads, size_t head_dim, size_t position_offset, float frequency_base);

void attention(const float* q, const float* k, const float* v, float* output, size_t tokens, size_t query_heads,
               size_t kv_heads, size_t head_dim, size_t query_offset = 0);

void residual_add(float* state, const float* branch, size_t count);

void silu_multiply(const float* gate, const float* up, float* output, size_t count);

void dequantize_embeddings(const void* packed, float* output, size_t rows, size_t width, size_t row_bytes,
                           ggml_type type);

uint32_t argmax(const float* logits, size_t vocabulary_size);

}  // namespace kernels
