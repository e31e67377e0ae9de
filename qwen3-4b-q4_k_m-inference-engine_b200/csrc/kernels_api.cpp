// C++ drop-in (include/Kernels.hpp, include/Weight.hpp) over the C ABI:
// status codes are turned back into the reference's exception types
// (std::invalid_argument, std::out_of_range, std::runtime_error).
#include "../../include/Kernels.hpp"

#include <stdexcept>
#include <string>
#include <utility>

#include "../../include/q4k_b200.h"

#define Q4K_CXX_API __attribute__((visibility("default")))

namespace {

void raise(int status) {
    if (status == Q4K_OK) return;
    const std::string msg = q4k_last_error();
    if (status == Q4K_EINVAL) throw std::invalid_argument(msg);
    if (status == Q4K_ERANGE) throw std::out_of_range(msg);
    throw std::runtime_error(msg);
}

void cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + cudaGetErrorString(e));
}

}  // namespace

// ------------------------------------------------------------ DeviceBuffer
// Every buffer is one stream-ordered allocation on its own stream; the
// owning handle is (data, bytes, stream) and a moved-from buffer is empty.
// Errors: a null host source for a non-empty upload is the caller's mistake
// (std::invalid_argument); anything CUDA reports is std::runtime_error, and
// a failed upload releases the allocation before throwing.
namespace {

void* stream_allocate(std::size_t n, cudaStream_t s) {
    void* p = nullptr;
    if (n == 0) return p;
    const cudaError_t e = cudaMallocAsync(&p, n, s);
    if (e != cudaSuccess) {
        // an allocation failure is not sticky: clear it so that the next
        // launch check does not report it again
        (void)cudaGetLastError();
        throw std::runtime_error(std::string("DeviceBuffer allocation: ") + cudaGetErrorString(e));
    }
    return p;
}

void stream_release(void* p, cudaStream_t s) noexcept {
    if (p) cudaFreeAsync(p, s);
}

}  // namespace

Q4K_CXX_API DeviceBuffer::DeviceBuffer(std::size_t n, cudaStream_t s)
    : data(stream_allocate(n, s)), bytes(n), stream(s) {}

Q4K_CXX_API DeviceBuffer::DeviceBuffer(const void* source, std::size_t n, cudaStream_t s)
    : DeviceBuffer((n > 0 && !source) ? throw std::invalid_argument("DeviceBuffer: no host bytes to upload") : n, s) {
    if (n == 0) return;
    // the copy is complete before the constructor returns, so the caller
    // may release the host bytes at once (the reference relies on this)
    cudaError_t e = cudaMemcpyAsync(data, source, n, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        stream_release(std::exchange(data, nullptr), stream);
        bytes = 0;
        throw std::runtime_error(std::string("DeviceBuffer upload: ") + cudaGetErrorString(e));
    }
}

Q4K_CXX_API DeviceBuffer::~DeviceBuffer() { stream_release(data, stream); }

Q4K_CXX_API DeviceBuffer::DeviceBuffer(DeviceBuffer&& o) noexcept : data(o.data), bytes(o.bytes), stream(o.stream) {
    o.data = nullptr;
    o.bytes = 0;
    o.stream = nullptr;
}

Q4K_CXX_API DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& o) noexcept {
    // take o's buffer into a temporary and swap: the old one is released
    // by the temporary's destructor, and self-assignment is a no-op swap
    DeviceBuffer taken(std::move(o));
    std::swap(data, taken.data);
    std::swap(bytes, taken.bytes);
    std::swap(stream, taken.stream);
    return *this;
}

// ------------------------------------------------------------------ Weight
Q4K_CXX_API Weight::Weight(std::string tensor_name, ggml_type type, std::vector<std::int64_t> dims,
                           const void* gguf_bytes)
    : name(std::move(tensor_name)), datatype(type), dimension(std::move(dims)) {
    const std::int64_t ne0 = dimension.size() > 0 ? dimension[0] : 0;
    std::int64_t ne1 = 1;
    for (std::size_t i = 1; i < dimension.size(); ++i) ne1 *= dimension[i];
    const std::size_t bytes = q4k_weight_device_bytes(static_cast<int>(type), ne0, ne1);
    if (bytes == 0) throw std::invalid_argument("Unsupported tensor type or shape for " + name);
    device_buffer = DeviceBuffer(bytes);
    raise(q4k_weight_upload(static_cast<int>(type), ne0, ne1, gguf_bytes, device_buffer.data, device_buffer.stream));
}

// ---------------------------------------------------------------- kernels
namespace kernels::detail {

Q4K_CXX_API int get_sm_count() {
    int device = 0;
    cuda(cudaGetDevice(&device), "CUDA device query failed: ");
    int count = 0;
    cuda(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device), "CUDA SM count query failed: ");
    return count;
}

Q4K_CXX_API void check_launch() {
    const auto error = cudaGetLastError();
    if (error != cudaSuccess) throw std::runtime_error(std::string("CUDA kernel launch failed: ") + cudaGetErrorString(error));
}

}  // namespace kernels::detail

namespace kernels {

namespace {
void stream_check(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA stream error: ") + cudaGetErrorString(e));
}
}  // namespace

Q4K_CXX_API CudaStream::CudaStream() { stream_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking)); }

Q4K_CXX_API CudaStream::~CudaStream() {
    if (stream_) cudaStreamDestroy(stream_);
}

Q4K_CXX_API CudaStream::CudaStream(CudaStream&& o) noexcept : stream_(std::exchange(o.stream_, nullptr)) {}

Q4K_CXX_API CudaStream& CudaStream::operator=(CudaStream&& o) noexcept {
    if (this != &o) {
        if (stream_) cudaStreamDestroy(stream_);
        stream_ = std::exchange(o.stream_, nullptr);
    }
    return *this;
}

Q4K_CXX_API cudaStream_t CudaStream::get() const {
    if (!stream_) throw std::logic_error("CUDA stream was moved from");
    return stream_;
}

Q4K_CXX_API void CudaStream::synchronize() const { stream_check(cudaStreamSynchronize(get())); }

Q4K_CXX_API bool CudaStream::ready() const {
    const auto e = cudaStreamQuery(get());
    if (e == cudaErrorNotReady) return false;
    stream_check(e);
    return true;
}

Q4K_CXX_API void rms_norm(const float* input, const Weight& scale, float* output, size_t rows, size_t width,
                          float epsilon) {
    if (rows == 0) return;
    // rms_norm.cu:34-36
    if (width == 0 || !(epsilon > 0.0f) || scale.datatype != GGML_TYPE_F32 || scale.dimension.empty() ||
        static_cast<size_t>(scale.dimension[0]) != width)
        throw std::invalid_argument("RMSNorm requires an F32 scale matching the row width and positive epsilon");
    raise(q4k_rms_norm(input, static_cast<const float*>(scale.device_buffer.data), output, rows, width, epsilon,
                       nullptr));
}

Q4K_CXX_API void matmul(const float* input, const Weight& weight, float* output, size_t rows, cudaStream_t stream) {
    // matmul.cu:132-136
    if (weight.datatype != GGML_TYPE_Q4_K && weight.datatype != GGML_TYPE_Q6_K)
        throw std::invalid_argument("matmul supports Q4_K and Q6_K weights only");
    if (weight.dimension.size() < 2 || weight.dimension[0] <= 0 || weight.dimension[0] % 256 != 0 ||
        weight.dimension[1] <= 0)
        throw std::invalid_argument("Invalid matmul weight dimensions");
    if (rows == 0) return;
    raise(q4k_matmul(input, weight.device_buffer.data, static_cast<int>(weight.datatype), weight.dimension[0],
                     weight.dimension[1], output, rows, stream));
}

Q4K_CXX_API void matmul(const float* input, const Weight& weight, float* output, size_t rows,
                        const CudaStream& stream) {
    matmul(input, weight, output, rows, stream.get());
}

Q4K_CXX_API void rope(float* input, size_t tokens, size_t heads, size_t head_dim, size_t position_offset,
                      float frequency_base) {
    raise(q4k_rope(input, tokens, heads, head_dim, position_offset, frequency_base, nullptr));
}

Q4K_CXX_API void attention(const float* q, const float* k, const float* v, float* output, size_t tokens,
                           size_t query_heads, size_t kv_heads, size_t head_dim, size_t query_offset) {
    raise(q4k_attention(q, k, v, output, tokens, query_heads, kv_heads, head_dim, query_offset, nullptr));
}

Q4K_CXX_API void residual_add(float* state, const float* branch, size_t count) {
    raise(q4k_residual_add(state, branch, count, nullptr));
}

Q4K_CXX_API void silu_multiply(const float* gate, const float* up, float* output, size_t count) {
    raise(q4k_silu_multiply(gate, up, output, count, nullptr));
}

Q4K_CXX_API void dequantize_embeddings(const void* packed, float* output, size_t rows, size_t width, size_t row_bytes,
                                       ggml_type type) {
    raise(q4k_dequantize_embeddings(packed, output, rows, width, row_bytes, static_cast<int>(type), nullptr));
}

Q4K_CXX_API uint32_t argmax(const float* logits, size_t vocabulary_size) {
    uint32_t result = 0;
    raise(q4k_argmax(logits, vocabulary_size, &result, nullptr));
    return result;
}

}  // namespace kernels
