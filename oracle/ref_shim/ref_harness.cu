// C entry points over the reference engine's own CUDA kernels
// (src/cuda/*.cu compiled unmodified), so tests can run the reference on the
// same device buffers as this library and compare. Written for this
// repository; test infrastructure only (the GPU-side checker).
//
// ref_forward replays Engine::inference (src/Engine.cpp:37-114) with the
// reference kernels, including the EmbedLookup host gather + H2D copy +
// dequantize_embeddings sequence (src/EmbedLookup.cpp:49-78).
#include "GGUF.hpp"
#include "Kernels.hpp"
#include "Weight.hpp"

#include <cuda_fp16.h>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#define REF_API extern "C" __attribute__((visibility("default")))

namespace refstub {
void put(const std::string& name, ggml_type type, int64_t ne0, int64_t ne1, const void* data, size_t bytes);
void drop(const std::string& name);
}  // namespace refstub

namespace {
thread_local std::string g_last_error;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_last_error = e.what();
        return 1;
    } catch (const std::out_of_range& e) {
        g_last_error = e.what();
        return 2;
    } catch (const std::length_error& e) {
        g_last_error = e.what();
        return 2;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return 3;
    }
}

// The fp16-KV configuration stores K/V in half precision; the reference keeps
// fp32. The replay rounds each newly written row to fp16 and back so both see
// the same cache contents.
__global__ void round_rows_f16(float* data, size_t count) {
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < count) data[i] = __half2float(__float2half_rn(data[i]));
}

enum { SLOT_ATTN_NORM, SLOT_Q, SLOT_K, SLOT_V, SLOT_Q_NORM, SLOT_K_NORM, SLOT_O, SLOT_FFN_NORM, SLOT_GATE, SLOT_UP,
       SLOT_DOWN, SLOTS };
}  // namespace

REF_API const char* ref_last_error() { return g_last_error.c_str(); }

REF_API int ref_weight_create(const char* name, int type, int64_t ne0, int64_t ne1, const void* host, size_t bytes,
                              void** out) {
    return guarded([&] {
        refstub::put(name, static_cast<ggml_type>(type), ne0, ne1, host, bytes);
        try {
            GGUF model("memory", false);
            *out = new Weight(model, name);
        } catch (...) {
            refstub::drop(name);
            throw;
        }
        refstub::drop(name);
    });
}

REF_API int ref_weight_set_rows(void* w, int64_t ne1) {
    return guarded([&] { static_cast<Weight*>(w)->dimension.at(1) = ne1; });
}

REF_API void* ref_weight_data(void* w) { return static_cast<Weight*>(w)->device_buffer.data; }

REF_API void ref_weight_destroy(void* w) { delete static_cast<Weight*>(w); }

REF_API int ref_matmul(const float* x, void* w, float* y, size_t rows, void* stream) {
    return guarded([&] {
        kernels::matmul(x, *static_cast<Weight*>(w), y, rows, static_cast<cudaStream_t>(stream));
    });
}

REF_API int ref_rms_norm(const float* x, void* gamma, float* y, size_t rows, size_t width, float eps) {
    return guarded([&] { kernels::rms_norm(x, *static_cast<Weight*>(gamma), y, rows, width, eps); });
}

REF_API int ref_rope(float* x, size_t tokens, size_t heads, size_t head_dim, size_t pos, float base) {
    return guarded([&] { kernels::rope(x, tokens, heads, head_dim, pos, base); });
}

REF_API int ref_attention(const float* q, const float* k, const float* v, float* out, size_t tokens, size_t heads,
                          size_t kv_heads, size_t head_dim, size_t offset) {
    return guarded([&] { kernels::attention(q, k, v, out, tokens, heads, kv_heads, head_dim, offset); });
}

REF_API int ref_residual_add(float* state, const float* branch, size_t count) {
    return guarded([&] { kernels::residual_add(state, branch, count); });
}

REF_API int ref_silu_multiply(const float* gate, const float* up, float* out, size_t count) {
    return guarded([&] { kernels::silu_multiply(gate, up, out, count); });
}

REF_API int ref_dequantize_embeddings(const void* packed, float* out, size_t rows, size_t width, size_t row_bytes,
                                      int type) {
    return guarded([&] {
        kernels::dequantize_embeddings(packed, out, rows, width, row_bytes, static_cast<ggml_type>(type));
    });
}

REF_API int ref_argmax(const float* logits, size_t count, uint32_t* out) {
    return guarded([&] { *out = kernels::argmax(logits, count); });
}

REF_API int ref_synchronize() {
    return guarded([&] {
        const auto e = cudaDeviceSynchronize();
        if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
    });
}

// Engine::inference replay. weights: SLOTS*layers + 2 Weight handles (last two:
// output_norm, token_embd). embd_host: the packed token_embd table in host
// memory (EmbedLookup keeps it there). k_cache/v_cache: device fp32
// [layers][capacity][kv_heads*head_dim]. logits (vocab floats) and hidden
// ([layers+1][width], last token) are optional device outputs.
REF_API int ref_forward(void* const* weights, int layers, int width, int heads, int kv_heads, int head_dim, int ffn,
                        int vocab, float eps, float rope_base, const void* embd_host, size_t embd_row_bytes,
                        float* k_cache, float* v_cache, size_t capacity, const uint32_t* token_ids, size_t tokens,
                        size_t offset, int kv_round_f16, float* logits, float* hidden, uint32_t* next_token) {
    return guarded([&] {
        using namespace kernels;
        auto W = [&](int layer, int slot) -> const Weight& {
            return *static_cast<const Weight*>(weights[SLOTS * layer + slot]);
        };
        const Weight& output_norm = *static_cast<const Weight*>(weights[SLOTS * layers + 0]);
        const Weight& token_embd = *static_cast<const Weight*>(weights[SLOTS * layers + 1]);
        if (offset + tokens > capacity) throw std::length_error("Chat session cache capacity exceeded");
        const size_t kv_width = size_t(kv_heads) * head_dim;

        // EmbedLookup::lookup: host gather, H2D copy, GPU dequantisation.
        std::vector<std::byte> packed(tokens * embd_row_bytes);
        for (size_t i = 0; i < tokens; ++i) {
            if (token_ids[i] >= size_t(vocab)) throw std::out_of_range("Embedding token ID out of range");
            std::memcpy(packed.data() + i * embd_row_bytes,
                        static_cast<const std::byte*>(embd_host) + size_t(token_ids[i]) * embd_row_bytes,
                        embd_row_bytes);
        }
        DeviceBuffer device_rows(packed.data(), packed.size());
        DeviceBuffer token_buffer(tokens * width * sizeof(float));
        dequantize_embeddings(device_rows.data, static_cast<float*>(token_buffer.data), tokens, width,
                              embd_row_bytes, token_embd.datatype);

        DeviceBuffer normalized(tokens * width * sizeof(float));
        DeviceBuffer q(tokens * heads * head_dim * sizeof(float));
        DeviceBuffer k(tokens * kv_heads * head_dim * sizeof(float));
        DeviceBuffer q_normalized(tokens * heads * head_dim * sizeof(float));
        DeviceBuffer attended(tokens * heads * head_dim * sizeof(float));
        DeviceBuffer branch(tokens * width * sizeof(float));
        DeviceBuffer gate(tokens * ffn * sizeof(float));
        DeviceBuffer up(tokens * ffn * sizeof(float));
        DeviceBuffer activated(tokens * ffn * sizeof(float));
        auto fp = [](DeviceBuffer& b) { return static_cast<float*>(b.data); };
        auto snapshot = [&](int index) {
            if (!hidden) return;
            const auto e = cudaMemcpy(hidden + size_t(index) * width, fp(token_buffer) + (tokens - 1) * width,
                                      width * sizeof(float), cudaMemcpyDeviceToDevice);
            if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
        };
        snapshot(0);

        for (int i = 0; i < layers; ++i) {
            float* cached_k = k_cache + size_t(i) * capacity * kv_width;
            float* cached_v = v_cache + size_t(i) * capacity * kv_width;
            float* new_k = cached_k + offset * kv_width;
            float* new_v = cached_v + offset * kv_width;

            rms_norm(fp(token_buffer), W(i, SLOT_ATTN_NORM), fp(normalized), tokens, width, eps);
            matmul(fp(normalized), W(i, SLOT_Q), fp(q), tokens);
            matmul(fp(normalized), W(i, SLOT_K), fp(k), tokens);
            matmul(fp(normalized), W(i, SLOT_V), new_v, tokens);

            rms_norm(fp(q), W(i, SLOT_Q_NORM), fp(q_normalized), tokens * heads, head_dim, eps);
            rms_norm(fp(k), W(i, SLOT_K_NORM), new_k, tokens * kv_heads, head_dim, eps);
            rope(fp(q_normalized), tokens, heads, head_dim, offset, rope_base);
            rope(new_k, tokens, kv_heads, head_dim, offset, rope_base);
            if (kv_round_f16) {
                const size_t n = tokens * kv_width;
                round_rows_f16<<<(n + 255) / 256, 256>>>(new_k, n);
                round_rows_f16<<<(n + 255) / 256, 256>>>(new_v, n);
                detail::check_launch();
            }

            attention(fp(q_normalized), cached_k, cached_v, fp(attended), tokens, heads, kv_heads, head_dim, offset);

            matmul(fp(attended), W(i, SLOT_O), fp(branch), tokens);
            residual_add(fp(token_buffer), fp(branch), tokens * width);

            rms_norm(fp(token_buffer), W(i, SLOT_FFN_NORM), fp(normalized), tokens, width, eps);
            matmul(fp(normalized), W(i, SLOT_GATE), fp(gate), tokens);
            matmul(fp(normalized), W(i, SLOT_UP), fp(up), tokens);
            silu_multiply(fp(gate), fp(up), fp(activated), tokens * ffn);
            matmul(fp(activated), W(i, SLOT_DOWN), fp(branch), tokens);
            residual_add(fp(token_buffer), fp(branch), tokens * width);
            snapshot(i + 1);
        }

        rms_norm(fp(token_buffer) + (tokens - 1) * width, output_norm, fp(normalized), 1, width, eps);
        DeviceBuffer logit_buffer(size_t(vocab) * sizeof(float));
        matmul(fp(normalized), token_embd, fp(logit_buffer), 1);
        if (logits) {
            const auto e = cudaMemcpy(logits, logit_buffer.data, size_t(vocab) * sizeof(float),
                                      cudaMemcpyDeviceToDevice);
            if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
        }
        const uint32_t next = argmax(fp(logit_buffer), size_t(vocab));
        if (next_token) *next_token = next;
    });
}

// One block of Engine::inference (src/Engine.cpp:71-103) with the reference
// kernels on given residual-stream rows: layer_weights are the SLOTS Weight
// handles of one layer; x (device, [tokens][width]) is updated in place;
// k_cache / v_cache (device fp32 [capacity][kv_heads*head_dim]) are this
// layer's caches, rows [0, offset) the prefix, rows offset.. written here
// (rounded to fp16 when kv_round_f16, as the fp16-KV configuration stores
// them).
REF_API int ref_layer(void* const* layer_weights, int width, int heads, int kv_heads, int head_dim, int ffn, float eps,
                      float rope_base, float* x, float* k_cache, float* v_cache, size_t capacity, size_t tokens,
                      size_t offset, int kv_round_f16) {
    return guarded([&] {
        using namespace kernels;
        auto W = [&](int slot) -> const Weight& { return *static_cast<const Weight*>(layer_weights[slot]); };
        if (offset + tokens > capacity) throw std::length_error("Chat session cache capacity exceeded");
        const size_t kv_width = size_t(kv_heads) * head_dim;
        DeviceBuffer normalized(tokens * width * sizeof(float));
        DeviceBuffer q(tokens * heads * head_dim * sizeof(float));
        DeviceBuffer k(tokens * kv_width * sizeof(float));
        DeviceBuffer q_normalized(tokens * heads * head_dim * sizeof(float));
        DeviceBuffer attended(tokens * heads * head_dim * sizeof(float));
        DeviceBuffer branch(tokens * width * sizeof(float));
        DeviceBuffer gate(tokens * ffn * sizeof(float));
        DeviceBuffer up(tokens * ffn * sizeof(float));
        DeviceBuffer activated(tokens * ffn * sizeof(float));
        auto fp = [](DeviceBuffer& b) { return static_cast<float*>(b.data); };
        float* new_k = k_cache + offset * kv_width;
        float* new_v = v_cache + offset * kv_width;

        rms_norm(x, W(SLOT_ATTN_NORM), fp(normalized), tokens, width, eps);
        matmul(fp(normalized), W(SLOT_Q), fp(q), tokens);
        matmul(fp(normalized), W(SLOT_K), fp(k), tokens);
        matmul(fp(normalized), W(SLOT_V), new_v, tokens);
        rms_norm(fp(q), W(SLOT_Q_NORM), fp(q_normalized), tokens * heads, head_dim, eps);
        rms_norm(fp(k), W(SLOT_K_NORM), new_k, tokens * kv_heads, head_dim, eps);
        rope(fp(q_normalized), tokens, heads, head_dim, offset, rope_base);
        rope(new_k, tokens, kv_heads, head_dim, offset, rope_base);
        if (kv_round_f16) {
            const size_t n = tokens * kv_width;
            round_rows_f16<<<(n + 255) / 256, 256>>>(new_k, n);
            round_rows_f16<<<(n + 255) / 256, 256>>>(new_v, n);
            detail::check_launch();
        }
        attention(fp(q_normalized), k_cache, v_cache, fp(attended), tokens, heads, kv_heads, head_dim, offset);
        matmul(fp(attended), W(SLOT_O), fp(branch), tokens);
        residual_add(x, fp(branch), tokens * width);
        rms_norm(x, W(SLOT_FFN_NORM), fp(normalized), tokens, width, eps);
        matmul(fp(normalized), W(SLOT_GATE), fp(gate), tokens);
        matmul(fp(normalized), W(SLOT_UP), fp(up), tokens);
        silu_multiply(fp(gate), fp(up), fp(activated), tokens * ffn);
        matmul(fp(activated), W(SLOT_DOWN), fp(branch), tokens);
        residual_add(x, fp(branch), tokens * width);
        const auto e = cudaDeviceSynchronize();
        if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
    });
}
