// The C ABI (include/q4k_b200.h): argument checks that mirror the
// reference's (each cited), launches, and error-code translation.
#include <cuda_runtime.h>
#include <nccl.h>

#include <cmath>
#include <cstring>
#include <limits>
#include <string>
#include <vector>

#include "engine.h"
#include "gguf.h"
#include "nccl_api.h"
#include "ops.h"
#include "q4k_format.h"
#include "q4k_internal.h"

#define Q4K_API extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_last_error;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return Q4K_OK;
    } catch (const q4k::Error& e) {
        g_last_error = e.what();
        return e.status;
    } catch (const std::bad_alloc&) {
        g_last_error = "out of host memory";
        return Q4K_ECUDA;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return Q4K_ECUDA;
    }
}

// Entry points that touch the device: a launch error left by an earlier,
// unrelated call is not this call's error, so clear it first (sticky
// context errors persist regardless and surface on the next CUDA call).
template <class F>
int guarded_cuda(F&& f) {
    return guarded([&] {
        (void)cudaGetLastError();
        f();
    });
}

[[noreturn]] void invalid(const char* msg) { throw q4k::Error(Q4K_EINVAL, msg); }

void launched(cudaError_t e) { q4k::cuda_check(e, "CUDA kernel launch failed"); }

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool quantised(int type) { return type == Q4K_TYPE_Q4_K || type == Q4K_TYPE_Q6_K; }

void check_matrix(int type, int64_t ne0, int64_t ne1) {
    // matmul.cu:132-136
    if (!quantised(type)) invalid("matmul supports Q4_K and Q6_K weights only");
    if (ne0 <= 0 || ne0 % 256 != 0 || ne1 <= 0 || ne1 > (1 << 30))
        invalid("Invalid matmul weight dimensions");
    if (ne0 > 12288) invalid("matmul supports up to 12288 inputs per row (K)");
}

}  // namespace

Q4K_API const char* q4k_last_error(void) { return g_last_error.c_str(); }

Q4K_API int q4k_abi_version(void) { return 2; }

Q4K_API size_t q4k_weight_device_bytes(int type, int64_t ne0, int64_t ne1) {
    if (ne0 <= 0 || ne1 <= 0) return 0;
    if (quantised(type) && ne0 % 256) return 0;
    return (size_t)ne1 * q4k_device_row_bytes(type, (size_t)ne0);
}

Q4K_API int q4k_weight_upload(int type, int64_t ne0, int64_t ne1, const void* host_gguf, void* device, void* stream) {
    return guarded_cuda([&] {
        if (type == Q4K_TYPE_F32) {
            if (ne0 <= 0 || ne1 <= 0 || !host_gguf || !device) invalid("invalid F32 tensor");
            q4k::cuda_check(cudaMemcpyAsync(device, host_gguf, sizeof(float) * ne0 * ne1, cudaMemcpyHostToDevice,
                                            as_stream(stream)),
                            "upload");
            q4k::cuda_check(cudaStreamSynchronize(as_stream(stream)), "upload");
            return;
        }
        check_matrix(type, ne0, ne1);
        if (!host_gguf || !device || reinterpret_cast<uintptr_t>(device) % 16)
            invalid("upload needs host data and a 16-byte aligned device buffer");
        const size_t raw = (size_t)ne1 * q4k_gguf_row_bytes(type, (size_t)ne0);
        void* tmp = nullptr;
        q4k::cuda_check(cudaMallocAsync(&tmp, raw, as_stream(stream)), "cudaMallocAsync");
        cudaError_t e = cudaMemcpyAsync(tmp, host_gguf, raw, cudaMemcpyHostToDevice, as_stream(stream));
        if (e == cudaSuccess)
            e = q4k::relayout(tmp, type, (size_t)ne0, 0, (size_t)ne1, 0, (size_t)ne0 / 256, device, as_stream(stream));
        cudaFreeAsync(tmp, as_stream(stream));
        if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
        q4k::cuda_check(e, "Host-to-device copy failed");
    });
}

Q4K_API int q4k_synth_tensor_host(uint64_t seed, const char* name, int type, int64_t ne0, int64_t ne1,
                                  void* host_gguf) {
    return guarded([&] {
        if (!name || !host_gguf || ne0 <= 0 || ne1 <= 0) invalid("invalid synthetic tensor request");
        const uint64_t key = q4k_tensor_key(seed, name);
        uint8_t* out = static_cast<uint8_t*>(host_gguf);
        if (type == Q4K_TYPE_F32) {
            float* f = static_cast<float*>(host_gguf);
            for (int64_t i = 0; i < ne0 * ne1; ++i) f[i] = q4k_synth_gamma(key, (uint64_t)i);
        } else if (type == Q4K_TYPE_Q4_K || type == Q4K_TYPE_Q6_K) {
            if (ne0 % 256) invalid("quantised rows must hold whole super-blocks");
            const int64_t blocks = ne1 * (ne0 / 256);
            for (int64_t b = 0; b < blocks; ++b) {
                if (type == Q4K_TYPE_Q4_K)
                    q4k_synth_q4k_block(key, (uint64_t)b, out + b * Q4K_Q4_BLOCK);
                else
                    q4k_synth_q6k_block(key, (uint64_t)b, out + b * Q4K_Q6_BLOCK);
            }
        } else {
            invalid("unsupported synthetic tensor type");
        }
    });
}

Q4K_API int q4k_synth_tensor_device(uint64_t seed, const char* name, int type, int64_t ne0, int64_t ne1, void* device,
                                    void* stream) {
    return guarded_cuda([&] {
        if (!name || !device || ne0 <= 0 || ne1 <= 0) invalid("invalid synthetic tensor request");
        const uint64_t key = q4k_tensor_key(seed, name);
        cudaStream_t s = as_stream(stream);
        if (type == Q4K_TYPE_F32) {
            launched(q4k::synth_gamma(key, static_cast<float*>(device), (size_t)(ne0 * ne1), s));
            return;
        }
        check_matrix(type, ne0, ne1);
        const size_t raw = (size_t)ne1 * q4k_gguf_row_bytes(type, (size_t)ne0);
        void* tmp = nullptr;
        q4k::cuda_check(cudaMallocAsync(&tmp, raw, s), "cudaMallocAsync");
        cudaError_t e = q4k::synth_raw(key, type, (size_t)ne0, (size_t)ne1, tmp, s);
        if (e == cudaSuccess) e = q4k::relayout(tmp, type, (size_t)ne0, 0, (size_t)ne1, 0, (size_t)ne0 / 256, device, s);
        cudaFreeAsync(tmp, s);
        launched(e);
    });
}

// Elements [index_base, index_base + n) of the fp16 N(0,1) stream `name`.
Q4K_API int q4k_synth_f16_host(uint64_t seed, const char* name, uint64_t index_base, size_t n, uint16_t* out) {
    return guarded([&] {
        if (!name || (!out && n)) invalid("invalid synthetic request");
        const uint64_t key = q4k_tensor_key(seed, name);
        for (size_t i = 0; i < n; ++i) out[i] = q4k_synth_f16(key, index_base + i);
    });
}

// Elements [0, n) of the fp32 N(0,1) stream `name` (synthetic activations).
Q4K_API int q4k_synth_f32_host(uint64_t seed, const char* name, size_t n, float* out) {
    return guarded([&] {
        if (!name || (!out && n)) invalid("invalid synthetic request");
        const uint64_t key = q4k_tensor_key(seed, name);
        for (size_t i = 0; i < n; ++i) out[i] = q4k_synth_f32(key, i);
    });
}

Q4K_API int q4k_synth_f32_device(uint64_t seed, const char* name, size_t n, float* out, void* stream) {
    return guarded_cuda([&] {
        if (!name || (!out && n)) invalid("invalid synthetic request");
        if (n) launched(q4k::synth_f32(q4k_tensor_key(seed, name), out, n, as_stream(stream)));
    });
}

Q4K_API int q4k_rms_norm(const float* input, const float* scale, float* output, size_t rows, size_t width,
                         float epsilon, void* stream) {
    return guarded_cuda([&] {
        if (rows == 0) return;
        // rms_norm.cu:34-36
        if (width == 0 || !(epsilon > 0.0f) || !scale || !input || !output)
            invalid("RMSNorm requires an F32 scale matching the row width and positive epsilon");
        launched(q4k::rms_norm(input, scale, output, rows, width, epsilon, as_stream(stream)));
    });
}

Q4K_API int q4k_matmul(const float* input, const void* weight, int type, int64_t ne0, int64_t ne1, float* output,
                       size_t rows, void* stream) {
    return guarded_cuda([&] {
        check_matrix(type, ne0, ne1);
        if (rows == 0) return;
        if (!input || !weight || !output) invalid("matmul requires device buffers");
        if (reinterpret_cast<uintptr_t>(input) % 16 || reinterpret_cast<uintptr_t>(weight) % 16)
            invalid("matmul input and weight must be 16-byte aligned");
        if (rows > (size_t)std::numeric_limits<int>::max() / 8) invalid("too many rows");
        q4k::GemvRequest r;
        r.nseg = 1;
        r.seg[0] = {static_cast<const uint8_t*>(weight), output, type, (int)ne1};
        r.K = (int)ne0;
        r.M = (int)rows;
        r.x = input;
        r.ldy = (int)ne1;
        r.epilogue = q4k::EPI_STORE;
        // programmatic dependent launch: the weight stream starts while the
        // preceding kernel on the stream finishes; the input is read and the
        // output written only after the dependency wait, and a preceding
        // kernel that does not signal early (everything that writes weights)
        // still completes first
        r.pdl = true;
        launched(q4k::launch_gemv(r, as_stream(stream)));
    });
}

Q4K_API int q4k_rope(float* input, size_t tokens, size_t heads, size_t head_dim, size_t position_offset,
                     float frequency_base, void* stream) {
    return guarded_cuda([&] {
        if (tokens == 0) return;
        // rope.cu:34-35
        if (heads == 0 || head_dim == 0 || head_dim % 2 != 0 || !(frequency_base > 0.0f))
            invalid("RoPE requires heads, an even head dimension and a positive frequency base");
        if (!input) invalid("RoPE requires a buffer");
        launched(q4k::rope(input, tokens, heads, head_dim, position_offset, frequency_base, as_stream(stream)));
    });
}

Q4K_API int q4k_attention(const float* q, const float* k, const float* v, float* output, size_t tokens,
                          size_t query_heads, size_t kv_heads, size_t head_dim, size_t query_offset, void* stream) {
    return guarded_cuda([&] {
        if (tokens == 0) return;
        // attention.cu:98-105
        if (!q || !k || !v || !output || kv_heads == 0 || query_heads == 0 || query_heads % kv_heads != 0 ||
            head_dim == 0 || head_dim > 256 ||
            tokens > static_cast<size_t>(std::numeric_limits<int>::max()) / query_heads ||
            tokens > std::numeric_limits<size_t>::max() / query_heads / head_dim / sizeof(float))
            invalid("Attention requires valid buffers, divisible Q/KV heads and head_dim in [1, 256]");
        const size_t max_cached = std::numeric_limits<size_t>::max() / kv_heads / head_dim / sizeof(float);
        if (tokens > max_cached || query_offset > max_cached - tokens) invalid("Attention cache dimensions overflow");
        launched(q4k::attention_f32(q, k, v, output, tokens, query_heads, kv_heads, head_dim, query_offset,
                                    as_stream(stream)));
    });
}

Q4K_API int q4k_residual_add(float* state, const float* branch, size_t count, void* stream) {
    return guarded_cuda([&] {
        if (count == 0) return;
        if (!state || !branch) invalid("residual_add requires buffers");
        launched(q4k::residual_add(state, branch, count, as_stream(stream)));
    });
}

Q4K_API int q4k_silu_multiply(const float* gate, const float* up, float* output, size_t count, void* stream) {
    return guarded_cuda([&] {
        if (count == 0) return;
        if (!gate || !up || !output) invalid("silu_multiply requires buffers");
        launched(q4k::silu_multiply(gate, up, output, count, as_stream(stream)));
    });
}

Q4K_API int q4k_dequantize_embeddings(const void* packed, float* output, size_t rows, size_t width, size_t row_bytes,
                                      int type, void* stream) {
    return guarded_cuda([&] {
        if (rows == 0) return;
        // embedding.cu:69-70
        if (!quantised(type)) invalid("Unsupported embedding storage type");
        if (!packed || !output || width == 0 || width % 256 ||
            row_bytes < q4k_gguf_row_bytes(type, width))
            invalid("dequantize_embeddings requires whole super-blocks per row");
        launched(q4k::dequantize_raw(packed, output, rows, width, row_bytes, type, as_stream(stream)));
    });
}

Q4K_API int q4k_argmax(const float* logits, size_t vocabulary_size, uint32_t* result, void* stream) {
    return guarded_cuda([&] {
        // argmax.cu:73-74
        if (!logits || vocabulary_size == 0 || vocabulary_size > UINT32_MAX || !result)
            invalid("Invalid argmax input");
        cudaStream_t s = as_stream(stream);
        const size_t scratch_bytes = q4k::argmax_scratch_bytes() + 64;
        void* scratch = nullptr;
        q4k::cuda_check(cudaMallocAsync(&scratch, scratch_bytes, s), "cudaMallocAsync");
        uint32_t* dev_result = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(scratch) + q4k::argmax_scratch_bytes());
        cudaError_t e = cudaMemsetAsync(scratch, 0, 256, s);
        if (e == cudaSuccess) e = q4k::argmax(logits, vocabulary_size, dev_result, scratch, s);
        uint32_t host = 0;
        if (e == cudaSuccess) e = cudaMemcpyAsync(&host, dev_result, sizeof host, cudaMemcpyDeviceToHost, s);
        cudaFreeAsync(scratch, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        q4k::cuda_check(e, "CUDA argmax failed");
        *result = host;
    });
}

Q4K_API size_t q4k_matmul_argmax_scratch_bytes(void) { return 256 + 1024 * 8; }

Q4K_API int q4k_matmul_ex(const float* input, const float* norm_gamma, float epsilon, int count,
                          const void* const* weights, const int* types, const int64_t* out_rows, float* const* outputs,
                          int64_t ne0, size_t rows, int epilogue, uint32_t* token_device, void* scratch,
                          void* stream) {
    return guarded_cuda([&] {
        if (count < 1 || count > q4k::kMaxSegments || !weights || !types || !out_rows || !outputs)
            invalid("matmul_ex needs 1..4 weights");
        if (epilogue < Q4K_EPI_STORE || epilogue > Q4K_EPI_ARGMAX) invalid("unknown epilogue");
        if (rows == 0) return;
        if (!input || reinterpret_cast<uintptr_t>(input) % 16) invalid("input must be a 16-byte aligned buffer");
        if (norm_gamma && !(epsilon > 0.0f)) invalid("RMSNorm requires a positive epsilon");
        q4k::GemvRequest r;
        r.nseg = count;
        for (int i = 0; i < count; ++i) {
            check_matrix(types[i], ne0, out_rows[i]);
            if (!weights[i] || reinterpret_cast<uintptr_t>(weights[i]) % 16) invalid("weights must be 16-byte aligned");
            float* y = epilogue == Q4K_EPI_SWIGLU ? outputs[0] : outputs[i];
            if (!y && epilogue != Q4K_EPI_ARGMAX) invalid("missing output buffer");
            r.seg[i] = {static_cast<const uint8_t*>(weights[i]), y, types[i], (int)out_rows[i]};
        }
        if (epilogue == Q4K_EPI_SWIGLU && (count != 2 || out_rows[0] != out_rows[1] || types[0] != types[1]))
            invalid("SWIGLU needs two weights of the same type and shape");
        if (epilogue == Q4K_EPI_ARGMAX) {
            if (count != 1 || rows != 1 || !token_device || !scratch) invalid("ARGMAX needs one weight, one row");
            uint8_t* sb = static_cast<uint8_t*>(scratch);
            r.argmax.counter = reinterpret_cast<unsigned*>(sb);
            r.argmax.cand_score = reinterpret_cast<float*>(sb + 256);
            r.argmax.cand_index = reinterpret_cast<uint32_t*>(sb + 256 + 1024 * 4);
            r.argmax.token = token_device;
        }
        if (epilogue != Q4K_EPI_ARGMAX && count > 1 && epilogue != Q4K_EPI_SWIGLU) {
            // independent outputs per weight: each [rows][out_rows[i]] when rows == 1
            if (rows != 1) invalid("several weights with separate outputs need rows == 1");
        }
        r.K = (int)ne0;
        r.M = (int)rows;
        r.x = input;
        r.gamma = norm_gamma;
        r.eps = epsilon;
        r.ldy = (int)out_rows[0];
        r.epilogue = epilogue;
        r.pdl = true;  // as in q4k_matmul
        launched(q4k::launch_gemv(r, as_stream(stream)));
    });
}

Q4K_API int q4k_matmul_batch(const float* input, const float* norm_gamma, float epsilon, int count,
                             const void* const* weights, const int* types, const int64_t* out_rows,
                             float* const* outputs, int64_t ld_out, int64_t ne0, size_t rows, int epilogue,
                             void* stream) {
    return guarded_cuda([&] {
        if (count < 1 || count > 3 || !weights || !types || !out_rows || !outputs)
            invalid("matmul_batch needs 1..3 weights");
        if (epilogue != Q4K_EPI_STORE && epilogue != Q4K_EPI_ADD && epilogue != Q4K_EPI_SWIGLU)
            invalid("matmul_batch epilogues: STORE, ADD, SWIGLU");
        if (rows == 0) return;
        if (rows > (1u << 20)) invalid("too many rows");
        if (!input || reinterpret_cast<uintptr_t>(input) % 16) invalid("input must be a 16-byte aligned buffer");
        if (norm_gamma && !(epsilon > 0.0f)) invalid("RMSNorm requires a positive epsilon");
        q4k::PrefillGemmArgs g;
        g.nseg = count;
        for (int i = 0; i < count; ++i) {
            check_matrix(types[i], ne0, out_rows[i]);
            if (!weights[i] || reinterpret_cast<uintptr_t>(weights[i]) % 16) invalid("weights must be 16-byte aligned");
            float* y = epilogue == Q4K_EPI_SWIGLU ? outputs[0] : outputs[i];
            if (!y) invalid("missing output buffer");
            g.seg[i] = {static_cast<const uint8_t*>(weights[i]), types[i], (int)out_rows[i], y};
        }
        if (epilogue == Q4K_EPI_SWIGLU && (count != 2 || out_rows[0] != out_rows[1] || types[0] != types[1]))
            invalid("SWIGLU needs two weights of the same type and shape");
        if (ld_out < out_rows[0] || ld_out > (int64_t)1 << 30) invalid("ld_out must cover the output rows");
        if (ne0 > 10240) invalid("at most 10240 inputs per row");
        const cudaStream_t s = as_stream(stream);
        // per-call workspace, as the reference's matmul allocates one (matmul.cu:142-145)
        void* ws = nullptr;
        const size_t a_bytes = ((2 * rows * (size_t)ne0 * 2 + 255) / 256) * 256;  // hi and lo planes
        const size_t rows_pad = (rows + 63) / 64 * 64;  // the group sums start 256-byte aligned
        const size_t s_bytes = ((sizeof(float) * (rows_pad + rows * (size_t)ne0 / 32) + 255) / 256) * 256;
        g.K = (int)ne0;
        g.M = (int)rows;
        g.epilogue = epilogue;
        const size_t part_floats = q4k::prefill_gemm_partial_floats(g);  // exactly the split-K partials it will use
        launched(cudaMallocAsync(&ws, a_bytes + s_bytes + part_floats * sizeof(float), s));
        uint16_t* a = static_cast<uint16_t*>(ws);
        float* scale = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + a_bytes);
        float* gsum = scale + rows_pad;  // [rows][ne0 / 32]
        g.partial = part_floats ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + a_bytes + s_bytes) : nullptr;
        g.partial_floats = part_floats;
        cudaError_t e = q4k::prefill_quantise(input, (int)ne0, norm_gamma, epsilon, (int)rows, (int)ne0, a, (int)rows,
                                              gsum, scale, s);
        if (e == cudaSuccess) {
            g.K = (int)ne0;
            g.M = (int)rows;
            g.ldy = (int)ld_out;
            g.epilogue = epilogue;
            g.a = a;
            g.row_scale = scale;
            g.gsum = gsum;
            e = q4k::prefill_gemm(g, s);
        }
        cudaFreeAsync(ws, s);
        launched(e);
    });
}

Q4K_API size_t q4k_attention_decode_scratch_bytes(int query_heads, int kv_heads) {
    if (kv_heads <= 0 || query_heads <= 0) return 0;
    const int splits = q4k::decode_attention_splits(kv_heads);
    return 256 + sizeof(float) * (size_t)query_heads * splits * (q4k::kDecodeHeadDim + 2);
}

// Allocation-free variant: the scratch is the library's fixed device array
// (attention_static_scratch.cu); the launch itself is the regular entry
// point's. Nothing is allocated: only the counters are cleared.
Q4K_API int q4k_attention_decode_f16_static(const float* qkv, const float* q_gamma, const float* k_gamma,
                                            uint16_t* k_cache, uint16_t* v_cache, int capacity,
                                            const int* position_device, int query_heads, int kv_heads, int head_dim,
                                            float epsilon, float rope_base, float* output, void* stream) {
    void* scratch = nullptr;
    const int rc = guarded_cuda([&] {
        if (head_dim != q4k::kDecodeHeadDim || kv_heads <= 0 || kv_heads > 64 || query_heads != 4 * kv_heads)
            invalid("decode attention supports head_dim 128 with 4 query heads per KV head (at most 64 KV heads)");
        const size_t need = 256 + sizeof(float) * (size_t)query_heads *
                                      q4k::decode_attention_splits(kv_heads) * (q4k::kDecodeHeadDim + 2);
        scratch = q4k::attention_static_scratch(need);  // the call below clears its counters
    });
    if (rc != Q4K_OK) return rc;
    return q4k_attention_decode_f16(qkv, q_gamma, k_gamma, k_cache, v_cache, capacity, position_device, query_heads,
                                    kv_heads, head_dim, epsilon, rope_base, output, scratch, stream);
}


Q4K_API int q4k_attention_decode_f16(const float* qkv, const float* q_gamma, const float* k_gamma, uint16_t* k_cache,
                                     uint16_t* v_cache, int capacity, const int* position_device, int query_heads,
                                     int kv_heads, int head_dim, float epsilon, float rope_base, float* output,
                                     void* scratch, void* stream) {
    return guarded_cuda([&] {
        if (!qkv || !q_gamma || !k_gamma || !k_cache || !v_cache || !position_device || !output || !scratch)
            invalid("decode attention requires device buffers");
        if (head_dim != q4k::kDecodeHeadDim || kv_heads <= 0 || kv_heads > 64 || query_heads != 4 * kv_heads ||
            capacity <= 0)
            invalid("decode attention supports head_dim 128 with 4 query heads per KV head (at most 64 KV heads)");
        if (!(epsilon > 0.0f) || !(rope_base > 0.0f)) invalid("epsilon and rope base must be positive");
        if (reinterpret_cast<uintptr_t>(k_cache) % 16 || reinterpret_cast<uintptr_t>(v_cache) % 16)
            invalid("KV caches must be 16-byte aligned");
        if (reinterpret_cast<uintptr_t>(scratch) % 16) invalid("scratch must be 16-byte aligned");
        const int splits = q4k::decode_attention_splits(kv_heads);
        uint8_t* sb = static_cast<uint8_t*>(scratch);
        q4k::DecodeAttnArgs a;
        a.qkv = qkv;
        a.q_gamma = q_gamma;
        a.k_gamma = k_gamma;
        a.k_cache = k_cache;
        a.v_cache = v_cache;
        a.capacity = capacity;
        a.position = position_device;
        a.heads = query_heads;
        a.kv_heads = kv_heads;
        a.eps = epsilon;
        a.rope_base = rope_base;
        a.counters = reinterpret_cast<unsigned*>(sb);
        a.partial_ml = reinterpret_cast<float*>(sb + 256);
        a.partial_o = a.partial_ml + (size_t)query_heads * splits * 2;
        a.out = output;
        a.err = nullptr;
        a.splits = splits;
        a.row_base = 0;
        q4k::KvTensorMap km, vm;
        q4k::cuda_check(q4k::make_kv_tensor_map(k_cache, (long long)kv_heads * capacity, &km), "K tensor map");
        q4k::cuda_check(q4k::make_kv_tensor_map(v_cache, (long long)kv_heads * capacity, &vm), "V tensor map");
        // the per-head counters start every call at zero, even after a
        // launch whose bounded waits gave up before its merge reset them
        q4k::cuda_check(cudaMemsetAsync(sb, 0, 256, as_stream(stream)), "clear attention counters");
        launched(q4k::decode_attention(a, km, vm, as_stream(stream), false));
    });
}

// ---------------------------------------------------------------- engine

struct q4k_engine {
    q4k::Engine impl;
    q4k_engine(const q4k_engine_config& c, const void* id) : impl(c, id) {}
};

Q4K_API void q4k_engine_config_qwen3_4b(q4k_engine_config* c, int capacity) {
    if (!c) return;
    std::memset(c, 0, sizeof *c);
    c->layers = 36;
    c->hidden = 2560;
    c->heads = 32;
    c->kv_heads = 8;
    c->head_dim = 128;
    c->ffn = 9728;
    c->vocab = 151936;
    c->eps = 1e-6f;
    c->rope_base = 1000000.0f;
    c->capacity = capacity;
    c->tp_rank = 0;
    c->tp_world = 1;
    c->device = 0;
}

Q4K_API int q4k_model_tensor(const q4k_engine_config* cfg, int i, char* name, size_t name_len, int* type,
                             int64_t* ne0, int64_t* ne1) {
    return guarded([&] {
        if (!cfg) invalid("config required");
        const auto specs = q4k::model_tensors(*cfg);
        if (i < 0 || (size_t)i >= specs.size()) throw q4k::Error(Q4K_ERANGE, "tensor index out of range");
        const auto& t = specs[i];
        if (name && name_len) {
            std::strncpy(name, t.name.c_str(), name_len - 1);
            name[name_len - 1] = 0;
        }
        if (type) *type = t.type;
        if (ne0) *ne0 = t.ne0;
        if (ne1) *ne1 = t.ne1;
    });
}

// ------------------------------------------------------ GGUF model files

struct q4k_gguf {
    q4k::GgufFile file;
    explicit q4k_gguf(const char* path) : file(path) {}
};

Q4K_API int q4k_gguf_open(const char* path, q4k_gguf** out) {
    return guarded([&] {
        if (!path || !out) invalid("path and output required");
        *out = nullptr;
        *out = new q4k_gguf(path);
    });
}

Q4K_API int q4k_gguf_close(q4k_gguf* f) {
    return guarded([&] { delete f; });
}

Q4K_API int q4k_gguf_tensor_count(const q4k_gguf* f, int64_t* count) {
    return guarded([&] {
        if (!f || !count) invalid("file and output required");
        *count = (int64_t)f->file.tensors().size();
    });
}

Q4K_API int q4k_gguf_tensor_info(const q4k_gguf* f, int64_t i, char* name, size_t name_len, int* type, int64_t* ne0,
                                 int64_t* ne1, const void** data) {
    return guarded([&] {
        if (!f) invalid("file required");
        const auto& ts = f->file.tensors();
        if (i < 0 || (size_t)i >= ts.size()) throw q4k::Error(Q4K_ERANGE, "tensor index out of range");
        const q4k::GgufTensor& t = ts[(size_t)i];
        if (name && name_len) {
            std::strncpy(name, t.name.c_str(), name_len - 1);
            name[name_len - 1] = 0;
        }
        int64_t rows = 1;
        for (size_t d = 1; d < t.ne.size(); ++d) rows *= t.ne[d];
        if (type) *type = (int)t.type;
        if (ne0) *ne0 = t.ne[0];
        if (ne1) *ne1 = rows;
        if (data) *data = f->file.data(t);
    });
}

namespace {
const q4k::GgufValue& gguf_meta(const q4k_gguf* f, const char* key) {
    if (!f || !key) invalid("file and key required");
    const q4k::GgufValue* v = f->file.find(key);
    if (!v) throw q4k::Error(Q4K_ERANGE, std::string("no metadata key ") + key);
    return *v;
}
}  // namespace

Q4K_API int q4k_gguf_meta_int(const q4k_gguf* f, const char* key, int64_t* value) {
    return guarded([&] {
        if (!value) invalid("output required");
        if (!gguf_meta(f, key).as_int(*value)) throw q4k::Error(Q4K_ERANGE, std::string(key) + " is not an integer");
    });
}

Q4K_API int q4k_gguf_meta_float(const q4k_gguf* f, const char* key, double* value) {
    return guarded([&] {
        if (!value) invalid("output required");
        if (!gguf_meta(f, key).as_float(*value)) throw q4k::Error(Q4K_ERANGE, std::string(key) + " is not a number");
    });
}

Q4K_API int q4k_gguf_meta_string(const q4k_gguf* f, const char* key, char* value, size_t len) {
    return guarded([&] {
        if (!value || !len) invalid("output required");
        const q4k::GgufValue& v = gguf_meta(f, key);
        if (v.kind != q4k::GgufValue::kString) throw q4k::Error(Q4K_ERANGE, std::string(key) + " is not a string");
        std::strncpy(value, v.s.c_str(), len - 1);
        value[len - 1] = 0;
    });
}

Q4K_API int q4k_gguf_engine_config(const q4k_gguf* f, int capacity, q4k_engine_config* c) {
    return guarded([&] {
        if (!f || !c) invalid("file and config required");
        if (capacity <= 0) invalid("capacity must be positive");
        const q4k::GgufValue* arch_v = f->file.find("general.architecture");
        const std::string arch = arch_v && arch_v->kind == q4k::GgufValue::kString ? arch_v->s : "qwen3";
        auto need_int = [&](const std::string& key) {
            const q4k::GgufValue* v = f->file.find(key);
            int64_t n = 0;
            if (!v || !v->as_int(n) || n <= 0 || n > (1 << 24))
                throw q4k::Error(Q4K_EINVAL, "GGUF: missing or invalid " + key);
            return (int)n;
        };
        auto opt_float = [&](const std::string& key, double fallback) {
            const q4k::GgufValue* v = f->file.find(key);
            double x = fallback;
            if (v && !v->as_float(x)) throw q4k::Error(Q4K_EINVAL, "GGUF: invalid " + key);
            return x;
        };
        q4k_engine_config cfg{};
        cfg.layers = need_int(arch + ".block_count");
        cfg.hidden = need_int(arch + ".embedding_length");
        cfg.heads = need_int(arch + ".attention.head_count");
        cfg.kv_heads = need_int(arch + ".attention.head_count_kv");
        cfg.head_dim = f->file.find(arch + ".attention.key_length") ? need_int(arch + ".attention.key_length")
                                                                   : cfg.hidden / cfg.heads;
        cfg.ffn = need_int(arch + ".feed_forward_length");
        cfg.eps = (float)opt_float(arch + ".attention.layer_norm_rms_epsilon", 1e-6);
        cfg.rope_base = (float)opt_float(arch + ".rope.freq_base", 1e6);
        const q4k::GgufTensor* embd = f->file.tensor("token_embd.weight");
        if (!embd || embd->ne.size() < 2) throw q4k::Error(Q4K_EINVAL, "GGUF: no token_embd.weight matrix");
        cfg.vocab = (int)embd->ne[1];
        cfg.capacity = capacity;
        cfg.tp_rank = 0;
        cfg.tp_world = 1;
        cfg.device = 0;
        *c = cfg;
    });
}

Q4K_API int q4k_engine_load_gguf(q4k_engine* e, const q4k_gguf* f) {
    return guarded_cuda([&] {
        if (!e || !f) invalid("engine and file required");
        const auto specs = q4k::model_tensors(e->impl.config());
        // a layer's gate and up rows are worked together, so they must share a type
        for (int L = 0; L < e->impl.config().layers; ++L) {
            const std::string p = "blk." + std::to_string(L) + ".";
            const q4k::GgufTensor* g = f->file.tensor(p + "ffn_gate.weight");
            const q4k::GgufTensor* u = f->file.tensor(p + "ffn_up.weight");
            if (g && u && g->type != u->type)
                throw q4k::Error(Q4K_EINVAL, "GGUF: " + p + "ffn_gate and ffn_up must share a type");
        }
        for (const auto& t : specs) {
            const q4k::GgufTensor* g = f->file.tensor(t.name);
            if (!g) throw q4k::Error(Q4K_EINVAL, "GGUF: missing tensor " + t.name);
            int64_t rows = 1;
            for (size_t d = 1; d < g->ne.size(); ++d) rows *= g->ne[d];
            if (g->bytes == 0) throw q4k::Error(Q4K_EINVAL, "GGUF: tensor " + t.name + " has an unsupported type");
            e->impl.set_tensor(t.name, (int)g->type, g->ne[0], rows, f->file.data(*g));
        }
    });
}

Q4K_API int q4k_tp_shard(const q4k_engine_config* cfg, int i, int rank, int world, int64_t* n0, int64_t* n1,
                         int64_t* b0, int64_t* b1) {
    return guarded([&] {
        if (!cfg || world < 1 || rank < 0 || rank >= world || !n0 || !n1 || !b0 || !b1) invalid("bad shard request");
        const auto specs = q4k::model_tensors(*cfg);
        if (i < 0 || (size_t)i >= specs.size()) throw q4k::Error(Q4K_ERANGE, "tensor index out of range");
        const auto s = q4k::tp_slice(*cfg, specs[i], rank, world);
        *n0 = s.n0;
        *n1 = s.n1;
        *b0 = s.b0;
        *b1 = s.b1;
    });
}

Q4K_API int q4k_nccl_unique_id(void* id128) {
    return guarded([&] {
        if (!id128) invalid("buffer required");
        ncclUniqueId id;
        const auto& api = q4k::nccl();
        const ncclResult_t r = api.GetUniqueId(&id);
        if (r != ncclSuccess) throw q4k::Error(Q4K_ECUDA, std::string("ncclGetUniqueId: ") + api.GetErrorString(r));
        static_assert(sizeof id == 128, "NCCL unique id is 128 bytes");
        std::memcpy(id128, &id, sizeof id);
    });
}

Q4K_API int q4k_engine_create(const q4k_engine_config* cfg, const void* nccl_id, q4k_engine** out) {
    return guarded_cuda([&] {
        if (!cfg || !out) invalid("config and output required");
        *out = nullptr;
        *out = new q4k_engine(*cfg, nccl_id);
    });
}

Q4K_API int q4k_engine_destroy(q4k_engine* e) {
    return guarded_cuda([&] { delete e; });
}

Q4K_API int q4k_engine_load_synthetic(q4k_engine* e, uint64_t seed) {
    return guarded_cuda([&] {
        if (!e) invalid("engine required");
        e->impl.load_synthetic(seed);
    });
}

Q4K_API int q4k_engine_set_tensor(q4k_engine* e, const char* name, int type, int64_t ne0, int64_t ne1,
                                  const void* host_gguf) {
    return guarded_cuda([&] {
        if (!e || !name || !host_gguf) invalid("engine, name and data required");
        e->impl.set_tensor(name, type, ne0, ne1, host_gguf);
    });
}

Q4K_API int q4k_engine_fill_kv_synthetic(q4k_engine* e, uint64_t seed, int n) {
    return guarded_cuda([&] {
        if (!e) invalid("engine required");
        e->impl.fill_kv_synthetic(seed, n);
    });
}

Q4K_API int q4k_engine_read_kv(q4k_engine* e, int layer, uint16_t* k_host, uint16_t* v_host) {
    return guarded_cuda([&] {
        if (!e) invalid("engine required");
        e->impl.read_kv(layer, k_host, v_host);
    });
}

Q4K_API int q4k_engine_write_kv(q4k_engine* e, int layer, const uint16_t* k_host, const uint16_t* v_host) {
    return guarded_cuda([&] {
        if (!e) invalid("engine required");
        e->impl.write_kv(layer, k_host, v_host);
    });
}

Q4K_API int q4k_engine_decode(q4k_engine* e, uint32_t token, int position, uint32_t* next_token, float* logits_host,
                              float* hidden_host) {
    return guarded_cuda([&] {
        if (!e || !next_token) invalid("engine and output required");
        *next_token = e->impl.decode(token, position, logits_host, hidden_host);
    });
}

Q4K_API int q4k_engine_prefill(q4k_engine* e, const uint32_t* tokens, int n, int position, uint32_t* next_token,
                               float* logits_host) {
    return guarded_cuda([&] {
        if (!e || !next_token || !tokens) invalid("engine, tokens and output required");
        *next_token = e->impl.prefill(tokens, n, position, logits_host);
    });
}

Q4K_API int q4k_engine_prefill_seq(q4k_engine* e, int seq, const uint32_t* tokens, int n, int position,
                                   uint32_t* next_token, float* logits_host) {
    return guarded_cuda([&] {
        if (!e || !next_token || !tokens) invalid("engine, tokens and output required");
        *next_token = e->impl.prefill(tokens, n, position, logits_host, seq);
    });
}

Q4K_API int q4k_engine_decode_batch(q4k_engine* e, int n, const int* seqs, const uint32_t* tokens,
                                    const int* positions, uint32_t* next_tokens, float* logits_host) {
    return guarded_cuda([&] {
        if (!e || !seqs || !tokens || !positions || !next_tokens) invalid("engine, inputs and outputs required");
        e->impl.decode_batch(n, seqs, tokens, positions, next_tokens, logits_host);
    });
}

Q4K_API int q4k_engine_generate(q4k_engine* e, uint32_t token, int position, int steps, int advance,
                                uint32_t* tokens_host) {
    return guarded_cuda([&] {
        if (!e) invalid("engine required");
        e->impl.generate(token, position, steps, advance, tokens_host);
    });
}

Q4K_API int q4k_engine_layer(q4k_engine* e, int layer, const float* x_host, int position, float* x_out_host) {
    return guarded_cuda([&] {
        if (!e || !x_host || !x_out_host) invalid("engine and buffers required");
        e->impl.layer_step(layer, x_host, position, x_out_host);
    });
}

Q4K_API int q4k_engine_layer_rows(q4k_engine* e, int layer, int seq, int n, int position, const float* x_host,
                                  float* x_out_host) {
    return guarded_cuda([&] {
        if (!e || !x_host || !x_out_host) invalid("engine and buffers required");
        e->impl.layer_rows(layer, seq, n, position, x_host, x_out_host);
    });
}

Q4K_API int q4k_engine_layer_batch(q4k_engine* e, int layer, int n, const int* seqs, const int* positions,
                                   const float* x_host, float* x_out_host) {
    return guarded_cuda([&] {
        if (!e || !seqs || !positions || !x_host || !x_out_host) invalid("engine, rows and buffers required");
        e->impl.layer_batch(layer, n, seqs, positions, x_host, x_out_host);
    });
}

Q4K_API int q4k_engine_trace(q4k_engine* e, uint32_t token, int position, unsigned long long* records_host,
                             size_t max_records, size_t* count) {
    return guarded_cuda([&] {
        if (!e || !count) invalid("engine and count required");
        *count = e->impl.trace_step(token, position, records_host, max_records);
    });
}

Q4K_API void* q4k_engine_stream(q4k_engine* e) { return e ? static_cast<void*>(e->impl.stream()) : nullptr; }

Q4K_API int q4k_engine_set_limits(q4k_engine* e, uint64_t device_wait_ns, int host_wait_ms) {
    return guarded([&] {
        if (!e) invalid("engine required");
        e->impl.set_limits(device_wait_ns, host_wait_ms);
    });
}

Q4K_API int q4k_engine_abort(q4k_engine* e) {
    return guarded([&] {
        if (!e) invalid("engine required");
        e->impl.abort();
    });
}

Q4K_API int q4k_tp_sum_parts(const void* parts, int world, int64_t count, uint32_t tag, const float* residual,
                             float* out, uint64_t wait_ns, int* err_device, void* stream) {
    return guarded_cuda([&] {
        if (!parts || !out || !err_device) invalid("tp_sum_parts needs parts, out and an error word");
        if (world < 1 || world > 8 || count < 0 || count % 4) invalid("1 <= world <= 8 and count a multiple of 4");
        if (reinterpret_cast<uintptr_t>(parts) % 16 || reinterpret_cast<uintptr_t>(out) % 16 ||
            (residual && reinterpret_cast<uintptr_t>(residual) % 16))
            invalid("tp_sum_parts buffers must be 16-byte aligned");
        if (wait_ns == 0) invalid("wait_ns must be positive");
        cudaStream_t s = as_stream(stream);
        q4k::cuda_check(cudaMemsetAsync(err_device, 0, sizeof(int), s), "memset");
        launched(q4k::tp_sum_parts(static_cast<const unsigned long long*>(parts), world, (size_t)count, tag,
                                   residual, out, wait_ns, err_device, s));
        int err = 0;
        q4k::cuda_check(cudaMemcpyAsync(&err, err_device, sizeof(int), cudaMemcpyDeviceToHost, s), "read err");
        q4k::cuda_check(cudaStreamSynchronize(s), "tp_sum_parts");
        if (err) throw q4k::Error(Q4K_ETIMEOUT, "tp_sum_parts: a partial sum never carried the tag (wait gave up)");
    });
}
