// Element-wise, normalisation, rotary, attention, dequantisation and argmax
// kernels behind the reference's launch signatures (include/Kernels.hpp:54-77
// of the reference), plus the layout/synthetic-data kernels of this library.
#include <cuda_runtime.h>

#include <algorithm>

#include <math_constants.h>

#include "ops.h"
#include "q4k_device.cuh"
#include "dequant_device.cuh"

namespace q4k {
namespace {

constexpr int kThreads = 256;

unsigned blocks_for(size_t n, unsigned per = kThreads) { return (unsigned)((n + per - 1) / per); }

// ---------------------------------------------------------------------------
// RMSNorm (rms_norm.cu:6-24): one CTA per row, fp32 sum of squares,
// y = (x * rsqrt(mean + eps)) * gamma.
// ---------------------------------------------------------------------------
__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ gamma, float* __restrict__ y,
                                size_t width, float eps) {
    __shared__ float partial[kThreads / 32];
    const float* xr = x + blockIdx.x * width;
    float* yr = y + blockIdx.x * width;
    float ss = 0.0f;
    for (size_t i = threadIdx.x; i < width; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total += partial[w];
    const float inv = rsqrtf(total / (float)width + eps);
    for (size_t i = threadIdx.x; i < width; i += blockDim.x) yr[i] = (xr[i] * inv) * gamma[i];
}

// ---------------------------------------------------------------------------
// RoPE (rope.cu:7-24): pair (j, j + d/2) of every head rotated by
// float(pos) * powf(base, -2j/d).
// ---------------------------------------------------------------------------
__global__ void rope_kernel(float* x, size_t pairs, size_t heads, size_t head_dim, size_t position_offset,
                            float base) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= pairs) return;
    const size_t half = head_dim / 2;
    const size_t head = i / half, j = i % half;
    const size_t position = position_offset + head / heads;
    const float angle = (float)position * powf(base, -2.0f * (float)j / (float)head_dim);
    float sn, cs;
    sincosf(angle, &sn, &cs);
    const size_t at = head * head_dim + j;
    const float a = x[at], b = x[at + half];
    x[at] = a * cs - b * sn;
    x[at + half] = a * sn + b * cs;
}

// ---------------------------------------------------------------------------
// Causal grouped-query attention over fp32 K/V (attention.cu:23-91
// semantics). One CTA per (query token, query head); each warp keeps its own
// online-softmax state over a strided subset of the keys, and the warps are
// merged at the end. head_dim <= 256.
// ---------------------------------------------------------------------------
constexpr int kAttnWarps = 4;

__global__ void attention_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                     const float* __restrict__ v, float* __restrict__ out, size_t heads,
                                     size_t kv_heads, size_t head_dim, size_t offset) {
    __shared__ float s_m[kAttnWarps], s_l[kAttnWarps];
    __shared__ float s_o[kAttnWarps][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row = blockIdx.x;
    const size_t token = row / heads, head = row % heads;
    const size_t kvh = head / (heads / kv_heads);
    const size_t keys = offset + token + 1;
    const size_t kv_width = kv_heads * head_dim;
    const float* qr = q + row * head_dim;
    const float scale = rsqrtf((float)head_dim);
    float qv[8], o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const size_t d = lane + 32 * i;
        qv[i] = d < head_dim ? qr[d] : 0.0f;
        o[i] = 0.0f;
    }
    float m = -CUDART_INF_F, l = 0.0f;
    for (size_t p = warp; p < keys; p += kAttnWarps) {
        const float* kr = k + p * kv_width + kvh * head_dim;
        const float* vr = v + p * kv_width + kvh * head_dim;
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const size_t d = lane + 32 * i;
            if (d < head_dim) dot += qv[i] * kr[d];
        }
        const float s = warp_sum(dot) * scale;
        const float m_new = fmaxf(m, s);
        const float rescale = expf(m - m_new);
        const float w = expf(s - m_new);
        l = l * rescale + w;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const size_t d = lane + 32 * i;
            o[i] = o[i] * rescale + (d < head_dim ? w * vr[d] : 0.0f);
        }
        m = m_new;
    }
    if (lane == 0) {
        s_m[warp] = m;
        s_l[warp] = l;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < 256) s_o[warp][d] = o[i];
    }
    __syncthreads();
    float mt = -CUDART_INF_F;
    for (int w = 0; w < kAttnWarps; ++w) mt = fmaxf(mt, s_m[w]);
    float lt = 0.0f, f[kAttnWarps];
    for (int w = 0; w < kAttnWarps; ++w) {
        f[w] = s_l[w] > 0.0f ? expf(s_m[w] - mt) : 0.0f;
        lt += s_l[w] * f[w];
    }
    for (size_t d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float acc = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) acc += s_o[w][d] * f[w];
        out[row * head_dim + d] = acc / lt;
    }
}

__global__ void residual_add_kernel(float* state, const float* branch, size_t count) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) state[i] += branch[i];
}

// The receiving side of the fused tensor-parallel sum: 4 outputs per thread,
// every slot's words read (bounded) until they carry `tag`, then summed in
// rank order and added to the residual, as the product prologue does
// (gemv_device.cuh quantise_rows).
__global__ void tp_sum_parts_kernel(const unsigned long long* parts, int world, size_t n4, unsigned tag,
                                    const float* residual, float* out, unsigned long long wait_ns, int* err) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 sum = sum_tagged4<kMaxRanks>(parts + 4 * i, 4 * n4, world, tag, wait_ns, err, ERR_WAIT_TIMEOUT_PEER);
        float4 x = residual ? reinterpret_cast<const float4*>(residual)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        x.x += sum.x;
        x.y += sum.y;
        x.z += sum.z;
        x.w += sum.w;
        reinterpret_cast<float4*>(out)[i] = x;
    }
}

__global__ void silu_multiply_kernel(const float* gate, const float* up, float* out, size_t count) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) {
        const float g = gate[i];
        out[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}

// ---------------------------------------------------------------------------
// Dequantisation of GGUF-layout rows (embedding.cu:6-59). Products d*sc*q
// are exact in fp32, so the result is bit-identical to the reference.
// ---------------------------------------------------------------------------
__global__ void dequantize_raw_kernel(const uint8_t* packed, float* out, size_t count, size_t width, size_t row_bytes,
                                      int type) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const size_t column = i % width;
    const uint8_t* row = packed + (i / width) * row_bytes;
    const unsigned position = column % 256;
    if (type == Q4K_TYPE_Q4_K) {
        out[i] = q4k_value(row + (column / 256) * 144, position);
    } else {
        const uint8_t* block = row + (column / 256) * 210;
        const float d = half_bits_to_float(block[208] | (block[209] << 8));
        const int scale = reinterpret_cast<const int8_t*>(block + 192)[position / 16];
        out[i] = (d * (float)scale) * (float)q6_code(block, block + 128, position);
    }
}

__global__ void embed_rows_kernel(const uint8_t* table, int type, size_t width, size_t vocab, const uint32_t* tokens,
                                  size_t count, float* out, int* err) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t t = blockIdx.y;
    if (t >= count) return;
    const uint32_t token = tokens[t];
    if (token >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && err) atomicOr(err, ERR_BAD_TOKEN);
        return;
    }
    const size_t row_bytes = q4k_device_row_bytes(type, width);
    const uint8_t* row = table + (size_t)token * row_bytes;
    for (size_t c = (size_t)blockIdx.x * blockDim.x + threadIdx.x; c < width; c += (size_t)gridDim.x * blockDim.x)
        out[t * width + c] = device_layout_value(row, type, width / 256, c);
}

// ---------------------------------------------------------------------------
// Argmax (argmax.cu:25-98): per-CTA best, then the last CTA reduces the CTA
// candidates in index order. Larger value wins; ties go to the lower index;
// NaN never wins; no candidate -> 0xffffffff.
// ---------------------------------------------------------------------------
__global__ void argmax_kernel(const float* __restrict__ logits, size_t count, float* cand_score, uint32_t* cand_index,
                              unsigned* counter, uint32_t* result) {
    __shared__ float s_score[kThreads / 32];
    __shared__ uint32_t s_index[kThreads / 32];
    __shared__ bool s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float bs = -CUDART_INF_F;
    uint32_t bi = 0xffffffffu;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        const float s = logits[i];
        if (candidate_better(s, (uint32_t)i, bs, bi)) {
            bs = s;
            bi = (uint32_t)i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float os = __shfl_xor_sync(0xffffffffu, bs, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (candidate_better(os, oi, bs, bi)) {
            bs = os;
            bi = oi;
        }
    }
    if (lane == 0) {
        s_score[warp] = bs;
        s_index[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (candidate_better(s_score[w], s_index[w], bs, bi)) {
                bs = s_score[w];
                bi = s_index[w];
            }
        cand_score[blockIdx.x] = bs;
        cand_index[blockIdx.x] = bi;
        __threadfence();
        s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (s_last && warp == 0) {
        __threadfence();
        bs = -CUDART_INF_F;
        bi = 0xffffffffu;
        for (unsigned c = lane; c < gridDim.x; c += 32) {
            const float s = __ldcg(cand_score + c);
            const uint32_t ix = __ldcg(cand_index + c);
            if (candidate_better(s, ix, bs, bi)) {
                bs = s;
                bi = ix;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float os = __shfl_xor_sync(0xffffffffu, bs, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (candidate_better(os, oi, bs, bi)) {
                bs = os;
                bi = oi;
            }
        }
        if (lane == 0) {
            *result = bi;
            *counter = 0u;
        }
    }
}

// ---------------------------------------------------------------------------
// Layout and synthetic-data kernels.
// ---------------------------------------------------------------------------
__global__ void synth_q4k_kernel(uint64_t key, uint8_t* out, size_t blocks) {
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b < blocks) q4k_synth_q4k_block(key, b, out + b * Q4K_Q4_BLOCK);
}

__global__ void synth_q6k_kernel(uint64_t key, uint8_t* out, size_t blocks) {
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b < blocks) q4k_synth_q6k_block(key, b, out + b * Q4K_Q6_BLOCK);
}

// Rows [n0, n1) and super-blocks [b0, b1) of a GGUF-layout matrix (nb_full
// blocks per row) into the device layout of a (b1-b0)*256-input matrix.
__global__ void relayout_kernel(const uint8_t* raw, int type, size_t nb_full, size_t n0, size_t n1, size_t b0,
                                size_t b1, uint8_t* out) {
    const size_t nb = b1 - b0;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (n1 - n0) * nb) return;
    const size_t r = i / nb, b = i % nb;
    if (type == Q4K_TYPE_Q4_K) {
        const uint4* src = reinterpret_cast<const uint4*>(raw + ((n0 + r) * nb_full + b0 + b) * Q4K_Q4_BLOCK);
        uint4* dst = reinterpret_cast<uint4*>(out + (r * nb + b) * Q4K_Q4_BLOCK);
        for (int k = 0; k < Q4K_Q4_BLOCK / 16; ++k) dst[k] = src[k];
    } else {
        uint8_t* row = out + r * q4k_q6p_row_bytes(nb);
        q4k_q6_to_planar(raw + ((n0 + r) * nb_full + b0 + b) * Q4K_Q6_BLOCK, row, nb, b);
        if (b == nb - 1)  // zero the d plane's padding so the layout is deterministic
            for (size_t i = nb * 210; i < q4k_q6p_row_bytes(nb); ++i) row[i] = 0;
    }
}

__global__ void synth_gamma_kernel(uint64_t key, float* out, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = q4k_synth_gamma(key, i);
}

__global__ void synth_f32_kernel(uint64_t key, float* out, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = q4k_synth_f32(key, i);
}

__global__ void synth_f16_kernel(uint64_t key, uint16_t* out, size_t n, size_t index_base) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = q4k_synth_f16(key, index_base + i);
}

}  // namespace

cudaError_t rms_norm(const float* x, const float* gamma, float* y, size_t rows, size_t width, float eps,
                     cudaStream_t s) {
    rms_norm_kernel<<<(unsigned)rows, kThreads, 0, s>>>(x, gamma, y, width, eps);
    return cudaGetLastError();
}

cudaError_t rope(float* x, size_t tokens, size_t heads, size_t head_dim, size_t pos, float base, cudaStream_t s) {
    const size_t pairs = tokens * heads * (head_dim / 2);
    rope_kernel<<<blocks_for(pairs), kThreads, 0, s>>>(x, pairs, heads, head_dim, pos, base);
    return cudaGetLastError();
}

cudaError_t attention_f32(const float* q, const float* k, const float* v, float* out, size_t tokens, size_t heads,
                          size_t kv_heads, size_t head_dim, size_t offset, cudaStream_t s) {
    attention_f32_kernel<<<(unsigned)(tokens * heads), kAttnWarps * 32, 0, s>>>(q, k, v, out, heads, kv_heads,
                                                                               head_dim, offset);
    return cudaGetLastError();
}

cudaError_t residual_add(float* state, const float* branch, size_t count, cudaStream_t s) {
    residual_add_kernel<<<blocks_for(count), kThreads, 0, s>>>(state, branch, count);
    return cudaGetLastError();
}

cudaError_t tp_sum_parts(const unsigned long long* parts, int world, size_t count, unsigned tag,
                         const float* residual, float* out, unsigned long long wait_ns, int* err, cudaStream_t s) {
    const size_t n4 = count / 4;
    const unsigned blocks = (unsigned)std::min<size_t>((n4 + kThreads - 1) / kThreads, 4 * 148);
    if (n4 == 0) return cudaSuccess;
    tp_sum_parts_kernel<<<blocks, kThreads, 0, s>>>(parts, world, n4, tag, residual, out, wait_ns, err);
    return cudaGetLastError();
}

cudaError_t silu_multiply(const float* gate, const float* up, float* out, size_t count, cudaStream_t s) {
    silu_multiply_kernel<<<blocks_for(count), kThreads, 0, s>>>(gate, up, out, count);
    return cudaGetLastError();
}

cudaError_t dequantize_raw(const void* packed, float* out, size_t rows, size_t width, size_t row_bytes, int type,
                           cudaStream_t s) {
    const size_t count = rows * width;
    dequantize_raw_kernel<<<blocks_for(count), kThreads, 0, s>>>(static_cast<const uint8_t*>(packed), out, count,
                                                                 width, row_bytes, type);
    return cudaGetLastError();
}

cudaError_t embed_rows(const void* table, int type, size_t width, size_t vocab, const uint32_t* tokens, size_t count,
                       float* out, int* err, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((width + kThreads - 1) / kThreads), (unsigned)count);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, embed_rows_kernel, static_cast<const uint8_t*>(table), type, width, vocab, tokens,
                              count, out, err);
}

size_t argmax_scratch_bytes() { return 1024 * (sizeof(float) + sizeof(uint32_t)) + 256; }

cudaError_t argmax(const float* logits, size_t count, uint32_t* result, void* scratch, cudaStream_t s) {
    const unsigned grid = (unsigned)std::min<size_t>(std::max(1, 2 * sm_count()), std::max<size_t>(1, (count + kThreads - 1) / kThreads));
    uint8_t* base = static_cast<uint8_t*>(scratch);
    unsigned* counter = reinterpret_cast<unsigned*>(base);
    float* score = reinterpret_cast<float*>(base + 256);
    uint32_t* index = reinterpret_cast<uint32_t*>(base + 256 + 1024 * sizeof(float));
    argmax_kernel<<<grid, kThreads, 0, s>>>(logits, count, score, index, counter, result);
    return cudaGetLastError();
}

cudaError_t relayout(const void* raw, int type, size_t K_full, size_t n0, size_t n1, size_t b0, size_t b1,
                     void* out, cudaStream_t s) {
    if (type != Q4K_TYPE_Q4_K && type != Q4K_TYPE_Q6_K) return cudaErrorInvalidValue;
    const size_t n = (n1 - n0) * (b1 - b0);
    if (n == 0) return cudaSuccess;
    relayout_kernel<<<blocks_for(n), kThreads, 0, s>>>(static_cast<const uint8_t*>(raw), type, K_full / 256, n0, n1,
                                                       b0, b1, static_cast<uint8_t*>(out));
    return cudaGetLastError();
}

cudaError_t synth_raw(uint64_t key, int type, size_t K, size_t N, void* out, cudaStream_t s) {
    const size_t blocks = N * (K / 256);
    if (type == Q4K_TYPE_Q4_K) {
        synth_q4k_kernel<<<blocks_for(blocks), kThreads, 0, s>>>(key, static_cast<uint8_t*>(out), blocks);
    } else if (type == Q4K_TYPE_Q6_K) {
        synth_q6k_kernel<<<blocks_for(blocks), kThreads, 0, s>>>(key, static_cast<uint8_t*>(out), blocks);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t synth_gamma(uint64_t key, float* out, size_t n, cudaStream_t s) {
    synth_gamma_kernel<<<blocks_for(n), kThreads, 0, s>>>(key, out, n);
    return cudaGetLastError();
}

cudaError_t synth_f32(uint64_t key, float* out, size_t n, cudaStream_t s) {
    synth_f32_kernel<<<blocks_for(n), kThreads, 0, s>>>(key, out, n);
    return cudaGetLastError();
}

cudaError_t synth_f16(uint64_t key, uint16_t* out, size_t n, size_t index_base, cudaStream_t s) {
    synth_f16_kernel<<<blocks_for(n), kThreads, 0, s>>>(key, out, n, index_base);
    return cudaGetLastError();
}

}  // namespace q4k
