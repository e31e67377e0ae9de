// Prompt prefill (q4k_engine_prefill): the steps between the batched
// products of one layer for M prompt tokens at positions pos0 .. pos0+M-1.
//
//   prefill_qk_kernel: per token and head, the QK RMSNorm (rms_norm.cu:17-19
//     over head_dim 128 with the q/k gammas), RoPE (rope.cu:21-22) and, for
//     the KV heads, the fp16 K and V rows appended to the cache: the same
//     arithmetic as the decode attention's prologue (attention_decode.cu).
//   prefill_attention_kernel: causal GQA attention of every prompt token over
//     the cache positions 0 .. its own (attention.cu:23-110 semantics: scale
//     1/sqrt(d), online softmax with expf, normalised at the end), fp32
//     arithmetic on the fp16 cache. One CTA per (token, query head); its four
//     warps take every fourth position and merge their (m, l, o) at the end.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "attention_device.cuh"
#include "ops.h"
#include "q4k_device.cuh"

namespace q4k {
namespace {

using namespace attn_dev;  // D = 128, rope_angle

__global__ void __launch_bounds__(64) prefill_qk_kernel(PrefillQkArgs a) {
    const int t = blockIdx.x, h = blockIdx.y, j = threadIdx.x, lane = j & 31, warp = j >> 5;
    const int pos = a.pos0 + t;
    const bool is_q = h < a.heads;
    const int kvh = is_q ? 0 : h - a.heads;
    const float* row = a.qkv + (size_t)t * a.ld_qkv + (is_q ? (size_t)h * D : (size_t)a.heads * D + (size_t)kvh * D);
    const float* gamma = is_q ? a.q_gamma : a.k_gamma;
    float x0 = row[j], x1 = row[j + 64];
    __shared__ float red[2];
    const float ss = warp_sum(x0 * x0 + x1 * x1);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    const float inv = rsqrtf((red[0] + red[1]) / (float)D + a.eps);  // rms_norm.cu:17
    x0 = (x0 * inv) * gamma[j];                                     // rms_norm.cu:19
    x1 = (x1 * inv) * gamma[j + 64];
    float sn, cs;
    sincosf(rope_angle(pos, j, a.rope_base), &sn, &cs);
    const float r0 = x0 * cs - x1 * sn, r1 = x0 * sn + x1 * cs;  // rope.cu:21-22
    if (is_q) {
        float* q = a.q_out + (size_t)t * a.heads * D + (size_t)h * D;
        q[j] = r0;
        q[j + 64] = r1;
    } else {
        const size_t at = ((size_t)kvh * a.capacity + pos) * D;
        a.k_cache[at + j] = q4k_f32_to_f16(r0);
        a.k_cache[at + j + 64] = q4k_f32_to_f16(r1);
        const float* v =
            a.qkv + (size_t)t * a.ld_qkv + (size_t)a.heads * D + (size_t)a.kv_heads * D + (size_t)kvh * D;
        a.v_cache[at + j] = q4k_f32_to_f16(v[j]);
        a.v_cache[at + j + 64] = q4k_f32_to_f16(v[j + 64]);
    }
}

__global__ void __launch_bounds__(128) prefill_attention_kernel(PrefillAttnArgs a) {
    const int t = blockIdx.x, h = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int last = a.pos0 + t;                 // causal: positions 0 .. last
    const int kvh = h / (a.heads / a.kv_heads);  // GQA group
    const float scale = rsqrtf((float)D);        // attention.cu:40
    const float4 q = reinterpret_cast<const float4*>(a.q + ((size_t)t * a.heads + h) * D)[lane];
    const uint16_t* kbase = a.k_cache + (size_t)kvh * a.capacity * D + 4 * lane;
    const uint16_t* vbase = a.v_cache + (size_t)kvh * a.capacity * D + 4 * lane;
    float m = -CUDART_INF_F, l = 0.0f, o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
    for (int p = warp; p <= last; p += 4) {
        const uint2 kw = *reinterpret_cast<const uint2*>(kbase + (size_t)p * D);
        const uint2 vw = *reinterpret_cast<const uint2*>(vbase + (size_t)p * D);
        float s = q.x * q4k_f16_to_f32(kw.x & 0xffffu) + q.y * q4k_f16_to_f32(kw.x >> 16) +
                  q.z * q4k_f16_to_f32(kw.y & 0xffffu) + q.w * q4k_f16_to_f32(kw.y >> 16);
        s = warp_sum(s) * scale;
        const float m_new = fmaxf(m, s);
        const float r = expf(m - m_new), e = expf(s - m_new);
        l = l * r + e;
        o0 = o0 * r + e * q4k_f16_to_f32(vw.x & 0xffffu);
        o1 = o1 * r + e * q4k_f16_to_f32(vw.x >> 16);
        o2 = o2 * r + e * q4k_f16_to_f32(vw.y & 0xffffu);
        o3 = o3 * r + e * q4k_f16_to_f32(vw.y >> 16);
        m = m_new;
    }
    __shared__ float wm[4], wl[4];
    __shared__ float4 wo[4][32];
    if (lane == 0) {
        wm[warp] = m;
        wl[warp] = l;
    }
    wo[warp][lane] = make_float4(o0, o1, o2, o3);
    __syncthreads();
    if (warp == 0) {
        float M = wm[0];
        for (int w = 1; w < 4; ++w) M = fmaxf(M, wm[w]);
        float L = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < 4; ++w) {
            if (!(wl[w] > 0.0f)) continue;  // a warp that had no position (last < 3)
            const float f = expf(wm[w] - M);
            L += wl[w] * f;
            const float4 v = wo[w][lane];
            acc.x += v.x * f;
            acc.y += v.y * f;
            acc.z += v.z * f;
            acc.w += v.w * f;
        }
        float4* out = reinterpret_cast<float4*>(a.out + ((size_t)t * a.heads + h) * D);
        out[lane] = make_float4(acc.x / L, acc.y / L, acc.z / L, acc.w / L);
    }
}

}  // namespace

cudaError_t prefill_qk(const PrefillQkArgs& a, int tokens, cudaStream_t s) {
    if (tokens <= 0 || a.heads <= 0 || a.kv_heads <= 0) return cudaErrorInvalidValue;
    prefill_qk_kernel<<<dim3(tokens, a.heads + a.kv_heads), 64, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t prefill_attention(const PrefillAttnArgs& a, int tokens, cudaStream_t s) {
    if (tokens <= 0 || a.heads <= 0 || a.kv_heads <= 0 || a.heads % a.kv_heads) return cudaErrorInvalidValue;
    prefill_attention_kernel<<<dim3(tokens, a.heads), 128, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace q4k
