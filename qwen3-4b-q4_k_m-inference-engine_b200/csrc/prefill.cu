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
#include <cuda.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include <cstring>
#include <mutex>

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

// ---------------------------------------------------------------------------
// Tensor-core form of the same attention (G = 4 query heads per KV head):
// one CTA per (16 prompt tokens, KV head). Each of its 4 compute warps owns
// 16 MMA rows = 4 tokens x the group's 4 heads and walks the K/V tiles of
// positions 0 .. its last token's position (64 per tile, loaded by TMA
// through the decode attention's tensor maps): S = Q K^T and O += P V on
// mma.sync m16n8k16 with fp16 K/V (the cache's own values) and Q and P each
// split into fp16 high and low parts (fp32-level accuracy), an online
// softmax per row with the causal limit pos0 + token (attention.cu:45-90).
// ---------------------------------------------------------------------------
constexpr int kTcTokens = 16;
constexpr int kTcWarps = 4;
constexpr int kTcStages = 2;
constexpr int kTcStageBytes = 2 * kTileBytes;  // K + V tiles, 32 KB

struct TcSmem {
    uint4 qf[kTcWarps][8][32][2];  // Q A-fragments per warp, k-step, lane: fp16 high, low parts
    uint64_t full[kTcStages];
    uint64_t empty[kTcStages];
};
constexpr int kTcSmemBytes = kTcStages * kTcStageBytes + (int)sizeof(TcSmem) + 1024;

__device__ __forceinline__ void mma_m16n8k16(float (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float quad_max(float v) {
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

__global__ void __launch_bounds__((kTcWarps + 1) * 32, 2)
    prefill_attention_tc_kernel(const PrefillAttnArgs a, const __grid_constant__ CUtensorMap kmap,
                                const __grid_constant__ CUtensorMap vmap, int tokens) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    TcSmem& sm = *reinterpret_cast<TcSmem*>(smem + kTcStages * kTcStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvh = blockIdx.y, t0 = blockIdx.x * kTcTokens;
    const int t_last = min(t0 + kTcTokens, tokens) - 1;
    const int ntiles = (a.pos0 + t_last) / kAttnTile + 1;  // tiles holding positions 0 .. the CTA's last row
    const int row0 = a.row_base + kvh * a.capacity;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kTcWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kTcWarps) {
        // ---------------- producer: K and V tiles
        if (lane == 0) {
            for (int t = 0; t < ntiles; ++t) {
                const int s = t % kTcStages, use = t / kTcStages;
                if (use > 0 && !mbar_wait_bounded(&sm.empty[s], (use - 1) & 1, a.err, ERR_WAIT_TIMEOUT_EMPTY)) break;
                uint8_t* st = smem + s * kTcStageBytes;
                const int y = row0 + t * kAttnTile;
                mbar_arrive_expect_tx(&sm.full[s], kTcStageBytes);
                tma_load_2d(st, &kmap, 0, y, &sm.full[s]);
                tma_load_2d(st + kBox, &kmap, 64, y, &sm.full[s]);
                tma_load_2d(st + kTileBytes, &vmap, 0, y, &sm.full[s]);
                tma_load_2d(st + kTileBytes + kBox, &vmap, 64, y, &sm.full[s]);
            }
        }
        return;
    }

    // ---------------- compute warps
    const int g = lane >> 2, tq = lane & 3;
    const int tok_lo = t0 + 4 * warp + (g >> 2), tok_hi = tok_lo + 2;  // MMA rows g and g + 8
    const int head = 4 * kvh + (g & 3);
    const bool ok_lo = tok_lo < tokens, ok_hi = tok_hi < tokens;
    {
        const float* qlo = a.q + ((size_t)(ok_lo ? tok_lo : 0) * a.heads + head) * D;
        const float* qhi = a.q + ((size_t)(ok_hi ? tok_hi : 0) * a.heads + head) * D;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int k0 = 16 * s + 2 * tq;
            const float2 x0 = ok_lo ? *reinterpret_cast<const float2*>(qlo + k0) : make_float2(0.f, 0.f);
            const float2 x1 = ok_hi ? *reinterpret_cast<const float2*>(qhi + k0) : make_float2(0.f, 0.f);
            const float2 x2 = ok_lo ? *reinterpret_cast<const float2*>(qlo + k0 + 8) : make_float2(0.f, 0.f);
            const float2 x3 = ok_hi ? *reinterpret_cast<const float2*>(qhi + k0 + 8) : make_float2(0.f, 0.f);
            uint4 hi, lo;
            split2(x0.x, x0.y, hi.x, lo.x);
            split2(x1.x, x1.y, hi.y, lo.y);
            split2(x2.x, x2.y, hi.z, lo.z);
            split2(x3.x, x3.y, hi.w, lo.w);
            sm.qf[warp][s][lane][0] = hi;
            sm.qf[warp][s][lane][1] = lo;
        }
    }
    __syncwarp();
    // causal limits: a row attends to positions 0 .. pos0 + token (none for rows past the prompt)
    const int lim_lo = ok_lo ? a.pos0 + tok_lo : -1, lim_hi = ok_hi ? a.pos0 + tok_hi : -1;
    const int warp_last = min(t0 + 4 * warp + 3, tokens - 1);
    const int warp_tiles = t0 + 4 * warp < tokens ? (a.pos0 + warp_last) / kAttnTile + 1 : 0;
    const float scale = rsqrtf((float)D);  // attention.cu:40
    float m_lo = -CUDART_INF_F, m_hi = -CUDART_INF_F, l_lo = 0.0f, l_hi = 0.0f;
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;

    for (int t = 0; t < ntiles; ++t) {
        const int s = t % kTcStages;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&sm.full[s], (t / kTcStages) & 1, a.err, ERR_WAIT_TIMEOUT_FULL)))
            break;
        if (t < warp_tiles) {
            const uint32_t kbase = smem_addr(smem + s * kTcStageBytes);
            const uint32_t vbase = kbase + kTileBytes;
            // S = Q K^T for 8 column tiles of 8 positions
            float sc[8][4];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float ch[4] = {0.f, 0.f, 0.f, 0.f}, cl[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int s2 = 0; s2 < 8; s2 += 2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kbase + tile_off(8 * j + (lane & 7), 2 * s2 + (lane >> 3)), b0, b1, b2, b3);
                    mma_m16n8k16(ch, sm.qf[warp][s2][lane][0], b0, b1);
                    mma_m16n8k16(cl, sm.qf[warp][s2][lane][1], b0, b1);
                    mma_m16n8k16(ch, sm.qf[warp][s2 + 1][lane][0], b2, b3);
                    mma_m16n8k16(cl, sm.qf[warp][s2 + 1][lane][1], b2, b3);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int pos = t * kAttnTile + 8 * j + 2 * tq + (i & 1);
                    const bool keep = pos <= (i < 2 ? lim_lo : lim_hi);
                    sc[j][i] = keep ? (ch[i] + cl[i]) * scale : -CUDART_INF_F;
                }
            }
            // online softmax of rows g (lo) and g + 8 (hi); selects keep an
            // all-masked row at m = -inf, l = 0 without a NaN
            float mx_lo = -CUDART_INF_F, mx_hi = -CUDART_INF_F;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                mx_lo = fmaxf(mx_lo, fmaxf(sc[j][0], sc[j][1]));
                mx_hi = fmaxf(mx_hi, fmaxf(sc[j][2], sc[j][3]));
            }
            const float mn_lo = fmaxf(m_lo, quad_max(mx_lo)), mn_hi = fmaxf(m_hi, quad_max(mx_hi));
            const bool any_lo = mn_lo != -CUDART_INF_F, any_hi = mn_hi != -CUDART_INF_F;
            const float r_lo = any_lo ? expf(m_lo - mn_lo) : 1.0f, r_hi = any_hi ? expf(m_hi - mn_hi) : 1.0f;
            float ps_lo = 0.0f, ps_hi = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                sc[j][0] = any_lo ? expf(sc[j][0] - mn_lo) : 0.0f;
                sc[j][1] = any_lo ? expf(sc[j][1] - mn_lo) : 0.0f;
                sc[j][2] = any_hi ? expf(sc[j][2] - mn_hi) : 0.0f;
                sc[j][3] = any_hi ? expf(sc[j][3] - mn_hi) : 0.0f;
                ps_lo += sc[j][0] + sc[j][1];
                ps_hi += sc[j][2] + sc[j][3];
            }
            l_lo = l_lo * r_lo + quad_sum(ps_lo);
            l_hi = l_hi * r_hi + quad_sum(ps_hi);
            m_lo = mn_lo;
            m_hi = mn_hi;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                o[j][0] *= r_lo;
                o[j][1] *= r_lo;
                o[j][2] *= r_hi;
                o[j][3] *= r_hi;
            }
            // O += P V, 16 positions per k-step
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                uint4 ph, pl;
                split2(sc[2 * kk][0], sc[2 * kk][1], ph.x, pl.x);
                split2(sc[2 * kk][2], sc[2 * kk][3], ph.y, pl.y);
                split2(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph.z, pl.z);
                split2(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph.w, pl.w);
#pragma unroll
                for (int jn = 0; jn < 16; jn += 2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(vbase + tile_off(16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8, jn + (lane >> 4)), b0, b1,
                              b2, b3);
                    mma_m16n8k16(o[jn], ph, b0, b1);
                    mma_m16n8k16(o[jn], pl, b0, b1);
                    mma_m16n8k16(o[jn + 1], ph, b2, b3);
                    mma_m16n8k16(o[jn + 1], pl, b2, b3);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
    }
    // normalised once at the end (attention.cu:92-95)
    if (ok_lo) {
        float* out = a.out + ((size_t)tok_lo * a.heads + head) * D;
        const float inv = 1.0f / l_lo;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            *reinterpret_cast<float2*>(out + 8 * j + 2 * tq) = make_float2(o[j][0] * inv, o[j][1] * inv);
    }
    if (ok_hi) {
        float* out = a.out + ((size_t)tok_hi * a.heads + head) * D;
        const float inv = 1.0f / l_hi;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            *reinterpret_cast<float2*>(out + 8 * j + 2 * tq) = make_float2(o[j][2] * inv, o[j][3] * inv);
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
    if (a.kmap && a.vmap && a.heads == G * a.kv_heads) {
        static std::once_flag once;
        static cudaError_t attr = cudaSuccess;
        std::call_once(once, [] {
            attr = cudaFuncSetAttribute(prefill_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kTcSmemBytes);
        });
        if (attr != cudaSuccess) return attr;
        CUtensorMap km, vm;
        std::memcpy(&km, a.kmap, sizeof km);
        std::memcpy(&vm, a.vmap, sizeof vm);
        const dim3 grid((tokens + kTcTokens - 1) / kTcTokens, a.kv_heads);
        prefill_attention_tc_kernel<<<grid, (kTcWarps + 1) * 32, kTcSmemBytes, s>>>(a, km, vm, tokens);
        return cudaGetLastError();
    }
    prefill_attention_kernel<<<dim3(tokens, a.heads), 128, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace q4k
