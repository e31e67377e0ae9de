// Split-K flash-decode GQA attention for one new token over an fp16 KV cache.
//
// Semantics follow the reference's decode path for a single token
// (src/Engine.cpp:87-92 and src/cuda/attention.cu:23-91): the new token's q
// and k are RMS-normalised per head (rms_norm.cu:6-24), rotated by RoPE at
// the token's position (rope.cu:7-24), the new k and v rows are stored in
// the cache, and every query head attends causally over positions
// [0, pos] with scale 1/sqrt(d) and a softmax.
//
// B200 structure: grid (splits, kv_heads). The CTA for (split, kv head)
// takes a contiguous range of positions and serves all G = heads/kv_heads
// query heads of its group, so each K/V row is read from HBM once per
// group (the reference re-reads it per query head). A producer warp streams
// 64-position K and V tiles (16 KB each, contiguous in the head-major cache
// layout) into a two-stage shared-memory ring with cp.async.bulk, starting
// before griddepcontrol.wait. Eight compute warps do the scores, an online
// softmax and the weighted V sum in fp32. Each CTA writes an unnormalised
// partial (o, max, sum); the last CTA of a KV head to finish merges the
// partials (log-sum-exp) and writes the attended output.
#include <cuda_runtime.h>

#include <math_constants.h>

#include "ops.h"
#include "q4k_device.cuh"

namespace q4k {
namespace {

constexpr int D = kDecodeHeadDim;  // 128
constexpr int G = 4;               // query heads per KV head
constexpr int T = 64;              // positions per tile
constexpr int kStages = 2;
constexpr int kComputeWarps = 8;
constexpr int kComputeThreads = kComputeWarps * 32;

struct Smem {
    uint16_t k[kStages][T * D];
    uint16_t v[kStages][T * D];
    float q[G][D];
    float w[G][T];
    uint16_t k_new[D];
    uint16_t v_new[D];
    float red[kComputeWarps][2];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    int last;
    int abort;
};

__device__ __forceinline__ float rope_angle(int pos, int j, float base) {
    // rope.cu:19-20
    return (float)pos * powf(base, -2.0f * (float)j / (float)D);
}

__global__ void __launch_bounds__(kComputeThreads + 32, 1) decode_attention_kernel(const __grid_constant__ DecodeAttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, splits = gridDim.x;

    const int pos = *a.position;
    if (pos < 0 || pos >= a.capacity) {
        if (tid == 0 && split == 0 && kvh == 0 && a.err) atomicOr(a.err, ERR_BAD_POSITION);
        return;
    }
    const int n_keys = pos + 1;
    const int chunk = (n_keys + splits - 1) / splits;
    const int p0 = min(split * chunk, n_keys), p1 = min(p0 + chunk, n_keys);
    const int tiles = (p1 - p0 + T - 1) / T;
    const size_t head_base = (size_t)kvh * a.capacity * D;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kComputeWarps) {
        // ---------------- producer: cached rows [p0, min(p1, pos)) ----------------
        if (lane == 0) {
            for (int t = 0; t < tiles; ++t) {
                const int s = t % kStages, use = t / kStages;
                if (use > 0 && !mbar_wait_bounded(&sm.empty[s], (use - 1) & 1, a.err, ERR_WAIT_TIMEOUT_EMPTY)) break;
                const int lo = p0 + t * T;
                const int hi = min(min(lo + T, p1), pos);
                const int rows = max(hi - lo, 0);
                mbar_arrive_expect_tx(&sm.full[s], (uint32_t)(2 * rows * D * 2));
                if (rows > 0) {
                    bulk_g2s(sm.k[s], a.k_cache + head_base + (size_t)lo * D, (uint32_t)(rows * D * 2), &sm.full[s]);
                    bulk_g2s(sm.v[s], a.v_cache + head_base + (size_t)lo * D, (uint32_t)(rows * D * 2), &sm.full[s]);
                }
            }
        }
        return;
    }

    // ---------------- compute warps: q (and the new k/v) of this token ----------------
    pdl_wait();
    const float* q_raw = a.qkv + (size_t)kvh * G * D;
    const float* k_raw = a.qkv + (size_t)a.heads * D + (size_t)kvh * D;
    const float* v_raw = a.qkv + (size_t)a.heads * D + (size_t)a.kv_heads * D + (size_t)kvh * D;
    const bool owner = pos >= p0 && pos < p1;
    {
        // Thread t handles pair (j, j + 64) of head h = t / 64 (4 heads x 64 pairs).
        const int h = tid >> 6, j = tid & 63;
        float x0 = q_raw[h * D + j], x1 = q_raw[h * D + j + 64];
        float ss = warp_sum(x0 * x0 + x1 * x1);
        float kx0 = 0.0f, kx1 = 0.0f, kss = 0.0f;
        if (owner && h == 0) {
            kx0 = k_raw[j];
            kx1 = k_raw[j + 64];
            kss = warp_sum(kx0 * kx0 + kx1 * kx1);
        }
        if (lane == 0) {
            sm.red[warp][0] = ss;
            sm.red[warp][1] = kss;
        }
        named_barrier(1, kComputeThreads);
        const float qsum = sm.red[2 * h][0] + sm.red[2 * h + 1][0];
        const float inv = rsqrtf(qsum / (float)D + a.eps);  // rms_norm.cu:17
        x0 = (x0 * inv) * a.q_gamma[j];
        x1 = (x1 * inv) * a.q_gamma[j + 64];
        float sn, cs;
        sincosf(rope_angle(pos, j, a.rope_base), &sn, &cs);
        sm.q[h][j] = x0 * cs - x1 * sn;  // rope.cu:21-22
        sm.q[h][j + 64] = x0 * sn + x1 * cs;
        if (owner && h == 0) {
            const float kinv = rsqrtf((sm.red[0][1] + sm.red[1][1]) / (float)D + a.eps);
            kx0 = (kx0 * kinv) * a.k_gamma[j];
            kx1 = (kx1 * kinv) * a.k_gamma[j + 64];
            const uint16_t k0 = q4k_f32_to_f16(kx0 * cs - kx1 * sn);
            const uint16_t k1 = q4k_f32_to_f16(kx0 * sn + kx1 * cs);
            const uint16_t v0 = q4k_f32_to_f16(v_raw[j]), v1 = q4k_f32_to_f16(v_raw[j + 64]);
            sm.k_new[j] = k0;
            sm.k_new[j + 64] = k1;
            sm.v_new[j] = v0;
            sm.v_new[j + 64] = v1;
            const size_t at = head_base + (size_t)pos * D;
            a.k_cache[at + j] = k0;
            a.k_cache[at + j + 64] = k1;
            a.v_cache[at + j] = v0;
            a.v_cache[at + j + 64] = v1;
        }
        named_barrier(1, kComputeThreads);
    }

    // ---------------- tiles ----------------
    const float scale = rsqrtf((float)D);  // attention.cu:40
    const int h = tid >> 6;                // head of this thread (score and PV phases)
    const int pp = tid & 63;               // position slot in the tile (score phase)
    const int d0 = 2 * (tid & 63);         // dims d0, d0+1 (PV phase)
    float m_run = -CUDART_INF_F, l_run = 0.0f, o0 = 0.0f, o1 = 0.0f;
    if (tid == 0) sm.abort = 0;
    named_barrier(1, kComputeThreads);
    for (int t = 0; t < tiles; ++t) {
        const int s = t % kStages, use = t / kStages;
        // A thread that gives up flags the CTA; all compute threads leave
        // together after the next barrier, so none is left waiting at it.
        const bool landed = mbar_wait_bounded(&sm.full[s], use & 1, a.err, ERR_WAIT_TIMEOUT_FULL);
        if (!landed) sm.abort = 1;
        const int lo = p0 + t * T;
        const int n = min(T, p1 - lo);
        // scores
        float score = -CUDART_INF_F;
        if (landed && pp < n) {
            const uint16_t* krow = (lo + pp == pos) ? sm.k_new : sm.k[s] + pp * D;
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int c = (i + pp) & 15;
                const uint4 kv = *reinterpret_cast<const uint4*>(krow + c * 8);
                const float4 qa = *reinterpret_cast<const float4*>(&sm.q[h][c * 8]);
                const float4 qb = *reinterpret_cast<const float4*>(&sm.q[h][c * 8 + 4]);
                const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kv.x));
                const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kv.y));
                const float2 k45 = __half22float2(*reinterpret_cast<const __half2*>(&kv.z));
                const float2 k67 = __half22float2(*reinterpret_cast<const __half2*>(&kv.w));
                dot += qa.x * k01.x + qa.y * k01.y + qa.z * k23.x + qa.w * k23.y;
                dot += qb.x * k45.x + qb.y * k45.y + qb.z * k67.x + qb.w * k67.y;
            }
            score = dot * scale;
        }
        // online softmax over this tile, per head (64 threads = warps 2h, 2h+1)
        float tmax = warp_max(score);
        if (lane == 0) sm.red[warp][0] = tmax;
        named_barrier(1, kComputeThreads);
        if (sm.abort) break;
        tmax = fmaxf(sm.red[2 * h][0], sm.red[2 * h + 1][0]);
        const float m_new = fmaxf(m_run, tmax);
        const float wgt = pp < n ? expf(score - m_new) : 0.0f;
        sm.w[h][pp] = wgt;
        float tsum = warp_sum(wgt);
        if (lane == 0) sm.red[warp][1] = tsum;
        named_barrier(1, kComputeThreads);
        tsum = sm.red[2 * h][1] + sm.red[2 * h + 1][1];
        const float rescale = expf(m_run - m_new);
        l_run = l_run * rescale + tsum;
        m_run = m_new;
        // weighted V
        o0 *= rescale;
        o1 *= rescale;
        for (int r = 0; r < n; ++r) {
            const uint16_t* vrow = (lo + r == pos) ? sm.v_new : sm.v[s] + r * D;
            const float2 vv = __half22float2(*reinterpret_cast<const __half2*>(vrow + d0));
            const float wr = sm.w[h][r];
            o0 += wr * vv.x;
            o1 += wr * vv.y;
        }
        named_barrier(1, kComputeThreads);
        if (tid == 0) mbar_arrive(&sm.empty[s]);
    }

    // ---------------- partials and the cross-split merge ----------------
    const int hq = h;  // query head within the group
    const size_t pidx = ((size_t)kvh * splits + split) * G + hq;
    a.partial_o[pidx * D + d0] = o0;
    a.partial_o[pidx * D + d0 + 1] = o1;
    if ((tid & 63) == 0) {
        a.partial_ml[pidx * 2 + 0] = m_run;
        a.partial_ml[pidx * 2 + 1] = l_run;
    }
    __threadfence();
    named_barrier(1, kComputeThreads);
    if (tid == 0) sm.last = atomicAdd(a.counters + kvh, 1u) == (unsigned)(splits - 1);
    named_barrier(1, kComputeThreads);
    if (!sm.last) return;
    __threadfence();
    float M = -CUDART_INF_F;
    for (int sp = 0; sp < splits; ++sp) {
        const size_t q = ((size_t)kvh * splits + sp) * G + hq;
        if (__ldcg(a.partial_ml + q * 2 + 1) > 0.0f) M = fmaxf(M, __ldcg(a.partial_ml + q * 2));
    }
    float L = 0.0f, acc0 = 0.0f, acc1 = 0.0f;
    for (int sp = 0; sp < splits; ++sp) {
        const size_t q = ((size_t)kvh * splits + sp) * G + hq;
        const float l = __ldcg(a.partial_ml + q * 2 + 1);
        if (!(l > 0.0f)) continue;
        const float f = expf(__ldcg(a.partial_ml + q * 2) - M);
        L += l * f;
        acc0 += __ldcg(a.partial_o + q * D + d0) * f;
        acc1 += __ldcg(a.partial_o + q * D + d0 + 1) * f;
    }
    float* out = a.out + ((size_t)kvh * G + hq) * D;
    out[d0] = acc0 / L;
    out[d0 + 1] = acc1 / L;
    if (tid == 0) a.counters[kvh] = 0u;
}

}  // namespace

int decode_attention_splits(int kv_heads) {
    const int s = sm_count() / (kv_heads > 0 ? kv_heads : 1);
    return s < 1 ? 1 : s;
}

size_t decode_attention_scratch_floats(int heads, int kv_heads, int splits) {
    (void)kv_heads;
    return (size_t)heads * splits * (D + 2);
}

cudaError_t decode_attention(const DecodeAttnArgs& a, cudaStream_t s, bool pdl) {
    if (a.kv_heads <= 0 || a.heads != a.kv_heads * G || a.splits <= 0 || a.capacity <= 0) return cudaErrorInvalidValue;
    static bool attr_done = false;
    if (!attr_done) {
        const cudaError_t e = cudaFuncSetAttribute(decode_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)sizeof(Smem));
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, a.kv_heads);
    cfg.blockDim = dim3(kComputeThreads + 32);
    cfg.dynamicSmemBytes = sizeof(Smem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, decode_attention_kernel, a);
}

}  // namespace q4k
