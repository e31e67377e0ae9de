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
// takes a contiguous range of positions and serves all G = 4 query heads of
// its group, so each K/V row is read from HBM once per group. A producer
// warp streams 64-position K and V tiles into a shared-memory ring with 2-D
// TMA loads (cp.async.bulk.tensor, 128-byte swizzle), starting before
// griddepcontrol.wait. Each of the eight compute warps owns 8 positions of
// every tile and runs its own online softmax with tensor-core MMAs:
//   scores  S[4 x 8] = Q[4 x 128] K^T         (mma.m16n8k16, rows 4..15 zero)
//   output  O[4 x 128] += P[4 x 8] V[8 x 128]  (mma.m16n8k8)
// Q and P are fp32 values split into fp16 hi + lo parts (two MMAs each), and
// K/V are exact fp16, so the products carry ~22 bits like the reference's
// fp32 arithmetic. The warps' (max, sum, O) are merged in shared memory, each
// CTA writes an unnormalised partial, and the last CTA of a KV head to finish
// merges the partials (log-sum-exp) and writes the attended output.
#include <cuda.h>
#include <cuda_runtime.h>

#include <math_constants.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "ops.h"
#include "q4k_device.cuh"
#include "attention_device.cuh"
#include "gemv_device.cuh"

namespace q4k {
namespace {

using namespace attn_dev;
constexpr int T = kAttnTile;  // positions per tile
constexpr int kComputeWarps = 8;
constexpr int kComputeThreads = kComputeWarps * 32;
constexpr int kStageBytes = 2 * kTileBytes;  // K + V
// Ring depth: a multiple of the two consumer groups, so that slot t % kStages
// is only ever consumed by group t % 2 and each group waits on its slots'
// mbarrier phases in order (with a depth the groups do not divide, a group
// running ahead could wait on a slot whose last phase is two uses old, see
// its parity as complete and read the slot early).
constexpr int kStages = 4;
// The merging CTA takes its splits 32 at a time, one per lane.
constexpr int kMergeBatch = 32;  // one split per lane
constexpr int kMaxSplits = 1024;

struct Args {
    const float* qkv;
    const float* q_gamma;
    const float* k_gamma;
    uint16_t* k_cache;  // this layer: [kv_heads][capacity][128]
    uint16_t* v_cache;
    int row_base;       // row of this layer's head 0, position 0 in the tensor maps
    int capacity;
    const int* position;
    int heads, kv_heads;
    float eps, rope_base;
    float* partial_o;
    float* partial_ml;
    unsigned* counters;
    float* out;
    int* err;
    int stages;
    unsigned long long* trace;
    int trace_tag;
    L2Prefetch prefetch[kMaxPrefetch];  // the next kernel's operands, after this CTA's first tiles
    ActImage out_image;                 // optional: the output quantised for the O product
    const int* seq_of;                  // batched decode: sequence of each token (nullptr: z)
    int ld_qkv;                         // floats between the tokens' projections
    long long seq_cache_elems;          // fp16 elements between sequences' caches
};

struct SmemTail {
    uint4 qf[8][32];
    float q[G][D];
    uint16_t k_new[D];
    uint16_t v_new[D];
    float red[kComputeWarps][2];
    uint64_t full[8];
    uint64_t empty[8];
    int last;
    int abort[4];  // [group][parity of the group's tile]: a fast warp's next tile never sets the flag its group is reading
};

__global__ void __launch_bounds__(kComputeThreads + 32, 1)
    decode_attention_kernel(const __grid_constant__ Args a, const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap) {
    // the 128-byte TMA swizzle is keyed to 1024-byte smem address blocks
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int S = a.stages;
    SmemTail& sm = *reinterpret_cast<SmemTail*>(smem + S * kStageBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, kvh = blockIdx.y, splits = gridDim.x;
    // Batched decode: block z serves the z-th token of the step, in sequence
    // seq_of[z] (z without a map): its projections, output, position and
    // split partials are row z of theirs, its cache that sequence's.
    const int z = blockIdx.z;
    const int sq = a.seq_of ? a.seq_of[z] : z;
    const float* qkv = a.qkv + (size_t)z * a.ld_qkv;
    uint16_t* k_cache = a.k_cache + (size_t)sq * a.seq_cache_elems;
    uint16_t* v_cache = a.v_cache + (size_t)sq * a.seq_cache_elems;
    float* partial_o = a.partial_o + (size_t)z * a.heads * splits * D;
    float* partial_ml = a.partial_ml + (size_t)z * a.heads * splits * 2;
    unsigned* counters = a.counters + (size_t)z * a.kv_heads;
    unsigned long long* trace = z == 0 ? a.trace : nullptr;
    if (threadIdx.x == 0) trace_at(trace, a.trace_tag, 0);

    const int pos = a.position[z];
    if (pos < 0 || pos >= a.capacity) {
        if (tid == 0 && split == 0 && kvh == 0 && a.err) atomicOr(a.err, ERR_BAD_POSITION);
        return;
    }
    const int n_keys = pos + 1;
    const int chunk = (n_keys + splits - 1) / splits;
    const int p0 = min(split * chunk, n_keys), p1 = min(p0 + chunk, n_keys);
    const int tiles = (p1 - p0 + T - 1) / T;
    // tensor-map row of (kvh, position 0) in this sequence's cache
    const int row0 = a.row_base + sq * (int)(a.seq_cache_elems / D) + kvh * a.capacity;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        sm.abort[0] = sm.abort[1] = sm.abort[2] = sm.abort[3] = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kComputeWarps) {
        // ---------------- producer: K and V tiles (rows past p1 are masked) ----------------
        if (lane == 0) {
            for (int t = 0; t < tiles; ++t) {
                const int s = t % S, use = t / S;
                if (use > 0 && !mbar_wait_bounded(&sm.empty[s], (use - 1) & 1, a.err, ERR_WAIT_TIMEOUT_EMPTY)) break;
                const int y = row0 + p0 + t * T;
                uint8_t* st = smem + s * kStageBytes;
                mbar_arrive_expect_tx(&sm.full[s], kStageBytes);
                tma_load_2d(st, &kmap, 0, y, &sm.full[s]);
                tma_load_2d(st + kBox, &kmap, 64, y, &sm.full[s]);
                tma_load_2d(st + kTileBytes, &vmap, 0, y, &sm.full[s]);
                tma_load_2d(st + kTileBytes + kBox, &vmap, 64, y, &sm.full[s]);
                if (t == min(S, tiles) - 1)
                    if (z == 0) issue_l2_prefetch(a.prefetch, split + splits * kvh, splits * gridDim.y);
            }
            if (tiles == 0) if (z == 0) issue_l2_prefetch(a.prefetch, split + splits * kvh, splits * gridDim.y);
        }
        return;
    }

    // ---------------- compute warps: q (and the new k/v) of this token ----------------
    const size_t head_base = (size_t)kvh * a.capacity * D;
    const float* q_raw = qkv + (size_t)kvh * G * D;
    const float* k_raw = qkv + (size_t)a.heads * D + (size_t)kvh * D;
    const float* v_raw = qkv + (size_t)a.heads * D + (size_t)a.kv_heads * D + (size_t)kvh * D;
    const bool owner = pos >= p0 && pos < p1;
    {
        // Thread t handles pair (j, j + 64) of head h = t / 64 (4 heads x 64 pairs).
        const int h = tid >> 6, j = tid & 63;
        // weights and the rotation angle do not depend on the previous kernel
        const float gq0 = a.q_gamma[j], gq1 = a.q_gamma[j + 64];
        const float gk0 = a.k_gamma[j], gk1 = a.k_gamma[j + 64];
        float sn, cs;
        sincosf(rope_angle(pos, j, a.rope_base), &sn, &cs);
        pdl_wait();
        float x0 = q_raw[h * D + j], x1 = q_raw[h * D + j + 64];
        float kx0 = 0.0f, kx1 = 0.0f, vx0 = 0.0f, vx1 = 0.0f;
        if (owner && h == 0) {
            kx0 = k_raw[j];
            kx1 = k_raw[j + 64];
            vx0 = v_raw[j];
            vx1 = v_raw[j + 64];
        }
        const float ss = warp_sum(x0 * x0 + x1 * x1);
        const float kss = (owner && h == 0) ? warp_sum(kx0 * kx0 + kx1 * kx1) : 0.0f;
        if (lane == 0) {
            sm.red[warp][0] = ss;
            sm.red[warp][1] = kss;
        }
        named_barrier(1, kComputeThreads);
        const float qsum = sm.red[2 * h][0] + sm.red[2 * h + 1][0];
        const float inv = rsqrtf(qsum / (float)D + a.eps);  // rms_norm.cu:17
        x0 = (x0 * inv) * gq0;
        x1 = (x1 * inv) * gq1;
        sm.q[h][j] = x0 * cs - x1 * sn;  // rope.cu:21-22
        sm.q[h][j + 64] = x0 * sn + x1 * cs;
        if (owner && h == 0) {
            const float kinv = rsqrtf((sm.red[0][1] + sm.red[1][1]) / (float)D + a.eps);
            kx0 = (kx0 * kinv) * gk0;
            kx1 = (kx1 * kinv) * gk1;
            const uint16_t k0 = q4k_f32_to_f16(kx0 * cs - kx1 * sn);
            const uint16_t k1 = q4k_f32_to_f16(kx0 * sn + kx1 * cs);
            const uint16_t v0 = q4k_f32_to_f16(vx0), v1 = q4k_f32_to_f16(vx1);
            sm.k_new[j] = k0;
            sm.k_new[j + 64] = k1;
            sm.v_new[j] = v0;
            sm.v_new[j + 64] = v1;
            const size_t at = head_base + (size_t)pos * D;
            k_cache[at + j] = k0;
            k_cache[at + j + 64] = k1;
            v_cache[at + j] = v0;
            v_cache[at + j + 64] = v1;
        }
        named_barrier(1, kComputeThreads);
    }

    // Q as MMA A-fragments (rows = heads, only rows 0..3 live), shared by all
    // warps: for k-step s, lane (g, t) = (l / 4, l % 4) holds q[g][16s + 2t, +1]
    // (a0) and q[g][16s + 8 + 2t, +1] (a2), each as fp16 hi and lo parts.
    const int g = lane >> 2, tq = lane & 3;
    {
        const int s = tid >> 5, l = tid & 31, gg = l >> 2, tt = l & 3;  // 256 threads: 8 k-steps x 32 lanes
        uint4 f = make_uint4(0u, 0u, 0u, 0u);
        if (gg < G) {
            split2(sm.q[gg][16 * s + 2 * tt], sm.q[gg][16 * s + 2 * tt + 1], f.x, f.y);
            split2(sm.q[gg][16 * s + 8 + 2 * tt], sm.q[gg][16 * s + 8 + 2 * tt + 1], f.z, f.w);
        }
        sm.qf[s][l] = f;
    }
    named_barrier(1, kComputeThreads);
    if (tid == 0) trace_at(trace, a.trace_tag, 1);

    // ---------------- tiles ----------------
    // The eight warps form two groups of four: group k takes tiles k, k + 2,
    // ...; warp wg of a group owns positions [16 wg, 16 wg + 16) of each of
    // its tiles. Per 16 positions a warp runs 16 QK and 16 PV MMAs of shape
    // m16n8k16 whose A rows 0-3 carry the fp16 hi parts of the 4 heads' Q (or
    // P) and rows 8-11 their lo parts, so one MMA yields both products:
    //   scores   S[h][pos] = D[h][pos] + D[h + 8][pos],  B = K^T (16 dims x 8 positions)
    //   output   O[h][dim] += D[h][dim] + D[h + 8][dim], B = V (16 positions x 8 dims)
    const int grp = warp >> 2, wg = warp & 3;
    const float scale = rsqrtf((float)D);  // attention.cu:40
    float m_run = -CUDART_INF_F, l_run = 0.0f;  // per head g (lanes with g < 4)
    float o[16][4];  // dim chunk c: hi rows (O[g][8c + 2tq, +1]) and lo rows (the same dims)
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    const int rA = 16 * wg + (lane & 7);                      // K rows: positions 0-7, then 8-15, of the slab
    const int vr = 16 * wg + (lane & 7) + 8 * ((lane >> 3) & 1);  // V rows for the transposed loads
    const int gbar = 2 + grp;                                 // named barrier of this warp's group

    for (int t = grp; t < tiles; t += 2) {
        const int s = t % S, use = t / S;
        // A warp whose wait gave up flags the CTA; its group still meets at
        // the end-of-tile barrier, after which the group leaves.
        const bool landed = mbar_wait_bounded(&sm.full[s], use & 1, a.err, ERR_WAIT_TIMEOUT_FULL);
        if (tid == 0 && t == 0) trace_at(trace, a.trace_tag, 2);
        if (warp == 0 && lane == 0 && t + 2 >= tiles) trace_at(trace, a.trace_tag, 3);
        const int flag = 2 * grp + ((t >> 1) & 1);
        if (!__all_sync(0xffffffffu, landed) && lane == 0) sm.abort[flag] = 1;
        const int lo = p0 + t * T;
        const int n = min(T, p1 - lo);
        uint8_t* kt = smem + s * kStageBytes;
        uint8_t* vt = kt + kTileBytes;
        // the new token's row: this warp's slab holds it in the owner CTA
        const int prow = pos - lo;
        const bool mine = owner && prow >= 16 * wg && prow < 16 * wg + 16;
        if (mine) {
            if (lane < 16) {
                *reinterpret_cast<uint4*>(kt + tile_off(prow, lane)) = *reinterpret_cast<const uint4*>(sm.k_new + 8 * lane);
                *reinterpret_cast<uint4*>(vt + tile_off(prow, lane)) = *reinterpret_cast<const uint4*>(sm.v_new + 8 * lane);
            }
            __syncwarp();
        }
        // scores of positions 0-7 (sa: even k-steps, sb: odd) and 8-15 (ta, tb) of the slab
        float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        float ta[4] = {0.0f, 0.0f, 0.0f, 0.0f}, tb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const uint32_t kbase = smem_addr(kt);
#pragma unroll
        for (int s2 = 0; s2 < 8; s2 += 2) {
            uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
            ldsm_x4(kbase + tile_off(rA, 2 * s2 + (lane >> 3)), a0, a1, a2, a3);
            ldsm_x4(kbase + tile_off(rA + 8, 2 * s2 + (lane >> 3)), b0, b1, b2, b3);
            const uint4 fa = sm.qf[s2][lane], fb = sm.qf[s2 + 1][lane];
            mma16816_hilo(sa, fa, a0, a1);
            mma16816_hilo(sb, fb, a2, a3);
            mma16816_hilo(ta, fa, b0, b1);
            mma16816_hilo(tb, fb, b2, b3);
        }
        // online softmax over the slab (lane (g, tq): positions 2tq, 2tq+1, 2tq+8, 2tq+9)
        const int c0 = 16 * wg + 2 * tq;
        const float x0 = c0 < n ? ((sa[0] + sb[0]) + (sa[2] + sb[2])) * scale : -CUDART_INF_F;
        const float x1 = c0 + 1 < n ? ((sa[1] + sb[1]) + (sa[3] + sb[3])) * scale : -CUDART_INF_F;
        const float x2 = c0 + 8 < n ? ((ta[0] + tb[0]) + (ta[2] + tb[2])) * scale : -CUDART_INF_F;
        const float x3 = c0 + 9 < n ? ((ta[1] + tb[1]) + (ta[3] + tb[3])) * scale : -CUDART_INF_F;
        float tmax = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        const float m_new = fmaxf(m_run, tmax);
        // branch-free: selects give the values of the empty case (every
        // score so far masked) without a branch around the exponentials
        const bool any = m_new != -CUDART_INF_F;
        const float e0 = expf(x0 - m_new), e1 = expf(x1 - m_new), e2 = expf(x2 - m_new), e3 = expf(x3 - m_new);
        const float er = expf(m_run - m_new);
        const float q0 = any ? e0 : 0.0f, q1 = any ? e1 : 0.0f, q2 = any ? e2 : 0.0f, q3 = any ? e3 : 0.0f;
        const float rescale = any ? er : 1.0f;
        float psum = (q0 + q1) + (q2 + q3);
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        l_run = l_run * rescale + psum;
        m_run = m_new;
        uint32_t ph0, pl0, ph1, pl1;
        split2(q0, q1, ph0, pl0);
        split2(q2, q3, ph1, pl1);
        if (g >= G) ph0 = pl0 = ph1 = pl1 = 0u;
        // O += P V over the slab's 16 positions, 128 dims in 16 chunks of 8
        const uint32_t vbase = smem_addr(vt);
#pragma unroll
        for (int c2 = 0; c2 < 16; c2 += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vbase + tile_off(vr, c2 + (lane >> 4)), b0, b1, b2, b3);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                o[c2][q] *= rescale;
                o[c2 + 1][q] *= rescale;
            }
            mma16816_acc(o[c2], ph0, pl0, ph1, pl1, b0, b1);
            mma16816_acc(o[c2 + 1], ph0, pl0, ph1, pl1, b2, b3);
        }
        if (mine) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes before the next TMA
        __syncwarp();
        // the slot is reused only when the ring wraps; then it is free once
        // the four warps of this group are done with it
        if (t + S < tiles) {
            named_barrier(gbar, kComputeThreads / 2);
            if (wg == 0 && lane == 0) mbar_arrive(&sm.empty[s]);
            if (sm.abort[flag]) break;
        }
    }
    named_barrier(1, kComputeThreads);

    // ---------------- merge the 8 warps (stage buffers reused as scratch) ----------------
    float* wm = reinterpret_cast<float*>(smem);            // [warps][G]
    float* wl = wm + kComputeWarps * G;                    // [warps][G]
    float* wo = wl + kComputeWarps * G;                    // [warps][G][D]
    const bool aborted = (sm.abort[0] | sm.abort[1] | sm.abort[2] | sm.abort[3]) != 0;
    if (!aborted) {
        if (g < G) {
            if (tq == 0) {
                wm[warp * G + g] = m_run;
                wl[warp * G + g] = l_run;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                wo[(warp * G + g) * D + 8 * j + 2 * tq] = o[j][0] + o[j][2];
                wo[(warp * G + g) * D + 8 * j + 2 * tq + 1] = o[j][1] + o[j][3];
            }
        }
    }
    named_barrier(1, kComputeThreads);
    const int hq = tid >> 6;          // query head within the group
    const int d0 = 2 * (tid & 63);    // dims d0, d0+1
    float M = -CUDART_INF_F;
    for (int w = 0; w < kComputeWarps; ++w) M = fmaxf(M, wm[w * G + hq]);
    float L = 0.0f, acc0 = 0.0f, acc1 = 0.0f;
    // branch-free (a select keeps each sum unchanged for an empty warp), so
    // that the exponentials of all warps are in flight at once
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) {
        const float l = wl[w * G + hq];
        const bool live = l > 0.0f;
        const float f = expf(wm[w * G + hq] - M);
        L = live ? L + l * f : L;
        acc0 = live ? acc0 + wo[(w * G + hq) * D + d0] * f : acc0;
        acc1 = live ? acc1 + wo[(w * G + hq) * D + d0 + 1] * f : acc1;
    }
    if (aborted) {
        M = -CUDART_INF_F;
        L = acc0 = acc1 = 0.0f;
    }

    // ---------------- partials and the cross-split merge ----------------
    const size_t pidx = ((size_t)kvh * splits + split) * G + hq;
    partial_o[pidx * D + d0] = acc0;
    partial_o[pidx * D + d0 + 1] = acc1;
    if ((tid & 63) == 0) {
        partial_ml[pidx * 2 + 0] = M;
        partial_ml[pidx * 2 + 1] = L;
    }
    __threadfence();
    named_barrier(1, kComputeThreads);
    if (tid == 0) trace_at(trace, a.trace_tag, 4);
    if (tid == 0) sm.last = atomicAdd(counters + kvh, 1u) == (unsigned)(splits - 1);
    named_barrier(1, kComputeThreads);
    if (!sm.last) {
        if (tid == 0) trace_at(trace, a.trace_tag, 7);
        return;
    }
    __threadfence();
    if (tid == 0) trace_at(trace, a.trace_tag, 3);  // the merging CTA: last arrival seen
    // The merge is on the critical path of the step. Lane u of each warp
    // takes splits u, u + 32, ...: the head's maximum and the splits'
    // weights are found across lanes (one exponential per lane, sums in a
    // fixed shuffle order), and the o partials of 32 splits at a time are
    // loaded in the same round trip as every split's (m, l).
    constexpr int kBatch = kMergeBatch;
    const float2* po = reinterpret_cast<const float2*>(partial_o + ((size_t)kvh * splits * G + hq) * D + d0);
    float2 v[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
        v[u] = u < splits ? __ldcg(po + (size_t)u * (G * D / 2)) : make_float2(0.0f, 0.0f);
    const float* mlh = partial_ml + ((size_t)kvh * splits * G + hq) * 2;  // split sp at mlh + sp * G * 2
    float my_m = -CUDART_INF_F, my_l = 0.0f;  // split `lane`
    float MM = -CUDART_INF_F;
    for (int sp = lane; sp < splits; sp += 32) {
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(mlh + (size_t)sp * G * 2));
        if (sp == lane) {
            my_m = ml.x;
            my_l = ml.y;
        }
        MM = fmaxf(MM, ml.y > 0.0f ? ml.x : -CUDART_INF_F);
    }
    MM = warp_max(MM);
    if (tid == 0) trace_at(trace, a.trace_tag, 5);
    float LL = 0.0f, o0 = 0.0f, o1 = 0.0f;
    for (int sp0 = 0; sp0 < splits; sp0 += kBatch) {
        float m = my_m, l = my_l;
        if (sp0 > 0) {
            m = -CUDART_INF_F;
            l = 0.0f;
            if (sp0 + lane < splits) {
                const float2 ml = __ldcg(reinterpret_cast<const float2*>(mlh + (size_t)(sp0 + lane) * G * 2));
                m = ml.x;
                l = ml.y;
            }
#pragma unroll
            for (int u = 0; u < kBatch; ++u)
                v[u] = sp0 + u < splits ? __ldcg(po + (size_t)(sp0 + u) * (G * D / 2)) : make_float2(0.0f, 0.0f);
        }
        const bool live = sp0 + lane < splits && l > 0.0f;
        const float f = live ? expf(m - MM) : 0.0f;
        LL += warp_sum(live ? l * f : 0.0f);
        // a dead split's weight is 0 and its partial 0: adding nothing
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const float fu = __shfl_sync(0xffffffffu, f, u);
            o0 += v[u].x * fu;
            o1 += v[u].y * fu;
        }
    }
    float* out = a.out + (size_t)z * a.heads * D + ((size_t)kvh * G + hq) * D;
    out[d0] = o0 / LL;
    out[d0 + 1] = o1 / LL;
    if (a.out_image.base) {
        // this KV head's G x 128 outputs are 16 whole 32-value groups of the
        // O product's activation, each held by a half-warp two values per
        // lane: quantise them from registers
        const gemv_dev::ImageParts img = gemv_dev::image_parts(a.out_image.base, a.out_image.K);
        gemv_dev::quantise_pair(o0 / LL, o1 / LL, ((kvh * G + hq) * D) + d0, a.out_image.K, img.q4, img.q6, img.xs,
                                img.xsum16, img.xsum32, lane);
    }
    if (tid == 0) {
        counters[kvh] = 0u;
        trace_at(trace, a.trace_tag, 6);  // slot 6 marks the merging CTA
        trace_at(trace, a.trace_tag, 7);
    }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() { return reinterpret_cast<EncodeTiled>(tensor_map_encoder()); }

size_t smem_bytes(int stages) { return (size_t)stages * kStageBytes + sizeof(SmemTail) + 1024; }

}  // namespace

void* tensor_map_encoder() {
    static void* fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = p;
    });
    return fn;
}

cudaError_t make_kv_tensor_map(const uint16_t* base, long long rows, KvTensorMap* out) {
    static_assert(sizeof(KvTensorMap) == sizeof(CUtensorMap), "tensor map storage size");
    EncodeTiled enc = encoder();
    if (!enc) return cudaErrorNotSupported;
    if (reinterpret_cast<uintptr_t>(base) % 16 || rows <= 0) return cudaErrorInvalidValue;
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)T};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    std::memcpy(out, &map, sizeof map);
    return cudaSuccess;
}

// One CTA per SM and KV head share by default (Q4K_ATTN_CTAS_PER_SM raises
// it; the CTAs then run in waves, one per SM at a time, as the kernel keeps
// all its registers for the tile loop): more splits shorten each CTA's KV
// stream but lengthen the cross-split merge, and one per SM measured faster.
int decode_attention_splits(int kv_heads) {
    const char* env = std::getenv("Q4K_ATTN_CTAS_PER_SM");
    int per_sm = env && *env ? std::atoi(env) : 1;
    per_sm = per_sm < 1 ? 1 : per_sm > 64 ? 64 : per_sm;
    const int s = per_sm * sm_count() / (kv_heads > 0 ? kv_heads : 1);
    return s < 1 ? 1 : s > kMaxSplits ? kMaxSplits : s;
}

size_t decode_attention_scratch_floats(int heads, int kv_heads, int splits) {
    (void)kv_heads;
    return (size_t)heads * splits * (D + 2);
}

cudaError_t decode_attention(const DecodeAttnArgs& in, const KvTensorMap& kmap, const KvTensorMap& vmap,
                             cudaStream_t s, bool pdl) {
    if (in.kv_heads <= 0 || in.heads != in.kv_heads * G || in.splits <= 0 || in.splits > kMaxSplits ||
        in.capacity <= 0)
        return cudaErrorInvalidValue;
    Args a;
    a.qkv = in.qkv;
    a.q_gamma = in.q_gamma;
    a.k_gamma = in.k_gamma;
    a.k_cache = in.k_cache;
    a.v_cache = in.v_cache;
    a.row_base = in.row_base;
    a.capacity = in.capacity;
    a.position = in.position;
    a.heads = in.heads;
    a.kv_heads = in.kv_heads;
    a.eps = in.eps;
    a.rope_base = in.rope_base;
    a.partial_o = in.partial_o;
    a.partial_ml = in.partial_ml;
    a.counters = in.counters;
    a.out = in.out;
    a.err = in.err;
    a.trace = in.trace;
    a.trace_tag = in.trace_tag;
    for (int e = 0; e < kMaxPrefetch; ++e) a.prefetch[e] = in.prefetch[e];
    a.out_image = in.out_image;
    if (a.out_image.base && (a.out_image.K != in.heads * D || a.out_image.K % 256 != 0)) return cudaErrorInvalidValue;
    a.seq_of = in.seq_of;
    a.ld_qkv = in.ld_qkv;
    a.seq_cache_elems = in.seq_cache_elems;
    if (in.batch < 1 || (in.batch > 1 && (a.out_image.base || in.ld_qkv <= 0))) return cudaErrorInvalidValue;
    a.stages = kStages;
    const size_t smem = smem_bytes(a.stages);
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(decode_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem_bytes(kStages));
    });
    if (attr != cudaSuccess) return attr;
    CUtensorMap km, vm;
    std::memcpy(&km, &kmap, sizeof km);
    std::memcpy(&vm, &vmap, sizeof vm);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(in.splits, in.kv_heads, in.batch);
    cfg.blockDim = dim3(kComputeThreads + 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, decode_attention_kernel, a, km, vm);
}

}  // namespace q4k
