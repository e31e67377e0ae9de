// Q4_K / Q6_K dequantise-fused matrix-vector (and small-batch) product.
//
// Arithmetic follows the reference engine's project<Type> kernel
// (src/cuda/matmul.cu:24-125): the fp32 activation is first quantised to
// int8 with one fp32 scale per 32 values (matmul.cu:8-22), then every
// 32-value group contributes  xs[g] * (d*sc*sum(q*xq) - dmin*m*sum(xq))
// for Q4_K and every 16-value run  xs[g] * (d*sc*sum((q-32)*xq))  for Q6_K,
// with the integer dot products done by dp4a.
//
// B200 structure (HBM-bound; one or two CTAs per SM):
//   * warp W (the last one) is a producer: one lane streams "stages" of R
//     consecutive weight rows (20-35 KB, one cp.async.bulk per matrix) into a
//     ring of S shared-memory buffers, completing on mbarriers. The bulk-copy
//     engine reaches full HBM bandwidth only with copies of >= 16 KB and
//     >= 64 KB in flight per SM, hence the large stages. The producer starts
//     before griddepcontrol.wait, so under programmatic dependent launch a
//     product's weights stream in while the previous kernel drains.
//   * warps 0..W-1 are consumers in T teams of TW warps; team k consumes the
//     stages k, k+T, ... . T divides the ring depth S, so every ring slot
//     is only ever taken by one team and its mbarrier phases are waited on
//     in order (a team waiting on a slot another team has not yet released
//     could match a parity two phases old). Within a team, LPR lanes work on one row (so a
//     team covers R = TW*32/LPR rows per stage); lane f of a row takes the
//     64-value chunks f, f+LPR, ... . Rows are reduced with xor-shuffles in a
//     fixed order, so results are deterministic.
//   * before the rows, the consumers quantise the activation into shared
//     memory (optionally RMSNorm-ing it first, which fuses rms_norm.cu:6-24
//     into the product). Codes are stored in a per-block permuted order so
//     that the 16-byte code loads of the lanes on one row are conflict free.
//   * a lane's 64-value chunk is two whole 32-value groups for Q4_K (the
//     low and high nibbles of 32 bytes) and four 16-value runs for Q6_K, so
//     each scale is decoded once per chunk and no partial crosses lanes
//     before the row reduction.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "q4k_device.cuh"
#include "q4k_internal.h"

namespace q4k {
namespace {

constexpr int kTeamWarps = 4;  // warps per consumer team
constexpr int kAllConsumersBarrier = 8;

struct GemvPlan {
    GemvSegment seg[kMaxSegments];
    int stage_start[kMaxSegments + 1];  // first stage index of each segment
    int nseg;
    int K, nb, M, ldx, ldy;
    const float* x;
    const float* gamma;
    float eps;
    int epilogue;
    int total_stages;
    int rows_per_stage;  // R: output rows per stage
    int lpr;             // lanes per row
    int S;               // ring depth (a multiple of teams)
    int teams;           // consumer teams that take stages (slot i % S always belongs to team i % teams)
    int stage_bytes;
    int row_bytes[kMaxSegments];
    int off_xq4, off_xq6, off_xs, off_xsum16, off_xsum32, off_bufs, off_bars, off_misc;
    ArgmaxTarget argmax;
    int* err;
    unsigned long long* trace;
    int trace_tag;
};

// Segment, first local row and row count of stage i.
__device__ __forceinline__ void stage_rows(const GemvPlan& p, int i, int& seg, int& r0, int& nr) {
    seg = 0;
    while (seg + 1 < p.nseg && i >= p.stage_start[seg + 1]) ++seg;
    r0 = (i - p.stage_start[seg]) * p.rows_per_stage;
    nr = min(p.rows_per_stage, p.seg[seg].rows - r0);
}

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 16-byte unit, within its 256-code block, where the activation codes of
// piece s (codes 16s..16s+15 of the block) are stored for the Q4_K and Q6_K
// lane mappings below. For the pieces that the lanes of one row read at the
// same time, consecutive blocks land on disjoint halves of the 8 bank
// groups, so a row's 16-byte loads are conflict free.
__device__ __forceinline__ int perm_q4(int s, int b) {
    // s = 4j + q: pair-chunk j, piece q of it
    const int j = s >> 2, q = s & 3;
    return 8 * (q >> 1) + 4 * ((q & 1) ^ (b & 1)) + j;
}
__device__ __forceinline__ int perm_q6(int s, int b) {
    // s = 8h + 2g + l: half h, 32-group g of it, 16-run l of the group
    const int h = s >> 3, g = (s >> 1) & 3, l = s & 1;
    return 8 * (g >> 1) + 4 * ((g & 1) ^ (b & 1)) + 2 * h + l;
}

// Q4_K pair-chunk p of a row: block b = p/4, j = p%4 covers the 32 nibble
// bytes at 16 + 32j of the block, i.e. the whole 32-value groups 2j (low
// nibbles) and 2j+1 (high nibbles) (matmul.cu:24-54). A lane's j is fixed
// (LPR is a multiple of 4), so its scale/min bytes come from fixed places.
// The high nibbles are dotted in place (16x) with an unsigned-byte dp4a.
template <int MT, int NR>
__device__ __forceinline__ void q4_pair(const uint8_t* const (&rows)[NR], int p, int j, const uint8_t* xq,
                                        const float* xs, const float* xsumf, int K, int mcount,
                                        float (&acc)[NR][MT]) {
    const int b = p >> 2;
    const int sh = (j & 1) * 16;
    uint32_t lo[NR][8], hi[NR][8];
    float ds0[NR], ds1[NR], dm0[NR], dm1[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const uint8_t* blk = rows[r] + b * 144;
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j);
        const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * j);
        // the 6-bit scales (SC) and mins (MN) of groups 0..3 or 4..7 as bytes
        const uint32_t SC = j < 2 ? (hdr.y & 0x3f3f3f3fu) : ((hdr.w & 0x0f0f0f0fu) | ((hdr.y >> 2) & 0x30303030u));
        const uint32_t MN =
            j < 2 ? (hdr.z & 0x3f3f3f3fu) : (((hdr.w >> 4) & 0x0f0f0f0fu) | ((hdr.z >> 2) & 0x30303030u));
        const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
        ds0[r] = d * (float)((SC >> sh) & 0xffu);
        ds1[r] = d * (float)((SC >> (sh + 8)) & 0xffu);
        dm0[r] = dmin * (float)((MN >> sh) & 0xffu);
        dm1[r] = dmin * (float)((MN >> (sh + 8)) & 0xffu);
        const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            lo[r][k] = w[k] & 0x0f0f0f0fu;
            hi[r][k] = w[k] & 0xf0f0f0f0u;
        }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < mcount) {
            const uint8_t* xb = xq + m * K + b * 256;
            uint4 xv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) xv[q] = *reinterpret_cast<const uint4*>(xb + 16 * perm_q4(4 * j + q, b));
            const float2 s2 = *reinterpret_cast<const float2*>(xs + m * (K / 32) + b * 8 + 2 * j);
            const float2 t2 = *reinterpret_cast<const float2*>(xsumf + m * (K / 32) + b * 8 + 2 * j);
            const uint32_t xl[8] = {xv[0].x, xv[0].y, xv[0].z, xv[0].w, xv[1].x, xv[1].y, xv[1].z, xv[1].w};
            const uint32_t xh[8] = {xv[2].x, xv[2].y, xv[2].z, xv[2].w, xv[3].x, xv[3].y, xv[3].z, xv[3].w};
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                int dl = 0, dh = 0;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    dl = __dp4a((int)lo[r][k], (int)xl[k], dl);
                    dh = dp4a_us(hi[r][k], xh[k], dh);
                }
                dh >>= 4;  // exact: every term is a multiple of 16
                acc[r][m] += s2.x * (ds0[r] * (float)dl - dm0[r] * t2.x);
                acc[r][m] += s2.y * (ds1[r] * (float)dh - dm1[r] * t2.y);
            }
        }
    }
}

// Q6_K quarter p of a planar row: block b = p/4, i = p%4 -> half h = i/2,
// l = i%2 covers positions 16l..16l+15 of every 32-group g = 0..3 of half h,
// i.e. the 16-value runs 8h + 2g + l. The 16 ql bytes at 64h + 16l (groups
// 0, 2) and 64h + 32 + 16l (groups 1, 3) carry the low nibbles, the 16 qh
// bytes at 32h + 16l the top two bits (matmul.cu:56-84, embedding.cu:42-58).
// A lane's i is fixed. xs16 holds 32 * (code sum) of each run, ordered so
// that a quarter's four runs are adjacent.
template <int MT, int NR>
__device__ __forceinline__ void q6_quarter(const uint8_t* const (&rows)[NR], int nb, int p, int i,
                                           const uint8_t* xq, const float* xs, const int* xs16, int K, int mcount,
                                           float (&acc)[NR][MT]) {
    const int b = p >> 2, h = i >> 1, l = i & 1;
    uint32_t q[NR][4][4];  // [row][group g][word]
    float dsc[NR][4];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const uint8_t* row = rows[r];
        const uint4 A = *reinterpret_cast<const uint4*>(row + b * 128 + 64 * h + 16 * l);
        const uint4 B = *reinterpret_cast<const uint4*>(row + b * 128 + 64 * h + 32 + 16 * l);
        const uint4 Q = *reinterpret_cast<const uint4*>(row + nb * 128 + b * 64 + 32 * h + 16 * l);
        const uint2 scw = *reinterpret_cast<const uint2*>(row + nb * 192 + b * 16 + 8 * h);
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + nb * 208 + b * 2));
        // run 8h + 2g + l: scale byte l + 2g of the 8 at 8h
        dsc[r][0] = d * (float)(int8_t)(scw.x >> (8 * l));
        dsc[r][1] = d * (float)(int8_t)(scw.x >> (8 * l + 16));
        dsc[r][2] = d * (float)(int8_t)(scw.y >> (8 * l));
        dsc[r][3] = d * (float)(int8_t)(scw.y >> (8 * l + 16));
        const uint32_t a[4] = {A.x, A.y, A.z, A.w}, bb[4] = {B.x, B.y, B.z, B.w}, qh[4] = {Q.x, Q.y, Q.z, Q.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            q[r][0][w] = (a[w] & 0x0f0f0f0fu) | ((qh[w] << 4) & 0x30303030u);
            q[r][1][w] = (bb[w] & 0x0f0f0f0fu) | ((qh[w] << 2) & 0x30303030u);
            q[r][2][w] = ((a[w] >> 4) & 0x0f0f0f0fu) | (qh[w] & 0x30303030u);
            q[r][3][w] = ((bb[w] >> 4) & 0x0f0f0f0fu) | ((qh[w] >> 2) & 0x30303030u);
        }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < mcount) {
            const uint8_t* xb = xq + m * K + b * 256;
            const float4 s4 = *reinterpret_cast<const float4*>(xs + m * (K / 32) + b * 8 + 4 * h);
            const int4 c4 = *reinterpret_cast<const int4*>(xs16 + m * (K / 16) + b * 16 + 4 * i);
            const float sg[4] = {s4.x, s4.y, s4.z, s4.w};
            const int cg[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const uint4 xv = *reinterpret_cast<const uint4*>(xb + 16 * perm_q6(8 * h + 2 * g + l, b));
#pragma unroll
                for (int r = 0; r < NR; ++r) {
                    // codes are in [0, 63], so signed dp4a is exact; the -32
                    // is applied through the run sums
                    int dd = __dp4a((int)q[r][g][0], (int)xv.x, 0);
                    dd = __dp4a((int)q[r][g][1], (int)xv.y, dd);
                    dd = __dp4a((int)q[r][g][2], (int)xv.z, dd);
                    dd = __dp4a((int)q[r][g][3], (int)xv.w, dd);
                    acc[r][m] += sg[g] * (dsc[r][g] * (float)(dd - cg[g]));
                }
            }
        }
    }
}

__device__ __forceinline__ int8_t q8_code(float v, float amax) {
    // matmul.cu:19: roundf((value / maximum) * 127), IEEE division.
    return amax == 0.0f ? 0 : static_cast<int8_t>(roundf(__fmul_rn(__fdiv_rn(v, amax), 127.0f)));
}

// Quantise MT activation rows into shared memory: codes (in the Q4_K and/or
// Q6_K permuted order), one fp32 scale per 32 values, code sums per 16 and
// per 32 values. Called by all W*32 consumer threads.
__device__ __forceinline__ void quantise_activation(const GemvPlan& p, int m0, int mcount, uint8_t* smem, int tid,
                                                    int lane, int warp, int nthreads) {
    const int K = p.K;
    uint8_t* xq4 = p.off_xq4 >= 0 ? smem + p.off_xq4 : nullptr;
    uint8_t* xq6 = p.off_xq6 >= 0 ? smem + p.off_xq6 : nullptr;
    float* xs = reinterpret_cast<float*>(smem + p.off_xs);
    int* xsum16 = reinterpret_cast<int*>(smem + p.off_xsum16);
    float* xsum32 = reinterpret_cast<float*>(smem + p.off_xsum32);
    float* red = reinterpret_cast<float*>(smem + p.off_misc);
    const int nvec = K / 4;
    constexpr int kHeld = 12;  // float4s of the row a thread keeps in registers (K <= 12 * 4 * nthreads)
    for (int m = 0; m < mcount; ++m) {
        const float4* xr = reinterpret_cast<const float4*>(p.x + (size_t)(m0 + m) * p.ldx);
        // one pass over the row: every load in flight at once, kept for both uses
        float4 held[kHeld];
#pragma unroll
        for (int k = 0; k < kHeld; ++k) {
            const int i = tid + k * nthreads;
            if (i < nvec) held[k] = xr[i];
        }
        float inv = 1.0f;
        if (p.gamma) {
            float ss = 0.0f;
#pragma unroll
            for (int k = 0; k < kHeld; ++k) {
                const int i = tid + k * nthreads;
                if (i < nvec) {
                    const float4 v = held[k];
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            named_barrier(kAllConsumersBarrier, nthreads);
            float total = 0.0f;
            for (int i = 0; i < nthreads / 32; ++i) total += red[i];
            inv = rsqrtf(total / (float)K + p.eps);  // rms_norm.cu:17
            named_barrier(kAllConsumersBarrier, nthreads);
        }
        // element e = 4*i of the row; the 8 lanes i..i+7 hold one 32-group
#pragma unroll
        for (int k = 0; k < kHeld; ++k) {
            const int i = tid + k * nthreads;
            if (i >= nvec) break;
            const int e = 4 * i;
            float4 v = held[k];
            if (p.gamma) {
                const float4 gm = reinterpret_cast<const float4*>(p.gamma)[i];
                v.x = (v.x * inv) * gm.x;  // rms_norm.cu:19: input * inverse_rms * scale
                v.y = (v.y * inv) * gm.y;
                v.z = (v.z * inv) * gm.z;
                v.w = (v.w * inv) * gm.w;
            }
            float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
            const int8_t c0 = q8_code(v.x, amax), c1 = q8_code(v.y, amax);
            const int8_t c2 = q8_code(v.z, amax), c3 = q8_code(v.w, amax);
            const uint32_t word = (uint32_t)(uint8_t)c0 | ((uint32_t)(uint8_t)c1 << 8) |
                                  ((uint32_t)(uint8_t)c2 << 16) | ((uint32_t)(uint8_t)c3 << 24);
            int run = (int)c0 + (int)c1 + (int)c2 + (int)c3;
            run += __shfl_xor_sync(0xffffffffu, run, 1);
            run += __shfl_xor_sync(0xffffffffu, run, 2);
            const int group = run + __shfl_xor_sync(0xffffffffu, run, 4);
            const int b = e >> 8, r16 = (e & 255) >> 4, o = e & 15;
            if (xq4) *reinterpret_cast<uint32_t*>(xq4 + m * K + b * 256 + 16 * perm_q4(r16, b) + o) = word;
            if (xq6) *reinterpret_cast<uint32_t*>(xq6 + m * K + b * 256 + 16 * perm_q6(r16, b) + o) = word;
            // run r16 = 8h + 2g + l is stored at quarter (2h + l), slot g
            if ((lane & 3) == 0)
                xsum16[m * (K / 16) + b * 16 + 4 * (2 * (r16 >> 3) + (r16 & 1)) + ((r16 >> 1) & 3)] = 32 * run;
            if ((lane & 7) == 0) {
                xsum32[m * (K / 32) + (e >> 5)] = (float)group;
                xs[m * (K / 32) + (e >> 5)] = amax / 127.0f;  // matmul.cu:18
            }
        }
    }
    named_barrier(kAllConsumersBarrier, nthreads);
}

template <int MT, int NR>
__global__ void __launch_bounds__(17 * 32, 1) gemv_kernel(const __grid_constant__ GemvPlan p) {
    constexpr bool PAIR = NR == 2;  // gate and up rows worked together (SwiGLU)
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint64_t t_start = p.trace ? global_timer_ns() : 0;
    const int W = (int)(blockDim.x >> 5) - 1;  // consumer warps
    const int T = p.teams;                     // teams taking stages (<= W / kTeamWarps)
    const int S = p.S;
    const int K = p.K;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
    uint64_t* empty = full + S;
    uint8_t* bufs = smem + p.off_bufs;
    int* team_abort = reinterpret_cast<int*>(smem + p.off_misc) + 64;

    const int G = gridDim.x;
    const int s_begin = (int)((long long)p.total_stages * blockIdx.x / G);
    const int s_end = (int)((long long)p.total_stages * (blockIdx.x + 1) / G);
    const int m0 = blockIdx.y * MT;
    const int mcount = min(MT, p.M - m0);

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        for (int k = 0; k < 4; ++k) team_abort[k] = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == W) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();
            for (int i = 0, st = s_begin; st < s_end; ++i, ++st) {
                const int slot = i % S, use = i / S;
                uint64_t* fb = full + slot;
                if (use > 0 && !mbar_wait_bounded(empty + slot, (use - 1) & 1, p.err, ERR_WAIT_TIMEOUT_EMPTY)) break;
                int seg, r0, nr;
                stage_rows(p, st, seg, r0, nr);
                const int rb = p.row_bytes[seg];
                uint8_t* dst = bufs + (size_t)slot * p.stage_bytes;
                if (PAIR) {
                    mbar_arrive_expect_tx(fb, 2 * nr * rb);
                    bulk_g2s_hint(dst, p.seg[0].w + (size_t)r0 * rb, nr * rb, fb, policy);
                    bulk_g2s_hint(dst + p.rows_per_stage * rb, p.seg[1].w + (size_t)r0 * rb, nr * rb, fb, policy);
                } else {
                    mbar_arrive_expect_tx(fb, nr * rb);
                    bulk_g2s_hint(dst, p.seg[seg].w + (size_t)r0 * rb, nr * rb, fb, policy);
                }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();
    const int nthreads = W * 32;
    quantise_activation(p, m0, mcount, smem, tid, lane, warp, nthreads);
    const uint8_t* xq4 = p.off_xq4 >= 0 ? smem + p.off_xq4 : nullptr;
    const uint8_t* xq6 = p.off_xq6 >= 0 ? smem + p.off_xq6 : nullptr;
    const float* xs = reinterpret_cast<const float*>(smem + p.off_xs);
    const int* xsum16 = reinterpret_cast<const int*>(smem + p.off_xsum16);
    const float* xsum32 = reinterpret_cast<const float*>(smem + p.off_xsum32);

    const int team = warp / kTeamWarps;
    const int team_threads = kTeamWarps * 32;
    const int LPR = p.lpr;
    const int sub = lane % LPR;                                        // lane within the row's lanes
    const int slot_row = (warp % kTeamWarps) * (32 / LPR) + lane / LPR;  // row of the stage
    const int chunks = p.nb * 4;  // 64-value pair-chunks (Q4_K) or quarters (Q6_K) per row
    const int iters = (chunks + LPR - 1) / LPR;
    const int lane_part = sub & 3;  // the lane's chunk within a block (LPR is a multiple of 4)
    float best_score = -__int_as_float(0x7f800000);
    uint32_t best_index = 0xffffffffu;

    // Stage i always lands in slot i % S and is taken by team i % T; as T
    // divides S, each slot is only ever waited on by one team, in order, so
    // a parity wait can never see a phase two uses old.
    for (int i = team, st = s_begin + team; team < T && st < s_end; i += T, st += T) {
        const int slot = i % S, use = i / S;
        if (!mbar_wait_bounded(full + slot, use & 1, p.err, ERR_WAIT_TIMEOUT_FULL)) team_abort[team] = 1;
        int seg, r0, nr;
        stage_rows(p, st, seg, r0, nr);
        const int rb = p.row_bytes[seg];
        const uint8_t* buf = bufs + (size_t)slot * p.stage_bytes;
        const int rr = slot_row < nr ? slot_row : 0;  // idle rows alias row 0; dropped below
        const uint8_t* rows[NR];
        rows[0] = buf + rr * rb;
        if (PAIR) rows[NR - 1] = buf + (p.rows_per_stage + rr) * rb;
        float acc[NR][MT];
#pragma unroll
        for (int r = 0; r < NR; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;
        if (p.seg[seg].type == Q4K_TYPE_Q4_K) {
#pragma unroll 2
            for (int k = 0; k < iters; ++k) {
                const int f = sub + LPR * k;
                if (f < chunks) q4_pair<MT, NR>(rows, f, lane_part, xq4, xs, xsum32, K, mcount, acc);
            }
        } else {
#pragma unroll 2
            for (int k = 0; k < iters; ++k) {
                const int f = sub + LPR * k;
                if (f < chunks) q6_quarter<MT, NR>(rows, p.nb, f, lane_part, xq6, xs, xsum16, K, mcount, acc);
            }
        }
        // all of this team's reads of the stage are done: release it
        named_barrier(1 + team, team_threads);
        if (warp % kTeamWarps == 0 && lane == 0) mbar_arrive(empty + slot);
        const bool abort_now = team_abort[team] != 0;
        // reduce each row over its LPR lanes (fixed xor order)
#pragma unroll
        for (int r = 0; r < NR; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m)
                for (int o = LPR >> 1; o > 0; o >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], o);
        if (abort_now) break;
        if (sub == 0 && slot_row < nr) {
            float* y = p.seg[seg].y;
            const int row = r0 + slot_row;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m >= mcount) break;
                float* out = y ? y + (size_t)(m0 + m) * p.ldy + row : nullptr;
                if (p.epilogue == EPI_STORE) {
                    *out = acc[0][m];
                } else if (p.epilogue == EPI_ADD) {
                    *out += acc[0][m];
                } else if (p.epilogue == EPI_SWIGLU) {
                    const float g = acc[0][m], u = acc[NR - 1][m];
                    *out = (g / (1.0f + expf(-g))) * u;  // silu_multiply.cu:9-10
                } else {
                    if (out) *out = acc[0][m];
                    if (candidate_better(acc[0][m], (uint32_t)row, best_score, best_index)) {
                        best_score = acc[0][m];
                        best_index = (uint32_t)row;
                    }
                }
            }
        }
    }

    if (p.epilogue == EPI_ARGMAX) {
        // CTA best, then the last CTA to finish reduces all CTAs in index
        // order (argmax.cu:25-61, :89-97).
        __shared__ float s_score[32];
        __shared__ uint32_t s_index[32];
        __shared__ bool s_last;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float os = __shfl_xor_sync(0xffffffffu, best_score, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_index, o);
            if (candidate_better(os, oi, best_score, best_index)) {
                best_score = os;
                best_index = oi;
            }
        }
        if (lane == 0) {
            s_score[warp] = best_score;
            s_index[warp] = best_index;
        }
        named_barrier(kAllConsumersBarrier, nthreads);
        if (tid == 0) {
            float bs = s_score[0];
            uint32_t bi = s_index[0];
            for (int w = 1; w < W; ++w)
                if (candidate_better(s_score[w], s_index[w], bs, bi)) {
                    bs = s_score[w];
                    bi = s_index[w];
                }
            p.argmax.cand_score[blockIdx.x] = bs;
            p.argmax.cand_index[blockIdx.x] = bi;
            __threadfence();
            const unsigned done = atomicAdd(p.argmax.counter, 1u);
            s_last = done == (unsigned)(G - 1);
        }
        named_barrier(kAllConsumersBarrier, nthreads);
        if (s_last && warp == 0) {
            __threadfence();
            float bs = -__int_as_float(0x7f800000);
            uint32_t bi = 0xffffffffu;
            for (int c = lane; c < G; c += 32) {
                const float s = __ldcg(p.argmax.cand_score + c);
                const uint32_t ix = __ldcg(p.argmax.cand_index + c);
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
                *p.argmax.token = bi == 0xffffffffu ? bi : bi + p.argmax.index_base;
                if (p.argmax.score) *p.argmax.score = bs;
                *p.argmax.counter = 0u;
            }
        }
    }
    if (tid == 0) trace_record(p.trace, p.trace_tag, t_start);
}

template <int MT, int NR>
cudaError_t launch_instance(const GemvPlan& plan, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl) {
    static std::once_flag once;
    static cudaError_t attr_status = cudaSuccess;
    static size_t max_dynamic = 0;
    std::call_once(once, [] {
        // static + dynamic shared memory must fit the 227 KB per-block limit
        cudaFuncAttributes fa{};
        attr_status = cudaFuncGetAttributes(&fa, gemv_kernel<MT, NR>);
        if (attr_status != cudaSuccess) return;
        max_dynamic = 227 * 1024 - fa.sharedSizeBytes;
        attr_status = cudaFuncSetAttribute(gemv_kernel<MT, NR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)max_dynamic);
    });
    if (attr_status != cudaSuccess) return attr_status;
    if (smem > max_dynamic) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_kernel<MT, NR>, plan);
}

int align_up(int v, int a) { return (v + a - 1) / a * a; }

int env_int(const char* name, int fallback) {
    const char* v = std::getenv(name);
    return v && *v ? std::atoi(v) : fallback;
}

}  // namespace

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

cudaError_t launch_gemv(const GemvRequest& rq, cudaStream_t stream) {
    if (rq.nseg < 1 || rq.nseg > kMaxSegments || rq.K <= 0 || rq.K % 256 != 0 || rq.M <= 0 || !rq.x)
        return cudaErrorInvalidValue;
    const bool pair = rq.epilogue == EPI_SWIGLU;
    if (pair && (rq.nseg != 2 || rq.seg[0].rows != rq.seg[1].rows || rq.seg[0].type != rq.seg[1].type))
        return cudaErrorInvalidValue;
    if (rq.epilogue == EPI_ARGMAX &&
        (rq.M != 1 || rq.nseg != 1 || !rq.argmax.cand_score || !rq.argmax.cand_index || !rq.argmax.counter ||
         !rq.argmax.token))
        return cudaErrorInvalidValue;

    GemvPlan p = {};
    p.K = rq.K;
    p.nb = rq.K / 256;
    p.M = rq.M;
    p.ldx = rq.ldx ? rq.ldx : rq.K;
    p.x = rq.x;
    p.gamma = rq.gamma;
    p.eps = rq.eps;
    p.epilogue = rq.epilogue;
    p.argmax = rq.argmax;
    p.err = rq.err;
    p.trace = rq.trace;
    p.trace_tag = rq.trace_tag;
    bool need_q4 = false, need_q6 = false;
    int max_row = 0;
    for (int s = 0; s < rq.nseg; ++s) {
        const GemvSegment& g = rq.seg[s];
        if ((g.type != Q4K_TYPE_Q4_K && g.type != Q4K_TYPE_Q6_K) || g.rows <= 0 || !g.w ||
            reinterpret_cast<uintptr_t>(g.w) % 16 != 0)
            return cudaErrorInvalidValue;
        if (!g.y && rq.epilogue != EPI_ARGMAX) return cudaErrorInvalidValue;
        p.seg[s] = g;
        p.row_bytes[s] = (int)q4k_device_row_bytes(g.type, rq.K);
        max_row = std::max(max_row, p.row_bytes[s]);
        need_q4 |= g.type == Q4K_TYPE_Q4_K;
        need_q6 |= g.type == Q4K_TYPE_Q6_K;
    }
    p.ldy = rq.ldy ? rq.ldy : rq.seg[0].rows;

    // Batch tile: as many activation rows as fit in ~48 KB of shared memory.
    const int per_row_x = (need_q4 ? rq.K : 0) + (need_q6 ? rq.K : 0) + rq.K / 32 * 8 + rq.K / 16 * 4;
    int MT = 1;
    while (MT < rq.M && MT < 8) MT <<= 1;
    while (MT > 1 && MT * per_row_x > 48 * 1024) MT >>= 1;
    if (MT * per_row_x > 160 * 1024) return cudaErrorInvalidValue;

    int off = 0;
    p.off_xq4 = -1;
    p.off_xq6 = -1;
    if (need_q4) {
        p.off_xq4 = off;
        off += MT * rq.K;
    }
    if (need_q6) {
        p.off_xq6 = off;
        off += MT * rq.K;
    }
    p.off_xs = off;
    off += MT * (rq.K / 32) * 4;
    p.off_xsum16 = off;
    off += MT * (rq.K / 16) * 4;
    p.off_xsum32 = off;
    off += MT * (rq.K / 32) * 4;
    p.off_misc = off;
    off += 128 * 4;
    off = align_up(off, 128);

    // Lanes per row: about five 64-value chunks per lane per stage.
    const int chunks = p.nb * 4;
    int lpr = env_int("Q4K_GEMV_LPR", chunks <= 48 ? 8 : chunks <= 80 ? 16 : 32);
    if (lpr != 8 && lpr != 16 && lpr != 32) lpr = 32;
    // consumer warps: teams of four (8 by default); K/4 float4s of the
    // activation row must fit the prologue's registers (12 per thread)
    int W = env_int("Q4K_GEMV_WARPS", 16);
    if (W != 8 && W != 12 && W != 16) W = 16;
    if (rq.K / 4 > 12 * W * 32) return cudaErrorInvalidValue;
    const int R = kTeamWarps * 32 / lpr;
    const int rows_in_stage = pair ? 2 * R : R;
    const int stage_bytes = align_up(rows_in_stage * max_row, 128);
    const int budget = std::max(env_int("Q4K_GEMV_SMEM_KB", 200) * 1024 - off, stage_bytes);
    int S = std::min(budget / stage_bytes, 8);
    if (S < 2) S = 2;
    // every ring slot belongs to one team: teams <= S and S a multiple of it
    const int teams = std::min(W / kTeamWarps, S);
    S -= S % teams;
    if (off + S * stage_bytes + 2 * S * 8 > 220 * 1024) return cudaErrorInvalidValue;
    p.lpr = lpr;
    p.rows_per_stage = R;
    p.stage_bytes = stage_bytes;
    p.S = S;
    p.teams = teams;
    p.off_bufs = off;
    off += S * stage_bytes;
    p.off_bars = off;
    off += 2 * S * 8;
    const size_t smem = (size_t)off;

    // stages of R output rows, never crossing a segment
    int stages = 0;
    const int stage_segs = pair ? 1 : rq.nseg;
    for (int s = 0; s < stage_segs; ++s) {
        p.stage_start[s] = stages;
        stages += (rq.seg[s].rows + R - 1) / R;
    }
    for (int s = stage_segs; s <= kMaxSegments; ++s) p.stage_start[s] = stages;
    p.nseg = stage_segs;
    p.total_stages = stages;

    int ctas = rq.ctas > 0 ? rq.ctas : env_int("Q4K_GEMV_CTAS_PER_SM", 1) * sm_count();
    ctas = std::min(ctas, stages);
    if (rq.epilogue == EPI_ARGMAX) ctas = std::min(ctas, 1024);
    const dim3 grid(ctas, (rq.M + MT - 1) / MT), block((W + 1) * 32);

    const int NR = pair ? 2 : 1;
    switch (MT * 4 + NR) {
        case 1 * 4 + 1: return launch_instance<1, 1>(p, grid, block, smem, stream, rq.pdl);
        case 2 * 4 + 1: return launch_instance<2, 1>(p, grid, block, smem, stream, rq.pdl);
        case 4 * 4 + 1: return launch_instance<4, 1>(p, grid, block, smem, stream, rq.pdl);
        case 8 * 4 + 1: return launch_instance<8, 1>(p, grid, block, smem, stream, rq.pdl);
        case 1 * 4 + 2: return launch_instance<1, 2>(p, grid, block, smem, stream, rq.pdl);
        case 2 * 4 + 2: return launch_instance<2, 2>(p, grid, block, smem, stream, rq.pdl);
        case 4 * 4 + 2: return launch_instance<4, 2>(p, grid, block, smem, stream, rq.pdl);
        case 8 * 4 + 2: return launch_instance<8, 2>(p, grid, block, smem, stream, rq.pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace q4k
