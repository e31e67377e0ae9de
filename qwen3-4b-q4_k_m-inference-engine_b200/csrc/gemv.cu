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
#include <type_traits>

#include "q4k_device.cuh"
#include "q4k_internal.h"
#include "gemv_device.cuh"

namespace q4k {
namespace {

using namespace gemv_dev;

constexpr int kTeamWarps = 4;  // warps per consumer team
constexpr int kHeldVec4 = 6;   // activation float4s a consumer thread holds while quantising
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
    int off_xq4, off_xq6, off_xs, off_xsum16, off_xsum32, off_bufs, off_bars, off_misc, off_mred;
    int off_gamma;  // RMSNorm gamma staged in shared memory (-1: no norm)
    int mma;  // Q4_K stages run on the tensor cores (M == 1, 16 rows or 8 + 8 SwiGLU rows per stage)
    ArgmaxTarget argmax;
    int* err;
    unsigned long long* trace;
    int trace_tag;
    L2Prefetch prefetch[kMaxPrefetch];  // the next kernel's operands, after this CTA's first S stages
    ActImage in_image;   // copy this quantised activation instead of quantising x (M == 1)
    ActImage out_image;  // SwiGLU: quantise this CTA's output rows into it (M == 1)
    int inflight;        // stages the producer keeps in flight (issued, not landed); 0: the whole ring
    int prefetch_landed; // issue the L2 prefetch once the first ring of stages has landed
    int gamma_bulk;      // the RMSNorm weight comes in by one bulk copy, ahead of the ring
    int off_resid;       // >= 0 (EPI_ADD, one segment, image input): this CTA's residual rows, fetched
                         // with the image so that the epilogue adds from shared memory
    int group_stages;    // stages per 32-row group: CTA shares start on group boundaries (out_image)
    int off_ostage;      // this CTA's output rows (out_image)
    PeerOut peer_out;    // EPI_PEER
    PeerIn peer_in;      // sum the ranks' partial sums into x first
};

// Segment, first local row and row count of stage i.
__device__ __forceinline__ void stage_rows(const GemvPlan& p, int i, int& seg, int& r0, int& nr) {
    seg = 0;
    while (seg + 1 < p.nseg && i >= p.stage_start[seg + 1]) ++seg;
    r0 = (i - p.stage_start[seg]) * p.rows_per_stage;
    nr = min(p.rows_per_stage, p.seg[seg].rows - r0);
}

template <int HELD>
__device__ __forceinline__ void quantise_activation(const GemvPlan& p, int m0, int mcount, uint8_t* smem, int tid,
                                                    int lane, int warp, int nthreads) {
    const float* gamma = p.gamma ? reinterpret_cast<const float*>(smem + p.off_gamma) : nullptr;
    const PeerIn& pin = p.peer_in;
    // tensor parallelism: every rank's partial sums of this step, read until
    // each word carries this step's tag
    const unsigned tag = pin.world > 0 ? (unsigned)(*pin.epoch + 1) : 0u;
    quantise_rows<HELD>(p.x, p.ldx, m0, mcount, gamma, p.eps, p.K, p.off_xq4 >= 0 ? smem + p.off_xq4 : nullptr,
                  p.off_xq6 >= 0 ? smem + p.off_xq6 : nullptr, reinterpret_cast<float*>(smem + p.off_xs),
                  reinterpret_cast<int*>(smem + p.off_xsum16), reinterpret_cast<float*>(smem + p.off_xsum32),
                  reinterpret_cast<float*>(smem + p.off_misc), tid, lane, warp, nthreads, kAllConsumersBarrier,
                  p.trace, p.trace_tag, pin.world > 0 ? pin.parts : nullptr, pin.world, tag, p.err, pin.wait_ns,
                  ERR_WAIT_TIMEOUT_PEER, pin.world >= 0 && blockIdx.x == 0 ? pin.x_out : nullptr);
}

// Batch of one whose activation the preceding kernel already quantised:
// copy the image's parts this product uses into shared memory, all loads
// of a thread in flight at once (16-byte units; at most 4 per thread).
__device__ __forceinline__ void copy_image(const GemvPlan& p, uint8_t* smem, int tid, int nthreads, int resid_row0,
                                           int resid_rows) {
    const int K = p.K;
    const ImageParts src = image_parts(p.in_image.base, K);
    const int n4 = p.off_xq4 >= 0 ? K / 16 : 0, n6 = p.off_xq6 >= 0 ? K / 16 : 0;
    const int ns = K / 128, n16 = K / 64;
    const int total = n4 + n6 + ns + n16 + ns;
    auto unit = [&](int u, const uint4*& from, uint4*& to) {
        if (u < n4) {
            from = reinterpret_cast<const uint4*>(src.q4) + u;
            to = reinterpret_cast<uint4*>(smem + p.off_xq4) + u;
            return;
        }
        u -= n4;
        if (u < n6) {
            from = reinterpret_cast<const uint4*>(src.q6) + u;
            to = reinterpret_cast<uint4*>(smem + p.off_xq6) + u;
            return;
        }
        u -= n6;
        if (u < ns) {
            from = reinterpret_cast<const uint4*>(src.xs) + u;
            to = reinterpret_cast<uint4*>(smem + p.off_xs) + u;
            return;
        }
        u -= ns;
        if (u < n16) {
            from = reinterpret_cast<const uint4*>(src.xsum16) + u;
            to = reinterpret_cast<uint4*>(smem + p.off_xsum16) + u;
            return;
        }
        u -= n16;
        from = reinterpret_cast<const uint4*>(src.xsum32) + u;
        to = reinterpret_cast<uint4*>(smem + p.off_xsum32) + u;
    };
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int u = tid + k * nthreads;
        if (u < total) {
            const uint4* from;
            uint4* to;
            unit(u, from, to);
            v[k] = __ldcg(from);  // written by the preceding kernel
        }
    }
    // the residual rows this CTA adds to, in the same round trip
    float rv = 0.0f;
    const bool resid = p.off_resid >= 0 && tid < resid_rows;
    if (resid) rv = __ldcg(p.seg[0].y + resid_row0 + tid);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int u = tid + k * nthreads;
        if (u < total) {
            const uint4* from;
            uint4* to;
            unit(u, from, to);
            *to = v[k];
        }
    }
    if (resid) reinterpret_cast<float*>(smem + p.off_resid)[tid] = rv;
    named_barrier(kAllConsumersBarrier, nthreads);
}

// SwiGLU with an output image: this CTA's rows [lo, hi) of the output are
// whole 32-value groups (its stages start on a group boundary), and their
// values were also kept in shared memory (off_ostage) by the epilogue.
// Each warp quantises 4 groups per pass, 8 lanes each; lanes past the last
// group only take part in their warp's shuffles. Called by all consumer
// threads after a barrier that follows the last output row.
__device__ __forceinline__ void quantise_output_groups(const GemvPlan& p, int lo, int hi, const uint8_t* smem, int lane,
                                                       int warp, int nthreads) {
    const ActImage& im = p.out_image;
    const ImageParts img = image_parts(im.base, im.K);
    const float* ostage = reinterpret_cast<const float*>(smem + p.off_ostage);
    const int ng = (hi - lo) / 32;
    for (int j0 = 0; j0 < ng; j0 += 4 * (nthreads / 32)) {
        const int j = j0 + warp * 4 + lane / 8;
        const bool valid = j < ng;
        const int local = 32 * (valid ? j : 0) + 4 * (lane & 7);
        const float4 v = *reinterpret_cast<const float4*>(ostage + local);
        quantise_vec4(v, lo + local, im.K, 0, img.q4, img.q6, img.xs, img.xsum16, img.xsum32, lane, valid);
    }
}

// MMA: the tensor-core stage path is compiled in (a separate instance, so
// that the default instances keep their registers for the dp4a loop).
// TYPES: the weight types the instance handles (1: Q4_K, 2: Q6_K, 3: both).
// HELD: activation float4s a consumer thread holds while quantising (0: the
// input is an already quantised image, copied). Each launch runs its code
// cold, so an instance compiles in only the paths it takes: instruction
// fetch, not arithmetic, was the leading stall of the decode products.
template <int MT, int NR, bool MMA, int TYPES, int HELD>
__global__ void __launch_bounds__(17 * 32, 1) gemv_kernel(const __grid_constant__ GemvPlan p) {
    static_assert(!MMA || MT == 1, "tensor-core stages take a batch of one");
    constexpr bool PAIR = NR == 2;  // gate and up rows worked together (SwiGLU)
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (threadIdx.x == 0) trace_at(p.trace, p.trace_tag, 0);
    const int W = (int)(blockDim.x >> 5) - 1;  // consumer warps
    const int T = p.teams;                     // teams taking stages (<= W / kTeamWarps)
    const int S = p.S;
    const int K = p.K;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
    uint64_t* empty = full + S;
    uint8_t* bufs = smem + p.off_bufs;
    int* team_abort = reinterpret_cast<int*>(smem + p.off_misc) + 64;

    const int G = gridDim.x;
    // shares in units of group_stages stages (1 unless an output image is written)
    const int u = p.group_stages;
    const int units = (p.total_stages + u - 1) / u;
    const int s_begin = u * (int)((long long)units * blockIdx.x / G);
    const int s_end = min(u * (int)((long long)units * (blockIdx.x + 1) / G), p.total_stages);
    const int m0 = blockIdx.y * MT;
    const int mcount = min(MT, p.M - m0);

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full + i, 1);
            // a slot is free once every warp of its team has read it (one
            // arrival per warp); tensor-core stages release it once, after
            // their team barrier
            mbar_init(empty + i, MMA ? 1 : kTeamWarps);
        }
        for (int k = 0; k < 4; ++k) team_abort[k] = 0;
        if (p.gamma_bulk) mbar_init(full + 2 * S, 1);
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == W) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();
            if (p.gamma_bulk) {
                // a weight, independent of the preceding kernel: first in the
                // copy engine's queue, so that no consumer waits for it
                mbar_arrive_expect_tx(full + 2 * S, (uint32_t)K * 4u);
                bulk_g2s(smem + p.off_gamma, p.gamma, (uint32_t)K * 4u, full + 2 * S);
            }
            for (int i = 0, st = s_begin; st < s_end; ++i, ++st) {
                const int slot = i % S, use = i / S;
                uint64_t* fb = full + slot;
                if (use > 0 && !mbar_wait_bounded(empty + slot, (use - 1) & 1, p.err, ERR_WAIT_TIMEOUT_EMPTY)) break;
                // bounded queue: stage i is issued once stage i - inflight has
                // landed (its slot is not re-armed before stage i is issued,
                // so the parity names that stage's phase)
                if (p.inflight > 0 && i >= p.inflight) {
                    const int j = i - p.inflight;
                    if (!mbar_wait_bounded(full + j % S, (j / S) & 1, p.err, ERR_WAIT_TIMEOUT_FULL)) break;
                }
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
                // the ring is full (or this CTA's stages are all issued):
                // let HBM go on with the next kernel's operands, either at
                // once or once those stages have landed (prefetch_landed), so
                // that the prefetch does not share HBM with this CTA's own ring
                if ((i == S - 1 || st == s_end - 1) && blockIdx.y == 0) {
                    if (p.prefetch_landed && !mbar_wait_bounded(fb, use & 1, p.err, ERR_WAIT_TIMEOUT_FULL)) break;
                    issue_l2_prefetch(p.prefetch, blockIdx.x, G);
                }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    if (p.gamma && !p.gamma_bulk) {
        // a weight: independent of the preceding kernel, so it is staged
        // before the wait and the quantisation needs one global round trip
        float4* g4 = reinterpret_cast<float4*>(smem + p.off_gamma);
        for (int i = tid; i < K / 4; i += W * 32) g4[i] = __ldg(reinterpret_cast<const float4*>(p.gamma) + i);
    }
    pdl_wait();
    // the bulk-copied RMSNorm weight (issued first at the CTA's start)
    if (p.gamma_bulk && !mbar_wait_bounded(full + 2 * S, 0, p.err, ERR_WAIT_TIMEOUT_FULL)) team_abort[0] = 1;
    if (tid == 0) trace_at(p.trace, p.trace_tag, 1);
    const int nthreads = W * 32;
    const int resid_row0 = s_begin * p.rows_per_stage;
    const int resid_rows = p.off_resid >= 0 ? min(s_end * p.rows_per_stage, p.seg[0].rows) - resid_row0 : 0;
    if constexpr (HELD == 0)
        copy_image(p, smem, tid, nthreads, resid_row0, resid_rows);
    else
        quantise_activation<HELD>(p, m0, mcount, smem, tid, lane, warp, nthreads);
    if (tid == 0) trace_at(p.trace, p.trace_tag, 2);
    const uint8_t* xq4 = p.off_xq4 >= 0 ? smem + p.off_xq4 : nullptr;
    const uint8_t* xq6 = p.off_xq6 >= 0 ? smem + p.off_xq6 : nullptr;
    const float* xs = reinterpret_cast<const float*>(smem + p.off_xs);
    const int* xsum16 = reinterpret_cast<const int*>(smem + p.off_xsum16);
    const float* xsum32 = reinterpret_cast<const float*>(smem + p.off_xsum32);

    // the step's tag of EPI_PEER words (read after the dependency wait)
    const unsigned peer_tag = p.epilogue == EPI_PEER ? (unsigned)(*p.peer_out.epoch + 1) : 0u;
    const int team = warp / kTeamWarps;
    const int team_threads = kTeamWarps * 32;
    const int LPR = p.lpr;
    const int sub = lane % LPR;                                        // lane within the row's lanes
    const int slot_row = (warp % kTeamWarps) * (32 / LPR) + lane / LPR;  // row of the stage
    const int chunks = p.nb * 4;  // 64-value pair-chunks (Q4_K) or quarters (Q6_K) per row
    const int full_iters = chunks / LPR;  // chunks every lane of a row takes
    const int lane_part = sub & 3;  // the lane's chunk within a block (LPR is a multiple of 4)
    float best_score = -__int_as_float(0x7f800000);
    uint32_t best_index = 0xffffffffu;

    // Stage i always lands in slot i % S and is taken by team i % T; as T
    // divides S, each slot is only ever waited on by one team, in order, so
    // a parity wait can never see a phase two uses old.
    for (int i = team, st = s_begin + team; team < T && st < s_end; i += T, st += T) {
        const int slot = i % S, use = i / S;
        const bool landed = __all_sync(0xffffffffu, mbar_wait_bounded(full + slot, use & 1, p.err, ERR_WAIT_TIMEOUT_FULL));
        if (!landed) team_abort[team] = 1;
        if (tid == 0 && i == 0) trace_at(p.trace, p.trace_tag, 3);
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
        // tensor-core stages: 16 rows (8 gate + 8 up rows for SwiGLU), the
        // team's 4 warps take every 4th super-block
        const bool mma = MMA && (TYPES & 1) != 0 && p.seg[seg].type == Q4K_TYPE_Q4_K;
        const int par = (i / T) & 1;  // double buffer of the cross-warp partials
        float* mred = reinterpret_cast<float*>(smem + p.off_mred) + (team * 2 + par) * kTeamWarps * 16;
        if (mma) {
            const int gq = lane >> 2, tq = lane & 3, wt = warp % kTeamWarps;
            const int rg = gq < nr ? gq : 0;
            const uint8_t* row_g = buf + rg * rb;
            const uint8_t* row_h = PAIR ? buf + (p.rows_per_stage + rg) * rb : buf + (gq + 8 < nr ? gq + 8 : 0) * rb;
            float ag = 0.0f, ah = 0.0f;
            q4_rows_mma<2>(row_g, row_h, wt, kTeamWarps, p.nb, xq4, xs, xsum32, gq, tq, ag, ah);
            ag += __shfl_xor_sync(0xffffffffu, ag, 1);
            ag += __shfl_xor_sync(0xffffffffu, ag, 2);
            ah += __shfl_xor_sync(0xffffffffu, ah, 1);
            ah += __shfl_xor_sync(0xffffffffu, ah, 2);
            if (tq == 0) {
                mred[wt * 16 + gq] = ag;
                mred[wt * 16 + gq + 8] = ah;
            }
        } else if (TYPES == 1 || (TYPES == 3 && p.seg[seg].type == Q4K_TYPE_Q4_K)) {
            if constexpr ((TYPES & 1) != 0) {
                // unconditional chunks, then at most one guarded remainder (no
                // branch inside the unrolled loop)
#pragma unroll 2
                for (int k = 0; k < full_iters; ++k)
                    q4_pair<MT, NR>(rows, sub + LPR * k, lane_part, xq4, xs, xsum32, K, mcount, acc);
                if (sub + LPR * full_iters < chunks)
                    q4_pair<MT, NR>(rows, sub + LPR * full_iters, lane_part, xq4, xs, xsum32, K, mcount, acc);
            }
        } else {
            if constexpr ((TYPES & 2) != 0) {
#pragma unroll 2
                for (int k = 0; k < full_iters; ++k)
                    q6_quarter<MT, NR>(rows, p.nb, sub + LPR * k, lane_part, xq6, xs, xsum16, K, mcount, acc);
                if (sub + LPR * full_iters < chunks)
                    q6_quarter<MT, NR>(rows, p.nb, sub + LPR * full_iters, lane_part, xq6, xs, xsum16, K, mcount,
                                       acc);
            }
        }
        // this warp's reads of the stage are done (its results are computed):
        // release its share of the slot; no team barrier on the dp4a path,
        // where a row's lanes are all in one warp
        if (MMA) {
            named_barrier(1 + team, team_threads);
            if (warp % kTeamWarps == 0 && lane == 0) mbar_arrive(empty + slot);
        } else {
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + slot);
        }
        const bool abort_now = MMA ? team_abort[team] != 0 : !landed;
        bool owner;
        int out_row;
        if (mma) {
            // warp 0 of the team: lane r sums the four warps' partials of row r
            owner = warp % kTeamWarps == 0 && lane < (PAIR ? 8 : 16);
            out_row = lane;
            if (owner) {
                float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
                for (int w = 0; w < kTeamWarps; ++w) {
                    v0 += mred[w * 16 + lane];
                    if (PAIR) v1 += mred[w * 16 + lane + 8];
                }
                acc[0][0] = v0;
                acc[NR - 1][0] = PAIR ? v1 : v0;
            }
        } else {
            // reduce each row over its LPR lanes (fixed xor order)
#pragma unroll
            for (int r = 0; r < NR; ++r)
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    for (int o = LPR >> 1; o > 0; o >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], o);
            owner = sub == 0;
            out_row = slot_row;
        }
        if (abort_now) break;
        if (owner && out_row < nr) {
            float* y = p.seg[seg].y;
            const int row = r0 + out_row;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m >= mcount) break;
                float* out = y ? y + (size_t)(m0 + m) * p.ldy + row : nullptr;
                if (p.epilogue == EPI_STORE) {
                    *out = acc[0][m];
                } else if (p.epilogue == EPI_ADD) {
                    if (p.off_resid >= 0)
                        *out = reinterpret_cast<const float*>(smem + p.off_resid)[row - resid_row0] + acc[0][m];
                    else
                        *out += acc[0][m];
                } else if (p.epilogue == EPI_PEER) {
                    // this rank's partial sum of row `row` with this step's tag, one
                    // 8-byte word into every rank's receive slot
                    const unsigned long long word =
                        (unsigned long long)__float_as_uint(acc[0][m]) | ((unsigned long long)peer_tag << 32);
                    for (int r = 0; r < p.peer_out.world; ++r) p.peer_out.recv[r][row] = word;
                } else if (p.epilogue == EPI_SWIGLU) {
                    const float g = acc[0][m], up = acc[NR - 1][m];
                    const float a = (g / (1.0f + expf(-g))) * up;  // silu_multiply.cu:9-10
                    *out = a;
                    if (PAIR && p.out_image.base)
                        reinterpret_cast<float*>(smem + p.off_ostage)[row - s_begin * p.rows_per_stage] = a;
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

    if (tid == 0) trace_at(p.trace, p.trace_tag, 4);
    if (PAIR && p.out_image.base) {
        named_barrier(kAllConsumersBarrier, nthreads);  // every output row of this CTA is written
        quantise_output_groups(p, s_begin * p.rows_per_stage, min(s_end * p.rows_per_stage, p.seg[0].rows), smem,
                               lane, warp, nthreads);
        if (tid == 0) trace_at(p.trace, p.trace_tag, 6);
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
    if (tid == 0) trace_at(p.trace, p.trace_tag, 7);
}

template <int MT, int NR, bool MMA = false, int TYPES = 3, int HELD = kHeldVec4>
cudaError_t launch_instance(const GemvPlan& plan, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl) {
    static std::once_flag once;
    static cudaError_t attr_status = cudaSuccess;
    static size_t max_dynamic = 0;
    std::call_once(once, [] {
        // static + dynamic shared memory must fit the 227 KB per-block limit
        cudaFuncAttributes fa{};
        attr_status = cudaFuncGetAttributes(&fa, gemv_kernel<MT, NR, MMA, TYPES, HELD>);
        if (attr_status != cudaSuccess) return;
        max_dynamic = 227 * 1024 - fa.sharedSizeBytes;
        attr_status = cudaFuncSetAttribute(gemv_kernel<MT, NR, MMA, TYPES, HELD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
    return cudaLaunchKernelEx(&cfg, gemv_kernel<MT, NR, MMA, TYPES, HELD>, plan);
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
    for (int e = 0; e < kMaxPrefetch; ++e) p.prefetch[e] = rq.prefetch[e];
    p.in_image = rq.in_image;
    p.out_image = rq.out_image;
    p.peer_out = rq.peer_out;
    p.peer_in = rq.peer_in;
    if (rq.epilogue == EPI_PEER) {
        if (rq.M != 1 || rq.nseg != 1 || p.peer_out.world < 1 || p.peer_out.world > kMaxRanks)
            return cudaErrorInvalidValue;
        if (!p.peer_out.epoch) return cudaErrorInvalidValue;
        for (int r = 0; r < p.peer_out.world; ++r)
            if (!p.peer_out.recv[r]) return cudaErrorInvalidValue;
    }
    if (p.peer_in.world >= 0 && (rq.M != 1 || !rq.gamma || p.peer_in.world > kMaxRanks ||
                                 (p.peer_in.world > 0 && (!p.peer_in.parts || !p.peer_in.epoch))))
        return cudaErrorInvalidValue;
    if (p.in_image.base && (rq.M != 1 || rq.gamma || p.in_image.K != rq.K)) return cudaErrorInvalidValue;
    if (p.out_image.base && (!pair || rq.M != 1 || p.out_image.K != rq.seg[0].rows || p.out_image.K % 256 != 0))
        return cudaErrorInvalidValue;
    bool need_q4 = false, need_q6 = false;
    int max_row = 0;
    for (int s = 0; s < rq.nseg; ++s) {
        const GemvSegment& g = rq.seg[s];
        if ((g.type != Q4K_TYPE_Q4_K && g.type != Q4K_TYPE_Q6_K) || g.rows <= 0 || !g.w ||
            reinterpret_cast<uintptr_t>(g.w) % 16 != 0)
            return cudaErrorInvalidValue;
        if (!g.y && rq.epilogue != EPI_ARGMAX && rq.epilogue != EPI_PEER) return cudaErrorInvalidValue;
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
    p.off_gamma = -1;
    if (rq.gamma) {
        p.off_gamma = off;
        off += rq.K * 4;
    }
    p.off_mred = off;
    off += 4 * 2 * kTeamWarps * 16 * 4;  // [team][2][warp][16 rows] partials of tensor-core stages
    off = align_up(off, 128);

    // Lanes per row: about five 64-value chunks per lane per stage.
    const int chunks = p.nb * 4;
    int lpr = env_int("Q4K_GEMV_LPR", chunks <= 48 ? 8 : chunks <= 80 ? 16 : 32);
    if (lpr != 8 && lpr != 16 && lpr != 32) lpr = 32;
    // Tensor-core stages need 16 rows (8 gate + 8 up for SwiGLU): for a
    // batch of one with Q4_K rows of up to 3072 inputs (bank-friendly row
    // strides), pick the lane split that gives that stage height.
    const bool any_q4 = need_q4;
    // Opt-in (Q4K_GEMV_MMA=1): measured no faster than the dp4a path here.
    const bool mma = rq.M == 1 && any_q4 && rq.K <= 3072 && env_int("Q4K_GEMV_MMA", 0) != 0;
    if (mma) lpr = pair ? 16 : 8;
    // consumer warps: teams of four, 12 by default (measured 1.6% faster
    // than 16 in the decode step); K/4 float4s of an activation row that is
    // quantised here must fit the prologue's registers (kHeldVec4 per
    // thread), which takes 16 warps past K = 9216
    const int R = kTeamWarps * 32 / lpr;
    // long products (the output head: dozens of stages per CTA) stream in
    // steady state, where 16 warps keep up with HBM better
    long long total_rows = 0;
    for (int s2 = 0; s2 < (pair ? 1 : rq.nseg); ++s2) total_rows += rq.seg[s2].rows;
    const bool long_product = total_rows / R > 8LL * sm_count();
    int W = env_int("Q4K_GEMV_WARPS", long_product ? 16 : 12);
    if (W != 8 && W != 12 && W != 16) W = 12;
    if (!rq.in_image.base && rq.K / 4 > kHeldVec4 * W * 32) W = 16;
    if (!rq.in_image.base && rq.K / 4 > kHeldVec4 * W * 32) return cudaErrorInvalidValue;
    const int rows_in_stage = pair ? 2 * R : R;
    const int stage_bytes = align_up(rows_in_stage * max_row, 128);

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
    // SwiGLU with an output image: CTA shares start on 32-row groups, so
    // that each CTA quantises whole groups of its own rows
    p.group_stages = 1;
    p.off_ostage = -1;
    if (p.out_image.base) {
        if (32 % R != 0) return cudaErrorInvalidValue;
        p.group_stages = 32 / R;
        const int units = (stages + p.group_stages - 1) / p.group_stages;
        ctas = std::min(ctas, units);
        const int max_rows = p.group_stages * ((units + ctas - 1) / ctas) * R;
        p.off_ostage = off;
        off += align_up(max_rows * 4, 128);
    }
    p.off_resid = -1;
    if (rq.epilogue == EPI_ADD && rq.M == 1 && p.nseg == 1 && p.in_image.base && p.group_stages == 1 &&
        env_int("Q4K_RESID_PREFETCH", 1) != 0) {
        const int max_rows = ((stages + ctas - 1) / ctas) * R;
        if (max_rows <= W * 32) {  // one row per consumer thread
            p.off_resid = off;
            off += align_up(max_rows * 4, 128);
        }
    }
    const int budget = std::max(env_int("Q4K_GEMV_SMEM_KB", 200) * 1024 - off, stage_bytes);
    int S = std::min(budget / stage_bytes, 8);
    if (S < 2) S = 2;
    // every ring slot belongs to one team: teams <= S and S a multiple of it
    const int teams = std::min(W / kTeamWarps, S);
    S -= S % teams;
    if (off + S * stage_bytes + (2 * S + 1) * 8 > 220 * 1024) return cudaErrorInvalidValue;
    p.lpr = lpr;
    p.inflight = std::max(0, env_int("Q4K_GEMV_INFLIGHT", 0));
    p.prefetch_landed = env_int("Q4K_PREFETCH_LANDED", 0) != 0;
    p.gamma_bulk = rq.gamma && reinterpret_cast<uintptr_t>(rq.gamma) % 16 == 0 && env_int("Q4K_GAMMA_BULK", 1) != 0;
    if (p.inflight >= S) p.inflight = 0;
    p.mma = mma ? 1 : 0;
    p.rows_per_stage = R;
    p.stage_bytes = stage_bytes;
    p.S = S;
    p.teams = teams;
    p.off_bufs = off;
    off += S * stage_bytes;
    p.off_bars = off;
    off += (2 * S + 1) * 8;  // full, empty, and the RMSNorm weight's copy
    const size_t smem = (size_t)off;
    const dim3 grid(ctas, (rq.M + MT - 1) / MT), block((W + 1) * 32);

    const int NR = pair ? 2 : 1;
    if (MT == 1 && !mma) {
        // batch of one: an instance with only the weight types and input path used
        const int types = (need_q4 ? 1 : 0) | (need_q6 ? 2 : 0);
        const int held = p.in_image.base ? 0 : rq.K / 4 <= 2 * W * 32 ? 2 : kHeldVec4;
        auto pick = [&](auto nr_tag) -> cudaError_t {
            constexpr int R_ = decltype(nr_tag)::value;
            auto by_held = [&](auto types_tag) -> cudaError_t {
                constexpr int T_ = decltype(types_tag)::value;
                if (held == 0) return launch_instance<1, R_, false, T_, 0>(p, grid, block, smem, stream, rq.pdl);
                if (held == 2) return launch_instance<1, R_, false, T_, 2>(p, grid, block, smem, stream, rq.pdl);
                return launch_instance<1, R_, false, T_, kHeldVec4>(p, grid, block, smem, stream, rq.pdl);
            };
            if (types == 1) return by_held(std::integral_constant<int, 1>{});
            if (types == 2) return by_held(std::integral_constant<int, 2>{});
            return by_held(std::integral_constant<int, 3>{});
        };
        return NR == 2 ? pick(std::integral_constant<int, 2>{}) : pick(std::integral_constant<int, 1>{});
    }
    switch (MT * 4 + NR) {
        case 1 * 4 + 1:
            return mma ? launch_instance<1, 1, true>(p, grid, block, smem, stream, rq.pdl)
                       : launch_instance<1, 1>(p, grid, block, smem, stream, rq.pdl);
        case 2 * 4 + 1: return launch_instance<2, 1>(p, grid, block, smem, stream, rq.pdl);
        case 4 * 4 + 1: return launch_instance<4, 1>(p, grid, block, smem, stream, rq.pdl);
        case 8 * 4 + 1: return launch_instance<8, 1>(p, grid, block, smem, stream, rq.pdl);
        case 1 * 4 + 2:
            return mma ? launch_instance<1, 2, true>(p, grid, block, smem, stream, rq.pdl)
                       : launch_instance<1, 2>(p, grid, block, smem, stream, rq.pdl);
        case 2 * 4 + 2: return launch_instance<2, 2>(p, grid, block, smem, stream, rq.pdl);
        case 4 * 4 + 2: return launch_instance<4, 2>(p, grid, block, smem, stream, rq.pdl);
        case 8 * 4 + 2: return launch_instance<8, 2>(p, grid, block, smem, stream, rq.pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace q4k
