// Persistent decode-step kernel: one launch decodes one token.
//
// The same work as the per-product launch sequence of the engine
// (embed, 36 x [QKV, attention, O, gate/up, down], output head + argmax,
// src/Engine.cpp:37-114), but with one CTA per SM running every phase:
//
//   * warp 8 of each CTA is a producer that streams, in order, every weight
//     stage and every K/V tile this CTA will consume during the whole step
//     into a 4-slot shared-memory ring (cp.async.bulk for weights, 2-D TMA for
//     the KV cache). Weights and the cache do not depend on the step's
//     activations, so the producer never waits for a phase: while the
//     consumers wait for the previous phase to finish everywhere, the next
//     phase's bytes are already arriving. HBM never drains between products.
//   * warps 0..7 are consumers. Before phase p they wait until every CTA has
//     finished phase dep(p) (a per-phase arrivals counter in global memory,
//     release/acquire), then do their share: a range of row stages of a
//     product (2 teams of 4 warps, the per-lane arithmetic of gemv.cu) or one
//     (KV head, split) unit of attention (attention_decode.cu's arithmetic,
//     each team taking whole 64-position tiles), then arrive on phase p.
//   * 9 warps allow 168 registers per thread, so every phase is inlined with
//     no local memory: under a saturated HBM stream a spill that misses L1
//     costs microseconds.
//
// Every wait is bounded (kWaitLimitNs); a CTA that gives up raises the shared
// abort flag, records an error bit and stops, and every other wait polls the
// flag, so a failure ends the launch instead of hanging it.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <math_constants.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "attention_device.cuh"
#include "decode_step.h"
#include "dequant_device.cuh"
#include "gemv_device.cuh"
#include "q4k_device.cuh"
#include "q4k_format.h"

namespace q4k {
namespace {

using namespace gemv_dev;
using namespace attn_dev;

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kTeams = 2;
constexpr int kTeamWarps = 4;
constexpr int kTeamThreads = kTeamWarps * 32;
constexpr int kS = kStepSlots;
constexpr int kSlot = kStepSlotBytes;
constexpr int kBarConsumers = 8;  // named barrier of all consumer warps (1..4: teams)
constexpr int kBarPrologue = 9;   // attention prologue: consumer warps 0..7
constexpr int kPrologueThreads = 256;
constexpr int kKvStage = 2 * kTileBytes;  // K + V tile
static_assert(kKvStage <= kSlot, "a K/V tile must fit a ring slot");
static_assert(kS % kTeams == 0, "every ring slot belongs to one team");
static_assert(sizeof(StepPhase) % 4 == 0, "phase descriptors are copied as words");
static_assert(kSlot % 1024 == 0, "slots keep the 1024-byte alignment of the TMA swizzle");

struct Tail {
    uint4 qf[8][32];  // Q MMA fragments (hi/lo) of the current attention unit
    float q[G][D];
    uint16_t k_new[D];
    uint16_t v_new[D];
    float red[64];
    float am_score[32];
    uint32_t am_index[32];
    uint64_t full[kS];
    uint64_t empty[kS];
    uint64_t xbar;  // the activation's bulk copy into the staging buffer
    float mred[kTeams][2][kTeamWarps][16];  // cross-warp partials of tensor-core stages
    // the current phase's descriptor for the consumers and, separately, for
    // the producer (which runs ahead): read from shared memory on every stage
    // instead of from global memory
    StepPhase phase_c;
    StepPhase phase_p;
    int team_abort[kTeams];
    int abort_local;
    int last;
    volatile int issued;  // stages the producer has issued (read on the exit path)
};

constexpr int kStageXBytes = 40 * 1024;  // fp32 activation (+ gamma) of a phase: K <= 10240
constexpr int kSmemBytes = kS * kSlot + kStepUnionBytes + kStageXBytes + (int)sizeof(Tail) + 1024;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool abort_raised(const StepArgs& a) {
    return *reinterpret_cast<volatile const unsigned*>(a.sync + a.nphases) != 0u;
}

__device__ __forceinline__ void raise_abort(const StepArgs& a, int code) {
    atomicOr(a.err, code);
    atomicExch(a.sync + a.nphases, 1u);
}

// Ring-slot wait: bounded, and it also gives up once another CTA aborted.
// The producer passes a sleep between polls so that its waiting does not
// take issue slots from the consumer warps of its scheduler.
__device__ bool slot_wait(uint64_t* bar, uint32_t parity, const StepArgs& a, int code, unsigned sleep_ns = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (unsigned it = 1;; ++it) {
        if (sleep_ns) __nanosleep(sleep_ns);
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 31u) == 0u) {
            if (abort_raised(a)) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
                raise_abort(a, code);
                return false;
            }
        }
    }
}

// Waits until `target` CTAs have arrived on phase `dep`.
__device__ bool dep_wait(const StepArgs& a, int dep, unsigned target) {
    const unsigned* flag = a.sync + dep;
    if (ld_acquire(flag) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (ld_acquire(flag) >= target) return true;
        if (abort_raised(a)) return false;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            raise_abort(a, ERR_WAIT_TIMEOUT_DEP);
            return false;
        }
        __nanosleep(20);
    }
}

__device__ __forceinline__ void stage_rows(const StepPhase& P, int st, int& seg, int& r0, int& nr) {
    seg = 0;
    while (seg + 1 < P.nseg && st >= P.stage_start[seg + 1]) ++seg;
    r0 = (st - P.stage_start[seg]) * P.R;
    nr = min(P.R, P.rows[seg] - r0);
}

struct AttnUnit {
    bool active;
    int kvh, p0, p1, tiles;
};

__device__ __forceinline__ AttnUnit attn_unit(const StepArgs& a, int cta, int pos) {
    AttnUnit u;
    u.active = cta < a.kv_heads * a.splits;
    const int n_keys = pos + 1;
    const int chunk = (n_keys + a.splits - 1) / a.splits;
    const int split = u.active ? cta % a.splits : 0;
    u.kvh = u.active ? cta / a.splits : 0;
    u.p0 = min(split * chunk, n_keys);
    u.p1 = min(u.p0 + chunk, n_keys);
    u.tiles = u.active ? (u.p1 - u.p0 + kAttnTile - 1) / kAttnTile : 0;
    return u;
}

__device__ __forceinline__ void gemv_range(const StepPhase& P, int cta, int ctas, int& s_begin, int& n) {
    s_begin = (int)((long long)P.total_stages * cta / ctas);
    n = (int)((long long)P.total_stages * (cta + 1) / ctas) - s_begin;
}

// ---------------------------------------------------------------- producer
__device__ __forceinline__ void producer(const StepArgs& a, const CUtensorMap* kmap, const CUtensorMap* vmap, uint8_t* ring,
                         Tail& tl, int pos) {
    const uint64_t policy = policy_evict_first();
    const int cta = blockIdx.x, ctas = gridDim.x;
    int i = 0;
    for (int ph = 0; ph < a.nphases; ++ph) {
        {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(a.phases + ph);
            uint32_t* dst = reinterpret_cast<uint32_t*>(&tl.phase_p);
            for (int w = 0; w < (int)(sizeof(StepPhase) / 4); ++w) dst[w] = __ldg(src + w);
        }
        const StepPhase& P = tl.phase_p;
        int n = 0, s_begin = 0;
        AttnUnit u{};
        if (P.kind == kStepGemv) {
            gemv_range(P, cta, ctas, s_begin, n);
        } else if (P.kind == kStepAttention) {
            u = attn_unit(a, cta, pos);
            n = u.tiles;
        }
        unsigned long long pwait = 0;  // trace only: ns the producer waited for free slots
        for (int k = 0; k < n; ++k, ++i) {
            const int slot = i % kS, use = i / kS;
            const uint64_t w0 = a.trace ? global_timer_ns() : 0;
            if (use > 0 && !slot_wait(&tl.empty[slot], (use - 1) & 1, a, ERR_WAIT_TIMEOUT_EMPTY, 200)) return;
            if (a.trace) pwait += global_timer_ns() - w0;
            // keep at most `inflight` stages on the way: a deeper queue of
            // weight bytes in front of this SM delays the activation loads
            // that every phase starts with
            if (a.inflight < kS && i >= a.inflight) {
                const int j = i - a.inflight;
                if (!slot_wait(&tl.full[j % kS], (j / kS) & 1, a, ERR_WAIT_TIMEOUT_FULL, 200)) return;
            }
            uint8_t* dst = ring + (size_t)slot * kSlot;
            uint64_t* fb = &tl.full[slot];
            if (P.kind == kStepGemv) {
                int seg, r0, nr;
                stage_rows(P, s_begin + k, seg, r0, nr);
                const int rb = P.row_bytes[seg];
                if (P.pair) {
                    mbar_arrive_expect_tx(fb, 2 * nr * rb);
                    bulk_g2s_hint(dst, P.w[0] + (size_t)r0 * rb, nr * rb, fb, policy);
                    bulk_g2s_hint(dst + P.R * rb, P.w[1] + (size_t)r0 * rb, nr * rb, fb, policy);
                } else {
                    mbar_arrive_expect_tx(fb, nr * rb);
                    bulk_g2s_hint(dst, P.w[seg] + (size_t)r0 * rb, nr * rb, fb, policy);
                }
            } else {
                const int y = (P.layer * a.kv_heads + u.kvh) * a.capacity + u.p0 + k * kAttnTile;
                mbar_arrive_expect_tx(fb, kKvStage);
                tma_load_2d(dst, kmap, 0, y, fb);
                tma_load_2d(dst + kBox, kmap, 64, y, fb);
                tma_load_2d(dst + kTileBytes, vmap, 0, y, fb);
                tma_load_2d(dst + kTileBytes + kBox, vmap, 64, y, fb);
            }
            tl.issued = i + 1;
        }
        if (a.trace && P.kind == kStepGemv)
            a.trace[((size_t)ph * kTraceCtas + blockIdx.x) * kTraceSlots + 6] = pwait;
    }
}

// ------------------------------------------------------- product phases
struct XArea {
    uint8_t* xq4;
    uint8_t* xq6;
    float* xs;
    int* xsum16;
    float* xsum32;
};

__device__ __forceinline__ XArea x_area(uint8_t* uni, const StepPhase& P) {
    XArea x;
    const int K = P.K;
    x.xq4 = P.q4 ? uni : nullptr;
    x.xq6 = P.q6 ? uni + (P.q4 ? K : 0) : nullptr;
    uint8_t* f = uni + K * (P.q4 + P.q6);
    x.xs = reinterpret_cast<float*>(f);
    x.xsum16 = reinterpret_cast<int*>(f + K / 8);
    x.xsum32 = reinterpret_cast<float*>(f + K / 8 + K / 4);
    return x;
}

// The phase's activation into shared memory: one bulk copy brings x (and
// the RMSNorm gamma) into the staging buffer, then the consumers RMSNorm it
// (when the phase has a gamma) and write the Q8 codes. Working from shared
// memory keeps almost nothing live per thread, so nothing spills. Returns
// false if the copy did not land (the launch is aborting).
__device__ __forceinline__ bool quantise_phase(const StepArgs& a, const StepPhase& P, const XArea& xa, float* xst,
                                               Tail& tl, int use, int tid, int lane, int warp, int ph) {
    const int K = P.K, nvec = K / 4;
    const bool norm = P.gamma != nullptr;
    if (tid == 0) {
        // x was written by other CTAs (generic proxy) and is read here by the
        // bulk-copy (async) proxy; the staging buffer was last read generically
        asm volatile("fence.proxy.async;" ::: "memory");
        mbar_arrive_expect_tx(&tl.xbar, (uint32_t)(K * 4 * (norm ? 2 : 1)));
        bulk_g2s(xst, P.x, (uint32_t)(K * 4), &tl.xbar);
        if (norm) bulk_g2s(xst + K, P.gamma, (uint32_t)(K * 4), &tl.xbar);
    }
    const bool landed = slot_wait(&tl.xbar, use & 1, a, ERR_WAIT_TIMEOUT_FULL);
    if (named_barrier_or(kBarConsumers, kConsumerThreads, !landed)) return false;
    if (tid == 0) trace_at(a.trace, ph, 4);
    const float4* x4 = reinterpret_cast<const float4*>(xst);
    const float4* g4 = reinterpret_cast<const float4*>(xst + K);
    float inv = 1.0f;
    if (norm) {
        float ss = 0.0f;
#pragma unroll 1
        for (int i = tid; i < nvec; i += kConsumerThreads) {
            const float4 v = x4[i];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        ss = warp_sum(ss);
        if (lane == 0) tl.red[warp] = ss;
        named_barrier(kBarConsumers, kConsumerThreads);
        float total = 0.0f;
        for (int w = 0; w < kConsumerWarps; ++w) total += tl.red[w];
        inv = rsqrtf(total / (float)K + a.eps);  // rms_norm.cu:17
    }
    // nvec is a multiple of 64, so every warp's lanes stay together
#pragma unroll 2
    for (int i = tid; i < nvec; i += kConsumerThreads) {
        float4 v = x4[i];
        if (norm) {
            const float4 g = g4[i];
            // rms_norm.cu:19: input * inverse_rms * scale
            v = make_float4((v.x * inv) * g.x, (v.y * inv) * g.y, (v.z * inv) * g.z, (v.w * inv) * g.w);
        }
        quantise_vec4(v, 4 * i, K, 0, xa.xq4, xa.xq6, xa.xs, xa.xsum16, xa.xsum32, lane);
    }
    named_barrier(kBarConsumers, kConsumerThreads);
    return true;
}

template <int NR>
__device__ __forceinline__ void gemv_phase(const StepArgs& a, const StepPhase& P, int ph, uint8_t* ring, uint8_t* uni,
                                           Tail& tl, int& i, int tid, int lane, int warp) {
    const int cta = blockIdx.x, ctas = gridDim.x;
    int s_begin, n;
    gemv_range(P, cta, ctas, s_begin, n);
    const XArea xa = x_area(uni, P);
    const int K = P.K;

    const int team = warp / kTeamWarps;
    const int LPR = P.lpr;
    const int sub = lane % LPR;
    const int slot_row = (warp % kTeamWarps) * (32 / LPR) + lane / LPR;
    const int chunks = P.nb * 4;
    const int iters = (chunks + LPR - 1) / LPR;
    const int part = sub & 3;
    const int epilogue = P.epilogue;
    float best_score = -CUDART_INF_F;
    uint32_t best_index = 0xffffffffu;
    // stage k of this phase is sequence index i + k: slot (i+k) % S, team (i+k) % T
    const int k0 = ((team - i) % kTeams + kTeams) % kTeams;
    unsigned long long waited = 0;  // trace only: ns this thread spent waiting for stages
    for (int k = k0; k < n; k += kTeams) {
        const int idx = i + k, slot = idx % kS, use = idx / kS;
        const uint64_t w0 = a.trace ? global_timer_ns() : 0;
        const bool landed = slot_wait(&tl.full[slot], use & 1, a, ERR_WAIT_TIMEOUT_FULL);
        if (a.trace) waited += global_timer_ns() - w0;
        // trace only: per-stage times of team 0 in layer 5's phases (launch 255)
        const int dk = (k - k0) / kTeams;
        if (a.trace && tid == 0 && dk < 4 && ph >= 26 && ph <= 30)
            a.trace[((size_t)(255 - (30 - ph)) * kTraceCtas + blockIdx.x) * kTraceSlots + 2 * dk] = global_timer_ns();
        if (tid == 0 && k == k0) trace_at(a.trace, ph, 2);
        int seg, r0, nr;
        stage_rows(P, s_begin + k, seg, r0, nr);
        const int rb = P.row_bytes[seg];
        const uint8_t* buf = ring + (size_t)slot * kSlot;
        const int rr = slot_row < nr ? slot_row : 0;  // idle rows alias row 0; dropped below
        const uint8_t* rows[NR];
        rows[0] = buf + rr * rb;
        if (NR == 2) rows[NR - 1] = buf + (P.R + rr) * rb;
        float acc[NR][1];
#pragma unroll
        for (int r = 0; r < NR; ++r) acc[r][0] = 0.0f;
        const bool mma = P.mma && P.type[seg] == Q4K_TYPE_Q4_K;
        float* mred = &tl.mred[team][(k / kTeams) & 1][0][0];
        if (mma) {
            const int gq = lane >> 2, tq = lane & 3, wt = warp % kTeamWarps;
            const int rg = gq < nr ? gq : 0;
            const uint8_t* row_g = buf + rg * rb;
            const uint8_t* row_h = NR == 2 ? buf + (P.R + rg) * rb : buf + (gq + 8 < nr ? gq + 8 : 0) * rb;
            float ag = 0.0f, ah = 0.0f;
            q4_rows_mma<3>(row_g, row_h, wt, kTeamWarps, P.nb, xa.xq4, xa.xs, xa.xsum32, gq, tq, ag, ah);
            ag += __shfl_xor_sync(0xffffffffu, ag, 1);
            ag += __shfl_xor_sync(0xffffffffu, ag, 2);
            ah += __shfl_xor_sync(0xffffffffu, ah, 1);
            ah += __shfl_xor_sync(0xffffffffu, ah, 2);
            if (tq == 0) {
                mred[wt * 16 + gq] = ag;
                mred[wt * 16 + gq + 8] = ah;
            }
        } else if (P.type[seg] == Q4K_TYPE_Q4_K) {
#pragma unroll 4
            for (int it = 0; it < iters; ++it) {
                const int f = sub + LPR * it;
                if (f < chunks) q4_pair<1, NR>(rows, f, part, xa.xq4, xa.xs, xa.xsum32, K, 1, acc);
            }
        } else {
#pragma unroll 4
            for (int it = 0; it < iters; ++it) {
                const int f = sub + LPR * it;
                if (f < chunks) q6_quarter<1, NR>(rows, P.nb, f, part, xa.xq6, xa.xs, xa.xsum16, K, 1, acc);
            }
        }
        // every read of the slot by this team is done: release it
        const bool abort_now = named_barrier_or(1 + team, kTeamThreads, !landed);
        if (warp % kTeamWarps == 0 && lane == 0) {
            mbar_arrive(&tl.empty[slot]);
            if (abort_now) tl.team_abort[team] = 1;
        }
        if (a.trace && tid == 0 && dk < 4 && ph >= 26 && ph <= 30)
            a.trace[((size_t)(255 - (30 - ph)) * kTraceCtas + blockIdx.x) * kTraceSlots + 2 * dk + 1] = global_timer_ns();
        bool owner;
        int out_row;
        if (mma) {
            // warp 0 of the team: lane r sums the four warps' partials of row r
            owner = warp % kTeamWarps == 0 && lane < (NR == 2 ? 8 : 16);
            out_row = lane;
            if (owner) {
                float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
                for (int w = 0; w < kTeamWarps; ++w) {
                    v0 += mred[w * 16 + lane];
                    if (NR == 2) v1 += mred[w * 16 + lane + 8];
                }
                acc[0][0] = v0;
                acc[NR - 1][0] = NR == 2 ? v1 : v0;
            }
        } else {
#pragma unroll
            for (int r = 0; r < NR; ++r)
                for (int o = LPR >> 1; o > 0; o >>= 1) acc[r][0] += __shfl_xor_sync(0xffffffffu, acc[r][0], o);
            owner = sub == 0;
            out_row = slot_row;
        }
        if (abort_now) break;
        if (owner && out_row < nr) {
            const int row = r0 + out_row;
            float* y = P.y[seg];
            if (epilogue == EPI_STORE) {
                y[row] = acc[0][0];
            } else if (epilogue == EPI_ADD) {
                y[row] = __ldcg(y + row) + acc[0][0];
            } else if (epilogue == EPI_SWIGLU) {
                const float g = acc[0][0], u = acc[NR - 1][0];
                y[row] = (g / (1.0f + expf(-g))) * u;  // silu_multiply.cu:9-10
            } else {
                if (y) y[row] = acc[0][0];
                if (candidate_better(acc[0][0], (uint32_t)row, best_score, best_index)) {
                    best_score = acc[0][0];
                    best_index = (uint32_t)row;
                }
            }
        }
    }
    i += n;
    if (tid == 0) trace_at(a.trace, ph, 3);
    if (tid == 0 && a.trace) a.trace[((size_t)ph * kTraceCtas + blockIdx.x) * kTraceSlots + 5] = waited;

    if (epilogue == EPI_ARGMAX) {
        // CTA best, then the last CTA reduces the CTAs in index order
        // (argmax.cu:25-61, :89-97) and finishes the step.
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
            tl.am_score[warp] = best_score;
            tl.am_index[warp] = best_index;
        }
        named_barrier(kBarConsumers, kConsumerThreads);
        if (tid == 0) {
            float bs = tl.am_score[0];
            uint32_t bi = tl.am_index[0];
            for (int w = 1; w < kConsumerWarps; ++w)
                if (candidate_better(tl.am_score[w], tl.am_index[w], bs, bi)) {
                    bs = tl.am_score[w];
                    bi = tl.am_index[w];
                }
            a.argmax.cand_score[cta] = bs;
            a.argmax.cand_index[cta] = bi;
            __threadfence();
            tl.last = atomicAdd(a.argmax.counter, 1u) == (unsigned)(ctas - 1);
        }
        named_barrier(kBarConsumers, kConsumerThreads);
        if (tl.last && warp == 0) {
            __threadfence();
            float bs = -CUDART_INF_F;
            uint32_t bi = 0xffffffffu;
            for (int c = lane; c < ctas; c += 32) {
                const float s = __ldcg(a.argmax.cand_score + c);
                const uint32_t ix = __ldcg(a.argmax.cand_index + c);
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
                const uint32_t tok = bi == 0xffffffffu ? bi : bi + a.argmax.index_base;
                *a.token = tok;
                if (a.argmax.score) *a.argmax.score = bs;
                *a.argmax.counter = 0u;
                // finish the step: record the token, advance the position
                const unsigned hn = *a.history_n;
                if (hn < a.history_cap) a.history[hn] = tok;
                *a.history_n = hn + 1;
                *a.pos += *a.advance;
            }
        }
    }
}

// ------------------------------------------------------ attention phases
__device__ __forceinline__ void attention_phase(const StepArgs& a, const StepPhase& P, int ph, uint8_t* ring, uint8_t* uni, Tail& tl,
                                int& i, int tid, int lane, int warp, int pos) {
    const AttnUnit u = attn_unit(a, blockIdx.x, pos);
    if (!u.active) return;
    const int kvh = u.kvh, p0 = u.p0, p1 = u.p1, tiles = u.tiles;
    const bool owner = pos >= p0 && pos < p1;
    const float* qkv = a.qkv;
    const float* q_raw = qkv + (size_t)kvh * G * D;
    const float* k_raw = qkv + (size_t)a.heads * D + (size_t)kvh * D;
    const float* v_raw = qkv + (size_t)a.heads * D + (size_t)a.kv_heads * D + (size_t)kvh * D;
    const size_t head_base = ((size_t)P.layer * a.kv_heads + kvh) * a.capacity * D;

    // ---- prologue (warps 0..7): q/k RMSNorm + RoPE, the new K/V row, Q fragments
    if (tid < kPrologueThreads) {
        const int h = tid >> 6, j = tid & 63;
        const float gq0 = P.gamma[j], gq1 = P.gamma[j + 64];
        const float gk0 = P.gamma2[j], gk1 = P.gamma2[j + 64];
        float sn, cs;
        sincosf(rope_angle(pos, j, a.rope_base), &sn, &cs);
        float x0 = __ldcg(q_raw + h * D + j), x1 = __ldcg(q_raw + h * D + j + 64);
        float kx0 = 0.0f, kx1 = 0.0f, vx0 = 0.0f, vx1 = 0.0f;
        if (owner && h == 0) {
            kx0 = __ldcg(k_raw + j);
            kx1 = __ldcg(k_raw + j + 64);
            vx0 = __ldcg(v_raw + j);
            vx1 = __ldcg(v_raw + j + 64);
        }
        const float ss = warp_sum(x0 * x0 + x1 * x1);
        const float kss = (owner && h == 0) ? warp_sum(kx0 * kx0 + kx1 * kx1) : 0.0f;
        if (lane == 0) {
            tl.red[2 * warp] = ss;
            tl.red[2 * warp + 1] = kss;
        }
        named_barrier(kBarPrologue, kPrologueThreads);
        const float qsum = tl.red[2 * (2 * h)] + tl.red[2 * (2 * h + 1)];
        const float inv = rsqrtf(qsum / (float)D + a.eps);  // rms_norm.cu:17
        x0 = (x0 * inv) * gq0;
        x1 = (x1 * inv) * gq1;
        tl.q[h][j] = x0 * cs - x1 * sn;  // rope.cu:21-22
        tl.q[h][j + 64] = x0 * sn + x1 * cs;
        if (owner && h == 0) {
            const float kinv = rsqrtf((tl.red[1] + tl.red[3]) / (float)D + a.eps);
            kx0 = (kx0 * kinv) * gk0;
            kx1 = (kx1 * kinv) * gk1;
            const uint16_t k0 = q4k_f32_to_f16(kx0 * cs - kx1 * sn);
            const uint16_t k1 = q4k_f32_to_f16(kx0 * sn + kx1 * cs);
            const uint16_t v0 = q4k_f32_to_f16(vx0), v1 = q4k_f32_to_f16(vx1);
            tl.k_new[j] = k0;
            tl.k_new[j + 64] = k1;
            tl.v_new[j] = v0;
            tl.v_new[j + 64] = v1;
            const size_t at = head_base + (size_t)pos * D;
            a.kcache[at + j] = k0;
            a.kcache[at + j + 64] = k1;
            a.vcache[at + j] = v0;
            a.vcache[at + j + 64] = v1;
        }
        named_barrier(kBarPrologue, kPrologueThreads);
        {
            const int s = tid >> 5, l = tid & 31, gg = l >> 2, tt = l & 3;  // 8 k-steps x 32 lanes
            uint4 f = make_uint4(0u, 0u, 0u, 0u);
            if (gg < G) {
                split2(tl.q[gg][16 * s + 2 * tt], tl.q[gg][16 * s + 2 * tt + 1], f.x, f.y);
                split2(tl.q[gg][16 * s + 8 + 2 * tt], tl.q[gg][16 * s + 8 + 2 * tt + 1], f.z, f.w);
            }
            tl.qf[s][l] = f;
        }
    }
    named_barrier(kBarConsumers, kConsumerThreads);
    if (tid == 0) trace_at(a.trace, ph, 1);

    // ---- tiles: team (i+t) % 4 takes tile t; warp w of the team owns rows [16w, 16w + 16)
    const int team = warp / kTeamWarps, wt = warp % kTeamWarps;
    const int g = lane >> 2, tq = lane & 3;
    const float scale = rsqrtf((float)D);  // attention.cu:40
    float m_run = -CUDART_INF_F, l_run = 0.0f;
    float o[16][2];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = 0.0f;
    const int k0 = ((team - i) % kTeams + kTeams) % kTeams;
    for (int t = k0; t < tiles; t += kTeams) {
        const int idx = i + t, slot = idx % kS, use = idx / kS;
        const bool landed = slot_wait(&tl.full[slot], use & 1, a, ERR_WAIT_TIMEOUT_FULL);
        if (tid == 0 && t == k0) trace_at(a.trace, ph, 2);
        const int lo = p0 + t * kAttnTile;
        const int n = min(kAttnTile, p1 - lo);
        uint8_t* kt = ring + (size_t)slot * kSlot;
        uint8_t* vt = kt + kTileBytes;
        const int prow = pos - lo;
#pragma unroll 1
        for (int sl = 0; sl < 2; ++sl) {
            const int rb = 16 * wt + 8 * sl;  // first tile row of this 8-position slab
            const bool mine = owner && prow >= rb && prow < rb + 8;
            if (mine) {
                // the new token's row replaces the cache's stale copy in the tile
                if (lane < 16) {
                    *reinterpret_cast<uint4*>(kt + tile_off(prow, lane)) =
                        *reinterpret_cast<const uint4*>(tl.k_new + 8 * lane);
                    *reinterpret_cast<uint4*>(vt + tile_off(prow, lane)) =
                        *reinterpret_cast<const uint4*>(tl.v_new + 8 * lane);
                }
                __syncwarp();
            }
            const int r_lane = rb + (lane & 7);
            float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const uint32_t kbase = smem_addr(kt);
#pragma unroll
            for (int s2 = 0; s2 < 8; s2 += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kbase + tile_off(r_lane, 2 * s2 + (lane >> 3)), b0, b1, b2, b3);
                const uint4 fa = tl.qf[s2][lane], fb = tl.qf[s2 + 1][lane];
                mma16816(sc, fa.x, fa.z, b0, b1);
                mma16816(sc, fa.y, fa.w, b0, b1);
                mma16816(sc, fb.x, fb.z, b2, b3);
                mma16816(sc, fb.y, fb.w, b2, b3);
            }
            const int c0 = rb + 2 * tq;
            const float s0 = c0 < n ? sc[0] * scale : -CUDART_INF_F;
            const float s1 = c0 + 1 < n ? sc[1] * scale : -CUDART_INF_F;
            float tmax = fmaxf(s0, s1);
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
            const float m_new = fmaxf(m_run, tmax);
            float p0v = 0.0f, p1v = 0.0f, rescale = 1.0f;
            if (m_new != -CUDART_INF_F) {
                p0v = expf(s0 - m_new);
                p1v = expf(s1 - m_new);
                rescale = expf(m_run - m_new);
            }
            float psum = p0v + p1v;
            psum += __shfl_xor_sync(0xffffffffu, psum, 1);
            psum += __shfl_xor_sync(0xffffffffu, psum, 2);
            l_run = l_run * rescale + psum;
            m_run = m_new;
            uint32_t pa_h, pa_l;
            split2(p0v, p1v, pa_h, pa_l);
            if (g >= G) pa_h = pa_l = 0u;
            const uint32_t vbase = smem_addr(vt);
#pragma unroll
            for (int j4 = 0; j4 < 16; j4 += 4) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vbase + tile_off(r_lane, j4 + (lane >> 3)), b0, b1, b2, b3);
                const uint32_t bb[4] = {b0, b1, b2, b3};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float c0f = o[j4 + q][0] * rescale, c1f = o[j4 + q][1] * rescale;
                    mma1688(c0f, c1f, pa_h, bb[q]);
                    mma1688(c0f, c1f, pa_l, bb[q]);
                    o[j4 + q][0] = c0f;
                    o[j4 + q][1] = c1f;
                }
            }
            if (mine) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before the slot's next TMA
        }
        const bool abort_now = named_barrier_or(1 + team, kTeamThreads, !landed);
        if (wt == 0 && lane == 0) {
            mbar_arrive(&tl.empty[slot]);
            if (abort_now) tl.team_abort[team] = 1;
        }
        if (abort_now) break;
    }
    i += tiles;
    if (tid == 0) trace_at(a.trace, ph, 3);

    // ---- merge the consumer warps in the shared scratch (fixed order)
    float* wm = reinterpret_cast<float*>(uni);          // [warps][G]
    float* wl = wm + kConsumerWarps * G;                // [warps][G]
    float* wo = wl + kConsumerWarps * G;                // [warps][G][D]
    if (g < G) {
        if (tq == 0) {
            wm[warp * G + g] = m_run;
            wl[warp * G + g] = l_run;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            wo[(warp * G + g) * D + 8 * j + 2 * tq] = o[j][0];
            wo[(warp * G + g) * D + 8 * j + 2 * tq + 1] = o[j][1];
        }
    }
    named_barrier(kBarConsumers, kConsumerThreads);
    bool aborted = false;
    for (int t = 0; t < kTeams; ++t) aborted |= tl.team_abort[t] != 0;
    const int hq = (tid >> 6) & 3;   // query head of the group
    const int d0 = 2 * (tid & 63);
    const bool merger = tid < kPrologueThreads;
    float M = -CUDART_INF_F, L = 0.0f, acc0 = 0.0f, acc1 = 0.0f;
    if (merger) {
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, wm[w * G + hq]);
        for (int w = 0; w < kConsumerWarps; ++w) {
            const float l = wl[w * G + hq];
            if (!(l > 0.0f)) continue;
            const float f = expf(wm[w * G + hq] - M);
            L += l * f;
            acc0 += wo[(w * G + hq) * D + d0] * f;
            acc1 += wo[(w * G + hq) * D + d0 + 1] * f;
        }
        if (aborted) {
            M = -CUDART_INF_F;
            L = acc0 = acc1 = 0.0f;
        }
        const int split = blockIdx.x % a.splits;
        const size_t pidx = ((size_t)kvh * a.splits + split) * G + hq;
        a.partial_o[pidx * D + d0] = acc0;
        a.partial_o[pidx * D + d0 + 1] = acc1;
        if ((tid & 63) == 0) {
            a.partial_ml[pidx * 2 + 0] = M;
            a.partial_ml[pidx * 2 + 1] = L;
        }
    }
    __threadfence();
    named_barrier(kBarConsumers, kConsumerThreads);
    if (tid == 0) tl.last = atomicAdd(a.counters + kvh, 1u) == (unsigned)(a.splits - 1);
    named_barrier(kBarConsumers, kConsumerThreads);
    if (!tl.last) return;
    __threadfence();
    // ---- the last CTA of this KV head merges the splits (log-sum-exp)
    float* mls = wo;  // [splits][G][2], after the warp merge is read
    const float* ml_head = a.partial_ml + (size_t)kvh * a.splits * G * 2;
    for (int k = tid; k < a.splits * G * 2; k += kConsumerThreads) mls[k] = __ldcg(ml_head + k);
    named_barrier(kBarConsumers, kConsumerThreads);
    if (!merger) return;
    float MM = -CUDART_INF_F;
    for (int sp = 0; sp < a.splits; ++sp)
        if (mls[(sp * G + hq) * 2 + 1] > 0.0f) MM = fmaxf(MM, mls[(sp * G + hq) * 2]);
    float LL = 0.0f, o0 = 0.0f, o1 = 0.0f;
    const float2* po = reinterpret_cast<const float2*>(a.partial_o + ((size_t)kvh * a.splits * G + hq) * D + d0);
    constexpr int kBatch = 16;
    for (int sp0 = 0; sp0 < a.splits; sp0 += kBatch) {
        float2 v[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; ++k)
            v[k] = sp0 + k < a.splits ? __ldcg(po + (size_t)(sp0 + k) * (G * D / 2)) : make_float2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
            if (sp0 + k < a.splits) {
                const float l = mls[((sp0 + k) * G + hq) * 2 + 1];
                if (l > 0.0f) {
                    const float f = expf(mls[((sp0 + k) * G + hq) * 2] - MM);
                    LL += l * f;
                    o0 += v[k].x * f;
                    o1 += v[k].y * f;
                }
            }
        }
    }
    float* out = a.att + ((size_t)kvh * G + hq) * D;
    out[d0] = o0 / LL;
    out[d0 + 1] = o1 / LL;
    if (tid == 0) a.counters[kvh] = 0u;
}

// ------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(kThreads, 1)
    decode_step_kernel(const __grid_constant__ StepArgs a, const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* ring = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t* uni = ring + (size_t)kS * kSlot;
    float* xst = reinterpret_cast<float*>(uni + kStepUnionBytes);
    Tail& tl = *reinterpret_cast<Tail*>(uni + kStepUnionBytes + kStageXBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int pos = *a.pos;
    const uint32_t token = *a.token;
    if (pos < 0 || pos >= a.capacity || token >= (uint32_t)a.vocab) {
        // every CTA reads the same values and leaves before any wait
        if (blockIdx.x == 0 && tid == 0) atomicOr(a.err, token >= (uint32_t)a.vocab ? ERR_BAD_TOKEN : ERR_BAD_POSITION);
        return;
    }
    if (tid == 0) {
        for (int s = 0; s < kS; ++s) {
            mbar_init(&tl.full[s], 1);
            mbar_init(&tl.empty[s], 1);
        }
        mbar_init(&tl.xbar, 1);
        for (int t = 0; t < kTeams; ++t) tl.team_abort[t] = 0;
        tl.abort_local = 0;
        tl.issued = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        if (lane == 0) producer(a, &kmap, &vmap, ring, tl, pos);
        return;
    }

    int i = 0;     // ring sequence index of the next stage this CTA consumes
    int xuse = 0;  // activation copies so far (parity of tl.xbar)
    for (int ph = 0; ph < a.nphases; ++ph) {
        // the previous phase's readers of tl.phase_c passed the phase-end barriers
        if (tid < (int)(sizeof(StepPhase) / 4))
            reinterpret_cast<uint32_t*>(&tl.phase_c)[tid] = __ldg(reinterpret_cast<const uint32_t*>(a.phases + ph) + tid);
        const StepPhase& P = tl.phase_c;
        bool failed = false;
        if (tid == 0) {
            const int dep = __ldg(&a.phases[ph].dep);  // tl.phase_c is complete only after the barrier below
            failed = dep >= 0 && !dep_wait(a, dep, gridDim.x);
            trace_at(a.trace, ph, 0);
        }
        if (named_barrier_or(kBarConsumers, kConsumerThreads, failed)) {
            tl.abort_local = 1;
            break;
        }
        if (P.kind == kStepEmbed) {
            // this CTA's share of the token's embedding row (EmbedLookup.cpp:49-78)
            const int per = (a.hidden + gridDim.x - 1) / gridDim.x;
            const int c0 = blockIdx.x * per, c1 = min(c0 + per, a.hidden);
            const size_t row_bytes = q4k_device_row_bytes(a.embd_type, (size_t)a.hidden);
            const uint8_t* row = a.embd + (size_t)token * row_bytes;
            for (int c = c0 + tid; c < c1; c += kConsumerThreads)
                a.x[c] = device_layout_value(row, a.embd_type, (size_t)a.hidden / 256, (size_t)c);
        } else if (P.kind == kStepGemv) {
            if (!quantise_phase(a, P, x_area(uni, P), xst, tl, xuse++, tid, lane, warp, ph)) {
                tl.abort_local = 1;
                break;
            }
            if (tid == 0) trace_at(a.trace, ph, 1);
            if (P.pair)
                gemv_phase<2>(a, P, ph, ring, uni, tl, i, tid, lane, warp);
            else
                gemv_phase<1>(a, P, ph, ring, uni, tl, i, tid, lane, warp);
        } else {
            attention_phase(a, P, ph, ring, uni, tl, i, tid, lane, warp, pos);
        }
        named_barrier(kBarConsumers, kConsumerThreads);
        const bool team_failed = tl.team_abort[warp / kTeamWarps] != 0;
        if (named_barrier_or(kBarConsumers, kConsumerThreads, team_failed)) {
            tl.abort_local = 1;
            break;
        }
        if (tid == 0) {
            __threadfence();
            atomicAdd(a.sync + ph, 1u);
            trace_at(a.trace, ph, 7);
        }
    }
    if (tl.abort_local && tid == 0) {
        // let the copies the producer issued into this CTA's ring land
        // (bounded) before the CTA's shared memory is released
        const uint64_t t0 = global_timer_ns();
        while (global_timer_ns() - t0 < 1000000ull) {
            const int n = tl.issued;
            bool all = true;
            for (int k = (n > kS ? n - kS : 0); k < n; ++k)
                if (!mbar_try_wait(&tl.full[k % kS], (k / kS) & 1)) all = false;
            if (all) break;
        }
    }
}

}  // namespace

bool step_gemv_geometry(int K, int max_row_bytes, bool pair, bool q4, bool q6, int& lpr, int& R) {
    if (K <= 0 || K % 256) return false;
    const int x_bytes = K * ((q4 ? 1 : 0) + (q6 ? 1 : 0)) + K / 8 + K / 4 + K / 8;
    if (x_bytes > kStepUnionBytes) return false;
    const int chunks = K / 256 * 4;
    lpr = chunks <= 48 ? 8 : chunks <= 80 ? 16 : 32;
    for (;;) {
        R = kTeamThreads / lpr;
        if ((long long)R * max_row_bytes * (pair ? 2 : 1) <= kSlot) return true;
        if (lpr == 32) return false;
        lpr *= 2;
    }
}

int step_ctas(std::string* why) {
    static int ctas = -1;
    static std::string reason;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaError_t e = cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) {
            reason = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
            ctas = 0;
            return;
        }
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kThreads, kSmemBytes);
        if (e != cudaSuccess || per_sm < 1) {
            cudaFuncAttributes fa{};
            cudaFuncGetAttributes(&fa, decode_step_kernel);
            char buf[256];
            std::snprintf(buf, sizeof buf,
                          "the kernel does not fit one CTA per SM (regs %d, max threads %d, local %zu B, static smem "
                          "%zu B, dynamic %d B, max dynamic %d B)",
                          fa.numRegs, fa.maxThreadsPerBlock, fa.localSizeBytes, fa.sharedSizeBytes, kSmemBytes,
                          fa.maxDynamicSharedSizeBytes);
            reason = e != cudaSuccess ? std::string("occupancy query: ") + cudaGetErrorString(e) : std::string(buf);
            ctas = 0;
            return;
        }
        ctas = sm_count();
    });
    if (why) *why = reason;
    return ctas;
}

cudaError_t launch_decode_step(const StepArgs& a, const KvTensorMap& kmap, const KvTensorMap& vmap, int ctas,
                               cudaStream_t s) {
    if (ctas <= 0 || ctas > 1024 || a.kv_heads * a.splits > ctas || a.inflight < 1) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(a.sync, 0, sizeof(unsigned) * (a.nphases + 1), s);
    if (e != cudaSuccess) return e;
    CUtensorMap km, vm;
    static_assert(sizeof(CUtensorMap) == sizeof(KvTensorMap), "tensor map storage");
    memcpy(&km, &kmap, sizeof km);
    memcpy(&vm, &vmap, sizeof vm);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident at once: phases wait on each other
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_step_kernel, a, km, vm);
}

}  // namespace q4k
