// Device-side helpers for sm_100a: shared-memory mbarriers, bulk (TMA) copies
// from global to shared memory, programmatic dependent launch controls and
// bounded waits.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q4k_format.h"
#include "q4k_internal.h"

namespace q4k {

// Error bits a kernel may OR into its error word.
enum : int {
    ERR_WAIT_TIMEOUT_FULL = 1,   // a consumer gave up waiting for a copy to land
    ERR_WAIT_TIMEOUT_EMPTY = 2,  // the producer gave up waiting for a buffer to drain
    ERR_BAD_POSITION = 4,        // a position read from device memory was out of range
    ERR_BAD_TOKEN = 8,           // a token id read from device memory was out of range
    ERR_WAIT_TIMEOUT_DEP = 16,   // a CTA gave up waiting for the other CTAs to finish a phase
    ERR_WAIT_TIMEOUT_PEER = 32,  // a product gave up waiting for the other ranks' partial sums
};

// A waiting thread gives up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Two consecutive 8-byte words, each read whole (a 64-bit element is
// single-copy atomic), from L2 at system scope: words other GPUs store.
__device__ __forceinline__ void ld_words2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Four (value, tag) words (value in the low half, tag in the high half) that
// other GPUs store into this GPU's memory: read until every tag is `tag`,
// giving up after limit_ns of %globaltimer with `code` in *err (at once if
// another wait already gave up). Returns the four values.
__device__ __forceinline__ float4 tagged_load4(const unsigned long long* p, unsigned tag, uint64_t limit_ns, int* err,
                                               int code) {
    unsigned long long w0, w1, w2, w3;
    ld_words2(p, w0, w1);
    ld_words2(p + 2, w2, w3);
    auto ready = [&] {
        return (unsigned)(w0 >> 32) == tag && (unsigned)(w1 >> 32) == tag && (unsigned)(w2 >> 32) == tag &&
               (unsigned)(w3 >> 32) == tag;
    };
    if (!ready()) {
        const uint64_t start = global_timer_ns();
        for (;;) {
            if (err && (*reinterpret_cast<volatile int*>(err) & code)) break;
            __nanosleep(32);
            ld_words2(p, w0, w1);
            ld_words2(p + 2, w2, w3);
            if (ready()) break;
            if (global_timer_ns() - start > limit_ns) {
                if (err) atomicOr(err, code);
                break;
            }
        }
    }
    return make_float4(__uint_as_float((unsigned)w0), __uint_as_float((unsigned)w1), __uint_as_float((unsigned)w2),
                       __uint_as_float((unsigned)w3));
}

// Sum, in rank order, of the four (value, tag) words at p + r * stride of
// ranks r < nparts (nparts <= kRanks). Every rank's words are loaded back to
// back and their tags checked together, so the sum costs one memory round
// trip when all words are there; tagged_load4 per rank is the wait for words
// still in flight (no branch on a loaded value separates the first loads, which
// a per-rank check would: one round trip per rank). Both paths add the ranks
// in the same order, so the result does not depend on which one ran.
template <int kRanks>
__device__ __forceinline__ float4 sum_tagged4(const unsigned long long* p, size_t stride, int nparts, unsigned tag,
                                              uint64_t limit_ns, int* err, int code) {
    unsigned long long w[kRanks][4];
#pragma unroll
    for (int r = 0; r < kRanks; ++r) {
        w[r][0] = w[r][1] = w[r][2] = w[r][3] = 0ull;
        if (r < nparts) {
            ld_words2(p + r * stride, w[r][0], w[r][1]);
            ld_words2(p + r * stride + 2, w[r][2], w[r][3]);
        }
    }
    bool ready = true;
    float4 s = make_float4(__uint_as_float((unsigned)w[0][0]), __uint_as_float((unsigned)w[0][1]),
                           __uint_as_float((unsigned)w[0][2]), __uint_as_float((unsigned)w[0][3]));
#pragma unroll
    for (int r = 0; r < kRanks; ++r) {
        if (r >= nparts) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) ready &= (unsigned)(w[r][j] >> 32) == tag;
        if (r > 0) {
            s.x += __uint_as_float((unsigned)w[r][0]);
            s.y += __uint_as_float((unsigned)w[r][1]);
            s.z += __uint_as_float((unsigned)w[r][2]);
            s.w += __uint_as_float((unsigned)w[r][3]);
        }
    }
    if (ready) return s;
    s = tagged_load4(p, tag, limit_ns, err, code);
    for (int r = 1; r < nparts; ++r) {
        const float4 t = tagged_load4(p + r * stride, tag, limit_ns, err, code);
        s.x += t.x;
        s.y += t.y;
        s.z += t.z;
        s.w += t.w;
    }
    return s;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// The same test, but the thread may be suspended until the phase completes
// or kSuspendHintNs have passed (the hardware wakes it on completion).
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return done != 0;
}

// Waits for the barrier phase with the given parity to complete; returns
// false (and records `code` in *err) if it has not after kWaitLimitNs.
// After a first plain test, each poll lets the hardware suspend the thread
// until the phase completes (up to kSuspendHintNs), so a waiting warp takes
// no issue slots from the working ones and wakes on the completion itself;
// %globaltimer is read once per poll. Measured against polling with the
// default suspend limit and a clock read every 64 polls: decode step +0.7%,
// prompt prefill +1%.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (;;) {
        if (mbar_try_wait_suspend(bar, parity)) return true;
        if (global_timer_ns() - start > kWaitLimitNs) {
            if (err) atomicOr(err, code);
            return false;
        }
    }
}

// One bulk copy global -> shared, completing `bytes` of transaction count on
// `bar`. dst, src and bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Same, with an L2 eviction-priority policy (weights are streamed once).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Asks L2 to fetch [p, p + bytes) from HBM; nothing completes or waits on it.
// p and bytes must be multiples of 16.
__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Issues this CTA's share (CTA `cta` of `ctas`, cut at 256-byte boundaries
// of the concatenated ranges) of the prefetch list as bulk L2 prefetches of
// at most 32 KB each. Addresses are kept in bounds of every range.
static __device__ __noinline__ void issue_l2_prefetch(const L2Prefetch* pf, int cta, int ctas) {
    unsigned long long len[kMaxPrefetch];
    unsigned long long total = 0;
    for (int e = 0; e < kMaxPrefetch; ++e) {
        unsigned long long l = 0;
        if (pf[e].base && pf[e].count > 0) {
            l = pf[e].bytes;
            if (pf[e].position) {
                int pos = *reinterpret_cast<const volatile int*>(pf[e].position);
                if (pos < 0) pos = 0;
                l = (unsigned long long)(pos + 1) * pf[e].bytes;
                if (l > pf[e].stride) l = pf[e].stride;
            }
            total += l * (unsigned long long)pf[e].count;
        }
        len[e] = l;
    }
    if (total == 0 || ctas <= 0) return;
    const unsigned long long lo = (total * (unsigned long long)cta / ctas) & ~255ull;
    const unsigned long long hi =
        cta + 1 >= ctas ? total : (total * (unsigned long long)(cta + 1) / ctas) & ~255ull;
    unsigned long long at = 0;  // start of the current range in the concatenation
    for (int e = 0; e < kMaxPrefetch && at < hi; ++e) {
        if (!len[e]) continue;
        for (int k = 0; k < pf[e].count && at < hi; ++k, at += len[e]) {
            const unsigned long long a = at > lo ? at : lo;
            const unsigned long long b = at + len[e] < hi ? at + len[e] : hi;
            if (a >= b) continue;
            const uintptr_t range = reinterpret_cast<uintptr_t>(pf[e].base) + (uintptr_t)k * pf[e].stride;
            uintptr_t p = (range + (a - at) + 15) & ~(uintptr_t)15;
            const uintptr_t end = (range + (b - at)) & ~(uintptr_t)15;
            while (p < end) {
                const uint32_t piece = end - p < 32768 ? (uint32_t)(end - p) : 32768u;
                l2_prefetch_bulk(reinterpret_cast<const void*>(p), piece);
                p += piece;
            }
        }
    }
}

// Programmatic dependent launch: wait for the preceding kernel's results /
// allow the next kernel to start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Named barrier over `threads` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also ORs a predicate over its participants: every
// thread gets the same answer.
__device__ __forceinline__ bool named_barrier_or(int id, int threads, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Optional timeline records: trace[0] counts records, record i occupies
// trace[1 + 4i .. 4 + 4i] = {tag, block, start ns, end ns} (%globaltimer).
// Kernels write one record per CTA when given a trace buffer.
// Optional timeline: trace[(launch * kTraceCtas + cta) * kTraceSlots + slot]
// receives %globaltimer at checkpoint `slot` of CTA `cta` of kernel launch
// `launch` (plain stores, no atomics, so tracing barely perturbs timing).
// Slot 0 is the CTA's start and slot 7 its end.
constexpr int kTraceLaunches = 256;
constexpr int kTraceCtas = 1024;
constexpr int kTraceSlots = 8;
__device__ __forceinline__ void trace_at(unsigned long long* trace, int launch, int slot) {
    if (!trace) return;
    const unsigned cta = blockIdx.x + gridDim.x * blockIdx.y;
    if (launch < 0 || launch >= kTraceLaunches || cta >= (unsigned)kTraceCtas) return;
    trace[((size_t)launch * kTraceCtas + cta) * kTraceSlots + slot] = global_timer_ns();
}

__device__ __forceinline__ bool candidate_better(float s, uint32_t i, float bs, uint32_t bi) {
    return s > bs || (s == bs && i < bi);
}

}  // namespace q4k
