// Prompt-prefill products on the tensor cores (tcgen05, sm_100a).
//
// The reference multiplies Q8-quantised activations with Q4_K/Q6_K weights
// in integer group dots (src/cuda/matmul.cu:24-84):
//   y[m][n] = sum_g xs[m][g] * (d[n] sc[n][g] sum q*xq - dmin[n] m[n][g] sum xq).
// The GEMM here keeps every factor that varies along K exact and applies the
// per-super-block weight scales outside the tensor cores:
//   A  = code * xs / row_scale, as fp16 hi + lo parts   [2][M][K]  prefill_quantise
//   B  = sc * q (Q4_K) or sc * (q - 32) (Q6_K), fp16     [N][K]     exact integers,
//        dequantised per tile here
//   P_b = (A_hi + A_lo) . B^T over super-block b         fp32, in TMEM
//   y  = row_scale * sum_b (d[n][b] P_b - dmin[n][b] sum_g m[n][g] gsum[m][g])
// where gsum[m][g] is the group's sum of A (prefill_quantise). A's hi + lo
// split carries 22 of its 24 bits and B is exact, so a product differs from
// the reference's integer arithmetic only by fp32 rounding (~1e-7), not by
// the 2^-11 of an fp16 operand: the layers of a prompt pass stay as close to
// the reference as its own arithmetic in another summation order.
//
// One CTA computes 128 activation rows x 128 output columns (SwiGLU: 64 gate
// and the same 64 up columns), K in 64-value stages, four per super-block:
//   warp 0     TMA producer of the A stages (hi and lo boxes, 128 rows x 64
//              fp16 each, 128-byte swizzle).
//   warp 1     TMEM allocation; one thread issues 2 x 4 tcgen05.mma.kind::f16
//              (M 128, N 128, K 16) per stage into the super-block's
//              accumulator (two, used in turn) and commits each stage back to
//              its empty barriers and each super-block to its accumulator.
//   warp 2     TMA producer of each super-block's raw weight rows (64-row
//              boxes; Q6_K planes swizzled), after asking L2 for the CTA's
//              whole weight slice.
//   warps 3-18 build each stage's B tile (K-major, 128-byte swizzled fp16;
//              thread: one row, 16 values) and each super-block's d / dmin /
//              mins, then read the previous super-block's accumulator out of
//              TMEM (tcgen05.ld) and fold it into fp32 registers; at the end
//              the row scale and store / add / SwiGLU.
// Every wait is bounded (kWaitLimitNs): on a timeout the kernel records an
// error bit, drains what it issued and releases its TMEM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "gemv_device.cuh"
#include "ops.h"
#include "q4k_device.cuh"
#include "q4k_format.h"
#include "q4k_internal.h"

namespace q4k {
namespace {

constexpr int BM = 128;                  // activation rows per CTA (MMA M)
constexpr int BN = 128;                  // output columns per CTA (MMA N, TMEM columns per accumulator)
constexpr int KS = 64;                   // K per stage: one 128-byte swizzle row of fp16
constexpr int kStagesA = 2;              // activation stages (hi + lo boxes each)
constexpr int kStagesB = 4;              // weight-operand stages (4 x 16 KB with 2 activation stages measured +1.8% batched decode, +2.7% prefill over 3 + 3)
constexpr int kRawStages = 2;            // raw weight super-block stages (the slice is prefetched to L2)
constexpr int kDeqWarps = 16;
constexpr int kThreads = (3 + kDeqWarps) * 32;  // A producer, MMA, raw producer, operand builders
constexpr int kBoxA = BM * KS * 2;                   // 16 KB: one hi or lo box
constexpr int kStageA = 2 * kBoxA;                   // 32 KB
constexpr int kStageB = BN * KS * 2;                 // 16 KB
constexpr int kRawChunksQ4 = 9;                      // 144 B
constexpr int kRawChunksQ6 = 14;                     // ql 128 B, qh 64 B, scales 16 B, d 16 B
constexpr int kRawStage = kRawChunksQ6 * BN * 16;    // 28 KB
// TMEM: two accumulator sets, super-blocks in turn; a set is the product P
// (BN columns) and the Q4_K min term Q (BN columns)
constexpr int kAccSet = 2 * BN;
constexpr int kAccCols = 2 * kAccSet;
// per super-block and tile column: d and dmin, as floats
constexpr int kSideFloats = BN * 2;
// min-term operands of one super-block (K = 16, 32-byte swizzle): the 8
// group sums of each activation row (hi and lo parts, then 8 zeros) and the
// 8 group mins of each weight row (then 8 zeros)
constexpr int kTile32 = BM * 32;  // 4 KB
constexpr int kOffB = kStagesA * kStageA;
constexpr int kOffRaw = kOffB + kStagesB * kStageB;
constexpr int kOffMin = kOffRaw + kRawStages * kRawStage;  // G hi, G lo, M
constexpr int kOffSide = kOffMin + 3 * kTile32;
constexpr int kOffBars = kOffSide + 2 * kSideFloats * 4;
constexpr int kSmemBytes = kOffBars + 256 + 1024;    // barriers, TMEM slot, alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory of one CTA");

struct Params {
    int nseg;
    int tile_start[4];  // first column tile of each segment; tile_start[nseg] = tiles
    int rows[3], type[3];
    int col_off[3];     // column of each segment in the split-K partials
    float* y[3];
    const uint8_t* w[3];
    int K, nb, M, ldy, epilogue;
    int splits;         // K ranges per tile (gridDim.z); > 1: partial sums to `partial`
    int ntot;           // columns of a partial row (all segments)
    float* partial;     // [splits][M][ntot]
    const float* row_scale;
    const float* gsum;  // [M][K / 32] group sums of A (the Q4_K min term)
    int* err;
};

// Raw weight maps per segment: Q4_K [0] = 144-byte rows; Q6_K [0] = ql
// (128 B, 128-byte swizzle), [1] = qh (64 B, 64-byte swizzle), [2] = 16-byte
// scale and d chunks. 64-row boxes.
constexpr int kWeightMaps = 3;
struct Maps {
    CUtensorMap a;
    CUtensorMap w[3][kWeightMaps];
};

// Raw stage layout (row r of the CTA's 128 weight rows):
//   Q4_K  r * 144                      the block (header chunk, 8 nibble chunks)
//   Q6_K  kQl + r * 128 (swizzled)     ql;  kQh + r * 64 (swizzled) qh;
//         kSc + r * 16                 scales; kD + r * 16  d chunk
constexpr int kQl = 0, kQh = 128 * BN, kSc = kQh + 64 * BN, kD = kSc + 16 * BN;
static_assert(kD + 16 * BN <= kRawStage, "raw stage layout");

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// The same for a K-major tile of 32-byte rows (one K = 16 step of fp16)
// with the 32-byte swizzle, 8-row groups 256 bytes apart.
__device__ __forceinline__ uint64_t sw32_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(256 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)6 << 61);
}

// Byte offset of 16-byte chunk c (0, 1) of row r in a 128-row x 32-byte
// tile with the 32-byte swizzle.
__device__ __forceinline__ uint32_t swz32(int r, int c) { return (uint32_t)(r * 32 + ((c ^ ((r >> 2) & 1)) << 4)); }

// Instruction descriptor of kind::f16: fp16 A and B (K-major), fp32 D,
// M = BM, N = BN.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint4 ld16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

__device__ __forceinline__ uint32_t byte_of(const uint4& v, int i) { return (word_of(v, i >> 2) >> (8 * (i & 3))) & 0xFFu; }

// Byte offset of 16-byte chunk c (0..7) of row r in a 128-row x 128-byte
// tile with the 128-byte swizzle (the layout TMA writes and the MMA reads).
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Issue the raw bytes of super-block b for this CTA's 128 weight rows.
__device__ __forceinline__ void load_raw(uint8_t* dst, const Params& p, const Maps& maps, int seg, int n0, bool pair,
                                         int type, int b, uint64_t* bar) {
    const int nb = p.nb;
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
        const CUtensorMap* m = maps.w[pair ? hh : seg];
        const int y = pair ? n0 : n0 + 64 * hh;
        if (type == Q4K_TYPE_Q4_K) {
            tma_load_2d(dst + hh * 64 * 144, &m[0], b * 144, y, bar);
        } else {
            tma_load_2d(dst + kQl + hh * 64 * 128, &m[0], b * 128, y, bar);
            tma_load_2d(dst + kQh + hh * 64 * 64, &m[1], nb * 128 + b * 64, y, bar);
            tma_load_2d(dst + kSc + hh * 64 * 16, &m[2], nb * 192 + b * 16, y, bar);
            tma_load_2d(dst + kD + hh * 64 * 16, &m[2], nb * 208 + (b >> 3) * 16, y, bar);
        }
    }
}

// The weight operand: 16 values (quarter p of K-stage j of the super-block)
// of weight row r into its row of the stage's B tile, as exact fp16
// integers in packed half arithmetic: each code byte q becomes the half
// 1024 + q by a byte permute with 0x64 (0x6400 | q), an exact subtraction
// gives q (Q6_K: q - 32), then
//   Q4_K  (embedding.cu:14-31): q * sc, at most 15 * 63 = 945
//   Q6_K  (embedding.cu:42-58): (q - 32) * sc, at most 32 * 32 = 1024
// in magnitude, so every product is exact; the super-block's d and dmin are
// applied to its accumulator (block_side, read_out).
// Values k = 16p .. 16p+15 of the stage: 16-byte chunks 2p and 2p+1 of the
// row's 128 bytes.
__device__ __forceinline__ __half2 half2_bits(uint32_t v) { return *reinterpret_cast<const __half2*>(&v); }
__device__ __forceinline__ uint32_t bits_half2(__half2 v) { return *reinterpret_cast<const uint32_t*>(&v); }

// 6-bit scale (min = false) or min (min = true) of 32-value group g of a
// Q4_K block whose first 16 bytes are `head` (matmul.cu:40-47).
__device__ __forceinline__ uint32_t q4_field(const uint4& head, int g, bool min) {
    if (g < 4) return byte_of(head, (min ? 8 : 4) + g) & 63;
    return min ? (byte_of(head, 8 + g) >> 4) | ((byte_of(head, 4 + g) >> 6) << 4)
               : (byte_of(head, 8 + g) & 15) | ((byte_of(head, g) >> 6) << 4);
}

// The 4 scales a builder thread (weight row r, quarter p of each stage)
// applies in the 4 stages j of a super-block, decoded once per super-block:
// Q4_K group 2j + (p >> 1)'s 6-bit scale (matmul.cu:40-47: groups 0-3 from
// bytes 4-7, groups 4-7 from the low nibbles of bytes 12-15 and the top two
// bits of bytes 4-7), Q6_K the int8 scale 4j + p of the 16 (embedding.cu:42-58).
__device__ __forceinline__ void stage_scales(const uint8_t* raw, int type, int r, int p, __half2 (&sc)[4]) {
    if (type == Q4K_TYPE_Q4_K) {
        const uint4 head = ld16(raw + r * 144);
        const uint32_t lo = head.y & 0x3f3f3f3fu;                                       // groups 0-3
        const uint32_t hi = (head.w & 0x0f0f0f0fu) | ((head.y >> 2) & 0x30303030u);     // groups 4-7
        const int h = p >> 1;
        sc[0] = __float2half2_rn((float)((lo >> (8 * h)) & 0xffu));
        sc[1] = __float2half2_rn((float)((lo >> (8 * (2 + h))) & 0xffu));
        sc[2] = __float2half2_rn((float)((hi >> (8 * h)) & 0xffu));
        sc[3] = __float2half2_rn((float)((hi >> (8 * (2 + h))) & 0xffu));
    } else {
        const uint4 scw = ld16(raw + kSc + r * 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[j] = __float2half2_rn((float)(int8_t)byte_of(scw, 4 * j + p));
    }
}

__device__ __forceinline__ void dequant_q4(const uint8_t* raw, uint8_t* bt, int r, int p, int j, __half2 sc2) {
    const uint8_t* blk = raw + r * 144;
    const __half2 k1024 = half2_bits(0x64006400u);
    // nibbles of values 16(p&1) .. +15 of group g: bytes 16 + 32j + 16(p&1) .., low or high nibble
    const uint4 nb = ld16(blk + 16 * (1 + 2 * j + (p & 1)));
    const int shift = 4 * (p >> 1);
    uint32_t o[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t nib = (word_of(nb, t) >> shift) & 0x0F0F0F0Fu;
        const __half2 q01 = __hsub2(half2_bits(__byte_perm(nib, 0x64646464u, 0x5140u)), k1024);
        const __half2 q23 = __hsub2(half2_bits(__byte_perm(nib, 0x64646464u, 0x7362u)), k1024);
        o[2 * t] = bits_half2(__hmul2(q01, sc2));
        o[2 * t + 1] = bits_half2(__hmul2(q23, sc2));
    }
    *reinterpret_cast<uint4*>(bt + swz(r, 2 * p)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(bt + swz(r, 2 * p + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
}

__device__ __forceinline__ void dequant_q6(const uint8_t* raw, uint8_t* bt, int r, int p, int j, __half2 sc2) {
    // ql: bytes 64(j>>1) + 16p .. ; qh: bytes 32(j>>1) + 16(p&1) ..
    const int cl = (j >> 1) * 4 + p, ch = (j >> 1) * 2 + (p & 1);  // ql chunk 0..7, qh chunk 0..3
    const uint4 lq = ld16(raw + kQl + r * 128 + ((cl ^ (r & 7)) << 4));
    const uint4 hq = ld16(raw + kQh + r * 64 + ((ch ^ ((r >> 1) & 3)) << 4));
    const int s4 = 4 * (j & 1), s2 = 2 * (2 * (j & 1) + (p >> 1));
    const __half2 k1056 = half2_bits(0x64206420u);  // 1024 + 32
    uint32_t o[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t q = ((word_of(lq, t) >> s4) & 0x0F0F0F0Fu) | (((word_of(hq, t) >> s2) & 0x03030303u) << 4);
        const __half2 q01 = __hsub2(half2_bits(__byte_perm(q, 0x64646464u, 0x5140u)), k1056);
        const __half2 q23 = __hsub2(half2_bits(__byte_perm(q, 0x64646464u, 0x7362u)), k1056);
        o[2 * t] = bits_half2(__hmul2(q01, sc2));
        o[2 * t + 1] = bits_half2(__hmul2(q23, sc2));
    }
    *reinterpret_cast<uint4*>(bt + swz(r, 2 * p)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(bt + swz(r, 2 * p + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
}

// Per-column factors of super-block b for tile column r (weight row r of
// the raw stage): side[r] = d, side[BN + r] = dmin; for Q4_K also row r of
// the min-term operands: the 8 group mins of weight row r (M tile) and the 8
// group sums g8 of activation row r (G tiles, hi and lo parts), each
// followed by 8 zeros (the MMA's K is 16).
__device__ __forceinline__ void block_side(const uint8_t* raw, float* side, uint8_t* mins, int r, int type, int b,
                                           const float (&g8)[8]) {
    if (type == Q4K_TYPE_Q4_K) {
        const uint4 head = ld16(raw + r * 144);
        side[r] = half_bits_to_float(head.x & 0xFFFFu);
        side[BN + r] = half_bits_to_float(head.x >> 16);
        uint32_t mw[4], hw[4], lw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            mw[k] = bits_half2(
                __floats2half2_rn((float)q4_field(head, 2 * k, true), (float)q4_field(head, 2 * k + 1, true)));
            const __half2 hi = __floats2half2_rn(g8[2 * k], g8[2 * k + 1]);
            const float2 hf = __half22float2(hi);
            hw[k] = bits_half2(hi);
            lw[k] = bits_half2(__floats2half2_rn(g8[2 * k] - hf.x, g8[2 * k + 1] - hf.y));
        }
        const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
        uint8_t* gh = mins;
        uint8_t* gl = mins + kTile32;
        uint8_t* mt = mins + 2 * kTile32;
        *reinterpret_cast<uint4*>(mt + swz32(r, 0)) = make_uint4(mw[0], mw[1], mw[2], mw[3]);
        *reinterpret_cast<uint4*>(mt + swz32(r, 1)) = zero;
        *reinterpret_cast<uint4*>(gh + swz32(r, 0)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(gh + swz32(r, 1)) = zero;
        *reinterpret_cast<uint4*>(gl + swz32(r, 0)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        *reinterpret_cast<uint4*>(gl + swz32(r, 1)) = zero;
    } else {
        const uint4 dch = ld16(raw + kD + r * 16);
        side[r] = half_bits_to_float((word_of(dch, (b & 7) >> 1) >> (16 * (b & 1))) & 0xFFFFu);
        side[BN + r] = 0.0f;
    }
}

// Lane 0 polls the barrier (one poller per warp keeps the barrier traffic
// low); once it has seen the phase complete, every lane observes it with one
// try_wait that succeeds at once.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    bool ok = true;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait_bounded(bar, parity, err, code);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) (void)mbar_try_wait(bar, parity);
    return ok;
}

// Folds super-block b's accumulators (TMEM columns acc_addr.. of this warp's
// lanes: P, then Q BN columns on) into the thread's 32 running sums of row m,
// columns c0 .. c0+31:
//   acc += d[n] P[m][n] - dmin[n] Q[m][n]   (Q = sum_g min[n][g] gsum[m][g]; Q4_K)
//   acc += d[n] P[m][n]                     (Q6_K)
__device__ __forceinline__ void read_out(uint32_t acc_addr, const float* side, int c0, bool q4, float (&acc)[32]) {
    float v[32];
    tmem_ld32(acc_addr, v);
    const float4* d4 = reinterpret_cast<const float4*>(side + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 d = d4[i];
        acc[4 * i] = fmaf(d.x, v[4 * i], acc[4 * i]);
        acc[4 * i + 1] = fmaf(d.y, v[4 * i + 1], acc[4 * i + 1]);
        acc[4 * i + 2] = fmaf(d.z, v[4 * i + 2], acc[4 * i + 2]);
        acc[4 * i + 3] = fmaf(d.w, v[4 * i + 3], acc[4 * i + 3]);
    }
    if (q4) {
        tmem_ld32(acc_addr + BN, v);
        const float4* m4 = reinterpret_cast<const float4*>(side + BN + c0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 m = m4[i];
            acc[4 * i] = fmaf(-m.x, v[4 * i], acc[4 * i]);
            acc[4 * i + 1] = fmaf(-m.y, v[4 * i + 1], acc[4 * i + 1]);
            acc[4 * i + 2] = fmaf(-m.z, v[4 * i + 2], acc[4 * i + 2]);
            acc[4 * i + 3] = fmaf(-m.w, v[4 * i + 3], acc[4 * i + 3]);
        }
    }
    tc_fence_before();
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ Params p, const __grid_constant__ Maps maps) {
    extern __shared__ uint8_t smem_dyn[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
    uint64_t* a_full = bars;
    uint64_t* a_empty = a_full + kStagesA;
    uint64_t* b_full = a_empty + kStagesA;
    uint64_t* b_empty = b_full + kStagesB;
    uint64_t* raw_full = b_empty + kStagesB;
    uint64_t* raw_empty = raw_full + kRawStages;
    uint64_t* acc_full = raw_empty + kRawStages;  // [2]: a super-block's MMAs are done
    uint64_t* acc_empty = acc_full + 2;           // [2]: its accumulators have been read out
    uint64_t* min_full = acc_empty + 2;           // the min-term operands of a super-block are written
    uint64_t* min_done = min_full + 1;            // the min-term MMAs of a super-block are done
    uint64_t* done = min_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    float* sides = reinterpret_cast<float*>(smem + kOffSide);  // [2][kSideFloats]
    uint8_t* mins = smem + kOffMin;                             // G hi, G lo, M tiles

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool pair = p.epilogue == EPI_SWIGLU;
    // Programmatic dependent launch: the next kernel (the split-K reduce or
    // the next product's quantisation) may be scheduled once every CTA is
    // running; it waits for this grid itself. Here only the activation
    // operand, the group sums and the outputs depend on earlier kernels, so
    // set-up, the weight stream and the first weight operands run before
    // griddepcontrol.wait, overlapping the preceding kernel.
    pdl_launch_dependents();
    const int tile = blockIdx.y, m0 = blockIdx.x * BM;
    int seg = 0;
    while (seg + 1 < p.nseg && tile >= p.tile_start[seg + 1]) ++seg;
    if (pair) seg = 0;
    const int n0 = (tile - p.tile_start[seg]) * (pair ? BN / 2 : BN);
    const int type = p.type[seg];
    // this CTA's super-blocks [b_begin, b_end) of the K range
    const int split = blockIdx.z;
    const int b_begin = split * p.nb / p.splits, b_end = (split + 1) * p.nb / p.splits;
    const int nblk = b_end - b_begin;
    const int nsteps = nblk * 4;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStagesA; ++i) {
            mbar_init(a_full + i, 1);
            mbar_init(a_empty + i, 1);
        }
        for (int i = 0; i < kStagesB; ++i) {
            mbar_init(b_full + i, kDeqWarps);
            mbar_init(b_empty + i, 1);
        }
        for (int i = 0; i < kRawStages; ++i) {
            mbar_init(raw_full + i, 1);
            mbar_init(raw_empty + i, kDeqWarps);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(acc_full + i, 1);
            mbar_init(acc_empty + i, kDeqWarps);
        }
        mbar_init(min_full, kDeqWarps);
        mbar_init(min_done, 1);
        mbar_init(done, 1);
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kAccCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- producer of the activation stages (hi and lo boxes)
            pdl_wait();  // the activation operand is the preceding kernel's output
            int issued = 0;
            for (int s = 0; s < nsteps; ++s) {
                const int st = s % kStagesA;
                if (!mbar_wait_bounded(a_empty + st, ((s / kStagesA) & 1) ^ 1, p.err, ERR_WAIT_TIMEOUT_EMPTY)) break;
                mbar_arrive_expect_tx(a_full + st, kStageA);
                const int x = (4 * b_begin + s) * KS;
                tma_load_3d(smem + st * kStageA, &maps.a, x, m0, 0, a_full + st);
                tma_load_3d(smem + st * kStageA + kBoxA, &maps.a, x, m0, 1, a_full + st);
                ++issued;
            }
            // every copy issued has landed before the CTA can exit (the last
            // use of each stage is the latest phase of its barrier)
            for (int s = issued - 1; s >= 0 && s >= issued - kStagesA; --s)
                mbar_wait_bounded(a_full + s % kStagesA, (s / kStagesA) & 1, p.err, ERR_WAIT_TIMEOUT_FULL);
        }
        __syncwarp();
    } else if (warp == 2) {
        if (lane == 0) {
            // ---------------- producer of the raw weight stages (a warp of
            // its own: two spinning producers in one warp's divergent lanes
            // starve each other)
            const uint32_t raw_bytes = (type == Q4K_TYPE_Q4_K ? kRawChunksQ4 : kRawChunksQ6) * BN * 16;
            int issued = 0;
            for (int i = 0; i < nblk; ++i) {
                const int rs = i % kRawStages;
                if (!mbar_wait_bounded(raw_empty + rs, ((i / kRawStages) & 1) ^ 1, p.err, ERR_WAIT_TIMEOUT_EMPTY))
                    break;
                mbar_arrive_expect_tx(raw_full + rs, raw_bytes);
                load_raw(smem + kOffRaw + rs * kRawStage, p, maps, seg, n0, pair, type, b_begin + i, raw_full + rs);
                ++issued;
            }
            for (int i = issued - 1; i >= 0 && i >= issued - kRawStages; --i)
                mbar_wait_bounded(raw_full + i % kRawStages, (i / kRawStages) & 1, p.err, ERR_WAIT_TIMEOUT_FULL);
        } else {
            // the rest of the warp asks L2 for this CTA's whole weight slice up
            // front, so the raw stages find it there
            const int row_bytes = (int)q4k_device_row_bytes(type, p.K);
            for (int r = lane - 1; r < BN; r += 31) {
                const int hh = r >> 6;
                const int wrow = pair ? n0 + (r & 63) : n0 + r;
                const int rows = p.rows[pair ? hh : seg];
                if (wrow >= rows) continue;
                const uint8_t* w = (pair ? p.w[hh] : p.w[seg]) + (size_t)wrow * row_bytes;
                if (type == Q4K_TYPE_Q4_K) {
                    l2_prefetch_bulk(w + b_begin * 144, (uint32_t)nblk * 144);
                } else {
                    l2_prefetch_bulk(w + b_begin * 128, (uint32_t)nblk * 128);
                    l2_prefetch_bulk(w + p.nb * 128 + b_begin * 64, (uint32_t)nblk * 64);
                    l2_prefetch_bulk(w + p.nb * 192 + b_begin * 16, (uint32_t)nblk * 16);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issue: super-block i accumulates in set i & 1
            // (P, then Q BN columns on), once the read-out of super-block
            // i - 2 freed it
            const bool q4 = type == Q4K_TYPE_Q4_K;
            bool ok = true;
            for (int i = 0; i < nblk && ok; ++i) {
                const uint32_t acc = tmem + (uint32_t)((i & 1) * kAccSet);
                if (i >= 2 && !mbar_wait_bounded(acc_empty + (i & 1), ((i - 2) >> 1) & 1, p.err,
                                                 ERR_WAIT_TIMEOUT_EMPTY)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int j = 0; j < 4; ++j) {
                    const int s = 4 * i + j;
                    const int sa = s % kStagesA, sb = s % kStagesB;
                    if (!mbar_wait_bounded(a_full + sa, (s / kStagesA) & 1, p.err, ERR_WAIT_TIMEOUT_FULL) ||
                        !mbar_wait_bounded(b_full + sb, (s / kStagesB) & 1, p.err, ERR_WAIT_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_addr(smem + sa * kStageA);
                    const uint32_t b_addr = smem_addr(smem + kOffB + sb * kStageB);
#pragma unroll
                    for (int kk = 0; kk < KS / 16; ++kk) {
                        const uint64_t bd = sw128_desc(b_addr + kk * 32);
                        mma_f16(acc, sw128_desc(a_addr + kk * 32), bd, (j | kk) != 0);
                        mma_f16(acc, sw128_desc(a_addr + kBoxA + kk * 32), bd, 1u);
                    }
                    tc_commit(a_empty + sa);
                    tc_commit(b_empty + sb);
                }
                if (ok && q4) {
                    // Q = G . M^T over the super-block's 8 groups (K = 16 with
                    // 8 zeros), the group sums' hi and lo parts in turn
                    if (!mbar_wait_bounded(min_full, i & 1, p.err, ERR_WAIT_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t md = sw32_desc(smem_addr(mins + 2 * kTile32));
                    mma_f16(acc + BN, sw32_desc(smem_addr(mins)), md, 0u);
                    mma_f16(acc + BN, sw32_desc(smem_addr(mins + kTile32)), md, 1u);
                    tc_commit(min_done);
                }
                if (ok) tc_commit(acc_full + (i & 1));
            }
            tc_commit(done);  // also on an early exit: the epilogue and the TMEM release wait for it
            mbar_wait_bounded(done, 0, p.err, ERR_WAIT_TIMEOUT_FULL);
        }
        __syncwarp();
    } else {
        // ---------------- weight operands and accumulator read-outs
        const int t = (warp - 3) * 32 + lane, r = t & (BN - 1), part = t >> 7;
        const int quad = warp & 3, cg = (warp - 3) >> 2;  // TMEM lanes 32 quad.., columns 32 cg..
        const int row = 32 * quad + lane, m = m0 + row;
        const int c0 = 32 * cg;
        const bool q4 = type == Q4K_TYPE_Q4_K;
        const uint32_t tlane = tmem + ((uint32_t)(32 * quad) << 16);
        const int groups = p.K / 32;
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
        // group sums of activation row r (this thread's min-term row when
        // part == 0); rows past M read row 0's, whose results are never stored
        const float* grow = p.gsum + (size_t)(m0 + r < p.M ? m0 + r : 0) * groups + 8 * b_begin;
        // super-block i's accumulators are read out after super-block i + 1's
        // operands are built, so that the tensor cores always have work
        auto fold = [&](int i) {
            if (!warp_wait(acc_full + (i & 1), (i >> 1) & 1, p.err, ERR_WAIT_TIMEOUT_FULL)) return false;
            tc_fence_after();
            read_out(tlane + (uint32_t)((i & 1) * kAccSet + c0), sides + (i & 1) * kSideFloats, c0, q4, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + (i & 1));
            return true;
        };
        // A wait that gives up (bounded) stops this warp's work; the warps
        // agree at every super-block's barrier, so all leave the loop together.
        // Stage j of super-block i into its ring slot of B tiles.
        __half2 sc4[4];  // this super-block's 4 scales of this thread (stage_scales)
        auto build = [&](const uint8_t* raw, int i, int j) {
            const int s = 4 * i + j, st = s % kStagesB;
            if (!warp_wait(b_empty + st, ((s / kStagesB) & 1) ^ 1, p.err, ERR_WAIT_TIMEOUT_EMPTY)) return false;
            uint8_t* bt = smem + kOffB + st * kStageB;
            if (q4)
                dequant_q4(raw, bt, r, part, j, sc4[j]);
            else
                dequant_q6(raw, bt, r, part, j, sc4[j]);
            fence_proxy_async();  // generic stores -> the MMA's async-proxy reads
            __syncwarp();
            if (lane == 0) mbar_arrive(b_full + st);
            return true;
        };
        // Super-block i: its first two stages are built, then (every warp
        // past super-block i - 1) super-block i - 1's accumulators are read
        // out while the tensor cores work on those stages, then the last two
        // stages and super-block i's side factors and min-term tiles.
        bool good = true, ok = true;
        for (int i = 0; i < nblk; ++i) {
            const int rs = i % kRawStages, b = b_begin + i;
            if (good) good = warp_wait(raw_full + rs, (i / kRawStages) & 1, p.err, ERR_WAIT_TIMEOUT_FULL);
            const uint8_t* raw = smem + kOffRaw + rs * kRawStage;
            if (good) stage_scales(raw, type, r, part, sc4);
            for (int j = 0; j < 2 && good; ++j) good = build(raw, i, j);
            // every warp has written super-block i - 1's side factors and read
            // out super-block i - 2
            if (named_barrier_or(2, kDeqWarps * 32, !good)) {
                ok = false;
                break;
            }
            if (i >= 1) good = fold(i - 1);
            // this super-block's 8 group sums, loaded while the last stages are built
            if (i == 0) pdl_wait();  // the group sums come from the preceding kernel
            float g8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (q4 && part == 0) {
                const float4 u = __ldg(reinterpret_cast<const float4*>(grow + 8 * i));
                const float4 w = __ldg(reinterpret_cast<const float4*>(grow + 8 * i + 4));
                g8[0] = u.x, g8[1] = u.y, g8[2] = u.z, g8[3] = u.w;
                g8[4] = w.x, g8[5] = w.y, g8[6] = w.z, g8[7] = w.w;
            }
            for (int j = 2; j < 4 && good; ++j) good = build(raw, i, j);
            // side factors: buffer i & 1 was last read by super-block i - 2's
            // read-out (before the barrier above); the min-term tiles are
            // single, so super-block i - 1's MMAs on them must be done
            if (part == 0) {
                if (q4 && i >= 1 && good) good = warp_wait(min_done, (i - 1) & 1, p.err, ERR_WAIT_TIMEOUT_FULL);
                block_side(raw, sides + (i & 1) * kSideFloats, mins, r, type, b, g8);
                fence_proxy_async();  // generic stores -> the MMA's async-proxy reads
            }
            __syncwarp();
            if (lane == 0) {
                if (q4) mbar_arrive(min_full);
                mbar_arrive(raw_empty + rs);
            }
        }
        // the last super-block's side factors are visible to every warp
        if (named_barrier_or(2, kDeqWarps * 32, !(ok && good))) ok = false;
        pdl_wait();  // (again, for a CTA with no super-blocks) before the outputs are written
        if (ok && nblk > 0) ok = fold(nblk - 1);
        warp_wait(done, 0, p.err, ERR_WAIT_TIMEOUT_FULL);
        tc_fence_after();
        const float rsc = m < p.M ? p.row_scale[m] : 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] *= rsc;
        const int rows = p.rows[seg];
        // the stage buffers are free once `done` has fired: each warp turns
        // its 32 x 32 block around in shared memory so that the global
        // stores are whole row segments
        float* st = reinterpret_cast<float*>(smem) + (warp - 3) * 32 * 33;
        if (pair && p.splits == 1) {
            // SwiGLU: gate columns 0..63 and up columns 64..127 of the tile
            // are held by different warps; the up warps hand theirs over
            float* up = reinterpret_cast<float*>(smem + kOffB) + (size_t)(32 * quad + lane) * 65;
            named_barrier(2, kDeqWarps * 32);
            if (cg >= 2)
#pragma unroll
                for (int i = 0; i < 32; ++i) up[32 * (cg - 2) + i] = acc[i];
            named_barrier(2, kDeqWarps * 32);
            if (cg < 2)
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float gv = acc[i], uv = up[32 * cg + i];
                    acc[i] = (gv / (1.0f + expf(-gv))) * uv;  // silu_multiply.cu:9-10
                }
        }
        const bool active = !(pair && p.splits == 1) || cg < 2;
        if (ok && active) {
#pragma unroll
            for (int i = 0; i < 32; ++i) st[lane * 33 + i] = acc[i];
            __syncwarp();
            // a SwiGLU tile's columns 0..63 are gate rows n0.., 64..127 the same up rows
            const int pseg = pair ? (cg >> 1) : seg;
            const int n = n0 + (pair ? 32 * (cg & 1) : c0) + lane;
            const bool col_ok = n < rows;
            for (int rr = 0; rr < 32; ++rr) {
                const int mr = m0 + 32 * quad + rr;
                if (mr >= p.M || !col_ok) continue;
                const float a = st[rr * 33 + lane];
                if (p.splits > 1) {
                    // this K range's share, reduced in a fixed order by split_reduce_kernel
                    p.partial[((size_t)split * p.M + mr) * p.ntot + p.col_off[pseg] + n] = a;
                } else {
                    float* out = p.y[pair ? 0 : seg] + (size_t)mr * p.ldy + n;
                    if (p.epilogue == EPI_ADD)
                        *out += a;
                    else
                        *out = a;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kAccCols);
    }
}

// y (=, or += for EPI_ADD) the sum of the split-K partials, in split order.
// Each thread sums V consecutive columns of one segment (V = 4 when every
// column offset, width and row stride is a multiple of 4); the segments are
// picked by selects, so the arguments stay out of local memory.
struct ReduceArgs {
    const float* partial;
    int splits, M, ntot, nseg, ldy, add;
    int off1, off2;  // first column of segments 1 and 2 (ntot when absent)
    float *y0, *y1, *y2;
};

template <int V>
__global__ void __launch_bounds__(256) split_reduce_kernel(const ReduceArgs r) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * V;
    if (i >= (size_t)r.M * r.ntot) return;
    const int m = (int)(i / r.ntot), c = (int)(i % r.ntot);
    float acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0.0f;
    for (int z = 0; z < r.splits; ++z) {
        const float* src = r.partial + ((size_t)z * r.M + m) * r.ntot + c;
        if constexpr (V == 4) {
            const float4 t = *reinterpret_cast<const float4*>(src);
            acc[0] += t.x;
            acc[1] += t.y;
            acc[2] += t.z;
            acc[3] += t.w;
        } else {
            acc[0] += *src;
        }
    }
    const bool s2 = c >= r.off2, s1 = c >= r.off1;
    float* yb = s2 ? r.y2 : s1 ? r.y1 : r.y0;
    const int col = c - (s2 ? r.off2 : s1 ? r.off1 : 0);
    float* out = yb + (size_t)m * r.ldy + col;
#pragma unroll
    for (int v = 0; v < V; ++v) out[v] = r.add ? out[v] + acc[v] : acc[v];
}

// SwiGLU split-K: y = silu(sum of the gate partials) * (sum of the up
// partials), each sum in split order (gate columns 0..rows-1 of a partial
// row, up columns rows..2 rows-1).
__global__ void __launch_bounds__(256) split_reduce_swiglu_kernel(const ReduceArgs r) {
    pdl_launch_dependents();
    pdl_wait();
    const int rows = r.off1;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)r.M * rows) return;
    const int m = (int)(i / rows), n = (int)(i % rows);
    float gs = 0.0f, us = 0.0f;
    for (int z = 0; z < r.splits; ++z) {
        const float* src = r.partial + ((size_t)z * r.M + m) * r.ntot;
        gs += src[n];
        us += src[rows + n];
    }
    r.y0[(size_t)m * r.ldy + n] = (gs / (1.0f + expf(-gs))) * us;  // silu_multiply.cu:9-10
}

// Q8 codes of each row (matmul.cu:8-22) as the GEMM's A operand: the
// value v = code * (scale / row_scale) in fp32, stored as fp16 hi = fp16(v)
// and lo = fp16(v - hi) (hi + lo carry 22 of v's 24 bits), and each 32-value
// group's sum of v (the Q4_K min term). One CTA of NT threads per row;
// thread t holds elements NT i + t, so warp w's lanes hold 32-value group
// (NT / 32) i + w at step i and the row is read once. Wide rows take 512 or
// 1024 threads: a row's chain of loads, two CTA-wide reductions and stores
// is latency-bound, and more threads per row shorten each thread's share
// (a 64-row batch keeps only 64 SMs busy).
template <int NT, int kSteps>
__global__ void __launch_bounds__(NT) prefill_quantise_kernel(const float* x, int ldx, const float* gamma, float eps,
                                                              int K, __half* a_hi, __half* a_lo, float* gsum,
                                                              float* row_scale) {
    constexpr int NW = NT / 32;
    const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_launch_dependents();
    pdl_wait();
    const float* xr = x + (size_t)m * ldx;
    __shared__ float red[NW];
    float v[kSteps];
#pragma unroll
    for (int i = 0; i < kSteps; ++i) v[i] = NT * i + tid < K ? xr[NT * i + tid] : 0.0f;
    if (gamma) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < kSteps; ++i) ss += v[i] * v[i];
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float total = 0.0f;
#pragma unroll
        for (int i = 0; i < NW; ++i) total += red[i];
        const float inv = rsqrtf(total / (float)K + eps);  // rms_norm.cu:17
#pragma unroll
        for (int i = 0; i < kSteps; ++i)
            if (NT * i + tid < K) v[i] = (v[i] * inv) * gamma[NT * i + tid];  // rms_norm.cu:19
        __syncthreads();
    }
    float am[kSteps];
    float wmax = 0.0f;
#pragma unroll
    for (int i = 0; i < kSteps; ++i) {
        am[i] = warp_max(fabsf(v[i]));
        wmax = fmaxf(wmax, am[i]);
    }
    if (lane == 0) red[warp] = wmax;
    __syncthreads();
    float rmax = 0.0f;
#pragma unroll
    for (int i = 0; i < NW; ++i) rmax = fmaxf(rmax, red[i]);
    const float S = gemv_dev::q8_scale(rmax);  // the largest group scale (matmul.cu:18)
#pragma unroll
    for (int i = 0; i < kSteps; ++i) {
        // K is a multiple of 256, so a warp's 32 elements are all in or all out
        if (NT * i + tid >= K) break;
        const bool defined = gemv_dev::q8_codes_defined(am[i]);
        const int8_t code = defined ? gemv_dev::q8_code_r(v[i], gemv_dev::recip_refined(am[i])) : 0;
        const float r = S > 0.0f ? __fdiv_rn(gemv_dev::q8_scale(am[i]), S) : 0.0f;
        const float val = (float)code * r;
        const __half hi = __float2half_rn(val);
        const size_t at = (size_t)m * K + NT * i + tid;
        a_hi[at] = hi;
        a_lo[at] = __float2half_rn(val - __half2float(hi));
        // the group's code sum is an exact integer: one rounding for its value
        int cs = code;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
        if (lane == 0) gsum[(size_t)m * (K / 32) + NW * i + warp] = r * (float)cs;
    }
    if (tid == 0) row_scale[m] = S;
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

cudaError_t prefill_quantise(const float* x, int ldx, const float* gamma, float eps, int M, int K, uint16_t* a,
                             int a_rows, float* gsum, float* row_scale, cudaStream_t s) {
    if (M <= 0 || K <= 0 || K % 256 || K > 10240 || ldx < K || !x || !a || !gsum || !row_scale ||
        a_rows < M)
        return cudaErrorInvalidValue;
    __half* hi = reinterpret_cast<__half*>(a);
    __half* lo = hi + (size_t)a_rows * K;
    if (K <= 2560)
        return launch_pdl(prefill_quantise_kernel<512, 5>, dim3(M), dim3(512), 0, s, x, ldx, gamma, eps, K, hi, lo,
                          gsum, row_scale);
    if (K <= 4096)
        return launch_pdl(prefill_quantise_kernel<512, 8>, dim3(M), dim3(512), 0, s, x, ldx, gamma, eps, K, hi, lo,
                          gsum, row_scale);
    return launch_pdl(prefill_quantise_kernel<1024, 10>, dim3(M), dim3(1024), 0, s, x, ldx, gamma, eps, K, hi, lo,
                      gsum, row_scale);
}

cudaError_t make_weight_map(const uint8_t* w, int type, int K, int rows, KvTensorMap* out) {
    static_assert(sizeof(KvTensorMap) == sizeof(CUtensorMap), "tensor map storage size");
    const EncodeTiled enc = reinterpret_cast<EncodeTiled>(tensor_map_encoder());
    if (!enc) return cudaErrorNotSupported;
    if (!w || reinterpret_cast<uintptr_t>(w) % 16 || rows <= 0 || K <= 0 || K % 256 ||
        (type != Q4K_TYPE_Q4_K && type != Q4K_TYPE_Q6_K))
        return cudaErrorInvalidValue;
    const cuuint64_t row_bytes = q4k_device_row_bytes(type, K);
    const cuuint64_t dims[2] = {row_bytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t estr[2] = {1, 1};
    struct {
        cuuint32_t width;
        CUtensorMapSwizzle swizzle;
    } kinds[kWeightMaps] = {{144, CU_TENSOR_MAP_SWIZZLE_NONE}, {0, CU_TENSOR_MAP_SWIZZLE_NONE},
                            {0, CU_TENSOR_MAP_SWIZZLE_NONE}};
    if (type == Q4K_TYPE_Q6_K) {
        kinds[0] = {128, CU_TENSOR_MAP_SWIZZLE_128B};
        kinds[1] = {64, CU_TENSOR_MAP_SWIZZLE_64B};
        kinds[2] = {16, CU_TENSOR_MAP_SWIZZLE_NONE};
    }
    for (int i = 0; i < kWeightMaps; ++i) {
        CUtensorMap map;
        std::memset(&map, 0, sizeof map);
        if (kinds[i].width) {
            const cuuint32_t box[2] = {kinds[i].width, 64};
            if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, kinds[i].swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return cudaErrorInvalidValue;
        }
        std::memcpy(&out[i], &map, sizeof map);
    }
    return cudaSuccess;
}

cudaError_t make_act_map(const uint16_t* a, int K, int rows, KvTensorMap* out) {
    const EncodeTiled enc = reinterpret_cast<EncodeTiled>(tensor_map_encoder());
    if (!enc) return cudaErrorNotSupported;
    if (!a || reinterpret_cast<uintptr_t>(a) % 16 || rows <= 0 || K <= 0 || K % 256) return cudaErrorInvalidValue;
    // [2][rows][K]: the hi plane, then the lo plane
    const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, 2};
    const cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)K * 2 * (cuuint64_t)rows};
    const cuuint32_t box[3] = {KS, BM, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMap map;
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t*>(a), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    std::memcpy(out, &map, sizeof map);
    return cudaSuccess;
}

namespace {
// K splits for `tiles` column tiles of M rows and nb super-blocks: with one
// CTA per SM, s splits cost about ceil(ctas * s / SMs) waves of
// (ceil(nb / s) + 2) super-blocks (2 for a CTA's set-up and epilogue), plus
// one for the reduce; the cheapest s whose partials fit `partial_floats`
// wins, each split keeping at least two super-blocks.
int gemm_splits(int M, int tiles, int nb, int ntot, size_t partial_floats) {
    const long long ctas = (long long)((M + BM - 1) / BM) * tiles, sms = sm_count();
    long long best = (ctas + sms - 1) / sms * (nb + 2);
    int splits = 1;
    for (int sp = 2; sp <= std::min(16, nb / 2); ++sp) {
        if ((size_t)sp * M * ntot > partial_floats) break;
        const long long cost = (ctas * sp + sms - 1) / sms * ((nb + sp - 1) / sp + 2) + 1;
        if (cost < best) {
            best = cost;
            splits = sp;
        }
    }
    return splits;
}
}  // namespace

size_t prefill_gemm_partial_floats(const PrefillGemmArgs& g) {
    const bool pair = g.epilogue == EPI_SWIGLU;
    if (g.nseg < 1 || g.nseg > 3 || g.K <= 0 || g.K % 256 || g.M <= 0) return 0;
    int tiles = 0, ntot = 0;
    for (int i = 0; i < g.nseg; ++i) {
        ntot += g.seg[i].rows;
        if (!pair || i == 0) tiles += (g.seg[i].rows + (pair ? BN / 2 : BN) - 1) / (pair ? BN / 2 : BN);
    }
    const int sp = gemm_splits(g.M, tiles, g.K / 256, ntot, (size_t)-1);
    return sp > 1 ? (size_t)sp * g.M * ntot : 0;
}

cudaError_t prefill_gemm(const PrefillGemmArgs& g, cudaStream_t s) {
    const bool pair = g.epilogue == EPI_SWIGLU;
    if (g.nseg < 1 || g.nseg > 3 || g.K <= 0 || g.K % 256 || g.M <= 0 || g.ldy <= 0 || !g.a || !g.row_scale || !g.gsum ||
        (g.epilogue != EPI_STORE && g.epilogue != EPI_ADD && !pair))
        return cudaErrorInvalidValue;
    if (pair && (g.nseg != 2 || g.seg[0].type != g.seg[1].type || g.seg[0].rows != g.seg[1].rows))
        return cudaErrorInvalidValue;
    Params p{};
    Maps maps;
    p.nseg = g.nseg;
    p.K = g.K;
    p.nb = g.K / 256;
    p.M = g.M;
    p.ldy = g.ldy;
    p.epilogue = g.epilogue;
    p.row_scale = g.row_scale;
    p.gsum = g.gsum;
    p.err = g.err;
    int tiles = 0, ntot = 0;
    for (int i = 0; i < g.nseg; ++i) {
        const PrefillGemmSegment& sg = g.seg[i];
        p.col_off[i] = ntot;
        ntot += sg.rows;
        p.w[i] = sg.w;
        if (!sg.w || sg.rows <= 0 || (!sg.y && !(pair && i == 1)) || (sg.type != Q4K_TYPE_Q4_K && sg.type != Q4K_TYPE_Q6_K))
            return cudaErrorInvalidValue;
        p.rows[i] = sg.rows;
        p.type[i] = sg.type;
        p.y[i] = sg.y;
        p.tile_start[i] = tiles;
        if (!pair || i == 0) tiles += (sg.rows + (pair ? BN / 2 : BN) - 1) / (pair ? BN / 2 : BN);
        KvTensorMap m[kWeightMaps];
        const KvTensorMap* src = g.wmap[i];
        if (!src) {
            const cudaError_t e = make_weight_map(sg.w, sg.type, g.K, sg.rows, m);
            if (e != cudaSuccess) return e;
            src = m;
        }
        std::memcpy(&maps.w[i][0], src, sizeof(CUtensorMap) * kWeightMaps);
    }
    for (int i = g.nseg; i < 3; ++i) std::memset(&maps.w[i][0], 0, sizeof(CUtensorMap) * kWeightMaps);
    for (int i = g.nseg; i < 4; ++i) p.tile_start[i] = tiles;
    if (g.amap) {
        std::memcpy(&maps.a, g.amap, sizeof(CUtensorMap));
    } else {
        KvTensorMap m;
        const cudaError_t e = make_act_map(g.a, g.K, g.M, &m);
        if (e != cudaSuccess) return e;
        std::memcpy(&maps.a, &m, sizeof m);
    }
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(prefill_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    });
    if (attr != cudaSuccess) return attr;
    // Split K where it shortens the launch (deterministic: the partial sums
    // are reduced in split order; gemm_splits has the cost model)
    const int splits = g.partial ? gemm_splits(g.M, tiles, p.nb, ntot, g.partial_floats) : 1;
    const int mtiles = (g.M + BM - 1) / BM;
    p.splits = splits;
    p.ntot = ntot;
    p.partial = g.partial;
    const dim3 grid(mtiles, tiles, splits);
    cudaError_t e = launch_pdl(prefill_gemm_kernel, grid, dim3(kThreads), kSmemBytes, s, p, maps);
    if (e != cudaSuccess || splits == 1) return e;
    ReduceArgs r;
    r.partial = g.partial;
    r.splits = splits;
    r.M = g.M;
    r.ntot = ntot;
    r.nseg = g.nseg;
    r.ldy = g.ldy;
    r.add = g.epilogue == EPI_ADD;
    r.off1 = g.nseg > 1 ? p.col_off[1] : ntot;
    r.off2 = g.nseg > 2 ? p.col_off[2] : ntot;
    r.y0 = g.seg[0].y;
    r.y1 = g.nseg > 1 ? g.seg[1].y : g.seg[0].y;
    r.y2 = g.nseg > 2 ? g.seg[2].y : g.seg[0].y;
    bool vec = ntot % 4 == 0 && g.ldy % 4 == 0 && r.off1 % 4 == 0 && r.off2 % 4 == 0;
    for (int i = 0; i < g.nseg; ++i) vec = vec && reinterpret_cast<uintptr_t>(g.seg[i].y) % 16 == 0;
    vec = vec && reinterpret_cast<uintptr_t>(g.partial) % 16 == 0;
    if (pair) {
        const size_t nr = (size_t)g.M * g.seg[0].rows;
        return launch_pdl(split_reduce_swiglu_kernel, dim3((unsigned)((nr + 255) / 256)), dim3(256), 0, s, r);
    }
    const size_t n = (size_t)g.M * ntot;
    if (vec) return launch_pdl(split_reduce_kernel<4>, dim3((unsigned)((n / 4 + 255) / 256)), dim3(256), 0, s, r);
    return launch_pdl(split_reduce_kernel<1>, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, r);
}

}  // namespace q4k
