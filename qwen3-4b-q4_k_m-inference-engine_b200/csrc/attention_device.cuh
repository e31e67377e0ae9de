// Device routines of the fp16-KV decode attention shared by the per-layer
// kernel (attention_decode.cu) and the decode-step kernel (decode_step.cu):
// RoPE angle, TMA tile loads, the swizzled tile addressing, and the
// tensor-core fragments (fp32 values carried as fp16 hi + lo parts).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ops.h"
#include "q4k_device.cuh"

namespace q4k {
namespace attn_dev {

constexpr int D = kDecodeHeadDim;       // 128
constexpr int G = 4;                    // query heads per KV head
constexpr int kAttnTile = 64;           // positions per tile
constexpr int kBox = kAttnTile * 64 * 2;  // one 64-position x 64-dim fp16 box: 8 KB
constexpr int kTileBytes = 2 * kBox;    // K or V tile: 16 KB

__device__ __forceinline__ float rope_angle(int pos, int j, float base) {
    // rope.cu:19-20
    return (float)pos * powf(base, -2.0f * (float)j / (float)D);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Byte offset of (row r, 16-byte chunk c of the 128-dim row) inside a tile
// loaded as two 64-dim boxes with the 128-byte swizzle.
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
    return (uint32_t)((c >> 3) * kBox + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    // rows 8..15 of A are zero (a1 = a3 = 0)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// m16n8k16 with A rows 0-7 = (q or p) hi parts and rows 8-15 = lo parts:
// f = (a0 hi, a1 lo, a2 hi, a3 lo) of lane (g, t) as the fragments of rows g
// and g + 8.
__device__ __forceinline__ void mma16816_hilo(float (&c)[4], uint4 f, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(f.x), "r"(f.y), "r"(f.z), "r"(f.w), "r"(b0), "r"(b1));
}

// m16n8k16 with all four A fragments given.
__device__ __forceinline__ void mma16816_acc(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma1688(float& c0, float& c1, uint32_t a0, uint32_t b0) {
    float c2 = 0.0f, c3 = 0.0f;  // rows 8..15: zero A rows, results unused
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+f"(c0), "+f"(c1), "+f"(c2), "+f"(c3)
        : "r"(a0), "r"(0u), "r"(b0));
}

// fp32 pair -> packed fp16 (hi) and the fp16 residual (lo).
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

}  // namespace attn_dev
}  // namespace q4k
