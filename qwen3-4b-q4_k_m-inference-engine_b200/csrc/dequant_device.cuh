// Element-wise Q4_K / Q6_K dequantisation (embedding.cu:6-59 of the
// reference), shared by ops.cu and the decode-step kernel.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "q4k_device.cuh"
#include "q4k_format.h"

namespace q4k {

__device__ __forceinline__ float q4k_value(const uint8_t* block, unsigned position) {
    const unsigned group = position / 32;
    const uint8_t* s = block + 4;
    const int scale = group < 4 ? s[group] & 63 : (s[group + 4] & 15) | ((s[group - 4] >> 6) << 4);
    const int minimum = group < 4 ? s[group + 4] & 63 : (s[group + 4] >> 4) | ((s[group] >> 6) << 4);
    const unsigned code = (block[16 + (group / 2) * 32 + position % 32] >> ((group % 2) * 4)) & 15;
    const float d = half_bits_to_float(block[0] | (block[1] << 8));
    const float dmin = half_bits_to_float(block[2] | (block[3] << 8));
    return (d * (float)scale) * (float)code - dmin * (float)minimum;
}

__device__ __forceinline__ int q6_code(const uint8_t* ql, const uint8_t* qh, unsigned position) {
    const unsigned half = position / 128, group = (position % 128) / 32, lane = position % 32;
    const unsigned low = (ql[half * 64 + (group % 2) * 32 + lane] >> (4 * (group / 2))) & 15;
    const unsigned high = (qh[half * 32 + lane] >> (2 * group)) & 3;
    return (int)((high << 4) | low) - 32;
}

// Row `token` of a device-layout table into `out` (the engine's embedding
// lookup; EmbedLookup.cpp:49-78 does the same on the host + GPU).
__device__ __forceinline__ float device_layout_value(const uint8_t* row, int type, size_t nb, size_t column) {
    const unsigned position = column % 256;
    const size_t b = column / 256;
    if (type == Q4K_TYPE_Q4_K) return q4k_value(row + b * 144, position);
    const uint8_t* ql = row + b * 128;
    const uint8_t* qh = row + nb * 128 + b * 64;
    const int8_t* sc = reinterpret_cast<const int8_t*>(row + nb * 192 + b * 16);
    const uint8_t* dp = row + nb * 208 + b * 2;
    const float d = half_bits_to_float(dp[0] | (dp[1] << 8));
    return (d * (float)sc[position / 16]) * (float)q6_code(ql, qh, position);
}

}  // namespace q4k
