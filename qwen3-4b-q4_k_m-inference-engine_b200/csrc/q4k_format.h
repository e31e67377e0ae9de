// Block formats, device layouts and the seeded synthetic-tensor generator.
//
// Shared by host code (g++) and device code (nvcc). Everything here is
// integer or exactly-rounded IEEE arithmetic, so the host and the device
// produce identical bytes for the same (seed, tensor name, index).
//
// GGUF super-block formats (256 values per block), as the reference reads them:
//   Q4_K, 144 B: fp16 d @0, fp16 dmin @2, 12 B packed 6-bit scales/mins @4,
//                128 B of nibbles @16   (src/cuda/matmul.cu:24-54,
//                src/cuda/embedding.cu:6-32)
//   Q6_K, 210 B: ql[128] @0, qh[64] @128, int8 scales[16] @192, fp16 d @208
//                (src/cuda/matmul.cu:61-84, src/cuda/embedding.cu:34-59)
//
// Device layouts used by this library's matrix-vector kernels:
//   Q4_K  rows are kept verbatim (row = nb * 144 B; 144 = 9 * 16, so every row
//         and block starts on a 16-byte boundary when the base does).
//   Q6_K  rows are re-laid out "planar" per row, because 210-byte blocks are
//         only 2-byte aligned:  [ql: nb*128][qh: nb*64][scales: nb*16]
//         [d: nb*2, zero-padded to a multiple of 16].  Each block's bytes keep
//         their order inside each plane, so the arithmetic is unchanged.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define Q4K_HD __host__ __device__ __forceinline__
#else
#define Q4K_HD static inline
#endif

// GGML tensor type ids (same values as include/q4k_b200.h).
#ifndef Q4K_TYPE_F32
#define Q4K_TYPE_F32 0
#define Q4K_TYPE_F16 1
#define Q4K_TYPE_Q4_K 12
#define Q4K_TYPE_Q6_K 14
#endif

#define Q4K_QK 256
#define Q4K_Q4_BLOCK 144
#define Q4K_Q6_BLOCK 210

// Bytes of one Q6_K planar device row holding nb super-blocks.
Q4K_HD size_t q4k_q6p_row_bytes(size_t nb) { return nb * 208 + ((2 * nb + 15) & ~(size_t)15); }

// Bytes of one device row of a quantised matrix with K inputs (K % 256 == 0).
Q4K_HD size_t q4k_device_row_bytes(int type, size_t K) {
    const size_t nb = K / Q4K_QK;
    if (type == Q4K_TYPE_Q4_K) return nb * Q4K_Q4_BLOCK;
    if (type == Q4K_TYPE_Q6_K) return q4k_q6p_row_bytes(nb);
    if (type == Q4K_TYPE_F32) return K * 4;
    if (type == Q4K_TYPE_F16) return K * 2;
    return 0;
}

// Bytes of one row in the GGUF file layout.
Q4K_HD size_t q4k_gguf_row_bytes(int type, size_t K) {
    const size_t nb = K / Q4K_QK;
    if (type == Q4K_TYPE_Q4_K) return nb * Q4K_Q4_BLOCK;
    if (type == Q4K_TYPE_Q6_K) return nb * Q4K_Q6_BLOCK;
    if (type == Q4K_TYPE_F32) return K * 4;
    if (type == Q4K_TYPE_F16) return K * 2;
    return 0;
}

// Scatter one raw Q6_K block (210 B) into block slot b of a planar row.
Q4K_HD void q4k_q6_to_planar(const uint8_t* blk, uint8_t* row, size_t nb, size_t b) {
    uint8_t* ql = row + b * 128;
    uint8_t* qh = row + nb * 128 + b * 64;
    uint8_t* sc = row + nb * 192 + b * 16;
    uint8_t* d = row + nb * 208 + b * 2;
    for (int i = 0; i < 128; ++i) ql[i] = blk[i];
    for (int i = 0; i < 64; ++i) qh[i] = blk[128 + i];
    for (int i = 0; i < 16; ++i) sc[i] = blk[192 + i];
    d[0] = blk[208];
    d[1] = blk[209];
}

// Gather block slot b of a planar row back into a raw 210-byte Q6_K block.
Q4K_HD void q4k_planar_to_q6(const uint8_t* row, size_t nb, size_t b, uint8_t* blk) {
    const uint8_t* ql = row + b * 128;
    const uint8_t* qh = row + nb * 128 + b * 64;
    const uint8_t* sc = row + nb * 192 + b * 16;
    const uint8_t* d = row + nb * 208 + b * 2;
    for (int i = 0; i < 128; ++i) blk[i] = ql[i];
    for (int i = 0; i < 64; ++i) blk[128 + i] = qh[i];
    for (int i = 0; i < 16; ++i) blk[192 + i] = sc[i];
    blk[208] = d[0];
    blk[209] = d[1];
}

// ---------------------------------------------------------------------------
// IEEE binary16 conversions written out in integer arithmetic (round to
// nearest, ties to even), so host and device agree bit for bit.
// ---------------------------------------------------------------------------
Q4K_HD uint32_t q4k_f32_bits(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}

Q4K_HD float q4k_bits_f32(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

Q4K_HD uint16_t q4k_f32_to_f16(float f) {
    const uint32_t x = q4k_f32_bits(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exponent = (x >> 23) & 0xffu;
    uint32_t mantissa = x & 0x7fffffu;
    if (exponent == 0xffu) return (uint16_t)(sign | 0x7c00u | (mantissa ? 0x200u : 0u));
    const int e = (int)exponent - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mantissa |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = mantissa >> shift;
        const uint32_t rem = mantissa & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (mantissa >> 13);
    const uint32_t rem = mantissa & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

Q4K_HD float q4k_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exponent = (h >> 10) & 0x1fu;
    uint32_t mantissa = h & 0x3ffu;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            exponent = 127 - 15 + 1;
            while ((mantissa & 0x400u) == 0) {
                mantissa <<= 1;
                --exponent;
            }
            mantissa &= 0x3ffu;
            bits = sign | (exponent << 23) | (mantissa << 13);
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 127 - 15) << 23) | (mantissa << 13);
    }
    return q4k_bits_f32(bits);
}

// ---------------------------------------------------------------------------
// Seeded synthetic tensors.
//
// key(seed, name) = mix64(seed ^ fnv1a64(name)); word(key, i) is the i-th
// output of a splitmix64 stream started at key. A normal deviate is the
// Irwin-Hall sum of twelve 16-bit uniforms, centred and scaled in double
// (exact integer arithmetic until one final rounding), so every value is
// reproducible on any IEEE host or device. Tails are bounded at +-6 sigma.
// ---------------------------------------------------------------------------
Q4K_HD uint64_t q4k_mix64(uint64_t z) {
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return z;
}

Q4K_HD uint64_t q4k_word(uint64_t key, uint64_t i) { return q4k_mix64(key + (i + 1) * 0x9E3779B97F4A7C15ull); }

Q4K_HD double q4k_normal(uint64_t key, uint64_t i) {
    uint64_t s = 0;
    for (int k = 0; k < 3; ++k) {
        const uint64_t w = q4k_word(key, 3 * i + (uint64_t)k);
        s += (w & 0xffffu) + ((w >> 16) & 0xffffu) + ((w >> 32) & 0xffffu) + (w >> 48);
    }
    return ((double)s - 393210.0) / 65536.0;
}

static inline uint64_t q4k_fnv1a64(const char* s) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (; *s; ++s) {
        h ^= (uint8_t)*s;
        h *= 0x100000001b3ull;
    }
    return h;
}

static inline uint64_t q4k_tensor_key(uint64_t seed, const char* name) { return q4k_mix64(seed ^ q4k_fnv1a64(name)); }

// Second stream of a tensor, used for the fp16 block headers.
Q4K_HD uint64_t q4k_header_key(uint64_t key) { return q4k_mix64(key ^ 0x4844522D4B455931ull); }

Q4K_HD void q4k_put_word(uint8_t* dst, uint64_t w, int nbytes) {
    for (int i = 0; i < nbytes; ++i) dst[i] = (uint8_t)(w >> (8 * i));
}

// Q4_K block b: d, dmin = fp16(|N(0, 2e-3)|); 12 scale bytes and 128 quant
// bytes uniform in [0, 255] (so every 6-bit field is uniform in [0, 63]).
Q4K_HD void q4k_synth_q4k_block(uint64_t key, uint64_t b, uint8_t* blk) {
    const uint64_t hk = q4k_header_key(key);
    double n0 = q4k_normal(hk, 2 * b), n1 = q4k_normal(hk, 2 * b + 1);
    n0 = n0 < 0 ? -n0 : n0;
    n1 = n1 < 0 ? -n1 : n1;
    const uint16_t d = q4k_f32_to_f16((float)(n0 * 2e-3));
    const uint16_t dmin = q4k_f32_to_f16((float)(n1 * 2e-3));
    blk[0] = (uint8_t)d;
    blk[1] = (uint8_t)(d >> 8);
    blk[2] = (uint8_t)dmin;
    blk[3] = (uint8_t)(dmin >> 8);
    for (int k = 0; k < 18; ++k) {
        const uint64_t w = q4k_word(key, 18 * b + (uint64_t)k);
        const int off = 4 + 8 * k;
        q4k_put_word(blk + off, w, off + 8 <= 144 ? 8 : 144 - off);
    }
}

// Q6_K block b: ql/qh bytes uniform in [0, 255]; int8 scales uniform in
// [-32, 31]; d = fp16(|N(0, 1e-3)|).
Q4K_HD void q4k_synth_q6k_block(uint64_t key, uint64_t b, uint8_t* blk) {
    for (int k = 0; k < 24; ++k) q4k_put_word(blk + 8 * k, q4k_word(key, 26 * b + (uint64_t)k), 8);
    for (int k = 0; k < 2; ++k) {
        const uint64_t w = q4k_word(key, 26 * b + 24 + (uint64_t)k);
        for (int i = 0; i < 8; ++i) blk[192 + 8 * k + i] = (uint8_t)(int8_t)((int)((w >> (8 * i)) & 63u) - 32);
    }
    double n = q4k_normal(q4k_header_key(key), b);
    n = n < 0 ? -n : n;
    const uint16_t d = q4k_f32_to_f16((float)(n * 1e-3));
    blk[208] = (uint8_t)d;
    blk[209] = (uint8_t)(d >> 8);
}

// RMSNorm gamma element i: 1 + N(0, 0.02).
Q4K_HD float q4k_synth_gamma(uint64_t key, uint64_t i) { return (float)(1.0 + 0.02 * q4k_normal(key, i)); }

// Plain N(0, 1) fp32 element i (activations).
Q4K_HD float q4k_synth_f32(uint64_t key, uint64_t i) { return (float)q4k_normal(key, i); }

// fp16 N(0, 1) element i (KV-cache fill).
Q4K_HD uint16_t q4k_synth_f16(uint64_t key, uint64_t i) { return q4k_f32_to_f16((float)q4k_normal(key, i)); }
