// Device routines of the Q4_K / Q6_K matrix-vector product shared by the
// per-product kernel (gemv.cu) and the persistent decode-step kernel
// (decode_step.cu): activation quantisation and the per-lane dot products.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "q4k_device.cuh"

namespace q4k {
namespace gemv_dev {

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
        if (MT == 1 || m < mcount) {  // a batch of one: always (mcount is 1)
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

// Tensor-core integer product: D = A (16x32 u8) * B (32x8 s8), zero C.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Q4_K dot products of two rows (row_g, row_h: the A rows g and g+8 of lane
// (g, t) = (lane / 4, lane % 4)) over super-blocks b_begin, b_begin + b_step,
// ... < nb, on the tensor cores. For block b, MMA (j, h) takes nibble plane
// h of 32-byte chunk j of the warp's 16 rows as A (u8; the high plane as
// 16x its value) and the codes of the block's 8 groups as the 8 columns of
// B, so column 2j + h, the diagonal, is group 2j + h's dot product. Lane
// (g, t) keeps chunk t's two columns for its rows and applies the group
// scales exactly as q4_pair does (matmul.cu:24-54).
template <int UNROLL>
__device__ __forceinline__ void q4_rows_mma(const uint8_t* row_g, const uint8_t* row_h, int b_begin, int b_step,
                                            int nb, const uint8_t* xq, const float* xs, const float* xsumf, int g,
                                            int t, float& acc_g, float& acc_h) {
    const int sh = (t & 1) * 16;
    // UNROLL blocks in flight per warp: each block is a chain of shared
    // loads, MMAs and scale arithmetic, so independent blocks hide latency
#pragma unroll UNROLL
    for (int b = b_begin; b < nb; b += b_step) {
        const uint8_t* pg = row_g + b * 144;
        const uint8_t* ph = row_h + b * 144;
        const uint8_t* xb = xq + b * 256;
        // B: codes of group g at positions 4t.. (piece 2g) and 4t + 16.. (piece 2g + 1)
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xb + 16 * perm_q4(2 * g, b) + 4 * t);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xb + 16 * perm_q4(2 * g + 1, b) + 4 * t);
        int dlg = 0, dlh = 0, dhg = 0, dhh = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t g0 = *reinterpret_cast<const uint32_t*>(pg + 16 + 32 * j + 4 * t);
            const uint32_t g1 = *reinterpret_cast<const uint32_t*>(pg + 32 + 32 * j + 4 * t);
            const uint32_t h0 = *reinterpret_cast<const uint32_t*>(ph + 16 + 32 * j + 4 * t);
            const uint32_t h1 = *reinterpret_cast<const uint32_t*>(ph + 32 + 32 * j + 4 * t);
            int c[4];
            mma_u8s8(c, g0 & 0x0f0f0f0fu, h0 & 0x0f0f0f0fu, g1 & 0x0f0f0f0fu, h1 & 0x0f0f0f0fu, b0, b1);
            if (j == t) {
                dlg = c[0];
                dlh = c[2];
            }
            mma_u8s8(c, g0 & 0xf0f0f0f0u, h0 & 0xf0f0f0f0u, g1 & 0xf0f0f0f0u, h1 & 0xf0f0f0f0u, b0, b1);
            if (j == t) {
                dhg = c[1] >> 4;  // exact: every term is a multiple of 16
                dhh = c[3] >> 4;
            }
        }
        const float2 s2 = *reinterpret_cast<const float2*>(xs + b * 8 + 2 * t);
        const float2 t2 = *reinterpret_cast<const float2*>(xsumf + b * 8 + 2 * t);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint4 hdr = *reinterpret_cast<const uint4*>(r == 0 ? pg : ph);
            const uint32_t SC =
                t < 2 ? (hdr.y & 0x3f3f3f3fu) : ((hdr.w & 0x0f0f0f0fu) | ((hdr.y >> 2) & 0x30303030u));
            const uint32_t MN =
                t < 2 ? (hdr.z & 0x3f3f3f3fu) : (((hdr.w >> 4) & 0x0f0f0f0fu) | ((hdr.z >> 2) & 0x30303030u));
            const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
            const float ds0 = d * (float)((SC >> sh) & 0xffu), ds1 = d * (float)((SC >> (sh + 8)) & 0xffu);
            const float dm0 = dmin * (float)((MN >> sh) & 0xffu), dm1 = dmin * (float)((MN >> (sh + 8)) & 0xffu);
            const int dl = r == 0 ? dlg : dlh, dh = r == 0 ? dhg : dhh;
            float& acc = r == 0 ? acc_g : acc_h;
            acc += s2.x * (ds0 * (float)dl - dm0 * t2.x);
            acc += s2.y * (ds1 * (float)dh - dm1 * t2.y);
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
        if (MT == 1 || m < mcount) {  // a batch of one: always (mcount is 1)
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

// 1/a for a positive finite float a, as a double with relative error below
// 2^-51: the hardware's approximate double reciprocal refined by two
// Newton-Raphson steps r <- r + r (1 - a r) (each roughly squares the
// relative error, down to the double rounding). Every float, normal or
// subnormal, is a normal double, so no range needs special handling.
__device__ __forceinline__ double recip_refined(float a) {
    const double ad = (double)a;
    double r;
    asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(r) : "d"(ad));
    r = fma(r, fma(-ad, r, 1.0), r);
    r = fma(r, fma(-ad, r, 1.0), r);
    return r;
}

// The reference's code roundf(fl(fl(v / amax) * 127)) (matmul.cu:19) bit
// for bit, without a division or a branch, given ra = recip_refined(amax)
// for a positive finite amax (and |v| <= amax).
// Why fl(v / amax) = fl32(v * ra): write v = V 2^i, amax = A 2^j (V, A
// integers below 2^24) and a float32 rounding boundary (midpoint) as
// M = N 2^k with N odd, 2^24 <= N < 2^25. The quotient v / amax is never
// exactly M (V = A N 2^(j+k-i) would need a factor N >= 2^24 in V), and
// when it is not, |v - amax M| >= min(2^i, 2^(j+k)), i.e. the quotient is at
// least 2^-50 (relative) from every midpoint in the normal range. v * ra is
// within 2^-51 * 1.5 of it, so both round to the same float. Quotients
// below 2^-126 give codes of 0 either way (127 t < 0.5). The product with
// 127 and the rounding (halves away from zero, as roundf) then follow the
// reference exactly: u - trunc(u) is exact.
__device__ __forceinline__ int8_t q8_code_r(float v, double ra) {
    const float t = __double2float_rn(__dmul_rn((double)v, ra));
    const float u = __fmul_rn(t, 127.0f);
    const float tr = truncf(u);
    const float c = fabsf(u - tr) >= 0.5f ? tr + copysignf(1.0f, u) : tr;
    return static_cast<int8_t>(static_cast<int>(c));
}

// Whether q8_code_r applies (amax positive and finite); otherwise every code
// of the group is 0, as the reference's for a zero maximum.
__device__ __forceinline__ bool q8_codes_defined(float amax) { return amax > 0.0f && amax <= 3.402823466e38f; }

// The group scale fl(amax / 127) (matmul.cu:18), bit for bit, without a
// division: amax * fl64(1/127) is within 2^-52 (relative) of amax / 127,
// which is never a float32 midpoint (127 is odd) and, as above, at least
// 2^-50 from one, subnormal results included (their grid is coarser).
// Infinities and NaNs pass through as amax / 127 would.
__device__ __forceinline__ float q8_scale(float amax) {
    return __double2float_rn(__dmul_rn((double)amax, 1.0 / 127.0));
}

// Quantise MT activation rows into shared memory: codes (in the Q4_K and/or
// Q6_K permuted order), one fp32 scale per 32 values, code sums per 16 and
// per 32 values. Called by all W*32 consumer threads.
// Q8-quantise the 4 values of element e = 4i of activation row m (already
// RMSNorm-ed if the product has a norm): the 8 lanes i..i+7 of a warp hold
// one 32-group (matmul.cu:8-22). Stores the codes (Q4_K and/or Q6_K
// permuted order), the group scale, and the 16- and 32-value code sums.
// quantise_vec4 for N float4s of a thread side by side (their dependent
// chains interleave); vector n is element e[n] of row m.
template <int N>
__device__ __forceinline__ void quantise_vecs(const float4 (&v)[N], const int (&e)[N], int K, int m, uint8_t* xq4,
                                              uint8_t* xq6, float* xs, int* xsum16, float* xsum32, int lane,
                                              bool store = true) {
    float amax[N];
#pragma unroll
    for (int n = 0; n < N; ++n) amax[n] = fmaxf(fmaxf(fabsf(v[n].x), fabsf(v[n].y)), fmaxf(fabsf(v[n].z), fabsf(v[n].w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int n = 0; n < N; ++n) amax[n] = fmaxf(amax[n], __shfl_xor_sync(0xffffffffu, amax[n], o));
    uint32_t word[N];
    int run[N];
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const bool defined = q8_codes_defined(amax[n]);
        const double ra = recip_refined(defined ? amax[n] : 1.0f);
        const int8_t c0 = defined ? q8_code_r(v[n].x, ra) : 0, c1 = defined ? q8_code_r(v[n].y, ra) : 0;
        const int8_t c2 = defined ? q8_code_r(v[n].z, ra) : 0, c3 = defined ? q8_code_r(v[n].w, ra) : 0;
        word[n] = (uint32_t)(uint8_t)c0 | ((uint32_t)(uint8_t)c1 << 8) | ((uint32_t)(uint8_t)c2 << 16) |
                  ((uint32_t)(uint8_t)c3 << 24);
        run[n] = (int)c0 + (int)c1 + (int)c2 + (int)c3;
    }
#pragma unroll
    for (int n = 0; n < N; ++n) run[n] += __shfl_xor_sync(0xffffffffu, run[n], 1);
#pragma unroll
    for (int n = 0; n < N; ++n) run[n] += __shfl_xor_sync(0xffffffffu, run[n], 2);
    int group[N];
#pragma unroll
    for (int n = 0; n < N; ++n) group[n] = run[n] + __shfl_xor_sync(0xffffffffu, run[n], 4);
    if (!store) return;  // a lane that only took part in its warp's shuffles
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const int b = e[n] >> 8, r16 = (e[n] & 255) >> 4, o = e[n] & 15;
        if (xq4) *reinterpret_cast<uint32_t*>(xq4 + m * K + b * 256 + 16 * perm_q4(r16, b) + o) = word[n];
        if (xq6) *reinterpret_cast<uint32_t*>(xq6 + m * K + b * 256 + 16 * perm_q6(r16, b) + o) = word[n];
        // run r16 = 8h + 2g + l is stored at quarter (2h + l), slot g
        if ((lane & 3) == 0)
            xsum16[m * (K / 16) + b * 16 + 4 * (2 * (r16 >> 3) + (r16 & 1)) + ((r16 >> 1) & 3)] = 32 * run[n];
        if ((lane & 7) == 0) {
            xsum32[m * (K / 32) + (e[n] >> 5)] = (float)group[n];
            xs[m * (K / 32) + (e[n] >> 5)] = q8_scale(amax[n]);  // matmul.cu:18
        }
    }
}

__device__ __forceinline__ void quantise_vec4(float4 v, int e, int K, int m, uint8_t* xq4, uint8_t* xq6, float* xs,
                                              int* xsum16, float* xsum32, int lane, bool store = true) {
    const float4 vv[1] = {v};
    const int ee[1] = {e};
    quantise_vecs<1>(vv, ee, K, m, xq4, xq6, xs, xsum16, xsum32, lane, store);
}

// Q8-quantise elements e and e + 1 (e even) of a row whose 32-value group
// is held two values per lane by the 16 lanes (lane & 15) = (e & 31) / 2 of
// a half-warp (all 32 lanes of the warp take part). Bit for bit what
// quantise_vec4 computes for the same group.
__device__ __forceinline__ void quantise_pair(float v0, float v1, int e, int K, uint8_t* xq4, uint8_t* xq6, float* xs,
                                              int* xsum16, float* xsum32, int lane) {
    float amax = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const bool defined = q8_codes_defined(amax);
    const double ra = recip_refined(defined ? amax : 1.0f);
    const int8_t c0 = defined ? q8_code_r(v0, ra) : 0, c1 = defined ? q8_code_r(v1, ra) : 0;
    int run = (int)c0 + (int)c1;
    run += __shfl_xor_sync(0xffffffffu, run, 1);
    run += __shfl_xor_sync(0xffffffffu, run, 2);
    run += __shfl_xor_sync(0xffffffffu, run, 4);
    const int group = run + __shfl_xor_sync(0xffffffffu, run, 8);
    const uint16_t word = (uint16_t)((uint32_t)(uint8_t)c0 | ((uint32_t)(uint8_t)c1 << 8));
    const int b = e >> 8, r16 = (e & 255) >> 4, o = e & 15;
    if (xq4) *reinterpret_cast<uint16_t*>(xq4 + b * 256 + 16 * perm_q4(r16, b) + o) = word;
    if (xq6) *reinterpret_cast<uint16_t*>(xq6 + b * 256 + 16 * perm_q6(r16, b) + o) = word;
    if ((lane & 7) == 0)
        xsum16[b * 16 + 4 * (2 * (r16 >> 3) + (r16 & 1)) + ((r16 >> 1) & 3)] = 32 * run;
    if ((lane & 15) == 0) {
        xsum32[e >> 5] = (float)group;
        xs[e >> 5] = q8_scale(amax);  // matmul.cu:18
    }
}

// The parts of an ActImage (q4k_internal.h) for K inputs.
struct ImageParts {
    uint8_t* q4;
    uint8_t* q6;
    float* xs;
    int* xsum16;
    float* xsum32;
};
__device__ __forceinline__ ImageParts image_parts(uint8_t* base, int K) {
    ImageParts v;
    v.q4 = base;
    v.q6 = base + K;
    v.xs = reinterpret_cast<float*>(base + 2 * K);
    v.xsum16 = reinterpret_cast<int*>(base + 2 * K + K / 8);
    v.xsum32 = reinterpret_cast<float*>(base + 2 * K + K / 8 + K / 4);
    return v;
}

template <int kHeld>
__device__ __forceinline__ void quantise_rows(const float* x, int ldx, int m0, int mcount, const float* gamma,
                                              float eps, int K, uint8_t* xq4, uint8_t* xq6, float* xs, int* xsum16,
                                              float* xsum32, float* red, int tid, int lane, int warp, int nthreads,
                                              int barrier_id, unsigned long long* trace = nullptr,
                                              int trace_tag = 0, const unsigned long long* parts = nullptr,
                                              int nparts = 0, unsigned parts_tag = 0, int* err = nullptr,
                                              uint64_t wait_ns = 0, int err_code = 0, float* x_out = nullptr) {
    const int nvec = K / 4;
    // kHeld: float4s of the row a thread keeps in registers (K <= kHeld * 4 * nthreads)
    for (int m = 0; m < mcount; ++m) {
        const float4* xr = reinterpret_cast<const float4*>(x + (size_t)(m0 + m) * ldx);
        // one pass over the row: every load in flight at once, kept for both uses
        float4 held[kHeld];
#pragma unroll
        for (int k = 0; k < kHeld; ++k) {
            const int i = tid + k * nthreads;
            if (i < nvec) held[k] = __ldcg(xr + i);  // may have been written by other SMs in this launch
        }
        if (parts && m == 0) {
            // tensor parallelism: x + the ranks' partial sums (rank order), the
            // residual stream every rank computes alike
#pragma unroll
            for (int k = 0; k < kHeld; ++k) {
                const int i = tid + k * nthreads;
                if (i >= nvec) continue;
                const float4 sum =
                    sum_tagged4<kMaxRanks>(parts + 4 * (size_t)i, (size_t)K, nparts, parts_tag, wait_ns, err, err_code);
                held[k].x += sum.x;
                held[k].y += sum.y;
                held[k].z += sum.z;
                held[k].w += sum.w;
            }
        }
        if (x_out && m == 0) {
#pragma unroll
            for (int k = 0; k < kHeld; ++k) {
                const int i = tid + k * nthreads;
                if (i < nvec) reinterpret_cast<float4*>(x_out)[i] = held[k];
            }
        }
        if (trace && tid == 0 && m == 0) {
            // timeline: when thread 0's first activation load has landed
            float landed;
            asm volatile("mov.b32 %0, %1;" : "=f"(landed) : "f"(held[0].x));
            asm volatile("" ::"f"(landed));
            trace_at(trace, trace_tag, 5);
        }
        float inv = 1.0f;
        if (gamma) {
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
            named_barrier(barrier_id, nthreads);
            // every warp sums the per-warp partials in the same shuffle tree
            const float total = warp_sum(lane < nthreads / 32 ? red[lane] : 0.0f);
            inv = rsqrtf(total / (float)K + eps);  // rms_norm.cu:17
            // `red` is written again only for the next row
            if (m + 1 < mcount) named_barrier(barrier_id, nthreads);
        }
        // element e = 4*i of the row; the 8 lanes i..i+7 hold one 32-group
        auto normed = [&](int k) {
            const int i = tid + k * nthreads;
            float4 v = held[k];
            if (gamma && i < nvec) {
                const float4 gm = reinterpret_cast<const float4*>(gamma)[i];
                v.x = (v.x * inv) * gm.x;  // rms_norm.cu:19: input * inverse_rms * scale
                v.y = (v.y * inv) * gm.y;
                v.z = (v.z * inv) * gm.z;
                v.w = (v.w * inv) * gm.w;
            }
            return v;
        };
        if constexpr (kHeld == 2) {
            // a thread's two float4s side by side (which warps hold a second
            // one is warp-uniform: nvec and nthreads are multiples of 32)
            if (tid + nthreads < nvec) {
                const float4 vv[2] = {normed(0), normed(1)};
                const int ee[2] = {4 * tid, 4 * (tid + nthreads)};
                quantise_vecs<2>(vv, ee, K, m, xq4, xq6, xs, xsum16, xsum32, lane);
            } else if (tid < nvec) {
                quantise_vec4(normed(0), 4 * tid, K, m, xq4, xq6, xs, xsum16, xsum32, lane);
            }
        } else {
#pragma unroll
            for (int k = 0; k < kHeld; ++k) {
                const int i = tid + k * nthreads;
                if (i >= nvec) break;
                quantise_vec4(normed(k), 4 * i, K, m, xq4, xq6, xs, xsum16, xsum32, lane);
            }
        }
    }
    named_barrier(barrier_id, nthreads);
}

}  // namespace gemv_dev
}  // namespace q4k
