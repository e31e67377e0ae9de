// Q4_K / Q6_K dequantise-fused matrix-vector (and small-batch) product.
//
// Arithmetic follows the reference engine's project<Type> kernel
// (src/cuda/matmul.cu:24-125): the fp32 activation is first quantised to
// int8 with one fp32 scale per 32 values (matmul.cu:8-22), then every
// 32-value group contributes  xs[g] * (d*sc*sum(q*xq) - dmin*m*sum(xq))
// for Q4_K and  xs[g] * (d*sc*sum((q-32)*xq))  for Q6_K, with the integer
// dot products done by dp4a.
//
// B200 structure (one CTA per SM, HBM-bound):
//   * warp W (the last one) is a producer: one lane streams whole weight rows
//     from HBM into shared memory with cp.async.bulk (TMA bulk copies)
//     completing on mbarriers. It starts before griddepcontrol.wait, so under
//     programmatic dependent launch the weights of this product stream in
//     while the previous kernel is still finishing.
//   * warps 0..W-1 are consumers. They quantise the activation into shared
//     memory (optionally applying RMSNorm first, which fuses
//     rms_norm.cu:6-24 into the product), then each warp owns a private ring
//     of S row buffers: row i of the CTA's range goes to warp i % W. A warp
//     reduces its row with shuffles and lane 0 writes the result, so the main
//     loop has no CTA-wide barrier.
//   * activation codes are stored in a permuted order per block so that the
//     16-byte shared loads of the 8 lanes working on one super-block hit 32
//     distinct banks.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "q4k_device.cuh"
#include "q4k_internal.h"

namespace q4k {
namespace {

struct GemvPlan {
    GemvSegment seg[kMaxSegments];
    int seg_start[kMaxSegments + 1];
    int nseg;
    int K, nb, M, ldx, ldy;
    const float* x;
    const float* gamma;
    float eps;
    int epilogue;
    int total_rows;
    int stages;      // S: buffers per consumer warp
    int slot_bytes;  // bytes per buffer (one job: 1 row, or 2 rows when paired)
    int row_bytes[kMaxSegments];
    int off_xq4, off_xq6, off_xs, off_xsum, off_bufs, off_bars, off_red;  // shared-memory offsets
    ArgmaxTarget argmax;
    int* err;
};

// 6-bit scale and min of 32-value group g of a Q4_K block, from the three
// header words holding bytes 4..15 (matmul.cu:40-48).
__device__ __forceinline__ void q4_scale_min(uint32_t w0, uint32_t w1, uint32_t w2, int g, int& sc, int& mn) {
    const int u = (g & 3) * 8;
    const int b0 = (w0 >> u) & 0xff, b1 = (w1 >> u) & 0xff, b2 = (w2 >> u) & 0xff;
    if (g < 4) {
        sc = b0 & 63;
        mn = b1 & 63;
    } else {
        sc = (b2 & 15) | ((b0 >> 6) << 4);
        mn = (b2 >> 4) | ((b1 >> 6) << 4);
    }
}

// Lane chunk f of a Q4_K row: block b = f/8, c = f%8 covers bytes
// 16 + 32*(c/2) + 16*(c%2) .. +16 of the block, i.e. positions 16*(c%2)..+15
// of groups 2*(c/2) (low nibbles) and 2*(c/2)+1 (high nibbles).
template <int MT, int JR>
__device__ __forceinline__ void q4_chunk(const uint8_t* const (&rows)[JR], int f, const uint8_t* xq, const float* xs,
                                         const int* xsum, int K, int mcount, float (&acc)[JR][MT]) {
    const int b = f >> 3, c = f & 7, j = c >> 1, h = c & 1;
    const int g0 = 2 * j;
    const int r_lo = b * 16 + 4 * j + h, r_hi = r_lo + 2;
    uint4 xlo[MT], xhi[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < mcount) {
            xlo[m] = *reinterpret_cast<const uint4*>(xq + m * K + b * 256 + 16 * c);
            xhi[m] = *reinterpret_cast<const uint4*>(xq + m * K + b * 256 + 128 + 16 * c);
        }
    }
#pragma unroll
    for (int r = 0; r < JR; ++r) {
        const uint8_t* blk = rows[r] + b * 144;
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 q = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j + 16 * h);
        const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
        int sc0, m0, sc1, m1;
        q4_scale_min(hdr.y, hdr.z, hdr.w, g0, sc0, m0);
        q4_scale_min(hdr.y, hdr.z, hdr.w, g0 + 1, sc1, m1);
        const float ds0 = d * (float)sc0, dm0 = dmin * (float)m0;
        const float ds1 = d * (float)sc1, dm1 = dmin * (float)m1;
        const uint32_t l0 = q.x & 0x0f0f0f0fu, l1 = q.y & 0x0f0f0f0fu, l2 = q.z & 0x0f0f0f0fu, l3 = q.w & 0x0f0f0f0fu;
        const uint32_t h0 = (q.x >> 4) & 0x0f0f0f0fu, h1 = (q.y >> 4) & 0x0f0f0f0fu;
        const uint32_t h2 = (q.z >> 4) & 0x0f0f0f0fu, h3 = (q.w >> 4) & 0x0f0f0f0fu;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m < mcount) {
                int dlo = __dp4a((int)l0, (int)xlo[m].x, 0);
                dlo = __dp4a((int)l1, (int)xlo[m].y, dlo);
                dlo = __dp4a((int)l2, (int)xlo[m].z, dlo);
                dlo = __dp4a((int)l3, (int)xlo[m].w, dlo);
                int dhi = __dp4a((int)h0, (int)xhi[m].x, 0);
                dhi = __dp4a((int)h1, (int)xhi[m].y, dhi);
                dhi = __dp4a((int)h2, (int)xhi[m].z, dhi);
                dhi = __dp4a((int)h3, (int)xhi[m].w, dhi);
                const float* xsm = xs + m * (K / 32) + b * 8;
                const int* sum = xsum + m * (K / 16);
                acc[r][m] += xsm[g0] * (ds0 * (float)dlo - dm0 * (float)sum[r_lo]) +
                             xsm[g0 + 1] * (ds1 * (float)dhi - dm1 * (float)sum[r_hi]);
            }
        }
    }
}

// Lane chunk f of a Q6_K planar row: block b = f/8, c = f%8 -> half = c/4,
// s = (c/2)%2, t = c%2. The 16 ql bytes at half*64 + s*32 + t*16 carry the
// low nibbles of 16-value runs A (32-group 4*half+s) and B (4*half+s+2);
// the 16 qh bytes at half*32 + t*16 carry their top two bits
// (matmul.cu:68-83, embedding.cu:42-58).
template <int MT, int JR>
__device__ __forceinline__ void q6_chunk(const uint8_t* const (&rows)[JR], int nb, int f, const uint8_t* xq,
                                         const float* xs, const int* xsum, int K, int mcount,
                                         float (&acc)[JR][MT]) {
    const int b = f >> 3, c = f & 7, half = c >> 2, s = (c >> 1) & 1, t = c & 1;
    const int rA = 8 * half + 2 * s + t, rB = rA + 4;
    const int gA = 4 * half + s, gB = gA + 2;
    const int shA = 2 * s, shB = 2 * s + 4;
    uint4 xa[MT], xb[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < mcount) {
            xa[m] = *reinterpret_cast<const uint4*>(xq + m * K + b * 256 + 16 * c);
            xb[m] = *reinterpret_cast<const uint4*>(xq + m * K + b * 256 + 128 + 16 * c);
        }
    }
#pragma unroll
    for (int r = 0; r < JR; ++r) {
        const uint8_t* row = rows[r];
        const uint4 ql = *reinterpret_cast<const uint4*>(row + b * 128 + half * 64 + s * 32 + t * 16);
        const uint4 qh = *reinterpret_cast<const uint4*>(row + nb * 128 + b * 64 + half * 32 + t * 16);
        const int8_t* sc = reinterpret_cast<const int8_t*>(row + nb * 192 + b * 16);
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + nb * 208 + b * 2));
        const float dA = d * (float)sc[rA], dB = d * (float)sc[rB];
        const uint32_t a0 = (ql.x & 0x0f0f0f0fu) | (((qh.x >> shA) & 0x03030303u) << 4);
        const uint32_t a1 = (ql.y & 0x0f0f0f0fu) | (((qh.y >> shA) & 0x03030303u) << 4);
        const uint32_t a2 = (ql.z & 0x0f0f0f0fu) | (((qh.z >> shA) & 0x03030303u) << 4);
        const uint32_t a3 = (ql.w & 0x0f0f0f0fu) | (((qh.w >> shA) & 0x03030303u) << 4);
        const uint32_t b0 = ((ql.x >> 4) & 0x0f0f0f0fu) | (((qh.x >> shB) & 0x03030303u) << 4);
        const uint32_t b1 = ((ql.y >> 4) & 0x0f0f0f0fu) | (((qh.y >> shB) & 0x03030303u) << 4);
        const uint32_t b2 = ((ql.z >> 4) & 0x0f0f0f0fu) | (((qh.z >> shB) & 0x03030303u) << 4);
        const uint32_t b3 = ((ql.w >> 4) & 0x0f0f0f0fu) | (((qh.w >> shB) & 0x03030303u) << 4);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m < mcount) {
                const int* sum = xsum + m * (K / 16) + b * 16;
                // codes are in [0, 63], so signed dp4a is exact; (q - 32) is
                // applied through the run sums.
                int da = __dp4a((int)a0, (int)xa[m].x, 0);
                da = __dp4a((int)a1, (int)xa[m].y, da);
                da = __dp4a((int)a2, (int)xa[m].z, da);
                da = __dp4a((int)a3, (int)xa[m].w, da);
                da -= 32 * sum[rA];
                int db = __dp4a((int)b0, (int)xb[m].x, 0);
                db = __dp4a((int)b1, (int)xb[m].y, db);
                db = __dp4a((int)b2, (int)xb[m].z, db);
                db = __dp4a((int)b3, (int)xb[m].w, db);
                db -= 32 * sum[rB];
                const float* xsm = xs + m * (K / 32) + b * 8;
                acc[r][m] += xsm[gA] * (dA * (float)da) + xsm[gB] * (dB * (float)db);
            }
        }
    }
}

// Permuted byte offset, inside its 256-value block, of the 16-value run r16
// for the Q4_K and Q6_K lane mappings above.
__device__ __forceinline__ int perm_q4(int r16) {
    const int j = r16 >> 2, lohi = (r16 >> 1) & 1, h = r16 & 1;
    return (lohi * 8 + 2 * j + h) * 16;
}
__device__ __forceinline__ int perm_q6(int r16) {
    const int half = r16 >> 3, ab = (r16 >> 2) & 1, s = (r16 >> 1) & 1, t = r16 & 1;
    return (ab * 8 + 4 * half + 2 * s + t) * 16;
}

__device__ __forceinline__ int8_t q8_code(float v, float amax) {
    // matmul.cu:19: roundf((value / maximum) * 127), IEEE division.
    return amax == 0.0f ? 0 : static_cast<int8_t>(roundf(__fmul_rn(__fdiv_rn(v, amax), 127.0f)));
}

template <int MT, int JR>
__global__ void __launch_bounds__(288, MT <= 2 ? 2 : 1) gemv_kernel(const __grid_constant__ GemvPlan p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int W = (int)(blockDim.x >> 5) - 1;  // consumer warps
    const int S = p.stages;
    const int K = p.K;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
    uint64_t* empty = full + W * S;
    uint8_t* bufs = smem + p.off_bufs;

    const int G = gridDim.x;
    const int r_begin = (int)((long long)p.total_rows * blockIdx.x / G);
    const int r_end = (int)((long long)p.total_rows * (blockIdx.x + 1) / G);
    const int m0 = blockIdx.y * MT;
    const int mcount = min(MT, p.M - m0);

    if (tid == 0) {
        for (int i = 0; i < W * S; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == W) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();
            int seg = 0;
            for (int i = 0, row = r_begin; row < r_end; ++i, ++row) {
                const int w = i % W, slot = (i / W) % S, use = i / (W * S);
                uint64_t* fb = full + w * S + slot;
                if (use > 0 && !mbar_wait_bounded(empty + w * S + slot, (use - 1) & 1, p.err, ERR_WAIT_TIMEOUT_EMPTY))
                    break;
                while (seg + 1 < p.nseg && row >= p.seg_start[seg + 1]) ++seg;
                const int local = row - p.seg_start[seg];
                uint8_t* dst = bufs + (size_t)(w * S + slot) * p.slot_bytes;
                if (JR == 2) {
                    const int rb = p.row_bytes[0];
                    mbar_arrive_expect_tx(fb, 2 * rb);
                    bulk_g2s_hint(dst, p.seg[0].w + (size_t)local * rb, rb, fb, policy);
                    bulk_g2s_hint(dst + rb, p.seg[1].w + (size_t)local * rb, rb, fb, policy);
                } else {
                    const int rb = p.row_bytes[seg];
                    mbar_arrive_expect_tx(fb, rb);
                    bulk_g2s_hint(dst, p.seg[seg].w + (size_t)local * rb, rb, fb, policy);
                }
            }
        }
        return;
    }

    // ---------------- consumers: quantise the activation ----------------
    pdl_wait();
    uint8_t* xq4 = p.off_xq4 >= 0 ? smem + p.off_xq4 : nullptr;
    uint8_t* xq6 = p.off_xq6 >= 0 ? smem + p.off_xq6 : nullptr;
    float* xs = reinterpret_cast<float*>(smem + p.off_xs);
    int* xsum = reinterpret_cast<int*>(smem + p.off_xsum);
    float* red = reinterpret_cast<float*>(smem + p.off_red);
    const int nthreads = W * 32;
    for (int m = 0; m < mcount; ++m) {
        const float* xr = p.x + (size_t)(m0 + m) * p.ldx;
        float inv = 1.0f;
        if (p.gamma) {
            float ss = 0.0f;
            for (int i = tid * 4; i < K; i += nthreads * 4) {
                const float4 v = *reinterpret_cast<const float4*>(xr + i);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            named_barrier(1, nthreads);
            float total = 0.0f;
            for (int i = 0; i < W; ++i) total += red[i];
            inv = rsqrtf(total / (float)K + p.eps);  // rms_norm.cu:17
            named_barrier(1, nthreads);
        }
        for (int g = warp * 4 + (lane >> 3); g < K / 32; g += W * 4) {
            const int e = g * 32 + (lane & 7) * 4;
            float4 v = *reinterpret_cast<const float4*>(xr + e);
            if (p.gamma) {
                const float4 gm = *reinterpret_cast<const float4*>(p.gamma + e);
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
            const int b = e >> 8, r16 = (e & 255) >> 4, o = e & 15;
            if (xq4) *reinterpret_cast<uint32_t*>(xq4 + m * K + b * 256 + perm_q4(r16) + o) = word;
            if (xq6) *reinterpret_cast<uint32_t*>(xq6 + m * K + b * 256 + perm_q6(r16) + o) = word;
            if ((lane & 3) == 0) xsum[m * (K / 16) + (e >> 4)] = run;
            if ((lane & 7) == 0) xs[m * (K / 32) + g] = amax / 127.0f;  // matmul.cu:18
        }
    }
    named_barrier(1, nthreads);

    // ---------------- consumers: rows ----------------
    float best_score = -__int_as_float(0x7f800000);
    uint32_t best_index = 0xffffffffu;
    int seg = 0;
    for (int i = warp, row = r_begin + warp; row < r_end; i += W, row += W) {
        const int slot = (i / W) % S, use = i / (W * S);
        // every lane waits; the warp leaves together if any lane gave up
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(full + warp * S + slot, use & 1, p.err, ERR_WAIT_TIMEOUT_FULL)))
            break;
        while (seg + 1 < p.nseg && row >= p.seg_start[seg + 1]) ++seg;
        const int jseg = JR == 2 ? 0 : seg;
        const int local = row - p.seg_start[jseg];
        const uint8_t* buf = bufs + (size_t)(warp * S + slot) * p.slot_bytes;
        const uint8_t* rows[JR];
#pragma unroll
        for (int r = 0; r < JR; ++r) rows[r] = buf + r * p.row_bytes[jseg];
        float acc[JR][MT];
#pragma unroll
        for (int r = 0; r < JR; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;
        const int chunks = p.nb * 8;
        if (p.seg[jseg].type == Q4K_TYPE_Q4_K) {
#pragma unroll(MT <= 2 ? 2 : 1)
            for (int f = lane; f < chunks; f += 32) q4_chunk<MT, JR>(rows, f, xq4, xs, xsum, K, mcount, acc);
        } else {
#pragma unroll(MT <= 2 ? 2 : 1)
            for (int f = lane; f < chunks; f += 32) q6_chunk<MT, JR>(rows, p.nb, f, xq6, xs, xsum, K, mcount, acc);
        }
#pragma unroll
        for (int r = 0; r < JR; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[r][m] = warp_sum(acc[r][m]);
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(empty + warp * S + slot);
            float* y = p.seg[jseg].y;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m >= mcount) break;
                float* out = y ? y + (size_t)(m0 + m) * p.ldy + local : nullptr;
                if (p.epilogue == EPI_STORE) {
                    *out = acc[0][m];
                } else if (p.epilogue == EPI_ADD) {
                    *out += acc[0][m];
                } else if (p.epilogue == EPI_SWIGLU) {
                    const float g = acc[0][m], u = acc[JR - 1][m];
                    *out = (g / (1.0f + expf(-g))) * u;  // silu_multiply.cu:9-10
                } else {
                    if (out) *out = acc[0][m];
                    if (candidate_better(acc[0][m], (uint32_t)local, best_score, best_index)) {
                        best_score = acc[0][m];
                        best_index = (uint32_t)local;
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
        if (lane == 0) {
            s_score[warp] = best_score;
            s_index[warp] = best_index;
        }
        named_barrier(1, nthreads);
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
        named_barrier(1, nthreads);
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
}

template <int MT, int JR>
cudaError_t launch_instance(const GemvPlan& plan, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl) {
    static std::once_flag once;
    static cudaError_t attr_status = cudaSuccess;
    std::call_once(once, [] {
        attr_status = cudaFuncSetAttribute(gemv_kernel<MT, JR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           227 * 1024);
    });
    if (attr_status != cudaSuccess) return attr_status;
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
    return cudaLaunchKernelEx(&cfg, gemv_kernel<MT, JR>, plan);
}

int align_up(int v, int a) { return (v + a - 1) / a * a; }

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
    p.nseg = rq.nseg;
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
    bool need_q4 = false, need_q6 = false;
    int max_row = 0, total = 0;
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
        p.seg_start[s] = total;
        if (!pair || s == 0) total += g.rows;
    }
    p.seg_start[rq.nseg] = total;
    if (pair) p.seg_start[1] = total;  // both segments index the same rows
    p.total_rows = total;
    p.ldy = rq.ldy ? rq.ldy : rq.seg[0].rows;

    // Batch tile: as many activation rows as fit in ~48 KB of shared memory.
    const int per_row_x = (need_q4 ? rq.K : 0) + (need_q6 ? rq.K : 0) + rq.K / 32 * 4 + rq.K / 16 * 4;
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
    p.off_xsum = off;
    off += MT * (rq.K / 16) * 4;
    p.off_red = off;
    off += 64 * 4;
    off = align_up(off, 128);

    const int JR = pair ? 2 : 1;
    p.slot_bytes = align_up(max_row * JR, 128);
    // Consumer warps and per-warp ring depth within ~110 KB (so that two
    // products can be resident on one SM while one drains and the next
    // prefetches), never fewer than 2 buffers per warp.
    const int budget = std::max(110 * 1024 - off, 0);
    int W = 8, S = budget / (W * p.slot_bytes);
    while (S < 2 && W > 2) {
        W >>= 1;
        S = budget / (W * p.slot_bytes);
    }
    S = std::min(S, 4);
    if (S < 1) S = 1;
    if (off + W * S * p.slot_bytes + 2 * W * S * 8 > 227 * 1024) return cudaErrorInvalidValue;
    p.stages = S;
    p.off_bufs = off;
    off += W * S * p.slot_bytes;
    p.off_bars = off;
    off += 2 * W * S * 8;
    const size_t smem = (size_t)off;

    int ctas = rq.ctas > 0 ? rq.ctas : sm_count();
    ctas = std::min(ctas, total);
    if (rq.epilogue == EPI_ARGMAX) ctas = std::min(ctas, 1024);
    const dim3 grid(ctas, (rq.M + MT - 1) / MT), block((W + 1) * 32);

    switch (MT * 4 + JR) {
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
