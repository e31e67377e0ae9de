// Checks the branch-free Q8 quantisation helpers of gemv_device.cuh against
// CUDA's own IEEE operations (test infrastructure):
//   q8_scale(a)       == a / 127.0f            for every non-negative float
//                                              bit pattern (2^31 values,
//                                              infinities and NaNs included)
//   q8_code_r(v, ra)  == roundf((v / a) * 127) for every mantissa of a at
//                                              exponents across the float range
//                                              (subnormal included), with v
//                                              drawn at and beside the code
//                                              boundaries (k + 0.5) a / 127 and
//                                              at random
// Prints the mismatch counts and exits non-zero if any is found.
#include <cstdio>
#include <cstdint>

#include "gemv_device.cuh"

using namespace q4k::gemv_dev;

__device__ unsigned long long g_bad_scale, g_bad_code, g_checked;

__device__ __forceinline__ int8_t code_ieee(float v, float amax) {
    return amax == 0.0f ? 0 : static_cast<int8_t>(roundf(__fmul_rn(__fdiv_rn(v, amax), 127.0f)));
}

__global__ void scale_kernel(uint32_t base) {
    const uint32_t bits = base + blockIdx.x * blockDim.x + threadIdx.x;  // bits < 2^31: sign 0
    const float a = __uint_as_float(bits);
    const float want = __fdiv_rn(a, 127.0f), got = q8_scale(a);
    const bool same = __float_as_uint(want) == __float_as_uint(got) || (isnan(want) && isnan(got));
    if (!same) atomicAdd(&g_bad_scale, 1ull);
}

__device__ __forceinline__ uint32_t mix(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// one thread per (mantissa, exponent): 48 values v for that amax
__global__ void code_kernel(int exp_field) {
    const uint32_t mant = blockIdx.x * blockDim.x + threadIdx.x;  // < 2^23
    const uint32_t bits = exp_field == 0 ? (mant ? mant : 1u) : ((uint32_t)exp_field << 23) | mant;
    const float amax = __uint_as_float(bits);
    const double ra = recip_refined(amax);
    unsigned long long bad = 0;
    for (int s = 0; s < 48; ++s) {
        const uint32_t h = mix(bits * 48u + (uint32_t)s);
        float v;
        if (s < 40) {
            // at or beside a boundary: (k + 0.5) * amax / 127, nudged by 0..3 ulps either way
            const int k = (int)(h % 127u);
            float b = __fmul_rn(__fdiv_rn((float)k + 0.5f, 127.0f), amax);
            const int nudge = (int)((h >> 8) % 7u) - 3;
            b = __uint_as_float(__float_as_uint(b) + nudge);
            v = fminf(b, amax);
        } else {
            v = __fmul_rn(amax, (float)(h >> 8) * (1.0f / 16777216.0f));
        }
        if ((h >> 31) & 1u) v = -v;
        if (code_ieee(v, amax) != q8_code_r(v, ra)) ++bad;
    }
    if (bad) atomicAdd(&g_bad_code, bad);
    atomicAdd(&g_checked, 48ull);
}

int main() {
    unsigned long long zero = 0, bad_scale = 0, bad_code = 0, checked = 0;
    cudaMemcpyToSymbol(g_bad_scale, &zero, sizeof zero);
    cudaMemcpyToSymbol(g_bad_code, &zero, sizeof zero);
    cudaMemcpyToSymbol(g_checked, &zero, sizeof zero);
    const uint32_t per_launch = 1u << 26;
    for (uint32_t base = 0; base < (1u << 31); base += per_launch) scale_kernel<<<per_launch / 256, 256>>>(base);
    // exponent fields: subnormal, the smallest normals, around 1, the largest
    const int exps[] = {0, 1, 2, 20, 60, 100, 126, 127, 128, 160, 200, 240, 253, 254};
    for (int e : exps) code_kernel<<<(1u << 23) / 256, 256>>>(e);
    const cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        std::printf("CUDA error: %s\n", cudaGetErrorString(err));
        return 2;
    }
    cudaMemcpyFromSymbol(&bad_scale, g_bad_scale, sizeof bad_scale);
    cudaMemcpyFromSymbol(&bad_code, g_bad_code, sizeof bad_code);
    cudaMemcpyFromSymbol(&checked, g_checked, sizeof checked);
    std::printf("scale: 2147483648 checked, %llu mismatches; codes: %llu checked, %llu mismatches\n", bad_scale,
                checked, bad_code);
    return bad_scale == 0 && bad_code == 0 ? 0 : 1;
}
