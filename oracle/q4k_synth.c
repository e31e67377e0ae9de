/* Seeded synthetic tensors for the CPU oracle and the reference arm.
 *
 * TEST INFRASTRUCTURE ONLY (tests/, smoke() and bench.py's CPU legs): it
 * lets the CPU baseline build the benchmark's model without loading the
 * product library. It restates, from their definitions, the seeded streams
 * the product library generates its synthetic model from, so both sides see
 * identical bytes (tests/test_oracle.py compares them over whole tensors):
 *
 *   key(seed, name) = mix(seed ^ FNV-1a-64(name)), mix = the splitmix64
 *                     finaliser (shifts 30/27/31, multipliers below);
 *   word(key, i)    = mix(key + (i + 1) * golden-ratio increment);
 *   normal(key, i)  = Irwin-Hall: the twelve 16-bit fields of words
 *                     3i, 3i+1, 3i+2 summed, minus 12 * 32767.5, over 65536;
 *   Q4_K block b    = fp16(|normal(hk, 2b)| * 2e-3), fp16(|normal(hk, 2b+1)|
 *                     * 2e-3) for d and dmin (hk = mix(key ^ "HDR-KEY1")),
 *                     then bytes 4..143 from words 18b .. 18b+17 (little
 *                     endian, the last word cut to 4 bytes);
 *   Q6_K block b    = bytes 0..191 from words 26b .. 26b+23, the 16 int8
 *                     scales from the low 6 bits of the bytes of words
 *                     26b+24, 26b+25 minus 32, d = fp16(|normal(hk, b)| * 1e-3);
 *   gamma i         = 1 + 0.02 * normal(key, i); KV fill = fp16(normal(key, i)).
 *
 * Blocks are numbered row-major over the whole tensor (GGUF layout).
 */
#include "q4k_oracle.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static uint64_t syn_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t syn_word(uint64_t key, uint64_t i) { return syn_mix(key + (i + 1) * 0x9E3779B97F4A7C15ull); }

static double syn_normal(uint64_t key, uint64_t i) {
    uint64_t sum = 0;
    for (uint64_t k = 0; k < 3; ++k) {
        uint64_t w = syn_word(key, 3 * i + k);
        for (int f = 0; f < 4; ++f, w >>= 16) sum += w & 0xffffu;
    }
    return ((double)sum - 12.0 * 32767.5) / 65536.0;
}

uint64_t orc_synth_key(uint64_t seed, const char* name) {
    uint64_t h = 0xcbf29ce484222325ull; /* FNV-1a 64 offset basis */
    for (const unsigned char* s = (const unsigned char*)name; *s; ++s) h = (h ^ *s) * 0x100000001b3ull;
    return syn_mix(seed ^ h);
}

static uint64_t syn_header_key(uint64_t key) { return syn_mix(key ^ 0x4844522D4B455931ull); }

static void syn_le_bytes(uint8_t* dst, uint64_t w, int n) {
    for (int i = 0; i < n; ++i) dst[i] = (uint8_t)(w >> (8 * i));
}

static uint16_t syn_abs_half(double v, double sigma) { return orc_float_to_half((float)(fabs(v) * sigma)); }

static void syn_q4k_block(uint64_t key, uint64_t b, uint8_t* blk) {
    const uint64_t hk = syn_header_key(key);
    const uint16_t d = syn_abs_half(syn_normal(hk, 2 * b), 2e-3);
    const uint16_t dmin = syn_abs_half(syn_normal(hk, 2 * b + 1), 2e-3);
    syn_le_bytes(blk, d, 2);
    syn_le_bytes(blk + 2, dmin, 2);
    for (int k = 0; k < 18; ++k) syn_le_bytes(blk + 4 + 8 * k, syn_word(key, 18 * b + (uint64_t)k), k < 17 ? 8 : 4);
}

static void syn_q6k_block(uint64_t key, uint64_t b, uint8_t* blk) {
    for (int k = 0; k < 24; ++k) syn_le_bytes(blk + 8 * k, syn_word(key, 26 * b + (uint64_t)k), 8);
    for (int k = 0; k < 2; ++k) {
        const uint64_t w = syn_word(key, 26 * b + 24 + (uint64_t)k);
        for (int i = 0; i < 8; ++i) blk[192 + 8 * k + i] = (uint8_t)(int8_t)((int)((w >> (8 * i)) & 63u) - 32);
    }
    syn_le_bytes(blk + 208, syn_abs_half(syn_normal(syn_header_key(key), b), 1e-3), 2);
}

int orc_synth_tensor(uint64_t seed, const char* name, int type, int64_t ne0, int64_t ne1, void* out) {
    if (!name || !out || ne0 <= 0 || ne1 <= 0) return 1;
    const uint64_t key = orc_synth_key(seed, name);
    if (type == ORC_F32) {
        float* f = (float*)out;
        for (int64_t i = 0; i < ne0 * ne1; ++i) f[i] = (float)(1.0 + 0.02 * syn_normal(key, (uint64_t)i));
        return 0;
    }
    if ((type != ORC_Q4_K && type != ORC_Q6_K) || ne0 % 256) return 1;
    const int64_t blocks = ne0 / 256 * ne1;
    uint8_t* p = (uint8_t*)out;
    if (type == ORC_Q4_K) {
#pragma omp parallel for schedule(static)
        for (int64_t b = 0; b < blocks; ++b) syn_q4k_block(key, (uint64_t)b, p + b * 144);
    } else {
#pragma omp parallel for schedule(static)
        for (int64_t b = 0; b < blocks; ++b) syn_q6k_block(key, (uint64_t)b, p + b * 210);
    }
    return 0;
}

void orc_synth_f16(uint64_t seed, const char* name, uint64_t index_base, size_t n, uint16_t* out) {
    const uint64_t key = orc_synth_key(seed, name);
    for (size_t i = 0; i < n; ++i) out[i] = orc_float_to_half((float)syn_normal(key, index_base + i));
}

void orc_synth_f32(uint64_t seed, const char* name, size_t n, float* out) {
    const uint64_t key = orc_synth_key(seed, name);
    for (size_t i = 0; i < n; ++i) out[i] = (float)syn_normal(key, i);
}

int orc_omp_threads(int requested) {
    int used = 1;
#ifdef _OPENMP
    if (requested > 0) {
#pragma omp parallel num_threads(requested)
        {
#pragma omp single
            used = omp_get_num_threads();
        }
    } else {
#pragma omp parallel
        {
#pragma omp single
            used = omp_get_num_threads();
        }
    }
#else
    (void)requested;
#endif
    return used;
}
