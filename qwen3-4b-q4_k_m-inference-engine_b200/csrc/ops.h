// Launchers for the non-GEMV kernels (ops.cu, attention_decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "q4k_internal.h"

namespace q4k {

cudaError_t rms_norm(const float* x, const float* gamma, float* y, size_t rows, size_t width, float eps,
                     cudaStream_t s);
cudaError_t rope(float* x, size_t tokens, size_t heads, size_t head_dim, size_t pos, float base, cudaStream_t s);
cudaError_t attention_f32(const float* q, const float* k, const float* v, float* out, size_t tokens, size_t heads,
                          size_t kv_heads, size_t head_dim, size_t offset, cudaStream_t s);
cudaError_t residual_add(float* state, const float* branch, size_t count, cudaStream_t s);
cudaError_t silu_multiply(const float* gate, const float* up, float* out, size_t count, cudaStream_t s);
// out = residual + sum over ranks of tagged partial sums (q4k_tp_sum_parts)
cudaError_t tp_sum_parts(const unsigned long long* parts, int world, size_t count, unsigned tag,
                         const float* residual, float* out, unsigned long long wait_ns, int* err, cudaStream_t s);
cudaError_t dequantize_raw(const void* packed, float* out, size_t rows, size_t width, size_t row_bytes, int type,
                           cudaStream_t s);
cudaError_t embed_rows(const void* table, int type, size_t width, size_t vocab, const uint32_t* tokens, size_t count,
                       float* out, int* err, cudaStream_t s, bool pdl);
size_t argmax_scratch_bytes();
cudaError_t argmax(const float* logits, size_t count, uint32_t* result, void* scratch, cudaStream_t s);
// Rows [n0, n1), super-blocks [b0, b1) of a GGUF-layout matrix with K_full
// inputs into the device layout (Q4_K verbatim, Q6_K planar).
cudaError_t relayout(const void* raw, int type, size_t K_full, size_t n0, size_t n1, size_t b0, size_t b1,
                     void* out, cudaStream_t s);
// Synthetic quantised matrix in GGUF layout (q4k_format.h generator).
cudaError_t synth_raw(uint64_t key, int type, size_t K, size_t N, void* out, cudaStream_t s);
cudaError_t synth_gamma(uint64_t key, float* out, size_t n, cudaStream_t s);
cudaError_t synth_f32(uint64_t key, float* out, size_t n, cudaStream_t s);
cudaError_t synth_f16(uint64_t key, uint16_t* out, size_t n, size_t index_base, cudaStream_t s);

// Split-K flash-decode attention over an fp16 KV cache for one new token,
// with the per-head QK RMSNorm and RoPE of that token fused in, and the new
// K/V row written into the cache (attention_decode.cu).
struct DecodeAttnArgs {
    const float* qkv;          // [H*D | KVH*D | KVH*D] raw projections of the new token
    const float* q_gamma;      // [D]
    const float* k_gamma;      // [D]
    uint16_t* k_cache;         // [KVH][capacity][D] fp16 (this layer)
    uint16_t* v_cache;         // [KVH][capacity][D] fp16
    int row_base;              // row of (this layer, head 0, position 0) in the tensor maps
    int capacity;
    const int* position;       // device scalar: index of the new token
    int heads, kv_heads;       // head_dim is 128
    float eps, rope_base;
    float* partial_o;          // [KVH][splits][G][D]
    float* partial_ml;         // [KVH][splits][G][2]
    unsigned* counters;        // [KVH], zero before the first launch; reset by the kernel
    float* out;                // [H*D] attended output
    int* err;
    int splits;                // CTAs per KV head
    unsigned long long* trace = nullptr;  // optional timeline records
    int trace_tag = 0;
    L2Prefetch prefetch[kMaxPrefetch];    // the next kernel's operands (optional)
    ActImage out_image;                   // optional: the attended output, quantised for the O product
    // Batched decode (one new token in each of `batch` sequences): qkv, out,
    // position, partial_o / partial_ml and counters hold one row / block per
    // token (qkv rows ld_qkv floats apart); token z's cache is that of
    // sequence seq_of[z] (z if null), seq_cache_elems fp16 elements per
    // sequence from k_cache / v_cache and from row_base in the tensor maps.
    int batch = 1;
    const int* seq_of = nullptr;
    int ld_qkv = 0;
    long long seq_cache_elems = 0;
};
constexpr int kDecodeHeadDim = 128;

// Prompt prefill (prefill.cu): M tokens at positions pos0 .. pos0+M-1.
struct PrefillQkArgs {
    const float* qkv = nullptr;  // [M][ld_qkv]: q (heads x 128) | k (kv_heads x 128) | v (kv_heads x 128)
    int ld_qkv = 0;
    const float* q_gamma = nullptr;  // [128]
    const float* k_gamma = nullptr;  // [128]
    float* q_out = nullptr;          // [M][heads x 128]: normed, rotated queries
    uint16_t* k_cache = nullptr;     // [kv_heads][capacity][128] fp16 (this layer)
    uint16_t* v_cache = nullptr;
    int capacity = 0, pos0 = 0, heads = 0, kv_heads = 0;
    float eps = 1e-6f, rope_base = 1e6f;
};
// Per token and head: QK RMSNorm and RoPE; for KV heads, K and V appended to the cache.
cudaError_t prefill_qk(const PrefillQkArgs& a, int tokens, cudaStream_t s);

// Opaque storage of a TMA tensor map (CUtensorMap); make_kv_tensor_map's
// views an fp16 KV cache as [rows][128]: 64-row x 64-dim boxes, 128-byte
// swizzle.
struct alignas(64) KvTensorMap {
    unsigned char bytes[128];
};
struct PrefillAttnArgs {
    const float* q = nullptr;             // [M][heads x 128]
    const uint16_t* k_cache = nullptr;    // [kv_heads][capacity][128] fp16, rows 0 .. pos0+M-1 written
    const uint16_t* v_cache = nullptr;
    float* out = nullptr;                 // [M][heads x 128]
    int capacity = 0, pos0 = 0, heads = 0, kv_heads = 0;
    // Optional: TMA maps of the whole cache (make_kv_tensor_map) and the map
    // row of this layer's KV head 0, position 0; with them and 4 query heads
    // per KV head the tensor-core kernel runs.
    const KvTensorMap* kmap = nullptr;
    const KvTensorMap* vmap = nullptr;
    int row_base = 0;
    int* err = nullptr;
};
// Causal GQA attention of every prompt token over cache positions 0 .. its own.
cudaError_t prefill_attention(const PrefillAttnArgs& a, int tokens, cudaStream_t s);
// Prompt-prefill products on the tensor cores (prefill_gemm.cu).
//
// prefill_quantise: each of M activation rows (optionally RMSNorm-ed with
// gamma) is Q8-quantised as the reference does (per 32 values, scale
// amax/127, code roundf(x/amax*127)); v = code * (scale / row_scale[m]),
// row_scale[m] being the row's largest group scale (|v| <= 127), is stored
// as fp16 hi and lo parts: a [2][a_rows][K] (hi plane, then lo plane), and
// gsum[m][g] = the sum of v over 32-value group g ([M][K / 32]).
cudaError_t prefill_quantise(const float* x, int ldx, const float* gamma, float eps, int M, int K, uint16_t* a,
                             int a_rows, float* gsum, float* row_scale, cudaStream_t s);
struct PrefillGemmSegment {
    const uint8_t* w = nullptr;  // device layout rows (q4k_format.h)
    int type = 0;                // Q4K_TYPE_Q4_K or Q4K_TYPE_Q6_K
    int rows = 0;
    float* y = nullptr;          // y[m * ldy + n]
};
struct PrefillGemmArgs {
    PrefillGemmSegment seg[3];
    // Prebuilt TMA maps (make_weight_map: kPrefillWeightMaps per segment;
    // make_act_map), or nullptr to encode them for this call. An activation
    // map may cover more rows than M.
    const KvTensorMap* wmap[3] = {nullptr, nullptr, nullptr};
    const KvTensorMap* amap = nullptr;
    int nseg = 0;
    int K = 0, M = 0, ldy = 0;
    int epilogue = 0;                 // EPI_STORE, EPI_ADD or EPI_SWIGLU (segments 0, 1 paired; output in seg[0].y)
    const uint16_t* a = nullptr;      // prefill_quantise output [2][rows of amap][K]
    const float* row_scale = nullptr;  // [M]
    const float* gsum = nullptr;       // [M][K / 32] (prefill_quantise)
    float* partial = nullptr;          // optional split-K workspace (STORE / ADD / SWIGLU products)
    size_t partial_floats = 0;
    int* err = nullptr;
};
// y = row_scale * sum over super-blocks of (d P - dmin mins . gsum), P the
// tensor-core product of a (hi + lo) with the exact integer weights.
cudaError_t prefill_gemm(const PrefillGemmArgs& g, cudaStream_t s);
// Floats of split-K workspace prefill_gemm would use for g's shapes given
// unlimited room (0: it would not split).
size_t prefill_gemm_partial_floats(const PrefillGemmArgs& g);
// TMA maps of the GEMM's operands: a weight matrix's raw rows as 64-row
// boxes (kPrefillWeightMaps maps written to out: one per Q4_K block or Q6_K
// plane width); the fp16 activation operand [2][rows][K] (hi and lo planes)
// as 64 x 128-row boxes of one plane, 128-byte swizzle.
constexpr int kPrefillWeightMaps = 3;
cudaError_t make_weight_map(const uint8_t* w, int type, int K, int rows, KvTensorMap* out);
cudaError_t make_act_map(const uint16_t* a, int K, int rows, KvTensorMap* out);
// cuTensorMapEncodeTiled from the driver (nullptr if unavailable).
void* tensor_map_encoder();
cudaError_t make_kv_tensor_map(const uint16_t* base, long long rows, KvTensorMap* out);
int decode_attention_splits(int kv_heads);
size_t decode_attention_scratch_floats(int heads, int kv_heads, int splits);
cudaError_t decode_attention(const DecodeAttnArgs& a, const KvTensorMap& kmap, const KvTensorMap& vmap,
                             cudaStream_t s, bool pdl);
// This device's fixed scratch for q4k_attention_decode_f16_static
// (attention_static_scratch.cu); throws q4k::Error if `need` does not fit.
void* attention_static_scratch(size_t need);
size_t attention_static_scratch_capacity();

}  // namespace q4k
