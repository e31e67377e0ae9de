/* CPU oracle for the Qwen3-4B Q4_K/Q6_K decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference
 * engine's arithmetic, used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py as the checker. The product library never
 * links, loads or calls it.
 *
 * Every function cites the reference file:line whose behaviour it restates
 * (paths relative to the poytaytoy/Qwen3-4B-Q4_K_M-Inference-Engine tree).
 * Weights are passed in the GGUF file layout (raw 144-byte Q4_K and 210-byte
 * Q6_K super-blocks, row-major, dimension[0] = K inputs per row).
 */
#ifndef Q4K_ORACLE_H
#define Q4K_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_K = 12, ORC_Q6_K = 14 };

float orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f);

/* embedding.cu:14-31 / :42-58 — one 256-value super-block to fp32. */
void orc_dequant_block_q4k(const uint8_t* block, float* out);
void orc_dequant_block_q6k(const uint8_t* block, float* out);

/* embedding.cu:65-84 (kernels::dequantize_embeddings) — rows of packed data. */
int orc_dequantize_rows(const void* packed, float* out, size_t rows, size_t width, size_t row_bytes, int type);

/* matmul.cu:8-22 (quantize) == MatmulReference.hpp:11-29: int8 codes and one
 * fp32 scale per 32 values; count must be a multiple of 32. */
void orc_quantize_q8(const float* x, size_t count, int8_t* codes, float* scales);

/* MatmulReference.hpp:42-64: Q8-quantise x, decode each weight row to fp32,
 * accumulate in double. y is [rows][N] (matmul.cu:123 output order).
 * OpenMP over output rows with `threads` threads (<= 0: all). */
int orc_matmul(const float* x, const void* weight, int type, size_t K, size_t N, size_t rows, double* y, int threads);

/* rms_norm.cu:6-24 — y = x * rsqrt(mean(x^2) + eps) * gamma, per row. */
void orc_rms_norm(const float* x, const float* gamma, float* y, size_t rows, size_t width, float eps);

/* rope.cu:7-24 — NeoX split-half rotation in place. */
void orc_rope(float* x, size_t tokens, size_t heads, size_t head_dim, size_t position_offset, float base);

/* attention.cu:23-91, AttentionReference.hpp:13-88 — causal GQA softmax(q.k/sqrt(d)).v
 * q/out: [tokens][heads][d]; k/v: [offset+tokens][kv_heads][d] (row stride
 * kv_heads*d). Query token t sits at absolute position offset + t. */
int orc_attention(const float* q, const float* k, const float* v, float* out, size_t tokens, size_t heads,
                  size_t kv_heads, size_t head_dim, size_t offset);

/* silu_multiply.cu:6-13 and residual_add.cu:6-9. */
void orc_silu_multiply(const float* gate, const float* up, float* out, size_t count);
void orc_residual_add(float* state, const float* branch, size_t count);

/* argmax.cu:25-98 — largest logit, lowest index on ties, NaN never wins;
 * UINT32_MAX when no logit beats -inf. */
uint32_t orc_argmax(const float* logits, size_t count);

/* One Engine::inference call (Engine.cpp:37-114) over `tokens` new tokens at
 * positions [pos, pos+tokens). Tensors are indexed layer*ORC_SLOTS + slot,
 * then ORC_SLOTS*layers + {0: output_norm, 1: token_embd}. K/V caches are
 * fp32 [layers][capacity][kv_heads*head_dim]; rows [0, pos) must hold the
 * prefix. If kv_round_f16 != 0 every new K/V row is rounded to fp16 as it is
 * stored (the fp16-KV configuration). logits (vocab floats, last token) and
 * hidden ([layers+1][hidden], last token's residual stream after the
 * embedding and after every layer) are optional outputs. */
enum {
    ORC_ATTN_NORM = 0, ORC_Q = 1, ORC_K = 2, ORC_V = 3, ORC_Q_NORM = 4, ORC_K_NORM = 5,
    ORC_O = 6, ORC_FFN_NORM = 7, ORC_GATE = 8, ORC_UP = 9, ORC_DOWN = 10, ORC_SLOTS = 11
};

typedef struct {
    int layers, hidden, heads, kv_heads, head_dim, ffn, vocab;
    float eps, rope_base;
    const void* const* tensors; /* ORC_SLOTS*layers + 2 pointers */
    const int* types;           /* same indexing */
} orc_model;

/* One block (Engine.cpp:71-103) on given rows x [tokens][hidden], updated in
 * place, at positions pos .. pos+tokens-1; k_cache / v_cache are this
 * layer's fp32 caches [capacity][kv_heads*head_dim] (rows [0, pos) the
 * prefix; the new rows are written, rounded to fp16 if kv_round_f16). */
int orc_layer(const orc_model* model, int layer, float* x, float* k_cache, float* v_cache, size_t capacity,
              size_t tokens, size_t pos, int kv_round_f16, int threads);

int orc_forward(const orc_model* model, float* k_cache, float* v_cache, size_t capacity, const uint32_t* token_ids,
                size_t tokens, size_t pos, int kv_round_f16, float* logits, float* hidden, uint32_t* next_token,
                int threads);

/* Seeded synthetic tensors (q4k_synth.c): the benchmark model's bytes
 * without the product library. orc_synth_tensor writes a GGUF-layout
 * Q4_K/Q6_K tensor or an F32 RMSNorm gamma (ne0 * ne1 values); the f16/f32
 * streams are the KV fill and synthetic activations. Returns 0 or 1 (bad
 * request). orc_omp_threads reports the threads an OpenMP region asked for
 * `requested` (<= 0: the default) actually gets. */
uint64_t orc_synth_key(uint64_t seed, const char* name);
int orc_synth_tensor(uint64_t seed, const char* name, int type, int64_t ne0, int64_t ne1, void* out);
void orc_synth_f16(uint64_t seed, const char* name, uint64_t index_base, size_t n, uint16_t* out);
void orc_synth_f32(uint64_t seed, const char* name, size_t n, float* out);
int orc_omp_threads(int requested);

#ifdef __cplusplus
}
#endif
#endif
