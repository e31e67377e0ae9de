/*
 * q4k_b200 — C ABI of the B200 (sm_100a) Qwen3-4B Q4_K_M decode hot path.
 *
 * Plain pointers and sizes only. Device pointers are CUDA device addresses
 * on the current device; `stream` is a cudaStream_t (NULL = legacy default
 * stream, as the reference's kernels use). Every function returns a status:
 *
 *   Q4K_OK (0)        success
 *   Q4K_EINVAL (1)    invalid argument   (the reference throws std::invalid_argument)
 *   Q4K_ERANGE (2)    size/capacity out of range (std::out_of_range / std::length_error)
 *   Q4K_ECUDA (3)     CUDA launch/runtime failure (std::runtime_error from check_launch)
 *   Q4K_ETIMEOUT (4)  a bounded wait gave up: inside a kernel (another rank's
 *                     partial sums, a copy that never landed) or on the host
 *                     (a tensor-parallel step that did not complete in time);
 *                     no counterpart in the reference, which has no waits
 *
 * and q4k_last_error() returns the calling thread's last message. Kernels
 * are asynchronous on `stream` unless stated otherwise; zero-size work
 * returns Q4K_OK without launching (the reference's behaviour).
 *
 * Reference paths below are relative to the poytaytoy/Qwen3-4B-Q4_K_M-
 * Inference-Engine source tree.
 */
#ifndef Q4K_B200_H
#define Q4K_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q4K_OK 0
#define Q4K_EINVAL 1
#define Q4K_ERANGE 2
#define Q4K_ECUDA 3
#define Q4K_ETIMEOUT 4

/* GGML tensor type ids (the GGUF file's values). */
#define Q4K_TYPE_F32 0
#define Q4K_TYPE_F16 1
#define Q4K_TYPE_Q4_K 12
#define Q4K_TYPE_Q6_K 14

/* Epilogues of q4k_matmul_ex. */
#define Q4K_EPI_STORE 0  /* y = W x                                   */
#define Q4K_EPI_ADD 1    /* y += W x (residual update)                */
#define Q4K_EPI_SWIGLU 2 /* y = silu(W0 x) * (W1 x), two weights      */
#define Q4K_EPI_ARGMAX 3 /* *token = argmax_n (W x)[n]; y optional    */

const char* q4k_last_error(void);
int q4k_abi_version(void);

/* ---------------------------------------------------------------- weights */

/* Device bytes of a tensor with ne0 inputs per row and ne1 rows in this
 * library's device layout (Q4_K: GGUF rows verbatim; Q6_K: per-row planar
 * re-layout of the same bytes; F32: as is). Replaces the size the
 * reference's Weight computes from the GGUF tensor (src/Weight.cpp:53-61). */
size_t q4k_weight_device_bytes(int type, int64_t ne0, int64_t ne1);

/* Copies a tensor given in GGUF file layout (host memory) into `device`
 * (q4k_weight_device_bytes(type, ne0, ne1) bytes, 16-byte aligned) in the
 * device layout. Replaces Weight::Weight(const GGUF&, name) +
 * DeviceBuffer(src, bytes) (src/Weight.cpp:6-23, :53-61); synchronises
 * `stream` before returning, as DeviceBuffer does. */
int q4k_weight_upload(int type, int64_t ne0, int64_t ne1, const void* host_gguf, void* device, void* stream);

/* Deterministic synthetic tensor `name` (seed, GGUF layout) into host memory
 * (ne1 * GGUF row bytes). Replaces GGUF::read_tensor_data for the model file
 * the tests use (src/GGUF.cpp:131-145); no counterpart in the reference's
 * arithmetic. */
int q4k_synth_tensor_host(uint64_t seed, const char* name, int type, int64_t ne0, int64_t ne1, void* host_gguf);

/* The same tensor generated on the device directly in the device layout. */
int q4k_synth_tensor_device(uint64_t seed, const char* name, int type, int64_t ne0, int64_t ne1, void* device,
                            void* stream);

/* Elements [index_base, index_base + n) of the fp16 N(0,1) stream `name`
 * (the KV-cache fill), and elements [0, n) of the fp32 N(0,1) stream
 * `name` (synthetic activations), on the host or the device. */
int q4k_synth_f16_host(uint64_t seed, const char* name, uint64_t index_base, size_t n, uint16_t* out);
int q4k_synth_f32_host(uint64_t seed, const char* name, size_t n, float* out);
int q4k_synth_f32_device(uint64_t seed, const char* name, size_t n, float* out, void* stream);

/* ------------------------------------------------ kernels (Kernels.hpp) */

/* kernels::rms_norm (include/Kernels.hpp:54-55, src/cuda/rms_norm.cu:30-39).
 * `scale` is the F32 gamma of `width` floats. */
int q4k_rms_norm(const float* input, const float* scale, float* output, size_t rows, size_t width, float epsilon,
                 void* stream);

/* kernels::matmul (include/Kernels.hpp:57-61, src/cuda/matmul.cu:130-166).
 * weight: device layout of a Q4_K/Q6_K tensor, ne0 = K inputs (multiple of
 * 256), ne1 = N output rows (only rows [0, ne1) are read). input [rows][K],
 * output [rows][N]. The activation is quantised to Q8 in the kernel (no
 * workspace), so concurrent calls on different streams are independent. */
int q4k_matmul(const float* input, const void* weight, int type, int64_t ne0, int64_t ne1, float* output,
               size_t rows, void* stream);

/* kernels::rope (include/Kernels.hpp:63-64, src/cuda/rope.cu:32-39). */
int q4k_rope(float* input, size_t tokens, size_t heads, size_t head_dim, size_t position_offset, float frequency_base,
             void* stream);

/* kernels::attention (include/Kernels.hpp:66-68, src/cuda/attention.cu:94-110):
 * fp32 causal GQA, q/output [tokens][query_heads][head_dim], k/v
 * [query_offset + tokens][kv_heads * head_dim], head_dim in [1, 256]. */
int q4k_attention(const float* q, const float* k, const float* v, float* output, size_t tokens, size_t query_heads,
                  size_t kv_heads, size_t head_dim, size_t query_offset, void* stream);

/* kernels::residual_add (include/Kernels.hpp:70, src/cuda/residual_add.cu:15-20). */
int q4k_residual_add(float* state, const float* branch, size_t count, void* stream);

/* kernels::silu_multiply (include/Kernels.hpp:72, src/cuda/silu_multiply.cu:15-23). */
int q4k_silu_multiply(const float* gate, const float* up, float* output, size_t count, void* stream);

/* kernels::dequantize_embeddings (include/Kernels.hpp:74-75,
 * src/cuda/embedding.cu:65-84): rows of GGUF-layout packed data (row_bytes
 * apart) to fp32, bit-identical to the reference. */
int q4k_dequantize_embeddings(const void* packed, float* output, size_t rows, size_t width, size_t row_bytes,
                              int type, void* stream);

/* kernels::argmax (include/Kernels.hpp:77, src/cuda/argmax.cu:72-98):
 * largest logit, lowest index on ties; synchronises and writes *result on
 * the host, as the reference does. */
int q4k_argmax(const float* logits, size_t vocabulary_size, uint32_t* result, void* stream);

/* ------------------------------------------ fused entry points (new) */

/* Fused product over 1..4 weights sharing one activation (the reference
 * issues one kernels::matmul per weight, src/Engine.cpp:83-85, :98-101).
 * norm_gamma (optional, K floats): RMSNorm the input rows first
 * (rms_norm.cu fused in). epilogue: Q4K_EPI_*. For SWIGLU pass two weights
 * (gate, up) and one output; for ARGMAX one weight, rows == 1, outputs[0]
 * optional logits, *token_device receives the index, and `scratch` must be
 * q4k_matmul_argmax_scratch_bytes() bytes zeroed once before first use. */
int q4k_matmul_ex(const float* input, const float* norm_gamma, float epsilon, int count, const void* const* weights,
                  const int* types, const int64_t* out_rows, float* const* outputs, int64_t ne0, size_t rows,
                  int epilogue, uint32_t* token_device, void* scratch, void* stream);
size_t q4k_matmul_argmax_scratch_bytes(void);

/* The same products for many activation rows (the reference's
 * kernels::matmul with rows = n prompt tokens, src/Engine.cpp:83-101) on the
 * tensor cores (tcgen05, fp32 accumulation in tensor memory). Each row is
 * Q8-quantised as the reference does (after RMSNorm with norm_gamma, if
 * given); the codes times their scales enter the tensor cores as fp16 hi +
 * lo parts against the exact integer products of the weight codes and
 * sub-block scales, and each super-block's d / dmin are applied in fp32, so
 * a product stays within ~1e-6 of the reference's integer dots.
 * count: 1..3 weights; outputs[i][m * ld_out + n] (SWIGLU: two weights of one
 * type and shape, output in outputs[0]). epilogue: Q4K_EPI_STORE, _ADD or
 * _SWIGLU. ne0 <= 10240. Allocates its workspace on the stream. Its kernels
 * launch with programmatic dependent launch: the first may start while the
 * stream's previous kernel runs, but reads its inputs (and writes its
 * outputs) only after that kernel has completed. */
int q4k_matmul_batch(const float* input, const float* norm_gamma, float epsilon, int count, const void* const* weights,
                     const int* types, const int64_t* out_rows, float* const* outputs, int64_t ld_out, int64_t ne0,
                     size_t rows, int epilogue, void* stream);

/* Decode attention for one token over an fp16 KV cache (new): fuses the
 * per-head q/k RMSNorm (src/Engine.cpp:87-88), RoPE (:89-90), the K/V cache
 * write and split-K attention (:92). qkv = [q | k | v] raw projections of
 * the token; caches are [kv_heads][capacity][128] fp16 for one layer;
 * *position_device is the token's position. head_dim must be 128,
 * query_heads == 4 * kv_heads and kv_heads <= 64 (the scratch's 256-byte
 * counter block). scratch: q4k_attention_decode_scratch_bytes
 * bytes, 16-byte aligned; the call clears its counter block on `stream`
 * before launching. The kernel's waits on its tile copies are bounded
 * (2 s): if one gives up, `output` is undefined, and this asynchronous
 * call does not report it (the decode engine reads such timeouts back
 * through its error word). */
int q4k_attention_decode_f16(const float* qkv, const float* q_gamma, const float* k_gamma, uint16_t* k_cache,
                             uint16_t* v_cache, int capacity, const int* position_device, int query_heads,
                             int kv_heads, int head_dim, float epsilon, float rope_base, float* output,
                             void* scratch, void* stream);
size_t q4k_attention_decode_scratch_bytes(int query_heads, int kv_heads);

/* No counterpart in the reference. q4k_attention_decode_f16 without a
 * scratch argument, for callers that may not allocate device memory: the
 * scratch is a fixed 1 MiB array in the library's device memory (one per
 * device), so nothing is allocated. Limit: 256 + 520 * query_heads * splits
 * bytes must fit in 1 MiB (2016 head-splits; with the default one CTA per SM
 * a B200 needs 592), else Q4K_ERANGE; at most 64 KV heads. The first call on
 * a device (with it current) looks up the array's address and should come
 * before any stream capture; the address is kept for the life of the
 * process, so resetting the device (cudaDeviceReset) after that first call
 * is not supported. Every call clears the per-head counters on
 * `stream` before launching. Calls on one device share the array: calls that
 * can overlap in time race and must be ordered by the caller. */
int q4k_attention_decode_f16_static(const float* qkv, const float* q_gamma, const float* k_gamma, uint16_t* k_cache,
                                    uint16_t* v_cache, int capacity, const int* position_device, int query_heads,
                                    int kv_heads, int head_dim, float epsilon, float rope_base, float* output,
                                    void* stream);

/* ------------------------------------------------------- decode engine */

/* Replaces Engine / ChatSession (src/Engine.cpp:14-114,
 * include/ChatSession.hpp:10-52) for the decode hot path: all weights and an
 * fp16 KV cache resident on one GPU (or sharded over tp_world GPUs, one
 * process each), the layer loop captured as one CUDA graph per step. */
typedef struct q4k_engine q4k_engine;

typedef struct {
    int layers, hidden, heads, kv_heads, head_dim, ffn, vocab;
    float eps, rope_base;
    int capacity; /* KV-cache positions */
    int tp_rank, tp_world;
    int device;
    /* Independent KV caches (sequences; ChatSession.hpp:10-52 each) the
     * engine holds; 0 or 1: one. The single-sequence calls work on
     * sequence 0; q4k_engine_prefill_seq and q4k_engine_decode_batch
     * address any of them. */
    int sequences;
} q4k_engine_config;

/* Qwen3-4B: 36 layers, 2560 hidden, 32/8 heads of 128, ffn 9728, vocab
 * 151936, eps 1e-6, rope base 1e6. */
void q4k_engine_config_qwen3_4b(q4k_engine_config* cfg, int capacity);

/* Tensor i (0 <= i < 11*layers + 2) of the model: GGUF name, type and
 * shape (ne0 inputs, ne1 rows) of the Q4_K_M synthetic model (Q6_K for
 * attn_v, the ffn_down of even layers and token_embd). Returns Q4K_ERANGE
 * past the end. */
int q4k_model_tensor(const q4k_engine_config* cfg, int i, char* name, size_t name_len, int* type, int64_t* ne0,
                     int64_t* ne1);

/* Rows [n0, n1) and super-blocks [b0, b1) of tensor i that rank `rank` of
 * `world` holds (Megatron-style: q/k/v/gate/up split by rows, attn_output
 * and ffn_down by whole super-blocks of their inputs, norms and token_embd
 * replicated). No reference counterpart: the reference runs on one GPU. */
int q4k_tp_shard(const q4k_engine_config* cfg, int i, int rank, int world, int64_t* n0, int64_t* n1, int64_t* b0,
                 int64_t* b1);

/* nccl_id: 128 bytes from q4k_nccl_unique_id on rank 0, shared by the
 * caller (NULL when tp_world == 1). */
int q4k_nccl_unique_id(void* id128);
int q4k_engine_create(const q4k_engine_config* cfg, const void* nccl_id, q4k_engine** out);
int q4k_engine_destroy(q4k_engine* engine);

/* Weights: all synthetic (device-generated, identical bytes to
 * q4k_synth_tensor_host), or one tensor at a time from GGUF-layout host
 * memory (this rank's shard is cut out here). */
int q4k_engine_load_synthetic(q4k_engine* engine, uint64_t seed);
int q4k_engine_set_tensor(q4k_engine* engine, const char* name, int type, int64_t ne0, int64_t ne1,
                          const void* host_gguf);

/* KV cache: positions [0, n) of every layer filled with fp16 N(0,1):
 * element (head, pos, d) of layer L is element
 * (head * 2^20 + pos) * 128 + d of stream "kv.{L}.k" / "kv.{L}.v"
 * (q4k_synth_f16_host), heads counted over all kv_heads. read_kv copies one
 * layer's [kv_heads/tp_world][capacity][128] K and V back to the host. */
int q4k_engine_fill_kv_synthetic(q4k_engine* engine, uint64_t seed, int n);
int q4k_engine_read_kv(q4k_engine* engine, int layer, uint16_t* k_host, uint16_t* v_host);
/* Replaces one layer's K/V (same layout as read_kv; either may be NULL),
 * e.g. to resume a saved session (ChatSession's cache, ChatSession.hpp:30-44). */
int q4k_engine_write_kv(q4k_engine* engine, int layer, const uint16_t* k_host, const uint16_t* v_host);

/* One decode step (Engine::inference for one new token, src/Engine.cpp:37-114):
 * embeds `token` at `position`, runs every layer and the output head, and
 * returns the greedy next token. logits_host (vocab floats, this rank's
 * shard when tp_world > 1; may be NULL) and hidden_host ((layers+1) * hidden
 * floats: the residual stream after the embedding and after each layer; may
 * be NULL, only with tp_world == 1) are optional. Synchronous. */
int q4k_engine_decode(q4k_engine* engine, uint32_t token, int position, uint32_t* next_token, float* logits_host,
                      float* hidden_host);

/* A whole prompt (Engine::inference's pass over the session's uncached
 * tokens, src/Engine.cpp:37-114 with tokens = n): embeds tokens[0..n) at
 * positions position .. position+n-1, runs every layer over all n rows
 * (batched products, causal GQA attention over the cache, the n K/V rows
 * written to the cache) and the output head on the last row only
 * (Engine.cpp:106-111). Returns the greedy next token; logits_host as for
 * q4k_engine_decode. Decoding continues at position + n. Token ids >= vocab
 * and position + n > capacity are Q4K_ERANGE. Synchronous. */
int q4k_engine_prefill(q4k_engine* engine, const uint32_t* tokens, int n, int position, uint32_t* next_token,
                       float* logits_host);

/* q4k_engine_prefill into sequence `seq` (0 <= seq < sequences). */
int q4k_engine_prefill_seq(q4k_engine* engine, int seq, const uint32_t* tokens, int n, int position,
                           uint32_t* next_token, float* logits_host);

/* One decode step for n tokens of n distinct sequences at once (the
 * reference serves one session per Engine::inference call; batching many
 * sequences into one step reads every weight once for all of them):
 * tokens[i] is embedded at positions[i] of sequence seqs[i]; next_tokens[i]
 * receives its greedy successor. The products run over all n rows (the
 * batched GEMV up to 8 rows, the tensor-core GEMM above), attention over
 * each sequence's own cache. logits_host (n x vocab floats; this rank's
 * vocabulary shard of each row when tp_world > 1) may be NULL. With
 * tp_world > 1 every rank calls it with the same rows: the row-parallel
 * sums are all-reduced and each row's greedy token is merged over the
 * ranks' head shards (lowest index on ties). 1 <= n <= min(sequences, 512).
 * Synchronous. */
int q4k_engine_decode_batch(q4k_engine* engine, int n, const int* seqs, const uint32_t* tokens, const int* positions,
                            uint32_t* next_tokens, float* logits_host);

/* `steps` greedy decode steps with the token fed back on the device; one
 * graph launch per step and no host synchronisation between steps.
 * advance != 0: position increases by one per step; advance == 0: every
 * step decodes at `position` again (fixed context). tokens_host receives
 * the `steps` generated tokens (may be NULL). Synchronous at the end. */
int q4k_engine_generate(q4k_engine* engine, uint32_t token, int position, int steps, int advance,
                        uint32_t* tokens_host);

/* One transformer block (src/Engine.cpp:71-103) applied to a given residual
 * stream x_host (hidden floats) for a token at `position`, result in
 * x_out_host; writes that layer's K/V row at `position`. For checking a
 * layer against another implementation on identical inputs. Synchronous. */
int q4k_engine_layer(q4k_engine* engine, int layer, const float* x_host, int position, float* x_out_host);

/* One transformer block of a prompt pass (src/Engine.cpp:71-103 with
 * tokens = n, as q4k_engine_prefill runs it: the products over all rows on
 * the tensor cores from 9 rows up) applied to given residual-stream rows
 * x_host [n][hidden] at positions position .. position+n-1 of sequence
 * `seq`; result in x_out_host [n][hidden]; writes the n K/V rows. n is at
 * most one prefill pass (512 rows). For checking a layer of the GEMM path
 * against another implementation on identical inputs. With tp_world > 1
 * every rank calls it (the row-parallel sums are all-reduced). Synchronous. */
int q4k_engine_layer_rows(q4k_engine* engine, int layer, int seq, int n, int position, const float* x_host,
                          float* x_out_host);

/* One transformer block of a batched decode step (q4k_engine_decode_batch's
 * products and per-sequence attention) on given rows: row i of x_host
 * [n][hidden] is the token at positions[i] of sequence seqs[i]; result in
 * x_out_host; writes each row's K/V. The reference serves each sequence as
 * its own session (Engine.cpp:71-103 per ChatSession). Synchronous. */
int q4k_engine_layer_batch(q4k_engine* engine, int layer, int n, const int* seqs, const int* positions,
                           const float* x_host, float* x_out_host);

/* Stream the engine launches on (cudaStream_t), e.g. to time with events. */
void* q4k_engine_stream(q4k_engine* engine);

/* Failure handling under tensor parallelism (no reference counterpart: the
 * reference runs on one GPU). device_wait_ns bounds every wait inside a
 * kernel for another rank's partial sums (default 2 s; 0 keeps the current
 * value): a wait that gives up makes the call fail with Q4K_ETIMEOUT, and
 * the kernels return, so the context stays usable. host_wait_ms bounds how
 * long a synchronous call waits for its step when tp_world > 1 (default 0:
 * no bound); past it the engine aborts its NCCL communicator and the call
 * fails with Q4K_ETIMEOUT. q4k_engine_abort may be called from any thread,
 * e.g. by a watchdog that learnt a peer process is gone: a call waiting on
 * the step returns Q4K_ETIMEOUT, and every later call on this engine fails
 * with Q4K_ETIMEOUT (destroy it and create a new one). */
int q4k_engine_set_limits(q4k_engine* engine, uint64_t device_wait_ns, int host_wait_ms);
int q4k_engine_abort(q4k_engine* engine);

/* The receiving side of the engine's fused tensor-parallel sum, on its own
 * (no reference counterpart). parts holds `world` slots of `count` 8-byte
 * words, slot r written by rank r: word i = (tag << 32) | bits of rank r's
 * partial sum i. Waits (bounded by wait_ns) until every word carries `tag`,
 * then out[i] = residual[i] + (slot 0 + slot 1 + ... in rank order) in fp32
 * (residual may be NULL: zero). count a multiple of 4, 1 <= world <= 8,
 * 16-byte aligned buffers; err_device is one int of device memory the call
 * clears. Synchronous: returns Q4K_ETIMEOUT if a wait gave up (out is then
 * undefined), Q4K_OK otherwise. */
int q4k_tp_sum_parts(const void* parts, int world, int64_t count, uint32_t tag, const float* residual, float* out,
                     uint64_t wait_ns, int* err_device, void* stream);

/* ------------------------------------------------------ GGUF model files */

/* A GGUF model file (format versions 2 and 3), mapped read-only: replaces
 * the reference's loader (src/GGUF.cpp:81-145) and its metadata reads
 * (src/Engine.cpp:49-55). Host-only: none of these touch a GPU except
 * q4k_engine_load_gguf. Opening fails with Q4K_EINVAL on a file that is not
 * well-formed GGUF (bad magic, truncation, tensors off their alignment or
 * past the end). */
typedef struct q4k_gguf q4k_gguf;
int q4k_gguf_open(const char* path, q4k_gguf** out);
int q4k_gguf_close(q4k_gguf* file);
int q4k_gguf_tensor_count(const q4k_gguf* file, int64_t* count);
/* Tensor i: name, ggml type, ne0 and ne1 (the product of the other
 * extents), and a pointer to its bytes inside the mapping (valid until
 * q4k_gguf_close). Q4K_ERANGE past the end. */
int q4k_gguf_tensor_info(const q4k_gguf* file, int64_t i, char* name, size_t name_len, int* type, int64_t* ne0,
                         int64_t* ne1, const void** data);
/* Metadata by key; Q4K_ERANGE when the key is absent or of another kind
 * (any integer type reads as int, any number as float). */
int q4k_gguf_meta_int(const q4k_gguf* file, const char* key, int64_t* value);
int q4k_gguf_meta_float(const q4k_gguf* file, const char* key, double* value);
int q4k_gguf_meta_string(const q4k_gguf* file, const char* key, char* value, size_t len);
/* Engine configuration from the metadata the reference reads
 * (Engine.cpp:49-55) under arch = general.architecture: {arch}.block_count,
 * .embedding_length, .attention.head_count, .attention.head_count_kv,
 * .attention.key_length (else hidden / heads), .feed_forward_length,
 * .attention.layer_norm_rms_epsilon, .rope.freq_base; vocab = rows of
 * token_embd.weight; the given KV capacity; one GPU (tp fields as for a
 * single device, device 0). */
int q4k_gguf_engine_config(const q4k_gguf* file, int capacity, q4k_engine_config* cfg);
/* Loads every tensor the engine needs from the file (this rank's shard when
 * tp_world > 1), checking name, shape and type: F32 norms, Q4_K or Q6_K
 * matrices (ffn_gate and ffn_up of a layer of one type). output.weight, if
 * present, is not used: the output head is token_embd.weight, as in the
 * reference. */
int q4k_engine_load_gguf(q4k_engine* engine, const q4k_gguf* file);

/* Diagnostics, no counterpart in the reference: one decode step (like
 * q4k_engine_decode) whose kernels store %globaltimer nanoseconds into a
 * [256 launches][1024 CTAs][8 slots] array of words: launch 5*layer + k
 * (k: 0 QKV, 1 attention, 2 O, 3 gate/up, 4 down), 5*layers the output
 * head; slot 0 a CTA's start, 7 its end, 1..6 kernel checkpoints; 0 where
 * nothing was recorded. Products: 1 dependency wait returned, 5 first
 * activation load landed, 2 activation quantised (or its image copied),
 * 3 first stage landed, 4 stages done, 6 output image written (SwiGLU).
 * Attention: 1 query ready, 2 / 3 first / last tile landed, 4 partials
 * written; the CTA that merged a head also records 3 (last split seen),
 * 5 (merge inputs loaded) and 6. Up to max_records words go to
 * records_host; *count receives how many. */
int q4k_engine_trace(q4k_engine* engine, uint32_t token, int position, unsigned long long* records_host,
                     size_t max_records, size_t* count);

#ifdef __cplusplus
}
#endif
#endif
