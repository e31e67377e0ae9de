// Decode engine: resident weights, fp16 KV cache, one CUDA graph per step,
// optional tensor parallelism over NCCL (one process per GPU).
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

#include <stdexcept>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/q4k_b200.h"
#include "decode_step.h"
#include "ops.h"

namespace q4k {

// Errors carry the C-ABI status they map to.
struct Error : std::runtime_error {
    int status;
    Error(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

void cuda_check(cudaError_t e, const char* what);

struct TensorSpec {
    std::string name;
    int type = 0;
    int64_t ne0 = 0, ne1 = 0;
    int layer = -1;  // -1: global tensor
    int slot = 0;    // 0..10 per layer; 0: output_norm, 1: token_embd for globals
};

// The synthetic Q4_K_M model's tensor list (q4k_model_tensor).
std::vector<TensorSpec> model_tensors(const q4k_engine_config& c);

// Part of a GGUF tensor that tensor-parallel rank `rank` of `world` holds:
// rows [n0, n1) and super-blocks [b0, b1) of every row.
struct TensorSlice {
    int64_t n0, n1, b0, b1;
};
TensorSlice tp_slice(const q4k_engine_config& c, const TensorSpec& t, int rank, int world);

class Engine {
public:
    Engine(const q4k_engine_config& cfg, const void* nccl_id);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    void load_synthetic(uint64_t seed);
    void set_tensor(const std::string& name, int type, int64_t ne0, int64_t ne1, const void* host_gguf);
    void fill_kv_synthetic(uint64_t seed, int n);
    void read_kv(int layer, uint16_t* k_host, uint16_t* v_host);
    void write_kv(int layer, const uint16_t* k_host, const uint16_t* v_host);
    uint32_t decode(uint32_t token, int position, float* logits_host, float* hidden_host);
    void generate(uint32_t token, int position, int steps, int advance, uint32_t* tokens_host);
    // A whole prompt at positions position .. position+n-1 (Engine.cpp:37-114
    // with tokens = n): every layer as batched products over the prompt rows,
    // the K/V rows written to the cache, the output head on the last row.
    // Returns the greedy next token.
    uint32_t prefill(const uint32_t* tokens_host, int n, int position, float* logits_host, int seq = 0);
    // One decode step for n tokens of n distinct sequences (tp_world == 1):
    // the products over all n rows, attention over each sequence's cache.
    void decode_batch(int n, const int* seqs, const uint32_t* tokens, const int* positions, uint32_t* next_host,
                      float* logits_host);
    // One block on a given residual-stream input (tp_world == 1 or all ranks).
    void layer_step(int layer, const float* x_host, int position, float* x_out_host);
    // One block of a prefill pass on given rows: n rows at positions
    // position .. position+n-1 of sequence seq (the products and attention
    // of prefill()), x_host [n][hidden] in, x_out_host [n][hidden] out.
    void layer_rows(int layer, int seq, int n, int position, const float* x_host, float* x_out_host);
    // One block of a batched decode step on given rows (decode_batch()'s
    // products and attention): row i at positions[i] of sequence seqs[i].
    void layer_batch(int layer, int n, const int* seqs, const int* positions, const float* x_host,
                     float* x_out_host);
    // Failure handling under tensor parallelism. device_wait_ns bounds every
    // in-kernel wait for another rank's partial sums (0 keeps the current
    // limit); host_wait_ms bounds how long a synchronous call waits for the
    // stream (0: no limit), after which the communicator is aborted and the
    // call fails with Q4K_ETIMEOUT. abort() may be called from any thread
    // (a watchdog that learnt a peer is gone): it aborts the communicator,
    // a synchronous call waiting on the stream returns Q4K_ETIMEOUT, and
    // every later call fails. The device limit is captured into the decode
    // graph, which is rebuilt on the next step.
    void set_limits(uint64_t device_wait_ns, int host_wait_ms);
    void abort();
    bool aborted() const { return aborted_.load(); }
    // One step with every kernel CTA's %globaltimer start/end recorded.
    size_t trace_step(uint32_t token, int position, unsigned long long* records_host, size_t max_records);
    cudaStream_t stream() const { return stream_; }
    const q4k_engine_config& config() const { return c_; }

private:
    struct Layer {
        float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *ffn_norm = nullptr;
        uint8_t *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *gate = nullptr, *up = nullptr, *down = nullptr;
        int tq = 0, tk = 0, tv = 0, to = 0, tgate = 0, tup = 0, tdown = 0;
    };
    using Slice = TensorSlice;

    void* alloc(size_t bytes);
    Slice shard_of(const TensorSpec& t) const;
    void** tensor_slot(const TensorSpec& t, int** type_slot);
    void place(const TensorSpec& t, const void* raw_device);
    void enqueue_step(bool record_hidden);
    // fused: the row-parallel sums go through the peer receive slots (the
    // decode step); otherwise through ncclAllReduce (layer_step)
    void enqueue_layer(int i, bool fused);
    // Tensor parallelism without a collective launch (tp_world > 1): maps
    // every rank's receive slots into this process (cudaIpc over NCCL).
    void setup_peer_slots();
    unsigned long long* peer_recv(int rank, int slot) const;  // rank's slot, [world][hidden] (value, tag) words
    void enqueue_head(bool fused);
    // Prompt rows per prefill pass and their buffers (allocated on first use).
    void ensure_prefill();
    void enqueue_prefill_layer(int i, int rows, int pos0, int seq);
    void ensure_prefill_maps();
    // One product over r.M rows: the tensor-core GEMM (with the given weight
    // maps) from pf_gemm_min_rows_ rows, else the batched GEMV.
    void enqueue_product(GemvRequest& r, const KvTensorMap* wmaps);
    const KvTensorMap* layer_maps(int layer, int slot) const;
    void ensure_batch();
    void enqueue_batch_layer(int i, int n, int splits);
    // Checks a batched step's rows and stages seqs / positions on the
    // device; returns the attention split count for them.
    int stage_batch(int n, const int* seqs, const uint32_t* tokens, const int* positions);
    // L2 prefetch descriptors of layer i's weights (q, k, v; o; gate, up; down).
    L2Prefetch weight_prefetch(const uint8_t* w, int type, int K, int rows) const;
    // the K and V cache rows 0..*pos_ of every KV head of `layer` (sequence 0), into f[0] and f[1]
    void kv_prefetch(int layer, L2Prefetch* f) const;
    void check_device_error(bool with_token = false);
    void ensure_graph();
    // Persistent decode-step kernel (tp_world == 1): one launch per token.
    void ensure_step_plan();
    void enqueue_step_kernel();

    q4k_engine_config c_;
    int rank_ = 0, world_ = 1;
    int Hl_ = 0, KVHl_ = 0, qd_ = 0, kvd_ = 0;
    int64_t ffn_b0_ = 0, ffn_b1_ = 0;
    int ffn_l_ = 0;
    int64_t vocab0_ = 0, vocab1_ = 0;
    int splits_ = 1;
    bool loaded_ = false;
    std::vector<bool> have_;

    cudaStream_t stream_ = nullptr;
    ncclComm_t comm_ = nullptr;
    std::vector<void*> allocations_;
    std::vector<Layer> layers_;
    float* output_norm_ = nullptr;
    uint8_t* token_embd_ = nullptr;
    int t_embd_ = 0;

    float *x_ = nullptr, *qkv_ = nullptr, *att_ = nullptr, *act_ = nullptr, *partial_ = nullptr,
          *logits_ = nullptr, *hidden_ = nullptr;
    // io_ (device) word layout; host_io_ (pinned) holds the words going in
    // at the same indices and those coming back from kHostOut on
    static constexpr int kIoToken = 0, kIoPos = 1, kIoAdvance = 2, kIoHistoryN = 3, kIoIn = 4, kIoErr = 4;
    static constexpr int kHostOut = 8;
    uint32_t* io_ = nullptr;
    void stage_io(uint32_t token, int position, uint32_t advance);
    uint32_t* token_ = nullptr;     // device: token to embed (and the step's result)
    int* pos_ = nullptr;            // device: position of the token
    int* advance_ = nullptr;        // device: position increment per step
    uint32_t* history_ = nullptr;   // device: generated tokens
    unsigned* history_n_ = nullptr; // device: count
    int* err_ = nullptr;
    uint16_t *kcache_ = nullptr, *vcache_ = nullptr;
    KvTensorMap kmap_{}, vmap_{};
    float *attn_part_o_ = nullptr, *attn_part_ml_ = nullptr;
    unsigned* attn_counters_ = nullptr;
    float* am_score_ = nullptr;
    uint32_t* am_index_ = nullptr;
    unsigned* am_counter_ = nullptr;
    float* tp_cand_local_ = nullptr;  // [2] score, index (as float bits)
    float* tp_cand_all_ = nullptr;    // [2 * world]
    uint32_t* host_io_ = nullptr;     // pinned: token, position, result

    int seqs_ = 1;             // KV caches held (sequences)
    size_t seq_elems_ = 0;     // fp16 elements of one sequence's K (or V) cache
    // decode_batch buffers (up to b_cap_ tokens per step)
    int b_cap_ = 0;
    float *b_x_ = nullptr, *b_qkv_ = nullptr, *b_att_ = nullptr, *b_act_ = nullptr, *b_logits_ = nullptr;
    float *b_part_o_ = nullptr, *b_part_ml_ = nullptr;
    unsigned* b_counters_ = nullptr;
    int *b_pos_ = nullptr, *b_seq_ = nullptr;
    uint32_t *b_tok_ = nullptr, *b_next_ = nullptr;
    float* b_partial_ = nullptr;   // tp_world > 1: row-parallel partial sums [B][hidden]
    uint32_t* b_cand_ = nullptr;   // tp_world > 1: [B] (score bits, global index) of this rank's head shard
    uint32_t* b_cand_all_ = nullptr;  // [world][B][2]
    KvTensorMap pf_head_map_[kPrefillWeightMaps];  // token_embd as the output head

    int pf_rows_ = 0;  // prompt rows one prefill pass holds
    uint32_t* pf_tokens_ = nullptr;
    float *pf_x_ = nullptr, *pf_qkv_ = nullptr, *pf_q_ = nullptr, *pf_att_ = nullptr, *pf_act_ = nullptr,
          *pf_partial_ = nullptr;
    bool pf_gemm_ = true;        // the tensor-core GEMM is available (prefill_gemm.cu)
    int pf_gemm_min_rows_ = 9;   // passes of fewer rows use the batched GEMV
    bool pf_maps_ready_ = false;  // pf_wmaps_ matches the placed tensors
    std::vector<KvTensorMap> pf_wmaps_;  // per layer: q, k, v, o, gate, up, down
    KvTensorMap pf_amap_[3];     // pf_a_ with K = hidden, q width, ffn width
    uint16_t* pf_a_ = nullptr;   // fp16 activation operand [2][rows][max K] (hi, lo planes)
    float* pf_gsum_ = nullptr;   // its 32-value group sums [rows][max K / 32]
    float* pf_rs_ = nullptr;     // its row scales
    float* pf_part_ = nullptr;   // split-K partial sums of the GEMM
    size_t pf_part_floats_ = 0;

    // Fused tensor-parallel sums (decode step): slot 2i takes layer i's
    // attn_output partial sums, 2i + 1 its ffn_down ones, from every rank;
    // one cudaMalloc per rank ([slots][world][hidden] words), mapped by the
    // others. xb_ is the second residual buffer (x_ and xb_ in turn).
    bool tp_fused_ = false;
    uint8_t* ar_base_ = nullptr;
    void* ar_peer_[8] = {};  // every rank's allocation (this rank's own at rank_)
    int* ar_epoch_ = nullptr;  // decode steps run, as every rank counts them
    float* xb_ = nullptr;
    cudaGraphExec_t exec_ = nullptr;
    uint64_t dev_wait_ns_ = 2000000000ull;  // in-kernel waits for other ranks' partial sums
    int host_wait_ms_ = 0;                  // synchronous calls under tensor parallelism (0: unbounded)
    std::atomic<bool> aborted_{false};
    std::mutex abort_mu_;                   // one ncclCommAbort, whichever thread gets there first
    bool comm_aborted_ = false;
    void host_wait(const char* what);
    void require_live() const;       // stream drained, bounded by host_wait_ms_ when world_ > 1
    // L2 prefetch plan. 1: each launch asks for the next launch's operands.
    // 2 (default, +0.8%): the attention launch also asks for the gate/up
    // weights and O for nothing: O is short, and a grid is complete only once
    // its prefetches are, so a 28 MB prefetch issued by O delayed gate/up's
    // dependency wait (1.66 -> 1.09 us). Moving more (the next layer's K/V
    // rows to ffn_down, its q/k/v weights to gate/up) measured 4.5% slower.
    int prefetch_plan_ = 2;
    bool l2_prefetch_ = true;        // each launch prefetches the next one's operands into L2
    bool act_images_ = true;         // SwiGLU and attention hand the next product a quantised activation
    ActImage act_img_, att_img_;     // quantised act_ (for ffn_down) and att_ (for attn_output)
    bool step_kernel_ = false;       // decode with decode_step.cu instead of the launch sequence
    bool step_ready_ = false;        // step_phases_ matches the placed tensors
    int step_ctas_ = 0;
    int step_splits_ = 0;
    int step_nphases_ = 0;
    StepPhase* step_phases_ = nullptr;  // device
    unsigned* step_sync_ = nullptr;     // device, [nphases + 1]
    unsigned long long* trace_ = nullptr;      // set only while a traced graph is captured
    unsigned long long* trace_buf_ = nullptr;
};

}  // namespace q4k
