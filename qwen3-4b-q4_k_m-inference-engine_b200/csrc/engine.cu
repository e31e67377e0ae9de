// Qwen3 decode engine (replaces Engine::inference / ChatSession of the
// reference for one new token per step: src/Engine.cpp:37-114,
// include/ChatSession.hpp:10-52).
//
// Per step, on one stream, captured once as a CUDA graph:
//   embed            token row of token_embd -> x            (EmbedLookup.cpp:49-78)
//   per layer:
//     gemv  QKV      rmsnorm(x, attn_norm) -> q|k|v          (Engine.cpp:82-85)
//     attention      q/k norm + RoPE + KV write + split-K     (Engine.cpp:87-92)
//     gemv  O        x += W_o att                            (Engine.cpp:94-95)
//     gemv  gate/up  act = silu(W_g n) * (W_u n), n = rmsnorm(x, ffn_norm)  (:97-100)
//     gemv  down     x += W_d act                            (Engine.cpp:101-102)
//   gemv  head       rmsnorm(x, output_norm), W_embd, argmax (Engine.cpp:105-111)
//   finish           record the token, advance the position
// Every kernel after the first is launched with programmatic stream
// serialisation, so each product's weight stream starts while its
// predecessor drains. With tp_world > 1 the projections are sharded
// Megatron-style and the row-parallel outputs are summed with NCCL.
#include "engine.h"

#include <cuda_runtime.h>
#include <math_constants.h>

#include <dlfcn.h>

#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <chrono>
#include <thread>
#include "nccl_api.h"

#include "ops.h"
#include "q4k_device.cuh"
#include "q4k_internal.h"

namespace q4k {

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Error(Q4K_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

static void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) throw Error(Q4K_ECUDA, std::string(what) + ": " + nccl().GetErrorString(r));
}

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    static std::string failure;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            failure = std::string("NCCL is not available: ") + dlerror();
            return;
        }
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        if (!api.GetUniqueId || !api.CommInitRank || !api.CommDestroy || !api.AllReduce || !api.AllGather ||
            !api.GetErrorString)
            failure = "NCCL library lacks a required symbol";
    });
    if (!failure.empty()) throw Error(Q4K_ECUDA, failure);
    return api;
}

namespace {

constexpr uint64_t kKvIndexStride = 1ull << 20;  // positions per head in the KV generator's index space

const char* const kSlotNames[11] = {"attn_norm", "attn_q",     "attn_k",   "attn_v",   "attn_q_norm", "attn_k_norm",
                                    "attn_output", "ffn_norm", "ffn_gate", "ffn_up",   "ffn_down"};

__global__ void finish_step_kernel(uint32_t* token, int* pos, const int* advance, uint32_t* history,
                                   unsigned* history_n, unsigned history_cap, const uint32_t* tp_cand, int world,
                                   int* epoch) {
    pdl_wait();
    if (threadIdx.x != 0) return;
    if (tp_cand) {
        // Greedy choice over the shards (argmax.cu ordering): larger logit,
        // then lower index.
        float bs = __uint_as_float(tp_cand[0]);
        uint32_t bi = tp_cand[1];
        for (int r = 1; r < world; ++r) {
            const float s = __uint_as_float(tp_cand[2 * r]);
            const uint32_t i = tp_cand[2 * r + 1];
            if (candidate_better(s, i, bs, bi)) {
                bs = s;
                bi = i;
            }
        }
        *token = bi;
    }
    const unsigned n = *history_n;
    if (n < history_cap) history[n] = *token;
    *history_n = n + 1;
    *pos += *advance;
    if (epoch) *epoch += 1;  // a decode step that used the peer receive slots
}

// Greedy token of each of n logit rows (argmax.cu:25-98 semantics: the
// largest value, the lowest index among equals). With `cand` set (a head
// sharded over tensor-parallel ranks) row r's best also goes to cand[2r]
// (score bits) and cand[2r+1] (index + index_base) for the cross-rank merge.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* logits, int vocab, uint32_t* out,
                                                           uint32_t* cand, uint32_t index_base) {
    const float* row = logits + (size_t)blockIdx.x * vocab;
    float bs = -CUDART_INF_F;
    uint32_t bi = 0xFFFFFFFFu;
    // four running candidates per thread over 16-byte loads keep several
    // loads in flight per thread (one CTA per row streams its 0.6 MB row);
    // candidate_better orders ties by index, so the merge order is free
    const int n4 = (reinterpret_cast<uintptr_t>(row) & 15u) == 0 ? vocab / 4 : 0;
    const float4* row4 = reinterpret_cast<const float4*>(row);
    float cs[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};
    uint32_t ci[4] = {0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu};
#pragma unroll 4
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = __ldcs(row4 + i);
        const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (candidate_better(e[c], (uint32_t)(4 * i + c), cs[c], ci[c])) {
                cs[c] = e[c];
                ci[c] = (uint32_t)(4 * i + c);
            }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
        if (candidate_better(cs[c], ci[c], bs, bi)) {
            bs = cs[c];
            bi = ci[c];
        }
    for (int i = 4 * n4 + threadIdx.x; i < vocab; i += blockDim.x)
        if (candidate_better(row[i], (uint32_t)i, bs, bi)) {
            bs = row[i];
            bi = (uint32_t)i;
        }
    __shared__ float ss[32];
    __shared__ uint32_t si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float s2 = __shfl_xor_sync(0xffffffffu, bs, o);
        const uint32_t i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        if (candidate_better(s2, i2, bs, bi)) {
            bs = s2;
            bi = i2;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        ss[threadIdx.x >> 5] = bs;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (candidate_better(ss[w], si[w], bs, bi)) {
                bs = ss[w];
                bi = si[w];
            }
        out[blockIdx.x] = bi;
        if (cand) {
            cand[2 * blockIdx.x] = __float_as_uint(bs);
            cand[2 * blockIdx.x + 1] = bi == 0xFFFFFFFFu ? bi : bi + index_base;
        }
    }
}

// Greedy token of row r over the ranks' shard winners cand_all[w][r][2]:
// the larger logit, then the lower global index (argmax.cu ordering).
__global__ void merge_row_candidates_kernel(const uint32_t* cand_all, int world, int n, uint32_t* out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    float bs = __uint_as_float(cand_all[2 * r]);
    uint32_t bi = cand_all[2 * r + 1];
    for (int w = 1; w < world; ++w) {
        const float sc = __uint_as_float(cand_all[((size_t)w * n + r) * 2]);
        const uint32_t ix = cand_all[((size_t)w * n + r) * 2 + 1];
        if (candidate_better(sc, ix, bs, bi)) {
            bs = sc;
            bi = ix;
        }
    }
    out[r] = bi;
}

}  // namespace

std::vector<TensorSpec> model_tensors(const q4k_engine_config& c) {
    std::vector<TensorSpec> out;
    char buf[96];
    for (int i = 0; i < c.layers; ++i) {
        for (int s = 0; s < 11; ++s) {
            std::snprintf(buf, sizeof buf, "blk.%d.%s.weight", i, kSlotNames[s]);
            TensorSpec t;
            t.name = buf;
            t.layer = i;
            t.slot = s;
            const int64_t qd = (int64_t)c.heads * c.head_dim, kvd = (int64_t)c.kv_heads * c.head_dim;
            switch (s) {
                case 0: case 7: t.type = Q4K_TYPE_F32; t.ne0 = c.hidden; t.ne1 = 1; break;
                case 4: case 5: t.type = Q4K_TYPE_F32; t.ne0 = c.head_dim; t.ne1 = 1; break;
                case 1: t.type = Q4K_TYPE_Q4_K; t.ne0 = c.hidden; t.ne1 = qd; break;
                case 2: t.type = Q4K_TYPE_Q4_K; t.ne0 = c.hidden; t.ne1 = kvd; break;
                case 3: t.type = Q4K_TYPE_Q6_K; t.ne0 = c.hidden; t.ne1 = kvd; break;
                case 6: t.type = Q4K_TYPE_Q4_K; t.ne0 = qd; t.ne1 = c.hidden; break;
                case 8: case 9: t.type = Q4K_TYPE_Q4_K; t.ne0 = c.hidden; t.ne1 = c.ffn; break;
                case 10: t.type = (i % 2 == 0) ? Q4K_TYPE_Q6_K : Q4K_TYPE_Q4_K; t.ne0 = c.ffn; t.ne1 = c.hidden; break;
            }
            out.push_back(t);
        }
    }
    TensorSpec on;
    on.name = "output_norm.weight";
    on.type = Q4K_TYPE_F32;
    on.ne0 = c.hidden;
    on.ne1 = 1;
    on.slot = 0;
    out.push_back(on);
    TensorSpec te;
    te.name = "token_embd.weight";
    te.type = Q4K_TYPE_Q6_K;
    te.ne0 = c.hidden;
    te.ne1 = c.vocab;
    te.slot = 1;
    out.push_back(te);
    return out;
}

// Megatron-style sharding (column-parallel q/k/v/gate/up, row-parallel
// attn_output/ffn_down on whole super-blocks, replicated norms and
// token_embd; the output head's vocab rows are split in enqueue_step).
TensorSlice tp_slice(const q4k_engine_config& c, const TensorSpec& t, int rank, int world) {
    const int64_t nb = t.ne0 / 256;
    TensorSlice s{0, t.ne1, 0, nb};
    if (t.layer < 0 || world <= 1) return s;
    const int64_t qd = (int64_t)c.heads / world * c.head_dim, kvd = (int64_t)c.kv_heads / world * c.head_dim;
    const int64_t fb = c.ffn / 256, f0 = fb * rank / world, f1 = fb * (rank + 1) / world;
    switch (t.slot) {
        case 1: s.n0 = rank * qd; s.n1 = s.n0 + qd; break;
        case 2: case 3: s.n0 = rank * kvd; s.n1 = s.n0 + kvd; break;
        case 6: s.b0 = rank * qd / 256; s.b1 = s.b0 + qd / 256; break;
        case 8: case 9: s.n0 = f0 * 256; s.n1 = f1 * 256; break;
        case 10: s.b0 = f0; s.b1 = f1; break;
        default: break;
    }
    return s;
}

Engine::Engine(const q4k_engine_config& cfg, const void* nccl_id) : c_(cfg) {
    const auto& c = c_;
    if (c.layers <= 0 || c.hidden <= 0 || c.hidden % 256 || c.heads <= 0 || c.kv_heads <= 0 ||
        c.head_dim != kDecodeHeadDim || c.heads != 4 * c.kv_heads || c.ffn <= 0 || c.ffn % 256 || c.vocab <= 0 ||
        c.capacity <= 0 || !(c.eps > 0.0f) || !(c.rope_base > 0.0f))
        throw Error(Q4K_EINVAL, "unsupported engine configuration (head_dim must be 128 and heads = 4 * kv_heads)");
    world_ = c.tp_world > 0 ? c.tp_world : 1;
    rank_ = c.tp_rank;
    if (rank_ < 0 || rank_ >= world_ || c.kv_heads % world_)
        throw Error(Q4K_EINVAL, "tp_world must divide kv_heads and 0 <= tp_rank < tp_world");
    Hl_ = c.heads / world_;
    KVHl_ = c.kv_heads / world_;
    qd_ = Hl_ * c.head_dim;
    kvd_ = KVHl_ * c.head_dim;
    const int64_t fb = c.ffn / 256;
    ffn_b0_ = fb * rank_ / world_;
    ffn_b1_ = fb * (rank_ + 1) / world_;
    ffn_l_ = (int)((ffn_b1_ - ffn_b0_) * 256);
    vocab0_ = (int64_t)c.vocab * rank_ / world_;
    vocab1_ = (int64_t)c.vocab * (rank_ + 1) / world_;
    if (ffn_l_ <= 0 || qd_ % 256) throw Error(Q4K_EINVAL, "tensor-parallel shards must hold whole super-blocks");
    if (c.sequences < 0 || c.sequences > 4096) throw Error(Q4K_EINVAL, "sequences must be in 0..4096");
    seqs_ = c.sequences > 1 ? c.sequences : 1;

    cuda_check(cudaSetDevice(c.device), "cudaSetDevice");
    cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    if (world_ > 1) {
        if (!nccl_id) throw Error(Q4K_EINVAL, "tp_world > 1 needs an NCCL unique id");
        ncclUniqueId id;
        std::memcpy(&id, nccl_id, sizeof id);
        nccl_check(nccl().CommInitRank(&comm_, world_, id, rank_), "ncclCommInitRank");
    }

    layers_.resize(c.layers);
    have_.assign(11 * (size_t)c.layers + 2, false);
    splits_ = decode_attention_splits(KVHl_);
    const int H = c.hidden;
    x_ = static_cast<float*>(alloc(sizeof(float) * H));
    qkv_ = static_cast<float*>(alloc(sizeof(float) * (qd_ + 2 * kvd_)));
    att_ = static_cast<float*>(alloc(sizeof(float) * qd_));
    act_ = static_cast<float*>(alloc(sizeof(float) * ffn_l_));
    if (const char* ai = std::getenv("Q4K_ACT_IMAGE")) act_images_ = ai[0] != '0';
    if (act_images_ && ffn_l_ % 256 == 0 && qd_ % 256 == 0) {
        act_img_ = {static_cast<uint8_t*>(alloc(act_image_bytes(ffn_l_))), ffn_l_};
        att_img_ = {static_cast<uint8_t*>(alloc(act_image_bytes(qd_))), qd_};
    } else {
        act_images_ = false;
    }
    partial_ = static_cast<float*>(alloc(sizeof(float) * H));
    logits_ = static_cast<float*>(alloc(sizeof(float) * (vocab1_ - vocab0_)));
    hidden_ = static_cast<float*>(alloc(sizeof(float) * H * (c.layers + 1)));
    // the step's small device words in one block, so that a decode call
    // moves them with one copy each way: token, position, advance and the
    // history count (host -> device), token .. error word (device -> host)
    io_ = static_cast<uint32_t*>(alloc(256));
    token_ = io_ + kIoToken;
    pos_ = reinterpret_cast<int*>(io_ + kIoPos);
    advance_ = reinterpret_cast<int*>(io_ + kIoAdvance);
    err_ = reinterpret_cast<int*>(io_ + kIoErr);
    history_ = static_cast<uint32_t*>(alloc(sizeof(uint32_t) * (size_t)c.capacity));
    history_n_ = io_ + kIoHistoryN;
    // [sequence][layer][kv head][position][128]: sequence 0 first
    seq_elems_ = (size_t)c.layers * KVHl_ * c.capacity * c.head_dim;
    const size_t kv_elems = seq_elems_ * seqs_;
    if ((long long)(kv_elems / c.head_dim) >= (1ll << 31)) throw Error(Q4K_EINVAL, "KV cache too large");
    kcache_ = static_cast<uint16_t*>(alloc(kv_elems * 2));
    vcache_ = static_cast<uint16_t*>(alloc(kv_elems * 2));
    // TMA views of the whole cache: rows = sequences * layers * kv_heads * capacity
    cuda_check(make_kv_tensor_map(kcache_, (long long)(kv_elems / c.head_dim), &kmap_), "K tensor map");
    cuda_check(make_kv_tensor_map(vcache_, (long long)(kv_elems / c.head_dim), &vmap_), "V tensor map");
    attn_part_o_ = static_cast<float*>(alloc(sizeof(float) * (size_t)Hl_ * splits_ * c.head_dim));
    attn_part_ml_ = static_cast<float*>(alloc(sizeof(float) * (size_t)Hl_ * splits_ * 2));
    attn_counters_ = static_cast<unsigned*>(alloc(sizeof(unsigned) * KVHl_));
    am_score_ = static_cast<float*>(alloc(sizeof(float) * 1024));
    am_index_ = static_cast<uint32_t*>(alloc(sizeof(uint32_t) * 1024));
    am_counter_ = static_cast<unsigned*>(alloc(64));
    tp_cand_local_ = static_cast<float*>(alloc(64));
    tp_cand_all_ = static_cast<float*>(alloc(sizeof(float) * 2 * world_ + 64));
    cuda_check(cudaMallocHost(&host_io_, 64), "cudaMallocHost");
    if (world_ > 1) setup_peer_slots();
    {
        // Q4K_STEP_KERNEL=1: decode with the persistent decode-step kernel
        // (or fail saying why it cannot run); otherwise the launch sequence,
        // which measures faster today
        if (const char* pf = std::getenv("Q4K_L2_PREFETCH")) l2_prefetch_ = pf[0] != '0';
        if (const char* pp = std::getenv("Q4K_PREFETCH_PLAN")) prefetch_plan_ = std::atoi(pp) == 1 ? 1 : 2;
        const char* env = std::getenv("Q4K_STEP_KERNEL");
        const bool wanted = env && env[0] == '1';
        std::string why;
        step_ctas_ = step_ctas(&why);
        step_splits_ = step_ctas_ > 0 ? step_ctas_ / KVHl_ : 0;
        if (world_ != 1) why = "tensor parallelism uses the launch sequence";
        else if (step_ctas_ > 0 && (step_splits_ < 1 || step_splits_ > splits_)) why = "attention split count";
        step_kernel_ = wanted && why.empty();
        if (wanted && !step_kernel_)
            throw Error(Q4K_EINVAL, "decode-step kernel unavailable: " + why);
        if (step_kernel_) {
            step_nphases_ = 2 + 5 * c.layers;
            step_phases_ = static_cast<StepPhase*>(alloc(sizeof(StepPhase) * step_nphases_));
            step_sync_ = static_cast<unsigned*>(alloc(sizeof(unsigned) * (step_nphases_ + 1)));
        }
    }
    cuda_check(cudaStreamSynchronize(stream_), "init");
}

Engine::~Engine() {
    if (exec_) cudaGraphExecDestroy(exec_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (int r = 0; r < world_ && r < kMaxRanks; ++r)
        if (r != rank_ && ar_peer_[r]) cudaIpcCloseMemHandle(ar_peer_[r]);
    if (comm_ && !comm_aborted_) nccl().CommDestroy(comm_);
    for (void* p : allocations_) cudaFree(p);
    if (host_io_) cudaFreeHost(host_io_);
    if (stream_) cudaStreamDestroy(stream_);
}

void* Engine::alloc(size_t bytes) {
    void* p = nullptr;
    cuda_check(cudaMalloc(&p, std::max<size_t>(bytes, 256)), "cudaMalloc");
    allocations_.push_back(p);
    cuda_check(cudaMemsetAsync(p, 0, std::max<size_t>(bytes, 256), stream_), "cudaMemset");
    return p;
}

Engine::Slice Engine::shard_of(const TensorSpec& t) const { return tp_slice(c_, t, rank_, world_); }

void** Engine::tensor_slot(const TensorSpec& t, int** type_slot) {
    *type_slot = nullptr;
    if (t.layer < 0) {
        if (t.slot == 0) return reinterpret_cast<void**>(&output_norm_);
        *type_slot = &t_embd_;
        return reinterpret_cast<void**>(&token_embd_);
    }
    Layer& L = layers_[t.layer];
    switch (t.slot) {
        case 0: return reinterpret_cast<void**>(&L.attn_norm);
        case 1: *type_slot = &L.tq; return reinterpret_cast<void**>(&L.q);
        case 2: *type_slot = &L.tk; return reinterpret_cast<void**>(&L.k);
        case 3: *type_slot = &L.tv; return reinterpret_cast<void**>(&L.v);
        case 4: return reinterpret_cast<void**>(&L.q_norm);
        case 5: return reinterpret_cast<void**>(&L.k_norm);
        case 6: *type_slot = &L.to; return reinterpret_cast<void**>(&L.o);
        case 7: return reinterpret_cast<void**>(&L.ffn_norm);
        case 8: *type_slot = &L.tgate; return reinterpret_cast<void**>(&L.gate);
        case 9: *type_slot = &L.tup; return reinterpret_cast<void**>(&L.up);
        default: *type_slot = &L.tdown; return reinterpret_cast<void**>(&L.down);
    }
}

// raw_device: the full tensor in GGUF layout on the device (F32: the values).
void Engine::place(const TensorSpec& t, const void* raw_device) {
    int* type_slot = nullptr;
    void** slot = tensor_slot(t, &type_slot);
    if (t.type == Q4K_TYPE_F32) {
        if (!*slot) *slot = alloc(sizeof(float) * t.ne0 * t.ne1);
        cuda_check(cudaMemcpyAsync(*slot, raw_device, sizeof(float) * t.ne0 * t.ne1, cudaMemcpyDeviceToDevice,
                                   stream_),
                   "copy tensor");
    } else {
        const Slice s = shard_of(t);
        const size_t bytes = (size_t)(s.n1 - s.n0) * q4k_device_row_bytes(t.type, (size_t)(s.b1 - s.b0) * 256);
        *slot = alloc(bytes);
        *type_slot = t.type;
        cuda_check(relayout(raw_device, t.type, (size_t)t.ne0, (size_t)s.n0, (size_t)s.n1, (size_t)s.b0,
                            (size_t)s.b1, *slot, stream_),
                   "relayout");
    }
}

void Engine::load_synthetic(uint64_t seed) {
    const auto specs = model_tensors(c_);
    size_t max_raw = 0;
    for (const auto& t : specs) max_raw = std::max(max_raw, (size_t)t.ne1 * q4k_gguf_row_bytes(t.type, t.ne0));
    void* tmp = nullptr;
    cuda_check(cudaMalloc(&tmp, max_raw), "cudaMalloc");
    try {
        for (size_t i = 0; i < specs.size(); ++i) {
            const auto& t = specs[i];
            const uint64_t key = q4k_tensor_key(seed, t.name.c_str());
            if (t.type == Q4K_TYPE_F32)
                cuda_check(synth_gamma(key, static_cast<float*>(tmp), (size_t)t.ne0 * t.ne1, stream_), "synth");
            else
                cuda_check(synth_raw(key, t.type, (size_t)t.ne0, (size_t)t.ne1, tmp, stream_), "synth");
            place(t, tmp);
            have_[i] = true;
        }
        cuda_check(cudaStreamSynchronize(stream_), "load_synthetic");
    } catch (...) {
        cudaStreamSynchronize(stream_);
        cudaFree(tmp);
        throw;
    }
    cudaFree(tmp);
    loaded_ = true;
    step_ready_ = false;
    pf_maps_ready_ = false;
}

void Engine::set_tensor(const std::string& name, int type, int64_t ne0, int64_t ne1, const void* host_gguf) {
    const auto specs = model_tensors(c_);
    size_t idx = specs.size();
    for (size_t i = 0; i < specs.size(); ++i)
        if (specs[i].name == name) idx = i;
    if (idx == specs.size()) throw Error(Q4K_EINVAL, "unknown tensor " + name);
    const auto& t = specs[idx];
    if (t.ne0 != ne0 || t.ne1 != ne1) throw Error(Q4K_EINVAL, "tensor " + name + " has the wrong shape");
    // norms are F32; every matrix may be Q4_K or Q6_K (a real Q4_K_M file
    // mixes them per layer)
    const bool matrix = t.type != Q4K_TYPE_F32;
    if (matrix ? (type != Q4K_TYPE_Q4_K && type != Q4K_TYPE_Q6_K) : type != Q4K_TYPE_F32)
        throw Error(Q4K_EINVAL, "tensor " + name + " has an unsupported type");
    TensorSpec ts = t;
    ts.type = type;
    const size_t bytes = (size_t)ne1 * q4k_gguf_row_bytes(type, ne0);
    void* tmp = nullptr;
    cuda_check(cudaMalloc(&tmp, bytes), "cudaMalloc");
    cudaError_t e = cudaMemcpyAsync(tmp, host_gguf, bytes, cudaMemcpyHostToDevice, stream_);
    if (e == cudaSuccess) {
        try {
            place(ts, tmp);
        } catch (...) {
            cudaStreamSynchronize(stream_);
            cudaFree(tmp);
            throw;
        }
        e = cudaStreamSynchronize(stream_);
    }
    cudaFree(tmp);
    cuda_check(e, "set_tensor");
    have_[idx] = true;
    loaded_ = std::all_of(have_.begin(), have_.end(), [](bool b) { return b; });
    step_ready_ = false;
    pf_maps_ready_ = false;
    if (exec_) {
        cudaGraphExecDestroy(exec_);
        exec_ = nullptr;
    }
}

void Engine::fill_kv_synthetic(uint64_t seed, int n) {
    if (n < 0 || n > c_.capacity) throw Error(Q4K_ERANGE, "KV fill beyond capacity");
    char name[64];
    for (int L = 0; L < c_.layers; ++L) {
        for (int kv = 0; kv < 2; ++kv) {
            std::snprintf(name, sizeof name, "kv.%d.%c", L, kv ? 'v' : 'k');
            const uint64_t key = q4k_tensor_key(seed, name);
            uint16_t* base = (kv ? vcache_ : kcache_) + (size_t)L * KVHl_ * c_.capacity * c_.head_dim;
            for (int h = 0; h < KVHl_; ++h) {
                const uint64_t hg = (uint64_t)rank_ * KVHl_ + h;
                cuda_check(synth_f16(key, base + (size_t)h * c_.capacity * c_.head_dim, (size_t)n * c_.head_dim,
                                     hg * kKvIndexStride * c_.head_dim, stream_),
                           "synth kv");
            }
        }
    }
    // every other sequence gets the same rows 0 .. n-1
    const size_t row_bytes = (size_t)n * c_.head_dim * 2, pitch = (size_t)c_.capacity * c_.head_dim * 2;
    for (int sq = 1; sq < seqs_ && n > 0; ++sq)
        for (uint16_t* cache : {kcache_, vcache_})
            cuda_check(cudaMemcpy2DAsync(cache + sq * seq_elems_, pitch, cache, pitch, row_bytes,
                                         (size_t)c_.layers * KVHl_, cudaMemcpyDeviceToDevice, stream_),
                       "copy kv");
    cuda_check(cudaStreamSynchronize(stream_), "fill_kv");
}

void Engine::read_kv(int layer, uint16_t* k_host, uint16_t* v_host) {
    if (layer < 0 || layer >= c_.layers) throw Error(Q4K_ERANGE, "layer out of range");
    const size_t n = (size_t)KVHl_ * c_.capacity * c_.head_dim;
    if (k_host)
        cuda_check(cudaMemcpyAsync(k_host, kcache_ + (size_t)layer * n, n * 2, cudaMemcpyDeviceToHost, stream_), "read");
    if (v_host)
        cuda_check(cudaMemcpyAsync(v_host, vcache_ + (size_t)layer * n, n * 2, cudaMemcpyDeviceToHost, stream_), "read");
    cuda_check(cudaStreamSynchronize(stream_), "read_kv");
}

void Engine::write_kv(int layer, const uint16_t* k_host, const uint16_t* v_host) {
    if (layer < 0 || layer >= c_.layers) throw Error(Q4K_ERANGE, "layer out of range");
    const size_t n = (size_t)KVHl_ * c_.capacity * c_.head_dim;
    if (k_host)
        cuda_check(cudaMemcpyAsync(kcache_ + (size_t)layer * n, k_host, n * 2, cudaMemcpyHostToDevice, stream_), "write");
    if (v_host)
        cuda_check(cudaMemcpyAsync(vcache_ + (size_t)layer * n, v_host, n * 2, cudaMemcpyHostToDevice, stream_), "write");
    cuda_check(cudaStreamSynchronize(stream_), "write_kv");
}

// Maps every rank's receive slots for the fused row-parallel sums. All ranks
// take part (two all-gathers over the engine's communicator) and agree: the
// fused path is used only if every rank exported its slots and opened every
// other rank's; otherwise every rank keeps the ncclAllReduce path.
// Q4K_TP_FUSED=0 turns it off.
void Engine::setup_peer_slots() {
    const int H = c_.hidden;
    bool want = world_ <= kMaxRanks;
    if (const char* e = std::getenv("Q4K_TP_FUSED")) want = want && e[0] != '0';
    ar_base_ = static_cast<uint8_t*>(alloc((size_t)2 * c_.layers * world_ * H * sizeof(unsigned long long)));
    ar_epoch_ = static_cast<int*>(alloc(64));
    xb_ = static_cast<float*>(alloc(sizeof(float) * H));
    constexpr size_t kRec = 128;  // per rank: IPC handle (64 bytes), then a status word
    static_assert(sizeof(cudaIpcMemHandle_t) <= 64, "IPC handle size");
    uint8_t* rec = static_cast<uint8_t*>(alloc(kRec * world_));
    std::vector<uint8_t> host(kRec * world_, 0), mine(kRec, 0);
    auto exchange = [&](int status) {
        mine[64] = (uint8_t)status;
        cuda_check(cudaMemcpyAsync(rec + kRec * rank_, mine.data(), kRec, cudaMemcpyHostToDevice, stream_), "h2d");
        nccl_check(nccl().AllGather(rec + kRec * rank_, rec, kRec, ncclUint8, comm_, stream_), "ncclAllGather");
        cuda_check(cudaMemcpyAsync(host.data(), rec, kRec * world_, cudaMemcpyDeviceToHost, stream_), "d2h");
        cuda_check(cudaStreamSynchronize(stream_), "peer slot exchange");
        bool all = true;
        for (int r = 0; r < world_; ++r) all = all && host[kRec * r + 64] == 1;
        return all;
    };
    cudaIpcMemHandle_t h{};
    int status = 0;
    if (want && cudaIpcGetMemHandle(&h, ar_base_) == cudaSuccess) {
        std::memcpy(mine.data(), &h, sizeof h);
        status = 1;
    }
    cudaGetLastError();
    if (!exchange(status)) return;
    status = 1;
    ar_peer_[rank_] = ar_base_;
    for (int r = 0; r < world_; ++r) {
        if (r == rank_) continue;
        cudaIpcMemHandle_t hr;
        std::memcpy(&hr, host.data() + kRec * r, sizeof hr);
        if (cudaIpcOpenMemHandle(&ar_peer_[r], hr, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            ar_peer_[r] = nullptr;
            status = 0;
        }
    }
    cudaGetLastError();
    if (!exchange(status)) {
        for (int r = 0; r < world_; ++r)
            if (r != rank_ && ar_peer_[r]) cudaIpcCloseMemHandle(ar_peer_[r]);
        std::fill(std::begin(ar_peer_), std::end(ar_peer_), nullptr);
        cudaGetLastError();
        return;
    }
    tp_fused_ = true;
}

unsigned long long* Engine::peer_recv(int rank, int slot) const {
    return static_cast<unsigned long long*>(ar_peer_[rank]) + (size_t)slot * world_ * c_.hidden;
}

// One transformer block (Engine.cpp:71-103) on the device buffers: x is
void Engine::kv_prefetch(int layer, L2Prefetch* f) const {
    if (!l2_prefetch_) return;
    const size_t kv_layer = (size_t)layer * KVHl_ * c_.capacity * c_.head_dim;
    for (int e = 0; e < 2; ++e) {
        f[e].base = (e == 0 ? kcache_ : vcache_) + kv_layer;
        f[e].bytes = (unsigned long long)c_.head_dim * 2;
        f[e].stride = (unsigned long long)c_.capacity * c_.head_dim * 2;
        f[e].count = KVHl_;
        f[e].position = pos_;
    }
}

L2Prefetch Engine::weight_prefetch(const uint8_t* w, int type, int K, int rows) const {
    L2Prefetch f;
    if (!l2_prefetch_ || !w) return f;
    f.base = w;
    f.bytes = (unsigned long long)q4k_device_row_bytes(type, K) * (unsigned long long)rows;
    f.stride = f.bytes;
    f.count = 1;
    return f;
}

// updated in place, layer i's K/V rows at *pos_ are written. With fused
// tensor parallelism the residual stream alternates between x_ and xb_ inside
// the layer (x_ again at its end, before the ffn_down ranks' partial sums
// are added by the next product).
void Engine::enqueue_layer(int i, bool fused) {
    const auto& c = c_;
    const int H = c.hidden;
    fused = fused && tp_fused_;
    // slot of layer l's attn_output (0) or ffn_down (1) partial sums
    auto slot = [&](int l, int k) { return 2 * l + k; };
    // EPI_PEER into every rank's slot s
    auto peer_out = [&](GemvRequest& r, int s_) {
        r.epilogue = EPI_PEER;
        r.seg[0].y = nullptr;
        r.peer_out.world = world_;
        r.peer_out.epoch = ar_epoch_;
        for (int k = 0; k < world_; ++k) r.peer_out.recv[k] = peer_recv(k, s_) + (size_t)rank_ * H;
    };
    // the product's input: x plus every rank's partial sums of slot s_ (none: s_ < 0), also stored to x_out
    auto peer_in = [&](GemvRequest& r, int s_, float* x_out) {
        r.peer_in.world = s_ >= 0 ? world_ : 0;
        r.peer_in.parts = s_ >= 0 ? peer_recv(rank_, s_) : nullptr;
        r.peer_in.epoch = ar_epoch_;
        r.peer_in.x_out = x_out;
        r.peer_in.wait_ns = dev_wait_ns_;
    };
    auto gemv = [&](GemvRequest& r) { cuda_check(launch_gemv(r, stream_), "gemv launch"); };
    auto all_reduce_into_x = [&]() {
        nccl_check(nccl().AllReduce(partial_, partial_, H, ncclFloat, ncclSum, comm_, stream_), "ncclAllReduce");
        cuda_check(residual_add(x_, partial_, H, stream_), "residual_add");
    };
    const Layer& L = layers_[i];
    const size_t kv_layer = (size_t)i * KVHl_ * c.capacity * c.head_dim;
    {
        GemvRequest r;
        r.nseg = 3;
        r.seg[0] = {L.q, qkv_, L.tq, qd_};
        r.seg[1] = {L.k, qkv_ + qd_, L.tk, kvd_};
        r.seg[2] = {L.v, qkv_ + qd_ + kvd_, L.tv, kvd_};
        r.K = H;
        r.x = x_;
        if (fused) peer_in(r, i > 0 ? slot(i - 1, 1) : -1, xb_);
        r.gamma = L.attn_norm;
        r.eps = c.eps;
        r.epilogue = EPI_STORE;
        r.err = err_;
        r.pdl = true;
        r.trace = trace_;
        r.trace_tag = 5 * i;
        kv_prefetch(i, r.prefetch);  // the attention's K and V rows
        gemv(r);
    }
    {
        DecodeAttnArgs a;
        a.qkv = qkv_;
        a.q_gamma = L.q_norm;
        a.k_gamma = L.k_norm;
        a.k_cache = kcache_ + kv_layer;
        a.v_cache = vcache_ + kv_layer;
        a.capacity = c.capacity;
        a.position = pos_;
        a.heads = Hl_;
        a.kv_heads = KVHl_;
        a.eps = c.eps;
        a.rope_base = c.rope_base;
        a.partial_o = attn_part_o_;
        a.partial_ml = attn_part_ml_;
        a.counters = attn_counters_;
        a.out = att_;
        a.err = err_;
        a.splits = splits_;
        a.row_base = i * KVHl_ * c.capacity;
        a.trace = trace_;
        a.trace_tag = 5 * i + 1;
        a.prefetch[0] = weight_prefetch(L.o, L.to, qd_, H);
        if (prefetch_plan_ == 2) {
            // the long attention launch also asks for the gate/up weights, so
            // that the short O launch ends without a 28 MB prefetch in flight
            a.prefetch[1] = weight_prefetch(L.gate, L.tgate, H, ffn_l_);
            a.prefetch[2] = weight_prefetch(L.up, L.tup, H, ffn_l_);
        }
        if (act_images_) a.out_image = att_img_;
        cuda_check(decode_attention(a, kmap_, vmap_, stream_, true), "attention launch");
    }
    {
        GemvRequest r;
        r.nseg = 1;
        r.seg[0] = {L.o, world_ > 1 ? partial_ : x_, L.to, H};
        r.K = qd_;
        r.x = att_;
        r.epilogue = world_ > 1 ? EPI_STORE : EPI_ADD;
        if (fused) peer_out(r, slot(i, 0));
        r.err = err_;
        r.pdl = true;
        r.trace = trace_;
        r.trace_tag = 5 * i + 2;
        if (prefetch_plan_ == 1) {
            r.prefetch[0] = weight_prefetch(L.gate, L.tgate, H, ffn_l_);
            r.prefetch[1] = weight_prefetch(L.up, L.tup, H, ffn_l_);
        }
        if (act_images_) r.in_image = att_img_;
        gemv(r);
        if (world_ > 1 && !fused) all_reduce_into_x();
    }
    {
        GemvRequest r;
        r.nseg = 2;
        r.seg[0] = {L.gate, act_, L.tgate, ffn_l_};
        r.seg[1] = {L.up, act_, L.tup, ffn_l_};
        r.K = H;
        r.x = x_;
        if (fused) {
            r.x = xb_;
            peer_in(r, slot(i, 0), x_);
        }
        r.gamma = L.ffn_norm;
        r.eps = c.eps;
        r.epilogue = EPI_SWIGLU;
        r.err = err_;
        r.pdl = true;
        r.trace = trace_;
        r.trace_tag = 5 * i + 3;
        r.prefetch[0] = weight_prefetch(L.down, L.tdown, ffn_l_, H);
        if (act_images_) r.out_image = act_img_;
        gemv(r);
    }
    {
        GemvRequest r;
        r.nseg = 1;
        r.seg[0] = {L.down, world_ > 1 ? partial_ : x_, L.tdown, H};
        r.K = ffn_l_;
        r.x = act_;
        r.epilogue = world_ > 1 ? EPI_STORE : EPI_ADD;
        if (fused) peer_out(r, slot(i, 1));
        r.err = err_;
        r.pdl = true;
        r.trace = trace_;
        r.trace_tag = 5 * i + 4;
        if (act_images_) r.in_image = act_img_;
        if (i + 1 < c.layers) {
            const Layer& N = layers_[i + 1];
            r.prefetch[0] = weight_prefetch(N.q, N.tq, H, qd_);
            r.prefetch[1] = weight_prefetch(N.k, N.tk, H, kvd_);
            r.prefetch[2] = weight_prefetch(N.v, N.tv, H, kvd_);
        }
        gemv(r);
        if (world_ > 1 && !fused) all_reduce_into_x();
    }
}

void Engine::enqueue_step(bool record_hidden) {
    const auto& c = c_;
    const int H = c.hidden;
    auto snapshot = [&](int i) {
        if (record_hidden)
            cuda_check(cudaMemcpyAsync(hidden_ + (size_t)i * H, x_, sizeof(float) * H, cudaMemcpyDeviceToDevice,
                                       stream_),
                       "snapshot");
    };

    cuda_check(embed_rows(token_embd_, t_embd_, H, c.vocab, token_, 1, x_, err_, stream_, false), "embed");
    snapshot(0);
    for (int i = 0; i < c.layers; ++i) {
        enqueue_layer(i, true);
        snapshot(i + 1);
    }
    enqueue_head(true);
}

// Output head on x_ (Engine.cpp:106-111): final RMSNorm, the token_embd
// product with the greedy choice fused, the shard merge when tp_world > 1, and
// the step's bookkeeping (token_, history, *pos_ += *advance_). fused: the
// last layer's ffn_down partial sums are still in the receive slots.
void Engine::enqueue_head(bool fused) {
    const auto& c = c_;
    const int H = c.hidden;
    fused = fused && tp_fused_;
    auto gemv = [&](GemvRequest& r) { cuda_check(launch_gemv(r, stream_), "gemv launch"); };
    {
        GemvRequest r;
        r.nseg = 1;
        const size_t row_bytes = q4k_device_row_bytes(t_embd_, H);
        r.seg[0] = {token_embd_ + (size_t)vocab0_ * row_bytes, logits_, t_embd_, (int)(vocab1_ - vocab0_)};
        r.K = H;
        r.x = x_;
        if (fused) {
            r.peer_in.world = world_;
            r.peer_in.parts = peer_recv(rank_, 2 * (c.layers - 1) + 1);
            r.peer_in.epoch = ar_epoch_;
            r.peer_in.wait_ns = dev_wait_ns_;
        }
        r.gamma = output_norm_;
        r.eps = c.eps;
        r.epilogue = EPI_ARGMAX;
        r.argmax.cand_score = am_score_;
        r.argmax.cand_index = am_index_;
        r.argmax.counter = am_counter_;
        r.argmax.index_base = (uint32_t)vocab0_;
        r.trace = trace_;
        r.trace_tag = 5 * c_.layers;
        // the next token's first product
        r.prefetch[0] = weight_prefetch(layers_[0].q, layers_[0].tq, H, qd_);
        r.prefetch[1] = weight_prefetch(layers_[0].k, layers_[0].tk, H, kvd_);
        r.prefetch[2] = weight_prefetch(layers_[0].v, layers_[0].tv, H, kvd_);
        if (world_ > 1) {
            r.argmax.token = reinterpret_cast<uint32_t*>(tp_cand_local_) + 1;
            r.argmax.score = tp_cand_local_;
        } else {
            r.argmax.token = token_;
        }
        r.err = err_;
        r.pdl = true;
        gemv(r);
    }
    if (world_ > 1)
        nccl_check(nccl().AllGather(tp_cand_local_, tp_cand_all_, 2, ncclUint32, comm_, stream_), "ncclAllGather");
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1);
        cfg.blockDim = dim3(32);
        cfg.stream = stream_;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cuda_check(cudaLaunchKernelEx(&cfg, finish_step_kernel, token_, pos_, (const int*)advance_, history_,
                                      history_n_, (unsigned)c.capacity,
                                      world_ > 1 ? reinterpret_cast<const uint32_t*>(tp_cand_all_) : nullptr, world_,
                                      fused ? ar_epoch_ : nullptr),
                   "finish launch");
    }
}

void Engine::ensure_step_plan() {
    if (step_ready_) return;
    const auto& c = c_;
    const int H = c.hidden;
    std::vector<StepPhase> ph;
    auto gemv_phase = [&](int dep, int layer, int epilogue, int K, const float* x, const float* gamma,
                          std::initializer_list<GemvSegment> segs, bool pair) {
        StepPhase p;
        p.kind = kStepGemv;
        p.dep = dep;
        p.layer = layer;
        p.epilogue = epilogue;
        p.K = K;
        p.nb = K / 256;
        p.pair = pair ? 1 : 0;
        p.x = x;
        p.gamma = gamma;
        int n = 0, max_row = 0;
        for (const GemvSegment& g : segs) {
            p.w[n] = g.w;
            p.y[n] = g.y;
            p.type[n] = g.type;
            p.rows[n] = g.rows;
            p.row_bytes[n] = (int)q4k_device_row_bytes(g.type, (size_t)K);
            max_row = std::max(max_row, p.row_bytes[n]);
            (g.type == Q4K_TYPE_Q4_K ? p.q4 : p.q6) = 1;
            ++n;
        }
        // the step kernel stages the fp32 activation (and gamma) in 40 KB of shared memory
        if (K * 4 * (gamma ? 2 : 1) > 40 * 1024 || !step_gemv_geometry(K, max_row, pair, p.q4, p.q6, p.lpr, p.R))
            throw Error(Q4K_EINVAL, "decode-step kernel: no stage geometry for this product");
        p.nseg = pair ? 1 : n;
        // Q4_K stages on the tensor cores where the stage is 16 rows (8 + 8 for
        // SwiGLU) and the row stride keeps the fragment loads bank-friendly
        // (opt-in with Q4K_GEMV_MMA=1, as in the per-product kernel)
        const char* mma_env = std::getenv("Q4K_GEMV_MMA");
        p.mma = mma_env && mma_env[0] == '1' && K <= 3072 && p.R == (pair ? 8 : 16) ? 1 : 0;
        int stages = 0;
        for (int s = 0; s < p.nseg; ++s) {
            p.stage_start[s] = stages;
            stages += (p.rows[s] + p.R - 1) / p.R;
        }
        for (int s = p.nseg; s <= kMaxSegments; ++s) p.stage_start[s] = stages;
        p.total_stages = stages;
        ph.push_back(p);
        return (int)ph.size() - 1;
    };
    StepPhase embed;
    embed.kind = kStepEmbed;
    ph.push_back(embed);
    int prev = 0;
    for (int i = 0; i < c.layers; ++i) {
        const Layer& L = layers_[i];
        const int qkv = gemv_phase(prev, i, EPI_STORE, H, x_, L.attn_norm,
                                   {{L.q, qkv_, L.tq, qd_}, {L.k, qkv_ + qd_, L.tk, kvd_},
                                    {L.v, qkv_ + qd_ + kvd_, L.tv, kvd_}},
                                   false);
        StepPhase at;
        at.kind = kStepAttention;
        at.dep = qkv;
        at.layer = i;
        at.gamma = L.q_norm;
        at.gamma2 = L.k_norm;
        ph.push_back(at);
        const int att = (int)ph.size() - 1;
        const int o = gemv_phase(att, i, EPI_ADD, qd_, att_, nullptr, {{L.o, x_, L.to, H}}, false);
        const int gu = gemv_phase(o, i, EPI_SWIGLU, H, x_, L.ffn_norm,
                                  {{L.gate, act_, L.tgate, ffn_l_}, {L.up, act_, L.tup, ffn_l_}}, true);
        prev = gemv_phase(gu, i, EPI_ADD, ffn_l_, act_, nullptr, {{L.down, x_, L.tdown, H}}, false);
    }
    gemv_phase(prev, c.layers, EPI_ARGMAX, H, x_, output_norm_, {{token_embd_, logits_, t_embd_, c.vocab}}, false);
    if ((int)ph.size() != step_nphases_) throw Error(Q4K_ECUDA, "decode-step plan size");
    cuda_check(cudaMemcpyAsync(step_phases_, ph.data(), sizeof(StepPhase) * ph.size(), cudaMemcpyHostToDevice,
                               stream_),
               "upload step plan");
    cuda_check(cudaStreamSynchronize(stream_), "upload step plan");
    step_ready_ = true;
}

void Engine::enqueue_step_kernel() {
    const auto& c = c_;
    StepArgs a;
    a.phases = step_phases_;
    a.nphases = step_nphases_;
    a.sync = step_sync_;
    a.err = err_;
    a.token = token_;
    a.pos = pos_;
    a.advance = advance_;
    a.history = history_;
    a.history_n = history_n_;
    a.history_cap = (unsigned)c.capacity;
    a.embd = token_embd_;
    a.embd_type = t_embd_;
    a.hidden = c.hidden;
    a.vocab = c.vocab;
    a.x = x_;
    a.qkv = qkv_;
    a.att = att_;
    a.kcache = kcache_;
    a.vcache = vcache_;
    a.capacity = c.capacity;
    a.heads = Hl_;
    a.kv_heads = KVHl_;
    a.splits = step_splits_;
    a.eps = c.eps;
    a.rope_base = c.rope_base;
    a.partial_o = attn_part_o_;
    a.partial_ml = attn_part_ml_;
    a.counters = attn_counters_;
    a.argmax.cand_score = am_score_;
    a.argmax.cand_index = am_index_;
    a.argmax.counter = am_counter_;
    a.argmax.token = token_;
    a.argmax.index_base = 0;
    a.trace = trace_;
    if (const char* env = std::getenv("Q4K_STEP_INFLIGHT")) a.inflight = std::max(1, std::atoi(env));
    cuda_check(launch_decode_step(a, kmap_, vmap_, step_ctas_, stream_), "decode-step launch");
}

void Engine::ensure_graph() {
    if (exec_) return;
    cudaGraph_t graph = nullptr;
    cuda_check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
        enqueue_step(false);
    } catch (...) {
        cudaStreamEndCapture(stream_, &graph);
        if (graph) cudaGraphDestroy(graph);
        throw;
    }
    cuda_check(cudaStreamEndCapture(stream_, &graph), "end capture");
    const cudaError_t e = cudaGraphInstantiate(&exec_, graph, 0);
    cudaGraphDestroy(graph);
    cuda_check(e, "graph instantiate");
}

void Engine::set_limits(uint64_t device_wait_ns, int host_wait_ms) {
    if (host_wait_ms < 0) throw Error(Q4K_EINVAL, "host_wait_ms must be >= 0");
    if (device_wait_ns && device_wait_ns != dev_wait_ns_) {
        dev_wait_ns_ = device_wait_ns;
        // the limit is a kernel parameter of the captured step: capture again
        if (exec_) cudaGraphExecDestroy(exec_);
        exec_ = nullptr;
    }
    host_wait_ms_ = host_wait_ms;
}

void Engine::abort() {
    aborted_.store(true);
    std::lock_guard<std::mutex> lock(abort_mu_);
    if (comm_ && !comm_aborted_) {
        // makes the NCCL kernels in flight on this rank return, so that the
        // stream drains; the communicator is freed and never used again
        const NcclApi& api = nccl();
        if (api.CommAbort) api.CommAbort(comm_);
        comm_aborted_ = true;
    }
}

void Engine::host_wait(const char* what) {
    if (world_ == 1 || (host_wait_ms_ == 0 && !aborted_.load())) {
        cuda_check(cudaStreamSynchronize(stream_), what);
        // an abort from another thread ends NCCL's kernels, so the stream
        // drains; the step did not complete
        if (aborted_.load()) throw Error(Q4K_ETIMEOUT, std::string(what) + ": tensor-parallel step aborted");
        return;
    }
    // tensor parallelism: poll, so that a peer that never arrives (or an
    // abort from another thread) ends the wait instead of blocking for good
    const auto start = std::chrono::steady_clock::now();
    for (long spins = 0;; ++spins) {
        const cudaError_t e = cudaStreamQuery(stream_);
        if (e == cudaSuccess) return;
        if (e != cudaErrorNotReady) cuda_check(e, what);
        const bool late = host_wait_ms_ > 0 && std::chrono::steady_clock::now() - start >
                                                    std::chrono::milliseconds(host_wait_ms_);
        if (late || aborted_.load()) {
            abort();
            // NCCL kernels end once the communicator is aborted, and every
            // wait inside this library's kernels is bounded: drain the stream
            // so that no kernel of this rank is left running
            cudaStreamSynchronize(stream_);
            throw Error(Q4K_ETIMEOUT, std::string(what) + ": tensor-parallel step " +
                                          (late ? "did not complete within the host limit" : "aborted") +
                                          "; the communicator is aborted");
        }
        if (spins > 1000) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

void Engine::check_device_error(bool with_token) {
    int err = 0;
    // with_token: the step's token and the error word in one copy
    if (with_token)
        cuda_check(cudaMemcpyAsync(&host_io_[kHostOut], io_, (kIoErr + 1) * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                   stream_),
                   "read token and err");
    else
        cuda_check(cudaMemcpyAsync(&host_io_[kHostOut + kIoErr], err_, sizeof(int), cudaMemcpyDeviceToHost, stream_),
                   "read err");
    host_wait("step");
    err = (int)host_io_[kHostOut + kIoErr];
    if (err) {
        cudaMemsetAsync(err_, 0, sizeof(int), stream_);
        cudaStreamSynchronize(stream_);
        char msg[96];
        std::snprintf(msg, sizeof msg, "device reported error bits 0x%x", err);
        int status = Q4K_ECUDA;
        if (err & (ERR_WAIT_TIMEOUT_FULL | ERR_WAIT_TIMEOUT_EMPTY | ERR_WAIT_TIMEOUT_DEP | ERR_WAIT_TIMEOUT_PEER))
            status = Q4K_ETIMEOUT;
        else if (err & (ERR_BAD_POSITION | ERR_BAD_TOKEN))
            status = Q4K_ERANGE;
        throw Error(status, msg);
    }
}

void Engine::require_live() const {
    if (aborted_.load()) throw Error(Q4K_ETIMEOUT, "the engine was aborted (tensor-parallel failure); create a new one");
}

void Engine::stage_io(uint32_t token, int position, uint32_t advance) {
    host_io_[kIoToken] = token;
    host_io_[kIoPos] = (uint32_t)position;
    host_io_[kIoAdvance] = advance;
    host_io_[kIoHistoryN] = 0;
    cuda_check(cudaMemcpyAsync(io_, host_io_, kIoIn * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_), "h2d");
}

uint32_t Engine::decode(uint32_t token, int position, float* logits_host, float* hidden_host) {
    require_live();
    if (!loaded_) throw Error(Q4K_EINVAL, "weights are not loaded");
    if (token >= (uint32_t)c_.vocab) throw Error(Q4K_ERANGE, "Token ID out of range");
    if (position < 0 || position >= c_.capacity) throw Error(Q4K_ERANGE, "KV cache capacity exceeded");
    if (hidden_host && world_ > 1) throw Error(Q4K_EINVAL, "hidden snapshots need tp_world == 1");
    stage_io(token, position, 0);
    if (hidden_host) {
        enqueue_step(true);
    } else if (step_kernel_) {
        ensure_step_plan();
        enqueue_step_kernel();
    } else {
        ensure_graph();
        cuda_check(cudaGraphLaunch(exec_, stream_), "graph launch");
    }
    if (logits_host)
        cuda_check(cudaMemcpyAsync(logits_host, logits_, sizeof(float) * (vocab1_ - vocab0_), cudaMemcpyDeviceToHost,
                                   stream_),
                   "d2h logits");
    if (hidden_host)
        cuda_check(cudaMemcpyAsync(hidden_host, hidden_, sizeof(float) * c_.hidden * (c_.layers + 1),
                                   cudaMemcpyDeviceToHost, stream_),
                   "d2h hidden");
    check_device_error(true);
    return host_io_[kHostOut + kIoToken];
}

void Engine::generate(uint32_t token, int position, int steps, int advance, uint32_t* tokens_host) {
    require_live();
    if (!loaded_) throw Error(Q4K_EINVAL, "weights are not loaded");
    if (token >= (uint32_t)c_.vocab) throw Error(Q4K_ERANGE, "Token ID out of range");
    if (steps < 0 || steps > c_.capacity) throw Error(Q4K_ERANGE, "too many steps");
    const long long last = (long long)position + (advance ? (long long)steps - 1 : 0);
    if (position < 0 || last >= c_.capacity) throw Error(Q4K_ERANGE, "KV cache capacity exceeded");
    if (steps == 0) return;
    if (step_kernel_)
        ensure_step_plan();
    else
        ensure_graph();
    stage_io(token, position, advance ? 1u : 0u);
    for (int s = 0; s < steps; ++s) {
        if (step_kernel_)
            enqueue_step_kernel();
        else
            cuda_check(cudaGraphLaunch(exec_, stream_), "graph launch");
    }
    if (tokens_host)
        cuda_check(cudaMemcpyAsync(tokens_host, history_, sizeof(uint32_t) * steps, cudaMemcpyDeviceToHost, stream_),
                   "d2h tokens");
    check_device_error();
}

size_t Engine::trace_step(uint32_t token, int position, unsigned long long* records_host, size_t max_records) {
    require_live();
    if (!loaded_) throw Error(Q4K_EINVAL, "weights are not loaded");
    if (token >= (uint32_t)c_.vocab) throw Error(Q4K_ERANGE, "Token ID out of range");
    if (position < 0 || position >= c_.capacity) throw Error(Q4K_ERANGE, "KV cache capacity exceeded");
    if (5 * c_.layers + 1 > kTraceLaunches) throw Error(Q4K_ERANGE, "too many layers to trace");
    const size_t words = (size_t)kTraceLaunches * kTraceCtas * kTraceSlots;
    if (!trace_buf_) trace_buf_ = static_cast<unsigned long long*>(alloc(words * 8));
    cuda_check(cudaMemsetAsync(trace_buf_, 0, words * 8, stream_), "memset trace");
    // a traced graph of its own; the normal graph stays untraced
    cudaGraphExec_t saved = exec_;
    exec_ = nullptr;
    trace_ = trace_buf_;
    const size_t n = std::min(words, max_records);
    try {
        if (step_kernel_)
            ensure_step_plan();
        else
            ensure_graph();
        stage_io(token, position, 0);
        if (step_kernel_)
            enqueue_step_kernel();
        else
            cuda_check(cudaGraphLaunch(exec_, stream_), "graph launch");
        cuda_check(cudaStreamSynchronize(stream_), "trace step");
        if (records_host && n)
            cuda_check(cudaMemcpy(records_host, trace_buf_, n * 8, cudaMemcpyDeviceToHost), "d2h trace");
    } catch (...) {
        if (exec_) cudaGraphExecDestroy(exec_);
        exec_ = saved;
        trace_ = nullptr;
        throw;
    }
    if (exec_) cudaGraphExecDestroy(exec_);
    exec_ = saved;
    trace_ = nullptr;
    check_device_error();
    return n;
}

// Rows of one prefill pass: longer prompts run as consecutive passes, each
// attending to the cache rows the previous passes wrote.
constexpr int kPrefillRows = 512;

void Engine::ensure_prefill() {
    if (pf_rows_) return;
    int rows = kPrefillRows;
    // Q4K_PREFILL_ROWS=r: r rows per pass (tests split prompts with it)
    if (const char* r = std::getenv("Q4K_PREFILL_ROWS")) rows = std::max(1, std::atoi(r));
    rows = std::min(rows, c_.capacity);
    const size_t H = c_.hidden;
    pf_tokens_ = static_cast<uint32_t*>(alloc(sizeof(uint32_t) * rows));
    pf_x_ = static_cast<float*>(alloc(sizeof(float) * rows * H));
    pf_qkv_ = static_cast<float*>(alloc(sizeof(float) * rows * (size_t)(qd_ + 2 * kvd_)));
    pf_q_ = static_cast<float*>(alloc(sizeof(float) * rows * (size_t)qd_));
    pf_att_ = static_cast<float*>(alloc(sizeof(float) * rows * (size_t)qd_));
    pf_act_ = static_cast<float*>(alloc(sizeof(float) * rows * (size_t)ffn_l_));
    if (world_ > 1) pf_partial_ = static_cast<float*>(alloc(sizeof(float) * rows * H));
    // Prompt products: the tensor-core GEMM for passes of 9 rows or more, the
    // batched dp4a GEMV (which streams each weight once per 8 rows) below
    // that, where it measured faster. Q4K_PREFILL_GEMM=0 / =1 forces one.
    if (const char* g = std::getenv("Q4K_PREFILL_GEMM")) {
        pf_gemm_ = g[0] != '0';
        pf_gemm_min_rows_ = pf_gemm_ ? 1 : INT32_MAX;
    }
    if (pf_gemm_) {
        const size_t max_k = std::max<size_t>({H, (size_t)qd_, (size_t)ffn_l_});
        pf_a_ = static_cast<uint16_t*>(alloc(sizeof(uint16_t) * 2 * rows * max_k));
        pf_gsum_ = static_cast<float*>(alloc(sizeof(float) * rows * (max_k / 32)));
        pf_rs_ = static_cast<float*>(alloc(sizeof(float) * rows));
        // split-K workspace: the most any product of a layer (or the batched
        // head) would use at any row count of a pass, so that the engine's
        // products take the same K splits as q4k_matmul_batch
        pf_part_floats_ = 0;
        for (int m = 1; m <= rows; ++m) {
            PrefillGemmArgs g;
            g.M = m;
            auto need = [&](int nseg, int K, int epi, std::initializer_list<int> outs) {
                g.nseg = nseg;
                g.K = K;
                g.epilogue = epi;
                int i = 0;
                for (int n : outs) g.seg[i++].rows = n;
                pf_part_floats_ = std::max(pf_part_floats_, prefill_gemm_partial_floats(g));
            };
            need(3, (int)H, EPI_STORE, {qd_, kvd_, kvd_});
            need(1, qd_, EPI_ADD, {(int)H});
            need(2, (int)H, EPI_SWIGLU, {ffn_l_, ffn_l_});
            need(1, ffn_l_, EPI_ADD, {(int)H});
            need(1, (int)H, EPI_STORE, {(int)(vocab1_ - vocab0_)});
        }
        pf_part_ = static_cast<float*>(alloc(sizeof(float) * pf_part_floats_));
        const int ks[3] = {(int)H, qd_, ffn_l_};
        for (int i = 0; i < 3; ++i) cuda_check(make_act_map(pf_a_, ks[i], rows, &pf_amap_[i]), "activation map");
    }
    pf_rows_ = rows;
}

// TMA maps of every layer's weights for the prefill GEMM, built once per
// placement of the tensors (encoding a map is host work).
void Engine::ensure_prefill_maps() {
    if (pf_maps_ready_) return;
    const int H = c_.hidden;
    pf_wmaps_.assign((size_t)c_.layers * 7 * kPrefillWeightMaps, KvTensorMap{});
    for (int i = 0; i < c_.layers; ++i) {
        const Layer& L = layers_[i];
        const struct {
            const uint8_t* w;
            int type, K, rows;
        } m[7] = {{L.q, L.tq, H, qd_},     {L.k, L.tk, H, kvd_},       {L.v, L.tv, H, kvd_},
                  {L.o, L.to, qd_, H},     {L.gate, L.tgate, H, ffn_l_}, {L.up, L.tup, H, ffn_l_},
                  {L.down, L.tdown, ffn_l_, H}};
        for (int j = 0; j < 7; ++j)
            cuda_check(make_weight_map(m[j].w, m[j].type, m[j].K, m[j].rows,
                                       &pf_wmaps_[((size_t)i * 7 + j) * kPrefillWeightMaps]),
                       "weight map");
    }
    const size_t row_bytes = q4k_device_row_bytes(t_embd_, H);
    cuda_check(make_weight_map(token_embd_ + (size_t)vocab0_ * row_bytes, t_embd_, H, (int)(vocab1_ - vocab0_),
                               pf_head_map_),
               "head map");
    pf_maps_ready_ = true;
}

const KvTensorMap* Engine::layer_maps(int layer, int slot) const {
    return &pf_wmaps_[((size_t)layer * 7 + slot) * kPrefillWeightMaps];
}

void Engine::enqueue_product(GemvRequest& r, const KvTensorMap* wmaps) {
    if (!pf_gemm_ || r.M < pf_gemm_min_rows_ || !wmaps) {
        cuda_check(launch_gemv(r, stream_), "gemv launch");
        return;
    }
    const int H = c_.hidden;
    cuda_check(prefill_quantise(r.x, r.ldx ? r.ldx : r.K, r.gamma, r.eps, r.M, r.K, pf_a_, pf_rows_, pf_gsum_, pf_rs_,
                                stream_),
               "prefill_quantise launch");
    PrefillGemmArgs g;
    g.nseg = r.nseg;
    for (int s = 0; s < r.nseg; ++s) {
        g.seg[s] = {r.seg[s].w, r.seg[s].type, r.seg[s].rows, r.seg[s].y};
        g.wmap[s] = wmaps + (size_t)s * kPrefillWeightMaps;
    }
    g.K = r.K;
    g.M = r.M;
    g.ldy = r.ldy;
    g.epilogue = r.epilogue;
    g.amap = &pf_amap_[r.K == H ? 0 : r.K == qd_ ? 1 : 2];
    g.a = pf_a_;
    g.row_scale = pf_rs_;
    g.gsum = pf_gsum_;
    g.partial = pf_part_;
    g.partial_floats = pf_part_floats_;
    g.err = err_;
    cuda_check(prefill_gemm(g, stream_), "prefill_gemm launch");
}

// One block (Engine.cpp:71-103) for `rows` prompt tokens at positions
// pos0 .. pos0+rows-1: each product runs once over all rows (the weights are
// streamed once per batch tile instead of once per token).
void Engine::enqueue_prefill_layer(int i, int rows, int pos0, int seq) {
    const auto& c = c_;
    const int H = c.hidden;
    const int W = qd_ + 2 * kvd_;
    // one product over all rows; slot: the product's first weight among the
    // layer's seven maps
    auto gemv = [&](GemvRequest& r, int slot) { enqueue_product(r, pf_gemm_ ? layer_maps(i, slot) : nullptr); };
    auto all_reduce_into_x = [&]() {
        const size_t n = (size_t)rows * H;
        nccl_check(nccl().AllReduce(pf_partial_, pf_partial_, n, ncclFloat, ncclSum, comm_, stream_),
                   "ncclAllReduce");
        cuda_check(residual_add(pf_x_, pf_partial_, n, stream_), "residual_add");
    };
    const Layer& L = layers_[i];
    const size_t kv_layer = (size_t)seq * seq_elems_ + (size_t)i * KVHl_ * c.capacity * c.head_dim;
    {
        GemvRequest r;
        r.nseg = 3;
        r.seg[0] = {L.q, pf_qkv_, L.tq, qd_};
        r.seg[1] = {L.k, pf_qkv_ + qd_, L.tk, kvd_};
        r.seg[2] = {L.v, pf_qkv_ + qd_ + kvd_, L.tv, kvd_};
        r.K = H;
        r.M = rows;
        r.ldx = H;
        r.ldy = W;
        r.x = pf_x_;
        r.gamma = L.attn_norm;
        r.eps = c.eps;
        r.epilogue = EPI_STORE;
        r.err = err_;
        r.pdl = true;
        gemv(r, 0);
    }
    {
        PrefillQkArgs a;
        a.qkv = pf_qkv_;
        a.ld_qkv = W;
        a.q_gamma = L.q_norm;
        a.k_gamma = L.k_norm;
        a.q_out = pf_q_;
        a.k_cache = kcache_ + kv_layer;
        a.v_cache = vcache_ + kv_layer;
        a.capacity = c.capacity;
        a.pos0 = pos0;
        a.heads = Hl_;
        a.kv_heads = KVHl_;
        a.eps = c.eps;
        a.rope_base = c.rope_base;
        cuda_check(prefill_qk(a, rows, stream_), "prefill_qk launch");
    }
    {
        PrefillAttnArgs a;
        a.q = pf_q_;
        a.k_cache = kcache_ + kv_layer;
        a.v_cache = vcache_ + kv_layer;
        a.out = pf_att_;
        a.capacity = c.capacity;
        a.pos0 = pos0;
        a.heads = Hl_;
        a.kv_heads = KVHl_;
        a.kmap = &kmap_;
        a.vmap = &vmap_;
        a.row_base = (int)(kv_layer / c.head_dim);
        a.err = err_;
        cuda_check(prefill_attention(a, rows, stream_), "prefill_attention launch");
    }
    {
        GemvRequest r;
        r.nseg = 1;
        r.seg[0] = {L.o, world_ > 1 ? pf_partial_ : pf_x_, L.to, H};
        r.K = qd_;
        r.M = rows;
        r.ldx = qd_;
        r.ldy = H;
        r.x = pf_att_;
        r.epilogue = world_ > 1 ? EPI_STORE : EPI_ADD;
        r.err = err_;
        r.pdl = true;
        gemv(r, 3);
        if (world_ > 1) all_reduce_into_x();
    }
    {
        GemvRequest r;
        r.nseg = 2;
        r.seg[0] = {L.gate, pf_act_, L.tgate, ffn_l_};
        r.seg[1] = {L.up, pf_act_, L.tup, ffn_l_};
        r.K = H;
        r.M = rows;
        r.ldx = H;
        r.ldy = ffn_l_;
        r.x = pf_x_;
        r.gamma = L.ffn_norm;
        r.eps = c.eps;
        r.epilogue = EPI_SWIGLU;
        r.err = err_;
        r.pdl = true;
        gemv(r, 4);
    }
    {
        GemvRequest r;
        r.nseg = 1;
        r.seg[0] = {L.down, world_ > 1 ? pf_partial_ : pf_x_, L.tdown, H};
        r.K = ffn_l_;
        r.M = rows;
        r.ldx = ffn_l_;
        r.ldy = H;
        r.x = pf_act_;
        r.epilogue = world_ > 1 ? EPI_STORE : EPI_ADD;
        r.err = err_;
        r.pdl = true;
        gemv(r, 6);
        if (world_ > 1) all_reduce_into_x();
    }
}

uint32_t Engine::prefill(const uint32_t* tokens_host, int n, int position, float* logits_host, int seq) {
    require_live();
    if (!loaded_) throw Error(Q4K_EINVAL, "weights are not loaded");
    if (seq < 0 || seq >= seqs_) throw Error(Q4K_ERANGE, "sequence out of range");
    if (n <= 0 || !tokens_host) throw Error(Q4K_EINVAL, "prefill needs at least one token");
    // Engine.cpp:126-128 (capacity) and EmbedLookup's token check
    if (position < 0 || (long long)position + n > c_.capacity) throw Error(Q4K_ERANGE, "KV cache capacity exceeded");
    for (int t = 0; t < n; ++t)
        if (tokens_host[t] >= (uint32_t)c_.vocab) throw Error(Q4K_ERANGE, "Token ID out of range");
    ensure_prefill();
    if (pf_gemm_) ensure_prefill_maps();
    const int H = c_.hidden;
    // the head's argmax writes the token; the position is the last row's
    stage_io(0, position + n - 1, 0);
    int rows = 0;
    for (int t0 = 0; t0 < n; t0 += pf_rows_) {
        rows = std::min(pf_rows_, n - t0);
        cuda_check(cudaMemcpyAsync(pf_tokens_, tokens_host + t0, sizeof(uint32_t) * rows, cudaMemcpyHostToDevice,
                                   stream_),
                   "h2d tokens");
        cuda_check(embed_rows(token_embd_, t_embd_, H, c_.vocab, pf_tokens_, rows, pf_x_, err_, stream_, false),
                   "embed");
        for (int i = 0; i < c_.layers; ++i) enqueue_prefill_layer(i, rows, position + t0, seq);
    }
    // Engine.cpp:106-111: only the last prompt token's state feeds the head
    cuda_check(cudaMemcpyAsync(x_, pf_x_ + (size_t)(rows - 1) * H, sizeof(float) * H, cudaMemcpyDeviceToDevice,
                               stream_),
               "last row");
    enqueue_head(false);
    if (logits_host)
        cuda_check(cudaMemcpyAsync(logits_host, logits_, sizeof(float) * (vocab1_ - vocab0_), cudaMemcpyDeviceToHost,
                                   stream_),
                   "d2h logits");
    check_device_error(true);
    return host_io_[kHostOut + kIoToken];
}

void Engine::ensure_batch() {
    if (b_cap_) return;
    const int B = std::min(seqs_, pf_rows_);
    const size_t H = c_.hidden, W = (size_t)qd_ + 2 * kvd_;
    b_x_ = static_cast<float*>(alloc(sizeof(float) * B * H));
    b_qkv_ = static_cast<float*>(alloc(sizeof(float) * B * W));
    b_att_ = static_cast<float*>(alloc(sizeof(float) * B * (size_t)qd_));
    b_act_ = static_cast<float*>(alloc(sizeof(float) * B * (size_t)ffn_l_));
    b_logits_ = static_cast<float*>(alloc(sizeof(float) * B * (size_t)(vocab1_ - vocab0_)));
    // split partials for up to splits_ CTAs per KV head (a batch of one)
    b_part_o_ = static_cast<float*>(alloc(sizeof(float) * B * (size_t)Hl_ * splits_ * c_.head_dim));
    b_part_ml_ = static_cast<float*>(alloc(sizeof(float) * B * (size_t)Hl_ * splits_ * 2));
    b_counters_ = static_cast<unsigned*>(alloc(sizeof(unsigned) * B * (size_t)KVHl_));
    cuda_check(cudaMemsetAsync(b_counters_, 0, sizeof(unsigned) * B * (size_t)KVHl_, stream_), "memset");
    b_pos_ = static_cast<int*>(alloc(sizeof(int) * B));
    b_seq_ = static_cast<int*>(alloc(sizeof(int) * B));
    b_tok_ = static_cast<uint32_t*>(alloc(sizeof(uint32_t) * B));
    b_next_ = static_cast<uint32_t*>(alloc(sizeof(uint32_t) * B));
    if (world_ > 1) {
        b_partial_ = static_cast<float*>(alloc(sizeof(float) * B * H));
        b_cand_ = static_cast<uint32_t*>(alloc(sizeof(uint32_t) * 2 * B));
        b_cand_all_ = static_cast<uint32_t*>(alloc(sizeof(uint32_t) * 2 * B * (size_t)world_));
    }
    b_cap_ = B;
}

// One block (Engine.cpp:71-103) for n tokens of n sequences: the products
// over all rows, attention per token over its own sequence's cache.
void Engine::enqueue_batch_layer(int i, int n, int splits) {
    const auto& c = c_;
    const int H = c.hidden;
    const int W = qd_ + 2 * kvd_;
    auto product = [&](GemvRequest& r, int slot) { enqueue_product(r, pf_gemm_ ? layer_maps(i, slot) : nullptr); };
    // tp_world > 1: the row-parallel products write partial sums, summed over
    // the ranks and added to the residual stream (Engine.cpp:94-95, :101-102)
    auto all_reduce_into_x = [&]() {
        const size_t cnt = (size_t)n * H;
        nccl_check(nccl().AllReduce(b_partial_, b_partial_, cnt, ncclFloat, ncclSum, comm_, stream_),
                   "ncclAllReduce");
        cuda_check(residual_add(b_x_, b_partial_, cnt, stream_), "residual_add");
    };
    const Layer& L = layers_[i];
    const size_t kv_layer = (size_t)i * KVHl_ * c.capacity * c.head_dim;
    {
        GemvRequest r;
        r.nseg = 3;
        r.seg[0] = {L.q, b_qkv_, L.tq, qd_};
        r.seg[1] = {L.k, b_qkv_ + qd_, L.tk, kvd_};
        r.seg[2] = {L.v, b_qkv_ + qd_ + kvd_, L.tv, kvd_};
        r.K = H;
        r.M = n;
        r.ldx = H;
        r.ldy = W;
        r.x = b_x_;
        r.gamma = L.attn_norm;
        r.eps = c.eps;
        r.epilogue = EPI_STORE;
        r.err = err_;
        r.pdl = true;
        product(r, 0);
    }
    {
        DecodeAttnArgs a;
        a.qkv = b_qkv_;
        a.q_gamma = L.q_norm;
        a.k_gamma = L.k_norm;
        a.k_cache = kcache_ + kv_layer;
        a.v_cache = vcache_ + kv_layer;
        a.capacity = c.capacity;
        a.position = b_pos_;
        a.heads = Hl_;
        a.kv_heads = KVHl_;
        a.eps = c.eps;
        a.rope_base = c.rope_base;
        a.partial_o = b_part_o_;
        a.partial_ml = b_part_ml_;
        a.counters = b_counters_;
        a.out = b_att_;
        a.err = err_;
        a.splits = splits;
        a.row_base = i * KVHl_ * c.capacity;
        a.batch = n;
        a.seq_of = b_seq_;
        a.ld_qkv = W;
        a.seq_cache_elems = (long long)seq_elems_;
        cuda_check(decode_attention(a, kmap_, vmap_, stream_, true), "attention launch");
    }
    {
        GemvRequest r;
        r.nseg = 1;
        r.seg[0] = {L.o, world_ > 1 ? b_partial_ : b_x_, L.to, H};
        r.K = qd_;
        r.M = n;
        r.ldx = qd_;
        r.ldy = H;
        r.x = b_att_;
        r.epilogue = world_ > 1 ? EPI_STORE : EPI_ADD;
        r.err = err_;
        r.pdl = true;
        product(r, 3);
        if (world_ > 1) all_reduce_into_x();
    }
    {
        GemvRequest r;
        r.nseg = 2;
        r.seg[0] = {L.gate, b_act_, L.tgate, ffn_l_};
        r.seg[1] = {L.up, b_act_, L.tup, ffn_l_};
        r.K = H;
        r.M = n;
        r.ldx = H;
        r.ldy = ffn_l_;
        r.x = b_x_;
        r.gamma = L.ffn_norm;
        r.eps = c.eps;
        r.epilogue = EPI_SWIGLU;
        r.err = err_;
        r.pdl = true;
        product(r, 4);
    }
    {
        GemvRequest r;
        r.nseg = 1;
        r.seg[0] = {L.down, world_ > 1 ? b_partial_ : b_x_, L.tdown, H};
        r.K = ffn_l_;
        r.M = n;
        r.ldx = ffn_l_;
        r.ldy = H;
        r.x = b_act_;
        r.epilogue = world_ > 1 ? EPI_STORE : EPI_ADD;
        r.err = err_;
        r.pdl = true;
        product(r, 6);
        if (world_ > 1) all_reduce_into_x();
    }
}

int Engine::stage_batch(int n, const int* seqs, const uint32_t* tokens, const int* positions) {
    if (!loaded_) throw Error(Q4K_EINVAL, "weights are not loaded");
    ensure_prefill();
    if (n < 1 || n > std::min(seqs_, pf_rows_)) throw Error(Q4K_ERANGE, "batch size out of range");
    if (!seqs || !positions) throw Error(Q4K_EINVAL, "batched step needs sequences and positions");
    std::vector<char> used(seqs_, 0);
    for (int b = 0; b < n; ++b) {
        if (seqs[b] < 0 || seqs[b] >= seqs_) throw Error(Q4K_ERANGE, "sequence out of range");
        if (used[seqs[b]]++) throw Error(Q4K_EINVAL, "a sequence appears twice in one step");
        if (tokens && tokens[b] >= (uint32_t)c_.vocab) throw Error(Q4K_ERANGE, "Token ID out of range");
        if (positions[b] < 0 || positions[b] >= c_.capacity) throw Error(Q4K_ERANGE, "KV cache capacity exceeded");
    }
    if (pf_gemm_) ensure_prefill_maps();
    ensure_batch();
    // Attention CTAs per token and KV head: with one CTA per SM, a split count
    // s costs about ceil(n * kv_heads * s / SMs) waves of ceil(tiles / s)
    // 64-position tiles each, plus about a tile for the cross-split merge;
    // take the cheapest (the smallest s on ties). One token gets the
    // single-token count.
    int max_pos = 0;
    for (int b = 0; b < n; ++b) max_pos = std::max(max_pos, positions[b]);
    const long long tiles = max_pos / 64 + 1, sms = sm_count();
    int splits = 1;
    long long best = -1;
    for (int sp = 1; sp <= splits_; ++sp) {
        const long long waves = ((long long)n * KVHl_ * sp + sms - 1) / sms;
        const long long cost = waves * ((tiles + sp - 1) / sp) + (sp > 1 ? 1 : 0);
        if (best < 0 || cost < best) {
            best = cost;
            splits = sp;
        }
    }
    if (n == 1) splits = splits_;
    if (const char* e = std::getenv("Q4K_BATCH_SPLITS")) splits = std::min(std::max(1, std::atoi(e)), splits_);
    cuda_check(cudaMemcpyAsync(b_seq_, seqs, sizeof(int) * n, cudaMemcpyHostToDevice, stream_), "h2d");
    cuda_check(cudaMemcpyAsync(b_pos_, positions, sizeof(int) * n, cudaMemcpyHostToDevice, stream_), "h2d");
    if (tokens) cuda_check(cudaMemcpyAsync(b_tok_, tokens, sizeof(uint32_t) * n, cudaMemcpyHostToDevice, stream_), "h2d");
    return splits;
}

void Engine::decode_batch(int n, const int* seqs, const uint32_t* tokens, const int* positions, uint32_t* next_host,
                          float* logits_host) {
    require_live();
    if (!tokens) throw Error(Q4K_EINVAL, "batched decode needs tokens");
    const int splits = stage_batch(n, seqs, tokens, positions);
    const int H = c_.hidden;
    const int vocab_l = (int)(vocab1_ - vocab0_);
    cuda_check(embed_rows(token_embd_, t_embd_, H, c_.vocab, b_tok_, n, b_x_, err_, stream_, false), "embed");
    for (int i = 0; i < c_.layers; ++i) enqueue_batch_layer(i, n, splits);
    {
        // output head on every row (Engine.cpp:106-111), then each row's argmax
        GemvRequest r;
        r.nseg = 1;
        const size_t row_bytes = q4k_device_row_bytes(t_embd_, H);
        r.seg[0] = {token_embd_ + (size_t)vocab0_ * row_bytes, b_logits_, t_embd_, vocab_l};
        r.K = H;
        r.M = n;
        r.ldx = H;
        r.ldy = vocab_l;
        r.x = b_x_;
        r.gamma = output_norm_;
        r.eps = c_.eps;
        r.epilogue = EPI_STORE;
        r.err = err_;
        r.pdl = true;
        enqueue_product(r, pf_gemm_ ? pf_head_map_ : nullptr);
    }
    argmax_rows_kernel<<<n, 1024, 0, stream_>>>(b_logits_, vocab_l, b_next_, world_ > 1 ? b_cand_ : nullptr,
                                                (uint32_t)vocab0_);
    cuda_check(cudaGetLastError(), "argmax launch");
    if (world_ > 1) {
        // each rank's shard winners, then the lowest-index-first merge per row
        nccl_check(nccl().AllGather(b_cand_, b_cand_all_, 2 * (size_t)n, ncclUint32, comm_, stream_),
                   "ncclAllGather");
        merge_row_candidates_kernel<<<(n + 127) / 128, 128, 0, stream_>>>(b_cand_all_, world_, n, b_next_);
        cuda_check(cudaGetLastError(), "merge launch");
    }
    cuda_check(cudaMemcpyAsync(next_host, b_next_, sizeof(uint32_t) * n, cudaMemcpyDeviceToHost, stream_), "d2h");
    if (logits_host)
        cuda_check(cudaMemcpyAsync(logits_host, b_logits_, sizeof(float) * n * (size_t)vocab_l, cudaMemcpyDeviceToHost,
                                   stream_),
                   "d2h logits");
    check_device_error();
}

void Engine::layer_batch(int layer, int n, const int* seqs, const int* positions, const float* x_host,
                         float* x_out_host) {
    require_live();
    if (layer < 0 || layer >= c_.layers) throw Error(Q4K_ERANGE, "layer out of range");
    if (!x_host || !x_out_host) throw Error(Q4K_EINVAL, "layer rows need input and output");
    const int splits = stage_batch(n, seqs, nullptr, positions);
    const size_t bytes = sizeof(float) * (size_t)n * c_.hidden;
    cuda_check(cudaMemcpyAsync(b_x_, x_host, bytes, cudaMemcpyHostToDevice, stream_), "h2d x");
    enqueue_batch_layer(layer, n, splits);
    cuda_check(cudaMemcpyAsync(x_out_host, b_x_, bytes, cudaMemcpyDeviceToHost, stream_), "d2h x");
    check_device_error();
}

void Engine::layer_rows(int layer, int seq, int n, int position, const float* x_host, float* x_out_host) {
    require_live();
    if (!loaded_) throw Error(Q4K_EINVAL, "weights are not loaded");
    if (layer < 0 || layer >= c_.layers) throw Error(Q4K_ERANGE, "layer out of range");
    if (seq < 0 || seq >= seqs_) throw Error(Q4K_ERANGE, "sequence out of range");
    if (!x_host || !x_out_host || n <= 0) throw Error(Q4K_EINVAL, "layer rows need at least one row");
    if (position < 0 || (long long)position + n > c_.capacity) throw Error(Q4K_ERANGE, "KV cache capacity exceeded");
    ensure_prefill();
    if (n > pf_rows_) throw Error(Q4K_ERANGE, "more rows than one prefill pass holds");
    if (pf_gemm_) ensure_prefill_maps();
    const size_t bytes = sizeof(float) * (size_t)n * c_.hidden;
    cuda_check(cudaMemcpyAsync(pf_x_, x_host, bytes, cudaMemcpyHostToDevice, stream_), "h2d x");
    enqueue_prefill_layer(layer, n, position, seq);
    cuda_check(cudaMemcpyAsync(x_out_host, pf_x_, bytes, cudaMemcpyDeviceToHost, stream_), "d2h x");
    check_device_error();
}

void Engine::layer_step(int layer, const float* x_host, int position, float* x_out_host) {
    require_live();
    if (!loaded_) throw Error(Q4K_EINVAL, "weights are not loaded");
    if (layer < 0 || layer >= c_.layers) throw Error(Q4K_ERANGE, "layer out of range");
    if (position < 0 || position >= c_.capacity) throw Error(Q4K_ERANGE, "KV cache capacity exceeded");
    host_io_[kIoPos] = (uint32_t)position;
    cuda_check(cudaMemcpyAsync(pos_, &host_io_[kIoPos], 4, cudaMemcpyHostToDevice, stream_), "h2d");
    cuda_check(cudaMemcpyAsync(x_, x_host, sizeof(float) * c_.hidden, cudaMemcpyHostToDevice, stream_), "h2d x");
    enqueue_layer(layer, false);
    cuda_check(cudaMemcpyAsync(x_out_host, x_, sizeof(float) * c_.hidden, cudaMemcpyDeviceToHost, stream_), "d2h x");
    check_device_error();
}

}  // namespace q4k
