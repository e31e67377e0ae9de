// Internal launch interfaces shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

namespace q4k {

// Launch with programmatic stream serialisation: the kernel may start while
// its predecessor in the stream runs; each kernel here calls
// griddepcontrol.wait before it reads what earlier kernels wrote or writes
// what they may still read.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// Quantised matrix-vector / small-batch matrix product.
// ---------------------------------------------------------------------------
enum Epilogue : int {
    EPI_STORE = 0,   // y[m][n] = dot
    EPI_ADD = 1,     // y[m][n] += dot            (residual stream update)
    EPI_SWIGLU = 2,  // y[m][n] = silu(gate) * up (segments 0 and 1 paired row by row)
    EPI_ARGMAX = 3,  // greedy token over all rows (M == 1), optional logits in y
    EPI_PEER = 4,    // tensor-parallel partial sums (M == 1) stored into every rank's receive slot (PeerOut)
};

// Tensor-parallel row-parallel product (EPI_PEER): output row n's partial
// sum goes, as one 8-byte word (value in the low half, tag in the high
// half), to recv[r][n] of every rank r (rank r's receive slot for this
// product, this rank's row of it; peer memory mapped over NVLink). The tag
// is *epoch + 1, the decode step's number as every rank counts it, so a
// reader knows a word is this step's without a separate flag, fence or
// atomic.
constexpr int kMaxRanks = 8;
struct PeerOut {
    unsigned long long* recv[kMaxRanks] = {};
    int world = 0;
    const int* epoch = nullptr;
};

// The consuming side (a product with an RMSNorm prologue): its input row is
// x + sum over ranks r = 0 .. world-1, in that order, of the values of
// parts[r * K ..] (waiting, bounded, until every word carries this step's
// tag *epoch + 1); the row is also written to x_out (the residual stream for
// the products after this one). world may be 0: x is only copied to x_out.
struct PeerIn {
    const unsigned long long* parts = nullptr;
    int world = -1;  // < 0: not used
    const int* epoch = nullptr;
    float* x_out = nullptr;
    unsigned long long wait_ns = 2000000000ull;
};

constexpr int kMaxSegments = 4;

struct GemvSegment {
    const uint8_t* w = nullptr;  // rows in the device layout (q4k_format.h)
    float* y = nullptr;          // output of this segment: y[m * ldy + n]
    int type = 0;                // Q4K_TYPE_Q4_K or Q4K_TYPE_Q6_K
    int rows = 0;                // N of this segment
};

// Bytes that a kernel's producer asks L2 to fetch for the kernel after it,
// once its own copies are issued, so that HBM keeps streaming while the
// current kernel computes and the next one finds its operands in L2:
// `count` ranges of `bytes` each, `stride` bytes apart from `base`. With
// `position` set, a range is (*position + 1) * bytes long, clamped to
// `stride` (a KV cache up to the new token). Only a hint: nothing waits on it.
struct L2Prefetch {
    const void* base = nullptr;
    unsigned long long bytes = 0;
    unsigned long long stride = 0;
    int count = 0;
    const int* position = nullptr;
};
constexpr int kMaxPrefetch = 5;

// A batch-of-one activation already quantised the way the product kernel
// holds it in shared memory (gemv_device.cuh), written by the kernel that
// produces the activation, so that the product kernel only copies it. For
// K inputs, from `base`: codes in the Q4_K order [K], codes in the Q6_K
// order [K], scales [K/32] f32, 16-value code sums [K/16] i32, 32-value
// code sums [K/32] f32 (act_image_bytes(K) bytes; K a multiple of 256).
struct ActImage {
    uint8_t* base = nullptr;
    int K = 0;
};
inline size_t act_image_bytes(int K) { return (size_t)K * 2 + (size_t)K / 8 + (size_t)K / 4 + (size_t)K / 8; }

struct ArgmaxTarget {
    float* cand_score = nullptr;     // [grid] per-CTA best logit
    uint32_t* cand_index = nullptr;  // [grid] per-CTA best row
    unsigned* counter = nullptr;     // zero before the first launch; reset by the kernel
    uint32_t* token = nullptr;       // result: best row + index_base
    uint32_t index_base = 0;         // global index of row 0 (sharded heads)
    float* score = nullptr;          // optional: best logit
};

struct GemvRequest {
    GemvSegment seg[kMaxSegments];
    int nseg = 0;
    int K = 0;                     // inputs per row (multiple of 256)
    int M = 1;                     // activation rows
    int ldx = 0;                   // floats between activation rows (0: K)
    int ldy = 0;                   // floats between output rows (0: segment rows)
    const float* x = nullptr;      // fp32 activations [M][ldx]
    const float* gamma = nullptr;  // optional RMSNorm weight applied to x first
    float eps = 1e-6f;
    int epilogue = EPI_STORE;
    ArgmaxTarget argmax;
    int* err = nullptr;  // optional device error word (bits of q4k_device.cuh)
    unsigned long long* trace = nullptr;  // optional timeline records (q4k_device.cuh)
    int trace_tag = 0;
    int ctas = 0;        // 0: one CTA per SM
    bool pdl = false;    // launch with programmatic stream serialisation
    L2Prefetch prefetch[kMaxPrefetch];  // the next kernel's operands (optional)
    ActImage in_image;   // M == 1, no gamma: copy this quantised activation instead of quantising x
    ActImage out_image;  // EPI_SWIGLU, M == 1: also quantise the output rows into this image
    PeerOut peer_out;    // EPI_PEER
    PeerIn peer_in;      // M == 1: sum the ranks' partial sums into x first (with gamma)
};

// Plans and launches one product. Returns cudaErrorInvalidValue for shapes it
// does not support (the caller validates user-facing arguments first).
cudaError_t launch_gemv(const GemvRequest& rq, cudaStream_t stream);

int sm_count();

}  // namespace q4k
