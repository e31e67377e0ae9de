// Persistent decode-step kernel: one launch runs a whole token (embedding,
// 36 blocks, output head) on one CTA per SM (decode_step.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "ops.h"
#include "q4k_internal.h"

namespace q4k {

enum StepPhaseKind : int { kStepEmbed = 0, kStepGemv = 1, kStepAttention = 2 };

// One phase of the step. A phase starts on a CTA once every CTA has finished
// phase `dep` (its arrivals counter reached the grid size).
struct StepPhase {
    int kind = kStepGemv;
    int dep = -1;
    int layer = 0;
    // matrix-vector phases (kStepGemv)
    int epilogue = EPI_STORE;
    int K = 0, nb = 0;              // inputs per row, super-blocks per row
    int lpr = 8, R = 16;            // lanes per row, rows per stage
    int nseg = 1, pair = 0;         // segments; pair: SwiGLU gate (w[0]) / up (w[1]) rows together
    int total_stages = 0;
    int q4 = 0, q6 = 0;             // which code layouts the activation needs
    int mma = 0;                    // Q4_K stages on the tensor cores (16 rows, or 8 gate + 8 up rows)
    int stage_start[kMaxSegments + 1] = {};
    int row_bytes[kMaxSegments] = {};
    int type[kMaxSegments] = {};
    int rows[kMaxSegments] = {};
    const uint8_t* w[kMaxSegments] = {};
    float* y[kMaxSegments] = {};
    const float* x = nullptr;       // fp32 activation
    const float* gamma = nullptr;   // RMSNorm gamma of x (gemv) / q_norm (attention)
    const float* gamma2 = nullptr;  // k_norm (attention)
};

constexpr int kStepSlotsDefaultInflight = 4;  // no throttle: every free ring slot is filled

struct StepArgs {
    const StepPhase* phases = nullptr;  // device array
    int nphases = 0;
    unsigned* sync = nullptr;  // [nphases + 1]: arrivals per phase, then the abort flag; zero at launch
    int* err = nullptr;
    uint32_t* token = nullptr;  // in: token to embed; out: the greedy next token
    int* pos = nullptr;         // in: position; advanced by *advance at the end
    const int* advance = nullptr;
    uint32_t* history = nullptr;
    unsigned* history_n = nullptr;
    unsigned history_cap = 0;
    const uint8_t* embd = nullptr;  // token_embd, device layout
    int embd_type = 0;
    int hidden = 0, vocab = 0;
    float* x = nullptr;  // residual stream
    const float* qkv = nullptr;
    float* att = nullptr;
    uint16_t* kcache = nullptr;  // [layers][kv_heads][capacity][128]
    uint16_t* vcache = nullptr;
    int capacity = 0, heads = 0, kv_heads = 0, splits = 0;
    float eps = 1e-6f, rope_base = 1e6f;
    float* partial_o = nullptr;   // [kv_heads][splits][4][128]
    float* partial_ml = nullptr;  // [kv_heads][splits][4][2]
    unsigned* counters = nullptr; // [kv_heads], self-resetting
    ArgmaxTarget argmax;
    unsigned long long* trace = nullptr;  // optional, q4k_device.cuh layout (launch = phase)
    int inflight = kStepSlotsDefaultInflight;  // ring stages the producer lets be in flight at once
};

constexpr int kStepSlots = 4;
constexpr int kStepSlotBytes = 34 * 1024;     // one ring slot: a weight stage or a 64-position K+V tile
constexpr int kStepUnionBytes = 33 * 1024 + 512;  // activation codes, or the attention merge scratch

// Lanes per row and rows per stage for a product phase; false if no
// geometry fits the ring slot and the activation area.
bool step_gemv_geometry(int K, int max_row_bytes, bool pair, bool q4, bool q6, int& lpr, int& R);
// CTAs a launch uses (one per SM), and whether the device can hold them all
// at once (the phases wait on one another).
int step_ctas(std::string* why = nullptr);
cudaError_t launch_decode_step(const StepArgs& a, const KvTensorMap& kmap, const KvTensorMap& vmap, int ctas,
                               cudaStream_t s);

}  // namespace q4k
