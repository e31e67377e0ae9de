// Fixed device storage for the split-K decode attention's scratch, for the
// allocation-free entry point q4k_attention_decode_f16_static (capi.cpp).
//
// Who needs it: callers that may not allocate device memory on their token
// path. A serving process that hands all free HBM to its own KV-block pool
// at start-up has nothing left for cudaMalloc; a latency-critical loop must
// not call cudaMalloc/cudaFree (or a caching allocator such as torch's)
// because those can synchronise the device or grow a pool mid-stream. The
// regular entry point needs a caller-supplied scratch buffer, which such a
// caller could only get by allocating.
//
// The storage is one file-scope __device__ array per device (every device
// gets its own copy with the module). Its address is taken once per device
// with cudaGetSymbolAddress, with that device current, on the first call
// made while it is current; that first call should come before any stream
// capture begins; the address is kept for the life of the process, so a
// device reset after that first call is not supported. Layout is the regular scratch layout: 256 bytes of per-KV-
// head counters (they must be zero when a launch starts; static storage
// starts zeroed, the merging CTA of each head resets its counter, and the
// entry point clears them before every launch), then the split partials,
// which need no initial value. All calls on one device share the array, so
// calls that can overlap in time (different streams, or several host
// threads) race on it and must be ordered by the caller.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "engine.h"

namespace q4k {
namespace {

constexpr size_t kStaticScratchBytes = size_t(1) << 20;  // 1 MiB: up to 2016 (query head, split) partials
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_attention_scratch[kStaticScratchBytes];

std::mutex g_mutex;
void* g_address[kMaxDevices] = {};

}  // namespace

size_t attention_static_scratch_capacity() { return kStaticScratchBytes; }

// Device address of this device's static scratch; `need` bytes must fit.
void* attention_static_scratch(size_t need) {
    if (need > kStaticScratchBytes)
        throw Error(Q4K_ERANGE, "decode attention needs " + std::to_string(need) +
                                    " bytes of scratch; the static scratch holds " +
                                    std::to_string(kStaticScratchBytes) + " (use q4k_attention_decode_f16)");
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) throw Error(Q4K_ERANGE, "device ordinal out of range for static scratch");
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_address[dev]) {
        void* p = nullptr;
        cuda_check(cudaGetSymbolAddress(&p, g_attention_scratch), "cudaGetSymbolAddress(static attention scratch)");
        g_address[dev] = p;
    }
    return g_address[dev];
}

}  // namespace q4k
