// gk_noalloc.cu - gk_puct_search_hash_noalloc: the injected-evaluator search
// with its scratch in a fixed device array instead of a caller workspace.
//
// Who needs it: callers that can hand over device buffers for inputs and
// outputs but cannot allocate device memory on the call path - a binding
// from a host language with no CUDA allocator of its own (a cgo, JNI or
// plain ctypes stub that only holds pointers it was given), or a service
// whose device memory budget is fixed at start-up and may not grow while it
// serves requests. Everything else in this library takes its scratch from
// the caller (sized by *_workspace_bytes); this entry point is the one
// exception.
//
// Scratch: one file-scope __device__ array of GK_NOALLOC_SCRATCH_BYTES per
// device, reserved by the driver when this module loads. Its address is
// resolved once per device with cudaGetSymbolAddress, on the first call
// made with that device current; make that first call before any stream
// capture. The search itself is gk_puct_search_hash on that array. All calls
// on a device share the array, so calls that overlap in time (two streams,
// two host threads) race on it: the caller serialises them.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "../../include/gk.h"
#include "gk_launch.cuh"

namespace {

static __device__ __align__(256) uint8_t g_search_scratch[GK_NOALLOC_SCRATCH_BYTES];

// Address of g_search_scratch on each device (null until resolved). Two host
// threads resolving the same device concurrently store the same value.
std::atomic<void*> g_scratch_address[64];

int scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return GK_EINVAL;
    void* p = g_scratch_address[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
        e = cudaGetSymbolAddress(&p, g_search_scratch);
        if (e != cudaSuccess) return (int)e;
        if (p == nullptr) return (int)cudaErrorInvalidSymbol;
        g_scratch_address[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return 0;
}

}  // namespace

extern "C" {

int gk_puct_search_hash_noalloc(int64_t batch, int simulations, const uint32_t* root_bits,
                                const gk_puct_options* options, const gk_puct_results_t* results, void* stream) {
    if (batch < 1 || simulations < 1 || root_bits == nullptr || options == nullptr || results == nullptr)
        return GK_EINVAL;
    const int capacity = simulations + 1;
    const size_t need = gk_puct_workspace_bytes(batch, capacity);
    if (need == 0) return GK_EINVAL;
    if (need > (size_t)GK_NOALLOC_SCRATCH_BYTES) return GK_ENOSPC;
    void* ws = nullptr;
    int s = scratch_for_current_device(&ws);
    if (s) return s;
    // The search draws no root noise, so the noise rows must read as zero;
    // the array still holds the previous call's trees. Everything else is
    // initialised by the search's own begin step.
    gk_puct_buffers_t bufs;
    if ((s = gk_puct_buffers(ws, batch, capacity, &bufs))) return s;
    const cudaError_t e =
        cudaMemsetAsync(bufs.noise, 0, (size_t)batch * GK_ACTIONS * sizeof(float), gk::as_stream(stream));
    if (e != cudaSuccess) return (int)e;
    return gk_puct_search_hash(ws, batch, simulations, root_bits, options, results, stream);
}

}  // extern "C"
