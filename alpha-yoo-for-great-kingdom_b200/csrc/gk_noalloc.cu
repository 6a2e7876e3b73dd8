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
// device, reserved by the driver when this module loads into a context. In
// host code the array's name is only a host-side stand-in, so its device
// address is resolved with cudaGetSymbolAddress, with the device current, on
// the first call made in each CUDA context (set-up; make that first call
// before any stream capture). The address is cached per device together with
// the context's unique id: after a device reset, or in another context on the
// same device, the module is loaded again and the address is resolved again.
// The search itself is gk_puct_search_hash on that array. All calls on a
// device share the array, so calls that overlap in time (two streams, two
// host threads) race on it: the caller serialises them.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/gk.h"
#include "gk_launch.cuh"

namespace {

static __device__ __align__(256) uint8_t g_search_scratch[GK_NOALLOC_SCRATCH_BYTES];

// Per device: the unique id of the context the address was resolved in, and
// the address (0 / null until resolved). Two host threads resolving in the
// same context store the same pair.
struct ScratchSlot {
    std::mutex lock;
    unsigned long long context_id = 0;
    void* address = nullptr;
};
ScratchSlot g_scratch[64];

// The two driver calls that name the current context, fetched through the
// runtime so the library needs no link-time dependency on the driver library.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;
std::once_flag g_driver_once;
cudaError_t g_driver_status = cudaSuccess;

cudaError_t load_driver_calls() {
    std::call_once(g_driver_once, [] {
        cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound, q2 = q1;
        void* f1 = nullptr;
        void* f2 = nullptr;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f1, 12000, cudaEnableDefault, &q1);
        if (e == cudaSuccess)
            e = cudaGetDriverEntryPointByVersion("cuCtxGetId", &f2, 12000, cudaEnableDefault, &q2);
        if (e == cudaSuccess && (q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess || !f1 || !f2))
            e = cudaErrorSymbolNotFound;
        g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
        g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f2);
        g_driver_status = e;
    });
    return g_driver_status;
}

int scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return GK_EINVAL;
    if ((e = load_driver_calls()) != cudaSuccess) return (int)e;
    CUcontext ctx = nullptr;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) return (int)cudaErrorInitializationError;
    void* p = nullptr;
    if (ctx == nullptr) {
        // The runtime has not made a context current on this thread yet:
        // resolving the symbol does, then the context is known.
        if ((e = cudaGetSymbolAddress(&p, g_search_scratch)) != cudaSuccess) return (int)e;
        if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return (int)cudaErrorInitializationError;
    }
    unsigned long long id = 0;
    if (g_ctx_get_id(ctx, &id) != CUDA_SUCCESS) return (int)cudaErrorInitializationError;
    ScratchSlot& slot = g_scratch[dev];
    std::lock_guard<std::mutex> guard(slot.lock);
    if (slot.address == nullptr || slot.context_id != id) {
        if (p == nullptr && (e = cudaGetSymbolAddress(&p, g_search_scratch)) != cudaSuccess) return (int)e;
        if (p == nullptr) return (int)cudaErrorInvalidSymbol;
        slot.address = p;
        slot.context_id = id;
    }
    *out = slot.address;
    return 0;
}

}  // namespace

extern "C" {

int gk_puct_search_hash_noalloc(int64_t batch, int simulations, const uint32_t* root_bits,
                                const gk_puct_options* options, const gk_puct_results_t* results, void* stream) {
    if (batch < 1 || simulations < 1 || root_bits == nullptr || options == nullptr || results == nullptr)
        return GK_EINVAL;
    // This search draws no root noise; a nonzero weight would mix in noise
    // rows that nobody drew.
    if (options->dirichlet_epsilon != 0.0) return GK_EINVAL;
    // Every node holds at least its 64-byte state: bound the request before
    // any size arithmetic can overflow.
    constexpr int64_t kMaxNodes = (int64_t)(GK_NOALLOC_SCRATCH_BYTES / 64);
    if (simulations >= kMaxNodes || batch > kMaxNodes / (simulations + 1)) return GK_ENOSPC;
    const int capacity = simulations + 1;
    const size_t need = gk_puct_workspace_bytes(batch, capacity);
    if (need == 0) return GK_EINVAL;
    if (need > (size_t)GK_NOALLOC_SCRATCH_BYTES) return GK_ENOSPC;
    void* ws = nullptr;
    const int s = scratch_for_current_device(&ws);
    if (s) return s;
    // The array still holds the previous call's trees; the search's begin
    // step writes every per-tree field it reads, and with no root noise the
    // noise rows are never read.
    return gk_puct_search_hash(ws, batch, simulations, root_bits, options, results, stream);
}

}  // extern "C"
