// gk_launch.cuh - launch helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#define GK_EINVAL (-22)

namespace gk {

// 148 SMs on B200; grids for streaming kernels are capped at a multiple of it
// and loop grid-stride, so every SM gets equal work.
constexpr int kSmCount = 148;

inline int launch_status() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : (int)e;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
__device__ __forceinline__ bool aligned16_dev(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// One-time per-device kernel attribute setup (cudaFuncSetAttribute is per device).
template <typename F>
inline bool once_per_device(bool (&done)[64], F&& setup) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    if (done[dev]) return true;
    if (!setup()) return false;
    done[dev] = true;
    return true;
}

inline int blocks_for(int64_t n, int per_block, int cap) {
    int64_t b = (n + per_block - 1) / per_block;
    if (b < 1) b = 1;
    if (b > cap) b = cap;
    return (int)b;
}

}  // namespace gk
