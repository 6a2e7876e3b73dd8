// gk_replay.cu - validation of replay rows on the GPU.
//
// The checks of the reference's ReplayBuffer ingest (_validate_rows,
// python/kingdom_ai/replay.py:35-74), evaluated for every row in one pass over
// the rows (one warp per row: lanes cover the 81 cells of the ten planes and
// the 82 actions). Each failed check sets its bit in one status word; the
// caller reports the lowest bit, which is the first check in the reference's
// order that some row fails.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/gk.h"
#include "gk_launch.cuh"

namespace gk {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ bool binary(float x) { return x == 0.0f || x == 1.0f; }

__global__ void __launch_bounds__(256) replay_validate_kernel(const float* features, const uint8_t* masks,
                                                              const float* policy, const float* value,
                                                              const int8_t* to_play, int64_t n, uint32_t* out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    uint32_t bad = 0u;
    for (int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; row < n; row += warps) {
        const float* f = features + row * GK_FEATURES;
        const uint8_t* m = masks + row * GK_ACTIONS;
        const float* p = policy + row * GK_ACTIONS;
        // Cells: lane, lane + 32, lane + 64 (< 81). Planes 5..8 hold one value
        // per row, taken from cell 0.
        float first[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) first[s] = __ldg(f + (5 + s) * GK_CELLS);
        float neutral = 0.0f;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int c = lane + 32 * k;
            if (c >= GK_CELLS) continue;
            float x[GK_PLANES];
#pragma unroll
            for (int q = 0; q < GK_PLANES; ++q) x[q] = __ldg(f + q * GK_CELLS + c);
#pragma unroll
            for (int q = 0; q < GK_PLANES; ++q) {
                if (!isfinite(x[q])) bad |= GK_REPLAY_NONFINITE;
                if (x[q] < 0.0f || x[q] > 1.0f) bad |= GK_REPLAY_RANGE;
            }
            if (!binary(x[0]) || !binary(x[1]) || !binary(x[2]) || !binary(x[3]) || !binary(x[4]) ||
                !binary(x[5]) || !binary(x[9]))
                bad |= GK_REPLAY_BINARY;
#pragma unroll
            for (int s = 0; s < 4; ++s)
                if (x[5 + s] != first[s]) bad |= GK_REPLAY_SCALAR;
            if ((x[9] != 0.0f) != (m[c] != 0)) bad |= GK_REPLAY_MASK;
            if (x[0] + x[1] + x[2] > 1.0f) bad |= GK_REPLAY_STONES;
            if (x[3] + x[4] > 1.0f) bad |= GK_REPLAY_TERRITORY;
            neutral += x[2];
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) neutral += __shfl_xor_sync(kFull, neutral, off);
        if (neutral > 1.0f) bad |= GK_REPLAY_NEUTRAL;
        // Actions: lane, lane + 32, lane + 64 (< 82). The sum is taken in
        // double; the reference sums in float32 (replay.py:70-71).
        double total = 0.0;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int a = lane + 32 * k;
            if (a >= GK_ACTIONS) continue;
            const float x = __ldg(p + a);
            if (!isfinite(x)) bad |= GK_REPLAY_NONFINITE;
            if (x < 0.0f || (m[a] == 0 && x != 0.0f)) bad |= GK_REPLAY_POLICY;
            total += (double)x;
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) total += __shfl_xor_sync(kFull, total, off);
        if (lane == 0) {
            const int actor = to_play[row];
            const float v = value[row];
            if (actor != 1 && actor != 2) bad |= GK_REPLAY_ACTOR;
            if (first[0] != (actor == 1 ? 1.0f : 0.0f)) bad |= GK_REPLAY_PERSPECTIVE;
            if (first[3] != 0.0f && first[3] != 0.5f) bad |= GK_REPLAY_TERMINAL;
            if (m[GK_PASS] == 0) bad |= GK_REPLAY_PASS;
            if (!(fabs(total - 1.0) <= 1e-6)) bad |= GK_REPLAY_SUM;
            if (!(v == 1.0f || v == -1.0f)) bad |= GK_REPLAY_VALUE;
        }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) bad |= __shfl_xor_sync(kFull, bad, off);
    if (lane == 0 && bad) atomicOr(out, bad);
}

}  // namespace
}  // namespace gk

extern "C" {

int gk_replay_validate(const float* features, const uint8_t* masks, const float* policy, const float* value,
                       const int8_t* to_play, int64_t n, uint32_t* violations, void* stream) {
    using namespace gk;
    if (n < 0 || violations == nullptr) return GK_EINVAL;
    if (n > 0 && (features == nullptr || masks == nullptr || policy == nullptr || value == nullptr ||
                  to_play == nullptr))
        return GK_EINVAL;
    cudaError_t e = cudaMemsetAsync(violations, 0, sizeof(uint32_t), as_stream(stream));
    if (e != cudaSuccess) return (int)e;
    if (n == 0) return 0;
    replay_validate_kernel<<<blocks_for(n, 8, kSmCount * 8), 256, 0, as_stream(stream)>>>(features, masks, policy,
                                                                                          value, to_play, n,
                                                                                          violations);
    return launch_status();
}

}  // extern "C"
