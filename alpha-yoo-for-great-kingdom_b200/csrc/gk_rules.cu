// gk_rules.cu - batched rules, encoder, playout and position-generator kernels
// and their C-ABI entry points (declared in include/gk.h).
//
// Layouts in HBM
//   wire records  int32 [N,170]  (python/kingdom_ai/gpu_rules.py:16-33)
//   packed states uint32[N,16]   (gk_bits, 64 B; include/gk_common.h)
//   features      fp32  [N,10,9,9], masks bool [N,82]
// Wire-record kernels stage whole blocks of records through shared memory
// with coalesced 16-byte loads and stores; one thread then owns one state in
// registers. The packed-state transition reads and writes each 64-byte state
// directly, and the packed-state encoder builds its output rows in shared
// memory and writes them with bulk (TMA) stores.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/gk.h"
#include "gk_device.cuh"
#include "gk_launch.cuh"
#include "gk_tc.cuh"

namespace gk {

constexpr int kRecBlock = 128;  // records per block in the wire-format kernels
constexpr int kBitsBlock = 256; // packed states per block

// ---- cooperative global<->shared copies (vectorised when aligned) -------------
template <typename T>
__device__ __forceinline__ void block_copy_in(T* dst, const T* src, int64_t count) {
    const int64_t bytes = count * (int64_t)sizeof(T);
    if (aligned16_dev(src) && (bytes & 15) == 0) {
        const int4* s = reinterpret_cast<const int4*>(src);
        int4* d = reinterpret_cast<int4*>(dst);
        for (int64_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = s[i];
    } else {
        for (int64_t i = threadIdx.x; i < count; i += blockDim.x) dst[i] = src[i];
    }
}
template <typename T>
__device__ __forceinline__ void block_copy_out(T* dst, const T* src, int64_t count) {
    const int64_t bytes = count * (int64_t)sizeof(T);
    if (aligned16_dev(dst) && (bytes & 15) == 0) {
        const int4* s = reinterpret_cast<const int4*>(src);
        int4* d = reinterpret_cast<int4*>(dst);
        for (int64_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = s[i];
    } else {
        for (int64_t i = threadIdx.x; i < count; i += blockDim.x) dst[i] = src[i];
    }
}

__device__ __forceinline__ int read_action(const void* actions, int action_bytes, int64_t i) {
    if (action_bytes == 8) {
        const int64_t a = reinterpret_cast<const int64_t*>(actions)[i];
        return (a >= 0 && a < GK_ACTIONS) ? (int)a : -1;
    }
    return reinterpret_cast<const int32_t*>(actions)[i];
}

// ---- encoder output from per-position planes held in shared memory ----------
struct PlaneSmem {
    uint32_t bits[kRecBlock][18];  // own, enemy, neutral, own_terr, enemy_terr, legal
    float consts[kRecBlock][4];    // black_to_play, own/enemy remaining, passes
    uint32_t pass_legal[kRecBlock];
};

__device__ __forceinline__ void store_planes(PlaneSmem& p, int t, const EncodePlanes& e) {
    const gk_b96 v[6] = {e.own, e.enemy, e.neutral, e.own_terr, e.enemy_terr, e.legal};
#pragma unroll
    for (int k = 0; k < 6; ++k) {
        p.bits[t][3 * k] = v[k].w[0];
        p.bits[t][3 * k + 1] = v[k].w[1];
        p.bits[t][3 * k + 2] = v[k].w[2];
    }
    p.consts[t][0] = e.black_to_play;
    p.consts[t][1] = e.own_remaining;
    p.consts[t][2] = e.enemy_remaining;
    p.consts[t][3] = e.passes;
    p.pass_legal[t] = e.pass_legal ? 1u : 0u;
}

__device__ __forceinline__ float plane_value(const PlaneSmem& p, int pos, int plane, int cell) {
    if (plane >= 5 && plane <= 8) return p.consts[pos][plane - 5];
    const int k = plane == 9 ? 5 : plane;
    const int bit = cell + cell / 9;
    return ((p.bits[pos][3 * k + (bit >> 5)] >> (bit & 31)) & 1u) ? 1.0f : 0.0f;
}

__device__ __forceinline__ uint32_t mask_byte(const PlaneSmem& p, int pos, int action) {
    if (action == GK_PASS) return p.pass_legal[pos];
    const int bit = action + action / 9;
    return (p.bits[pos][15 + (bit >> 5)] >> (bit & 31)) & 1u;
}

// Writes `count` positions' features (count*810 floats) and masks (count*82
// bytes) starting at the block's first position, with 16 B / 4 B stores.
__device__ void write_encoded(const PlaneSmem& p, int count, float* features, uint8_t* masks) {
    const int total = count * GK_FEATURES;
    int vec = 0;
    if (aligned16_dev(features)) {
        vec = total / 4;
        float4* out4 = reinterpret_cast<float4*>(features);
        for (int j = threadIdx.x; j < vec; j += blockDim.x) {
            int f = 4 * j;
            int pos = f / GK_FEATURES;
            int rem = f - pos * GK_FEATURES;
            int plane = rem / GK_CELLS;
            int cell = rem - plane * GK_CELLS;
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[q] = plane_value(p, pos, plane, cell);
                if (++cell == GK_CELLS) {
                    cell = 0;
                    if (++plane == GK_PLANES) {
                        plane = 0;
                        ++pos;
                    }
                }
            }
            out4[j] = make_float4(v[0], v[1], v[2], v[3]);
        }
        vec *= 4;
    }
    for (int f = vec + threadIdx.x; f < total; f += blockDim.x) {
        const int pos = f / GK_FEATURES, rem = f - pos * GK_FEATURES;
        features[f] = plane_value(p, pos, rem / GK_CELLS, rem % GK_CELLS);
    }
    const int mbytes = count * GK_ACTIONS;
    int mvec = 0;
    if ((reinterpret_cast<uintptr_t>(masks) & 3u) == 0) {
        mvec = mbytes / 4;
        uint32_t* out = reinterpret_cast<uint32_t*>(masks);
        for (int j = threadIdx.x; j < mvec; j += blockDim.x) {
            uint32_t word = 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int b = 4 * j + q;
                const int pos = b / GK_ACTIONS;
                word |= mask_byte(p, pos, b - pos * GK_ACTIONS) << (8 * q);
            }
            out[j] = word;
        }
        mvec *= 4;
    }
    for (int b = mvec + threadIdx.x; b < mbytes; b += blockDim.x) {
        const int pos = b / GK_ACTIONS;
        masks[b] = (uint8_t)mask_byte(p, pos, b - pos * GK_ACTIONS);
    }
}

// ---- kernels ---------------------------------------------------------------------

__global__ void initial_records_kernel(int32_t* recs, int64_t n, int neutral) {
    const int64_t total = n * GK_STATE_WIDTH;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int f = (int)(i % GK_STATE_WIDTH);
        int32_t v = 0;
        if (f == neutral) v = 3;
        else if (f == GK_ACTOR) v = 1;
        else if (f == GK_BLACK_STOCK || f == GK_WHITE_STOCK) v = GK_STONES;
        recs[i] = v;
    }
}

__global__ void initial_bits_kernel(gk_bits* bits, int64_t n, int neutral) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        bits[i] = initial_bits(neutral);
}

__global__ void __launch_bounds__(kRecBlock) play_records_kernel(int32_t* recs, const void* actions, int action_bytes,
                                                                  uint8_t* accepted, int64_t n) {
    extern __shared__ __align__(16) int32_t smem_rec[];
    for (int64_t base = (int64_t)blockIdx.x * kRecBlock; base < n; base += (int64_t)gridDim.x * kRecBlock) {
        const int count = (int)(n - base < kRecBlock ? n - base : kRecBlock);
        block_copy_in(smem_rec, recs + base * GK_STATE_WIDTH, (int64_t)count * GK_STATE_WIDTH);
        __syncthreads();
        const int t = threadIdx.x;
        if (t < count) {
            int32_t* rec = smem_rec + t * GK_STATE_WIDTH;
            gk_bits s = pack_record(rec);
            const bool ok = play(s, read_action(actions, action_bytes, base + t));
            accepted[base + t] = ok ? 1 : 0;
            if (ok) unpack_record(s, rec);
        }
        __syncthreads();
        block_copy_out(recs + base * GK_STATE_WIDTH, smem_rec, (int64_t)count * GK_STATE_WIDTH);
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kRecBlock) encode_records_kernel(const int32_t* recs, float* features,
                                                                    uint8_t* masks, int64_t n) {
    extern __shared__ __align__(16) int32_t smem_rec[];
    PlaneSmem& planes = *reinterpret_cast<PlaneSmem*>(smem_rec + kRecBlock * GK_STATE_WIDTH);
    for (int64_t base = (int64_t)blockIdx.x * kRecBlock; base < n; base += (int64_t)gridDim.x * kRecBlock) {
        const int count = (int)(n - base < kRecBlock ? n - base : kRecBlock);
        block_copy_in(smem_rec, recs + base * GK_STATE_WIDTH, (int64_t)count * GK_STATE_WIDTH);
        __syncthreads();
        if ((int)threadIdx.x < count) {
            const gk_bits s = pack_record(smem_rec + threadIdx.x * GK_STATE_WIDTH);
            store_planes(planes, threadIdx.x, encode_planes(s));
        }
        __syncthreads();
        write_encoded(planes, count, features + base * GK_FEATURES, masks + base * GK_ACTIONS);
        __syncthreads();
    }
}

// Encoder from packed states, in chunks of kEncChunk positions per block:
//   1. one thread per position computes its planes (registers -> shared);
//   2. one thread per (position, cell) writes the cell's 10 plane values and
//      its mask byte into a shared-memory image of the chunk's output rows,
//      which are contiguous in HBM (kEncChunk * 3,240 + kEncChunk * 82 bytes);
//   3. one thread hands the image to the TMA engine as two bulk stores.
// Two images alternate, so a chunk is computed while the previous one drains.
// Outputs that are not 16-byte aligned, and a final partial chunk, are
// copied out with ordinary stores instead.
constexpr int kEncChunk = 16;
constexpr int kEncThreads = 256;

struct EncodeStage {
    float feat[2][kEncChunk * GK_FEATURES];   // 2 x 51,840 B (16-byte aligned)
    uint8_t mask[2][kEncChunk * GK_ACTIONS];  // 2 x 1,312 B
    uint32_t bits[kEncChunk][18];              // own, enemy, neutral, own_terr, enemy_terr, legal
    float consts[kEncChunk][4];
    uint32_t pass_legal[kEncChunk];
};
constexpr size_t kEncSmem = sizeof(EncodeStage);

template <bool kBulk>
__global__ void __launch_bounds__(kEncThreads) encode_bits_kernel(const gk_bits* bits, float* features,
                                                                   uint8_t* masks, int64_t n) {
    extern __shared__ __align__(128) uint8_t enc_smem[];
    EncodeStage& st = *reinterpret_cast<EncodeStage*>(enc_smem);
    const int64_t chunks = (n + kEncChunk - 1) / kEncChunk;
    int buf = 0;
    for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x, buf ^= 1) {
        const int64_t base = c * kEncChunk;
        const int count = (int)(n - base < kEncChunk ? n - base : kEncChunk);
        if ((int)threadIdx.x < count) {
            const EncodePlanes e = encode_planes(bits[base + threadIdx.x]);
            const gk_b96 v[6] = {e.own, e.enemy, e.neutral, e.own_terr, e.enemy_terr, e.legal};
#pragma unroll
            for (int k = 0; k < 6; ++k) {
                st.bits[threadIdx.x][3 * k] = v[k].w[0];
                st.bits[threadIdx.x][3 * k + 1] = v[k].w[1];
                st.bits[threadIdx.x][3 * k + 2] = v[k].w[2];
            }
            st.consts[threadIdx.x][0] = e.black_to_play;
            st.consts[threadIdx.x][1] = e.own_remaining;
            st.consts[threadIdx.x][2] = e.enemy_remaining;
            st.consts[threadIdx.x][3] = e.passes;
            st.pass_legal[threadIdx.x] = e.pass_legal ? 1u : 0u;
        }
        // The image in `buf` went to a bulk store two chunks ago; it must have
        // been read out before it is overwritten.
        if (kBulk && threadIdx.x == 0) tc::bulk_wait_read<1>();
        __syncthreads();
        float* out = st.feat[buf];
        uint8_t* mout = st.mask[buf];
        for (int i = threadIdx.x; i < count * GK_CELLS; i += blockDim.x) {
            const int pos = i / GK_CELLS, cell = i - pos * GK_CELLS;
            const int bit = cell + cell / 9;
            const int w = bit >> 5, sh = bit & 31;
            const uint32_t* b = st.bits[pos];
            float* o = out + pos * GK_FEATURES + cell;
#pragma unroll
            for (int k = 0; k < 5; ++k) o[k * GK_CELLS] = ((b[3 * k + w] >> sh) & 1u) ? 1.0f : 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) o[(5 + k) * GK_CELLS] = st.consts[pos][k];
            const uint32_t legal = (b[15 + w] >> sh) & 1u;
            o[9 * GK_CELLS] = legal ? 1.0f : 0.0f;
            mout[pos * GK_ACTIONS + cell] = (uint8_t)legal;
        }
        if ((int)threadIdx.x < count) mout[threadIdx.x * GK_ACTIONS + GK_PASS] = (uint8_t)st.pass_legal[threadIdx.x];
        if (kBulk) tc::fence_proxy_async_smem();  // generic-proxy writes -> visible to the bulk copy
        __syncthreads();
        if (kBulk && count == kEncChunk) {
            if (threadIdx.x == 0) {
                tc::bulk_s2g(features + base * GK_FEATURES, tc::smem_u32(out), kEncChunk * GK_FEATURES * 4);
                tc::bulk_s2g(masks + base * GK_ACTIONS, tc::smem_u32(mout), kEncChunk * GK_ACTIONS);
                tc::bulk_commit();
            }
        } else {
            float* fdst = features + base * GK_FEATURES;
            for (int i = threadIdx.x; i < count * GK_FEATURES; i += blockDim.x) fdst[i] = out[i];
            uint8_t* mdst = masks + base * GK_ACTIONS;
            for (int i = threadIdx.x; i < count * GK_ACTIONS; i += blockDim.x) mdst[i] = mout[i];
        }
    }
    if (kBulk && threadIdx.x == 0) tc::bulk_wait<0>();
}

__global__ void __launch_bounds__(kRecBlock) records_to_bits_kernel(const int32_t* recs, gk_bits* bits,
                                                                     uint32_t* status, int64_t n) {
    extern __shared__ __align__(16) int32_t smem_rec[];
    for (int64_t base = (int64_t)blockIdx.x * kRecBlock; base < n; base += (int64_t)gridDim.x * kRecBlock) {
        const int count = (int)(n - base < kRecBlock ? n - base : kRecBlock);
        block_copy_in(smem_rec, recs + base * GK_STATE_WIDTH, (int64_t)count * GK_STATE_WIDTH);
        __syncthreads();
        if ((int)threadIdx.x < count) {
            const int32_t* rec = smem_rec + threadIdx.x * GK_STATE_WIDTH;
            if (status != nullptr && !record_in_range(rec)) atomicOr(status, GK_ERR_BAD_INPUT);
            bits[base + threadIdx.x] = pack_record(rec);
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kRecBlock) bits_to_records_kernel(const gk_bits* bits, int32_t* recs, int64_t n) {
    extern __shared__ __align__(16) int32_t smem_rec[];
    for (int64_t base = (int64_t)blockIdx.x * kRecBlock; base < n; base += (int64_t)gridDim.x * kRecBlock) {
        const int count = (int)(n - base < kRecBlock ? n - base : kRecBlock);
        if ((int)threadIdx.x < count) {
            int32_t* rec = smem_rec + threadIdx.x * GK_STATE_WIDTH;
            unpack_record(bits[base + threadIdx.x], rec);
            rec[GK_RESERVED] = 0;
        }
        __syncthreads();
        block_copy_out(recs + base * GK_STATE_WIDTH, smem_rec, (int64_t)count * GK_STATE_WIDTH);
        __syncthreads();
    }
}

// One state per thread, grid-stride. Each thread reads and writes its own
// 64-byte state directly (four 16-byte accesses when the array is 16-byte
// aligned); with no block-wide staging a state whose transition runs long
// (big flood fills) delays only its own warp. Rejected states are not
// written back.
template <bool kVector>
__global__ void __launch_bounds__(kBitsBlock) play_bits_kernel(gk_bits* bits, const void* actions, int action_bytes,
                                                                uint8_t* accepted, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        gk_bits s;
        if (kVector) {
            const uint4* src = reinterpret_cast<const uint4*>(bits + i);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 v = __ldcs(src + q);
                s.w[4 * q] = v.x;
                s.w[4 * q + 1] = v.y;
                s.w[4 * q + 2] = v.z;
                s.w[4 * q + 3] = v.w;
            }
        } else {
            s = bits[i];
        }
        const bool ok = play(s, read_action(actions, action_bytes, i));
        accepted[i] = ok ? 1 : 0;
        if (!ok) continue;
        if (kVector) {
            uint4* dst = reinterpret_cast<uint4*>(bits + i);
#pragma unroll
            for (int q = 0; q < 4; ++q)
                __stcs(dst + q, make_uint4(s.w[4 * q], s.w[4 * q + 1], s.w[4 * q + 2], s.w[4 * q + 3]));
        } else {
            bits[i] = s;
        }
    }
}

// Uniform-random playout per game (PCG32 stream (seed, game_id)); legal set in
// action-index order, placements then pass (engine/src/State.cpp:183-198).
__global__ void random_playouts_kernel(uint64_t seed, uint64_t first_game, int64_t n, int neutral, int8_t* boards,
                                       int32_t* infos) {
    for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < n; g += (int64_t)gridDim.x * blockDim.x) {
        gk_pcg32 rng = gk_pcg32_seed(seed, first_game + (uint64_t)g);
        gk_bits s = initial_bits(neutral);
        int plies = 0;
        while (gk_reason(&s) == GK_NONE) {
            const gk_b96 legal = legal_placements(s);
            const int count = gk_popc(legal) + 1;
            const int j = (int)gk_pcg32_bounded(&rng, (uint32_t)count);
            const int action = j == count - 1 ? GK_PASS : gk_bit_cell(select_bit(legal, j));
            play(s, action);
            ++plies;
        }
        const gk_b96 black = gk_get(&s, GK_PLANE_BLACK), white = gk_get(&s, GK_PLANE_WHITE);
        const gk_b96 neutral_b = gk_get(&s, GK_PLANE_NEUTRAL);
        int8_t* board = boards + g * GK_CELLS;
        for (int i = 0; i < GK_CELLS; ++i) {
            const int b = gk_cell_bit(i);
            board[i] = gk_test(black, b) ? 1 : gk_test(white, b) ? 2 : gk_test(neutral_b, b) ? 3 : 0;
        }
        const gk_b96 E = empty_cells(s);
        const int reason = gk_reason(&s);
        int32_t* info = infos + g * 5;
        info[0] = gk_winner(&s);
        info[1] = reason == GK_CAPTURE ? GK_CPP_CAPTURE : reason == GK_SUICIDE ? GK_CPP_SUICIDE : GK_CPP_TWO_PASSES;
        info[2] = gk_popc(gk_and(E, gk_get(&s, GK_PLANE_OWN_BLACK)));
        info[3] = gk_popc(gk_and(E, gk_get(&s, GK_PLANE_OWN_WHITE)));
        info[4] = plies;
    }
}

// Mid-game position generator: k ~ U[0,60] uniform legal moves from the default
// start, restarting with a fresh k from the same stream when the game ends
// within them (at most 64 attempts, then the start position).
__global__ void gen_positions_kernel(uint64_t seed, uint64_t first, int64_t n, gk_bits* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        gk_pcg32 rng = gk_pcg32_seed(seed, first + (uint64_t)i);
        gk_bits result = initial_bits(40);
        for (int attempt = 0; attempt < 64; ++attempt) {
            const int k = (int)gk_pcg32_bounded(&rng, 61u);
            gk_bits s = initial_bits(40);
            bool ok = true;
            for (int m = 0; m < k; ++m) {
                const gk_b96 legal = legal_placements(s);
                const int count = gk_popc(legal) + 1;
                const int j = (int)gk_pcg32_bounded(&rng, (uint32_t)count);
                play(s, j == count - 1 ? GK_PASS : gk_bit_cell(select_bit(legal, j)));
                if (gk_reason(&s) != GK_NONE) {
                    ok = false;
                    break;
                }
            }
            if (ok) {
                result = s;
                break;
            }
        }
        out[i] = result;
    }
}

constexpr size_t kRecSmem = (size_t)kRecBlock * GK_STATE_WIDTH * sizeof(int32_t);

int rec_grid(int64_t n) { return blocks_for(n, kRecBlock, kSmCount * 16); }

bool configure_rules_kernels() {
    static bool done[64] = {};
    return once_per_device(done, [] {
        return cudaFuncSetAttribute(play_records_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kRecSmem) == cudaSuccess &&
               cudaFuncSetAttribute(encode_records_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)(kRecSmem + sizeof(PlaneSmem))) == cudaSuccess &&
               cudaFuncSetAttribute(records_to_bits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kRecSmem) == cudaSuccess &&
               cudaFuncSetAttribute(bits_to_records_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kRecSmem) == cudaSuccess &&
               cudaFuncSetAttribute(encode_bits_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kEncSmem) == cudaSuccess &&
               cudaFuncSetAttribute(encode_bits_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kEncSmem) == cudaSuccess;
    });
}

}  // namespace gk

using namespace gk;

extern "C" {

int gk_initial_records(int32_t* recs, int64_t n, int neutral_cell, void* stream) {
    if (recs == nullptr || n < 0) return GK_EINVAL;
    if (n == 0) return 0;
    initial_records_kernel<<<blocks_for(n * GK_STATE_WIDTH, 256, kSmCount * 8), 256, 0, as_stream(stream)>>>(
        recs, n, neutral_cell >= 0 && neutral_cell < GK_CELLS ? neutral_cell : -1);
    return launch_status();
}

int gk_initial_bits(uint32_t* bits, int64_t n, int neutral_cell, void* stream) {
    if (bits == nullptr || n < 0) return GK_EINVAL;
    if (n == 0) return 0;
    initial_bits_kernel<<<blocks_for(n, 256, kSmCount * 8), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<gk_bits*>(bits), n, neutral_cell);
    return launch_status();
}

int gk_play_records(int32_t* recs, const void* actions, int action_bytes, uint8_t* accepted, int64_t n, void* stream) {
    if (recs == nullptr || actions == nullptr || accepted == nullptr || n < 0) return GK_EINVAL;
    if (action_bytes != 4 && action_bytes != 8) return GK_EINVAL;
    if (n == 0) return 0;
    if (!configure_rules_kernels()) return launch_status();
    play_records_kernel<<<rec_grid(n), kRecBlock, kRecSmem, as_stream(stream)>>>(recs, actions, action_bytes, accepted, n);
    return launch_status();
}

int gk_encode_records(const int32_t* recs, float* features, uint8_t* masks, int64_t n, void* stream) {
    if (recs == nullptr || features == nullptr || masks == nullptr || n < 0) return GK_EINVAL;
    if (n == 0) return 0;
    if (!configure_rules_kernels()) return launch_status();
    encode_records_kernel<<<rec_grid(n), kRecBlock, kRecSmem + sizeof(PlaneSmem), as_stream(stream)>>>(
        recs, features, masks, n);
    return launch_status();
}

int gk_records_to_bits(const int32_t* recs, uint32_t* bits, uint32_t* status, int64_t n, void* stream) {
    if (recs == nullptr || bits == nullptr || n < 0) return GK_EINVAL;
    if (n == 0) return 0;
    if (!configure_rules_kernels()) return launch_status();
    records_to_bits_kernel<<<rec_grid(n), kRecBlock, kRecSmem, as_stream(stream)>>>(
        recs, reinterpret_cast<gk_bits*>(bits), status, n);
    return launch_status();
}

int gk_bits_to_records(const uint32_t* bits, int32_t* recs, int64_t n, void* stream) {
    if (recs == nullptr || bits == nullptr || n < 0) return GK_EINVAL;
    if (n == 0) return 0;
    if (!configure_rules_kernels()) return launch_status();
    bits_to_records_kernel<<<rec_grid(n), kRecBlock, kRecSmem, as_stream(stream)>>>(
        reinterpret_cast<const gk_bits*>(bits), recs, n);
    return launch_status();
}

int gk_play_bits(uint32_t* bits, const void* actions, int action_bytes, uint8_t* accepted, int64_t n, void* stream) {
    if (bits == nullptr || actions == nullptr || accepted == nullptr || n < 0) return GK_EINVAL;
    if (action_bytes != 4 && action_bytes != 8) return GK_EINVAL;
    if (n == 0) return 0;
    const int grid = blocks_for(n, kBitsBlock, kSmCount * 8);
    if (aligned16(bits))
        play_bits_kernel<true><<<grid, kBitsBlock, 0, as_stream(stream)>>>(reinterpret_cast<gk_bits*>(bits), actions,
                                                                          action_bytes, accepted, n);
    else
        play_bits_kernel<false><<<grid, kBitsBlock, 0, as_stream(stream)>>>(reinterpret_cast<gk_bits*>(bits), actions,
                                                                           action_bytes, accepted, n);
    return launch_status();
}

int gk_encode_bits(const uint32_t* bits, float* features, uint8_t* masks, int64_t n, void* stream) {
    if (bits == nullptr || features == nullptr || masks == nullptr || n < 0) return GK_EINVAL;
    if (n == 0) return 0;
    if (!configure_rules_kernels()) return launch_status();
    const int grid = blocks_for(n, kEncChunk, kSmCount * 2);
    const gk_bits* states = reinterpret_cast<const gk_bits*>(bits);
    if (aligned16(features) && aligned16(masks))
        encode_bits_kernel<true><<<grid, kEncThreads, kEncSmem, as_stream(stream)>>>(states, features, masks, n);
    else
        encode_bits_kernel<false><<<grid, kEncThreads, kEncSmem, as_stream(stream)>>>(states, features, masks, n);
    return launch_status();
}

int gk_random_playouts(uint64_t seed, uint64_t first_game, int64_t n, int neutral_cell, int8_t* boards,
                       int32_t* infos, void* stream) {
    if (boards == nullptr || infos == nullptr || n < 0) return GK_EINVAL;
    if (n == 0) return 0;
    random_playouts_kernel<<<blocks_for(n, 128, kSmCount * 16), 128, 0, as_stream(stream)>>>(
        seed, first_game, n, neutral_cell >= 0 && neutral_cell < GK_CELLS ? neutral_cell : -1, boards, infos);
    return launch_status();
}

int gk_gen_positions(uint64_t seed, uint64_t first, int64_t n, uint32_t* bits, void* stream) {
    if (bits == nullptr || n < 0) return GK_EINVAL;
    if (n == 0) return 0;
    gen_positions_kernel<<<blocks_for(n, 128, kSmCount * 16), 128, 0, as_stream(stream)>>>(
        seed, first, n, reinterpret_cast<gk_bits*>(bits));
    return launch_status();
}

}  // extern "C"
