// gk_net.cu - policy/value network on sm_100a tensor cores (tcgen05 + TMEM).
//
// Semantics: the batch-norm PolicyValueNet (python/kingdom_ai/model.py:30-84
// with BN folded into the convolutions and a 64-unit value hidden layer):
//   stem 3x3 (10->C) + ReLU, R residual blocks of two 3x3 convs, then
//   policy 1x1 (C->2) + ReLU -> FC 162->82, value 1x1 (C->1) + ReLU ->
//   FC 81->64 -> ReLU -> FC 64->1 -> tanh.
//
// Tower kernel (persistent, one CTA per SM, 320 threads: a weight producer,
// an MMA warp and eight epilogue warps):
//   * Images are processed in groups of G whole images, so a CTA never needs
//     another CTA's halo. Each image is stored as 100 rows (a 10x10 grid,
//     row r*10+c; column 9 and row 9 are zero padding shared by neighbours),
//     each row holding C channels in bf16.
//   * A 3x3 convolution is 9 shifted GEMMs: for tap (dr,dc) the A operand is
//     the same activation buffer shifted by dr*10+dc rows. With the K-major
//     no-swizzle layout ([C/8 chunks][rows][8 channels], 16-byte rows) a row
//     shift is just a 16-byte move of the descriptor's start address.
//   * D[128 x C] accumulates in TMEM (fp32), 9 taps x C/16 MMAs of
//     128 x C x 16 per 128-row tile. The MMA warp runs a fully unrolled
//     issue loop on warp-uniform descriptors and one elected lane issues
//     each instruction, so an MMA costs a couple of uniform adds.
//   * Weights stream from L2 into a ring of tap slots with bulk (TMA) copies
//     (no multicast) so the next taps arrive while this one runs: 11 slots
//     for C=64 (all 9 taps resident, tiles issued tile-major), 3 for C=128.
//   * Eight epilogue warps (two per TMEM lane quadrant, each owning half of
//     the channels, biases held in registers) drain TMEM (tcgen05.ld), add
//     the folded-BN bias and the residual, apply ReLU, zero the padding rows
//     and write the next layer's bf16 rows back to shared memory. After the
//     last layer a head pass computes the two 1x1 head convolutions
//     (3 channels, fp32 weights staged in shared memory).
// Heads kernel: the fully connected heads and, in search mode, the masked
// softmax, written straight into the PUCT workspace.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/gk.h"
#include "gk_device.cuh"
#include "gk_launch.cuh"
#include "gk_puct.cuh"
#include "gk_tc.cuh"

namespace gk {

template <int C>
struct NetCfg {
    static_assert(C == 32 || C == 64 || C == 128, "channels must be 32, 64 or 128");
    static constexpr int G = C == 128 ? 2 : 5;  // images per group
    static constexpr int T = C == 128 ? 2 : 4;  // 128-row tiles per group (>= 100*G rows)
    // 32 channels: two CTAs per SM (256 TMEM columns and <= 102 registers
    // each) so one CTA's epilogue latency overlaps the other's.
    static constexpr int MIN_BLOCKS = C == 32 ? 2 : 1;
    static constexpr int TMEM_COLS = 2 * T * C <= 256 ? 256 : 512;
    static constexpr int HALO = 11;              // max |tap row shift| = 10 + 1
    // Rows a kept output reads: the group's G*100 rows and a zero halo either
    // side. The tail of the last tile (rows G*100 .. T*128-1) is computed but
    // never stored; its MMAs read up to TAIL rows past a chunk, i.e. into the
    // next chunk or buffer, or into the weight slots after the last buffer.
    static constexpr int ROWS = G * 100 + 2 * HALO;
    static constexpr int TAIL = T * 128 - G * 100;
    static constexpr int CHUNK = ROWS * 16;      // bytes between 8-channel chunks
    static constexpr int ACT = (C / 8) * CHUNK;  // one activation buffer
    static constexpr int SLOT = C * C * 2;       // one tap of weights (bf16)
    static constexpr int NSLOT = C <= 64 ? 11 : 3;
    static constexpr bool TILE_OUTER = C <= 64;  // all 9 taps resident: tile-major issue order
    static constexpr int EPI_WARPS = 8;          // two per TMEM lane quadrant, each half the channels
    static constexpr int HALF = C / 2;           // channels of one epilogue warp
    static constexpr int W = HALF < 32 ? HALF : 32;  // TMEM columns per load
    // GroupNorm partial sums: [image][group][32-row chunk of the image, <= 5]
    static constexpr int GN_PARTS = G * 8 * 5;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int NBARS = 2 * NSLOT + 2 * T + 1;  // + mma_idle
    static constexpr int HEADW = (3 * C + 3 + 3) / 4 * 4;  // head 1x1 weights + biases (floats)
    static constexpr int SMEM = 2 * ACT + NSLOT * SLOT + NBARS * 8 + 16 + HEADW * 4 + 2 * GN_PARTS * 4;
    static constexpr uint32_t IDESC = tc::idesc_bf16(128, C);
    static_assert(2 * T * C <= 512, "two layers of accumulators must fit in TMEM");
    static_assert(TAIL >= 0 && TAIL * 16 <= NSLOT * SLOT, "tail reads stay inside the shared-memory allocation");
    static_assert(SMEM <= 232448, "shared memory per CTA");
};

struct NetParams {
    int channels, blocks;
    int norm;               // 0 batch norm folded, 1 GroupNorm (include/gk.h, gk_net_t)
    const float* norm_w;    // [layers][C] GroupNorm weight (norm 1)
    const float* norm_b;    // [layers][C] GroupNorm bias (norm 1)
    const float* head_norm; // [6] head GroupNorm weights and biases (norm 1)
    const uint8_t* conv_w;  // per layer, per tap: [Cin/8][Cout][8] bf16 (stem Cin padded to 16)
    const float* conv_b;    // [layers][C]
    const float* head_w;    // [3][C]: policy 1x1 (2 rows) then value 1x1 (BN folded)
    const float* head_b;    // [3]
    const float* pol_w;     // [162][82] feature-major
    const float* pol_b;     // [82]
    const float* val_w1;    // [81][H] feature-major, H = 64 (norm 0) or C (norm 1)
    const float* val_b1;    // [H]
    const float* val_w2;    // [H]
    const float* val_b2;    // [1]
};

struct NetInput {
    const gk_bits* states;    // packed states, or null
    const float* features;    // fp32 [N][10][81], or null
    const int32_t* index;     // optional gather: image i reads slot index[i]
    const int32_t* count_ptr; // optional device-side count (<= n)
    int64_t n;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ int input_count(const NetInput& in) {
    int64_t n = in.n;
    if (in.count_ptr) {
        const int64_t c = *in.count_ptr;
        n = c < n ? c : n;
    }
    return (int)(n < 0 ? 0 : n);
}

// Stem input row m of a group: 10 planes as bf16 (channels 10-15 zero).
template <int C>
__device__ __forceinline__ void build_input_row(uint8_t* buf, int m, int base_img, int nimg, const NetInput& in) {
    using K = NetCfg<C>;
    const int img = m / 100, pos = m - img * 100, r = pos / 10, c = pos - r * 10;
    uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
    if (img < nimg && r < 9 && c < 9) {
        const int idx = base_img + img;
        const int src = in.index ? in.index[idx] : idx;
        float v[10];
        if (in.states) {
            const gk_bits s = in.states[src];
            const EncodePlanes e = encode_planes(s);
            const int bit = r * 10 + c;
            v[0] = (float)gk_test(e.own, bit);
            v[1] = (float)gk_test(e.enemy, bit);
            v[2] = (float)gk_test(e.neutral, bit);
            v[3] = (float)gk_test(e.own_terr, bit);
            v[4] = (float)gk_test(e.enemy_terr, bit);
            v[5] = e.black_to_play;
            v[6] = e.own_remaining;
            v[7] = e.enemy_remaining;
            v[8] = e.passes;
            v[9] = (float)gk_test(e.legal, bit);
        } else {
            const float* f = in.features + (int64_t)src * GK_FEATURES + r * 9 + c;
#pragma unroll
            for (int k = 0; k < 10; ++k) v[k] = f[k * GK_CELLS];
        }
        lo = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                        pack_bf16x2(v[6], v[7]));
        hi = make_uint4(pack_bf16x2(v[8], v[9]), 0u, 0u, 0u);
    }
    *reinterpret_cast<uint4*>(buf + (K::HALO + m) * 16) = lo;
    *reinterpret_cast<uint4*>(buf + K::CHUNK + (K::HALO + m) * 16) = hi;
}

struct MmaBarriers {
    uint32_t slot_full, slot_free, acc_full, epi_done;
    uint32_t* status;
};

// Lane 0 waits; the outcome is broadcast so the warp's control flow stays uniform.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, uint32_t* status, bool leader) {
    int ok = 1;
    if (leader) ok = tc::mbar_wait(bar, parity, status) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    tc::tc_fence_after();
    return ok != 0;
}

// All MMAs of one 3x3 layer for the T tiles of a group, issued by the whole
// (converged) MMA warp with one elected lane per instruction. KS = K steps of
// 16 input channels per tap (1 for the stem). `a_lo`/`a_hi` are the halves of
// the descriptor of row 0 of the input buffer, `b_lo`/`b_hi` of weight slot 0;
// `c` is the running tap count that selects weight slots. A row shift or K
// step is an add to a descriptor's low half (the 14-bit start-address field
// holds addresses below 2^18 and never carries into the stride fields);
// where the loops are unrolled the added offsets are compile-time constants.
// Returns false if a bounded wait gave up.
template <int C, int KS>
__device__ __forceinline__ bool issue_layer(uint32_t tmem_d, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                            uint32_t b_hi, int c, uint32_t epi_parity, const MmaBarriers& mb,
                                            bool leader) {
    using K = NetCfg<C>;
    constexpr uint32_t kChunk16 = K::CHUNK / 16;  // A K-chunk stride in 16-byte units
    constexpr uint32_t kBChunk16 = C;             // B K-chunk stride (C rows x 16 B) in 16-byte units
    constexpr uint32_t kSlot16 = K::SLOT / 16;
    int sl = c % K::NSLOT;                         // weight slot of the layer's first tap
    uint32_t par = (uint32_t)(c / K::NSLOT) & 1u;  // and the parity of its fill
    if (K::TILE_OUTER) {
        // Weight slot and fill parity of each tap of this layer.
        int slot[9];
        uint32_t parity[9];
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
            slot[tap] = sl;
            parity[tap] = par;
            if (++sl == K::NSLOT) {
                sl = 0;
                par ^= 1u;
            }
        }
#pragma unroll
        for (int t = 0; t < K::T; ++t) {
            // Input rows of tile t come from tiles t-1..t+1 of the previous epilogue.
#pragma unroll
            for (int nb = (t == 0 ? 0 : t + 1); nb <= t + 1 && nb < K::T; ++nb)
                if (!warp_wait(mb.epi_done + 8 * nb, epi_parity, mb.status, leader)) return false;
#pragma unroll
            for (int tap = 0; tap < 9; ++tap) {
                if (t == 0 && !warp_wait(mb.slot_full + 8 * slot[tap], parity[tap], mb.status, leader)) return false;
                const int off = (tap / 3 - 1) * 10 + (tap % 3 - 1);
                const uint32_t a = a_lo + (uint32_t)(t * 128 + off);
                const uint32_t b = b_lo + (uint32_t)slot[tap] * kSlot16;
#pragma unroll
                for (int s = 0; s < KS; ++s)
                    tc::mma_bf16_warp(tmem_d + t * C, a + 2 * s * kChunk16, a_hi, b + 2 * s * kBChunk16, b_hi,
                                      K::IDESC, (tap | s) != 0);
                if (t == K::T - 1) tc::mma_commit_warp(mb.slot_free + 8 * slot[tap]);
            }
            tc::mma_commit_warp(mb.acc_full + 8 * t);
        }
    } else {
        // The tap loop stays rolled here: unrolled over 9 taps x T tiles x KS
        // steps the issue code no longer stays in the instruction cache next
        // to the epilogue's, and the tower ran twice as long.
#pragma unroll 1
        for (int tap = 0; tap < 9; ++tap) {
            if (!warp_wait(mb.slot_full + 8 * sl, par, mb.status, leader)) return false;
            const int off = (tap / 3 - 1) * 10 + (tap % 3 - 1);
            const uint32_t b = b_lo + (uint32_t)sl * kSlot16;
#pragma unroll
            for (int t = 0; t < K::T; ++t) {
                if (tap == 0) {
#pragma unroll
                    for (int nb = (t == 0 ? 0 : t + 1); nb <= t + 1 && nb < K::T; ++nb)
                        if (!warp_wait(mb.epi_done + 8 * nb, epi_parity, mb.status, leader)) return false;
                }
                const uint32_t a = a_lo + (uint32_t)(t * 128 + off);
#pragma unroll
                for (int s = 0; s < KS; ++s)
                    tc::mma_bf16_warp(tmem_d + t * C, a + 2 * s * kChunk16, a_hi, b + 2 * s * kBChunk16, b_hi,
                                      K::IDESC, (tap | s) != 0);
                if (tap == 8) tc::mma_commit_warp(mb.acc_full + 8 * t);
            }
            tc::mma_commit_warp(mb.slot_free + 8 * sl);
            if (++sl == K::NSLOT) {
                sl = 0;
                par ^= 1u;
            }
        }
    }
    return true;
}

// W TMEM columns (16 or 32) of this thread's lane.
template <int W>
__device__ __forceinline__ void tmem_ldw(uint32_t taddr, float (&v)[W]) {
    if constexpr (W == 16) tc::tmem_ld16(taddr, v);
    else tc::tmem_ld32(taddr, v);
}

// GroupNorm statistics of the reference network (GroupNorm(gcd(8, C), C),
// python/kingdom_ai/model.py:17-23, 46-47): per image and group of C/8
// channels, over the 81 cells. A 32-row chunk k of a group's rows meets at
// most two images; image `img` spans chunks gn_first(img) .. gn_last(img),
// at most five, and each chunk's warp stores its partial sums in slot
// [img][group][k - gn_first(img)], so the combine below adds them in a fixed
// order and the statistics do not depend on warp timing.
__device__ __forceinline__ int gn_first(int img) { return img * 100 / 32; }
__device__ __forceinline__ int gn_last(int img) { return (img * 100 + 99) / 32; }

__device__ __forceinline__ float gn_total(const float* parts, int img, int grp) {
    const float* p = parts + (img * 8 + grp) * 5;
    float s = 0.0f;
    for (int j = 0, n = gn_last(img) - gn_first(img); j <= n; ++j) s += p[j];
    return s;
}

// One pass of this warp over the accumulator of tile t: per group of the
// warp's half (four groups), the sums over valid cells of x and of x^2,
// reduced over the warp separately for the two images a chunk can meet (one
// reduction when the chunk lies inside one image), into `sums` and `squares`.
template <int C>
__device__ __forceinline__ void gn_partials(uint32_t tacc, int t, int q, int lane, int col0, int nimg, float* sums,
                                            float* squares) {
    using K = NetCfg<C>;
    constexpr int W = K::W, CG = C / 8;
    const int m0 = t * 128 + q * 32, m = m0 + lane;
    const int img = m / 100, pos = m - img * 100, r = pos / 10, cc = pos - r * 10;
    const bool valid = img < nimg && r < 9 && cc < 9;
    const int g0 = col0 / CG;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sq[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int cb = 0; cb < K::HALF / W; ++cb) {
        float v[W];
        tmem_ldw<W>(tacc + (uint32_t)(col0 + cb * W), v);
#pragma unroll
        for (int j = 0; j < W; ++j) {
            const int gi = (cb * W + j) / CG;
            const float x = valid ? v[j] : 0.0f;
            acc[gi] += x;
            sq[gi] = fmaf(x, x, sq[gi]);
        }
    }
    const int img0 = m0 / 100;
    const bool straddles = (m0 + 31) / 100 != img0;  // warp-uniform
    const bool second = img != img0;
    const int k = t * 4 + q;
#pragma unroll
    for (int gi = 0; gi < 4; ++gi) {
        float a = second ? 0.0f : acc[gi], b = second ? 0.0f : sq[gi];
        float c = second ? acc[gi] : 0.0f, d = second ? sq[gi] : 0.0f;
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            a += __shfl_xor_sync(0xffffffffu, a, off);
            b += __shfl_xor_sync(0xffffffffu, b, off);
            if (straddles) {
                c += __shfl_xor_sync(0xffffffffu, c, off);
                d += __shfl_xor_sync(0xffffffffu, d, off);
            }
        }
        if (lane == 0) {
            if (img0 < K::G) {
                const int slot = (img0 * 8 + g0 + gi) * 5 + (k - gn_first(img0));
                sums[slot] = a;
                squares[slot] = b;
            }
            if (straddles && img0 + 1 < K::G) {
                const int slot = ((img0 + 1) * 8 + g0 + gi) * 5 + (k - gn_first(img0 + 1));
                sums[slot] = c;
                squares[slot] = d;
            }
        }
    }
}

// GN: the reference's GroupNorm network (p.norm == 1); otherwise batch norm
// folded into conv_b. Two instantiations keep the batch-norm epilogue free of
// the GroupNorm passes.
template <int C, bool GN>
__global__ void __launch_bounds__(NetCfg<C>::THREADS, NetCfg<C>::MIN_BLOCKS)
    net_tower_kernel(NetParams p, NetInput in, float* headfeat, uint32_t* status) {
    using K = NetCfg<C>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* const bufP = smem;
    uint8_t* const bufQ = smem + K::ACT;
    uint8_t* const slots = smem + 2 * K::ACT;
    uint64_t* const bars = reinterpret_cast<uint64_t*>(slots + K::NSLOT * K::SLOT);
    uint32_t* const tmem_holder = reinterpret_cast<uint32_t*>(bars + K::NBARS);
    float* const headw = reinterpret_cast<float*>(tmem_holder + 4);  // [3][C] then [3] biases
    float* const gn_sum = headw + K::HEADW;    // GroupNorm partial sums (norm 1)
    float* const gn_sq = gn_sum + K::GN_PARTS;  // and squares
    const uint32_t slot_full = tc::smem_u32(bars);
    const uint32_t slot_free = slot_full + 8 * K::NSLOT;
    const uint32_t acc_full = slot_free + 8 * K::NSLOT;
    const uint32_t epi_done = acc_full + 8 * K::T;
    const uint32_t mma_idle = epi_done + 8 * K::T;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NL = 1 + 2 * p.blocks;  // MMA layers per group
    const int count = input_count(in);
    const int groups = (count + K::G - 1) / K::G;

    // Zero both activation buffers (halo and padding rows stay zero forever).
    for (int i = threadIdx.x; i < 2 * K::ACT / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < 3 * C; i += blockDim.x) headw[i] = p.head_w[i];
    if (threadIdx.x < 3) headw[3 * C + threadIdx.x] = p.norm ? 0.0f : p.head_b[threadIdx.x];
    tc::fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        // epi_done completes when every epilogue warp has arrived.
        for (int b = 0; b < K::NBARS; ++b) {
            const uint32_t bar = slot_full + 8 * b;
            const bool per_warp = bar >= epi_done && bar < mma_idle;
            tc::mbar_init(bar, per_warp ? (uint32_t)K::EPI_WARPS : 1u);
        }
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tc::smem_u32(tmem_holder), K::TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0 && lane == 0) {
        // ---------------- weight producer ----------------
        int c = 0;
        for (int g = blockIdx.x; g < groups; g += gridDim.x) {
            for (int l = 0; l < NL; ++l) {
                for (int tap = 0; tap < 9; ++tap, ++c) {
                    const int slot = c % K::NSLOT, round = c / K::NSLOT;
                    if (round > 0 && !tc::mbar_wait(slot_free + 8 * slot, (round - 1) & 1, status)) goto done;
                    const uint32_t bytes = l == 0 ? 16u * C * 2u : (uint32_t)K::SLOT;
                    const uint8_t* src = l == 0 ? p.conv_w + tap * bytes
                                                : p.conv_w + 9 * 16 * C * 2 + ((size_t)(l - 1) * 9 + tap) * K::SLOT;
                    tc::mbar_expect_tx(slot_full + 8 * slot, bytes);
                    tc::bulk_g2s(tc::smem_u32(slots + slot * K::SLOT), src, bytes, slot_full + 8 * slot);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: the whole warp runs the loop, one lane issues ----------------
        const MmaBarriers mb{slot_full, slot_free, acc_full, epi_done, status};
        const uint64_t bdesc = tc::smem_desc(tc::smem_u32(slots), C * 16, 128);
        const uint64_t adescP = tc::smem_desc(tc::smem_u32(bufP) + K::HALO * 16, K::CHUNK, 128);
        const uint64_t adescQ = tc::smem_desc(tc::smem_u32(bufQ) + K::HALO * 16, K::CHUNK, 128);
        const uint32_t a_hi = (uint32_t)(adescP >> 32), b_lo = (uint32_t)bdesc, b_hi = (uint32_t)(bdesc >> 32);
        const bool leader = lane == 0;
        bool ok = true;
        int c = 0, i = 0;
        for (int g = blockIdx.x; ok && g < groups; g += gridDim.x, ++i) {
            for (int l = 0; ok && l < NL; ++l, c += 9) {
                const int a = i * NL + l;  // accumulator phase index
                const uint32_t epi_parity = (uint32_t)(i * NL + l) & 1u;  // epilogue layer l of group i
                const uint32_t tmem_d = tmem + (uint32_t)((a & 1) * K::T * C);
                const uint32_t a_lo = (uint32_t)(l % 2 == 0 ? adescQ : adescP);
                ok = l == 0 ? issue_layer<C, 1>(tmem_d, a_lo, a_hi, b_lo, b_hi, c, epi_parity, mb, leader)
                            : issue_layer<C, C / 16>(tmem_d, a_lo, a_hi, b_lo, b_hi, c, epi_parity, mb, leader);
            }
        }
        // Drain: every MMA issued above completes before TMEM is released.
        __syncwarp();
        tc::mma_commit_warp(mma_idle);
        if (leader) tc::mbar_wait(mma_idle, 0, status);
        __syncwarp();
    } else if (warp >= 2) {
        // ------- epilogue: 8 warps; warp -> (TMEM lane quadrant, half of the channels) -------
        constexpr int HALF = K::HALF, W = K::W, CG = C / 8;
        const int e = warp - 2;
        const int q = warp & 3;          // TMEM lanes 32q..32q+31 = tile rows
        const int col0 = (e >> 2) * HALF; // this warp's channels [col0, col0 + C/2)
        const int etid = threadIdx.x - 64;
        constexpr bool gn = GN;
        // A wait of all eight epilogue warps: warp 0 polls the barrier
        // (bounded) and named barrier 1 releases the other seven with the
        // outcome, so they sleep instead of polling shared memory while the
        // MMAs read their operands from it; a timeout ends all eight together.
        auto group_wait = [&](uint32_t bar, uint32_t parity) -> bool {
            int ok = 1;
            if (e == 0 && lane == 0) ok = tc::mbar_wait(bar, parity, status) ? 1 : 0;
            __syncwarp();
            const bool all_ok = tc::named_barrier_and(1, 32 * K::EPI_WARPS, ok != 0);
            tc::tc_fence_after();
            return all_ok;
        };
        int i = 0;
        for (int g = blockIdx.x; g < groups; g += gridDim.x, ++i) {
            const int base_img = g * K::G;
            const int nimg = count - base_img < K::G ? count - base_img : K::G;
            // Epilogue layer 0: build the stem input (channels 0-15 of buffer Q).
            for (int m = etid; m < K::G * 100; m += 32 * K::EPI_WARPS) build_input_row<C>(bufQ, m, base_img, nimg, in);
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0)
                for (int t = 0; t < K::T; ++t) tc::mbar_arrive(epi_done + 8 * t);
            for (int l = 0; l < NL; ++l) {
                const int a = i * NL + l;
                const uint32_t colbase = (uint32_t)((a & 1) * K::T * C);
                const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + colbase;  // this quadrant's accumulators
                uint8_t* const out = l % 2 == 0 ? bufP : bufQ;
                const bool residual = l >= 2 && l % 2 == 0;
                const bool last = l == NL - 1;
                float bias[GN ? 1 : HALF];
                if constexpr (!GN) {
#pragma unroll
                    for (int j = 0; j < HALF; ++j) bias[j] = __ldg(p.conv_b + l * C + col0 + j);
                }
                if constexpr (GN) {
                    // GroupNorm statistics: sums of x and x^2 per (image,
                    // group) slot, then a named barrier of the eight warps.
                    for (int t = 0; t < K::T; ++t) {
                        if (!group_wait(acc_full + 8 * t, (uint32_t)a & 1u)) goto epi_done_label;
                        gn_partials<C>(tq + t * C, t, q, lane, col0, nimg, gn_sum, gn_sq);
                    }
                    // Every warp's partial sums are written (no warp leaves between
                    // the waits above and this barrier).
                    __syncwarp();
                    tc::named_barrier(2, 32 * K::EPI_WARPS);
                    __threadfence_block();
                }
                for (int t = 0; t < K::T; ++t) {
                    if (!gn && !group_wait(acc_full + 8 * t, (uint32_t)a & 1u)) goto epi_done_label;
                    const int m = t * 128 + q * 32 + lane;
                    const int img = m / 100, pos = m - img * 100, r = pos / 10, cc = pos - r * 10;
                    const bool valid = img < nimg && r < 9 && cc < 9;
                    const bool stored = m < K::G * 100;  // tail rows of the last tile are dropped
                    uint8_t* const row = out + (K::HALO + m) * 16;
                    float mean[4] = {0.0f, 0.0f, 0.0f, 0.0f}, rstd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    if (gn && valid) {
#pragma unroll
                        for (int gi = 0; gi < 4; ++gi) {
                            const int grp = col0 / CG + gi;
                            mean[gi] = gn_total(gn_sum, img, grp) / (float)(81 * CG);
                            const float var = gn_total(gn_sq, img, grp) / (float)(81 * CG) - mean[gi] * mean[gi];
                            rstd[gi] = 1.0f / sqrtf(fmaxf(var, 0.0f) + 1e-5f);
                        }
                    }
#pragma unroll
                    for (int cb = 0; cb < HALF / W; ++cb) {
                        const int ch0 = col0 + cb * W;
                        float v[W];
                        tmem_ldw<W>(tq + t * C + ch0, v);
                        uint4 res[W / 8];
                        if (residual && stored) {
#pragma unroll
                            for (int k = 0; k < W / 8; ++k)
                                res[k] = *reinterpret_cast<const uint4*>(row + (ch0 / 8 + k) * K::CHUNK);
                        }
#pragma unroll
                        for (int j = 0; j < W; ++j) {
                            float x;
                            if constexpr (GN) {
                                // torch's fused GroupNorm form: y = a x + b, a = rstd w, b = bias - a mean
                                const int gi = (cb * W + j) / CG;
                                const float sa = rstd[gi] * __ldg(p.norm_w + l * C + ch0 + j);
                                x = sa * v[j] + (__ldg(p.norm_b + l * C + ch0 + j) - sa * mean[gi]);
                            } else {
                                x = v[j] + bias[cb * W + j];
                            }
                            if (residual) {
                                const uint4 rv = res[j >> 3];
                                const uint32_t w = (j & 7) < 2 ? rv.x : (j & 7) < 4 ? rv.y : (j & 7) < 6 ? rv.z : rv.w;
                                x += (j & 1) ? bf16_hi(w) : bf16_lo(w);
                            }
                            v[j] = valid ? fmaxf(x, 0.0f) : 0.0f;
                        }
#pragma unroll
                        for (int k = 0; k < W / 8 && stored; ++k) {
                            const uint4 o = make_uint4(pack_bf16x2(v[8 * k], v[8 * k + 1]),
                                                       pack_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                                                       pack_bf16x2(v[8 * k + 4], v[8 * k + 5]),
                                                       pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
                            *reinterpret_cast<uint4*>(row + (ch0 / 8 + k) * K::CHUNK) = o;
                        }
                    }
                    tc::tc_fence_before();
                    if (!last) {
                        tc::fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(epi_done + 8 * t);
                    }
                }
            }
            // Head pass: the 1x1 policy (2) and value (1) convolutions over the
            // final rows, once all eight warps have written them.
            __syncwarp();
            tc::named_barrier(3, 32 * K::EPI_WARPS);
            for (int m = etid; m < K::T * 128; m += 32 * K::EPI_WARPS) {
                const int img = m / 100, pos = m - img * 100, r = pos / 10, cc = pos - r * 10;
                if (!(img < nimg && r < 9 && cc < 9)) continue;
                const uint8_t* row = bufP + (K::HALO + m) * 16;
                float h0 = headw[3 * C], h1 = headw[3 * C + 1], h2 = headw[3 * C + 2];
#pragma unroll 4
                for (int k = 0; k < C / 8; ++k) {
                    const uint4 rv = *reinterpret_cast<const uint4*>(row + k * K::CHUNK);
                    const uint32_t w[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float x = (j & 1) ? bf16_hi(w[j >> 1]) : bf16_lo(w[j >> 1]);
                        const int ch = k * 8 + j;
                        h0 = fmaf(x, headw[ch], h0);
                        h1 = fmaf(x, headw[C + ch], h1);
                        h2 = fmaf(x, headw[2 * C + ch], h2);
                    }
                }
                float* hf = headfeat + (int64_t)(base_img + img) * 243 + r * 9 + cc;
                // With GroupNorm the heads kernel normalises the raw outputs first.
                hf[0] = gn ? h0 : fmaxf(h0, 0.0f);
                hf[81] = gn ? h1 : fmaxf(h1, 0.0f);
                hf[162] = gn ? h2 : fmaxf(h2, 0.0f);
            }
        }
    epi_done_label:;
    }
done:
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, K::TMEM_COLS);
    }
}

// ---- 64-channel tower with column-fused taps ----------------------------------
// For C = 64 an MMA of N = 64 output channels is bound by shared-memory operand
// traffic (A 4 KB + B 2 KB per 128x64x16 step): the nine-tap issue pattern
// measured 2,078 cycles per 128-row tile on B200, against 1,410 for the
// pattern used here. The column taps dc = 0 and dc = +1 of each row offset dr
// share one MMA of N = 128: B = [W(dr,0) | W(dr,+1)] on A shifted by 10 dr
// rows, so the accumulator holds P0[m] (dc = 0) and P1[m] = sum_dr x[m + 10 dr]
// W(dr,+1). The tap dc = -1 is an N = 64 MMA on A shifted by 10 dr - 1 rows
// that accumulates straight into P0. The output row is then
//     y[m] = P0[m] + P1[m+1],
// a one-row shift the epilogue applies with a warp shuffle and, at TMEM
// lane-quadrant boundaries, a shared-memory exchange. Tiles start every 127
// rows: a tile's 128th row only supplies P1 to its 127th, so tiles need no
// data from one another and two sets of eight epilogue warps finish
// alternate tiles concurrently (the epilogue, not the MMA, limits a tile).
// Accumulators take 128 TMEM columns, four in a ring; tile c (a running count
// over groups, layers and tiles) waits for the epilogue of tile c-3, which
// drains its buffer (c-4) and finishes every input row it reads. Weight slot
// dr holds one row offset's [Cin/8][3][64][8] block, which gk_net_t.conv_w
// stores contiguously for 64 channels (one bulk copy); the N = 128 operand is
// its rows 64..191 (dc = 0, +1), the N = 64 operand rows 0..63 (dc = -1).
struct Cols64 {
    static constexpr int C = 64, G = 5, T = 4, HALO = 11;
    static constexpr int STRIDE = 127;            // rows between tile starts (T * 127 >= G * 100)
    static constexpr int ROWS = G * 100 + 2 * HALO;
    static constexpr int TAIL = (T - 1) * STRIDE + 128 - G * 100;
    static constexpr int CHUNK = ROWS * 16;
    static constexpr int ACT = (C / 8) * CHUNK;
    static constexpr int NACC = 2 * C;            // 128 accumulator columns per tile
    static constexpr int NBUF = 4;                // accumulators in the TMEM ring
    static constexpr int BCHUNK = 3 * C * 16;     // 3072 B per 8-channel chunk of a slot
    static constexpr int SLOT = (C / 8) * BCHUNK; // 24,576 B: one row offset's weights
    static constexpr int NSLOT = 3;
    static constexpr int SETS = 2;                // epilogue warp sets and MMA warps, alternate tiles
    static constexpr int EPI_WARPS = 8 * SETS;    // per set: 4 lane quadrants x 2 channel halves
    static constexpr int EPI0 = 1 + SETS;         // first epilogue warp (warp 0 loads weights)
    static constexpr int THREADS = 32 * (EPI0 + EPI_WARPS);
    static constexpr int NDONE = 8;               // epilogue-done barriers, a ring over tiles
    // slot_full[3], slot_free[3], acc_full[4], epi_done[8], input_ready, mma_idle, heads_ready, heads_done
    static constexpr int NBARS = 2 * NSLOT + NBUF + NDONE + 4;
    static constexpr int HEADW = (3 * C + 3 + 3) / 4 * 4;
    static constexpr int XFLOATS = SETS * 3 * 4 * 2 * 32;  // [set][3 tiles][4 quadrants][2 halves][32]
    static constexpr int SMEM = 2 * ACT + NSLOT * SLOT + NBARS * 8 + 16 + HEADW * 4 + XFLOATS * 4;
    static constexpr uint32_t IDESC128 = tc::idesc_bf16(128, 2 * C);
    static constexpr uint32_t IDESC64 = tc::idesc_bf16(128, C);
    static_assert(NBUF * NACC <= 512, "accumulators fit in TMEM");
    static_assert(T * STRIDE >= G * 100, "tiles cover the group");
    static_assert(TAIL >= 0 && TAIL * 16 <= NSLOT * SLOT, "tail reads stay inside the allocation");
    static_assert(SMEM <= 232448, "shared memory per CTA");
};

// ReLU(pre + p1) of 32 channels of one output row (zero on padding rows),
// stored as bf16 into four 8-channel chunks.
__device__ __forceinline__ void store_row32(uint8_t* row, const float (&pre)[32], const float (&p1)[32], bool valid) {
#pragma unroll
    for (int k2 = 0; k2 < 4; ++k2) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = valid ? fmaxf(pre[8 * k2 + j] + p1[8 * k2 + j], 0.0f) : 0.0f;
        *reinterpret_cast<uint4*>(row + k2 * Cols64::CHUNK) =
            make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
    }
}

// The k-th image group of CTA b out of P for `count` images. Rounds of full
// groups (5 images, 4 tiles) come first; the images left over after the last
// full round are spread over as many CTAs as take at least two each (2 to 5
// images), so the last round keeps every SM busy with shorter groups instead
// of a few SMs with full ones. A group has at least two tiles, so both MMA
// warps and both epilogue sets have work in every layer.
struct ColsGroup {
    int base, nimg, tiles;
};

__device__ __forceinline__ bool cols_group(int k, int b, int P, int count, ColsGroup& g) {
    const int full_rounds = count / (Cols64::G * P);
    if (k < full_rounds) {
        g.base = (k * P + b) * Cols64::G;
        g.nimg = Cols64::G;
        g.tiles = Cols64::T;
        return true;
    }
    const int tail0 = full_rounds * Cols64::G * P, tail = count - tail0;
    if (k > full_rounds || tail <= 0) return false;
    const int m = tail >= 2 * P ? P : (tail / 2 > 0 ? tail / 2 : 1);  // CTAs that take a tail group
    if (b >= m) return false;
    const int per = tail / m, extra = tail % m;
    g.nimg = per + (b < extra ? 1 : 0);
    g.base = tail0 + b * per + (b < extra ? b : extra);
    const int t = (g.nimg * 100 + Cols64::STRIDE - 1) / Cols64::STRIDE;
    g.tiles = t < 2 ? 2 : t;
    return true;
}

__global__ void __launch_bounds__(Cols64::THREADS, 1)
    net_tower_cols_kernel(NetParams p, NetInput in, float* headfeat, uint32_t* status) {
    using K = Cols64;
    constexpr int C = K::C;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* const bufP = smem;
    uint8_t* const bufQ = smem + K::ACT;
    uint8_t* const slots = smem + 2 * K::ACT;
    uint64_t* const bars = reinterpret_cast<uint64_t*>(slots + K::NSLOT * K::SLOT);
    uint32_t* const tmem_holder = reinterpret_cast<uint32_t*>(bars + K::NBARS);
    float* const headw = reinterpret_cast<float*>(tmem_holder + 4);  // [3][C] then [3] biases
    float* const xp1 = headw + K::HEADW;    // lane 0's P1 per set, tile, quadrant and half
    const uint32_t slot_full = tc::smem_u32(bars);
    const uint32_t slot_free = slot_full + 8 * K::NSLOT;
    const uint32_t acc_full = slot_free + 8 * K::NSLOT;
    const uint32_t epi_done = acc_full + 8 * K::NBUF;
    const uint32_t input_ready = epi_done + 8 * K::NDONE;
    const uint32_t mma_idle = input_ready + 8;
    const uint32_t heads_ready = mma_idle + 8;
    const uint32_t heads_done = heads_ready + 8;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NL = 1 + 2 * p.blocks;
    const int count = input_count(in);
    const int P = (int)gridDim.x, cta = (int)blockIdx.x;

    for (int i = threadIdx.x; i < 2 * K::ACT / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < 3 * C; i += blockDim.x) headw[i] = p.head_w[i];
    if (threadIdx.x < 3) headw[3 * C + threadIdx.x] = p.head_b[threadIdx.x];
    tc::fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        for (int b = 0; b < K::NBARS; ++b) {
            const uint32_t bar = slot_full + 8 * b;
            uint32_t n = 1u;                                           // producer / commit arrivals
            if ((bar >= slot_free && bar < acc_full) || bar == mma_idle) n = (uint32_t)K::SETS;  // each MMA warp
            if (bar >= epi_done && bar < input_ready) n = 8u;          // one epilogue set
            if (bar == input_ready || bar == heads_ready || bar == heads_done) n = (uint32_t)K::EPI_WARPS;
            tc::mbar_init(bar, n);
        }
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tc::smem_u32(tmem_holder), 512);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0 && lane == 0) {
        // ---------------- weight producer: slot dr <- row offset dr's [Cin/8][3][64][8] block ----------------
        int u = 0;  // layers issued so far (each layer fills every slot once)
        ColsGroup grp;
        for (int gk = 0; cols_group(gk, cta, P, count, grp); ++gk) {
            for (int l = 0; l < NL; ++l, ++u) {
                const int chunks = l == 0 ? 2 : C / 8;  // 8-channel input chunks (stem input padded to 16)
                for (int dr = 0; dr < 3; ++dr) {
                    if (u > 0 && !tc::mbar_wait(slot_free + 8 * dr, (uint32_t)(u - 1) & 1u, status)) goto done;
                    const uint32_t bytes = (uint32_t)(chunks * K::BCHUNK);
                    const uint8_t* src = l == 0 ? p.conv_w + dr * (2 * K::BCHUNK)
                                                : p.conv_w + 6 * K::BCHUNK + ((size_t)(l - 1) * 3 + dr) * K::SLOT;
                    tc::mbar_expect_tx(slot_full + 8 * dr, bytes);
                    tc::bulk_g2s(tc::smem_u32(slots + dr * K::SLOT), src, bytes, slot_full + 8 * dr);
                }
            }
        }
    } else if (warp >= 1 && warp < K::EPI0) {
        // ---------------- MMA warps: warp 1 + ms issues tiles c = ms, ms+2, ... ----------------
        // Two issuers keep the tensor pipe fed: while one waits on its next
        // tile's barriers (each a shared-memory round trip competing with
        // the operand traffic), the other's MMAs run.
        constexpr uint32_t kChunk16 = K::CHUNK / 16, kBChunk16 = K::BCHUNK / 16, kSlot16 = K::SLOT / 16;
        constexpr uint32_t kRows64 = C;  // rows 64.. of a slot chunk, in 16-byte units
        const uint64_t bdesc = tc::smem_desc(tc::smem_u32(slots), K::BCHUNK, 128);
        const uint64_t adescP = tc::smem_desc(tc::smem_u32(bufP) + K::HALO * 16, K::CHUNK, 128);
        const uint64_t adescQ = tc::smem_desc(tc::smem_u32(bufQ) + K::HALO * 16, K::CHUNK, 128);
        const uint32_t a_hi = (uint32_t)(adescP >> 32), b_lo = (uint32_t)bdesc, b_hi = (uint32_t)(bdesc >> 32);
        const bool leader = lane == 0;
        const int ms = warp - 1;
        int c = 0, u = 0, i = 0;
        ColsGroup grp;
        for (int gk = 0; cols_group(gk, cta, P, count, grp); ++gk, ++i) {
            const int T = grp.tiles;
            for (int l = 0; l < NL; ++l, ++u) {
                const uint32_t a_lo = (uint32_t)(l % 2 == 0 ? adescQ : adescP);
                const int ks = l == 0 ? 1 : C / 16;
                const int t_first = (ms - c) & 1;  // this warp's first tile of the layer (tiles alternate warps)
                for (int t = 0; t < T; ++t, ++c) {
                    if ((c & 1) != ms) continue;
                    const bool first_use = t == t_first;  // this warp's first tile of the layer waits for the weights
                    const bool last_use = t + 2 >= T;     // and its last one releases them
                    if (l == 0 && first_use && !warp_wait(input_ready, (uint32_t)i & 1u, status, leader))
                        goto mma_drain;
                    // Tile t reads the rows the previous layer's tiles t-1..t+1 wrote
                    // (tiles c-T-1, c-T, c-T+1), and tile c-4's epilogue frees this
                    // tile's accumulator. Each epilogue set finishes its tiles in order,
                    // so of c-T-1 and c-T+1 (the same set) the later one stands for
                    // both; the last tile has no tile below it and waits for c-T-1.
                    // The epilogue-done ring is NDONE deep: no tile waited for here can
                    // be overtaken NDONE tiles later before this tile is issued.
                    {
                        const int deps[3] = {c - 4, c - T, t == T - 1 ? c - T - 1 : c - T + 1};
#pragma unroll
                        for (int j = 0; j < 3; ++j) {
                            const int dep = deps[j];
                            if (dep >= 0 && !warp_wait(epi_done + 8 * (dep % K::NDONE),
                                                       (uint32_t)(dep / K::NDONE) & 1u, status, leader))
                                goto mma_drain;
                        }
                    }
                    const uint32_t d = tmem + (uint32_t)((c % K::NBUF) * K::NACC);
#pragma unroll
                    for (int dr = 0; dr < 3; ++dr) {
                        if (first_use && !warp_wait(slot_full + 8 * dr, (uint32_t)u & 1u, status, leader)) goto mma_drain;
                        const uint32_t a = a_lo + (uint32_t)(t * K::STRIDE + (dr - 1) * 10);
                        const uint32_t b = b_lo + (uint32_t)dr * kSlot16;
                        for (int s = 0; s < ks; ++s)  // dc = 0, +1 -> columns 0..127
                            tc::mma_bf16_warp(d, a + 2 * s * kChunk16, a_hi, b + kRows64 + 2 * s * kBChunk16, b_hi,
                                              K::IDESC128, (dr | s) != 0);
                        for (int s = 0; s < ks; ++s)  // dc = -1 -> columns 0..63
                            tc::mma_bf16_warp(d, a - 1 + 2 * s * kChunk16, a_hi, b + 2 * s * kBChunk16, b_hi,
                                              K::IDESC64, 1u);
                        if (last_use) tc::mma_commit_warp(slot_free + 8 * dr);
                    }
                    tc::mma_commit_warp(acc_full + 8 * (c % K::NBUF));
                }
            }
        }
    mma_drain:
        __syncwarp();
        tc::mma_commit_warp(mma_idle);
        if (leader) tc::mbar_wait(mma_idle, 0, status);
        __syncwarp();
    } else if (warp >= K::EPI0) {
        // ------- epilogue: set s takes tiles c = s, s+2, ...; warp -> (quadrant q, channel half h) -------
        const int e = warp - K::EPI0;
        const int s = e >> 3;
        const int q = warp & 3;
        const int h = (e & 7) >> 2;
        const int ch0 = 32 * h;
        const int etid = threadIdx.x - 32 * K::EPI0;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        // A wait of the whole set: its first warp polls the barrier (bounded)
        // and the set's named barrier releases the other seven with the
        // outcome, so they sleep instead of polling shared memory (which the
        // MMA operand reads saturate). Named barrier 1 + s belongs to set s,
        // 3 + s to its P1 exchange; a timeout ends all eight warps together.
        auto set_wait = [&](uint32_t bar, uint32_t parity) -> bool {
            int ok = 1;
            if ((e & 7) == 0 && lane == 0) ok = tc::mbar_wait(bar, parity, status) ? 1 : 0;
            __syncwarp();
            const bool all_ok = tc::named_barrier_and(1 + s, 256, ok != 0);
            tc::tc_fence_after();
            return all_ok;
        };
        int c = 0, i = 0;
        bool first = true;
        ColsGroup grp;
        for (int gk = 0; cols_group(gk, cta, P, count, grp); ++gk, ++i) {
            const int base_img = grp.base;
            const int nimg = grp.nimg;
            const int T = grp.tiles;
            if (first) {
                for (int m = etid; m < K::G * 100; m += 32 * K::EPI_WARPS) build_input_row<C>(bufQ, m, base_img, nimg, in);
                tc::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(input_ready);
                first = false;
            } else {
                // The previous group's head pass (all warps) must have read buffer P.
                if (!set_wait(heads_done, (uint32_t)(i - 1) & 1u)) goto epi_exit;
            }
            for (int l = 0; l < NL; ++l) {
                uint8_t* const out = l % 2 == 0 ? bufP : bufQ;
                const bool residual = l >= 2 && l % 2 == 0;
                const float* const bias = p.conv_b + l * C + ch0;
                for (int t = 0; t < T; ++t, ++c) {
                    if ((c & 1) != s) continue;
                    const int b = c % K::NBUF, k = c >> 1;  // k: this set's tile count
                    const int x = k % 3;
                    const int m = t * K::STRIDE + q * 32 + lane;
                    uint8_t* const row = out + (K::HALO + m) * 16 + (ch0 / 8) * K::CHUNK;
                    // Bias plus residual (the block input, which this warp wrote two
                    // layers ago and now overwrites in place) before the accumulator
                    // is ready. Row 127 belongs to the next tile and is not stored.
                    float pre[32];
                    // Eight 16-byte loads (bias + 32 h is 128-byte aligned), not 32 scalar ones:
                    // the L1 data pipe is the one the MMA operands and the stores use.
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 b4 = __ldg(reinterpret_cast<const float4*>(bias) + j);
                        pre[4 * j] = b4.x;
                        pre[4 * j + 1] = b4.y;
                        pre[4 * j + 2] = b4.z;
                        pre[4 * j + 3] = b4.w;
                    }
                    if (residual) {
#pragma unroll
                        for (int k2 = 0; k2 < 4; ++k2) {
                            const uint4 rv = *reinterpret_cast<const uint4*>(row + k2 * K::CHUNK);
                            const uint32_t w[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                            for (int j = 0; j < 8; ++j) pre[8 * k2 + j] += (j & 1) ? bf16_hi(w[j >> 1]) : bf16_lo(w[j >> 1]);
                        }
                    }
                    if (!set_wait(acc_full + 8 * b, (uint32_t)(c / K::NBUF) & 1u)) goto epi_exit;
                    const uint32_t taddr = tmem + lane_base + (uint32_t)(b * K::NACC + ch0);
                    float p1[32], p0[16];
                    tc::tmem_ld32_16(taddr + C, taddr, p1, p0);
                    if (q > 0 && lane == 0) {
                        // Publish lane 0's P1: the last row of the quadrant above needs it.
                        float4* const w = reinterpret_cast<float4*>(xp1 + (((s * 3 + x) * 4 + q) * 2 + h) * 32);
#pragma unroll
                        for (int j = 0; j < 8; ++j) w[j] = make_float4(p1[4 * j], p1[4 * j + 1], p1[4 * j + 2], p1[4 * j + 3]);
                    }
                    __syncwarp();
                    // y[m] = P0[m] + P1[m + 1]: P1 of the next row comes from the next lane.
#pragma unroll
                    for (int j = 0; j < 32; ++j) p1[j] = __shfl_down_sync(0xffffffffu, p1[j], 1);
#pragma unroll
                    for (int j = 0; j < 16; ++j) pre[j] += p0[j];
                    tc::tmem_ld16(taddr + 16, p0);
#pragma unroll
                    for (int j = 0; j < 16; ++j) pre[16 + j] += p0[j];
                    const int img = m / 100, pos = m - img * 100, r = pos / 10, cc = pos - r * 10;
                    const bool valid = img < nimg && r < 9 && cc < 9;
                    // Lane 31's next row is lane 0 of the quadrant below, published
                    // above; the wait comes after this warp's own TMEM reads so the
                    // other warps' publishing overlaps them. Quadrant 3's lane 31 is
                    // row 127, which belongs to the next tile and is not stored.
                    tc::named_barrier(3 + s, 256);
                    // Only lane 31 loads: a load every lane issues returns 512 bytes
                    // per 16-byte load through the shared-memory pipe.
                    if (q < 3 && lane == 31) {
                        const float4* const nb = reinterpret_cast<const float4*>(xp1 + (((s * 3 + x) * 4 + q + 1) * 2 + h) * 32);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float4 v = nb[j];
                            p1[4 * j] = v.x;
                            p1[4 * j + 1] = v.y;
                            p1[4 * j + 2] = v.z;
                            p1[4 * j + 3] = v.w;
                        }
                    }
                    if (m < K::G * 100 && !(q == 3 && lane == 31)) store_row32(row, pre, p1, valid);
                    tc::tc_fence_before();
                    tc::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(epi_done + 8 * (c % K::NDONE));
                }
            }
            // Build the next group's stem input (buffer Q) before the head pass,
            // so its MMAs can start, once the group's last MMAs (which read Q)
            // are complete: the last tile of each MMA warp.
            {
                ColsGroup next;
                if (cols_group(gk + 1, cta, P, count, next)) {
                    for (int cl = c - 2; cl < c; ++cl)  // the last tile of each MMA warp
                        if (!set_wait(acc_full + 8 * (cl % K::NBUF), (uint32_t)(cl / K::NBUF) & 1u)) goto epi_exit;
                    const int nb = next.base;
                    const int nn = next.nimg;
                    for (int mm = etid; mm < K::G * 100; mm += 32 * K::EPI_WARPS) build_input_row<C>(bufQ, mm, nb, nn, in);
                    tc::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(input_ready);
                }
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(heads_ready);
            if (!set_wait(heads_ready, (uint32_t)i & 1u)) goto epi_exit;
            for (int mm = etid; mm < K::G * 100; mm += 32 * K::EPI_WARPS) {
                const int img = mm / 100, pos = mm - img * 100, r = pos / 10, cc = pos - r * 10;
                if (!(img < nimg && r < 9 && cc < 9)) continue;
                const uint8_t* row = bufP + (K::HALO + mm) * 16;
                float h0 = headw[3 * C], h1 = headw[3 * C + 1], h2 = headw[3 * C + 2];
#pragma unroll 4
                for (int kk = 0; kk < C / 8; ++kk) {
                    const uint4 rv = *reinterpret_cast<const uint4*>(row + kk * K::CHUNK);
                    const uint32_t w[4] = {rv.x, rv.y, rv.z, rv.w};
                    // The 8 channels' weights of the three head rows as 16-byte broadcast loads.
                    float hw[3][8];
#pragma unroll
                    for (int o = 0; o < 3; ++o) {
                        const float4 lo = *reinterpret_cast<const float4*>(headw + o * C + kk * 8);
                        const float4 hi = *reinterpret_cast<const float4*>(headw + o * C + kk * 8 + 4);
                        hw[o][0] = lo.x, hw[o][1] = lo.y, hw[o][2] = lo.z, hw[o][3] = lo.w;
                        hw[o][4] = hi.x, hw[o][5] = hi.y, hw[o][6] = hi.z, hw[o][7] = hi.w;
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float xv = (j & 1) ? bf16_hi(w[j >> 1]) : bf16_lo(w[j >> 1]);
                        h0 = fmaf(xv, hw[0][j], h0);
                        h1 = fmaf(xv, hw[1][j], h1);
                        h2 = fmaf(xv, hw[2][j], h2);
                    }
                }
                float* hf = headfeat + (int64_t)(base_img + img) * 243 + r * 9 + cc;
                hf[0] = fmaxf(h0, 0.0f);
                hf[81] = fmaxf(h1, 0.0f);
                hf[162] = fmaxf(h2, 0.0f);
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(heads_done);
        }
    epi_exit:;
    }
done:
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

int launch_tower_cols(const NetParams& p, const NetInput& in, float* headfeat, uint32_t* status,
                      cudaStream_t stream) {
    using K = Cols64;
    static bool done[64] = {};
    if (!once_per_device(done, [] {
            return cudaFuncSetAttribute(net_tower_cols_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, K::SMEM) ==
                   cudaSuccess;
        }))
        return launch_status();
    // Every CTA of a tail round takes at least two images (cols_group).
    const int64_t half = (in.n + 1) / 2;
    const int grid = (int)(half < kSmCount ? half : kSmCount);
    net_tower_cols_kernel<<<grid < 1 ? 1 : grid, K::THREADS, K::SMEM, stream>>>(p, in, headfeat, status);
    return launch_status();
}

// ---- fully connected heads -------------------------------------------------------
struct HeadOut {
    float* logits;       // raw mode: [n][82]
    float* values;       // raw mode: [n]
    float* policy;       // search mode: [B][82] masked softmax, row index[i]
    float* leaf_value;   // search mode: [B]
    const gk_bits* states;  // search mode: leaf states for the legal mask
    const int32_t* leaf;    // search mode: [B] leaf node (0: the root, masked by root_allow too)
    const uint32_t* root_allow;  // search mode: [B][3] root candidates, or null (no root narrowing)
};

constexpr int kHeadWarps = 8;   // per block
constexpr int kHeadPos = 4;     // positions per warp: each weight read from shared memory feeds four
// Shared memory of the heads kernel for a value head of H hidden units:
// the feature-major FC weights as they lie in global memory, then per warp
// the features of its positions.
constexpr size_t head_smem(int H) {
    return (size_t)(162 * GK_ACTIONS + 81 * H + kHeadWarps * kHeadPos * 244) * sizeof(float);
}

// Copies N floats (N a multiple of 4, both addresses 16-byte aligned) into
// shared memory as 16-byte asynchronous copies: every copy of the block is
// in flight at once. The caller commits and waits (cp.async.wait_all).
template <int N>
__device__ __forceinline__ void stage_floats(float* dst, const float* src) {
    static_assert(N % 4 == 0, "16-byte copies");
    for (int i = 4 * threadIdx.x; i < N; i += 4 * blockDim.x)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(tc::smem_u32(dst + i)), "l"(src + i) : "memory");
}

// H = value-head hidden units: 64 for the batch-norm layout, C for the
// reference's GroupNorm network (python/kingdom_ai/model.py:58-66).
template <int H>
__global__ void __launch_bounds__(32 * kHeadWarps) net_heads_kernel(NetParams p, const float* headfeat, NetInput in,
                                                               HeadOut out) {
    constexpr int HU = H / 32;  // hidden units per lane
    extern __shared__ __align__(16) float hs[];
    float* wp = hs;                      // [162][82]
    float* w1 = wp + 162 * GK_ACTIONS;   // [81][H]
    float* feat_all = w1 + 81 * H;
    stage_floats<162 * GK_ACTIONS>(wp, p.pol_w);
    stage_floats<81 * H>(w1, p.val_w1);
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* feat = feat_all + warp * (kHeadPos * 244);
    const int count = input_count(in);
    // Lane l owns actions l, l+32, l+64 (the last only for l < 18) and hidden
    // units l + 32k (k < H/32) of the value head, for each of the warp's kHeadPos
    // positions. Every accumulation runs over the features in order, so each
    // position's sums are those of a one-position loop.
    const float* wa = wp + lane;       // weights of actions lane, lane+32, lane+64 at feature j: [j * 82 + a]
    const float* wb = wp + lane + 32;
    const float* wc = wp + (lane + 64 < GK_ACTIONS ? lane + 64 : GK_ACTIONS - 1);
    const bool gn = p.norm != 0;
    for (int img0 = (blockIdx.x * kHeadWarps + warp) * kHeadPos; img0 < count;
         img0 += gridDim.x * kHeadWarps * kHeadPos) {
#pragma unroll
        for (int u = 0; u < kHeadPos; ++u) {
            const int img = img0 + u;
            const float* hf = headfeat + (int64_t)img * 243;
            float fv[8];
#pragma unroll
            for (int v = 0; v < 8; ++v) fv[v] = img < count && lane + 32 * v < 243 ? __ldg(hf + lane + 32 * v) : 0.f;
            if (gn) {
                // GroupNorm(1, 2) over the 162 policy features and
                // GroupNorm(1, 1) over the 81 value features, then ReLU
                // (python/kingdom_ai/model.py:51-63; eps 1e-5).
                float sp = 0.f, sv = 0.f;
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    const int idx = lane + 32 * v;
                    if (idx < 162) sp += fv[v];
                    else if (idx < 243) sv += fv[v];
                }
#pragma unroll
                for (int off = 16; off; off >>= 1) {
                    sp += __shfl_xor_sync(0xffffffffu, sp, off);
                    sv += __shfl_xor_sync(0xffffffffu, sv, off);
                }
                const float mp = sp / 162.f, mv = sv / 81.f;
                float qp = 0.f, qv = 0.f;
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    const int idx = lane + 32 * v;
                    if (idx < 162) qp += (fv[v] - mp) * (fv[v] - mp);
                    else if (idx < 243) qv += (fv[v] - mv) * (fv[v] - mv);
                }
#pragma unroll
                for (int off = 16; off; off >>= 1) {
                    qp += __shfl_xor_sync(0xffffffffu, qp, off);
                    qv += __shfl_xor_sync(0xffffffffu, qv, off);
                }
                const float rp = 1.0f / sqrtf(qp / 162.f + 1e-5f), rv = 1.0f / sqrtf(qv / 81.f + 1e-5f);
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    const int idx = lane + 32 * v;
                    if (idx >= 243) continue;
                    const int ch = idx < 81 ? 0 : idx < 162 ? 1 : 2;
                    const float w = __ldg(p.head_norm + (ch < 2 ? ch : 4)), b = __ldg(p.head_norm + (ch < 2 ? 2 + ch : 5));
                    const float mean = ch < 2 ? mp : mv, rstd = ch < 2 ? rp : rv;
                    const float a = rstd * w;
                    fv[v] = fmaxf(a * fv[v] + (b - a * mean), 0.f);
                }
            }
#pragma unroll
            for (int v = 0; v < 8; ++v)
                if (lane + 32 * v < 243) feat[u * 244 + lane + 32 * v] = fv[v];
        }
        __syncwarp();
        float la[kHeadPos], lb[kHeadPos], lc[kHeadPos];
#pragma unroll
        for (int u = 0; u < kHeadPos; ++u) la[u] = lb[u] = lc[u] = 0.f;
#pragma unroll 9
        for (int j = 0; j < 162; ++j) {
            const float xa = wa[j * GK_ACTIONS], xb = wb[j * GK_ACTIONS], xc = wc[j * GK_ACTIONS];
#pragma unroll
            for (int u = 0; u < kHeadPos; ++u) {
                const float f = feat[u * 244 + j];
                la[u] = fmaf(xa, f, la[u]);
                lb[u] = fmaf(xb, f, lb[u]);
                lc[u] = fmaf(xc, f, lc[u]);
            }
        }
        float hv[HU][kHeadPos];
#pragma unroll
        for (int k = 0; k < HU; ++k) {
            const float b = __ldg(p.val_b1 + lane + 32 * k);
#pragma unroll
            for (int u = 0; u < kHeadPos; ++u) hv[k][u] = b;
        }
#pragma unroll 9
        for (int j = 0; j < 81; ++j) {
            float x[HU];
#pragma unroll
            for (int k = 0; k < HU; ++k) x[k] = w1[j * H + lane + 32 * k];
#pragma unroll
            for (int u = 0; u < kHeadPos; ++u) {
                const float f = feat[u * 244 + 162 + j];
#pragma unroll
                for (int k = 0; k < HU; ++k) hv[k][u] = fmaf(x[k], f, hv[k][u]);
            }
        }
        const float pa = __ldg(p.pol_b + lane), pb = __ldg(p.pol_b + lane + 32);
        const float pc = lane + 64 < GK_ACTIONS ? __ldg(p.pol_b + lane + 64) : 0.f;
        float w2[HU];
#pragma unroll
        for (int k = 0; k < HU; ++k) w2[k] = __ldg(p.val_w2 + lane + 32 * k);
        const float b2 = __ldg(p.val_b2);
#pragma unroll
        for (int u = 0; u < kHeadPos; ++u) {
            const int img = img0 + u;
            if (img >= count) break;  // warp-uniform
            float logit[3];
            logit[0] = la[u] + pa;
            logit[1] = lb[u] + pb;
            logit[2] = lane + 64 < GK_ACTIONS ? lc[u] + pc : 0.f;
            float vpart = 0.f;
#pragma unroll
            for (int k = 0; k < HU; ++k) vpart = fmaf(fmaxf(hv[k][u], 0.f), w2[k], vpart);
#pragma unroll
            for (int off = 16; off; off >>= 1) vpart += __shfl_xor_sync(0xffffffffu, vpart, off);
            const float value = tanhf(vpart + b2);
            if (out.logits) {
#pragma unroll
                for (int k = 0; k < 3; ++k)
                    if (lane + 32 * k < GK_ACTIONS) out.logits[(int64_t)img * GK_ACTIONS + lane + 32 * k] = logit[k];
                if (lane == 0) out.values[img] = value;
            } else {
                // Masked softmax over the leaf's legal actions (gpu_puct.py:500-501).
                const int tree = in.index ? in.index[img] : img;
                const gk_bits s = out.states[tree];
                const gk_b96 placements = legal_placements(s);
                bool legal[3];
                float mx = -INFINITY;
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    const int a = lane + 32 * k;
                    legal[k] = a < GK_ACTIONS && (a == GK_PASS ? true : gk_test(placements, a + a / 9) != 0) &&
                               (out.root_allow == nullptr || out.leaf[tree] != 0 ||
                                ((out.root_allow[tree * 3 + k] >> lane) & 1u) != 0u);
                    if (legal[k]) mx = fmaxf(mx, logit[k]);
                }
#pragma unroll
                for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                float e[3], sum = 0.f;
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    e[k] = legal[k] ? __expf(logit[k] - mx) : 0.f;
                    sum += e[k];
                }
#pragma unroll
                for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
#pragma unroll
                for (int k = 0; k < 3; ++k)
                    if (lane + 32 * k < GK_ACTIONS) out.policy[(int64_t)tree * GK_ACTIONS + lane + 32 * k] = e[k] / sum;
                if (lane == 0) out.leaf_value[tree] = value;
            }
        }
        __syncwarp();
    }
}

// ---- tensor-core self-test ---------------------------------------------------------
// One 128x64x16 bf16 MMA from operands staged in the same K-major no-swizzle
// layout the tower uses (A: chunk stride 2048 B, B: chunk stride 1024 B, 8-row
// groups 128 B apart). The operands sit in a 64 KB buffer sized so that every
// address stays inside it even if the two descriptor strides were read the
// other way round; the result is compared on the host.
constexpr int kSelfTestSmem = 65536;

__global__ void __launch_bounds__(128, 1)
    mma_selftest_kernel(const uint16_t* a, const uint16_t* b, float* d, uint32_t* status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_holder;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kSelfTestSmem / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    // A[m][k] (128 x 16) -> chunk (k/8) at 2048*(k/8) + 16*m; B[n][k] (64 x 16) at 32768 + 1024*(k/8) + 16*n.
    for (int i = threadIdx.x; i < 128 * 16; i += blockDim.x) {
        const int m = i / 16, k = i % 16;
        reinterpret_cast<uint16_t*>(smem + 2048 * (k / 8) + 16 * m)[k % 8] = a[i];
    }
    for (int i = threadIdx.x; i < 64 * 16; i += blockDim.x) {
        const int n = i / 16, k = i % 16;
        reinterpret_cast<uint16_t*>(smem + 32768 + 1024 * (k / 8) + 16 * n)[k % 8] = b[i];
    }
    tc::fence_proxy_async_smem();
    const uint32_t barp = tc::smem_u32(&bar);
    if (threadIdx.x == 0) {
        tc::mbar_init(barp, 1);
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tc::smem_u32(&tmem_holder), 512);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = tmem_holder;
    if (threadIdx.x == 0) {
        const uint32_t base = tc::smem_u32(smem);
        tc::mma_bf16(tmem, tc::smem_desc(base, 2048, 128), tc::smem_desc(base + 32768, 1024, 128),
                     tc::idesc_bf16(128, 64), 0);
        tc::mma_commit(barp);
    }
    __syncwarp();
    const bool ok = tc::mbar_wait(barp, 0, status);
    tc::tc_fence_after();
    if (ok) {
#pragma unroll 1
        for (int cb = 0; cb < 2; ++cb) {
            float v[32];
            tc::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + cb * 32, v);
            const int m = warp * 32 + lane;
            for (int j = 0; j < 32; ++j) d[m * 64 + cb * 32 + j] = v[j];
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

inline NetParams make_params(const gk_net_t* net) {
    NetParams p;
    p.channels = net->channels;
    p.blocks = net->blocks;
    p.conv_w = static_cast<const uint8_t*>(net->conv_w);
    p.conv_b = net->conv_b;
    p.head_w = net->head_w;
    p.head_b = net->head_b;
    p.pol_w = net->pol_w;
    p.pol_b = net->pol_b;
    p.val_w1 = net->val_w1;
    p.val_b1 = net->val_b1;
    p.val_w2 = net->val_w2;
    p.val_b2 = net->val_b2;
    p.norm = net->norm;
    p.norm_w = net->norm_w;
    p.norm_b = net->norm_b;
    p.head_norm = net->head_norm;
    return p;
}

template <int C, bool GN>
int launch_tower(const NetParams& p, const NetInput& in, float* headfeat, uint32_t* status, cudaStream_t stream) {
    using K = NetCfg<C>;
    static bool done[64] = {};
    if (!once_per_device(done, [] {
            return cudaFuncSetAttribute(net_tower_kernel<C, GN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        K::SMEM) == cudaSuccess;
        }))
        return launch_status();
    const int64_t groups = (in.n + K::G - 1) / K::G;
    const int64_t slots = (int64_t)kSmCount * K::MIN_BLOCKS;
    const int grid = (int)(groups < slots ? groups : slots);
    net_tower_kernel<C, GN><<<grid < 1 ? 1 : grid, K::THREADS, K::SMEM, stream>>>(p, in, headfeat, status);
    return launch_status();
}

template <int H>
int launch_heads_h(const NetParams& p, const float* headfeat, const NetInput& in, const HeadOut& out,
                   cudaStream_t stream) {
    static bool done[64] = {};
    if (!once_per_device(done, [] {
            return cudaFuncSetAttribute(net_heads_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)head_smem(H)) == cudaSuccess;
        }))
        return launch_status();
    int64_t blocks = (in.n + kHeadWarps * kHeadPos - 1) / (kHeadWarps * kHeadPos);
    if (blocks > 2 * kSmCount) blocks = 2 * kSmCount;
    net_heads_kernel<H><<<(int)(blocks < 1 ? 1 : blocks), 32 * kHeadWarps, head_smem(H), stream>>>(p, headfeat, in,
                                                                                                   out);
    return launch_status();
}

int launch_heads(const NetParams& p, const float* headfeat, const NetInput& in, const HeadOut& out,
                 cudaStream_t stream) {
    const int hidden = p.norm ? p.channels : 64;
    return hidden == 32    ? launch_heads_h<32>(p, headfeat, in, out, stream)
           : hidden == 128 ? launch_heads_h<128>(p, headfeat, in, out, stream)
                           : launch_heads_h<64>(p, headfeat, in, out, stream);
}

inline bool valid_net(const gk_net_t* net) {
    if (!net || (net->channels != 32 && net->channels != 64 && net->channels != 128) || net->blocks < 0 ||
        net->blocks > 64 || !net->conv_w || !net->head_w || !net->pol_w || !net->pol_b || !net->val_w1 ||
        !net->val_b1 || !net->val_w2 || !net->val_b2 || !aligned16(net->conv_w) || !aligned16(net->pol_w) ||
        !aligned16(net->val_w1))  // 16-byte copies and loads
        return false;
    if (net->norm == 0) return net->conv_b && aligned16(net->conv_b) && net->head_b;
    return net->norm == 1 && net->norm_w && net->norm_b && net->head_norm;
}

// Records `e` on `stream`; inside a stream capture as an external event node,
// so that replays of the graph record it (and its times can be read).
inline void record_event(cudaEvent_t e, cudaStream_t stream) {
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &capturing) == cudaSuccess && capturing == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(e, stream, cudaEventRecordExternal);
    else
        cudaEventRecord(e, stream);
}

int run_forward(const gk_net_t* net, const NetInput& in, float* headfeat, const HeadOut& out, uint32_t* status,
                cudaStream_t stream, cudaEvent_t tower_start = nullptr, cudaEvent_t tower_stop = nullptr) {
    const NetParams p = make_params(net);
    if (tower_start) record_event(tower_start, stream);
    // The column-fused kernel serves the 64-channel batch-norm layout; GroupNorm
    // needs whole-image statistics between layers, which the templated tower
    // gathers (its conv_w is per tap for every width).
    int s;
    if (net->norm == 0) {
        s = net->channels == 64   ? launch_tower_cols(p, in, headfeat, status, stream)
            : net->channels == 32 ? launch_tower<32, false>(p, in, headfeat, status, stream)
                                  : launch_tower<128, false>(p, in, headfeat, status, stream);
    } else {
        s = net->channels == 32   ? launch_tower<32, true>(p, in, headfeat, status, stream)
            : net->channels == 64 ? launch_tower<64, true>(p, in, headfeat, status, stream)
                                  : launch_tower<128, true>(p, in, headfeat, status, stream);
    }
    if (tower_stop) record_event(tower_stop, stream);
    if (s) return s;
    return launch_heads(p, headfeat, in, out, stream);
}

int net_evaluate(const gk_net_t* net, void* ws, int64_t batch, int capacity, float* headfeat, uint32_t* status,
                 cudaStream_t stream, cudaEvent_t tower_start, cudaEvent_t tower_stop) {
    if (!valid_net(net) || ws == nullptr || batch <= 0 || capacity < 1 || headfeat == nullptr || status == nullptr)
        return GK_EINVAL;
    int s = gk_puct_compact(ws, batch, capacity, stream);
    if (s) return s;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    NetInput in{v.leaf_bits, nullptr, v.active, v.active_count, batch};
    HeadOut out{nullptr, nullptr, v.policy, v.leaf_value, v.leaf_bits, v.leaf, v.root_allow};
    return run_forward(net, in, headfeat, out, status, stream, tower_start, tower_stop);
}

}  // namespace gk

using namespace gk;

extern "C" {

size_t gk_net_weight_bytes(int channels, int blocks) {
    if ((channels != 32 && channels != 64 && channels != 128) || blocks < 0) return 0;
    return (size_t)9 * 16 * channels * 2 + (size_t)blocks * 2 * 9 * channels * channels * 2;
}

size_t gk_net_headfeat_bytes(int64_t n) { return n <= 0 ? 0 : (size_t)n * 243 * sizeof(float); }

int gk_mma_selftest(const uint16_t* a, const uint16_t* b, float* d, uint32_t* status, void* stream) {
    if (a == nullptr || b == nullptr || d == nullptr || status == nullptr) return GK_EINVAL;
    static bool done[64] = {};
    if (!once_per_device(done, [] {
            return cudaFuncSetAttribute(mma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kSelfTestSmem) == cudaSuccess;
        }))
        return launch_status();
    mma_selftest_kernel<<<1, 128, kSelfTestSmem, as_stream(stream)>>>(a, b, d, status);
    return launch_status();
}

int gk_net_forward(const gk_net_t* net, const uint32_t* states, const float* features, int64_t n, float* headfeat,
                   float* logits, float* values, uint32_t* status, void* stream) {
    if (!valid_net(net) || n < 0 || headfeat == nullptr || logits == nullptr || values == nullptr ||
        status == nullptr || (states == nullptr) == (features == nullptr))
        return GK_EINVAL;
    if (n == 0) return 0;
    NetInput in{reinterpret_cast<const gk_bits*>(states), features, nullptr, nullptr, n};
    HeadOut out{logits, values, nullptr, nullptr, nullptr, nullptr, nullptr};
    return run_forward(net, in, headfeat, out, status, as_stream(stream));
}

int gk_net_evaluate_puct(const gk_net_t* net, void* ws, int64_t batch, int capacity, float* headfeat,
                         uint32_t* status, void* stream) {
    return net_evaluate(net, ws, batch, capacity, headfeat, status, as_stream(stream), nullptr, nullptr);
}

int gk_net_evaluate_states(const gk_net_t* net, const uint32_t* states, const int32_t* active,
                           const int32_t* active_count, int64_t n, float* policy, float* value, float* headfeat,
                           uint32_t* status, void* stream) {
    if (!valid_net(net) || states == nullptr || active == nullptr || active_count == nullptr || n <= 0 ||
        policy == nullptr || value == nullptr || headfeat == nullptr || status == nullptr)
        return GK_EINVAL;
    const gk_bits* bits = reinterpret_cast<const gk_bits*>(states);
    NetInput in{bits, nullptr, active, active_count, n};
    HeadOut out{nullptr, nullptr, policy, value, bits, nullptr, nullptr};
    return run_forward(net, in, headfeat, out, status, as_stream(stream));
}

}  // extern "C"
