// gk_bpuct.cu - BatchedPUCT on the GPU: leaf batches under virtual loss and
// subtree reuse, for many independent searchers at once.
//
// Reference: kingdom::BatchedPUCT (mcts/src/BatchedPUCT.cpp, declared in
// mcts/include/BatchedPUCT.h:38-60), the evaluation searcher of
// python/kingdom_ai/evaluation.py:174-231. One workspace holds T trees (one per
// game and model); each search runs in waves, and a wave collects up to L
// pending leaves per tree, evaluates all of them in one batch and backs them up
// in collection order:
//
//   select           BatchedPUCT.cpp:143-196  (virtual loss of one per pending
//                    simulation; a subtree holding only pending leaves is
//                    skipped for the next-scored edge)
//   reserve/release  BatchedPUCT.cpp:198-216
//   backup           BatchedPUCT.cpp:218-227
//   expand           BatchedPUCT.cpp:72-81 (checks), 229-250 (priors)
//   search loop      BatchedPUCT.cpp:328-442
//   advance          BatchedPUCT.cpp:290-326
//
// One warp owns one tree in every kernel; lanes cover the 82 edges of a node
// (three each) or the steps of a path. The reference walks the tree depth
// first and backtracks out of subtrees whose every path ends in a pending leaf.
// Here such nodes carry a "blocked" flag, kept exact as leaves are reserved
// (a node is blocked when it is pending, or expanded with every legal edge
// leading to a blocked child) and cleared when the wave's leaves are released,
// so selection is one greedy descent over unblocked children: the same leaf
// the backtracking walk reaches, with the same nodes created.
//
// Double arithmetic follows the reference operation by operation through
// GK_DADD/GK_DMUL (no FMA contraction); sums over actions run in action order.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/gk.h"
#include "gk_device.cuh"
#include "gk_launch.cuh"
#include "gk_puct.cuh"

namespace gk {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kWarps = 4;  // warps (trees) per block

enum : uint8_t { kExpanded = 1, kPending = 2, kBlocked = 4 };
enum : int32_t { kIdle = 0, kSearching = 1, kTerminalRoot = 2 };
enum { kStEvals, kStBatches, kStMaxBatch, kStReused, kStInherited, kStAdvances, kStReuseHits, kStats };

// Device workspace for T trees of C nodes and L leaf slots each. Node arrays
// are [T][C], edge arrays [T][C][82] indexed by action, slot arrays [T][L].
struct BpuctView {
    gk_bits* node_state;
    int32_t* node_visits;
    int32_t* node_reserved;
    uint8_t* node_flags;
    double* prior;
    double* wsum;
    int32_t* visits;
    int32_t* reserved;
    int32_t* child;
    // per tree
    int32_t* count;        // nodes held (0 = empty tree)
    int32_t* mode;         // kIdle / kSearching / kTerminalRoot for the current search
    int32_t* budget;       // simulations of the current search
    int32_t* sims;         // simulations completed in the current search
    int32_t* pending;      // leaves collected by the current wave
    int32_t* stats;        // [T][kStats]
    uint32_t* errors;      // GK_ERR_* of the current search
    double* root_terminal; // terminal root value (kTerminalRoot)
    int32_t* init_visits;  // [T][82] root edge visits when the search began
    double* init_wsum;     // [T][82]
    // slots
    int32_t* slot_node;
    int32_t* slot_len;
    int32_t* slot_path;    // [T*L][P] parent nodes
    uint8_t* slot_act;     // [T*L][P] actions
    gk_bits* slot_bits;
    uint8_t* slot_needs;
    double* slot_policy;   // [T*L][82] evaluator weights
    double* slot_value;
    float* slot_policy_f;  // [T*L][82] native network output
    float* slot_value_f;
    int32_t* active;       // compacted slot indices
    int32_t* active_count;
    int32_t* remaining;    // max over trees of budget - sims after a wave
    int32_t* remap;        // [T][C] advance scratch
};

size_t bpuct_layout(void* base, int64_t T, int C, int L, BpuctView* out) {
    const int64_t N = T * (int64_t)C, E = N * GK_ACTIONS, S = T * (int64_t)L, P = path_cap(C);
    size_t off = 0;
    char* b = static_cast<char*>(base);
    auto take = [&](size_t bytes) -> void* {
        void* p = b ? b + off : nullptr;
        off = align256(off + bytes);
        return p;
    };
    BpuctView v;
    v.node_state = (gk_bits*)take(N * sizeof(gk_bits));
    v.node_visits = (int32_t*)take(N * 4);
    v.node_reserved = (int32_t*)take(N * 4);
    v.node_flags = (uint8_t*)take(N);
    v.prior = (double*)take(E * 8);
    v.wsum = (double*)take(E * 8);
    v.visits = (int32_t*)take(E * 4);
    v.reserved = (int32_t*)take(E * 4);
    v.child = (int32_t*)take(E * 4);
    v.count = (int32_t*)take(T * 4);
    v.mode = (int32_t*)take(T * 4);
    v.budget = (int32_t*)take(T * 4);
    v.sims = (int32_t*)take(T * 4);
    v.pending = (int32_t*)take(T * 4);
    v.stats = (int32_t*)take(T * kStats * 4);
    v.errors = (uint32_t*)take(T * 4);
    v.root_terminal = (double*)take(T * 8);
    v.init_visits = (int32_t*)take(T * GK_ACTIONS * 4);
    v.init_wsum = (double*)take(T * GK_ACTIONS * 8);
    v.slot_node = (int32_t*)take(S * 4);
    v.slot_len = (int32_t*)take(S * 4);
    v.slot_path = (int32_t*)take(S * P * 4);
    v.slot_act = (uint8_t*)take(S * P);
    v.slot_bits = (gk_bits*)take(S * sizeof(gk_bits));
    v.slot_needs = (uint8_t*)take(S);
    v.slot_policy = (double*)take(S * GK_ACTIONS * 8);
    v.slot_value = (double*)take(S * 8);
    v.slot_policy_f = (float*)take(S * GK_ACTIONS * 4);
    v.slot_value_f = (float*)take(S * 4);
    v.active = (int32_t*)take(S * 4);
    v.active_count = (int32_t*)take(4);
    v.remaining = (int32_t*)take(4);
    v.remap = (int32_t*)take(N * 4);
    if (out) *out = v;
    return off;
}

// ---- small helpers -------------------------------------------------------------
__device__ __forceinline__ bool legal_at(const gk_b96& placements, const gk_bits& s, int a) {
    if (gk_reason(&s) != GK_NONE) return false;
    return a == GK_PASS ? true : gk_test(placements, a + a / 9) != 0;
}

__device__ __forceinline__ double terminal_value(const gk_bits& s) {
    return gk_winner(&s) == gk_actor(&s) ? 1.0 : -1.0;
}

// BatchedPUCT.cpp:52-67: the position, its history counters and its result;
// the settled-territory flag is a cache and is ignored.
__device__ __forceinline__ bool same_state(const gk_bits& a, const gk_bits& b) {
    bool eq = true;
#pragma unroll
    for (int i = 0; i < 15; ++i) eq &= a.w[i] == b.w[i];
    return eq && ((a.w[15] ^ b.w[15]) & (GK_META_SETTLED - 1u)) == 0u;
}

// Sum in action order of v[k] (action lane + 32k) over the actions with use[k].
// The values pass through the warp's slice of a block-wide scratch (every
// tree kernel runs kWarps warps per block), unselected ones as +0.0: the
// callers' values are >= +0 or differences of sums that start at +0, so the
// running total is never -0 and adding +0.0 equals skipping the action.
__device__ __forceinline__ double ordered_sum(const double (&v)[3], const bool (&use)[3]) {
    __shared__ double scratch[kWarps][96];
    const int lane = threadIdx.x & 31;
    double* const sc = scratch[threadIdx.x >> 5];
#pragma unroll
    for (int k = 0; k < 3; ++k)
        if (lane + 32 * k < GK_ACTIONS) sc[lane + 32 * k] = use[k] ? v[k] : 0.0;
    __syncwarp();
    double total = 0.0;
#pragma unroll 8
    for (int a = 0; a < GK_ACTIONS; ++a) total = GK_DADD(total, sc[a]);
    __syncwarp();  // every lane has read the scratch before it is written again
    return total;
}

// ---- begin ---------------------------------------------------------------------
// BatchedPUCT.cpp:339-367: drop a tree that does not continue from this root,
// handle a finished root, create or keep the root, and queue the root for
// evaluation when it is not expanded yet.
__device__ void begin_tree(const BpuctView& v, int64_t t, int C, int L, const gk_bits* roots, const uint8_t* mask,
                           int simulations, int reuse, int lane) {
    const int64_t tb = t * C;
    if (mask && !mask[t]) {
        if (lane == 0) {
            v.mode[t] = kIdle;
            v.pending[t] = 0;
        }
        for (int i = lane; i < L; i += 32) v.slot_needs[t * L + i] = 0;
        return;
    }
    int pend = 0;
    if (lane == 0) {
        const gk_bits r = roots[t];
        int count = v.count[t];
        int32_t* st = v.stats + t * kStats;
        st[kStEvals] = st[kStBatches] = st[kStMaxBatch] = st[kStReused] = st[kStInherited] = 0;
        v.errors[t] = 0u;
        v.sims[t] = 0;
        v.budget[t] = simulations;
        if (!reuse || (count > 0 && !same_state(v.node_state[tb], r))) count = 0;
        if (gk_reason(&r) != GK_NONE) {
            count = 0;
            v.mode[t] = kTerminalRoot;
            v.root_terminal[t] = terminal_value(r);
        } else {
            v.mode[t] = kSearching;
            if (count == 0) {
                v.node_state[tb] = r;
                v.node_visits[tb] = 0;
                v.node_reserved[tb] = 0;
                v.node_flags[tb] = 0;
                count = 1;
            } else {
                st[kStReused] = count;
                st[kStInherited] = v.node_visits[tb];
            }
            if (!(v.node_flags[tb] & kExpanded)) {
                const int64_t s = t * L;
                v.slot_node[s] = 0;
                v.slot_len[s] = 0;
                v.slot_bits[s] = v.node_state[tb];
                pend = 1;
            }
        }
        v.count[t] = count;
        v.pending[t] = pend;
    }
    pend = __shfl_sync(kFull, pend, 0);
    for (int i = lane; i < L; i += 32) v.slot_needs[t * L + i] = i < pend ? 1 : 0;
}

// ---- expansion -----------------------------------------------------------------
// Expands node `leaf` from slot s's evaluation (BatchedPUCT.cpp:72-81, 229-250).
// Returns false when the evaluation is rejected, with the reference's first
// failing check as the tree's error: the value (GK_ERR_BAD_EVAL), a weight
// (GK_BPUCT_ERR_POLICY), or no positive weight on a legal action
// (GK_BPUCT_ERR_NO_WEIGHT).
__device__ bool expand_slot(const BpuctView& v, int64_t t, int C, int64_t s, int leaf, bool float_eval, int lane,
                            double& value) {
    const int64_t vtx = t * C + leaf, eb = vtx * GK_ACTIONS, row = s * GK_ACTIONS;
    const gk_bits st = v.node_state[vtx];
    const gk_b96 placements = legal_placements(st);
    value = float_eval ? (double)v.slot_value_f[s] : v.slot_value[s];
    const bool bad_value = !(isfinite(value) && value >= -1.0 && value <= 1.0);
    bool bad = false;
    double w[3];
    bool use[3];
    double largest = 0.0;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int a = lane + 32 * k;
        w[k] = 0.0;
        use[k] = false;
        if (a >= GK_ACTIONS) continue;
        w[k] = float_eval ? (double)v.slot_policy_f[row + a] : v.slot_policy[row + a];
        bad |= !(isfinite(w[k]) && w[k] >= 0.0);
        use[k] = legal_at(placements, st, a);
        if (use[k]) largest = fmax(largest, w[k]);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) largest = fmax(largest, __shfl_xor_sync(kFull, largest, off));
    bad = __any_sync(kFull, bad);
    if (bad_value || bad || !(largest > 0.0)) {
        if (lane == 0)
            v.errors[t] |= bad_value ? GK_ERR_BAD_EVAL : bad ? GK_BPUCT_ERR_POLICY : GK_BPUCT_ERR_NO_WEIGHT;
        return false;
    }
    double scaled[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) scaled[k] = use[k] ? w[k] / largest : 0.0;
    const double total = ordered_sum(scaled, use);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int a = lane + 32 * k;
        if (a >= GK_ACTIONS) continue;
        v.prior[eb + a] = use[k] ? scaled[k] / total : 0.0;
        v.wsum[eb + a] = 0.0;
        v.visits[eb + a] = 0;
        v.reserved[eb + a] = 0;
        v.child[eb + a] = -1;
    }
    if (lane == 0) v.node_flags[vtx] = kExpanded;
    return true;
}

// Root expansion of a search that starts from an unexpanded root (its own
// batch of one, BatchedPUCT.cpp:361-365), then the snapshot of the root edges
// that results are measured against (368-375).
__device__ void root_expand_tree(const BpuctView& v, int64_t t, int C, int L, bool float_eval, int lane) {
    if (v.mode[t] != kSearching) return;
    const int64_t tb = t * C;
    if (v.pending[t] > 0) {
        double value;
        const bool ok = expand_slot(v, t, C, t * L, 0, float_eval, lane, value);
        if (lane == 0) {
            v.pending[t] = 0;
            v.slot_needs[t * L] = 0;
            if (ok) {
                int32_t* st = v.stats + t * kStats;
                st[kStEvals] += 1;
                st[kStBatches] += 1;
                if (st[kStMaxBatch] < 1) st[kStMaxBatch] = 1;
            }
        }
        __syncwarp();
        if (!ok) return;
    }
    for (int a = lane; a < GK_ACTIONS; a += 32) {
        v.init_visits[t * GK_ACTIONS + a] = v.visits[tb * GK_ACTIONS + a];
        v.init_wsum[t * GK_ACTIONS + a] = v.wsum[tb * GK_ACTIONS + a];
    }
}

// ---- selection -----------------------------------------------------------------
// One greedy descent from the root over unblocked children, creating the
// chosen child when it is missing (BatchedPUCT.cpp:143-196). The path goes to
// `path`/`acts`. Returns the leaf node, -1 when the root is blocked, or -2 on
// a capacity or consistency failure (error bit set).
__device__ int select_leaf(const BpuctView& v, int64_t t, int C, double c_puct, int lane, int32_t* path,
                           uint8_t* acts, int& depth, gk_bits& leaf_state) {
    const int64_t tb = t * C;
    const int P = path_cap(C);
    int node = 0;
    depth = 0;
    uint8_t flags = v.node_flags[tb];
    if (flags & kBlocked) return -1;
    gk_bits st = v.node_state[tb];
    for (;;) {
        if (gk_reason(&st) != GK_NONE || !(flags & kExpanded)) {
            leaf_state = st;
            return node;
        }
        const int64_t vtx = tb + node, eb = vtx * GK_ACTIONS;
        const double scale = sqrt(GK_DADD((double)v.node_visits[vtx], (double)v.node_reserved[vtx]));
        const gk_b96 placements = legal_placements(st);
        int best = -1, best_child = -1;
        double best_score = 0.0, best_prior = 0.0;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int a = lane + 32 * k;
            if (a >= GK_ACTIONS || !legal_at(placements, st, a)) continue;
            const int n = v.visits[eb + a], r = v.reserved[eb + a], ch = v.child[eb + a];
            // Only a reserved edge can lead to a blocked child.
            if (r > 0 && ch >= 0 && (v.node_flags[tb + ch] & kBlocked)) continue;
            const double p = v.prior[eb + a];
            const double eff = GK_DADD((double)n, (double)r);
            const double q = eff == 0.0 ? 0.0 : GK_DSUB(v.wsum[eb + a], (double)r) / eff;
            const double u = GK_DMUL(p, scale) / GK_DADD(1.0, eff);
            const double score = c_puct >= 1.0 ? GK_DADD(q / c_puct, u) : GK_DADD(q, GK_DMUL(c_puct, u));
            if (best < 0 || score > best_score || (score == best_score && p > best_prior)) {
                best = a;
                best_child = ch;
                best_score = score;
                best_prior = p;
            }
        }
        // Warp argmax (higher score, then higher prior, then lower action).
        // Each lane's candidate is already the best of its own edges in that
        // order, so a single lane holding the highest score has the answer;
        // ties (and no candidate) take the full reduction.
        int ch;
        {
            double top = best >= 0 ? best_score : -INFINITY;
#pragma unroll
            for (int off = 16; off; off >>= 1) top = fmax(top, __shfl_xor_sync(kFull, top, off));
            const unsigned holders = __ballot_sync(kFull, best >= 0 && best_score == top);
            if (__popc(holders) == 1) {
                const int src = __ffs(holders) - 1;
                best = __shfl_sync(kFull, best, src);
                ch = __shfl_sync(kFull, best_child, src);
            } else {
#pragma unroll
                for (int off = 16; off; off >>= 1) {
                    const double os = __shfl_down_sync(kFull, best_score, off);
                    const double op = __shfl_down_sync(kFull, best_prior, off);
                    const int oa = __shfl_down_sync(kFull, best, off);
                    const int oc = __shfl_down_sync(kFull, best_child, off);
                    if (oa >= 0 && (best < 0 || os > best_score ||
                                    (os == best_score && (op > best_prior || (op == best_prior && oa < best))))) {
                        best = oa;
                        best_child = oc;
                        best_score = os;
                        best_prior = op;
                    }
                }
                best = __shfl_sync(kFull, best, 0);
                ch = __shfl_sync(kFull, best_child, 0);
            }
        }
        if (best < 0 || depth >= P) {
            if (lane == 0) v.errors[t] |= GK_ERR_CAPACITY;
            return -2;
        }
        if (ch < 0) {
            gk_bits next = st;
            const bool ok = play(next, best);
            if (lane == 0) ch = v.count[t];
            ch = __shfl_sync(kFull, ch, 0);
            if (!ok || ch >= C) {
                if (lane == 0) v.errors[t] |= GK_ERR_CAPACITY;
                return -2;
            }
            if (lane == 0) {
                v.count[t] = ch + 1;
                v.node_state[tb + ch] = next;
                v.node_visits[tb + ch] = 0;
                v.node_reserved[tb + ch] = 0;
                v.node_flags[tb + ch] = 0;
                v.child[eb + best] = ch;
            }
            st = next;
            flags = 0;
        } else {
            st = v.node_state[tb + ch];
            flags = v.node_flags[tb + ch];
        }
        if (lane == 0) {
            path[depth] = node;
            acts[depth] = (uint8_t)best;
        }
        ++depth;
        node = ch;
    }
}

// Backup of `value` (from the leaf player's view) along a path
// (BatchedPUCT.cpp:218-227). Lanes own path steps; the caller orders it.
__device__ __forceinline__ void backup_path(const BpuctView& v, int64_t t, int C, const int32_t* path,
                                            const uint8_t* acts, int depth, int leaf, int leaf_actor, double value,
                                            int lane) {
    const int64_t tb = t * C;
    if (lane == 0) v.node_visits[tb] += 1;
    for (int d = lane; d < depth; d += 32) {
        const int parent = path[d];
        const int next = d + 1 < depth ? path[d + 1] : leaf;
        const int64_t e = (tb + parent) * GK_ACTIONS + acts[d];
        const int parent_actor = (int)(v.node_state[tb + parent].w[15] & 3u);
        v.wsum[e] = GK_DADD(v.wsum[e], parent_actor == leaf_actor ? value : -value);
        v.visits[e] += 1;
        v.node_visits[tb + next] += 1;
    }
}

// Adds `delta` reservations along a path (BatchedPUCT.cpp:198-216).
__device__ __forceinline__ void reserve_path(const BpuctView& v, int64_t t, int C, const int32_t* path,
                                             const uint8_t* acts, int depth, int leaf, int delta, int lane) {
    const int64_t tb = t * C;
    if (lane == 0) v.node_reserved[tb] += delta;
    for (int d = lane; d < depth; d += 32) {
        const int next = d + 1 < depth ? path[d + 1] : leaf;
        v.reserved[(tb + path[d]) * GK_ACTIONS + acts[d]] += delta;
        v.node_reserved[tb + next] += delta;
        if (delta < 0) v.node_flags[tb + path[d]] &= (uint8_t)~kBlocked;
    }
}

// After `leaf` became pending: mark it blocked, then each ancestor whose legal
// edges all lead to blocked children, stopping at the first that has an open one.
__device__ void propagate_blocked(const BpuctView& v, int64_t t, int C, const int32_t* path, int depth, int leaf,
                                  int lane) {
    const int64_t tb = t * C;
    if (lane == 0) v.node_flags[tb + leaf] |= kPending | kBlocked;
    __syncwarp();
    for (int j = depth - 1; j >= 0; --j) {
        const int node = path[j];
        const int64_t vtx = tb + node, eb = vtx * GK_ACTIONS;
        const gk_bits st = v.node_state[vtx];
        const gk_b96 placements = legal_placements(st);
        bool open = false;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int a = lane + 32 * k;
            if (a >= GK_ACTIONS || !legal_at(placements, st, a)) continue;
            const int ch = v.child[eb + a];
            open |= ch < 0 || !(v.node_flags[tb + ch] & kBlocked);
        }
        if (__any_sync(kFull, open)) return;
        if (lane == 0) v.node_flags[vtx] |= kBlocked;
        __syncwarp();
    }
}

// ---- one wave's collection -----------------------------------------------------
// BatchedPUCT.cpp:377-404: select leaves until the wave holds min(remaining, L)
// of them; finished leaves are backed up at once with their exact value and
// take no slot.
__device__ void collect_tree(const BpuctView& v, int64_t t, int C, int L, double c_puct, int lane) {
    const int P = path_cap(C);
    int pend = 0;
    if (v.mode[t] == kSearching && v.errors[t] == 0u) {
        const int budget = v.budget[t];
        int sims = v.sims[t];
        const int remaining = budget - sims;
        const int cap = remaining < L ? remaining : L;
        // Every pass either adds a slot, completes a simulation or stops.
        for (int guard = 0; guard <= cap + remaining && pend < cap && pend < budget - sims; ++guard) {
            const int64_t s = t * L + pend;
            int32_t* path = v.slot_path + s * P;
            uint8_t* acts = v.slot_act + s * P;
            int depth = 0;
            gk_bits leaf_state;
            const int leaf = select_leaf(v, t, C, c_puct, lane, path, acts, depth, leaf_state);
            __syncwarp();
            if (leaf < 0) break;
            if (gk_reason(&leaf_state) != GK_NONE) {
                backup_path(v, t, C, path, acts, depth, leaf, gk_actor(&leaf_state), terminal_value(leaf_state), lane);
                ++sims;
                __syncwarp();
                continue;
            }
            if (lane == 0) {
                v.slot_node[s] = leaf;
                v.slot_len[s] = depth;
                v.slot_bits[s] = leaf_state;
            }
            reserve_path(v, t, C, path, acts, depth, leaf, 1, lane);
            __syncwarp();
            propagate_blocked(v, t, C, path, depth, leaf, lane);
            __syncwarp();
            ++pend;
        }
        if (lane == 0) v.sims[t] = sims;
    }
    if (lane == 0) v.pending[t] = pend;
    for (int i = lane; i < L; i += 32) v.slot_needs[t * L + i] = i < pend ? 1 : 0;
}

// ---- one wave's expansion and backup -------------------------------------------
// BatchedPUCT.cpp:405-413: expand, release and back up each collected leaf in
// collection order.
__device__ void expand_tree(const BpuctView& v, int64_t t, int C, int L, bool float_eval, int lane) {
    const int P = path_cap(C);
    const int pend = v.pending[t];
    if (v.mode[t] != kSearching) return;
    bool ok = v.errors[t] == 0u;
    for (int i = 0; i < pend && ok; ++i) {
        const int64_t s = t * L + i;
        const int leaf = v.slot_node[s], depth = v.slot_len[s];
        const int32_t* path = v.slot_path + s * P;
        const uint8_t* acts = v.slot_act + s * P;
        double value;
        ok = expand_slot(v, t, C, s, leaf, float_eval, lane, value);
        if (!ok) break;
        reserve_path(v, t, C, path, acts, depth, leaf, -1, lane);
        backup_path(v, t, C, path, acts, depth, leaf, gk_actor(&v.slot_bits[s]), value, lane);
        __syncwarp();
    }
    if (lane == 0) {
        if (ok) {
            v.sims[t] += pend;
            if (pend > 0) {
                int32_t* st = v.stats + t * kStats;
                st[kStEvals] += pend;
                st[kStBatches] += 1;
                if (st[kStMaxBatch] < pend) st[kStMaxBatch] = pend;
            }
            const int left = v.budget[t] - v.sims[t];
            if (left > 0) atomicMax(v.remaining, left);
        }
        v.pending[t] = 0;
    }
    for (int i = lane; i < L; i += 32) v.slot_needs[t * L + i] = 0;
}

// ---- injected evaluator ----------------------------------------------------------
__device__ __forceinline__ void hash_eval_slot(const BpuctView& v, int64_t s, int lane) {
    uint64_t words[GK_EVAL_WORDS];
    const gk_bits st = v.slot_bits[s];
    gk_eval_words_from_bits(&st, words);
    const uint64_t h = gk_eval_hash_words(words);
    for (int a = lane; a < GK_ACTIONS; a += 32) v.slot_policy[s * GK_ACTIONS + a] = (double)gk_eval_weight(h, a);
    if (lane == 0) v.slot_value[s] = (double)gk_eval_value(h);
}

__device__ __forceinline__ void hash_eval_tree(const BpuctView& v, int64_t t, int L, int lane) {
    for (int i = 0; i < L; ++i)
        if (v.slot_needs[t * L + i]) hash_eval_slot(v, t * L + i, lane);
}

// ---- results ---------------------------------------------------------------------
struct BpuctOut {
    int64_t* actions;
    int32_t* visits;
    double* priors;
    double* move_values;
    uint8_t* legal;
    int32_t* sims;
    int32_t* nodes;
    double* root_values;
    double* best_values;
    int32_t* stats;
    uint32_t* errors;
    uint32_t* status;
};

// BatchedPUCT.cpp:415-441: visits and values gained in this search, the best
// move by (visits, value, prior, lower action), and the root value. A failed
// search clears its tree (BatchedPUCT.cpp:435-440).
__device__ void finish_tree(const BpuctView& v, int64_t t, int C, const BpuctOut& out, int lane) {
    const int64_t tb = t * C, eb = tb * GK_ACTIONS, row = t * GK_ACTIONS;
    const int mode = v.mode[t];
    const int sims = v.sims[t];
    uint32_t err = v.errors[t];
    const gk_bits root = v.node_state[tb];
    const bool live = mode == kSearching && err == 0u && v.count[t] > 0;
    const gk_b96 placements = legal_placements(root);
    bool use[3];
    double sum[3];
    int best = -1, best_n = 0;
    double best_q = 0.0, best_p = 0.0;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int a = lane + 32 * k;
        use[k] = false;
        sum[k] = 0.0;
        if (a >= GK_ACTIONS) continue;
        use[k] = live && legal_at(placements, root, a);
        int n = 0;
        double p = 0.0, q = 0.0;
        if (use[k]) {
            n = v.visits[eb + a] - v.init_visits[row + a];
            sum[k] = GK_DSUB(v.wsum[eb + a], v.init_wsum[row + a]);
            p = v.prior[eb + a];
            q = n == 0 ? 0.0 : sum[k] / (double)n;
            if (best < 0 || n > best_n || (n == best_n && (q > best_q || (q == best_q && p > best_p)))) {
                best = a;
                best_n = n;
                best_q = q;
                best_p = p;
            }
        }
        out.visits[row + a] = n;
        out.priors[row + a] = p;
        out.move_values[row + a] = q;
        out.legal[row + a] = use[k] ? 1 : 0;
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const int oa = __shfl_down_sync(kFull, best, off);
        const int on = __shfl_down_sync(kFull, best_n, off);
        const double oq = __shfl_down_sync(kFull, best_q, off);
        const double op = __shfl_down_sync(kFull, best_p, off);
        if (oa >= 0 && (best < 0 || on > best_n ||
                        (on == best_n && (oq > best_q || (oq == best_q && (op > best_p || (op == best_p && oa < best))))))) {
            best = oa;
            best_n = on;
            best_q = oq;
            best_p = op;
        }
    }
    const double root_sum = ordered_sum(sum, use);
    if (lane == 0) {
        if (live && (best < 0 || best_n == 0)) err |= GK_ERR_CAPACITY;
        const bool ok = live && err == 0u;
        if (mode == kSearching && !ok) v.count[t] = 0;
        if (!ok && mode == kSearching) {
            for (int a = 0; a < GK_ACTIONS; ++a) {
                out.visits[row + a] = 0;
                out.priors[row + a] = 0.0;
                out.move_values[row + a] = 0.0;
                out.legal[row + a] = 0;
            }
        }
        out.actions[t] = ok ? best : -1;
        out.sims[t] = ok ? sims : 0;
        out.nodes[t] = ok ? v.count[t] : 0;
        out.root_values[t] = ok ? root_sum / (double)sims : mode == kTerminalRoot ? v.root_terminal[t] : 0.0;
        out.best_values[t] = ok ? best_q : 0.0;
        for (int i = 0; i < kStats; ++i) out.stats[t * kStats + i] = v.stats[t * kStats + i];
        out.errors[t] = mode == kSearching ? err : 0u;
        if (mode == kSearching && err && out.status) atomicOr(out.status, err);
    }
}

// ---- advance ---------------------------------------------------------------------
// BatchedPUCT.cpp:290-326: keep the played move's subtree and compact it to
// the front of the tree. Nodes are renumbered in their existing order (a
// child is always created after its parent, so the new root takes index 0 and
// every node moves down or stays), which lets the copy run in place.
__device__ void advance_tree(const BpuctView& v, int64_t t, int C, const int32_t* actions, const uint8_t* mask,
                             int reuse, uint8_t* advanced, int lane) {
    if (mask && !mask[t]) {
        if (lane == 0 && advanced) advanced[t] = 0;
        return;
    }
    const int64_t tb = t * C;
    int32_t* st = v.stats + t * kStats;
    const int count = v.count[t];
    if (lane == 0) st[kStAdvances] += 1;
    if (!reuse || count == 0) {
        if (lane == 0) {
            v.count[t] = 0;
            if (advanced) advanced[t] = 0;
        }
        return;
    }
    const gk_bits root = v.node_state[tb];
    const int a = actions[t];
    const bool legal = a >= 0 && a < GK_ACTIONS && legal_at(legal_placements(root), root, a);
    if (!legal) {
        if (lane == 0 && advanced) advanced[t] = 0;
        return;
    }
    const int ch = (v.node_flags[tb] & kExpanded) ? v.child[tb * GK_ACTIONS + a] : -1;
    if (ch < 0) {
        if (lane == 0) {
            v.count[t] = 0;
            if (advanced) advanced[t] = 0;
        }
        return;
    }
    int32_t* remap = v.remap + tb;
    // 1. Mark the subtree: children always follow their parent, so one pass
    //    in index order from `ch` reaches every descendant. Each chunk of 32
    //    nodes is rescanned until no marked, expanded node in it is left
    //    unvisited (a node can mark later nodes of its own chunk).
    for (int i = ch + lane; i < count; i += 32) remap[i] = i == ch ? 0 : -1;
    __syncwarp();
    for (int base = ch; base < count; base += 32) {
        const int i = base + lane;
        unsigned done = 0u;
        for (int guard = 0; guard < 33; ++guard) {
            const bool marked = i < count && remap[i] >= 0 && (v.node_flags[tb + i] & kExpanded);
            const unsigned todo = __ballot_sync(kFull, marked) & ~done;
            if (!todo) break;
            const int j = __ffs(todo) - 1;
            done |= 1u << j;
            const int64_t eb = (tb + base + j) * GK_ACTIONS;
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const int e = lane + 32 * k;
                if (e >= GK_ACTIONS) continue;
                const int c = v.child[eb + e];
                if (c >= 0) remap[c] = 0;
            }
            __syncwarp();
        }
    }
    __syncwarp();
    // 2. New indices: the rank of each kept node among the kept nodes.
    int kept = 0;
    for (int base = ch; base < count; base += 32) {
        const int i = base + lane;
        const bool keep = i < count && remap[i] >= 0;
        const unsigned bal = __ballot_sync(kFull, keep);
        if (i < count) remap[i] = keep ? kept + __popc(bal & ((1u << lane) - 1u)) : -1;
        kept += __popc(bal);
    }
    __syncwarp();
    // 3. Move each kept node to its new index, children renumbered.
    for (int base = ch; base < count; base += 32) {
        const int i = base + lane;
        unsigned todo = __ballot_sync(kFull, i < count && remap[i] >= 0);
        while (todo) {
            const int j = __ffs(todo) - 1;
            todo &= todo - 1u;
            const int from = base + j;
            const int to = remap[from];
            const int64_t src = tb + from, dst = tb + to;
            const uint8_t flags = v.node_flags[src];
            if (lane < 16) v.node_state[dst].w[lane] = v.node_state[src].w[lane];
            if (flags & kExpanded) {
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    const int e = lane + 32 * k;
                    if (e >= GK_ACTIONS) continue;
                    const int64_t se = src * GK_ACTIONS + e, de = dst * GK_ACTIONS + e;
                    const int c = v.child[se];
                    const double p = v.prior[se], w = v.wsum[se];
                    const int n = v.visits[se], r = v.reserved[se];
                    v.prior[de] = p;
                    v.wsum[de] = w;
                    v.visits[de] = n;
                    v.reserved[de] = r;
                    v.child[de] = c >= 0 ? remap[c] : -1;
                }
            }
            if (lane == 0) {
                const int nv = v.node_visits[src], nr = v.node_reserved[src];
                v.node_visits[dst] = nv;
                v.node_reserved[dst] = nr;
                v.node_flags[dst] = flags;
            }
            __syncwarp();
        }
    }
    if (lane == 0) {
        v.count[t] = kept;
        st[kStReuseHits] += 1;
        if (advanced) advanced[t] = 1;
    }
}

// ---- kernels -----------------------------------------------------------------------
#define GK_TREE_WARP()                                                          \
    const int lane = threadIdx.x & 31;                                          \
    const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;   \
    if (t >= T) return

__global__ void __launch_bounds__(32 * kWarps) bpuct_init_kernel(BpuctView v, int64_t T, int L) {
    GK_TREE_WARP();
    if (lane == 0) {
        v.count[t] = 0;
        v.mode[t] = kIdle;
        v.pending[t] = 0;
        v.errors[t] = 0u;
        v.sims[t] = 0;
        v.budget[t] = 0;
        for (int i = 0; i < kStats; ++i) v.stats[t * kStats + i] = 0;
    }
    for (int i = lane; i < L; i += 32) v.slot_needs[t * L + i] = 0;
}

__global__ void __launch_bounds__(32 * kWarps) bpuct_clear_kernel(BpuctView v, int64_t T, const uint8_t* mask) {
    GK_TREE_WARP();
    if (lane == 0 && (!mask || mask[t])) v.count[t] = 0;
}

__global__ void __launch_bounds__(32 * kWarps)
    bpuct_begin_kernel(BpuctView v, int64_t T, int C, int L, const gk_bits* roots, const uint8_t* mask,
                       int simulations, int reuse) {
    GK_TREE_WARP();
    begin_tree(v, t, C, L, roots, mask, simulations, reuse, lane);
}

__global__ void __launch_bounds__(32 * kWarps) bpuct_root_expand_kernel(BpuctView v, int64_t T, int C, int L,
                                                                        int float_eval) {
    GK_TREE_WARP();
    root_expand_tree(v, t, C, L, float_eval != 0, lane);
}

__global__ void __launch_bounds__(32 * kWarps) bpuct_collect_kernel(BpuctView v, int64_t T, int C, int L,
                                                                    double c_puct) {
    GK_TREE_WARP();
    if (t == 0 && lane == 0) *v.remaining = 0;
    collect_tree(v, t, C, L, c_puct, lane);
}

__global__ void __launch_bounds__(32 * kWarps) bpuct_hash_eval_kernel(BpuctView v, int64_t S) {
    const int lane = threadIdx.x & 31;
    const int64_t s = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    if (s < S && v.slot_needs[s]) hash_eval_slot(v, s, lane);
}

__global__ void __launch_bounds__(1024) bpuct_compact_kernel(BpuctView v, int64_t S) {
    __shared__ int warp_sums[32];
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t base = 0; base < S; base += blockDim.x) {
        const int64_t s = base + threadIdx.x;
        const int flag = (s < S && v.slot_needs[s]) ? 1 : 0;
        const unsigned ballot = __ballot_sync(kFull, flag);
        const int in_warp = __popc(ballot & ((1u << lane) - 1u));
        if (lane == 31) warp_sums[warp] = in_warp + flag;
        __syncthreads();
        if (warp == 0) {
            int x = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(kFull, x, off);
                if (lane >= off) x += y;
            }
            warp_sums[lane] = x;
        }
        __syncthreads();
        const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + in_warp;
        if (flag) v.active[carry + before] = (int32_t)s;
        __syncthreads();
        if (threadIdx.x == 0) carry += warp_sums[(blockDim.x >> 5) - 1];
        __syncthreads();
    }
    if (threadIdx.x == 0) *v.active_count = carry;
}

__global__ void __launch_bounds__(32 * kWarps) bpuct_expand_kernel(BpuctView v, int64_t T, int C, int L,
                                                                   int float_eval) {
    GK_TREE_WARP();
    expand_tree(v, t, C, L, float_eval != 0, lane);
}

__global__ void __launch_bounds__(32 * kWarps) bpuct_finish_kernel(BpuctView v, int64_t T, int C, BpuctOut out) {
    GK_TREE_WARP();
    finish_tree(v, t, C, out, lane);
}

__global__ void __launch_bounds__(32 * kWarps) bpuct_advance_kernel(BpuctView v, int64_t T, int C,
                                                                    const int32_t* actions, const uint8_t* mask,
                                                                    int reuse, uint8_t* advanced) {
    GK_TREE_WARP();
    advance_tree(v, t, C, actions, mask, reuse, advanced, lane);
}

// A whole injected-evaluator search in one launch, one warp per tree: the
// evaluator is a pure function of the leaf, so no tree waits for another and
// each warp runs its waves back to back. Each wave completes at least one
// simulation, so budget + 1 waves bound the loop. Seven blocks per SM (72
// registers) keep 4,144 trees resident at once; at 128 registers only four
// fit and a 4,096-tree search ran in two rounds of blocks (7.91 -> 6.68 ms
// for 4,096 trees x 128 simulations on a B200).
__global__ void __launch_bounds__(32 * kWarps, 7) bpuct_search_hash_kernel(BpuctView v, int64_t T, int C, int L,
                                                                        const gk_bits* roots, const uint8_t* mask,
                                                                        int simulations, int reuse, double c_puct,
                                                                        BpuctOut out) {
    GK_TREE_WARP();
    begin_tree(v, t, C, L, roots, mask, simulations, reuse, lane);
    __syncwarp();
    if (v.mode[t] == kSearching) {
        hash_eval_tree(v, t, L, lane);
        __syncwarp();
        root_expand_tree(v, t, C, L, false, lane);
        __syncwarp();
        for (int wave = 0; wave <= simulations && v.errors[t] == 0u && v.sims[t] < v.budget[t]; ++wave) {
            collect_tree(v, t, C, L, c_puct, lane);
            __syncwarp();
            hash_eval_tree(v, t, L, lane);
            __syncwarp();
            expand_tree(v, t, C, L, false, lane);
            __syncwarp();
        }
        if (lane == 0 && v.errors[t] == 0u && v.sims[t] < v.budget[t]) v.errors[t] |= GK_ERR_CAPACITY;
        __syncwarp();
    }
    finish_tree(v, t, C, out, lane);
}

#undef GK_TREE_WARP

inline int tree_grid(int64_t T) { return blocks_for(T, kWarps, 1 << 30); }

inline bool valid(const void* ws, int64_t T, int C, int L) {
    return ws != nullptr && T > 0 && T < (1ll << 24) && C >= 1 && C < (1 << 24) && L >= 1 && L <= 4096 &&
           T * (int64_t)L < (1ll << 31);
}

inline BpuctView view_of(void* ws, int64_t T, int C, int L) {
    BpuctView v;
    bpuct_layout(ws, T, C, L, &v);
    return v;
}

inline bool valid_out(const gk_bpuct_results_t* o) {
    return o && o->actions && o->visits && o->priors && o->move_values && o->legal && o->simulations && o->nodes &&
           o->root_values && o->best_values && o->stats && o->errors;
}

inline BpuctOut out_of(const gk_bpuct_results_t* o) {
    return BpuctOut{o->actions, o->visits,      o->priors,      o->move_values, o->legal,  o->simulations,
                    o->nodes,   o->root_values, o->best_values, o->stats,       o->errors, o->status};
}

}  // namespace
}  // namespace gk

extern "C" {

size_t gk_bpuct_workspace_bytes(int64_t trees, int capacity, int leaf_batch) {
    using namespace gk;
    if (!valid(reinterpret_cast<void*>(1), trees, capacity, leaf_batch)) return 0;
    return bpuct_layout(nullptr, trees, capacity, leaf_batch, nullptr);
}

int gk_bpuct_buffers(void* ws, int64_t trees, int capacity, int leaf_batch, gk_bpuct_buffers_t* out) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch) || out == nullptr) return GK_EINVAL;
    const BpuctView v = view_of(ws, trees, capacity, leaf_batch);
    out->needs_eval = v.slot_needs;
    out->leaf_bits = reinterpret_cast<uint32_t*>(v.slot_bits);
    out->policy = v.slot_policy;
    out->value = v.slot_value;
    out->policy_f = v.slot_policy_f;
    out->value_f = v.slot_value_f;
    out->active = v.active;
    out->active_count = v.active_count;
    out->pending = v.pending;
    out->node_count = v.count;
    out->remaining = v.remaining;
    out->stats = v.stats;
    return 0;
}

int gk_bpuct_init(void* ws, int64_t trees, int capacity, int leaf_batch, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch)) return GK_EINVAL;
    bpuct_init_kernel<<<tree_grid(trees), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), trees, leaf_batch);
    return launch_status();
}

int gk_bpuct_clear(void* ws, int64_t trees, int capacity, int leaf_batch, const uint8_t* mask, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch)) return GK_EINVAL;
    bpuct_clear_kernel<<<tree_grid(trees), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), trees, mask);
    return launch_status();
}

int gk_bpuct_begin(void* ws, int64_t trees, int capacity, int leaf_batch, const uint32_t* roots, const uint8_t* mask,
                   int simulations, int reuse, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch) || roots == nullptr || simulations < 1) return GK_EINVAL;
    bpuct_begin_kernel<<<tree_grid(trees), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), trees, capacity, leaf_batch,
        reinterpret_cast<const gk_bits*>(roots), mask, simulations, reuse);
    return launch_status();
}

int gk_bpuct_root_expand(void* ws, int64_t trees, int capacity, int leaf_batch, int float_eval, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch)) return GK_EINVAL;
    bpuct_root_expand_kernel<<<tree_grid(trees), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), trees, capacity, leaf_batch, float_eval);
    return launch_status();
}

int gk_bpuct_collect(void* ws, int64_t trees, int capacity, int leaf_batch, double c_puct, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch) || !(c_puct > 0.0) || !isfinite(c_puct)) return GK_EINVAL;
    bpuct_collect_kernel<<<tree_grid(trees), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), trees, capacity, leaf_batch, c_puct);
    return launch_status();
}

int gk_bpuct_hash_eval(void* ws, int64_t trees, int capacity, int leaf_batch, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch)) return GK_EINVAL;
    const int64_t S = trees * leaf_batch;
    bpuct_hash_eval_kernel<<<tree_grid(S), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), S);
    return launch_status();
}

int gk_bpuct_compact(void* ws, int64_t trees, int capacity, int leaf_batch, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch)) return GK_EINVAL;
    bpuct_compact_kernel<<<1, 1024, 0, as_stream(stream)>>>(view_of(ws, trees, capacity, leaf_batch),
                                                            trees * leaf_batch);
    return launch_status();
}

int gk_bpuct_expand(void* ws, int64_t trees, int capacity, int leaf_batch, int float_eval, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch)) return GK_EINVAL;
    bpuct_expand_kernel<<<tree_grid(trees), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), trees, capacity, leaf_batch, float_eval);
    return launch_status();
}

int gk_bpuct_finish(void* ws, int64_t trees, int capacity, int leaf_batch, const gk_bpuct_results_t* out,
                    void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch) || !valid_out(out)) return GK_EINVAL;
    if (out->status) {
        const cudaError_t e = cudaMemsetAsync(out->status, 0, sizeof(uint32_t), as_stream(stream));
        if (e != cudaSuccess) return (int)e;
    }
    bpuct_finish_kernel<<<tree_grid(trees), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), trees, capacity, out_of(out));
    return launch_status();
}

int gk_bpuct_advance(void* ws, int64_t trees, int capacity, int leaf_batch, const int32_t* actions,
                     const uint8_t* mask, int reuse, uint8_t* advanced, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch) || actions == nullptr) return GK_EINVAL;
    bpuct_advance_kernel<<<tree_grid(trees), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), trees, capacity, actions, mask, reuse, advanced);
    return launch_status();
}

int gk_bpuct_search_hash(void* ws, int64_t trees, int capacity, int leaf_batch, const uint32_t* roots,
                         const uint8_t* mask, int simulations, int reuse, double c_puct,
                         const gk_bpuct_results_t* out, void* stream) {
    using namespace gk;
    if (!valid(ws, trees, capacity, leaf_batch) || roots == nullptr || simulations < 1 || !(c_puct > 0.0) ||
        !isfinite(c_puct) || !valid_out(out))
        return GK_EINVAL;
    if (out->status) {
        const cudaError_t e = cudaMemsetAsync(out->status, 0, sizeof(uint32_t), as_stream(stream));
        if (e != cudaSuccess) return (int)e;
    }
    bpuct_search_hash_kernel<<<tree_grid(trees), 32 * kWarps, 0, as_stream(stream)>>>(
        view_of(ws, trees, capacity, leaf_batch), trees, capacity, leaf_batch, reinterpret_cast<const gk_bits*>(roots),
        mask, simulations, reuse, c_puct, out_of(out));
    return launch_status();
}

// Copies every tree of a workspace into one with more nodes per tree (the
// slot arrays are scratch of a single search and are not copied).
int gk_bpuct_grow(const void* src, int capacity, void* dst, int new_capacity, int64_t trees, int leaf_batch,
                  void* stream) {
    using namespace gk;
    if (!valid(const_cast<void*>(src), trees, capacity, leaf_batch) || !valid(dst, trees, new_capacity, leaf_batch) ||
        new_capacity < capacity || path_cap(new_capacity) < path_cap(capacity))
        return GK_EINVAL;
    const BpuctView a = view_of(const_cast<void*>(src), trees, capacity, leaf_batch);
    const BpuctView b = view_of(dst, trees, new_capacity, leaf_batch);
    const cudaStream_t s = as_stream(stream);
    cudaError_t e = cudaSuccess;
    auto rows = [&](void* to, const void* from, size_t per_node) {
        if (e != cudaSuccess) return;
        e = cudaMemcpy2DAsync(to, per_node * new_capacity, from, per_node * capacity, per_node * capacity, trees,
                              cudaMemcpyDeviceToDevice, s);
    };
    auto flat = [&](void* to, const void* from, size_t bytes) {
        if (e != cudaSuccess) return;
        e = cudaMemcpyAsync(to, from, bytes, cudaMemcpyDeviceToDevice, s);
    };
    rows(b.node_state, a.node_state, sizeof(gk_bits));
    rows(b.node_visits, a.node_visits, 4);
    rows(b.node_reserved, a.node_reserved, 4);
    rows(b.node_flags, a.node_flags, 1);
    rows(b.prior, a.prior, 8 * GK_ACTIONS);
    rows(b.wsum, a.wsum, 8 * GK_ACTIONS);
    rows(b.visits, a.visits, 4 * GK_ACTIONS);
    rows(b.reserved, a.reserved, 4 * GK_ACTIONS);
    rows(b.child, a.child, 4 * GK_ACTIONS);
    flat(b.count, a.count, trees * 4);
    flat(b.mode, a.mode, trees * 4);
    flat(b.budget, a.budget, trees * 4);
    flat(b.sims, a.sims, trees * 4);
    flat(b.pending, a.pending, trees * 4);
    flat(b.stats, a.stats, trees * kStats * 4);
    flat(b.errors, a.errors, trees * 4);
    flat(b.root_terminal, a.root_terminal, trees * 8);
    flat(b.init_visits, a.init_visits, trees * GK_ACTIONS * 4);
    flat(b.init_wsum, a.init_wsum, trees * GK_ACTIONS * 8);
    flat(b.slot_needs, a.slot_needs, trees * leaf_batch);
    return e == cudaSuccess ? 0 : (int)e;
}

}  // extern "C"
