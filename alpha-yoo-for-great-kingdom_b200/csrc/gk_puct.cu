// gk_puct.cu - batched PUCT over structure-of-arrays trees in HBM.
//
// One warp owns one tree in select, expand/backup and finish: lanes score the
// 82 edges of a node in parallel (3 per lane) and a warp argmax picks the
// edge; the serial dependencies of the reference (the prior normaliser and the
// root value are sums in action order) are evaluated in action order through
// warp shuffles so every double is bit-identical to the reference search.
//
// Reference semantics followed:
//   select            mcts/src/PUCT.cpp:118-142, python/kingdom_ai/gpu_puct.py:182-258
//   expand (priors)   mcts/src/PUCT.cpp:53-86,  gpu_puct.py:277-324
//   root noise mix    gpu_puct.py:308-321 (mix and renormalise as PUCT.cpp:88-116)
//   backup            mcts/src/PUCT.cpp:228-236, gpu_puct.py:325-340
//   finish            mcts/src/PUCT.cpp:246-267, gpu_puct.py:343-379
// Double arithmetic goes through GK_DADD/GK_DMUL (__dadd_rn/__dmul_rn) so no
// FMA contraction changes a bit; division and sqrt are IEEE round-to-nearest.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/gk.h"
#include "gk_device.cuh"
#include "gk_launch.cuh"
#include "gk_puct.cuh"
#include "gk_random.cuh"

namespace gk {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kWarpsPerBlock = 4;

__device__ __forceinline__ bool action_legal(const gk_b96& placements, bool pass_ok, int a) {
    return a == GK_PASS ? pass_ok : gk_test(placements, a + a / 9) != 0;
}

// This lane's root-candidate bits for actions lane, lane+32, lane+64 of tree
// t's node `node`: the root's words, all ones elsewhere.
__device__ __forceinline__ void allow_bits(const PuctView& v, int64_t t, int node, int lane, bool (&ok)[3]) {
#pragma unroll
    for (int k = 0; k < 3; ++k) ok[k] = node != 0 || ((v.root_allow[t * 3 + k] >> lane) & 1u) != 0u;
}

__device__ __forceinline__ float terminal_value(const gk_bits& s) {
    return gk_winner(&s) == gk_actor(&s) ? 1.0f : -1.0f;
}

// Per-warp shared scratch of an ordered sum: one double per action.
constexpr int kSumScratch = 96;

// Sum of per-lane values v[k] (action a = lane + 32k) over selected actions in
// increasing action order; every lane returns the same total. The values pass
// through the warp's scratch `sc`, unselected ones as +0.0: every caller's
// selected values are >= +0 or sums that start at +0, so the running total is
// never -0 and adding +0.0 leaves it bit-identical to skipping the action.
__device__ __forceinline__ double ordered_sum(const double (&v)[3], const bool (&use)[3], double* sc, int lane) {
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

__global__ void puct_begin_kernel(PuctView v, int64_t B, int C, const gk_bits* roots) {
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < B; t += (int64_t)gridDim.x * blockDim.x) {
        const gk_bits r = roots[t];
        const int64_t vtx = t * C;
        const bool live = gk_reason(&r) == GK_NONE;
        v.node_state[vtx] = r;
        v.node_visits[vtx] = 0;
        v.node_value[vtx] = 0.0f;
        v.expanded[vtx] = 0;
        v.node_count[t] = live ? 1 : 0;
        v.leaf[t] = 0;
        v.path_len[t] = 0;
        v.sims[t] = 0;
        v.evals[t] = 0;
        v.errors[t] = 0u;
        v.needs_eval[t] = live ? 1 : 0;
        v.leaf_bits[t] = r;
        v.leaf_value[t] = live ? 0.0f : terminal_value(r);
        v.root_allow[t * 3] = 0xffffffffu;
        v.root_allow[t * 3 + 1] = 0xffffffffu;
        v.root_allow[t * 3 + 2] = (1u << (GK_ACTIONS - 64)) - 1u;
    }
}

// This lane's three edges (actions lane, lane+32, lane+64) of node vtx.
__device__ __forceinline__ void load_edges(const PuctView& v, int64_t vtx, int lane, int (&en)[3], double (&ep)[3],
                                           double (&ew)[3], int (&ech)[3]) {
    const int64_t ebase = vtx * GK_ACTIONS;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int a = lane + 32 * k;
        const bool in_row = a < GK_ACTIONS;
        en[k] = in_row ? v.visits[ebase + a] : 0;
        ep[k] = in_row ? v.prior[ebase + a] : 0.0;
        ew[k] = in_row ? v.wsum[ebase + a] : 0.0;
        ech[k] = in_row ? v.child[ebase + a] : -1;
    }
}

// A path entry: the action taken (bits 0-7) and the player to move at the
// parent (bits 8-9), so the backup needs neither the parent's state nor the
// edge's child index (the child of entry d is the node of entry d + 1).
__device__ __forceinline__ int32_t path_entry(int action, int actor) { return action | (actor << 8); }

// One selection pass of tree t by its warp (every lane calls it).
__device__ __forceinline__ void select_tree(const PuctView& v, int64_t t, int C, const PuctOptions& o, int lane) {
    const int P = path_cap(C);
    if (lane == 0) v.needs_eval[t] = 0;
    if (v.node_count[t] == 0) {  // terminal root: no tree, value fixed at begin
        if (lane == 0) v.path_len[t] = 0;
        return;
    }
    const int64_t tbase = t * C;
    int node = 0, depth = 0;
    // The current node's state and statistics stay in registers; a level
    // loads its edges (this lane's three: visits, prior, W, child) once the
    // node is known to be expanded. Loading a chosen child's edges together
    // with its state (one dependent round trip per level instead of two) was
    // measured and gained nothing in self-play or in the fused search. A child
    // created during this pass is known to be unexpanded, so no lane reads
    // memory another lane of this warp has just written.
    gk_bits st = v.node_state[tbase];
    bool expanded = v.expanded[tbase] != 0;
    int node_n = v.node_visits[tbase];
    float node_q = v.node_value[tbase];
    int en[3], ech[3];
    double ep[3], ew[3];
    bool fresh = false;
    for (;;) {
        const int64_t vtx = tbase + node;
        if (gk_reason(&st) != GK_NONE) {
            if (lane == 0) v.leaf_value[t] = terminal_value(st);
            break;
        }
        if (fresh || !expanded) {
            if (lane == 0) {
                v.needs_eval[t] = 1;
                v.leaf_bits[t] = st;
            }
            break;
        }
        const int64_t ebase = vtx * GK_ACTIONS;
        load_edges(v, vtx, lane, en, ep, ew, ech);
        const double scale = sqrt((double)node_n);
        const gk_b96 placements = legal_placements(st);
        bool allowed[3];
        allow_bits(v, t, node, lane, allowed);
        int best = -1;
        double best_score = 0.0, best_prior = 0.0;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int a = lane + 32 * k;
            if (a >= GK_ACTIONS || !allowed[k] || !action_legal(placements, true, a)) continue;
            const int n = en[k];
            const double p = ep[k];
            double q;
            if (n == 0) q = o.fpu_enabled != 0.0 ? GK_DSUB((double)node_q, o.fpu_reduction) : 0.0;
            else q = ew[k] / (double)n;
            const double expl = GK_DMUL(p, scale) / GK_DADD(1.0, (double)n);
            const double score = o.c_puct >= 1.0 ? GK_DADD(q / o.c_puct, expl) : GK_DADD(q, GK_DMUL(o.c_puct, expl));
            if (best < 0 || score > best_score || (score == best_score && p > best_prior)) {
                best = a;
                best_score = score;
                best_prior = p;
            }
        }
        // Warp argmax: higher score, then higher prior, then lower action index.
        // Each lane's candidate is already the best of its own edges in that
        // order, so when a single lane holds the highest score its candidate
        // is the answer; ties (and no candidate at all) take the full
        // reduction.
        {
            double top = best >= 0 ? best_score : -INFINITY;
#pragma unroll
            for (int off = 16; off; off >>= 1) top = fmax(top, __shfl_xor_sync(kFull, top, off));
            const unsigned holders = __ballot_sync(kFull, best >= 0 && best_score == top);
            if (__popc(holders) == 1) {
                best = __shfl_sync(kFull, best, __ffs(holders) - 1);
            } else {
#pragma unroll
                for (int off = 16; off; off >>= 1) {
                    const double os = __shfl_down_sync(kFull, best_score, off);
                    const double op = __shfl_down_sync(kFull, best_prior, off);
                    const int oa = __shfl_down_sync(kFull, best, off);
                    if (oa >= 0 && (best < 0 || os > best_score ||
                                    (os == best_score && (op > best_prior || (op == best_prior && oa < best))))) {
                        best = oa;
                        best_score = os;
                        best_prior = op;
                    }
                }
                best = __shfl_sync(kFull, best, 0);
            }
        }
        if (best < 0 || depth >= P) {
            if (lane == 0) {
                v.errors[t] |= GK_ERR_CAPACITY;
                v.leaf_value[t] = 0.0f;
            }
            break;
        }
        const int actor = gk_actor(&st);  // the parent's player, recorded with the action
        // The chosen edge's child index is already in the lane that owns it.
        const int slot = best >> 5;
        int ch = __shfl_sync(kFull, slot == 0 ? ech[0] : slot == 1 ? ech[1] : ech[2], best & 31);
        if (ch < 0) {
            gk_bits next = st;
            const bool ok = play(next, best);
            if (lane == 0) ch = v.node_count[t]++;
            ch = __shfl_sync(kFull, ch, 0);
            if (!ok || ch >= C) {
                if (lane == 0) {
                    v.errors[t] |= GK_ERR_CAPACITY;
                    v.leaf_value[t] = 0.0f;
                }
                break;
            }
            if (lane == 0) {
                v.node_state[tbase + ch] = next;
                v.node_visits[tbase + ch] = 0;
                v.node_value[tbase + ch] = 0.0f;
                v.expanded[tbase + ch] = 0;
                v.child[ebase + best] = ch;
            }
            st = next;
            fresh = true;
        } else {
            st = v.node_state[tbase + ch];
            expanded = v.expanded[tbase + ch] != 0;
            node_n = v.node_visits[tbase + ch];
            node_q = v.node_value[tbase + ch];
            fresh = false;
        }
        if (lane == 0) {
            v.path_nodes[t * P + depth] = node;
            v.path_actions[t * P + depth] = path_entry(best, actor);
        }
        ++depth;
        node = ch;
    }
    if (lane == 0) {
        v.leaf[t] = node;
        v.path_len[t] = depth;
    }
}

__global__ void __launch_bounds__(32 * kWarpsPerBlock, 7) puct_select_kernel(PuctView v, int64_t B, int C, PuctOptions o) {
    const int lane = threadIdx.x & 31;
    const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    if (t < B) select_tree(v, t, C, o, lane);
}

// Expansion of tree t's leaf with the evaluator's output and, if `backup`,
// the backup along the selected path, by the tree's warp.
__device__ __forceinline__ void expand_backup_tree(const PuctView& v, int64_t t, int C, const PuctOptions& o,
                                                   int backup, int lane, double* sc) {
    // The tree's scalars, its policy row and the path length are loaded
    // together, then the leaf's state with this lane's path entry, so the
    // expansion and the backup take three dependent global round trips.
    const int P = path_cap(C);
    const int64_t row = t * GK_ACTIONS;
    const int count = v.node_count[t];
    const int node = v.leaf[t];
    float leaf_value = v.leaf_value[t];
    const bool eval = v.needs_eval[t] != 0;
    const int len = backup ? v.path_len[t] : 0;
    float pol[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) pol[k] = lane + 32 * k < GK_ACTIONS ? v.policy[row + lane + 32 * k] : 0.0f;
    if (count == 0) return;
    const int64_t vtx = t * C + node;
    const gk_bits st = v.node_state[vtx];
    // Depth `lane` of the path: parent node, entry (action and the parent's
    // player) and child, the next entry's node or the leaf.
    int path_parent = 0, path_action = 0, path_child = 0;
    if (lane < len) {
        path_parent = v.path_nodes[t * P + lane];
        path_action = v.path_actions[t * P + lane];
        path_child = lane + 1 < len ? v.path_nodes[t * P + lane + 1] : node;
    }
    if (eval) {
        const gk_b96 placements = legal_placements(st);
        const int64_t ebase = vtx * GK_ACTIONS;
        const bool mix = node == 0 && o.epsilon != 0.0;
        bool allowed[3];
        allow_bits(v, t, node, lane, allowed);
        bool bad = !(isfinite(leaf_value) && fabsf(leaf_value) <= 1.0f);
        bool use[3];
        double w[3], nz[3];
        double largest = 0.0;
        int legal_count = 0;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int a = lane + 32 * k;
            use[k] = a < GK_ACTIONS && allowed[k] && action_legal(placements, true, a);
            w[k] = 0.0;
            nz[k] = 0.0;
            if (use[k]) {
                const float p = pol[k];
                bad |= !(isfinite(p) && p >= 0.0f);
                w[k] = (double)p;
                if (mix) nz[k] = (double)v.noise[row + a];
                largest = fmax(largest, w[k]);
                ++legal_count;
            }
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            largest = fmax(largest, __shfl_xor_sync(kFull, largest, off));
            legal_count += __shfl_xor_sync(kFull, legal_count, off);
        }
        bad = __any_sync(kFull, bad);
        double total = 0.0;
        if (!bad && largest > 0.0) {
            double scaled[3];
#pragma unroll
            for (int k = 0; k < 3; ++k) scaled[k] = use[k] ? w[k] / largest : 0.0;
            total = ordered_sum(scaled, use, sc, lane);
        }
        if (bad || legal_count == 0 || !(total > 0.0) || !isfinite(total)) {
            // Mirrors the reference's handling of a bad evaluation: flag it,
            // use a uniform policy over legal actions and a zero value.
            bad = true;
#pragma unroll
            for (int k = 0; k < 3; ++k) w[k] = use[k] ? 1.0 : 0.0;
            largest = 1.0;
            total = (double)legal_count;
            leaf_value = 0.0f;
        }
        double noise_total = 0.0;
        if (mix) noise_total = ordered_sum(nz, use, sc, lane);
        double prior[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            prior[k] = 0.0;
            if (!use[k]) continue;
            double weight = (w[k] / largest) / total;
            if (mix) {
                const double sampled = noise_total > 0.0 ? nz[k] / noise_total : 1.0 / (double)legal_count;
                weight = GK_DADD(GK_DMUL(GK_DSUB(1.0, o.epsilon), weight), GK_DMUL(o.epsilon, sampled));
            }
            prior[k] = weight;
        }
        if (mix) {
            bool all[3] = {true, true, lane + 64 < GK_ACTIONS};
            const double combined = ordered_sum(prior, all, sc, lane);
#pragma unroll
            for (int k = 0; k < 3; ++k) prior[k] = prior[k] / combined;
        }
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int a = lane + 32 * k;
            if (a < GK_ACTIONS) {
                v.prior[ebase + a] = prior[k];
                v.wsum[ebase + a] = 0.0;
                v.visits[ebase + a] = 0;
                v.child[ebase + a] = -1;
            }
        }
        if (lane == 0) {
            if (bad) v.errors[t] |= GK_ERR_BAD_EVAL;
            v.leaf_value[t] = leaf_value;
            v.node_value[vtx] = leaf_value;
            v.expanded[vtx] = 1;
            v.evals[t] += 1;
        }
    }
    if (!backup) return;
    const int leaf_actor = gk_actor(&st);
    const double lv = (double)leaf_value;
    const int64_t tbase = t * C;
    if (lane == 0) v.node_visits[tbase] += 1;
    for (int d = lane; d < len; d += 32) {
        const bool first = d == lane;
        const int parent = first ? path_parent : v.path_nodes[t * P + d];
        const int entry = first ? path_action : v.path_actions[t * P + d];
        const int child = first ? path_child : d + 1 < len ? v.path_nodes[t * P + d + 1] : node;
        const int64_t e = (tbase + parent) * GK_ACTIONS + (entry & 0xff);
        const double value = (entry >> 8) == leaf_actor ? lv : -lv;
        v.visits[e] += 1;
        v.wsum[e] = GK_DADD(v.wsum[e], value);
        v.node_visits[tbase + child] += 1;
    }
    if (lane == 0) v.sims[t] += 1;
}

__global__ void __launch_bounds__(32 * kWarpsPerBlock) puct_expand_backup_kernel(PuctView v, int64_t B, int C,
                                                                                 PuctOptions o, int backup) {
    const int lane = threadIdx.x & 31;
    const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    __shared__ double sum_scratch[kWarpsPerBlock][kSumScratch];
    if (t < B) expand_backup_tree(v, t, C, o, backup, lane, sum_scratch[threadIdx.x >> 5]);
}

struct PuctOutputs {
    int64_t* actions;
    int32_t* visits;
    float* policy;
    float* values;
    int32_t* sims;
    int32_t* evals;
    double* priors;
    float* best_values;
    int32_t* nodes;
    double* root_values;
    uint32_t* status;
};

__global__ void __launch_bounds__(32 * kWarpsPerBlock) puct_finish_kernel(PuctView v, int64_t B, int C, PuctOutputs out) {
    __shared__ double sum_scratch[kWarpsPerBlock][kSumScratch];
    const int lane = threadIdx.x & 31;
    const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    if (t >= B) return;
    const int64_t vtx = t * C, ebase = vtx * GK_ACTIONS, row = t * GK_ACTIONS;
    const gk_bits root = v.node_state[vtx];
    const uint32_t err = v.errors[t];
    if (lane == 0 && err && out.status) atomicOr(out.status, err);
    if (v.node_count[t] == 0) {
        for (int a = lane; a < GK_ACTIONS; a += 32) {
            if (out.visits) out.visits[row + a] = 0;
            if (out.policy) out.policy[row + a] = 0.0f;
            if (out.priors) out.priors[row + a] = 0.0;
        }
        if (lane == 0) {
            if (out.actions) out.actions[t] = -1;
            if (out.values) out.values[t] = terminal_value(root);
            if (out.best_values) out.best_values[t] = 0.0f;
            if (out.sims) out.sims[t] = 0;
            if (out.evals) out.evals[t] = 0;
            if (out.nodes) out.nodes[t] = 0;
            if (out.root_values) out.root_values[t] = (double)terminal_value(root);
        }
        return;
    }
    const int sims = v.sims[t];
    const gk_b96 placements = legal_placements(root);
    const bool expanded = v.expanded[vtx] != 0;
    bool allowed[3];
    allow_bits(v, t, 0, lane, allowed);
    bool use[3];
    double ws[3];
    int best = -1, best_n = 0;
    double best_q = 0.0, best_p = 0.0;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int a = lane + 32 * k;
        use[k] = expanded && a < GK_ACTIONS && allowed[k] && action_legal(placements, true, a);
        ws[k] = 0.0;
        if (a >= GK_ACTIONS) continue;
        const int n = expanded ? v.visits[ebase + a] : 0;
        const double p = expanded ? v.prior[ebase + a] : 0.0;
        if (out.visits) out.visits[row + a] = n;
        if (out.policy) out.policy[row + a] = sims > 0 ? __fdiv_rn((float)n, (float)sims) : 0.0f;
        if (out.priors) out.priors[row + a] = p;
        if (!use[k]) continue;
        ws[k] = v.wsum[ebase + a];
        const double q = n == 0 ? 0.0 : ws[k] / (double)n;
        if (best < 0 || n > best_n || (n == best_n && (q > best_q || (q == best_q && p > best_p)))) {
            best = a;
            best_n = n;
            best_q = q;
            best_p = p;
        }
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
    const double root_sum = ordered_sum(ws, use, sum_scratch[threadIdx.x >> 5], lane);
    if (lane == 0) {
        const double rv = sims > 0 ? root_sum / (double)sims : 0.0;
        if (out.actions) out.actions[t] = best;
        if (out.values) out.values[t] = (float)rv;
        if (out.best_values) out.best_values[t] = (float)best_q;
        if (out.sims) out.sims[t] = sims;
        if (out.evals) out.evals[t] = v.evals[t];
        if (out.nodes) out.nodes[t] = v.node_count[t];
        if (out.root_values) out.root_values[t] = rv;
    }
}

// Injected evaluator (include/gk_common.h): weights and value of tree t's
// leaf, by the tree's warp (lane l computes actions l, l+32, l+64).
__device__ __forceinline__ void hash_eval_tree(const PuctView& v, int64_t t, int lane) {
    if (!v.needs_eval[t]) return;
    uint64_t words[GK_EVAL_WORDS];
    const gk_bits s = v.leaf_bits[t];
    gk_eval_words_from_bits(&s, words);
    const uint64_t h = gk_eval_hash_words(words);
    for (int a = lane; a < GK_ACTIONS; a += 32) v.policy[t * GK_ACTIONS + a] = gk_eval_weight(h, a);
    if (lane == 0) v.leaf_value[t] = gk_eval_value(h);
}

__global__ void __launch_bounds__(32 * kWarpsPerBlock) puct_hash_eval_kernel(PuctView v, int64_t B) {
    const int lane = threadIdx.x & 31;
    const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    if (t < B) hash_eval_tree(v, t, lane);
}

// A whole injected-evaluator search, one warp per tree, in one launch: the
// evaluator is a pure function of the leaf, so trees need no batch-wide step
// and each warp runs root expansion and every simulation back to back. The
// per-tree arithmetic is that of the separate select / evaluate / expand
// kernels; __syncwarp orders each phase's writes before the next phase reads.
// Four blocks per SM: up to 128 registers, so the fused loop does not spill;
// the C3 search (1,024 trees) needs fewer than two blocks per SM.
__global__ void __launch_bounds__(32 * kWarpsPerBlock, 4) puct_search_hash_kernel(PuctView v, int64_t B, int C,
                                                                                  PuctOptions o, int simulations) {
    __shared__ double sum_scratch[kWarpsPerBlock][kSumScratch];
    const int lane = threadIdx.x & 31;
    const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    if (t >= B) return;
    hash_eval_tree(v, t, lane);
    __syncwarp();
    expand_backup_tree(v, t, C, o, 0, lane, sum_scratch[threadIdx.x >> 5]);
    __syncwarp();
    for (int i = 0; i < simulations; ++i) {
        select_tree(v, t, C, o, lane);
        __syncwarp();
        hash_eval_tree(v, t, lane);
        __syncwarp();
        expand_backup_tree(v, t, C, o, 1, lane, sum_scratch[threadIdx.x >> 5]);
        __syncwarp();
    }
}

// ---- root tactical checks ----------------------------------------------------
// GpuPUCT's tactical_checks (python/kingdom_ai/gpu_puct.py:84-161): each legal
// root action is played; an action that ends the game is a win (+1) or a
// loss (-1) for the mover, and one after which the opponent can win with its
// next move is a loss too. The opponent can win at once only by a second
// pass or by taking the last liberty of one of the mover's groups, so only
// those replies are tried, each with the ordinary transition. The root then
// keeps its winning actions if it has any, else its safe ones if it has any,
// else all of them.

// True when the player to move in `next` can win with one move against `mover`.
__device__ bool opponent_wins_next(const gk_bits& next, int mover) {
    const int opponent = gk_actor(&next);
    if (gk_passes(&next) == 1) {
        gk_bits reply = next;
        if (play(reply, GK_PASS) && gk_reason(&reply) != GK_NONE && gk_winner(&reply) == opponent) return true;
    }
    if (gk_stock(&next, opponent) < 1) return false;
    const gk_b96 own = gk_get(&next, mover == 1 ? GK_PLANE_BLACK : GK_PLANE_WHITE);
    const gk_b96 empty = empty_cells(next);
    gk_b96 pending = own;
    while (gk_any(pending)) {
        const gk_b96 group = gk_flood(own, lowest_bit(pending));
        pending = gk_andnot(pending, group);
        const gk_b96 libs = gk_and(gk_neighbours(group), empty);
        if (gk_popc(libs) != 1) continue;
        const int bit = libs.w[0] ? __ffs(libs.w[0]) - 1 : libs.w[1] ? 31 + __ffs(libs.w[1]) : 63 + __ffs(libs.w[2]);
        gk_bits reply = next;
        if (play(reply, gk_bit_cell(bit)) && gk_reason(&reply) == GK_CAPTURE && gk_winner(&reply) == opponent)
            return true;
    }
    return false;
}

// One warp per tree; lane l judges actions l, l+32, l+64 of the root.
__global__ void __launch_bounds__(32 * kWarpsPerBlock) puct_root_tactics_kernel(PuctView v, int64_t B, int C) {
    const int lane = threadIdx.x & 31;
    const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    if (t >= B || v.node_count[t] == 0) return;  // a finished root has no candidates
    const gk_bits root = v.node_state[t * C];
    const int mover = gk_actor(&root);
    const gk_b96 placements = legal_placements(root);
    bool cand[3];
    int outcome[3];
    bool win = false, safe = false;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int a = lane + 32 * k;
        cand[k] = a < GK_ACTIONS && action_legal(placements, true, a);
        outcome[k] = 0;
        if (!cand[k]) continue;
        gk_bits next = root;
        play(next, a);
        if (gk_reason(&next) != GK_NONE) outcome[k] = gk_winner(&next) == mover ? 1 : -1;
        else if (opponent_wins_next(next, mover)) outcome[k] = -1;
        win |= outcome[k] > 0;
        safe |= outcome[k] >= 0;
    }
    win = __any_sync(kFull, win);
    safe = __any_sync(kFull, safe);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const bool keep = cand[k] && (win ? outcome[k] > 0 : safe ? outcome[k] >= 0 : true);
        const uint32_t word = __ballot_sync(kFull, keep);
        if (lane == 0) v.root_allow[t * 3 + k] = word;
    }
}

// ---- root Dirichlet noise ---------------------------------------------------
// Stream per tree: PCG32 (seed, stream_base + tree); draws in gk_random.cuh.
__global__ void puct_noise_kernel(PuctView v, int64_t B, int C, uint64_t seed, uint64_t stream_base, double alpha) {
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < B; t += (int64_t)gridDim.x * blockDim.x) {
        gk_pcg32 r = gk_pcg32_seed(seed, stream_base + (uint64_t)t);
        root_noise(v.node_state[t * C], alpha, r, v.noise + t * GK_ACTIONS, v.root_allow + t * 3);
    }
}

// Ordered compaction of trees whose leaf needs the evaluator (single block).
__global__ void __launch_bounds__(1024) puct_compact_kernel(PuctView v, int64_t B) {
    // Each thread takes kPer consecutive trees, so one pass of the block covers
    // 4,096 trees; the active list keeps increasing tree order.
    constexpr int kPer = 4;
    __shared__ int warp_sums[32];
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int warps = (int)(blockDim.x >> 5);
    for (int64_t base = 0; base < B; base += (int64_t)blockDim.x * kPer) {
        const int64_t t0 = base + (int64_t)threadIdx.x * kPer;
        bool flag[kPer];
        int count = 0;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            flag[j] = t0 + j < B && v.needs_eval[t0 + j] != 0;
            count += flag[j] ? 1 : 0;
        }
        int x = count;  // inclusive prefix over the warp's threads
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(kFull, x, off);
            if (lane >= off) x += y;
        }
        if (lane == 31) warp_sums[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int w = lane < warps ? warp_sums[lane] : 0;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(kFull, w, off);
                if (lane >= off) w += y;
            }
            warp_sums[lane] = w;  // inclusive prefix over warps
        }
        __syncthreads();
        int pos = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + x - count;
#pragma unroll
        for (int j = 0; j < kPer; ++j)
            if (flag[j]) v.active[pos++] = (int32_t)(t0 + j);
        __syncthreads();
        if (threadIdx.x == 0) carry += warp_sums[warps - 1];
        __syncthreads();
    }
    if (threadIdx.x == 0) *v.active_count = carry;
}

inline PuctOptions make_options(const gk_puct_options* o) {
    PuctOptions p;
    p.c_puct = o ? o->c_puct : 1.5;
    p.epsilon = o ? o->dirichlet_epsilon : 0.0;
    p.fpu_enabled = o ? (double)o->fpu_enabled : 0.0;
    p.fpu_reduction = o ? o->fpu_reduction : 0.0;
    return p;
}

inline int warp_grid(int64_t B) {
    const int64_t blocks = (B + kWarpsPerBlock - 1) / kWarpsPerBlock;
    return (int)(blocks < 1 ? 1 : blocks);
}

inline bool valid_ws(const void* ws, int64_t B, int C) { return ws != nullptr && B > 0 && C >= 1 && C < (1 << 24); }

// Blocks of the fused search kernel that fit on the current device at once
// (resident blocks per SM x SMs), or 0 if the query fails.
inline int64_t fused_search_capacity() {
    static int64_t cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cached[dev] == 0) {
        int per_sm = 0, sms = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, puct_search_hash_kernel, 32 * kWarpsPerBlock, 0) !=
                cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return 0;
        cached[dev] = (int64_t)per_sm * sms;
    }
    return cached[dev];
}

}  // namespace gk

using namespace gk;

extern "C" {

size_t gk_puct_workspace_bytes(int64_t batch, int capacity) {
    // Beyond 2^40 nodes (a workspace of petabytes) the byte counts could wrap.
    if (batch <= 0 || capacity < 1 || capacity >= (1 << 24) || batch > ((int64_t)1 << 40) / capacity) return 0;
    return puct_layout(nullptr, batch, capacity, nullptr);
}

int gk_puct_buffers(void* ws, int64_t batch, int capacity, gk_puct_buffers_t* out) {
    if (!valid_ws(ws, batch, capacity) || out == nullptr) return GK_EINVAL;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    out->needs_eval = v.needs_eval;
    out->leaf_bits = reinterpret_cast<uint32_t*>(v.leaf_bits);
    out->leaf_value = v.leaf_value;
    out->policy = v.policy;
    out->noise = v.noise;
    out->active = v.active;
    out->active_count = v.active_count;
    out->errors = v.errors;
    out->leaf = v.leaf;
    out->root_allow = v.root_allow;
    out->node_visits = v.node_visits;
    return 0;
}

int gk_puct_root_tactics(void* ws, int64_t batch, int capacity, void* stream) {
    if (!valid_ws(ws, batch, capacity)) return GK_EINVAL;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    puct_root_tactics_kernel<<<warp_grid(batch), 32 * kWarpsPerBlock, 0, as_stream(stream)>>>(v, batch, capacity);
    return launch_status();
}

int gk_puct_begin(void* ws, int64_t batch, int capacity, const uint32_t* root_bits, void* stream) {
    if (!valid_ws(ws, batch, capacity) || root_bits == nullptr) return GK_EINVAL;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    puct_begin_kernel<<<blocks_for(batch, 256, kSmCount * 8), 256, 0, as_stream(stream)>>>(
        v, batch, capacity, reinterpret_cast<const gk_bits*>(root_bits));
    return launch_status();
}

int gk_puct_noise(void* ws, int64_t batch, int capacity, uint64_t seed, uint64_t stream_base, double alpha,
                  void* stream) {
    if (!valid_ws(ws, batch, capacity) || !(alpha > 0.0)) return GK_EINVAL;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    puct_noise_kernel<<<blocks_for(batch, 128, kSmCount * 8), 128, 0, as_stream(stream)>>>(v, batch, capacity, seed,
                                                                                             stream_base, alpha);
    return launch_status();
}

int gk_puct_hash_eval(void* ws, int64_t batch, int capacity, void* stream) {
    if (!valid_ws(ws, batch, capacity)) return GK_EINVAL;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    puct_hash_eval_kernel<<<warp_grid(batch), 32 * kWarpsPerBlock, 0, as_stream(stream)>>>(v, batch);
    return launch_status();
}

int gk_puct_compact(void* ws, int64_t batch, int capacity, void* stream) {
    if (!valid_ws(ws, batch, capacity)) return GK_EINVAL;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    puct_compact_kernel<<<1, 1024, 0, as_stream(stream)>>>(v, batch);
    return launch_status();
}

int gk_puct_select(void* ws, int64_t batch, int capacity, const gk_puct_options* options, void* stream) {
    if (!valid_ws(ws, batch, capacity) || options == nullptr || !(options->c_puct > 0.0)) return GK_EINVAL;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    puct_select_kernel<<<warp_grid(batch), 32 * kWarpsPerBlock, 0, as_stream(stream)>>>(v, batch, capacity,
                                                                                         make_options(options));
    return launch_status();
}

int gk_puct_expand_backup(void* ws, int64_t batch, int capacity, const gk_puct_options* options, int backup,
                          void* stream) {
    if (!valid_ws(ws, batch, capacity) || options == nullptr) return GK_EINVAL;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    puct_expand_backup_kernel<<<warp_grid(batch), 32 * kWarpsPerBlock, 0, as_stream(stream)>>>(
        v, batch, capacity, make_options(options), backup);
    return launch_status();
}

int gk_puct_finish(void* ws, int64_t batch, int capacity, const gk_puct_results_t* results, void* stream) {
    if (!valid_ws(ws, batch, capacity) || results == nullptr) return GK_EINVAL;
    PuctView v;
    puct_layout(ws, batch, capacity, &v);
    PuctOutputs o{results->actions, results->visits, results->policy, results->values, results->simulations,
                  results->network_evaluations, results->priors, results->best_values, results->nodes,
                  results->root_values, results->status};
    puct_finish_kernel<<<warp_grid(batch), 32 * kWarpsPerBlock, 0, as_stream(stream)>>>(v, batch, capacity, o);
    return launch_status();
}

int gk_puct_search_hash(void* ws, int64_t batch, int simulations, const uint32_t* root_bits,
                        const gk_puct_options* options, const gk_puct_results_t* results, void* stream) {
    if (simulations < 1 || options == nullptr || results == nullptr) return GK_EINVAL;
    const int capacity = simulations + 1;
    int s = gk_puct_begin(ws, batch, capacity, root_bits, stream);
    if (s) return s;
    const int64_t resident = fused_search_capacity();
    if (resident > 0 && 2 * (int64_t)warp_grid(batch) <= resident) {
        // At most half the resident warp slots hold trees: the per-phase
        // launches would be too small to hide their launch gaps, so one
        // launch runs every tree's whole search. (Measured on B200: 1024
        // trees x 800 simulations, 28.7 M vs 16.0 M simulations/s; at 4096
        // trees the per-phase launches win, 52.6 M vs 40.4 M.)
        PuctView v;
        puct_layout(ws, batch, capacity, &v);
        puct_search_hash_kernel<<<warp_grid(batch), 32 * kWarpsPerBlock, 0, as_stream(stream)>>>(
            v, batch, capacity, make_options(options), simulations);
        if ((s = launch_status())) return s;
    } else {
        // Enough trees to fill the GPU: step all trees one phase per launch.
        if ((s = gk_puct_hash_eval(ws, batch, capacity, stream))) return s;
        if ((s = gk_puct_expand_backup(ws, batch, capacity, options, 0, stream))) return s;
        for (int i = 0; i < simulations; ++i) {
            if ((s = gk_puct_select(ws, batch, capacity, options, stream))) return s;
            if ((s = gk_puct_hash_eval(ws, batch, capacity, stream))) return s;
            if ((s = gk_puct_expand_backup(ws, batch, capacity, options, 1, stream))) return s;
        }
    }
    return gk_puct_finish(ws, batch, capacity, results, stream);
}

}  // extern "C"
