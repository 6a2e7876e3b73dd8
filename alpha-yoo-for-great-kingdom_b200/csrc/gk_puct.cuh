// gk_puct.cuh - structure-of-arrays search workspace shared by the PUCT,
// evaluator and self-play translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/gk.h"

namespace gk {

// Per-search device workspace for `batch` trees of `capacity` nodes each.
// Node-major arrays are [batch][capacity], edge arrays [batch][capacity][82].
// Nothing needs clearing between searches: a node's edge rows are written in
// full when it is expanded, and its scalars when it is created.
struct PuctView {
    // tree nodes
    gk_bits* node_state;   // [B*C] packed state of the node
    int32_t* node_visits;  // [B*C]
    float* node_value;     // [B*C] evaluator value of the node (first-play urgency)
    uint8_t* expanded;     // [B*C]
    // edges
    double* prior;         // [B*C*82]
    double* wsum;          // [B*C*82] backed-up value sum from the parent's view
    int32_t* visits;       // [B*C*82]
    int32_t* child;        // [B*C*82] -1 = not created
    // per tree
    int32_t* node_count;   // [B]
    int32_t* leaf;         // [B]
    int32_t* path_len;     // [B]
    int32_t* path_nodes;   // [B*P]
    int32_t* path_actions; // [B*P]
    int32_t* sims;         // [B] completed simulations
    int32_t* evals;        // [B] evaluator calls
    uint32_t* errors;      // [B] GK_ERR_* bits
    // evaluator interface
    uint8_t* needs_eval;   // [B] leaf is a non-terminal unexpanded node
    gk_bits* leaf_bits;    // [B] state to evaluate
    float* leaf_value;     // [B] terminal value, or the evaluator's value
    float* policy;         // [B*82] evaluator policy (probabilities or weights)
    float* noise;          // [B*82] root noise (max-normalised gamma draws)
    int32_t* active;       // [B] compacted indices of trees needing evaluation
    int32_t* active_count; // [1]
    // root candidates: bit (a & 31) of word a >> 5 is set when the root may
    // choose action a (all actions after begin; narrowed by the tactical checks)
    uint32_t* root_allow;  // [B*3]
};

constexpr int kPathCap = GK_MAX_PLIES + 4;  // a path never exceeds the game length

__host__ __device__ inline int path_cap(int capacity) { return capacity < kPathCap ? capacity : kPathCap; }

inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Carves the workspace; returns the total byte size (base may be null).
inline size_t puct_layout(void* base, int64_t B, int C, PuctView* v) {
    const int64_t N = B * (int64_t)C, E = N * GK_ACTIONS, P = B * (int64_t)path_cap(C);
    size_t off = 0;
    char* b = static_cast<char*>(base);
    auto take = [&](size_t bytes) -> void* {
        void* p = b ? b + off : nullptr;
        off = align256(off + bytes);
        return p;
    };
    PuctView t;
    t.node_state = (gk_bits*)take(N * sizeof(gk_bits));
    t.node_visits = (int32_t*)take(N * 4);
    t.node_value = (float*)take(N * 4);
    t.expanded = (uint8_t*)take(N);
    t.prior = (double*)take(E * 8);
    t.wsum = (double*)take(E * 8);
    t.visits = (int32_t*)take(E * 4);
    t.child = (int32_t*)take(E * 4);
    t.node_count = (int32_t*)take(B * 4);
    t.leaf = (int32_t*)take(B * 4);
    t.path_len = (int32_t*)take(B * 4);
    t.path_nodes = (int32_t*)take(P * 4);
    t.path_actions = (int32_t*)take(P * 4);
    t.sims = (int32_t*)take(B * 4);
    t.evals = (int32_t*)take(B * 4);
    t.errors = (uint32_t*)take(B * 4);
    t.needs_eval = (uint8_t*)take(B);
    t.leaf_bits = (gk_bits*)take(B * sizeof(gk_bits));
    t.leaf_value = (float*)take(B * 4);
    t.policy = (float*)take(B * GK_ACTIONS * 4);
    t.noise = (float*)take(B * GK_ACTIONS * 4);
    t.active = (int32_t*)take(B * 4);
    t.active_count = (int32_t*)take(4);
    t.root_allow = (uint32_t*)take(B * 3 * 4);
    if (v) *v = t;
    return off;
}

// Native-network leaf evaluation of a search workspace (gk_net.cu); events,
// when given, are recorded around the tower kernel on `stream`.
int net_evaluate(const gk_net_t* net, void* ws, int64_t batch, int capacity, float* headfeat, uint32_t* status,
                 cudaStream_t stream, cudaEvent_t tower_start, cudaEvent_t tower_stop);

struct PuctOptions {
    double c_puct;
    double epsilon;       // root noise weight (0 disables)
    double fpu_enabled;   // nonzero: unvisited edges start at node value - reduction
    double fpu_reduction;
};

}  // namespace gk
