/*
 * gk_oracle.c - CPU oracle for the batched self-play path (TEST INFRASTRUCTURE).
 *
 * This file restates, in plain C on the int32[170] wire record, the reference
 * algorithms the CUDA path must reproduce bit for bit:
 *   - rules:   State::play        engine/src/State.cpp:92-167
 *              placement_error    engine/src/State.cpp:72-90
 *              score              engine/src/State.cpp:48-61
 *              claim_territory    engine/src/State.cpp:63-70
 *              Board::territory   engine/src/Board.cpp:149-198
 *              collect_group      engine/src/Board.cpp:41-61
 *              wire updates       python/kingdom_ai/gpu_rules.py:185-252
 *   - encoder: encode             mcts/src/BatchedPUCT.cpp:25-50
 *   - search:  PUCT::search       mcts/src/PUCT.cpp:177-268
 *              expand             mcts/src/PUCT.cpp:53-86
 *              select_edge        mcts/src/PUCT.cpp:118-142
 *              better_move        mcts/src/PUCT.cpp:151-157
 * plus the harness definitions that have no reference counterpart (the PCG32
 * playout and position generators and the injected evaluator, which live in
 * include/gk_common.h and are shared with the kernels).
 *
 * Only tests, the smoke check and the benchmark's CPU-baseline leg may load
 * this code; the product never does. Build with -ffp-contract=off.
 */
#include "gk_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "../include/gk_common.h"

/* ---------------------------------------------------------------- rules */

static int nbrs(int i, int* out) {
    int row = i / 9, col = i % 9, n = 0;
    if (row > 0) out[n++] = i - 9;
    if (row < 8) out[n++] = i + 9;
    if (col > 0) out[n++] = i - 1;
    if (col < 8) out[n++] = i + 1;
    return n;
}

static unsigned edge_mask(int i) {
    int row = i / 9, col = i % 9;
    return (row == 0 ? 1u : 0u) | (row == 8 ? 2u : 0u) | (col == 0 ? 4u : 0u) | (col == 8 ? 8u : 0u);
}

/* Board.cpp:41-61: breadth-first group of the stone at `start`. */
static int collect_group(const int32_t* cells, int start, int* queue) {
    int player = cells[start];
    if (player != 1 && player != 2) return 0;
    unsigned char visited[GK_CELLS];
    memset(visited, 0, sizeof visited);
    int length = 1;
    queue[0] = start;
    visited[start] = 1;
    for (int cursor = 0; cursor < length; ++cursor) {
        int nb[4];
        int count = nbrs(queue[cursor], nb);
        for (int n = 0; n < count; ++n) {
            int next = nb[n];
            if (!visited[next] && cells[next] == player) {
                visited[next] = 1;
                queue[length++] = next;
            }
        }
    }
    return length;
}

static int group_has_liberty(const int32_t* cells, const int* group, int length) {
    for (int i = 0; i < length; ++i) {
        int nb[4];
        int count = nbrs(group[i], nb);
        for (int n = 0; n < count; ++n)
            if (cells[nb[n]] == 0) return 1;
    }
    return 0;
}

/* Board.cpp:149-198 with allow_single_edge = true: owners[i] in {0,1,2}. */
static void territory(const int32_t* cells, int* owners) {
    for (int i = 0; i < GK_CELLS; ++i) owners[i] = 0;
    for (int player = 1; player <= 2; ++player) {
        int enemy = 3 - player;
        unsigned char visited[GK_CELLS];
        int queue[GK_CELLS];
        memset(visited, 0, sizeof visited);
        for (int start = 0; start < GK_CELLS; ++start) {
            if (visited[start] || cells[start] != 0) continue;
            int length = 1;
            queue[0] = start;
            visited[start] = 1;
            int contains_enemy = 0, has_own_boundary = 0;
            unsigned edges = 0;
            for (int cursor = 0; cursor < length; ++cursor) {
                int current = queue[cursor];
                edges |= edge_mask(current);
                contains_enemy |= cells[current] == enemy;
                int nb[4];
                int count = nbrs(current, nb);
                for (int n = 0; n < count; ++n) {
                    int next = nb[n];
                    if (cells[next] == player) {
                        has_own_boundary = 1;
                    } else if (cells[next] != 3 && !visited[next]) {
                        visited[next] = 1;
                        queue[length++] = next;
                    }
                }
            }
            if (contains_enemy || !has_own_boundary || edges == 15u) continue;
            for (int i = 0; i < length; ++i)
                if (cells[queue[i]] == 0) owners[queue[i]] = player;
        }
    }
}

static void claim_territory(int32_t* rec) {
    int detected[GK_CELLS];
    territory(rec, detected);
    for (int i = 0; i < GK_CELLS; ++i)
        if (rec[GK_CELLS + i] == 0 && detected[i] != 0) rec[GK_CELLS + i] = detected[i];
}

void gko_score(const int32_t* rec, int* black, int* white) {
    int b = 0, w = 0;
    for (int i = 0; i < GK_CELLS; ++i) {
        if (rec[i] != 0) continue;
        b += rec[GK_CELLS + i] == 1;
        w += rec[GK_CELLS + i] == 2;
    }
    *black = b;
    *white = w;
}

void gko_initial(int32_t* rec, int neutral_cell) {
    memset(rec, 0, GK_STATE_WIDTH * sizeof(int32_t));
    if (neutral_cell >= 0 && neutral_cell < GK_CELLS) rec[neutral_cell] = 3;
    rec[GK_ACTOR] = 1;
    rec[GK_BLACK_STOCK] = GK_STONES;
    rec[GK_WHITE_STOCK] = GK_STONES;
}

int gko_legal(const int32_t* rec, int action) {
    if (rec[GK_REASON] != GK_NONE || action < 0 || action >= GK_ACTIONS) return 0;
    if (action == GK_PASS) return 1;
    int stock = rec[rec[GK_ACTOR] == 1 ? GK_BLACK_STOCK : GK_WHITE_STOCK];
    return rec[action] == 0 && rec[GK_CELLS + action] == 0 && stock > 0;
}

int gko_play(int32_t* rec, int action) {
    if (!gko_legal(rec, action)) return 0;
    int actor = rec[GK_ACTOR], enemy = 3 - actor;
    if (action == GK_PASS) {
        ++rec[GK_PASSES];
        rec[GK_ACTOR] = enemy;
        if (rec[GK_PASSES] == 2) {
            int b, w;
            gko_score(rec, &b, &w);
            rec[GK_REASON] = GK_TWO_PASSES;
            rec[GK_WINNER] = b - w >= 3 ? 1 : 2;
            rec[GK_CAPTURED] = 0;
        }
        return 1;
    }
    rec[action] = actor;
    unsigned char examined[GK_CELLS], captured[GK_CELLS];
    memset(examined, 0, sizeof examined);
    memset(captured, 0, sizeof captured);
    int captured_count = 0;
    int nb[4], group[GK_CELLS];
    int count = nbrs(action, nb);
    for (int n = 0; n < count; ++n) {
        int next = nb[n];
        if (rec[next] != enemy || examined[next]) continue;
        int length = collect_group(rec, next, group);
        int surrounded = !group_has_liberty(rec, group, length);
        for (int i = 0; i < length; ++i) {
            examined[group[i]] = 1;
            if (surrounded) {
                captured[group[i]] = 1;
                ++captured_count;
            }
        }
    }
    int suicide = 0;
    if (captured_count == 0) {
        int length = collect_group(rec, action, group);
        suicide = !group_has_liberty(rec, group, length);
    }
    --rec[actor == 1 ? GK_BLACK_STOCK : GK_WHITE_STOCK];
    rec[GK_PASSES] = 0;
    rec[GK_ACTOR] = enemy;
    if (captured_count > 0) {
        for (int i = 0; i < GK_CELLS; ++i)
            if (captured[i]) rec[i] = 0;
        rec[GK_REASON] = GK_CAPTURE;
        rec[GK_WINNER] = actor;
        rec[GK_CAPTURED] = captured_count;
    } else if (suicide) {
        rec[GK_REASON] = GK_SUICIDE;
        rec[GK_WINNER] = enemy;
        rec[GK_CAPTURED] = 0;
    } else {
        claim_territory(rec);
    }
    return 1;
}

void gko_encode(const int32_t* rec, float* features, uint8_t* mask) {
    int actor = rec[GK_ACTOR], enemy = 3 - actor;
    int own_stock = rec[actor == 1 ? GK_BLACK_STOCK : GK_WHITE_STOCK];
    int enemy_stock = rec[actor == 1 ? GK_WHITE_STOCK : GK_BLACK_STOCK];
    float own_remaining = (float)((double)own_stock / 41.0);
    float enemy_remaining = (float)((double)enemy_stock / 41.0);
    float passes = (float)((double)rec[GK_PASSES] / 2.0);
    for (int a = 0; a < GK_ACTIONS; ++a) mask[a] = (uint8_t)gko_legal(rec, a);
    for (int i = 0; i < GK_CELLS; ++i) {
        features[0 * 81 + i] = rec[i] == actor ? 1.0f : 0.0f;
        features[1 * 81 + i] = rec[i] == enemy ? 1.0f : 0.0f;
        features[2 * 81 + i] = rec[i] == 3 ? 1.0f : 0.0f;
        features[3 * 81 + i] = rec[GK_CELLS + i] == actor ? 1.0f : 0.0f;
        features[4 * 81 + i] = rec[GK_CELLS + i] == enemy ? 1.0f : 0.0f;
        features[5 * 81 + i] = actor == 1 ? 1.0f : 0.0f;
        features[6 * 81 + i] = own_remaining;
        features[7 * 81 + i] = enemy_remaining;
        features[8 * 81 + i] = passes;
        features[9 * 81 + i] = mask[i] ? 1.0f : 0.0f;
    }
}

void gko_play_batch(int32_t* recs, const int32_t* actions, uint8_t* accepted, int64_t n) {
    for (int64_t i = 0; i < n; ++i) accepted[i] = (uint8_t)gko_play(recs + i * GK_STATE_WIDTH, actions[i]);
}

void gko_encode_batch(const int32_t* recs, float* features, uint8_t* masks, int64_t n) {
    for (int64_t i = 0; i < n; ++i)
        gko_encode(recs + i * GK_STATE_WIDTH, features + i * GK_FEATURES, masks + i * GK_ACTIONS);
}

/* ------------------------------------------------------ random playouts */

/* Legal actions in index order (placements by row*9+col, then pass), the
 * order of State::legal_moves (engine/src/State.cpp:183-198). */
static int legal_list(const int32_t* rec, int* out) {
    int n = 0;
    for (int a = 0; a < GK_ACTIONS; ++a)
        if (gko_legal(rec, a)) out[n++] = a;
    return n;
}

static int cpp_reason(int wire) {
    return wire == GK_CAPTURE ? GK_CPP_CAPTURE
         : wire == GK_SUICIDE ? GK_CPP_SUICIDE
         : wire == GK_TWO_PASSES ? GK_CPP_TWO_PASSES
                                 : GK_CPP_NONE;
}

void gko_random_playout(uint64_t seed, uint64_t game, int neutral_cell, int8_t* board, int32_t* info) {
    int32_t rec[GK_STATE_WIDTH];
    int legal[GK_ACTIONS];
    gk_pcg32 rng = gk_pcg32_seed(seed, game);
    gko_initial(rec, neutral_cell);
    int plies = 0;
    while (rec[GK_REASON] == GK_NONE) {
        int n = legal_list(rec, legal);
        int j = (int)gk_pcg32_bounded(&rng, (uint32_t)n);
        gko_play(rec, legal[j]);
        ++plies;
    }
    for (int i = 0; i < GK_CELLS; ++i) board[i] = (int8_t)rec[i];
    int b, w;
    gko_score(rec, &b, &w);
    info[0] = rec[GK_WINNER];
    info[1] = cpp_reason(rec[GK_REASON]);
    info[2] = b;
    info[3] = w;
    info[4] = plies;
}

void gko_random_playouts(uint64_t seed, uint64_t first_game, int64_t n, int neutral_cell, int8_t* boards,
                         int32_t* infos) {
    for (int64_t i = 0; i < n; ++i)
        gko_random_playout(seed, first_game + (uint64_t)i, neutral_cell, boards + i * GK_CELLS, infos + i * 5);
}

/* Position generator: stream (seed, index); draw k in [0, 60], play k uniform
 * legal moves from the default start; if the game ends within those k moves,
 * draw a fresh k from the same stream and restart (at most 64 attempts, then
 * the start position). */
void gko_gen_position(uint64_t seed, uint64_t index, int32_t* rec) {
    int legal[GK_ACTIONS];
    gk_pcg32 rng = gk_pcg32_seed(seed, index);
    for (int attempt = 0; attempt < 64; ++attempt) {
        int k = (int)gk_pcg32_bounded(&rng, 61u);
        gko_initial(rec, 40);
        int ok = 1;
        for (int i = 0; i < k; ++i) {
            int n = legal_list(rec, legal);
            int j = (int)gk_pcg32_bounded(&rng, (uint32_t)n);
            gko_play(rec, legal[j]);
            if (rec[GK_REASON] != GK_NONE) {
                ok = 0;
                break;
            }
        }
        if (ok) return;
    }
    gko_initial(rec, 40);
}

void gko_gen_positions(uint64_t seed, uint64_t first, int64_t n, int32_t* recs) {
    for (int64_t i = 0; i < n; ++i) gko_gen_position(seed, first + (uint64_t)i, recs + i * GK_STATE_WIDTH);
}

void gko_eval(const int32_t* rec, float* weights, float* value) {
    uint64_t words[GK_EVAL_WORDS];
    gk_eval_words_from_record(rec, words);
    uint64_t h = gk_eval_hash_words(words);
    for (int a = 0; a < GK_ACTIONS; ++a) weights[a] = gk_eval_weight(h, a);
    *value = gk_eval_value(h);
}

/* ------------------------------------------------------------------ PUCT */

typedef struct {
    int move;
    double prior;
    int64_t visits;
    double value_sum;
    int child; /* -1: none */
} o_edge;

typedef struct {
    int player;
    int64_t visits;
    int expanded;
    int nedges;
    o_edge* edges;
} o_node;

static double edge_value(const o_edge* e) { return e->visits == 0 ? 0.0 : e->value_sum / (double)e->visits; }

/* Evaluator used by the search: 0 = injected hash evaluator, 1 = uniform
 * (weight 1 for every action, value 0 - what a zero-weight network gives). */
static __thread int g_uniform_evaluator = 0;
/* Root candidates of a search with tactical checks (NULL: every legal action). */
static __thread const uint8_t* g_root_allow = NULL;

/* PUCT.cpp:53-86 */
static int expand(o_node* node, const int32_t* rec, o_edge* storage, double* leaf_value, int64_t* evaluations,
                  const uint8_t* allow) {
    int moves[GK_ACTIONS];
    int n = legal_list(rec, moves);
    if (allow) {
        int kept = 0;
        for (int i = 0; i < n; ++i)
            if (allow[moves[i]]) moves[kept++] = moves[i];
        n = kept;
    }
    if (n == 0) return -1;
    float w[GK_ACTIONS], v;
    if (g_uniform_evaluator) {
        for (int a = 0; a < GK_ACTIONS; ++a) w[a] = 1.0f;
        v = 0.0f;
    } else {
        gko_eval(rec, w, &v);
    }
    ++*evaluations;
    if (!isfinite(v) || v < -1.0f || v > 1.0f) return -2;
    for (int a = 0; a < GK_ACTIONS; ++a)
        if (!isfinite(w[a]) || w[a] < 0.0f) return -2;
    double largest = 0.0;
    for (int i = 0; i < n; ++i) largest = fmax(largest, (double)w[moves[i]]);
    if (largest == 0.0) return -2;
    double total = 0.0;
    for (int i = 0; i < n; ++i) total += (double)w[moves[i]] / largest;
    node->edges = storage;
    node->nedges = n;
    for (int i = 0; i < n; ++i) {
        storage[i].move = moves[i];
        storage[i].prior = ((double)w[moves[i]] / largest) / total;
        storage[i].visits = 0;
        storage[i].value_sum = 0.0;
        storage[i].child = -1;
    }
    node->expanded = 1;
    *leaf_value = (double)v;
    return 0;
}

/* PUCT.cpp:118-142 */
static int select_edge(const o_node* node, double c_puct) {
    double parent_scale = sqrt((double)node->visits);
    int best = 0;
    double best_score = -INFINITY;
    for (int i = 0; i < node->nedges; ++i) {
        const o_edge* e = &node->edges[i];
        double exploration = e->prior * parent_scale / (1.0 + (double)e->visits);
        double score = c_puct >= 1.0 ? edge_value(e) / c_puct + exploration : edge_value(e) + c_puct * exploration;
        const o_edge* prev = &node->edges[best];
        if (score > best_score ||
            (score == best_score && (e->prior > prev->prior || (e->prior == prev->prior && e->move < prev->move)))) {
            best = i;
            best_score = score;
        }
    }
    return best;
}

static double terminal_value(const int32_t* rec) { return rec[GK_WINNER] == rec[GK_ACTOR] ? 1.0 : -1.0; }

int gko_puct_search(const int32_t* root, int simulations, double c_puct, int32_t* visits, double* priors,
                    int32_t* stats, double* values) {
    for (int a = 0; a < GK_ACTIONS; ++a) {
        visits[a] = 0;
        priors[a] = 0.0;
    }
    stats[0] = -1;
    stats[1] = 0;
    stats[2] = 0;
    stats[3] = 0;
    values[1] = 0.0;
    if (root[GK_REASON] != GK_NONE) {
        values[0] = terminal_value(root);
        return 0;
    }
    int capacity = simulations + 1;
    o_node* tree = (o_node*)calloc((size_t)capacity, sizeof(o_node));
    o_edge* pool = (o_edge*)malloc((size_t)capacity * GK_ACTIONS * sizeof(o_edge));
    int* path_node = (int*)malloc((size_t)capacity * sizeof(int));
    int* path_edge = (int*)malloc((size_t)capacity * sizeof(int));
    int size = 1, status = 0;
    int64_t evaluations = 0;
    double ignored;
    tree[0].player = root[GK_ACTOR];
    if (expand(&tree[0], root, pool, &ignored, &evaluations, g_root_allow) != 0) {
        status = -2;
        goto done;
    }
    int64_t completed = 0;
    for (int iteration = 0; iteration < simulations; ++iteration) {
        int32_t sim[GK_STATE_WIDTH];
        memcpy(sim, root, sizeof sim);
        int node = 0, depth = 0;
        double leaf_value = 0.0;
        for (;;) {
            if (sim[GK_REASON] != GK_NONE) {
                leaf_value = terminal_value(sim);
                break;
            }
            if (!tree[node].expanded) {
                if (expand(&tree[node], sim, pool + (size_t)node * GK_ACTIONS, &leaf_value, &evaluations,
                           node == 0 ? g_root_allow : NULL) != 0) {
                    status = -2;
                    goto done;
                }
                break;
            }
            int e = select_edge(&tree[node], c_puct);
            o_edge* edge = &tree[node].edges[e];
            if (!gko_play(sim, edge->move)) {
                status = -1;
                goto done;
            }
            path_node[depth] = node;
            path_edge[depth] = e;
            ++depth;
            if (edge->child < 0) {
                if (size >= capacity) {
                    status = -1;
                    goto done;
                }
                edge->child = size;
                tree[size].player = sim[GK_ACTOR];
                ++size;
            }
            node = edge->child;
        }
        ++tree[0].visits;
        for (int d = 0; d < depth; ++d) {
            o_edge* edge = &tree[path_node[d]].edges[path_edge[d]];
            double value = tree[path_node[d]].player == sim[GK_ACTOR] ? leaf_value : -leaf_value;
            ++edge->visits;
            edge->value_sum += value;
            ++tree[edge->child].visits;
        }
        ++completed;
    }
    {
        double root_sum = 0.0;
        const o_edge* best = NULL;
        for (int i = 0; i < tree[0].nedges; ++i) {
            const o_edge* e = &tree[0].edges[i];
            visits[e->move] = (int32_t)e->visits;
            priors[e->move] = e->prior;
            root_sum += e->value_sum;
            if (best == NULL) {
                best = e;
                continue;
            }
            /* PUCT.cpp:151-157 over moves sorted by index (edge order). */
            int better;
            if (e->visits != best->visits) better = e->visits > best->visits;
            else if (edge_value(e) != edge_value(best)) better = edge_value(e) > edge_value(best);
            else if (e->prior != best->prior) better = e->prior > best->prior;
            else better = e->move < best->move;
            if (better) best = e;
        }
        stats[0] = best ? best->move : -1;
        stats[1] = (int32_t)completed;
        stats[2] = size;
        stats[3] = (int32_t)evaluations;
        values[0] = root_sum / (double)completed;
        values[1] = best ? edge_value(best) : 0.0;
    }
done:
    free(tree);
    free(pool);
    free(path_node);
    free(path_edge);
    return status;
}

/* Root tactical checks of the GPU search (python/kingdom_ai/gpu_puct.py:84-161).
 * After the mover's action the opponent can win at once only by a second
 * pass or by taking the last liberty of one of the mover's groups; each
 * candidate reply is checked with the ordinary transition. */
static int opponent_wins_next(const int32_t* next, int mover) {
    const int opponent = next[GK_ACTOR];
    int32_t reply[GK_STATE_WIDTH];
    if (next[GK_PASSES] == 1) {
        memcpy(reply, next, sizeof reply);
        if (gko_play(reply, GK_PASS) && reply[GK_REASON] != GK_NONE && reply[GK_WINNER] == opponent) return 1;
    }
    if (next[opponent == 1 ? GK_BLACK_STOCK : GK_WHITE_STOCK] < 1) return 0;
    unsigned char seen[GK_CELLS];
    memset(seen, 0, sizeof seen);
    int group[GK_CELLS];
    for (int point = 0; point < GK_CELLS; ++point) {
        if (next[point] != mover || seen[point]) continue;
        const int length = collect_group(next, point, group);
        int liberty = -1, several = 0;
        for (int i = 0; i < length; ++i) {
            seen[group[i]] = 1;
            int nb[4];
            const int count = nbrs(group[i], nb);
            for (int j = 0; j < count; ++j) {
                if (next[nb[j]] != 0) continue;
                if (liberty < 0) liberty = nb[j];
                else if (liberty != nb[j]) several = 1;
            }
        }
        if (several || liberty < 0) continue;
        memcpy(reply, next, sizeof reply);
        if (gko_play(reply, liberty) && reply[GK_REASON] == GK_CAPTURE && reply[GK_WINNER] == opponent) return 1;
    }
    return 0;
}

/* outcome[a] = +1 (the mover wins at once), -1 (loses at once or the
 * opponent can win with its next move), 0 otherwise or illegal; allow[a] =
 * the legal actions narrowed to the wins if any, else to the safe ones if
 * any, else all of them. */
void gko_root_tactics(const int32_t* rec, int8_t* outcome, uint8_t* allow) {
    int winning = 0, safe = 0;
    for (int a = 0; a < GK_ACTIONS; ++a) {
        outcome[a] = 0;
        allow[a] = (uint8_t)gko_legal(rec, a);
        if (!allow[a]) continue;
        int32_t next[GK_STATE_WIDTH];
        memcpy(next, rec, sizeof next);
        gko_play(next, a);
        if (next[GK_REASON] != GK_NONE) outcome[a] = next[GK_WINNER] == rec[GK_ACTOR] ? 1 : -1;
        else if (opponent_wins_next(next, rec[GK_ACTOR])) outcome[a] = -1;
        winning |= outcome[a] > 0;
        safe |= outcome[a] >= 0;
    }
    for (int a = 0; a < GK_ACTIONS; ++a) {
        if (winning) allow[a] = allow[a] && outcome[a] > 0;
        else if (safe) allow[a] = allow[a] && outcome[a] >= 0;
    }
}

/* The injected-evaluator search with the root narrowed by gko_root_tactics
 * (uniform = 1: the uniform evaluator). */
int gko_puct_search_tactics(const int32_t* rec, int simulations, double c_puct, int uniform, int32_t* visits,
                            double* priors, int32_t* stats, double* values) {
    int8_t outcome[GK_ACTIONS];
    uint8_t allow[GK_ACTIONS];
    gko_root_tactics(rec, outcome, allow);
    g_root_allow = allow;
    g_uniform_evaluator = uniform ? 1 : 0;
    int status = gko_puct_search(rec, simulations, c_puct, visits, priors, stats, values);
    g_uniform_evaluator = 0;
    g_root_allow = NULL;
    return status;
}

int gko_puct_search_uniform(const int32_t* rec, int simulations, double c_puct, int32_t* visits, double* priors,
                            int32_t* stats, double* values) {
    g_uniform_evaluator = 1;
    int status = gko_puct_search(rec, simulations, c_puct, visits, priors, stats, values);
    g_uniform_evaluator = 0;
    return status;
}

typedef struct {
    const int32_t* recs;
    int64_t begin, end;
    int simulations;
    double c_puct;
    int32_t* visits;
    int32_t* best;
    double* root_values;
    int status;
} batch_job;

static void* batch_worker(void* arg) {
    batch_job* job = (batch_job*)arg;
    double priors[GK_ACTIONS];
    for (int64_t i = job->begin; i < job->end; ++i) {
        int32_t stats[4];
        double values[2];
        int s = gko_puct_search(job->recs + i * GK_STATE_WIDTH, job->simulations, job->c_puct,
                                job->visits + i * GK_ACTIONS, priors, stats, values);
        if (s != 0) job->status = s;
        job->best[i] = stats[0];
        job->root_values[i] = values[0];
    }
    return NULL;
}

int gko_puct_search_batch(const int32_t* recs, int64_t n, int simulations, double c_puct, int32_t* visits,
                          int32_t* best, double* root_values, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    batch_job jobs[256];
    int64_t per = (n + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        int64_t b = (int64_t)t * per, e = b + per < n ? b + per : n;
        if (b >= e) break;
        jobs[t] = (batch_job){recs, b, e, simulations, c_puct, visits, best, root_values, 0};
        pthread_create(&tid[t], NULL, batch_worker, &jobs[t]);
        ++started;
    }
    int status = 0;
    for (int t = 0; t < started; ++t) {
        pthread_join(tid[t], NULL);
        if (jobs[t].status) status = jobs[t].status;
    }
    return status;
}

/* ------------------------------------------------------------ self-play */
/* One self-play game as the device engine plays it with the injected
 * evaluator and no root noise. Per ply (python/kingdom_ai/gpu_training.py:
 * 59-87): search, record the visit shares n / simulations as floats (:69-70),
 * then move. At temperature 0 the move is the search's best action (:76-77);
 * otherwise it is drawn with weights exp((log n - log n_max) / T) (:28-37),
 * which are the visit counts themselves at T = 1. The draw uses the PCG32
 * stream (sample_seed ^ GKO_SAMPLE_SALT, game * 256 + ply): at T = 1 an
 * integer u = bounded(simulations) picks the first action whose running visit
 * total exceeds u (exact integer arithmetic); at other temperatures
 * u = uniform01 * total picks the first positive-weight action whose running
 * weight total exceeds u. With `tactics` each search narrows its root by the
 * root tactical checks (gko_root_tactics), as the engine does with
 * tactical_checks set. */
#define GKO_SAMPLE_SALT 0x9E3779B97F4A7C15ULL

static double o_uniform01(gk_pcg32* r) {
    uint64_t hi = gk_pcg32_next(r) >> 5, lo = gk_pcg32_next(r) >> 6; /* 27 + 26 bits */
    return ((double)(hi * 67108864ull + lo) + 0.5) * (1.0 / 9007199254740992.0);
}

int gko_selfplay_hash_game(uint64_t sample_seed, uint64_t game, int neutral_cell, int simulations, double c_puct,
                           int temperature_moves, double temperature, double final_temperature, int tactics,
                           uint8_t* actions, float* policy, int32_t* rec) {
    gko_initial(rec, neutral_cell);
    for (int ply = 0; ply < GK_MAX_PLIES + 2; ++ply) {
        if (rec[GK_REASON] != GK_NONE) return ply;
        int32_t visits[GK_ACTIONS], stats[4];
        double priors[GK_ACTIONS], values[2];
        int status = tactics ? gko_puct_search_tactics(rec, simulations, c_puct, 0, visits, priors, stats, values)
                             : gko_puct_search(rec, simulations, c_puct, visits, priors, stats, values);
        if (status != 0) return status < 0 ? status : -1;
        const int sims = stats[1];
        for (int a = 0; a < GK_ACTIONS; ++a)
            policy[(size_t)ply * GK_ACTIONS + a] = sims > 0 ? (float)visits[a] / (float)sims : 0.0f;
        const double t = ply < temperature_moves ? temperature : final_temperature;
        int action = stats[0];
        if (t != 0.0 && sims > 0) {
            gk_pcg32 r = gk_pcg32_seed(sample_seed ^ GKO_SAMPLE_SALT, game * 256u + (uint64_t)ply);
            if (t == 1.0) {
                int64_t u = (int64_t)gk_pcg32_bounded(&r, (uint32_t)sims), run = 0;
                for (int a = 0; a < GK_ACTIONS; ++a) {
                    run += visits[a];
                    if (visits[a] > 0 && u < run) {
                        action = a;
                        break;
                    }
                }
            } else {
                int nmax = 0;
                for (int a = 0; a < GK_ACTIONS; ++a) nmax = visits[a] > nmax ? visits[a] : nmax;
                double w[GK_ACTIONS], total = 0.0;
                for (int a = 0; a < GK_ACTIONS; ++a) {
                    w[a] = visits[a] > 0 ? exp((log((double)visits[a]) - log((double)nmax)) / t) : 0.0;
                    total += w[a];
                }
                double u = o_uniform01(&r) * total, run = 0.0;
                for (int a = 0; a < GK_ACTIONS; ++a) {
                    const double before = run;
                    run += w[a];
                    if (w[a] > 0.0 && u >= before && u < run) {
                        action = a;
                        break;
                    }
                }
            }
        }
        if (action < 0 || !gko_play(rec, action)) return -1;
        actions[ply] = (uint8_t)action;
    }
    return rec[GK_REASON] != GK_NONE ? GK_MAX_PLIES + 2 : -1;
}

typedef struct {
    uint64_t sample_seed, first_game;
    int64_t begin, end;
    int neutral_cell, simulations, temperature_moves, tactics;
    double c_puct, temperature, final_temperature;
    uint8_t* actions;
    float* policy;
    int32_t* recs;
    int32_t* plies;
} selfplay_job;

static void* selfplay_worker(void* arg) {
    selfplay_job* j = (selfplay_job*)arg;
    for (int64_t i = j->begin; i < j->end; ++i)
        j->plies[i] = gko_selfplay_hash_game(j->sample_seed, j->first_game + (uint64_t)i, j->neutral_cell,
                                             j->simulations, j->c_puct, j->temperature_moves, j->temperature,
                                             j->final_temperature, j->tactics, j->actions + i * (GK_MAX_PLIES + 2),
                                             j->policy + i * (int64_t)(GK_MAX_PLIES + 2) * GK_ACTIONS,
                                             j->recs + i * GK_STATE_WIDTH);
    return NULL;
}

void gko_selfplay_hash_games(uint64_t sample_seed, uint64_t first_game, int64_t n, int neutral_cell,
                             int simulations, double c_puct, int temperature_moves, double temperature,
                             double final_temperature, int tactics, uint8_t* actions, float* policy, int32_t* recs,
                             int32_t* plies, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    selfplay_job jobs[256];
    int64_t per = (n + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        int64_t b = (int64_t)t * per, e = b + per < n ? b + per : n;
        if (b >= e) break;
        jobs[t] = (selfplay_job){sample_seed, first_game, b, e, neutral_cell, simulations, temperature_moves,
                                 tactics, c_puct, temperature, final_temperature, actions, policy, recs, plies};
        pthread_create(&tid[t], NULL, selfplay_worker, &jobs[t]);
        ++started;
    }
    for (int t = 0; t < started; ++t) pthread_join(tid[t], NULL);
}

/* ----------------------------------------------------------- BatchedPUCT */
/* The evaluation searcher of mcts/src/BatchedPUCT.cpp restated: leaf batches
 * gathered under a virtual loss of one per pending simulation (143-227), the
 * subtree promotion of advance() (290-326) and the search loop with its
 * per-search statistics (328-442). Selection is the reference's depth-first
 * walk: at each node the edges are tried in score order and a subtree that
 * holds only pending leaves is skipped for the next-scored edge. The tree is
 * one growable node array; edges are the legal actions in action order. */

typedef struct {
    int move;
    double prior;
    int64_t visits;
    double value_sum;
    int64_t reserved;
    int64_t child; /* -1: none */
} ob_edge;

typedef struct {
    int32_t rec[GK_STATE_WIDTH];
    int64_t visits;
    int64_t reserved;
    int expanded;
    int pending;
    int nedges;
    ob_edge edges[GK_ACTIONS];
} ob_node;

typedef struct {
    int64_t node;
    int depth;
    int64_t path_node[GK_MAX_PLIES + 4];
    int path_edge[GK_MAX_PLIES + 4];
} ob_leaf;

typedef struct {
    int64_t simulations;
    double c_puct;
    int64_t leaf_batch;
    int reuse;
    int evaluator;
    ob_node* tree;
    int64_t size, cap;
    int64_t stats[GKO_BPUCT_STATS];
} ob_search;

enum { OB_EVALS, OB_BATCHES, OB_MAX_BATCH, OB_REUSED, OB_INHERITED, OB_ADVANCES, OB_REUSE_HITS };

void* gko_bpuct_new(int64_t simulations, double c_puct, int64_t leaf_batch, int reuse, int evaluator) {
    if (simulations < 1 || !(c_puct > 0.0) || !isfinite(c_puct) || leaf_batch < 1) return NULL;
    ob_search* s = (ob_search*)calloc(1, sizeof(ob_search));
    if (!s) return NULL;
    s->simulations = simulations;
    s->c_puct = c_puct;
    s->leaf_batch = leaf_batch;
    s->reuse = reuse != 0;
    s->evaluator = evaluator;
    return s;
}

void gko_bpuct_free(void* h) {
    ob_search* s = (ob_search*)h;
    if (!s) return;
    free(s->tree);
    free(s);
}

void gko_bpuct_clear(void* h) { ((ob_search*)h)->size = 0; }

int64_t gko_bpuct_size(const void* h) { return ((const ob_search*)h)->size; }

void gko_bpuct_stats(const void* h, int64_t* out) {
    for (int i = 0; i < GKO_BPUCT_STATS; ++i) out[i] = ((const ob_search*)h)->stats[i];
}

static int64_t ob_push(ob_search* s, const int32_t* rec) {
    if (s->size == s->cap) {
        int64_t cap = s->cap ? 2 * s->cap : 64;
        ob_node* grown = (ob_node*)realloc(s->tree, (size_t)cap * sizeof(ob_node));
        if (!grown) return -1;
        s->tree = grown;
        s->cap = cap;
    }
    ob_node* n = &s->tree[s->size];
    memcpy(n->rec, rec, sizeof n->rec);
    n->visits = 0;
    n->reserved = 0;
    n->expanded = 0;
    n->pending = 0;
    n->nedges = 0;
    return s->size++;
}

/* BatchedPUCT.cpp:52-67: every field that defines a position, rules and result included. */
static int ob_same_state(const int32_t* a, const int32_t* b) {
    for (int i = 0; i <= GK_CAPTURED; ++i)
        if (a[i] != b[i]) return 0;
    return 1;
}

/* The evaluators of the search: the injected hash evaluator, a uniform one,
 * and the fixed evaluator of the reference's own tests
 * (tests/batched_puct_test.cpp:21-28: weight (i + 1) / 81 on cell i, none on
 * pass; value 0.25 for Black to play, -0.5 for White). */
static void ob_evaluate(int kind, const int32_t* rec, double* w, double* v) {
    if (kind == GKO_EVAL_UNIFORM) {
        for (int a = 0; a < GK_ACTIONS; ++a) w[a] = 1.0;
        *v = 0.0;
    } else if (kind == GKO_EVAL_RAMP) {
        for (int a = 0; a < GK_CELLS; ++a) w[a] = (double)(a + 1) / 81.0;
        w[GK_PASS] = 0.0;
        *v = rec[GK_ACTOR] == 1 ? 0.25 : -0.5;
    } else {
        float wf[GK_ACTIONS], vf;
        gko_eval(rec, wf, &vf);
        for (int a = 0; a < GK_ACTIONS; ++a) w[a] = (double)wf[a];
        *v = (double)vf;
    }
}

/* BatchedPUCT.cpp:72-81 (evaluation checks) and 229-250 (edges). */
static int ob_expand(ob_node* n, const double* w, double v) {
    if (!isfinite(v) || v < -1.0 || v > 1.0) return GKO_BPUCT_BAD_VALUE;
    for (int a = 0; a < GK_ACTIONS; ++a)
        if (!isfinite(w[a]) || w[a] < 0.0) return GKO_BPUCT_BAD_POLICY;
    int moves[GK_ACTIONS];
    const int count = legal_list(n->rec, moves);
    double largest = 0.0;
    for (int i = 0; i < count; ++i) largest = fmax(largest, w[moves[i]]);
    if (largest == 0.0) return GKO_BPUCT_ZERO_POLICY;
    double total = 0.0;
    for (int i = 0; i < count; ++i) total += w[moves[i]] / largest;
    for (int i = 0; i < count; ++i) {
        ob_edge* e = &n->edges[i];
        e->move = moves[i];
        e->prior = (w[moves[i]] / largest) / total;
        e->visits = 0;
        e->value_sum = 0.0;
        e->reserved = 0;
        e->child = -1;
    }
    n->nedges = count;
    n->expanded = 1;
    return 0;
}

/* BatchedPUCT.cpp:143-196. Returns 1 with the leaf and its path, 0 when
 * every path below `node` ends in a pending leaf, negative on failure. */
static int ob_select(ob_search* s, int64_t node, ob_leaf* leaf) {
    if (s->tree[node].pending) return 0;
    if (!s->tree[node].expanded || s->tree[node].rec[GK_REASON] != GK_NONE) {
        leaf->node = node;
        return 1;
    }
    const int count = s->tree[node].nedges;
    if (count == 0) return GKO_BPUCT_LOGIC;
    uint8_t tried[GK_ACTIONS] = {0};
    for (int attempt = 0; attempt < count; ++attempt) {
        const ob_node* n = &s->tree[node];
        const double scale = sqrt((double)n->visits + (double)n->reserved);
        int best = -1;
        double best_score = -INFINITY;
        for (int i = 0; i < count; ++i) {
            if (tried[i]) continue;
            const ob_edge* e = &n->edges[i];
            const double effective = (double)e->visits + (double)e->reserved;
            const double value = effective == 0.0 ? 0.0 : (e->value_sum - (double)e->reserved) / effective;
            const double exploration = e->prior * scale / (1.0 + effective);
            const double score = s->c_puct >= 1.0 ? value / s->c_puct + exploration : value + s->c_puct * exploration;
            if (best < 0 || score > best_score ||
                (score == best_score && (e->prior > n->edges[best].prior ||
                                         (e->prior == n->edges[best].prior && e->move < n->edges[best].move)))) {
                best = i;
                best_score = score;
            }
        }
        if (best < 0) return 0;
        tried[best] = 1;
        int64_t child = s->tree[node].edges[best].child;
        if (child < 0) {
            int32_t next[GK_STATE_WIDTH];
            memcpy(next, s->tree[node].rec, sizeof next);
            if (!gko_play(next, s->tree[node].edges[best].move)) return GKO_BPUCT_LOGIC;
            child = ob_push(s, next);
            if (child < 0) return GKO_BPUCT_LOGIC;
            s->tree[node].edges[best].child = child;
        }
        if (leaf->depth >= GK_MAX_PLIES + 4) return GKO_BPUCT_LOGIC;
        leaf->path_node[leaf->depth] = node;
        leaf->path_edge[leaf->depth] = best;
        ++leaf->depth;
        const int found = ob_select(s, child, leaf);
        if (found != 0) return found;
        --leaf->depth;
    }
    return 0;
}

/* BatchedPUCT.cpp:198-227 */
static void ob_reserve(ob_search* s, const ob_leaf* l, int64_t delta) {
    s->tree[l->node].pending = delta > 0;
    s->tree[0].reserved += delta;
    for (int d = 0; d < l->depth; ++d) {
        ob_edge* e = &s->tree[l->path_node[d]].edges[l->path_edge[d]];
        e->reserved += delta;
        s->tree[e->child].reserved += delta;
    }
}

static void ob_backup(ob_search* s, const ob_leaf* l, double value) {
    ++s->tree[0].visits;
    const int player = s->tree[l->node].rec[GK_ACTOR];
    for (int d = 0; d < l->depth; ++d) {
        ob_node* parent = &s->tree[l->path_node[d]];
        ob_edge* e = &parent->edges[l->path_edge[d]];
        e->value_sum += parent->rec[GK_ACTOR] == player ? value : -value;
        ++e->visits;
        ++s->tree[e->child].visits;
    }
}

static double ob_terminal_value(const int32_t* rec) { return rec[GK_WINNER] == rec[GK_ACTOR] ? 1.0 : -1.0; }

static void ob_note_batch(ob_search* s, int64_t rows) {
    s->stats[OB_EVALS] += rows;
    s->stats[OB_BATCHES] += 1;
    if (rows > s->stats[OB_MAX_BATCH]) s->stats[OB_MAX_BATCH] = rows;
}

/* BatchedPUCT.cpp:328-442. Outputs per action: visits and mean value gained
 * in this search, priors, legal (the root's edges); info = {best action,
 * simulations, nodes, network evaluations}; values = {root value, best value}.
 * Any failure clears the tree and returns a negative GKO_BPUCT_* code. */
int gko_bpuct_search(void* h, const int32_t* root, int32_t* visits, double* priors, double* move_values,
                     uint8_t* legal, int32_t* info, double* values) {
    ob_search* s = (ob_search*)h;
    for (int a = 0; a < GK_ACTIONS; ++a) {
        visits[a] = 0;
        priors[a] = 0.0;
        move_values[a] = 0.0;
        legal[a] = 0;
    }
    info[0] = -1;
    info[1] = info[2] = info[3] = 0;
    values[0] = values[1] = 0.0;
    for (int i = OB_EVALS; i <= OB_INHERITED; ++i) s->stats[i] = 0;
    if (!s->reuse || (s->size > 0 && !ob_same_state(s->tree[0].rec, root))) s->size = 0;
    if (root[GK_REASON] != GK_NONE) {
        s->size = 0;
        values[0] = ob_terminal_value(root);
        return 0;
    }
    if (s->size == 0) {
        if (ob_push(s, root) < 0) return GKO_BPUCT_LOGIC;
    } else {
        s->stats[OB_REUSED] = s->size;
        s->stats[OB_INHERITED] = s->tree[0].visits;
    }
    int status = 0;
    double w[GK_ACTIONS], v;
    if (!s->tree[0].expanded) {
        ob_evaluate(s->evaluator, s->tree[0].rec, w, &v);
        if ((status = ob_expand(&s->tree[0], w, v)) != 0) goto failed;
        ob_note_batch(s, 1);
    }
    int64_t initial_visits[GK_ACTIONS];
    double initial_values[GK_ACTIONS];
    for (int i = 0; i < s->tree[0].nedges; ++i) {
        initial_visits[i] = s->tree[0].edges[i].visits;
        initial_values[i] = s->tree[0].edges[i].value_sum;
    }
    ob_leaf* pending = (ob_leaf*)malloc((size_t)s->leaf_batch * sizeof(ob_leaf));
    double* weights = (double*)malloc((size_t)s->leaf_batch * GK_ACTIONS * sizeof(double));
    double* leaf_values = (double*)malloc((size_t)s->leaf_batch * sizeof(double));
    if (!pending || !weights || !leaf_values) {
        status = GKO_BPUCT_LOGIC;
        goto release;
    }
    int64_t sims = 0;
    while (sims < s->simulations) {
        const int64_t remaining = s->simulations - sims;
        const int64_t capacity = remaining < s->leaf_batch ? remaining : s->leaf_batch;
        int64_t count = 0;
        while (count < capacity && count < s->simulations - sims) {
            ob_leaf* l = &pending[count];
            l->depth = 0;
            const int found = ob_select(s, 0, l);
            if (found < 0) {
                status = found;
                goto release;
            }
            if (found == 0) break;
            if (s->tree[l->node].rec[GK_REASON] != GK_NONE) {
                ob_backup(s, l, ob_terminal_value(s->tree[l->node].rec));
                ++sims;
                continue;
            }
            ob_reserve(s, l, 1);
            ++count;
        }
        if (count > 0) {
            for (int64_t i = 0; i < count; ++i)
                ob_evaluate(s->evaluator, s->tree[pending[i].node].rec, weights + i * GK_ACTIONS, &leaf_values[i]);
            for (int64_t i = 0; i < count; ++i) {
                const double lv = leaf_values[i];
                if (!isfinite(lv) || lv < -1.0 || lv > 1.0) {
                    status = GKO_BPUCT_BAD_VALUE;
                    goto release;
                }
                for (int a = 0; a < GK_ACTIONS; ++a)
                    if (!isfinite(weights[i * GK_ACTIONS + a]) || weights[i * GK_ACTIONS + a] < 0.0) {
                        status = GKO_BPUCT_BAD_POLICY;
                        goto release;
                    }
            }
            ob_note_batch(s, count);
            for (int64_t i = 0; i < count; ++i) {
                if ((status = ob_expand(&s->tree[pending[i].node], weights + i * GK_ACTIONS, leaf_values[i])) != 0)
                    goto release;
                ob_reserve(s, &pending[i], -1);
                ob_backup(s, &pending[i], leaf_values[i]);
                ++sims;
            }
        } else if (sims < s->simulations) {
            status = GKO_BPUCT_LOGIC;
            goto release;
        }
    }
    {
        const ob_node* r = &s->tree[0];
        double root_sum = 0.0;
        int best = -1;
        int64_t best_visits = 0;
        double best_value = 0.0;
        for (int i = 0; i < r->nedges; ++i) {
            const ob_edge* e = &r->edges[i];
            const int64_t n = e->visits - initial_visits[i];
            const double sum = e->value_sum - initial_values[i];
            const double mean = n == 0 ? 0.0 : sum / (double)n;
            visits[e->move] = (int32_t)n;
            priors[e->move] = e->prior;
            move_values[e->move] = mean;
            legal[e->move] = 1;
            root_sum += sum;
            /* BatchedPUCT.cpp:118-123 over moves in action order. */
            int better;
            if (best < 0) better = 1;
            else if (n != best_visits) better = n > best_visits;
            else if (mean != best_value) better = mean > best_value;
            else if (e->prior != r->edges[best].prior) better = e->prior > r->edges[best].prior;
            else better = 0;
            if (better) {
                best = i;
                best_visits = n;
                best_value = mean;
            }
        }
        if (best < 0 || best_visits == 0) {
            status = GKO_BPUCT_LOGIC;
            goto release;
        }
        info[0] = r->edges[best].move;
        info[1] = (int32_t)sims;
        info[2] = (int32_t)s->size;
        info[3] = (int32_t)s->stats[OB_EVALS];
        values[0] = root_sum / (double)sims;
        values[1] = best_value;
    }
release:
    free(pending);
    free(weights);
    free(leaf_values);
failed:
    if (status != 0) s->size = 0;
    return status;
}

/* BatchedPUCT.cpp:290-326: keep and compact the played move's subtree. */
int gko_bpuct_advance(void* h, int action) {
    ob_search* s = (ob_search*)h;
    ++s->stats[OB_ADVANCES];
    if (!s->reuse || s->size == 0) {
        s->size = 0;
        return 0;
    }
    const ob_node* r = &s->tree[0];
    int found = -1;
    for (int i = 0; i < r->nedges; ++i)
        if (r->edges[i].move == action) found = i;
    if (found < 0 && !(action >= 0 && action < GK_ACTIONS && gko_legal(r->rec, action))) return 0;
    if (found < 0 || r->edges[found].child < 0) {
        s->size = 0;
        return 0;
    }
    int64_t* order = (int64_t*)malloc((size_t)s->size * sizeof(int64_t));
    int64_t* remap = (int64_t*)malloc((size_t)s->size * sizeof(int64_t));
    ob_node* kept = (ob_node*)malloc((size_t)s->size * sizeof(ob_node));
    if (!order || !remap || !kept) {
        free(order);
        free(remap);
        free(kept);
        s->size = 0;
        return 0;
    }
    int64_t count = 0;
    order[count++] = r->edges[found].child;
    for (int64_t next = 0; next < count; ++next) {
        const ob_node* n = &s->tree[order[next]];
        for (int i = 0; i < n->nedges; ++i)
            if (n->edges[i].child >= 0) order[count++] = n->edges[i].child;
    }
    for (int64_t i = 0; i < s->size; ++i) remap[i] = -1;
    for (int64_t i = 0; i < count; ++i) remap[order[i]] = i;
    for (int64_t i = 0; i < count; ++i) {
        kept[i] = s->tree[order[i]];
        for (int e = 0; e < kept[i].nedges; ++e)
            if (kept[i].edges[e].child >= 0) kept[i].edges[e].child = remap[kept[i].edges[e].child];
    }
    memcpy(s->tree, kept, (size_t)count * sizeof(ob_node));
    s->size = count;
    free(order);
    free(remap);
    free(kept);
    ++s->stats[OB_REUSE_HITS];
    return 1;
}
