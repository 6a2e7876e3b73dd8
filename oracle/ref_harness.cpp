// ref_harness.cpp - C-ABI driver around the reference C++ engine (TEST INFRASTRUCTURE).
//
// Compiled together with the reference's own sources (engine/src/*.cpp,
// mcts/src/PUCT.cpp, mcts/src/BatchedPUCT.cpp) by oracle/Makefile into
// oracle/_ref/libgkref.so. It pins the plain-C oracle and serves as the
// "reference" CPU baseline; nothing in the product links it.
//
// Reference entry points used:
//   kingdom::State / play / legal_moves / score   engine/include/board/State.h:16-81
//   kingdom::encode_puct_position                 mcts/include/BatchedPUCT.h:16
//   kingdom::PUCT::search                         mcts/include/PUCT.h:60-73
//   kingdom::BatchedPUCT search / advance / stats mcts/include/BatchedPUCT.h:38-60
// Wire translation follows tests/gpu_rules_test.py:30-39 (cpu_record).
#include "BatchedPUCT.h"
#include "PUCT.h"
#include "board/State.h"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <thread>
#include <vector>

#include "../include/gk_common.h"

using kingdom::Board;
using kingdom::Cell;
using kingdom::EndReason;
using kingdom::Move;
using kingdom::Position;
using kingdom::State;

namespace {

int wire_reason(EndReason reason) {
    switch (reason) {
        case EndReason::Capture: return GK_CAPTURE;
        case EndReason::Suicide: return GK_SUICIDE;
        case EndReason::TwoPasses: return GK_TWO_PASSES;
        default: return GK_NONE;
    }
}

void to_record(const State& s, int32_t* rec) {
    const auto& cells = s.board().cells();
    const auto& owners = s.ownership();
    for (int i = 0; i < GK_CELLS; ++i) {
        rec[i] = static_cast<int32_t>(cells[static_cast<std::size_t>(i)]);
        rec[GK_CELLS + i] = static_cast<int32_t>(owners[static_cast<std::size_t>(i)]);
    }
    rec[GK_ACTOR] = static_cast<int32_t>(s.to_play());
    rec[GK_BLACK_STOCK] = s.remaining_stones(Cell::Black);
    rec[GK_WHITE_STOCK] = s.remaining_stones(Cell::White);
    rec[GK_PASSES] = s.consecutive_passes();
    rec[GK_REASON] = wire_reason(s.result().reason);
    rec[GK_WINNER] = static_cast<int32_t>(s.result().winner);
    rec[GK_CAPTURED] = s.result().captured_stones;
    rec[GK_RESERVED] = 0;
}

Move to_move(int action) { return action == GK_PASS ? Move::pass() : Move::place(action / 9, action % 9); }

int action_of(const Move& m) { return m.is_pass() ? GK_PASS : m.point->row * 9 + m.point->col; }

std::optional<Position> neutral_of(int cell) {
    if (cell < 0 || cell >= GK_CELLS) return std::nullopt;
    return Position{cell / 9, cell % 9};
}

// Legal set by the MCTS::candidates rule (mcts/src/MCTS.cpp:28-51), which
// equals legal_moves() under the default rules (suicide loses).
int fast_legal(const State& s, int* out) {
    int n = 0;
    if (s.result().finished()) return 0;
    const Cell actor = s.to_play();
    if (s.remaining_stones(actor) > 0) {
        const auto& cells = s.board().cells();
        const auto& owners = s.ownership();
        for (int i = 0; i < GK_CELLS; ++i)
            if (cells[static_cast<std::size_t>(i)] == Cell::Empty && owners[static_cast<std::size_t>(i)] == Cell::Empty)
                out[n++] = i;
    }
    out[n++] = GK_PASS;
    return n;
}

int api_legal(const State& s, int* out) {
    int n = 0;
    for (const auto& m : s.legal_moves()) out[n++] = action_of(m);
    return n;
}

kingdom::PUCTEvaluation hash_eval(const State& s) {
    int32_t rec[GK_STATE_WIDTH];
    to_record(s, rec);
    uint64_t words[GK_EVAL_WORDS];
    gk_eval_words_from_record(rec, words);
    const uint64_t h = gk_eval_hash_words(words);
    kingdom::PUCTEvaluation e;
    for (int a = 0; a < GK_ACTIONS; ++a) e.policy[static_cast<std::size_t>(a)] = static_cast<double>(gk_eval_weight(h, a));
    e.value = static_cast<double>(gk_eval_value(h));
    return e;
}

State gen_position(uint64_t seed, uint64_t index) {
    gk_pcg32 rng = gk_pcg32_seed(seed, index);
    int legal[GK_ACTIONS];
    for (int attempt = 0; attempt < 64; ++attempt) {
        const int k = static_cast<int>(gk_pcg32_bounded(&rng, 61u));
        State s;
        bool ok = true;
        for (int i = 0; i < k; ++i) {
            const int n = api_legal(s, legal);
            const int j = static_cast<int>(gk_pcg32_bounded(&rng, static_cast<uint32_t>(n)));
            (void)s.play(to_move(legal[j]));
            if (s.result().finished()) {
                ok = false;
                break;
            }
        }
        if (ok) return s;
    }
    return State();
}

void playout(uint64_t seed, uint64_t game, int neutral, int fast, int8_t* board, int32_t* info) {
    gk_pcg32 rng = gk_pcg32_seed(seed, game);
    State s(kingdom::GameRules{}, neutral_of(neutral));
    int legal[GK_ACTIONS];
    int plies = 0;
    while (!s.result().finished()) {
        const int n = fast ? fast_legal(s, legal) : api_legal(s, legal);
        const int j = static_cast<int>(gk_pcg32_bounded(&rng, static_cast<uint32_t>(n)));
        (void)s.play(to_move(legal[j]));
        ++plies;
    }
    for (int i = 0; i < GK_CELLS; ++i) board[i] = static_cast<int8_t>(s.board().cells()[static_cast<std::size_t>(i)]);
    info[0] = static_cast<int32_t>(s.result().winner);
    info[1] = static_cast<int32_t>(s.result().reason);
    info[2] = s.result().score.black;
    info[3] = s.result().score.white;
    info[4] = plies;
}

template <class F>
void parallel_for(int64_t n, int threads, F&& body) {
    if (threads < 1) threads = 1;
    std::vector<std::thread> pool;
    const int64_t per = (n + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        const int64_t b = t * per, e = std::min<int64_t>(n, b + per);
        if (b >= e) break;
        pool.emplace_back([=, &body] {
            for (int64_t i = b; i < e; ++i) body(i);
        });
    }
    for (auto& th : pool) th.join();
}

// ---- BatchedPUCT -----------------------------------------------------------
// The batch callback sees only schema-1 positions, so the injected evaluator
// rebuilds the wire record of a non-terminal position from its planes
// (BatchedPUCT.cpp:25-50) before hashing it.
kingdom::PUCTEvaluation encoded_eval(int kind, const kingdom::EncodedPUCTPosition& e) {
    kingdom::PUCTEvaluation out;
    const float* f = e.features.data();
    if (kind == 1) {
        out.policy.fill(1.0);
        out.value = 0.0;
        return out;
    }
    if (kind == 2) {  // tests/batched_puct_test.cpp:21-28
        for (std::size_t i = 0; i < Board::kCellCount; ++i) out.policy[i] = static_cast<double>(i + 1) / 81.0;
        out.value = f[405] != 0.0F ? 0.25 : -0.5;
        return out;
    }
    int32_t rec[GK_STATE_WIDTH] = {};
    const int actor = f[405] != 0.0F ? 1 : 2, enemy = 3 - actor;
    for (int i = 0; i < GK_CELLS; ++i) {
        rec[i] = f[i] != 0.0F ? actor : f[81 + i] != 0.0F ? enemy : f[162 + i] != 0.0F ? 3 : 0;
        rec[GK_CELLS + i] = f[243 + i] != 0.0F ? actor : f[324 + i] != 0.0F ? enemy : 0;
    }
    const int own = static_cast<int>(std::lround(f[486] * 41.0)), other = static_cast<int>(std::lround(f[567] * 41.0));
    rec[GK_ACTOR] = actor;
    rec[GK_BLACK_STOCK] = actor == 1 ? own : other;
    rec[GK_WHITE_STOCK] = actor == 1 ? other : own;
    rec[GK_PASSES] = static_cast<int>(std::lround(f[648] * 2.0));
    uint64_t words[GK_EVAL_WORDS];
    gk_eval_words_from_record(rec, words);
    const uint64_t h = gk_eval_hash_words(words);
    for (int a = 0; a < GK_ACTIONS; ++a) out.policy[static_cast<std::size_t>(a)] = static_cast<double>(gk_eval_weight(h, a));
    out.value = static_cast<double>(gk_eval_value(h));
    return out;
}

struct BatchedHandle {
    kingdom::BatchedPUCT search;
    int evaluator;
    int64_t max_rows = 0;
};

}  // namespace

extern "C" {

void* gkr_state_new(int neutral_cell) { return new State(kingdom::GameRules{}, neutral_of(neutral_cell)); }

// cells[81] in {0,1,2,3}; to_play 1 or 2. Returns null on a rejected setup.
void* gkr_state_from_board(const int32_t* cells, int to_play) {
    try {
        Board::Cells c{};
        for (int i = 0; i < GK_CELLS; ++i) c[static_cast<std::size_t>(i)] = static_cast<Cell>(cells[i]);
        return new State(Board(c), static_cast<Cell>(to_play));
    } catch (const std::exception&) {
        return nullptr;
    }
}

void* gkr_state_copy(const void* h) { return new State(*static_cast<const State*>(h)); }
void gkr_state_free(void* h) { delete static_cast<State*>(h); }

int gkr_state_play(void* h, int action) {
    if (action < 0 || action >= GK_ACTIONS) return 0;
    return static_cast<State*>(h)->play(to_move(action)).accepted() ? 1 : 0;
}

void gkr_state_record(const void* h, int32_t* rec) { to_record(*static_cast<const State*>(h), rec); }

void gkr_state_score(const void* h, int32_t* out) {
    const auto s = static_cast<const State*>(h)->score();
    out[0] = s.black;
    out[1] = s.white;
}

int gkr_state_legal(const void* h, int32_t* out) {
    int tmp[GK_ACTIONS];
    const int n = api_legal(*static_cast<const State*>(h), tmp);
    for (int i = 0; i < n; ++i) out[i] = tmp[i];
    return n;
}

void gkr_state_encode(const void* h, float* features, uint8_t* mask) {
    const auto e = kingdom::encode_puct_position(*static_cast<const State*>(h));
    std::memcpy(features, e.features.data(), sizeof(float) * GK_FEATURES);
    for (int a = 0; a < GK_ACTIONS; ++a) mask[a] = e.legal_mask[static_cast<std::size_t>(a)] ? 1 : 0;
}

void gkr_random_playouts(uint64_t seed, uint64_t first, int64_t n, int neutral, int fast, int threads,
                         int8_t* boards, int32_t* infos) {
    parallel_for(n, threads, [&](int64_t i) {
        playout(seed, first + static_cast<uint64_t>(i), neutral, fast, boards + i * GK_CELLS, infos + i * 5);
    });
}

void gkr_gen_positions(uint64_t seed, uint64_t first, int64_t n, int threads, int32_t* recs) {
    parallel_for(n, threads, [&](int64_t i) {
        to_record(gen_position(seed, first + static_cast<uint64_t>(i)), recs + i * GK_STATE_WIDTH);
    });
}

void* gkr_gen_position_state(uint64_t seed, uint64_t index) { return new State(gen_position(seed, index)); }

void gkr_encode_positions(uint64_t seed, uint64_t first, int64_t n, int threads, float* features,
                          uint8_t* masks) {
    parallel_for(n, threads, [&](int64_t i) {
        const State s = gen_position(seed, first + static_cast<uint64_t>(i));
        const auto e = kingdom::encode_puct_position(s);
        std::memcpy(features + i * GK_FEATURES, e.features.data(), sizeof(float) * GK_FEATURES);
        for (int a = 0; a < GK_ACTIONS; ++a)
            masks[i * GK_ACTIONS + a] = e.legal_mask[static_cast<std::size_t>(a)] ? 1 : 0;
    });
}

// Generated positions held as kingdom::State, so the encoder can be timed
// without the generator.
void* gkr_states_generate(uint64_t seed, uint64_t first, int64_t n, int threads) {
    auto* v = new std::vector<State>(static_cast<std::size_t>(n));
    parallel_for(n, threads, [&](int64_t i) { (*v)[static_cast<std::size_t>(i)] = gen_position(seed, first + i); });
    return v;
}

void gkr_states_free(void* h) { delete static_cast<std::vector<State>*>(h); }

// kingdom::encode_puct_position over every held state on `threads` workers.
void gkr_states_encode(const void* h, int threads, float* features, uint8_t* masks) {
    const auto& v = *static_cast<const std::vector<State>*>(h);
    parallel_for(static_cast<int64_t>(v.size()), threads, [&](int64_t i) {
        const auto e = kingdom::encode_puct_position(v[static_cast<std::size_t>(i)]);
        std::memcpy(features + i * GK_FEATURES, e.features.data(), sizeof(float) * GK_FEATURES);
        for (int a = 0; a < GK_ACTIONS; ++a)
            masks[i * GK_ACTIONS + a] = e.legal_mask[static_cast<std::size_t>(a)] ? 1 : 0;
    });
}

// PUCT with the injected hash evaluator and no root noise.
// stats = {best_action, simulations, nodes, network_evaluations}; values = {root, best}.
int gkr_puct_search(const void* h, int simulations, double c_puct, int32_t* visits, double* priors,
                    int32_t* stats, double* values) {
    try {
        kingdom::PUCTOptions o;
        o.simulations = static_cast<std::size_t>(simulations);
        o.c_puct = c_puct;
        o.dirichlet_epsilon = 0.0;
        kingdom::PUCT search(o);
        const auto r = search.search(*static_cast<const State*>(h), hash_eval);
        for (int a = 0; a < GK_ACTIONS; ++a) {
            visits[a] = 0;
            priors[a] = 0.0;
        }
        for (const auto& m : r.moves) {
            visits[action_of(m.move)] = static_cast<int32_t>(m.visits);
            priors[action_of(m.move)] = m.prior;
        }
        stats[0] = r.best_move ? action_of(*r.best_move) : -1;
        stats[1] = static_cast<int32_t>(r.simulations);
        stats[2] = static_cast<int32_t>(r.nodes);
        stats[3] = static_cast<int32_t>(r.network_evaluations);
        values[0] = r.root_value;
        values[1] = r.best_value;
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

// One PUCT per generated position, spread over `threads` workers.
int gkr_puct_positions(uint64_t seed, uint64_t first, int64_t n, int simulations, double c_puct, int threads,
                       int32_t* visits, int32_t* best) {
    int status = 0;
    parallel_for(n, threads, [&](int64_t i) {
        const State s = gen_position(seed, first + static_cast<uint64_t>(i));
        double priors[GK_ACTIONS], values[2];
        int32_t stats[4];
        if (gkr_puct_search(&s, simulations, c_puct, visits + i * GK_ACTIONS, priors, stats, values) != 0) status = -1;
        best[i] = stats[0];
    });
    return status;
}

// PUCT with a caller-supplied evaluator (used to time the reference search
// with a CPU network). The callback receives schema-1 features and the mask
// and returns 82 non-negative policy weights and a value in [-1, 1].
typedef void (*gkr_eval_fn)(const float* features, const uint8_t* mask, double* policy, double* value, void* ctx);

int gkr_puct_search_cb(const void* h, int simulations, double c_puct, double alpha, double epsilon, uint64_t seed,
                       gkr_eval_fn fn, void* ctx, int32_t* visits, int32_t* stats) {
    try {
        kingdom::PUCTOptions o;
        o.simulations = static_cast<std::size_t>(simulations);
        o.c_puct = c_puct;
        o.dirichlet_alpha = alpha;
        o.dirichlet_epsilon = epsilon;
        o.seed = seed;
        kingdom::PUCT search(o);
        const auto r = search.search(*static_cast<const State*>(h), [&](const State& s) {
            const auto e = kingdom::encode_puct_position(s);
            uint8_t mask[GK_ACTIONS];
            for (int a = 0; a < GK_ACTIONS; ++a) mask[a] = e.legal_mask[static_cast<std::size_t>(a)] ? 1 : 0;
            kingdom::PUCTEvaluation out;
            fn(e.features.data(), mask, out.policy.data(), &out.value, ctx);
            return out;
        });
        for (int a = 0; a < GK_ACTIONS; ++a) visits[a] = 0;
        for (const auto& m : r.moves) visits[action_of(m.move)] = static_cast<int32_t>(m.visits);
        stats[0] = r.best_move ? action_of(*r.best_move) : -1;
        stats[1] = static_cast<int32_t>(r.simulations);
        stats[2] = static_cast<int32_t>(r.nodes);
        stats[3] = static_cast<int32_t>(r.network_evaluations);
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

// BatchedPUCT with one of the evaluators above (0 hash, 1 uniform, 2 the
// reference tests' fixed evaluator). Same outputs as gko_bpuct_search.
void* gkr_bpuct_new(int64_t simulations, double c_puct, int64_t leaf_batch, int reuse, int evaluator) {
    try {
        kingdom::PUCTOptions o;
        o.simulations = static_cast<std::size_t>(simulations);
        o.c_puct = c_puct;
        o.dirichlet_epsilon = 0.0;
        return new BatchedHandle{kingdom::BatchedPUCT(o, static_cast<std::size_t>(leaf_batch), reuse != 0), evaluator};
    } catch (const std::exception&) {
        return nullptr;
    }
}

void gkr_bpuct_free(void* h) { delete static_cast<BatchedHandle*>(h); }

void gkr_bpuct_clear(void* h) { static_cast<BatchedHandle*>(h)->search.clear(); }

int gkr_bpuct_search(void* h, const void* state, int32_t* visits, double* priors, double* move_values,
                     uint8_t* legal, int32_t* info, double* values) {
    auto* b = static_cast<BatchedHandle*>(h);
    for (int a = 0; a < GK_ACTIONS; ++a) {
        visits[a] = 0;
        priors[a] = 0.0;
        move_values[a] = 0.0;
        legal[a] = 0;
    }
    info[0] = -1;
    info[1] = info[2] = info[3] = 0;
    values[0] = values[1] = 0.0;
    try {
        const int kind = b->evaluator;
        const auto r = b->search.search(*static_cast<const State*>(state),
                                        [kind](const std::vector<kingdom::EncodedPUCTPosition>& positions) {
                                            std::vector<kingdom::PUCTEvaluation> out;
                                            out.reserve(positions.size());
                                            for (const auto& p : positions) out.push_back(encoded_eval(kind, p));
                                            return out;
                                        });
        for (const auto& m : r.moves) {
            const int a = action_of(m.move);
            visits[a] = static_cast<int32_t>(m.visits);
            priors[a] = m.prior;
            move_values[a] = m.value;
            legal[a] = 1;
        }
        info[0] = r.best_move ? action_of(*r.best_move) : -1;
        info[1] = static_cast<int32_t>(r.simulations);
        info[2] = static_cast<int32_t>(r.nodes);
        info[3] = static_cast<int32_t>(r.network_evaluations);
        values[0] = r.root_value;
        values[1] = r.best_value;
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

int gkr_bpuct_advance(void* h, int action) {
    auto* b = static_cast<BatchedHandle*>(h);
    return b->search.advance(to_move(action)) ? 1 : 0;
}

void gkr_bpuct_stats(const void* h, int64_t* out) {
    const auto& s = static_cast<const BatchedHandle*>(h)->search.stats();
    out[0] = static_cast<int64_t>(s.network_evaluations);
    out[1] = static_cast<int64_t>(s.inference_batches);
    out[2] = static_cast<int64_t>(s.max_observed_batch_size);
    out[3] = static_cast<int64_t>(s.reused_nodes);
    out[4] = static_cast<int64_t>(s.inherited_visits);
    out[5] = static_cast<int64_t>(s.advance_calls);
    out[6] = static_cast<int64_t>(s.reuse_hits);
}

}  // extern "C"

