/*
 * gk_oracle.h - CPU oracle (test infrastructure only).
 *
 * A plain-C restatement of the reference rules, encoder and PUCT search,
 * operating on the int32[170] wire record. It is the checker for the CUDA
 * path: only tests, the smoke check and the benchmark's CPU-baseline leg use
 * it. Nothing in the product links or calls it.
 *
 * Parity is pinned: tests compare it with the reference C++ engine compiled
 * from its own sources (oracle/_ref) and with golden vectors taken from the
 * reference's tests (tests/golden).
 */
#ifndef GK_ORACLE_H
#define GK_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void gko_initial(int32_t* rec, int neutral_cell);
int gko_legal(const int32_t* rec, int action);
int gko_play(int32_t* rec, int action);
void gko_score(const int32_t* rec, int* black, int* white);
void gko_encode(const int32_t* rec, float* features, uint8_t* mask);
void gko_play_batch(int32_t* recs, const int32_t* actions, uint8_t* accepted, int64_t n);
void gko_encode_batch(const int32_t* recs, float* features, uint8_t* masks, int64_t n);

/* Uniform-random playout: info = {winner, cpp_reason, score_black, score_white, plies}. */
void gko_random_playout(uint64_t seed, uint64_t game, int neutral_cell, int8_t* board, int32_t* info);
void gko_random_playouts(uint64_t seed, uint64_t first_game, int64_t n, int neutral_cell, int8_t* boards,
                         int32_t* infos);
/* Random mid-game position generator: k ~ U[0,60] uniform legal moves, non-terminal. */
void gko_gen_position(uint64_t seed, uint64_t index, int32_t* rec);
void gko_gen_positions(uint64_t seed, uint64_t first, int64_t n, int32_t* recs);

void gko_eval(const int32_t* rec, float* weights, float* value);

/* PUCT search with the injected evaluator and no root noise.
 * Outputs: visits[82], priors[82] (0 for illegal), stats = {best_action,
 * simulations, nodes, network_evaluations}, values = {root_value, best_value}. */
int gko_puct_search(const int32_t* rec, int simulations, double c_puct, int32_t* visits, double* priors,
                    int32_t* stats, double* values);
/* Same search with a uniform evaluator (all weights 1, value 0). */
int gko_puct_search_uniform(const int32_t* rec, int simulations, double c_puct, int32_t* visits, double* priors,
                            int32_t* stats, double* values);
/* Root tactical checks (python/kingdom_ai/gpu_puct.py:84-161): per action
 * outcome +1 / -1 / 0 and the narrowed root candidates. */
void gko_root_tactics(const int32_t* rec, int8_t* outcome, uint8_t* allow);
/* The search above with the root narrowed by gko_root_tactics. */
int gko_puct_search_tactics(const int32_t* rec, int simulations, double c_puct, int uniform, int32_t* visits,
                            double* priors, int32_t* stats, double* values);
int gko_puct_search_batch(const int32_t* recs, int64_t n, int simulations, double c_puct, int32_t* visits,
                          int32_t* best, double* root_values, int threads);

/* Self-play of one game with the injected evaluator and no root noise, as the
 * device engine plays it (temperature schedule of collect_gpu_puct_games,
 * move draws from PCG32 (sample_seed ^ salt, game * 256 + ply); tactics: the
 * root tactical checks narrow every root). Outputs:
 * actions[GK_MAX_PLIES + 2], policy[GK_MAX_PLIES + 2][82] (visit shares per
 * ply), the final record rec[170]. Returns the plies played, or < 0. */
int gko_selfplay_hash_game(uint64_t sample_seed, uint64_t game, int neutral_cell, int simulations, double c_puct,
                           int temperature_moves, double temperature, double final_temperature, int tactics,
                           uint8_t* actions, float* policy, int32_t* rec);
/* Games first_game .. first_game + n - 1 of the above on `threads` threads;
 * plies[n] receives each game's return value. */
void gko_selfplay_hash_games(uint64_t sample_seed, uint64_t first_game, int64_t n, int neutral_cell,
                             int simulations, double c_puct, int temperature_moves, double temperature,
                             double final_temperature, int tactics, uint8_t* actions, float* policy, int32_t* recs,
                             int32_t* plies, int threads);

/* BatchedPUCT (mcts/src/BatchedPUCT.cpp): a persistent searcher with leaf
 * batches under virtual loss and subtree reuse. `evaluator` picks the leaf
 * evaluator (GKO_EVAL_*). stats = {network_evaluations, inference_batches,
 * max_observed_batch_size, reused_nodes, inherited_visits, advance_calls,
 * reuse_hits}. */
#define GKO_BPUCT_STATS 7
#define GKO_EVAL_HASH 0
#define GKO_EVAL_UNIFORM 1
#define GKO_EVAL_RAMP 2 /* tests/batched_puct_test.cpp:21-28 */
#define GKO_BPUCT_BAD_VALUE (-2)   /* value not finite or outside [-1, 1] */
#define GKO_BPUCT_BAD_POLICY (-3)  /* a weight not finite or negative */
#define GKO_BPUCT_ZERO_POLICY (-4) /* no positive weight on a legal action */
#define GKO_BPUCT_LOGIC (-5)
void* gko_bpuct_new(int64_t simulations, double c_puct, int64_t leaf_batch, int reuse, int evaluator);
void gko_bpuct_free(void* h);
void gko_bpuct_clear(void* h);
int64_t gko_bpuct_size(const void* h);
void gko_bpuct_stats(const void* h, int64_t* out);
int gko_bpuct_search(void* h, const int32_t* root, int32_t* visits, double* priors, double* move_values,
                     uint8_t* legal, int32_t* info, double* values);
int gko_bpuct_advance(void* h, int action);

#ifdef __cplusplus
}
#endif
#endif
