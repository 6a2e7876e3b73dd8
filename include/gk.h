/*
 * gk.h - C ABI of libgk.so, the B200-native batched self-play engine.
 *
 * Conventions (all entry points)
 *   - Pointers are device pointers unless a parameter says "host".
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *     work is enqueued on it and the call returns without synchronising.
 *   - Return value: 0 on success, GK_EINVAL (-22) for a rejected argument
 *     (nothing is launched), otherwise the cudaError_t of a failed launch.
 *   - Hot entry points allocate nothing; scratch comes from the caller, sized
 *     by the matching *_workspace_bytes function.
 *   - Device-side failures never trap: they set bits (GK_ERR_* in
 *     gk_common.h) in a caller-supplied uint32 status word or per-lane word.
 *     Entry points whose kernels wait on barriers (gk_net_*, gk_mma_selftest,
 *     gk_selfplay_ply) take uint32 status[2]: every wait is bounded, and the
 *     first wait that gives up sets GK_ERR_TIMEOUT in status[0] and records
 *     its barrier's shared address | parity << 31 in status[1].
 *
 * Each declaration names the reference interface it replaces. The reference
 * launches NVRTC kernels through ctypes (python/kingdom_ai/gpu_runtime.py:179-221,
 * CudaModule.launch); these functions are what that FFI binds instead.
 */
#ifndef GK_H
#define GK_H

#include <stddef.h>
#include <stdint.h>

#include "gk_common.h"

#if defined(__GNUC__)
#define GK_API __attribute__((visibility("default")))
#else
#define GK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- rules */

/* Initial states in wire format. Replaces gpu_initial_batch
 * (python/kingdom_ai/gpu_rules.py:284-293) behind GpuStateBatch.initial
 * (gpu_rules.py:353-374). neutral_cell = row*9+col, or -1 for none. */
GK_API int gk_initial_records(int32_t* recs, int64_t n, int neutral_cell, void* stream);

/* Initial states in packed format (uint32[n,16]). Same semantics as
 * gk_initial_records (reference gpu_initial_batch, gpu_rules.py:284-293). */
GK_API int gk_initial_bits(uint32_t* bits, int64_t n, int neutral_cell, void* stream);

/* One transition per wire record, in place; accepted[n] gets 1/0 and rejected
 * records stay unchanged. actions are int32 (action_bytes 4) or int64 (8);
 * int64 values outside [0,82) are rejected without wrapping. Replaces
 * gpu_play_batch (gpu_rules.py:295-301) behind GpuStateBatch.play (:418-443). */
GK_API int gk_play_records(int32_t* recs, const void* actions, int action_bytes, uint8_t* accepted, int64_t n,
                    void* stream);

/* Schema-1 observation planes fp32[n,10,9,9] and legal mask bool[n,82].
 * Replaces gpu_encode_batch (gpu_rules.py:303-311) behind GpuStateBatch.encode
 * (:445-454) and the CPU encode_puct_batch (bindings/batched_puct.cpp:140-148). */
GK_API int gk_encode_records(const int32_t* recs, float* features, uint8_t* masks, int64_t n, void* stream);

/* Wire record -> packed state. If `status` is non-null, GK_ERR_BAD_INPUT is
 * OR-ed into it when a record holds a value outside the wire format's ranges.
 * Replaces the record copy of gpu_search_initialize (gpu_puct.py:163-180). */
GK_API int gk_records_to_bits(const int32_t* recs, uint32_t* bits, uint32_t* status, int64_t n, void* stream);

/* Packed state -> wire record (reserved field 169 written as 0); the export
 * side of the wire format of python/kingdom_ai/gpu_rules.py:16-33. */
GK_API int gk_bits_to_records(const uint32_t* bits, int32_t* recs, int64_t n, void* stream);

/* One transition per packed state, in place (the HBM-bound rules kernel).
 * Same rules as gpu_play (gpu_rules.py:185-252) / State::play (engine/src/State.cpp:92-167).
 * Packed states must come from gk_records_to_bits, gk_initial_bits or earlier
 * library transitions: the territory-settled flag (GK_META_SETTLED) that the
 * transitions set lets a placement re-examine only the empty component it
 * splits; hand-built states leave meta bits 27..31 zero. */
GK_API int gk_play_bits(uint32_t* bits, const void* actions, int action_bytes, uint8_t* accepted, int64_t n, void* stream);

/* Encoder from packed states; same outputs as gk_encode_records (reference
 * gpu_encode, gpu_rules.py:258-282; encode, mcts/src/BatchedPUCT.cpp:25-50). */
GK_API int gk_encode_bits(const uint32_t* bits, float* features, uint8_t* masks, int64_t n, void* stream);

/* Uniform-random complete playouts from the default start, one PCG32 stream
 * per game (seed, first_game + i). boards int8[n,81]; infos int32[n,5] =
 * {winner, C++ EndReason, score black, score white, plies}. No reference API
 * (the reference samples legal_moves() in tests/board_test.cpp:131-162). */
GK_API int gk_random_playouts(uint64_t seed, uint64_t first_game, int64_t n, int neutral_cell, int8_t* boards,
                       int32_t* infos, void* stream);

/* Random non-terminal mid-game positions (k ~ U[0,60] uniform legal moves,
 * stream (seed, first + i)) as packed states. No reference counterpart: a
 * workload generator for the encoder, search and network benchmarks. */
GK_API int gk_gen_positions(uint64_t seed, uint64_t first, int64_t n, uint32_t* bits, void* stream);

/* ----------------------------------------------------------------- PUCT */

/* Search options (python/kingdom_ai/gpu_puct.py:26-63, GpuPUCTOptions;
 * the device copy is the `options` tensor of gpu_puct.py:465-468). */
typedef struct {
    double c_puct;
    double dirichlet_epsilon; /* root noise weight; 0 disables */
    int fpu_enabled;          /* nonzero: unvisited edges start at node value - fpu_reduction */
    double fpu_reduction;
} gk_puct_options;

/* Device pointers into a search workspace that an external evaluator reads
 * and writes between gk_puct_select and gk_puct_expand_backup. */
typedef struct {
    uint8_t* needs_eval;   /* [B] 1: leaf_bits[t] needs policy/value */
    uint32_t* leaf_bits;   /* [B,16] packed leaf states */
    float* leaf_value;     /* [B] evaluator writes the value (current player's view) */
    float* policy;         /* [B,82] evaluator writes probabilities or weights >= 0 */
    float* noise;          /* [B,82] root noise written by gk_puct_noise */
    int32_t* active;       /* [B] compacted tree indices (gk_puct_compact) */
    int32_t* active_count; /* [1] */
    uint32_t* errors;      /* [B] GK_ERR_* per tree */
    int32_t* leaf;         /* [B] node of the leaf to evaluate (0: the root) */
    uint32_t* root_allow;  /* [B,3] root candidates: bit a%32 of word a/32 (all after gk_puct_begin) */
    int32_t* node_visits;  /* [B,capacity] visits of each node (node 0 the root; nodes >= the tree's node
                              count hold stale values) */
} gk_puct_buffers_t;

/* Search outputs (GpuSearchResult, gpu_puct.py:66-76); any pointer may be
 * NULL to skip that output. `status` receives the OR of all tree errors. */
typedef struct {
    int64_t* actions;             /* [B] best action, -1 for a terminal root */
    int32_t* visits;              /* [B,82] root visit counts */
    float* policy;                /* [B,82] visits / simulations */
    float* values;                /* [B] mean backed-up value for the root player */
    int32_t* simulations;         /* [B] */
    int32_t* network_evaluations; /* [B] */
    double* priors;               /* [B,82] root priors (after noise) */
    float* best_values;           /* [B] mean value of the best action */
    int32_t* nodes;               /* [B] tree size */
    double* root_values;          /* [B] root value in double (for exact comparison) */
    uint32_t* status;             /* [1] OR of GK_ERR_* bits */
} gk_puct_results_t;

/* Bytes of device workspace for `batch` trees of `capacity` nodes
 * (capacity = simulations + 1, gpu_puct.py:439). 0 for invalid sizes. */
GK_API size_t gk_puct_workspace_bytes(int64_t batch, int capacity);

/* Fill `out` (host struct) with device pointers into the workspace: the
 * leaf tensors the reference allocates in GpuPUCT._search (gpu_puct.py:445-471). */
GK_API int gk_puct_buffers(void* ws, int64_t batch, int capacity, gk_puct_buffers_t* out);

/* Reset the trees at the given packed roots. Replaces gpu_search_initialize
 * (gpu_puct.py:163-180). */
GK_API int gk_puct_begin(void* ws, int64_t batch, int capacity, const uint32_t* root_bits, void* stream);

/* Root tactical checks: narrow each root's candidate actions to the ones that
 * win at once if there are any, else to those after which the opponent has
 * no winning reply if there are any (else all stay). Call after gk_puct_begin
 * and before the root's evaluation; select, expand, noise, finish and the
 * native evaluator then honour the candidates. Replaces gpu_search_root_tactics
 * and gpu_search_root_filter (gpu_puct.py:84-161, launched at :475-479). */
GK_API int gk_puct_root_tactics(void* ws, int64_t batch, int capacity, void* stream);

/* Root Dirichlet noise over each root's legal actions, max-normalised, from
 * PCG32 stream (seed, stream_base + tree). Replaces the torch._standard_gamma
 * block of GpuPUCT._search (gpu_puct.py:509-517). */
GK_API int gk_puct_noise(void* ws, int64_t batch, int capacity, uint64_t seed, uint64_t stream_base, double alpha,
                  void* stream);

/* One selection pass per tree (one leaf per tree). Replaces gpu_search_select
 * (gpu_puct.py:182-258). */
GK_API int gk_puct_select(void* ws, int64_t batch, int capacity, const gk_puct_options* options, void* stream);

/* The injected evaluator: weights w_a = exp(z_a) and a uniform value, pure
 * functions of the leaf (gk_common.h). No reference counterpart: it stands in
 * for the evaluator callback of PUCT::search (mcts/include/PUCT.h:34). */
GK_API int gk_puct_hash_eval(void* ws, int64_t batch, int capacity, void* stream);

/* Ordered list of trees whose leaf needs evaluation (device-side; replaces
 * the host-synchronising nonzero() of gpu_puct.py:482). */
GK_API int gk_puct_compact(void* ws, int64_t batch, int capacity, void* stream);

/* Expand evaluated leaves ((w/max)/sum priors, root noise mix) and, when
 * `backup` is nonzero, back the leaf value up the path. Replaces
 * gpu_search_expand_backup (gpu_puct.py:260-341). */
GK_API int gk_puct_expand_backup(void* ws, int64_t batch, int capacity, const gk_puct_options* options, int backup,
                          void* stream);

/* Root statistics and best action. Replaces gpu_search_finish
 * (gpu_puct.py:343-379). `results` is a host struct of device pointers. */
GK_API int gk_puct_finish(void* ws, int64_t batch, int capacity, const gk_puct_results_t* results, void* stream);

/* A complete search with the injected evaluator, no host synchronisation:
 * begin, then one kernel in which each tree's warp runs the root evaluation
 * and `simulations` x (select, evaluate, expand/backup), then finish. Results
 * equal those of the separate gk_puct_* steps. The workspace must be sized
 * for capacity = simulations + 1. With options->dirichlet_epsilon != 0 the
 * root mixes in the workspace's noise rows, which gk_puct_noise must have
 * drawn (or the caller zeroed) first. Equivalent of PUCT::search
 * (mcts/src/PUCT.cpp:177-268) per tree. */
GK_API int gk_puct_search_hash(void* ws, int64_t batch, int simulations, const uint32_t* root_bits,
                        const gk_puct_options* options, const gk_puct_results_t* results, void* stream);

/* Scratch limit of gk_puct_search_hash_noalloc per device: 16 MiB, e.g. 20
 * trees of 400 simulations, 125 of 64 or 471 of 16. */
#define GK_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
/* Returned when a request needs more scratch than GK_NOALLOC_SCRATCH_BYTES. */
#define GK_ENOSPC (-28)

/* gk_puct_search_hash without a caller workspace; it has no reference
 * counterpart. For callers that can pass device buffers but cannot allocate
 * device memory on the call path: a host-language binding with no CUDA
 * allocator of its own (a cgo, JNI or ctypes stub holding only pointers it
 * was given), or a service whose device memory is fixed at start-up. The
 * trees live in a file-scope device array of GK_NOALLOC_SCRATCH_BYTES; a
 * request whose gk_puct_workspace_bytes(batch, simulations + 1) exceeds it
 * returns GK_ENOSPC and launches nothing. The first call in each CUDA context
 * on a device resolves the array's address with that device current
 * (set-up): make it before any stream capture. The search draws no root
 * noise: options->dirichlet_epsilon must be 0 (else GK_EINVAL). Each call
 * writes every per-tree field it reads, so the previous call's contents do
 * not matter. All calls on a device share the array, so calls that overlap in
 * time (other streams, other host threads) race: the caller serialises them.
 * Calls no allocator. */
GK_API int gk_puct_search_hash_noalloc(int64_t batch, int simulations, const uint32_t* root_bits,
                                       const gk_puct_options* options, const gk_puct_results_t* results,
                                       void* stream);

/* -------------------------------------------------------------- network */

/* Device pointers of a packed policy/value network. Layout of conv_w, for each
 * 3x3 layer (stem first, then two per residual block), the stem's Cin padded
 * from 10 to 16: for each of the 9 taps (row-major over (dr, dc)), bf16
 * [Cin/8][Cout][8]; except with 64 channels and batch norm, where it is for
 * each row offset dr (-1, 0, 1) bf16 [Cin/8][3 (dc = -1, 0, 1)][Cout][8], the
 * three column taps side by side. head_w/head_b: the 1x1 policy (2 rows) and
 * value (1 row) convolutions. pol_*, val_*: the fully connected heads.
 *
 * norm = 0: batch norm folded into the convolutions (the self-play workload
 * layout): conv_b fp32 [layers][C] is each layer's folded bias, the head
 * convolutions carry their folded biases, and the value head's hidden width is
 * 64. norm = 1: the reference's PolicyValueNet (python/kingdom_ai/model.py:
 * 13-84): bias-free convolutions, each followed by GroupNorm(gcd(8, C), C)
 * with norm_w/norm_b fp32 [layers][C] (eps 1e-5), the policy and value 1x1
 * convolutions by GroupNorm(1, 2) and GroupNorm(1, 1) with head_norm fp32[6] =
 * {policy weight[2], policy bias[2], value weight, value bias}, and a value
 * hidden width of C; conv_b and head_b are unused.
 *
 * conv_w, pol_w, val_w1 and (norm 0) conv_b must be 16-byte aligned: the
 * kernels read them with 16-byte copies. Anything else is GK_EINVAL. */
typedef struct {
    int channels; /* 32, 64 or 128 */
    int blocks;   /* residual blocks */
    const void* conv_w;
    const float* conv_b;
    const float* head_w; /* [3][C] */
    const float* head_b; /* [3] */
    const float* pol_w;  /* [162][82]: policy FC, feature-major (the transpose of torch's [82][162]) */
    const float* pol_b;  /* [82] */
    const float* val_w1; /* [81][H], H = 64 (norm 0) or C (norm 1): value FC, feature-major */
    const float* val_b1; /* [H] */
    const float* val_w2; /* [H] */
    const float* val_b2; /* [1] */
    int norm;                /* 0 batch norm folded, 1 GroupNorm */
    const float* norm_w;     /* [layers][C] (norm 1) */
    const float* norm_b;     /* [layers][C] (norm 1) */
    const float* head_norm;  /* [6] (norm 1) */
} gk_net_t;

/* Tensor-core self-test: D[128,64] (fp32) = A[128,16] x B[64,16]^T (bf16 bit
 * patterns, row-major) through one tcgen05.mma with the operand layout the
 * network kernels use. No reference counterpart: a pre-flight check of the
 * descriptor encodings, whose addresses stay in range by construction. */
GK_API int gk_mma_selftest(const uint16_t* a, const uint16_t* b, float* d, uint32_t* status, void* stream);

/* Bytes of packed bf16 convolution weights for this shape (0 if unsupported);
 * the packed form of the reference model's conv parameters
 * (python/kingdom_ai/model.py:43-50). */
GK_API size_t gk_net_weight_bytes(int channels, int blocks);

/* Bytes of the per-call head-feature workspace for n positions (the 1x1
 * head convolution outputs of python/kingdom_ai/model.py:51-69). */
GK_API size_t gk_net_headfeat_bytes(int64_t n);

/* Network forward for n positions given either packed states (`states`,
 * uint32[n,16]; the 10 observation planes are built on the fly) or schema-1
 * features (fp32[n,10,9,9]); exactly one must be non-null. Writes raw policy
 * logits fp32[n,82] and values fp32[n]. `headfeat` is workspace of
 * gk_net_headfeat_bytes(n). Replaces the model forward of the reference's
 * leaf evaluation (PolicyValueNet.forward, python/kingdom_ai/model.py:72-84,
 * called from GpuPUCT._search, gpu_puct.py:485). */
GK_API int gk_net_forward(const gk_net_t* net, const uint32_t* states, const float* features, int64_t n,
                          float* headfeat, float* logits, float* values, uint32_t* status, void* stream);

/* Leaf evaluation inside a search: compacts the trees whose leaf needs the
 * network (device-side, no host synchronisation), runs the network on those
 * leaves and writes the masked softmax policy and the value into the search
 * workspace. Replaces GpuPUCT._search's evaluate() (gpu_puct.py:481-502). */
GK_API int gk_net_evaluate_puct(const gk_net_t* net, void* ws, int64_t batch, int capacity, float* headfeat,
                                uint32_t* status, void* stream);

/* Network evaluation of a gathered set of packed states: for i <
 * *active_count, state active[i] (uint32[16] each) is evaluated and its masked
 * softmax policy over legal actions and its value are written to row
 * active[i] of policy fp32[n,82] and value fp32[n]. Used by the batched
 * evaluation search (gk_bpuct_*) for its leaf slots; the reference calls the
 * model through EncodedBatchedEvaluator (python/kingdom_ai/encoded_batching.py:71-95). */
GK_API int gk_net_evaluate_states(const gk_net_t* net, const uint32_t* states, const int32_t* active,
                                  const int32_t* active_count, int64_t n, float* policy, float* value,
                                  float* headfeat, uint32_t* status, void* stream);

/* ------------------------------------------------------------ self-play */

/* Per-ply self-play parameters (GpuPUCTOptions plus the temperature schedule
 * of collect_gpu_puct_games, python/kingdom_ai/gpu_training.py:124-175). */
typedef struct {
    int simulations;
    double c_puct;
    double dirichlet_alpha;
    double dirichlet_epsilon;
    int fpu_enabled;
    double fpu_reduction;
    int temperature_moves;    /* plies per game that use `temperature` */
    double temperature;       /* before temperature_moves (0 = best action) */
    double final_temperature; /* afterwards */
    uint64_t seed;            /* root noise (GpuPUCTOptions.seed) */
    uint64_t game_stride;     /* game-id step when a lane starts its next game */
    int neutral_cell;         /* start position's neutral stone, -1 for none */
    int tactical_checks;      /* nonzero: gk_puct_root_tactics at every root (GpuPUCTOptions.tactical_checks) */
    uint64_t sample_seed;     /* move sampling (the `seed` argument of collect_gpu_puct_games) */
    uint64_t game_limit;      /* 0: lanes play forever; else a lane whose next game id would reach
                                 game_limit parks on its finished position and plays no more */
} gk_selfplay_params_t;

/* Finished-game log of gk_selfplay_ply: the k-th game to finish (in device
 * order) goes to slot k % capacity. Its action history replays the game from
 * the start position through the rules (the record_history output of
 * collect_gpu_puct_games, gpu_training.py:50-51, 89-90, 113), and its replay
 * rows are rows first_row .. first_row + plies - 1 of the replay ring (ring
 * index = row % replay capacity). */
#define GK_GAME_ACTIONS (GK_MAX_PLIES + 2)
typedef struct {
    uint64_t* game_id;      /* [capacity] */
    uint64_t* first_row;    /* [capacity] replay rows written before this game's */
    int32_t* plies;         /* [capacity] moves played, = replay rows of the game */
    int8_t* winner;         /* [capacity] 1 black, 2 white */
    int8_t* reason;         /* [capacity] GPU reason code (GK_CAPTURE, GK_SUICIDE, GK_TWO_PASSES) */
    uint32_t* final_state;  /* [capacity][16] packed final position */
    uint8_t* actions;       /* [capacity][GK_GAME_ACTIONS] action of each ply (81 = pass) */
    int64_t capacity;
} gk_gamelog_t;

/* FIFO replay ring in the CPU ReplayBuffer's row schema
 * (python/kingdom_ai/replay.py:106-125): features f32[cap,10,9,9],
 * masks bool[cap,82], policy f32[cap,82], value f32[cap], to_play i8[cap]. */
typedef struct {
    float* features;
    uint8_t* masks;
    float* policy;
    float* value;
    int8_t* to_play;
    int64_t capacity;
} gk_replay_t;

/* Device pointers into a self-play workspace. counters (uint64[8]): moves,
 * finished games, replay rows written (monotone; ring index = rows % cap),
 * errors, black wins, white wins, capture endings, network evaluations. */
typedef struct {
    uint32_t* states;      /* [lanes,16] packed current positions (writable between plies) */
    int32_t* lane_ply;     /* [lanes] plies of the current game; -1 once parked */
    uint64_t* game_id;     /* [lanes] */
    uint64_t* counters;    /* [8] */
    int32_t* last_action;  /* [lanes] action played in the last ply, -1 if none */
    float* last_policy;    /* [lanes,82] visit shares of the last ply's search (the policy target) */
} gk_selfplay_buffers_t;

/* Bytes of self-play workspace for `lanes` concurrent games (positions,
 * per-game history of states and visit policies, counters). The device-side
 * equivalent of the history tensors of gpu_training.py:44-55. */
GK_API size_t gk_selfplay_workspace_bytes(int64_t lanes);

/* Start every lane at the initial position; lane i plays game first_game + i,
 * then first_game + i + game_stride, ... Zeroes the counters. Replaces the
 * GpuStateBatch.initial call of collect_gpu_puct_games (gpu_training.py:171). */
GK_API int gk_selfplay_reset(void* ws, int64_t lanes, int neutral_cell, uint64_t first_game, void* stream);

/* Fill `out` (host struct) with device pointers into the workspace. Same
 * role as the reference's history tensors (gpu_training.py:44-55). */
GK_API int gk_selfplay_buffers(void* ws, int64_t lanes, gk_selfplay_buffers_t* out);

/* One ply of batched self-play: a full search per lane with the native
 * network (no host synchronisation), then one move per lane; finished games
 * are written to `replay` and `games` (each may be NULL) and their lanes
 * restart, or park once params->game_limit is reached. `puct_ws` is a search
 * workspace for (lanes, simulations + 1); `headfeat` holds
 * gk_net_headfeat_bytes(lanes); `timer` (may be NULL, see gk_timer_create)
 * records the network tower's launches (inside a stream capture, as external
 * event nodes, so a graph replay records them). `net` may be NULL: leaves are then
 * scored by the injected evaluator (gk_puct_hash_eval) and headfeat may be
 * NULL. Replaces one iteration of the reference's per-ply loop
 * (gpu_training.py:59-87). */
GK_API int gk_selfplay_ply(void* sp_ws, void* puct_ws, int64_t lanes, const gk_net_t* net,
                           const gk_selfplay_params_t* params, const gk_replay_t* replay,
                           const gk_gamelog_t* games, float* headfeat, uint32_t* status, void* timer,
                           void* stream);

/* ------------------------------------------------------ batched search */

/* kingdom::BatchedPUCT (mcts/include/BatchedPUCT.h:38-60,
 * mcts/src/BatchedPUCT.cpp) for many searchers at once: one workspace holds
 * `trees` trees of at most `capacity` nodes, and each search runs in waves
 * that collect up to `leaf_batch` pending leaves per tree under a virtual
 * loss of one, evaluate them together and back them up in collection order.
 * Trees persist between searches; gk_bpuct_advance keeps the played move's
 * subtree (reuse). A search adds at most `simulations` nodes to a tree, so a
 * caller keeps capacity >= nodes held + simulations + 1 (gk_bpuct_grow).
 * Per-tree statistics, GK_BPUCT_STAT_* order (BatchedPUCTStatistics,
 * BatchedPUCT.h:21-31): */
#define GK_BPUCT_STAT_EVALS 0        /* network evaluations of the last search */
#define GK_BPUCT_STAT_BATCHES 1      /* inference batches of the last search */
#define GK_BPUCT_STAT_MAX_BATCH 2    /* largest batch of the last search */
#define GK_BPUCT_STAT_REUSED 3       /* nodes held when the last search began */
#define GK_BPUCT_STAT_INHERITED 4    /* root visits when the last search began */
#define GK_BPUCT_STAT_ADVANCES 5     /* advance calls (cumulative) */
#define GK_BPUCT_STAT_REUSE_HITS 6   /* advances that kept a subtree (cumulative) */
#define GK_BPUCT_STATS 7
/* Evaluation failures of a batched search, besides GK_ERR_BAD_EVAL (a value
 * not finite or outside [-1, 1], BatchedPUCT.cpp:73-75): */
#define GK_BPUCT_ERR_POLICY (1u << 4)    /* a weight not finite or negative (BatchedPUCT.cpp:76-80) */
#define GK_BPUCT_ERR_NO_WEIGHT (1u << 5) /* no positive weight on a legal action (BatchedPUCT.cpp:233-236) */

typedef struct {
    int64_t* actions;      /* [T] best action (BatchedPUCT.cpp:118-123), -1 when none */
    int32_t* visits;       /* [T,82] visits gained in this search */
    double* priors;        /* [T,82] root edge priors */
    double* move_values;   /* [T,82] mean value gained in this search */
    uint8_t* legal;        /* [T,82] the root's edges (its legal actions) */
    int32_t* simulations;  /* [T] */
    int32_t* nodes;        /* [T] tree size after the search */
    double* root_values;   /* [T] */
    double* best_values;   /* [T] */
    int32_t* stats;        /* [T,GK_BPUCT_STATS] */
    uint32_t* errors;      /* [T] GK_ERR_* of this search; a failed tree is cleared */
    uint32_t* status;      /* [1] OR of errors, or NULL */
} gk_bpuct_results_t;

typedef struct {
    uint8_t* needs_eval;   /* [T*L] slot holds a leaf to evaluate */
    uint32_t* leaf_bits;   /* [T*L,16] packed leaf states */
    double* policy;        /* [T*L,82] evaluator weights (read unless float_eval) */
    double* value;         /* [T*L] */
    float* policy_f;       /* [T*L,82] fp32 evaluator output (float_eval) */
    float* value_f;        /* [T*L] */
    int32_t* active;       /* [T*L] slots compacted by gk_bpuct_compact */
    int32_t* active_count; /* [1] */
    int32_t* pending;      /* [T] leaves of the current wave */
    int32_t* node_count;   /* [T] nodes held */
    int32_t* remaining;    /* [1] max over trees of simulations left after the last wave */
    int32_t* stats;        /* [T,GK_BPUCT_STATS] current statistics */
} gk_bpuct_buffers_t;

/* Bytes of a batched-search workspace (0 for invalid sizes). Stands in for
 * the per-searcher node vectors of BatchedPUCT::Impl (BatchedPUCT.cpp:134-140). */
GK_API size_t gk_bpuct_workspace_bytes(int64_t trees, int capacity, int leaf_batch);
/* Device pointers of the workspace's evaluator interface and counters. */
GK_API int gk_bpuct_buffers(void* ws, int64_t trees, int capacity, int leaf_batch, gk_bpuct_buffers_t* out);
/* Empty trees and zero counters (once, after allocating the workspace). */
GK_API int gk_bpuct_init(void* ws, int64_t trees, int capacity, int leaf_batch, void* stream);
/* BatchedPUCT::clear (BatchedPUCT.cpp:286) of the trees with mask[t] != 0 (NULL: all). */
GK_API int gk_bpuct_clear(void* ws, int64_t trees, int capacity, int leaf_batch, const uint8_t* mask,
                          void* stream);
/* Start a search of the trees with mask[t] != 0 (NULL: all) from packed roots
 * (BatchedPUCT.cpp:339-367): a tree that does not continue from its root, or
 * any tree when reuse is 0, is cleared; a finished root clears the tree and
 * gives its terminal value; an unexpanded root is queued in slot 0. */
GK_API int gk_bpuct_begin(void* ws, int64_t trees, int capacity, int leaf_batch, const uint32_t* roots,
                          const uint8_t* mask, int simulations, int reuse, void* stream);
/* Expand the queued roots from their evaluations (one batch of one each,
 * BatchedPUCT.cpp:361-365) and record the root edges results are measured from. */
GK_API int gk_bpuct_root_expand(void* ws, int64_t trees, int capacity, int leaf_batch, int float_eval,
                                void* stream);
/* One wave's selection (BatchedPUCT.cpp:377-404): per tree, leaves until the
 * wave holds min(simulations left, leaf_batch); finished leaves are backed up
 * at once. Also zeroes *remaining. */
GK_API int gk_bpuct_collect(void* ws, int64_t trees, int capacity, int leaf_batch, double c_puct, void* stream);
/* The injected evaluator (include/gk_common.h) on every slot that needs one;
 * stands in for the reference's batch callback (BatchedPUCT.cpp:252-268). */
GK_API int gk_bpuct_hash_eval(void* ws, int64_t trees, int capacity, int leaf_batch, void* stream);
/* Device-side list of the slots that need an evaluation (active, active_count):
 * the positions vector of BatchedPUCT.cpp:381-401, without a host round trip. */
GK_API int gk_bpuct_compact(void* ws, int64_t trees, int capacity, int leaf_batch, void* stream);
/* One wave's expansion, release and backup in collection order
 * (BatchedPUCT.cpp:405-413); a rejected evaluation (BatchedPUCT.cpp:72-81,
 * 233-236) sets GK_ERR_BAD_EVAL, GK_BPUCT_ERR_POLICY or GK_BPUCT_ERR_NO_WEIGHT
 * on its tree. */
GK_API int gk_bpuct_expand(void* ws, int64_t trees, int capacity, int leaf_batch, int float_eval, void* stream);
/* Results of the search (BatchedPUCT.cpp:415-434); failed trees are cleared. */
GK_API int gk_bpuct_finish(void* ws, int64_t trees, int capacity, int leaf_batch, const gk_bpuct_results_t* out,
                           void* stream);
/* BatchedPUCT::advance (BatchedPUCT.cpp:290-326) of the trees with mask[t] != 0
 * by actions[t]: advanced[t] = 1 when the subtree was kept; an illegal action
 * leaves the tree as it is; a legal one without a child clears it. */
GK_API int gk_bpuct_advance(void* ws, int64_t trees, int capacity, int leaf_batch, const int32_t* actions,
                            const uint8_t* mask, int reuse, uint8_t* advanced, void* stream);
/* A whole search with the injected evaluator in one launch (begin, waves,
 * finish): BatchedPUCT::search (BatchedPUCT.cpp:328-442) with the callback on the device. */
GK_API int gk_bpuct_search_hash(void* ws, int64_t trees, int capacity, int leaf_batch, const uint32_t* roots,
                                const uint8_t* mask, int simulations, int reuse, double c_puct,
                                const gk_bpuct_results_t* out, void* stream);
/* Copy every tree into a workspace with more nodes per tree (the reference's
 * node vector grows on demand, BatchedPUCT.cpp:183-185). */
GK_API int gk_bpuct_grow(const void* src, int capacity, void* dst, int new_capacity, int64_t trees,
                         int leaf_batch, void* stream);

/* --------------------------------------------------------------- replay */

/* Checks of a replay row, in the order the reference applies them
 * (python/kingdom_ai/replay.py:35-74, _validate_rows). */
#define GK_REPLAY_NONFINITE (1u << 0)    /* features or policy not finite */
#define GK_REPLAY_RANGE (1u << 1)        /* a feature outside [0, 1] */
#define GK_REPLAY_BINARY (1u << 2)       /* planes 0-5, 9 not 0/1 */
#define GK_REPLAY_SCALAR (1u << 3)       /* planes 5-8 not constant */
#define GK_REPLAY_ACTOR (1u << 4)        /* to_play not 1 or 2 */
#define GK_REPLAY_PERSPECTIVE (1u << 5)  /* plane 5 disagrees with to_play */
#define GK_REPLAY_TERMINAL (1u << 6)     /* passes plane not 0 or 0.5 */
#define GK_REPLAY_PASS (1u << 7)         /* pass not legal */
#define GK_REPLAY_MASK (1u << 8)         /* plane 9 disagrees with the mask */
#define GK_REPLAY_STONES (1u << 9)       /* stone planes overlap */
#define GK_REPLAY_NEUTRAL (1u << 10)     /* more than one neutral stone */
#define GK_REPLAY_TERRITORY (1u << 11)   /* territory planes overlap */
#define GK_REPLAY_POLICY (1u << 12)      /* negative or illegal policy mass */
#define GK_REPLAY_SUM (1u << 13)         /* policy sum not 1 within 1e-6 (summed in double) */
#define GK_REPLAY_VALUE (1u << 14)       /* value not -1 or +1 */

/* Validate n replay rows (features fp32[n,10,9,9], masks bool[n,82], policy
 * fp32[n,82], value fp32[n], to_play int8[n]): *violations (device) is set to
 * the OR over rows of the GK_REPLAY_* checks they fail; the lowest set bit is
 * the reference's error. One pass over the rows on the GPU. Replaces the CPU
 * _validate_rows of ReplayBuffer.extend (python/kingdom_ai/replay.py:35-74,
 * 133-161). */
GK_API int gk_replay_validate(const float* features, const uint8_t* masks, const float* policy, const float* value,
                              const int8_t* to_play, int64_t n, uint32_t* violations, void* stream);

/* CUDA-event timer for kernel launches inside gk_selfplay_ply: a host object
 * holding `pairs` start/stop event pairs (NULL on failure). No reference
 * counterpart: the reference times phases with perf_counter (loop.py:563-621). */
GK_API void* gk_timer_create(int pairs);

/* Destroy a timer and its events. No reference counterpart (see gk_timer_create). */
GK_API void gk_timer_destroy(void* timer);

/* Forget recorded pairs so the next plies start from the first pair. No
 * reference counterpart (see gk_timer_create). */
GK_API void gk_timer_reset(void* timer);

/* Sum of the recorded pairs' elapsed times; the stream must be synchronised.
 * No reference counterpart (see gk_timer_create). */
GK_API int gk_timer_read(void* timer, double* total_ms, int* pairs);

#ifdef __cplusplus
}
#endif
#endif /* GK_H */
