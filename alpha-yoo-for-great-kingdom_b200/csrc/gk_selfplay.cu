// gk_selfplay.cu - continuous batched self-play on one GPU.
//
// B lanes each play games back to back. One ply = one PUCT search per lane
// (root evaluation, root noise, `simulations` x select / evaluate /
// expand-backup, all with the native network) followed by one move per lane.
// The host issues one call per ply and never synchronises inside it.
//
// Semantics follow the reference's GPU self-play collection
// (python/kingdom_ai/gpu_training.py:40-121):
//   * the policy target is raw root visits / simulations, recorded before the
//     move is chosen (:69-70);
//   * moves are sampled from visits^(1/T) for the first `temperature_moves`
//     plies of each game and are the search's best action afterwards (:71-81);
//   * a finished game's samples get value +1 for the winner's turns and -1
//     otherwise (:114-117) and go into a FIFO replay ring laid out like the
//     CPU ReplayBuffer (python/kingdom_ai/replay.py:106-125);
//   * the actions played are kept per lane and logged with the finished game,
//     so the game replays from the start position (record_history, :50-51,
//     :89-90, :113).
// Random streams are keyed by (seed, game id, ply) - not by lane or GPU -
// so a game's moves do not depend on how games are sharded across GPUs.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <new>

#include "../../include/gk.h"
#include "gk_device.cuh"
#include "gk_launch.cuh"
#include "gk_puct.cuh"
#include "gk_random.cuh"

namespace gk {

constexpr int kHist = GK_MAX_PLIES + 2;  // plies of history per lane
constexpr uint64_t kNoiseSalt = 0x6A09E667F3BCC909ULL;
constexpr uint64_t kSampleSalt = 0x9E3779B97F4A7C15ULL;  // python/kingdom_ai/gpu_training.py:25

enum Counter { kMoves = 0, kGames, kRows, kErrors, kBlackWins, kWhiteWins, kCaptureEnds, kEvaluations, kCounters };

struct SelfPlayView {
    gk_bits* states;               // [B] current position of each lane
    int32_t* lane_ply;             // [B] plies played in the lane's current game
    uint64_t* game_id;             // [B]
    gk_bits* hist_bits;            // [kHist][B]
    float* hist_policy;            // [kHist][B][82]
    uint8_t* hist_action;          // [kHist][B] action played at each ply
    int32_t* last_action;          // [B] action played in the last ply (-1: none)
    float* last_policy;            // [B][82] visit shares of the last ply's search
    int64_t* best;                 // [B] best action of the last search
    unsigned long long* counters;  // [kCounters]
};

inline size_t selfplay_layout(void* base, int64_t B, SelfPlayView* v) {
    size_t off = 0;
    char* b = static_cast<char*>(base);
    auto take = [&](size_t bytes) -> void* {
        void* p = b ? b + off : nullptr;
        off = align256(off + bytes);
        return p;
    };
    SelfPlayView t;
    t.states = (gk_bits*)take(B * sizeof(gk_bits));
    t.lane_ply = (int32_t*)take(B * 4);
    t.game_id = (uint64_t*)take(B * 8);
    t.hist_bits = (gk_bits*)take((size_t)kHist * B * sizeof(gk_bits));
    t.hist_policy = (float*)take((size_t)kHist * B * GK_ACTIONS * 4);
    t.hist_action = (uint8_t*)take((size_t)kHist * B);
    t.last_action = (int32_t*)take(B * 4);
    t.last_policy = (float*)take((size_t)B * GK_ACTIONS * 4);
    t.best = (int64_t*)take(B * 8);
    t.counters = (unsigned long long*)take(kCounters * 8);
    if (v) *v = t;
    return off;
}

struct ReplayView {
    float* features;
    uint8_t* masks;
    float* policy;
    float* value;
    int8_t* to_play;
    int64_t capacity;
};

struct GameLogView {
    uint64_t* game_id;
    uint64_t* first_row;
    int32_t* plies;
    int8_t* winner;
    int8_t* reason;
    gk_bits* final_state;
    uint8_t* actions;
    int64_t capacity;
};

__global__ void selfplay_reset_kernel(SelfPlayView v, int64_t B, int neutral, uint64_t first_game) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        v.states[b] = initial_bits(neutral);
        v.lane_ply[b] = 0;
        v.game_id[b] = first_game + (uint64_t)b;
        v.best[b] = -1;
        v.last_action[b] = -1;
    }
    if (blockIdx.x == 0 && threadIdx.x < kCounters) v.counters[threadIdx.x] = 0ull;
}

// Root noise keyed by (game, ply) so it is independent of lane and GPU.
__global__ void selfplay_noise_kernel(SelfPlayView v, PuctView p, int64_t B, int C, uint64_t seed, double alpha) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        gk_pcg32 r = gk_pcg32_seed(seed ^ kNoiseSalt, v.game_id[b] * 256u + (uint64_t)v.lane_ply[b]);
        root_noise(p.node_state[b * C], alpha, r, p.noise + b * GK_ACTIONS, p.root_allow + b * 3);
    }
}

struct AdvanceParams {
    int temperature_moves;
    double temperature, final_temperature;
    uint64_t sample_seed, game_stride, game_limit;
    int neutral;
};

__device__ __forceinline__ float encoded_value(const EncodePlanes& e, int plane, int cell) {
    const int bit = cell + cell / 9;
    switch (plane) {
        case 0: return (float)gk_test(e.own, bit);
        case 1: return (float)gk_test(e.enemy, bit);
        case 2: return (float)gk_test(e.neutral, bit);
        case 3: return (float)gk_test(e.own_terr, bit);
        case 4: return (float)gk_test(e.enemy_terr, bit);
        case 5: return e.black_to_play;
        case 6: return e.own_remaining;
        case 7: return e.enemy_remaining;
        case 8: return e.passes;
        default: return (float)gk_test(e.legal, bit);
    }
}

__global__ void __launch_bounds__(128) selfplay_advance_kernel(SelfPlayView v, PuctView p, int64_t B, int C,
                                                               AdvanceParams ap, ReplayView rp, GameLogView gl) {
    constexpr unsigned kAll = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int64_t b = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    if (b >= B) return;
    const int ply = v.lane_ply[b];
    if (ply < 0 || (ap.game_limit != 0 && v.game_id[b] >= ap.game_limit)) {
        // Parked (the game limit was reached), or a lane that started past
        // the limit (more lanes than games): it plays nothing.
        if (lane == 0) {
            v.lane_ply[b] = -1;
            v.last_action[b] = -1;
        }
        return;
    }
    gk_bits s = v.states[b];
    if (ply >= kHist) {  // unreachable: no game outlasts 2*81+4 plies
        if (lane == 0) {
            atomicAdd(&v.counters[kErrors], 1ull);
            v.states[b] = initial_bits(ap.neutral);
            v.lane_ply[b] = 0;
            v.game_id[b] += ap.game_stride;
        }
        return;
    }
    const int64_t ebase = b * (int64_t)C * GK_ACTIONS;  // root node's edges
    const bool expanded = p.expanded[b * (int64_t)C] != 0;
    const int sims = p.sims[b];
    int n[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int a = lane + 32 * k;
        n[k] = (expanded && a < GK_ACTIONS) ? p.visits[ebase + a] : 0;
    }
    // Policy target: raw visit proportions, before temperature.
    float* hp = v.hist_policy + ((int64_t)ply * B + b) * GK_ACTIONS;
    float* lp = v.last_policy + b * GK_ACTIONS;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int a = lane + 32 * k;
        if (a < GK_ACTIONS) hp[a] = lp[a] = sims > 0 ? __fdiv_rn((float)n[k], (float)sims) : 0.0f;
    }
    if (lane == 0) v.hist_bits[(int64_t)ply * B + b] = s;

    const double temperature = ply < ap.temperature_moves ? ap.temperature : ap.final_temperature;
    int action = (int)v.best[b];
    if (temperature != 0.0 && sims > 0) {
        gk_pcg32 r = gk_pcg32_seed(ap.sample_seed ^ kSampleSalt, v.game_id[b] * 256u + (uint64_t)ply);
        double w[3];
        int nmax = max(n[0], max(n[1], n[2]));
#pragma unroll
        for (int off = 16; off; off >>= 1) nmax = max(nmax, __shfl_xor_sync(kAll, nmax, off));
        // exp((log n - log n_max) / T) as in gpu_training.py:28-37; T == 1 is exactly n / n_max.
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            if (n[k] <= 0) w[k] = 0.0;
            else if (temperature == 1.0) w[k] = (double)n[k];
            else w[k] = exp((log((double)n[k]) - log((double)nmax)) / fmax(temperature, 2.2250738585072014e-308));
        }
        double total = 0.0;
        for (int a = 0; a < GK_ACTIONS; ++a) {
            const int k = a >> 5;
            total += __shfl_sync(kAll, k == 0 ? w[0] : k == 1 ? w[1] : w[2], a & 31);
        }
        double u = 0.0;
        if (lane == 0) u = temperature == 1.0 ? (double)gk_pcg32_bounded(&r, (uint32_t)sims) : uniform01(r) * total;
        u = __shfl_sync(kAll, u, 0);
        double carry = 0.0;
        int chosen = -1;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            double x = w[k];
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const double y = __shfl_up_sync(kAll, x, off);
                if (lane >= off) x += y;
            }
            const double incl = carry + x, excl = incl - w[k];
            const bool hit = w[k] > 0.0 && u >= excl && u < incl;
            const unsigned m = __ballot_sync(kAll, hit);
            if (chosen < 0 && m) chosen = (__ffs(m) - 1) + 32 * k;
            carry += __shfl_sync(kAll, x, 31);
        }
        if (chosen >= 0) action = chosen;
    }
    int finished = 0, winner = 0;
    if (lane == 0) {
        const bool ok = play(s, action);
        if (!ok) atomicAdd(&v.counters[kErrors], 1ull);
        v.hist_action[(int64_t)ply * B + b] = (uint8_t)(action >= 0 && action < GK_ACTIONS ? action : 255);
        v.last_action[b] = action;
        atomicAdd(&v.counters[kMoves], 1ull);
        atomicAdd(&v.counters[kEvaluations], (unsigned long long)p.evals[b]);
        finished = gk_reason(&s) != GK_NONE;
        winner = gk_winner(&s);
    }
    finished = __shfl_sync(kAll, finished, 0);
    winner = __shfl_sync(kAll, winner, 0);
    if (!finished) {
        if (lane == 0) {
            v.states[b] = s;
            v.lane_ply[b] = ply + 1;
        }
        return;
    }
    const int rows = ply + 1;
    unsigned long long base = 0, order = 0;
    if (lane == 0) {
        base = atomicAdd(&v.counters[kRows], (unsigned long long)rows);
        order = atomicAdd(&v.counters[kGames], 1ull);
        atomicAdd(&v.counters[winner == 1 ? kBlackWins : kWhiteWins], 1ull);
        if (gk_reason(&s) == GK_CAPTURE) atomicAdd(&v.counters[kCaptureEnds], 1ull);
    }
    base = __shfl_sync(kAll, base, 0);
    order = __shfl_sync(kAll, order, 0);
    if (gl.capacity > 0) {
        const int64_t slot = (int64_t)(order % (unsigned long long)gl.capacity);
        for (int k = lane; k < rows; k += 32)
            gl.actions[slot * GK_GAME_ACTIONS + k] = v.hist_action[(int64_t)k * B + b];
        if (lane == 0) {  // only lane 0 played the move: its `s` is the final position
            gl.final_state[slot] = s;
            gl.game_id[slot] = v.game_id[b];
            gl.first_row[slot] = base;
            gl.plies[slot] = rows;
            gl.winner[slot] = (int8_t)winner;
            gl.reason[slot] = (int8_t)gk_reason(&s);
        }
    }
    if (rp.capacity > 0) {
        for (int k = 0; k < rows; ++k) {
            const int64_t row = (int64_t)((base + (unsigned long long)k) % (unsigned long long)rp.capacity);
            const gk_bits hs = v.hist_bits[(int64_t)k * B + b];
            const EncodePlanes e = encode_planes(hs);
            float* f = rp.features + row * GK_FEATURES;
            for (int i = lane; i < GK_FEATURES; i += 32) f[i] = encoded_value(e, i / GK_CELLS, i % GK_CELLS);
            const float* src = v.hist_policy + ((int64_t)k * B + b) * GK_ACTIONS;
            for (int a = lane; a < GK_ACTIONS; a += 32) {
                rp.policy[row * GK_ACTIONS + a] = src[a];
                rp.masks[row * GK_ACTIONS + a] =
                    a == GK_PASS ? (uint8_t)e.pass_legal : (uint8_t)gk_test(e.legal, a + a / 9);
            }
            if (lane == 0) {
                const int actor = gk_actor(&hs);
                rp.value[row] = actor == winner ? 1.0f : -1.0f;
                rp.to_play[row] = (int8_t)actor;
            }
        }
    }
    if (lane == 0) {
        const uint64_t next = v.game_id[b] + ap.game_stride;
        if (ap.game_limit != 0 && next >= ap.game_limit) {
            // Park on the finished position: later searches see a terminal
            // root and do no work for this lane.
            v.states[b] = s;
            v.lane_ply[b] = -1;
        } else {
            v.states[b] = initial_bits(ap.neutral);
            v.lane_ply[b] = 0;
            v.game_id[b] = next;
        }
    }
}

struct Timer {
    int capacity = 0, used = 0;
    cudaEvent_t* events = nullptr;  // 2 * capacity
};

}  // namespace gk

using namespace gk;

extern "C" {

size_t gk_selfplay_workspace_bytes(int64_t lanes) { return lanes <= 0 ? 0 : selfplay_layout(nullptr, lanes, nullptr); }

int gk_selfplay_reset(void* ws, int64_t lanes, int neutral_cell, uint64_t first_game, void* stream) {
    if (ws == nullptr || lanes <= 0) return GK_EINVAL;
    SelfPlayView v;
    selfplay_layout(ws, lanes, &v);
    selfplay_reset_kernel<<<blocks_for(lanes, 256, kSmCount * 8), 256, 0, as_stream(stream)>>>(
        v, lanes, neutral_cell >= 0 && neutral_cell < GK_CELLS ? neutral_cell : -1, first_game);
    return launch_status();
}

int gk_selfplay_buffers(void* ws, int64_t lanes, gk_selfplay_buffers_t* out) {
    if (ws == nullptr || lanes <= 0 || out == nullptr) return GK_EINVAL;
    SelfPlayView v;
    selfplay_layout(ws, lanes, &v);
    out->states = reinterpret_cast<uint32_t*>(v.states);
    out->lane_ply = v.lane_ply;
    out->game_id = v.game_id;
    out->counters = reinterpret_cast<uint64_t*>(v.counters);
    out->last_action = v.last_action;
    out->last_policy = v.last_policy;
    return 0;
}

void* gk_timer_create(int pairs) {
    if (pairs <= 0) return nullptr;
    Timer* t = new (std::nothrow) Timer();
    if (!t) return nullptr;
    t->events = static_cast<cudaEvent_t*>(std::calloc((size_t)pairs * 2, sizeof(cudaEvent_t)));
    if (!t->events) {
        delete t;
        return nullptr;
    }
    t->capacity = pairs;
    for (int i = 0; i < 2 * pairs; ++i) {
        if (cudaEventCreate(&t->events[i]) != cudaSuccess) {
            for (int j = 0; j < i; ++j) cudaEventDestroy(t->events[j]);
            std::free(t->events);
            delete t;
            return nullptr;
        }
    }
    return t;
}

void gk_timer_destroy(void* timer) {
    Timer* t = static_cast<Timer*>(timer);
    if (!t) return;
    for (int i = 0; i < 2 * t->capacity; ++i) cudaEventDestroy(t->events[i]);
    std::free(t->events);
    delete t;
}

void gk_timer_reset(void* timer) {
    if (timer) static_cast<Timer*>(timer)->used = 0;
}

int gk_timer_read(void* timer, double* total_ms, int* pairs) {
    Timer* t = static_cast<Timer*>(timer);
    if (!t || !total_ms || !pairs) return GK_EINVAL;
    double sum = 0.0;
    for (int i = 0; i < t->used; ++i) {
        float ms = 0.0f;
        const cudaError_t e = cudaEventElapsedTime(&ms, t->events[2 * i], t->events[2 * i + 1]);
        if (e != cudaSuccess) return (int)e;
        sum += ms;
    }
    *total_ms = sum;
    *pairs = t->used;
    return 0;
}

int gk_selfplay_ply(void* sp_ws, void* puct_ws, int64_t lanes, const gk_net_t* net, const gk_selfplay_params_t* prm,
                    const gk_replay_t* replay, const gk_gamelog_t* games, float* headfeat, uint32_t* status,
                    void* timer, void* stream) {
    if (sp_ws == nullptr || puct_ws == nullptr || lanes <= 0 || prm == nullptr ||
        (net != nullptr && headfeat == nullptr) || status == nullptr || prm->simulations < 1)
        return GK_EINVAL;
    const cudaStream_t st = as_stream(stream);
    const int C = prm->simulations + 1;
    SelfPlayView v;
    selfplay_layout(sp_ws, lanes, &v);
    PuctView pv;
    puct_layout(puct_ws, lanes, C, &pv);
    Timer* tm = static_cast<Timer*>(timer);
    auto evaluate = [&]() -> int {
        if (net == nullptr) return gk_puct_hash_eval(puct_ws, lanes, C, stream);
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        if (tm && tm->used < tm->capacity) {
            e0 = tm->events[2 * tm->used];
            e1 = tm->events[2 * tm->used + 1];
            ++tm->used;
        }
        return net_evaluate(net, puct_ws, lanes, C, headfeat, status, st, e0, e1);
    };
    gk_puct_options o{prm->c_puct, prm->dirichlet_epsilon, prm->fpu_enabled, prm->fpu_reduction};
    int s = gk_puct_begin(puct_ws, lanes, C, reinterpret_cast<const uint32_t*>(v.states), stream);
    if (s) return s;
    if (prm->tactical_checks && (s = gk_puct_root_tactics(puct_ws, lanes, C, stream))) return s;
    if ((s = evaluate())) return s;
    if (prm->dirichlet_epsilon != 0.0) {
        selfplay_noise_kernel<<<blocks_for(lanes, 128, kSmCount * 8), 128, 0, st>>>(v, pv, lanes, C, prm->seed,
                                                                                     prm->dirichlet_alpha);
        if ((s = launch_status())) return s;
    }
    if ((s = gk_puct_expand_backup(puct_ws, lanes, C, &o, 0, stream))) return s;
    for (int i = 0; i < prm->simulations; ++i) {
        if ((s = gk_puct_select(puct_ws, lanes, C, &o, stream))) return s;
        if ((s = evaluate())) return s;
        if ((s = gk_puct_expand_backup(puct_ws, lanes, C, &o, 1, stream))) return s;
    }
    gk_puct_results_t res{};
    res.actions = v.best;
    res.status = status;
    if ((s = gk_puct_finish(puct_ws, lanes, C, &res, stream))) return s;
    AdvanceParams ap{prm->temperature_moves, prm->temperature, prm->final_temperature, prm->sample_seed,
                     prm->game_stride, prm->game_limit,
                     prm->neutral_cell >= 0 && prm->neutral_cell < GK_CELLS ? prm->neutral_cell : -1};
    ReplayView rp{};
    if (replay) rp = ReplayView{replay->features, replay->masks, replay->policy, replay->value, replay->to_play,
                                replay->capacity};
    GameLogView gl{};
    if (games) gl = GameLogView{games->game_id, games->first_row, games->plies, games->winner, games->reason,
                                reinterpret_cast<gk_bits*>(games->final_state), games->actions, games->capacity};
    const int64_t blocks = (lanes + 3) / 4;
    selfplay_advance_kernel<<<(int)blocks, 128, 0, st>>>(v, pv, lanes, C, ap, rp, gl);
    return launch_status();
}

}  // extern "C"
