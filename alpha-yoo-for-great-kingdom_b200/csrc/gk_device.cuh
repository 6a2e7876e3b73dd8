// gk_device.cuh - device-side rules on register-resident 96-bit bitboards.
//
// Every function here runs in one thread on one packed state (gk_bits, 64 B).
// The algorithms are bitboard restatements of the reference rules:
//   State::play            engine/src/State.cpp:92-167  (gpu_play, gpu_rules.py:185-252)
//   Board::territory       engine/src/Board.cpp:149-198 (gpu_claim_territory, gpu_rules.py:124-172)
//   legal placements       gpu_legal, gpu_rules.py:174-183
// Flood fills are iterated 4-neighbour dilations masked by the passable set
// (small regions: stone groups), or run-filling floods (large regions: the
// territory passes); the padding column (bit r*10+9) is outside every mask,
// so horizontal shifts need no column masks and row runs never join.
#pragma once

#include <cstdint>

#include "../../include/gk_common.h"

namespace gk {

__device__ __forceinline__ gk_b96 lowest_bit(gk_b96 a) {
    gk_b96 r = gk_b(0u, 0u, 0u);
    if (a.w[0]) r.w[0] = a.w[0] & (0u - a.w[0]);
    else if (a.w[1]) r.w[1] = a.w[1] & (0u - a.w[1]);
    else r.w[2] = a.w[2] & (0u - a.w[2]);
    return r;
}

// Index of the j-th (0-based) set bit of a 96-bit value, j < popcount.
__device__ __forceinline__ int select_bit(gk_b96 a, int j) {
    int word = 0;
    int c0 = __popc(a.w[0]);
    uint32_t v = a.w[0];
    if (j >= c0) {
        j -= c0;
        int c1 = __popc(a.w[1]);
        if (j >= c1) {
            j -= c1;
            v = a.w[2];
            word = 2;
        } else {
            v = a.w[1];
            word = 1;
        }
    }
    // Binary search inside the 32-bit word.
    int base = 0;
#pragma unroll
    for (int width = 16; width >= 1; width >>= 1) {
        uint32_t lowmask = (width == 32) ? 0xffffffffu : ((1u << width) - 1u);
        int c = __popc(v & lowmask);
        if (j >= c) {
            j -= c;
            v >>= width;
            base += width;
        }
    }
    return word * 32 + base;
}

// ---- run-filling flood for large regions -------------------------------------
// Within one row a region is a union of runs of set bits, and runs of
// different rows are separated by the zero padding column. Adding the seeds
// to the mask carries from each seed to the top of its run, so
// ((m + x) ^ m) & m | x is every cell from a seed up to the end of its run;
// the same on bit-reversed words covers the cells below the seed. A flood
// then alternates a full horizontal closure with one vertical step, and
// needs one iteration per vertical turn of the region instead of one per
// cell of its radius.

__device__ __forceinline__ gk_b96 add96(gk_b96 a, gk_b96 b) {
    gk_b96 r;
    asm("add.cc.u32 %0, %3, %6;\n\t"
        "addc.cc.u32 %1, %4, %7;\n\t"
        "addc.u32 %2, %5, %8;"
        : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2])
        : "r"(a.w[0]), "r"(a.w[1]), "r"(a.w[2]), "r"(b.w[0]), "r"(b.w[1]), "r"(b.w[2]));
    return r;
}

// Bit i -> bit 95 - i.
__device__ __forceinline__ gk_b96 rev96(gk_b96 a) { return gk_b(__brev(a.w[2]), __brev(a.w[1]), __brev(a.w[0])); }

__device__ __forceinline__ gk_b96 xor96(gk_b96 a, gk_b96 b) {
    return gk_b(a.w[0] ^ b.w[0], a.w[1] ^ b.w[1], a.w[2] ^ b.w[2]);
}

// Cells of mask m (mr = rev96(m)) in a horizontal run that holds a cell of x (x within m).
__device__ __forceinline__ gk_b96 run_fill(gk_b96 m, gk_b96 mr, gk_b96 x) {
    const gk_b96 up = gk_or(gk_and(xor96(add96(m, x), m), m), x);
    const gk_b96 xr = rev96(x);
    const gk_b96 down = rev96(gk_or(gk_and(xor96(add96(mr, xr), mr), mr), xr));
    return gk_or(up, down);
}

// Same result as gk_flood(m, seed) for any region, fastest for large ones.
__device__ __forceinline__ gk_b96 flood_runs(gk_b96 m, gk_b96 seed) {
    const gk_b96 mr = rev96(m);
    gk_b96 x = run_fill(m, mr, gk_and(seed, m));
    for (;;) {
        const gk_b96 fresh = gk_andnot(gk_and(gk_or(gk_shl(x, 10), gk_shr(x, 10)), m), x);
        if (!gk_any(fresh)) return x;
        x = gk_or(x, run_fill(m, mr, fresh));
    }
}

// Two floods of one mask from two seed sets, advanced in the same loop.
__device__ __forceinline__ void flood_runs2(gk_b96 m, gk_b96 sa, gk_b96 sb, gk_b96& ra, gk_b96& rb) {
    const gk_b96 mr = rev96(m);
    gk_b96 a = run_fill(m, mr, gk_and(sa, m)), b = run_fill(m, mr, gk_and(sb, m));
    for (;;) {
        const gk_b96 fa = gk_andnot(gk_and(gk_or(gk_shl(a, 10), gk_shr(a, 10)), m), a);
        const gk_b96 fb = gk_andnot(gk_and(gk_or(gk_shl(b, 10), gk_shr(b, 10)), m), b);
        if (!gk_any(gk_or(fa, fb))) break;
        a = gk_or(a, run_fill(m, mr, fa));
        b = gk_or(b, run_fill(m, mr, fb));
    }
    ra = a;
    rb = b;
}

__device__ __forceinline__ gk_b96 empty_cells(const gk_bits& s) {
    gk_b96 occ = gk_or(gk_or(gk_get(&s, GK_PLANE_BLACK), gk_get(&s, GK_PLANE_WHITE)), gk_get(&s, GK_PLANE_NEUTRAL));
    return gk_andnot(gk_valid(), occ);
}

// Legal placements of the player to move (not including pass); empty if finished.
__device__ __forceinline__ gk_b96 legal_placements(const gk_bits& s) {
    if (gk_reason(&s) != GK_NONE) return gk_b(0u, 0u, 0u);
    int actor = gk_actor(&s);
    if (gk_stock(&s, actor) <= 0) return gk_b(0u, 0u, 0u);
    gk_b96 owned = gk_or(gk_get(&s, GK_PLANE_OWN_BLACK), gk_get(&s, GK_PLANE_OWN_WHITE));
    return gk_andnot(empty_cells(s), owned);
}

// Board::territory + State::claim_territory on bitboards. A territory for
// player P is an empty component that (1) has no opponent-adjacent cell (the
// reference flood passes through enemy stones and rejects such components),
// (2) touches a P stone, (3) does not touch all four edges. Ownership is sticky.
__device__ __forceinline__ void claim_territory(gk_bits& s) {
    const gk_b96 black = gk_get(&s, GK_PLANE_BLACK), white = gk_get(&s, GK_PLANE_WHITE);
    const gk_b96 E = empty_cells(s);
    gk_b96 near_black, near_white;
    flood_runs2(E, gk_and(E, gk_neighbours(black)), gk_and(E, gk_neighbours(white)), near_black, near_white);
    gk_b96 pb = gk_andnot(near_black, near_white);
    gk_b96 pw = gk_andnot(near_white, near_black);
    const gk_b96 C = gk_or(pb, pw);
    if (!gk_any(C)) return;
    // Components touching all four edges: nested floods by edge.
    gk_b96 t = flood_runs(C, gk_and(C, gk_b(GK_ROW0_0, 0u, 0u)));
    if (gk_any(t)) t = flood_runs(t, gk_and(t, gk_b(0u, 0u, GK_ROW8_2)));
    if (gk_any(t)) t = flood_runs(t, gk_and(t, gk_b(GK_COL0_0, GK_COL0_1, GK_COL0_2)));
    if (gk_any(t)) t = flood_runs(t, gk_and(t, gk_b(GK_COL8_0, GK_COL8_1, GK_COL8_2)));
    pb = gk_andnot(pb, t);
    pw = gk_andnot(pw, t);
    const gk_b96 ob = gk_get(&s, GK_PLANE_OWN_BLACK), ow = gk_get(&s, GK_PLANE_OWN_WHITE);
    const gk_b96 unowned = gk_andnot(gk_valid(), gk_or(ob, ow));
    gk_put(&s, GK_PLANE_OWN_BLACK, gk_or(ob, gk_and(pb, unowned)));
    gk_put(&s, GK_PLANE_OWN_WHITE, gk_or(ow, gk_and(pw, unowned)));
}

__device__ __forceinline__ bool touches_four_edges(gk_b96 x) {
    return (x.w[0] & GK_ROW0_0) && (x.w[2] & GK_ROW8_2) &&
           ((x.w[0] & GK_COL0_0) | (x.w[1] & GK_COL0_1) | (x.w[2] & GK_COL0_2)) &&
           ((x.w[0] & GK_COL8_0) | (x.w[1] & GK_COL8_1) | (x.w[2] & GK_COL8_2));
}

// Union of the components of `m` that hold a cell of `seeds` and no cell of
// `hit` (with kEdges, and that do not touch all four edges). Each component
// grows one run closure and one vertical step at a time and is abandoned at
// its first `hit` cell; a seed on a `hit` cell settles its component at once.
// One loop runs over the steps of all components, so a thread's flood steps
// are not nested per component and the threads of a warp stay together.
template <bool kEdges>
__device__ __forceinline__ gk_b96 closed_components(gk_b96 m, gk_b96 hit, gk_b96 seeds) {
    gk_b96 result = gk_b(0u, 0u, 0u);
    seeds = gk_andnot(seeds, hit);
    if (!gk_any(seeds)) return result;
    const gk_b96 mr = rev96(m);
    gk_b96 x = gk_b(0u, 0u, 0u), f = lowest_bit(seeds);
    for (;;) {
        x = gk_or(x, run_fill(m, mr, f));
        if (gk_any(gk_and(x, hit))) {
            f = gk_b(0u, 0u, 0u);
            seeds = gk_andnot(seeds, x);
            x = f;
        } else {
            f = gk_andnot(gk_and(gk_or(gk_shl(x, 10), gk_shr(x, 10)), m), x);
            if (gk_any(f)) continue;
            // x is a whole component without a `hit` cell.
            if (!kEdges || !touches_four_edges(x)) result = gk_or(result, x);
            seeds = gk_andnot(seeds, x);
            x = f;
        }
        if (!gk_any(seeds)) return result;
        f = lowest_bit(seeds);
    }
}

// The same claim after a placement of `mover` next to the empty cells
// `around`, for a state whose territory was settled before the move
// (GK_META_SETTLED: every qualifying empty component already owned). No
// stone is removed by a non-final move, so an empty component that does not
// touch the new stone keeps its neighbours and its edges, qualifies exactly
// as before and is already owned. Only the pieces of the component the stone
// split are examined: each touches the mover's new stone, so it is territory
// of the mover unless it reaches a cell next to an enemy stone or touches all
// four edges. `E` is the empty set after the move.
__device__ __forceinline__ void claim_around(gk_bits& s, gk_b96 around, gk_b96 E, gk_b96 enemy, int mover) {
    const gk_b96 gained = closed_components<true>(E, gk_and(E, gk_neighbours(enemy)), gk_and(around, E));
    if (!gk_any(gained)) return;
    const gk_b96 ob = gk_get(&s, GK_PLANE_OWN_BLACK), ow = gk_get(&s, GK_PLANE_OWN_WHITE);
    const gk_b96 unowned = gk_andnot(gk_valid(), gk_or(ob, ow));
    if (mover == 1) gk_put(&s, GK_PLANE_OWN_BLACK, gk_or(ob, gk_and(gained, unowned)));
    else gk_put(&s, GK_PLANE_OWN_WHITE, gk_or(ow, gk_and(gained, unowned)));
}

// One transition; returns false (state unchanged) for rejected actions.
__device__ __forceinline__ bool play(gk_bits& s, int action) {
    const uint32_t meta = s.w[15];
    if (((meta >> GK_META_REASON_SHIFT) & 3u) != GK_NONE) return false;
    if (action < 0 || action >= GK_ACTIONS) return false;
    const int actor = (int)(meta & 3u);
    const int enemy = 3 - actor;
    int bstock = (int)((meta >> GK_META_BSTOCK_SHIFT) & 63u);
    int wstock = (int)((meta >> GK_META_WSTOCK_SHIFT) & 63u);
    int passes = (int)((meta >> GK_META_PASSES_SHIFT) & 3u);
    if (action == GK_PASS) {
        ++passes;
        int reason = GK_NONE, winner = gk_winner(&s);
        if (passes == 2) {
            const gk_b96 E = empty_cells(s);
            const int b = gk_popc(gk_and(E, gk_get(&s, GK_PLANE_OWN_BLACK)));
            const int w = gk_popc(gk_and(E, gk_get(&s, GK_PLANE_OWN_WHITE)));
            reason = GK_TWO_PASSES;
            winner = b - w >= 3 ? 1 : 2;
        }
        const int captured = reason == GK_NONE ? gk_captured(&s) : 0;
        s.w[15] = gk_pack_meta(enemy, bstock, wstock, passes, reason, winner, captured) |
                  (meta & 0xf8000000u);
        return true;
    }
    const int bit = gk_cell_bit(action);
    const gk_b96 here = gk_single(bit);
    gk_b96 black = gk_get(&s, GK_PLANE_BLACK), white = gk_get(&s, GK_PLANE_WHITE);
    const gk_b96 neutral = gk_get(&s, GK_PLANE_NEUTRAL);
    const gk_b96 owned = gk_or(gk_get(&s, GK_PLANE_OWN_BLACK), gk_get(&s, GK_PLANE_OWN_WHITE));
    const int stock = actor == 1 ? bstock : wstock;
    if (gk_test(gk_or(gk_or(black, white), gk_or(neutral, owned)), bit) || stock <= 0) return false;
    gk_b96 own = actor == 1 ? black : white;
    gk_b96 opp = actor == 1 ? white : black;
    own = gk_or(own, here);
    const gk_b96 E = gk_andnot(gk_valid(), gk_or(gk_or(own, opp), neutral));
    const gk_b96 lib = gk_neighbours(E);  // cells next to an empty cell
    const gk_b96 around = gk_neighbours(here);
    // Enemy groups next to the new stone with no liberty are captured.
    const gk_b96 captured = closed_components<false>(opp, gk_and(opp, lib), gk_and(around, opp));
    const int captured_count = gk_popc(captured);
    bool suicide = false;
    if (captured_count == 0) suicide = gk_any(closed_components<false>(own, gk_and(own, lib), here));
    if (actor == 1) --bstock;
    else --wstock;
    opp = gk_andnot(opp, captured);
    gk_put(&s, actor == 1 ? GK_PLANE_BLACK : GK_PLANE_WHITE, own);
    gk_put(&s, actor == 1 ? GK_PLANE_WHITE : GK_PLANE_BLACK, opp);
    int reason = GK_NONE, winner = gk_winner(&s), captured_field = gk_captured(&s);
    if (captured_count > 0) {
        reason = GK_CAPTURE;
        winner = actor;
        captured_field = captured_count;
    } else if (suicide) {
        reason = GK_SUICIDE;
        winner = enemy;
        captured_field = 0;
    }
    s.w[15] = gk_pack_meta(enemy, bstock, wstock, 0, reason, winner, captured_field) | (meta & 0xf8000000u);
    if (reason == GK_NONE) {
        if (meta & GK_META_SETTLED) claim_around(s, around, E, opp, actor);
        else claim_territory(s);
        s.w[15] |= GK_META_SETTLED;
    }
    return true;
}

__device__ __forceinline__ gk_bits initial_bits(int neutral_cell) {
    gk_bits s;
#pragma unroll
    for (int i = 0; i < 16; ++i) s.w[i] = 0u;
    if (neutral_cell >= 0 && neutral_cell < GK_CELLS) gk_put(&s, GK_PLANE_NEUTRAL, gk_single(gk_cell_bit(neutral_cell)));
    // No black or white stone: no territory, so the state is settled.
    s.w[15] = gk_pack_meta(1, GK_STONES, GK_STONES, 0, GK_NONE, 0, 0) | GK_META_SETTLED;
    return s;
}

// Wire record (int32[170], possibly in shared memory) -> packed state.
__device__ __forceinline__ gk_bits pack_record(const int32_t* rec) {
    gk_bits s;
#pragma unroll
    for (int i = 0; i < 16; ++i) s.w[i] = 0u;
    for (int i = 0; i < GK_CELLS; ++i) {
        const int bit = gk_cell_bit(i);
        const uint32_t m = 1u << (bit & 31);
        const int word = bit >> 5;
        const int c = rec[i];
        if (c == 1) s.w[word] |= m;
        else if (c == 2) s.w[3 + word] |= m;
        else if (c == 3) s.w[6 + word] |= m;
        const int o = rec[GK_CELLS + i];
        if (o == 1) s.w[9 + word] |= m;
        else if (o == 2) s.w[12 + word] |= m;
    }
    s.w[15] = gk_pack_meta(rec[GK_ACTOR] & 3, rec[GK_BLACK_STOCK] & 63, rec[GK_WHITE_STOCK] & 63,
                           rec[GK_PASSES] & 3, rec[GK_REASON] & 3, rec[GK_WINNER] & 3, rec[GK_CAPTURED] & 127);
    return s;
}

// True when the record's fields lie inside the ranges the packed state holds.
__device__ __forceinline__ bool record_in_range(const int32_t* rec) {
    bool ok = true;
    for (int i = 0; i < GK_CELLS; ++i) {
        ok &= (unsigned)rec[i] <= 3u;
        ok &= (unsigned)rec[GK_CELLS + i] <= 2u;
    }
    ok &= rec[GK_ACTOR] == 1 || rec[GK_ACTOR] == 2;
    ok &= (unsigned)rec[GK_BLACK_STOCK] <= 41u && (unsigned)rec[GK_WHITE_STOCK] <= 41u;
    ok &= (unsigned)rec[GK_PASSES] <= 2u && (unsigned)rec[GK_REASON] <= 3u;
    ok &= (unsigned)rec[GK_WINNER] <= 2u && (unsigned)rec[GK_CAPTURED] <= 81u;
    return ok;
}

// Packed state -> wire record fields 0..168 (169, reserved, is left alone).
__device__ __forceinline__ void unpack_record(const gk_bits& s, int32_t* rec) {
    for (int i = 0; i < GK_CELLS; ++i) {
        const int bit = gk_cell_bit(i);
        const int word = bit >> 5, sh = bit & 31;
        const int b = (s.w[word] >> sh) & 1u, w = (s.w[3 + word] >> sh) & 1u, n = (s.w[6 + word] >> sh) & 1u;
        rec[i] = b ? 1 : w ? 2 : n ? 3 : 0;
        const int ob = (s.w[9 + word] >> sh) & 1u, ow = (s.w[12 + word] >> sh) & 1u;
        rec[GK_CELLS + i] = ob ? 1 : ow ? 2 : 0;
    }
    rec[GK_ACTOR] = gk_actor(&s);
    rec[GK_BLACK_STOCK] = gk_stock(&s, 1);
    rec[GK_WHITE_STOCK] = gk_stock(&s, 2);
    rec[GK_PASSES] = gk_passes(&s);
    rec[GK_REASON] = gk_reason(&s);
    rec[GK_WINNER] = gk_winner(&s);
    rec[GK_CAPTURED] = gk_captured(&s);
}

// Actor-relative planes used by the encoder and by the network's stem.
struct EncodePlanes {
    gk_b96 own, enemy, neutral, own_terr, enemy_terr, legal;
    float black_to_play, own_remaining, enemy_remaining, passes;
    bool pass_legal;
};

__device__ __forceinline__ EncodePlanes encode_planes(const gk_bits& s) {
    EncodePlanes p;
    const int actor = gk_actor(&s);
    const gk_b96 black = gk_get(&s, GK_PLANE_BLACK), white = gk_get(&s, GK_PLANE_WHITE);
    const gk_b96 ob = gk_get(&s, GK_PLANE_OWN_BLACK), ow = gk_get(&s, GK_PLANE_OWN_WHITE);
    p.own = actor == 1 ? black : white;
    p.enemy = actor == 1 ? white : black;
    p.neutral = gk_get(&s, GK_PLANE_NEUTRAL);
    p.own_terr = actor == 1 ? ob : ow;
    p.enemy_terr = actor == 1 ? ow : ob;
    p.legal = legal_placements(s);
    p.pass_legal = gk_reason(&s) == GK_NONE;
    p.black_to_play = actor == 1 ? 1.0f : 0.0f;
    // float(double(k) / 41.0) as in mcts/src/BatchedPUCT.cpp:34-35.
    p.own_remaining = (float)((double)gk_stock(&s, actor) / 41.0);
    p.enemy_remaining = (float)((double)gk_stock(&s, 3 - actor) / 41.0);
    p.passes = (float)gk_passes(&s) * 0.5f;
    return p;
}

}  // namespace gk
