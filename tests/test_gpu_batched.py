"""Batched evaluation search on the GPU (GpuBatchedPUCT, csrc/gk_bpuct.cu)
against the reference's kingdom::BatchedPUCT (mcts/src/BatchedPUCT.cpp).

The evaluation games in tests/golden/batched.npz were played by the
reference's own searcher; here every tree of a GpuBatchedPUCT replays one
game, all games of a configuration searched together, and every result field
and statistic must match bit for bit. The reference's tests
(tests/batched_puct_test.cpp) are replayed with their fixed evaluator as a
device callback.
"""

import sys

import numpy as np
import pytest
import torch

from test_oracle import batched_games, split_board_record

pytestmark = pytest.mark.gpu


# (i + 1) / 81 by true division, as the reference computes it (a CUDA tensor
# divided by a scalar is multiplied by the reciprocal, which can differ in the
# last bit).
RAMP = torch.tensor([(i + 1) / 81.0 for i in range(81)] + [0.0], dtype=torch.float64)


def ramp(features, masks):
    """tests/batched_puct_test.cpp:21-28 on the device: weight (i + 1) / 81 on
    cell i, none on pass; value 0.25 with Black to play, else -0.5."""
    n = features.shape[0]
    weights = RAMP.to(features.device).expand(n, -1).clone()
    values = torch.where(features[:, 5, 0, 0] != 0, 0.25, -0.5).to(torch.float64)
    return weights, values


def uniform(features, masks):
    n = features.shape[0]
    return (torch.ones((n, 82), dtype=torch.float64, device=features.device),
            torch.zeros(n, dtype=torch.float64, device=features.device))


def evaluator(kind):
    from kingdom_ai import HashEvaluator
    return {"hash": HashEvaluator(), "uniform": uniform, "ramp": ramp}[kind]


def searcher(trees, sims, leaf=8, reuse=True, c=1.5, **options):
    from kingdom_ai.batched_puct import GpuBatchedPUCT, PUCTOptions
    return GpuBatchedPUCT(trees, PUCTOptions(simulations=sims, c_puct=c, **options), leaf, reuse)


def packed(records):
    from kingdom_ai.gpu_rules import records_to_bits
    return records_to_bits(torch.from_numpy(np.ascontiguousarray(records, dtype=np.int32)).cuda())


def one(oracle_rec):
    return packed(np.asarray(oracle_rec)[None])


@pytest.mark.parametrize("fused", [True, False])
def test_golden_evaluation_games_bit_exact(golden, oracle, fused):
    from kingdom_ai.batched_puct import GpuBatchedPUCT, PUCTOptions, STAT_NAMES
    filler = oracle.initial(1)[0]
    checked = 0
    for g, ci, (sims, leaf, c, kind, reuse), games in batched_games(golden):
        T = len(games)
        # one configuration starts at the smallest capacity, so trees grow
        cap = sims + 1 if ci == 1 else None
        opts = PUCTOptions(simulations=sims, c_puct=c)
        pair = [GpuBatchedPUCT(T, opts, leaf, reuse, capacity=cap) for _ in range(2)]
        for s in pair:
            s._fuse_hash = fused
        ev = evaluator(kind)
        for ply in range(max(len(r) for r in games)):
            rows = np.asarray([r[ply] if ply < len(r) else -1 for r in games])
            live = rows >= 0
            recs = np.stack([g["root"][i] if i >= 0 else filler for i in rows])
            roots = packed(recs)
            actors = recs[:, 162]
            for who in (0, 1):
                active = live & (actors == (1 if who == 0 else 2))
                if not active.any():
                    continue
                r = pair[who].search(roots, ev, active=torch.from_numpy(active).cuda())
                stats = torch.stack([pair[who].stats[n] for n in STAT_NAMES], 1).cpu().numpy()
                for t in np.flatnonzero(active):
                    i = rows[t]
                    assert np.array_equal(r.visits[t].cpu().numpy(), g["visits"][i]), (ci, t, ply)
                    assert np.array_equal(r.priors[t].cpu().numpy(), g["priors"][i])
                    assert np.array_equal(r.move_values[t].cpu().numpy(), g["move_values"][i])
                    assert np.array_equal(r.legal[t].cpu().numpy().astype(np.uint8), g["legal"][i])
                    info = [r.actions[t].item(), r.simulations[t].item(), r.nodes[t].item(),
                            r.network_evaluations[t].item()]
                    assert info == g["info"][i].tolist(), (ci, t, ply)
                    assert [r.root_values[t].item(), r.best_values[t].item()] == g["values"][i].tolist()
                    assert stats[t].tolist() == g["stats"][i].tolist()
                    checked += 1
            live_t = torch.from_numpy(live).cuda()
            moves = np.where(live, g["move"][np.maximum(rows, 0)], 0)
            adv = [s.advance(torch.from_numpy(moves), active=live_t).cpu().numpy() for s in pair]
            for t in np.flatnonzero(live):
                assert [bool(adv[0][t]), bool(adv[1][t])] == g["advanced"][rows[t]].astype(bool).tolist()
            bad = np.where(live, g["bad_action"][np.maximum(rows, 0)], -100)
            has_bad = live & (bad != -100)
            if has_bad.any():
                mask = torch.from_numpy(has_bad).cuda()
                adv = [s.advance(torch.from_numpy(bad), active=mask).cpu().numpy() for s in pair]
                for t in np.flatnonzero(has_bad):
                    assert [bool(adv[0][t]), bool(adv[1][t])] == g["bad_advanced"][rows[t]].astype(bool).tolist()
            after = [torch.stack([s.stats[n] for n in STAT_NAMES], 1).cpu().numpy() for s in pair]
            for t in np.flatnonzero(live):
                assert [after[0][t].tolist(), after[1][t].tolist()] == g["stats_after"][rows[t]].tolist()
        if ci == 1:
            assert pair[0].capacity > sims + 1  # the workspace grew instead of truncating a tree
    assert checked == len(g["cfg"])


def test_reference_known_answers(oracle):
    """tests/batched_puct_test.cpp:89-209 on the GPU searcher."""
    # :89-115 budgets, one callback per batch, distinct positions per batch
    for count in (1, 7, 19, 301):
        calls, seen, largest = [], [0], [0]

        def counting(features, masks):
            calls.append(features.shape[0])
            assert 1 <= features.shape[0] <= 8
            assert torch.unique(features.reshape(features.shape[0], -1), dim=0).shape[0] == features.shape[0]
            return ramp(features, masks)

        s = searcher(1, count, leaf=8, reuse=False)
        r = s.search(one(oracle.initial(1)[0]), counting)
        st = {k: v.item() for k, v in s.stats.items()}
        assert r.simulations.item() == count and r.visits.sum().item() == count
        assert r.network_evaluations.item() == sum(calls) == st["network_evaluations"]
        assert st["inference_batches"] == len(calls) and st["max_observed_batch_size"] == max(calls)
        assert sum(calls) <= count + 1 and r.nodes.item() <= count + 1
        if count >= 8:
            assert max(calls) == 8
    # :117-150 reuse and per-search visits
    s = searcher(1, 64)
    root = oracle.initial(1)[0]
    first = s.search(one(root), ramp)
    assert s.stats["reused_nodes"].item() == 0
    repeated = s.search(one(root), ramp)
    assert s.stats["reused_nodes"].item() == first.nodes.item() and s.stats["inherited_visits"].item() == 64
    assert repeated.visits.sum().item() == 64 and repeated.network_evaluations.item() <= 64
    best = repeated.actions.item()
    assert s.advance([best]).item()
    root, _ = oracle.play(root[None].copy(), [best])
    after = s.search(one(root[0]), ramp)
    assert s.stats["reused_nodes"].item() > 0 and s.stats["inherited_visits"].item() > 0
    assert s.stats["advance_calls"].item() == 1 and s.stats["reuse_hits"].item() == 1
    assert after.visits.sum().item() == 64 and after.nodes.item() < repeated.nodes.item() + 65
    assert not s.advance([40]).item() and not s.advance([-1]).item()
    again = s.search(one(root[0]), ramp)
    assert s.stats["reused_nodes"].item() == after.nodes.item() and again.visits.sum().item() == 64
    assert s.stats["advance_calls"].item() == 3 and s.stats["reuse_hits"].item() == 1
    s.clear()
    assert s.search(one(root[0]), ramp).network_evaluations.item() > 0 and s.stats["reused_nodes"].item() == 0
    # :152-169 a state that differs in any field starts a new tree
    s = searcher(1, 16, leaf=4)
    start = oracle.initial(1)[0]
    s.search(one(start), ramp)
    passed, _ = oracle.play(start[None].copy(), [81])
    assert s.search(one(passed[0]), ramp).simulations.item() == 16 and s.stats["reused_nodes"].item() == 0
    setup = passed[0].copy()
    setup[165] = 0
    assert s.search(one(setup), ramp).simulations.item() == 16 and s.stats["reused_nodes"].item() == 0
    assert s.search(one(oracle.initial(1, -1)[0]), ramp).simulations.item() == 16
    assert s.stats["reused_nodes"].item() == 0
    # :171-209 capture values without the network, terminal roots
    for actor in (1, 2):
        calls = []
        s = searcher(1, 32)
        rec = split_board_record(oracle, actor)
        r = s.search(one(rec), lambda f, m: calls.append(1) or ramp(f, m))
        assert r.actions.item() == 40 and r.best_values.item() == 1.0 and r.visits.sum().item() == 32
        assert r.network_evaluations.item() == 1 and len(calls) == 1
        assert s.advance([40]).item()
        done, _ = oracle.play(rec[None].copy(), [40])
        t = s.search(one(done[0]), ramp)
        assert t.root_values.item() == -1.0 and t.actions.item() == -1
        assert s.stats["network_evaluations"].item() == 0
    two = oracle.initial(1)
    oracle.play(two, [81])
    oracle.play(two, [81])
    t = searcher(1, 8).search(one(two[0]), ramp)
    assert t.actions.item() == -1 and t.simulations.item() == 0 and not t.legal.any().item()
    assert t.root_values.item() == -1.0


def test_evaluation_failures_clear_the_tree_and_recover(oracle):
    """tests/batched_puct_test.cpp:211-260: a failing second batch leaves no
    reservations behind; the next search starts a fresh tree."""
    s = searcher(1, 16)
    root = one(oracle.initial(1)[0])
    for failure in range(5):
        calls = [0]

        def failing(features, masks):
            w, v = ramp(features, masks)
            calls[0] += 1
            if calls[0] == 2:
                if failure == 0:
                    raise RuntimeError("inference failed")
                if failure == 1:
                    return w[:-1], v[:-1]
                if failure == 2:
                    v[0] = float("nan")
                if failure == 3:
                    w[0, 0] = -1.0
                if failure == 4:
                    w[0].zero_()
            return w, v

        with pytest.raises((RuntimeError, ValueError)):
            s.search(root, failing)
        recovered = s.search(root, ramp)
        assert s.stats["reused_nodes"].item() == 0 and s.stats["inherited_visits"].item() == 0
        assert recovered.visits.sum().item() == 16
        s.clear()
    from kingdom_ai.batched_puct import GpuBatchedPUCT, PUCTOptions
    for bad in (dict(trees=1, leaf_batch_size=0), dict(trees=0), dict(trees=1, dirichlet=0.1)):
        with pytest.raises(ValueError):
            GpuBatchedPUCT(bad.get("trees", 1), PUCTOptions(simulations=8, dirichlet_epsilon=bad.get("dirichlet", 0.0)),
                           bad.get("leaf_batch_size", 8))


def test_deadline_and_large_finite_policy(oracle):
    """tests/batched_puct_test.cpp:253-290."""
    s = searcher(1, 100000, time_limit_ms=1)
    r = s.search(one(oracle.initial(1)[0]), ramp)
    assert 1 <= r.simulations.item() < 100000 and r.visits.sum().item() == r.simulations.item()
    big = sys.float_info.max

    def huge(features, masks):
        w, v = ramp(features, masks)
        return torch.full_like(w, big), v

    s = searcher(1, 16, leaf=4, reuse=False, c=big)
    r = s.search(one(oracle.initial(1)[0]), huge)
    assert r.visits.sum().item() == 16 and np.isfinite(r.root_values.item())
    assert torch.isfinite(r.priors).all().item()


def test_native_network_searches_many_games(oracle):
    """The tcgen05 network as the evaluator of 48 games at once, one searcher
    per game playing both colours: per tree the budget, legality, tree-size and
    statistics invariants of the reference search, and the played move's
    subtree carried into the next search."""
    from kingdom_ai.model import random_network
    T, sims = 48, 48
    net = random_network(64, 2, 13)
    s = searcher(T, sims, leaf=8)
    recs = oracle.gen_positions(5, T)
    previous = None
    for ply in range(8):
        live = recs[:, 166] == 0
        if not live.any():
            break
        r = s.search(packed(recs), net, active=torch.from_numpy(live).cuda())
        st = {k: v.cpu().numpy() for k, v in s.stats.items()}
        for t in np.flatnonzero(live):
            _, legal = oracle.encode(recs[t][None])
            assert np.array_equal(r.legal[t].cpu().numpy(), legal[0])
            assert r.visits[t].sum().item() == sims == r.simulations[t].item()
            assert legal[0][r.actions[t].item()]
            assert r.network_evaluations[t].item() == st["network_evaluations"][t] <= sims + 1
            assert r.nodes[t].item() <= st["reused_nodes"][t] + sims + 1
            # a tree whose every simulation ends in a finished game needs no batch
            assert st["max_observed_batch_size"][t] <= 8
            assert (st["max_observed_batch_size"][t] == 0) == (st["network_evaluations"][t] == 0)
            assert abs(r.root_values[t].item()) <= 1
            assert abs(r.priors[t].sum().item() - 1) < 1e-9
            if previous is not None:
                # the best move always has a child, so its subtree was kept
                # (with at least the visits this search gave it)
                assert st["reused_nodes"][t] >= 1 and st["inherited_visits"][t] >= previous[t]
        moves = r.actions.clamp(min=0).to(torch.int32)
        chosen = r.visits.gather(1, r.actions.clamp(min=0)[:, None]).flatten().cpu().numpy()
        advanced = s.advance(moves, active=torch.from_numpy(live).cuda()).cpu().numpy()
        assert advanced[live].all()
        previous = chosen
        for t in np.flatnonzero(live):
            nxt, ok = oracle.play(recs[t][None].copy(), [int(moves[t].item())])
            assert ok[0]
            recs[t] = nxt[0]
        previous = np.where(recs[:, 166] == 0, previous, -1)


def test_evaluation_games_between_models():
    """evaluate_models_gpu (evaluation.py:235-360 played on the GPU): with
    identical deterministic models every pair splits 1-1, because both games
    of a pair use the same seed (evaluation.py:252-256); counts are consistent
    from the candidate's side."""
    from kingdom_ai import evaluate_models_gpu
    from kingdom_ai.model import random_network
    same = random_network(64, 2, 21)
    r = evaluate_models_gpu(same, random_network(64, 2, 21), games=16, simulations=16, seed=9)
    assert r.games == 16 and r.wins == 8 and r.losses == 8 and r.win_rate == 0.5
    assert r.wins_as_black + r.wins_as_white == r.wins
    assert sum(r.endings.values()) == 16 and r.total_plies > 16
    other = evaluate_models_gpu(same, random_network(64, 2, 22), games=8, simulations=8, seed=3,
                                opening_moves=0)
    assert other.wins + other.losses == 8 and sum(other.endings.values()) == 8
    with pytest.raises(ValueError):
        evaluate_models_gpu(same, same, games=3)
