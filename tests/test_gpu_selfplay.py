"""Device-resident self-play engine: legality, replay rows, determinism, shard invariance."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def small_net(seed=3):
    from kingdom_ai.model import random_network
    return random_network(64, 2, seed)


def run_engine(lanes, plies, rank=0, world=1, seed=11, sims=16, replay=1 << 15, temperature_moves=4):
    from kingdom_ai.gpu_puct import GpuPUCTOptions
    from kingdom_ai.selfplay import SelfPlayEngine

    opts = GpuPUCTOptions(simulations=sims, c_puct=1.5, dirichlet_alpha=0.3, dirichlet_epsilon=0.25, seed=seed)
    engine = SelfPlayEngine(small_net(), lanes, opts, temperature_moves=temperature_moves, replay_capacity=replay,
                            rank=rank, world_size=world)
    engine.step(plies)
    torch.cuda.synchronize()
    engine.check()
    return engine


def rows_of(engine):
    n = engine.stats()["rows"]
    r = engine.replay
    n = min(n, r.capacity)
    return (r.features[:n].cpu().numpy(), r.masks[:n].cpu().numpy(), r.policy[:n].cpu().numpy(),
            r.value[:n].cpu().numpy(), r.to_play[:n].cpu().numpy())


def test_counters_and_replay_rows_are_consistent(oracle):
    lanes, plies = 96, 70
    engine = run_engine(lanes, plies)
    s = engine.stats()
    assert s["moves"] == lanes * plies and s["errors"] == 0
    assert s["games"] > 0 and s["black_wins"] + s["white_wins"] == s["games"]
    assert s["evaluations"] >= lanes * plies  # at least the root of every search
    feats, masks, policy, value, to_play = rows_of(engine)
    assert len(value) == s["rows"] > 0
    assert set(np.unique(value).tolist()) <= {-1.0, 1.0}
    assert set(np.unique(to_play).tolist()) <= {1, 2}
    # Observation planes are one-hot where they must be and agree with the mask.
    cells = feats[:, :3].reshape(len(feats), 3, 81)
    assert (cells.sum(axis=1) <= 1).all()
    assert np.array_equal(feats[:, 9].reshape(len(feats), 81) > 0, masks[:, :81])
    assert np.array_equal(feats[:, 5, 0, 0] == 1.0, to_play == 1)
    # Visit policies are distributions over legal actions only.
    assert np.allclose(policy.sum(axis=1), 1.0, atol=1e-5)
    assert (policy[~masks] == 0).all()


def keyset(rows):
    """Multiset of rows; games finishing in the same ply are written in atomic order."""
    feats, masks, policy, value, to_play = rows
    return sorted(hash((f.tobytes(), p.tobytes(), float(v), int(t)))
                  for f, p, v, t in zip(feats, policy, value, to_play))


def test_same_seed_same_games():
    a = run_engine(48, 40, seed=5)
    b = run_engine(48, 40, seed=5)
    assert a.stats() == b.stats()
    assert keyset(rows_of(a)) == keyset(rows_of(b))
    c = run_engine(48, 40, seed=6)
    assert keyset(rows_of(a)) != keyset(rows_of(c))


def test_games_do_not_depend_on_sharding():
    """One engine with 64 lanes = two ranks of 32 lanes: the same games, the same rows."""
    plies = 60
    whole = run_engine(64, plies, seed=9, temperature_moves=8)
    half0 = run_engine(32, plies, rank=0, world=2, seed=9, temperature_moves=8)
    half1 = run_engine(32, plies, rank=1, world=2, seed=9, temperature_moves=8)
    # Completed games are written in completion order, which differs between
    # layouts; compare the multisets of rows.
    w = rows_of(whole)
    h = [np.concatenate(parts) for parts in zip(rows_of(half0), rows_of(half1))]
    assert whole.stats()["games"] == half0.stats()["games"] + half1.stats()["games"]
    assert keyset(w) == keyset(h)


# --------------------------------------------------------------------------
# Parity of the engine's games against the oracle and the reference engine.

GPU_REASON, GPU_WINNER = 166, 167


def finished_games(engine):
    """Game log and replay rows of every game the engine finished (all in the ring)."""
    s = engine.stats()
    assert s["rows"] <= engine.replay.capacity and s["games"] <= engine.games.capacity
    log = engine.games.read(s["games"])
    return log, rows_of(engine)


@pytest.mark.parametrize("tactics", [False, True])
def test_injected_evaluator_games_equal_the_oracle_bit_for_bit(oracle, tactics):
    """No root noise, T = 1 for 10 plies then the best action: every finished
    game - its moves, visit-share targets, planes, masks, values and final
    position - equals the oracle's restatement of the same game id; with the
    root tactical checks on as well."""
    from kingdom_ai.gpu_puct import GpuPUCTOptions, HashEvaluator
    from kingdom_ai.gpu_rules import bits_to_records
    from kingdom_ai.selfplay import SelfPlayEngine

    lanes, plies, sims, seed = 256, 90, 32, 77
    opts = GpuPUCTOptions(simulations=sims, c_puct=1.5, dirichlet_epsilon=0.0, seed=3, tactical_checks=tactics)
    engine = SelfPlayEngine(HashEvaluator(), lanes, opts, temperature_moves=10, replay_capacity=1 << 16,
                            sample_seed=seed, game_log=4096)
    engine.step(plies)
    torch.cuda.synchronize()
    engine.check()
    log, (feats, masks, policy, value, to_play) = finished_games(engine)
    n = len(log["game_id"])
    assert n >= lanes, "every lane should finish at least one game in 90 plies"
    ids = log["game_id"].astype(np.int64)
    finals = bits_to_records(torch.from_numpy(log["final_state"]).cuda()).cpu().numpy()
    for gid in np.unique(ids):
        o_plies, o_actions, o_policy, o_final = oracle.selfplay_hash(seed, 1, sims, first_game=int(gid),
                                                                     tactics=tactics)
        slot = int(np.nonzero(ids == gid)[0][0])
        k, first = int(log["plies"][slot]), int(log["first_row"][slot])
        assert k == o_plies[0] > 0, gid
        assert np.array_equal(log["actions"][slot, :k], o_actions[0, :k]), gid
        assert np.array_equal(finals[slot], o_final[0]), gid
        assert int(log["winner"][slot]) == o_final[0, GPU_WINNER] and int(log["reason"][slot]) == o_final[0, GPU_REASON]
        rows = slice(first, first + k)
        assert np.array_equal(policy[rows], o_policy[0, :k]), gid
        # Replay the moves: each row holds the encoder's planes and mask of the position it was taken at.
        rec = oracle.initial(1)
        recs = []
        for a in o_actions[0, :k]:
            recs.append(rec.copy())
            rec, ok = oracle.play(rec, [int(a)])
            assert ok[0]
        ef, em = oracle.encode(np.concatenate(recs))
        assert np.array_equal(feats[rows], ef) and np.array_equal(masks[rows], em)
        movers = np.concatenate(recs)[:, 162]
        assert np.array_equal(to_play[rows], movers)
        assert np.array_equal(value[rows], np.where(movers == o_final[0, GPU_WINNER], 1.0, -1.0).astype(np.float32))


def test_engine_visit_targets_equal_gpupuct_searches(oracle):
    """Every position of every finished game, searched again by GpuPUCT with
    the same evaluator, gives the visit shares the engine recorded; where the
    engine played the best action (after ply 10) that is GpuPUCT's action."""
    from kingdom_ai.gpu_puct import GpuPUCT, GpuPUCTOptions, HashEvaluator
    from kingdom_ai.gpu_rules import GpuStateBatch
    from kingdom_ai.selfplay import SelfPlayEngine

    lanes, sims = 128, 48
    opts = GpuPUCTOptions(simulations=sims, c_puct=1.5, dirichlet_epsilon=0.0, seed=3)
    engine = SelfPlayEngine(HashEvaluator(), lanes, opts, temperature_moves=10, replay_capacity=1 << 15,
                            sample_seed=5, game_log=2048)
    engine.step(70)
    torch.cuda.synchronize()
    engine.check()
    log, (_, _, policy, _, _) = finished_games(engine)
    recs, targets, played, late = [], [], [], []
    for slot in range(len(log["game_id"])):
        k, first = int(log["plies"][slot]), int(log["first_row"][slot])
        rec = oracle.initial(1)
        for ply in range(k):
            a = int(log["actions"][slot, ply])
            recs.append(rec.copy())
            targets.append(policy[first + ply])
            played.append(a)
            late.append(ply >= 10)
            rec, ok = oracle.play(rec, [a])
            assert ok[0]
    recs = np.concatenate(recs)
    result = GpuPUCT(HashEvaluator(), opts).search(GpuStateBatch.from_records(recs))
    assert np.array_equal(result.policy.cpu().numpy(), np.stack(targets))
    late = np.array(late)
    assert np.array_equal(result.actions.cpu().numpy()[late], np.array(played)[late])
    # The oracle's search agrees on a sample of the positions.
    pick = np.arange(0, len(recs), max(1, len(recs) // 64))
    visits, best, _ = oracle.puct_batch(recs[pick], sims)
    assert np.array_equal(result.visits.cpu().numpy()[pick], visits)


@pytest.mark.parametrize("net,sims,plies", [("6x64", 400, 64), ("groupnorm32x2", 128, 80)])
def test_network_games_replay_in_the_reference_engine(oracle, reference, net, sims, plies):
    """C5 settings (6x64 network, Dirichlet 0.3 / 0.25, T = 1 for 10 plies then
    the best action, 400 simulations) on 256 lanes for 64 plies, and the
    Trainer's defaults (the reference's own 32 x 2 GroupNorm network, 128
    simulations): every finished game replays move by move in the reference's
    kingdom::State; every replay row carries that state's planes and mask, the
    mover, and +1 exactly on the winner's moves; the final position equals
    the reference's."""
    from kingdom_ai.gpu_puct import GpuPUCTOptions
    from kingdom_ai.gpu_rules import bits_to_records
    from kingdom_ai.model import random_groupnorm_network, random_network
    from kingdom_ai.selfplay import SelfPlayEngine
    from oracle.oracle import RefState

    model = random_network(64, 6, 7) if net == "6x64" else random_groupnorm_network(32, 2, 7)
    opts = GpuPUCTOptions(simulations=sims, c_puct=1.5, dirichlet_alpha=0.3, dirichlet_epsilon=0.25, seed=19)
    engine = SelfPlayEngine(model, 256, opts, temperature_moves=10, replay_capacity=1 << 16, game_log=4096)
    engine.step(plies)
    torch.cuda.synchronize()
    engine.check()
    log, (feats, masks, policy, value, to_play) = finished_games(engine)
    assert len(log["game_id"]) >= 32
    finals = bits_to_records(torch.from_numpy(log["final_state"]).cuda()).cpu().numpy()
    for slot in range(len(log["game_id"])):
        k, first = int(log["plies"][slot]), int(log["first_row"][slot])
        state = RefState.initial(reference)
        for ply in range(k):
            row = first + ply
            f, m = state.encode()
            assert np.array_equal(feats[row], f) and np.array_equal(masks[row], m), (slot, ply)
            rec = state.record()
            assert int(to_play[row]) == int(rec[162])
            p = policy[row]
            assert abs(float(p.sum()) - 1.0) < 1e-5 and not p[~m].any()
            assert state.play(int(log["actions"][slot, ply])), (slot, ply)
        final = state.record()
        assert final[GPU_REASON] != 0 and np.array_equal(final, finals[slot]), slot
        winner = int(log["winner"][slot])
        assert winner == final[GPU_WINNER]
        movers = to_play[first:first + k]
        assert np.array_equal(value[first:first + k], np.where(movers == winner, 1.0, -1.0).astype(np.float32))


def test_graph_replay_plays_the_same_games():
    """A captured ply replayed as a CUDA graph is the same computation as the
    direct launches: same counters, same replay rows, same game log."""
    from kingdom_ai.gpu_puct import GpuPUCTOptions
    from kingdom_ai.selfplay import SelfPlayEngine

    def run(graph):
        opts = GpuPUCTOptions(simulations=24, c_puct=1.5, dirichlet_alpha=0.3, dirichlet_epsilon=0.25, seed=4)
        engine = SelfPlayEngine(small_net(), 64, opts, temperature_moves=6, replay_capacity=1 << 14, game_log=1024)
        engine.step(1)
        if graph:
            engine.capture()
        engine.step(59)
        torch.cuda.synchronize()
        engine.check()
        return engine

    direct, replayed = run(False), run(True)
    assert direct.stats() == replayed.stats() and direct.stats()["games"] > 0
    assert keyset(rows_of(direct)) == keyset(rows_of(replayed))
    n = direct.stats()["games"]
    a, b = direct.games.read(n), replayed.games.read(n)
    order_a, order_b = a["game_id"].argsort(), b["game_id"].argsort()
    for key in ("game_id", "plies", "winner", "reason", "actions", "final_state"):
        assert np.array_equal(a[key][order_a], b[key][order_b]), key
