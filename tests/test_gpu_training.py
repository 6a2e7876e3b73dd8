"""collect_gpu_puct_games: complete games in the replay-sample schema.

Every recorded game is replayed from the default start with the oracle: each
sample's planes and legal mask must equal the oracle encoder of the position
it was taken at (as tests/gpu_training_test.py:97-123 checks against the C++
encoder), the mover must match, the final state must be terminal with the
returned winner and reason, and values must be +1 exactly for the winner's
moves.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GPU_ACTOR, GPU_REASON, GPU_WINNER = 162, 166, 167
# wire reason code -> EndReason value (C++ order None, Capture, TwoPasses, Suicide)
REASON_CODE = {1: 1, 2: 3, 3: 2}


def _collect(model, games, **kw):
    from kingdom_ai.gpu_puct import GpuPUCTOptions
    from kingdom_ai.training import collect_gpu_puct_games

    opts = GpuPUCTOptions(simulations=16, seed=kw.pop("noise_seed", 5))
    return collect_gpu_puct_games(model, games, options=opts, record_history=True, **kw)


def _replay_and_check(oracle, game):
    from kingdom_ai.training import Cell

    rec = oracle.initial(1)
    for ply, (sample, action) in enumerate(zip(game.samples, game.action_history)):
        feats, masks = oracle.encode(rec)
        assert np.array_equal(sample.features.numpy(), feats[0]), ply
        assert np.array_equal(sample.legal_mask.numpy(), masks[0]), ply
        assert sample.to_play == Cell(int(rec[0, GPU_ACTOR]))
        assert sample.value == (1.0 if sample.to_play == game.winner else -1.0)
        p = sample.policy.numpy()
        assert abs(float(p.sum()) - 1.0) < 1e-5 and not p[~masks[0]].any()
        assert masks[0][action], (ply, action)
        rec, accepted = oracle.play(rec, [action])
        assert accepted[0] == 1
    assert rec[0, GPU_REASON] != 0, "game did not end"
    assert int(rec[0, GPU_WINNER]) == int(game.winner)
    assert REASON_CODE[int(rec[0, GPU_REASON])] == int(game.reason)


def test_games_replay_exactly_with_the_oracle_hash_evaluator(oracle):
    from kingdom_ai.gpu_puct import HashEvaluator

    games = _collect(HashEvaluator(), 7, batch_size=4, temperature_moves=6, seed=11)
    assert len(games) == 7
    for game in games:
        assert len(game.samples) == len(game.action_history) >= 1
        _replay_and_check(oracle, game)


def test_games_replay_exactly_with_the_native_network(oracle):
    from kingdom_ai.model import random_network

    games = _collect(random_network(64, 1, 3), 5, batch_size=5, temperature=1.0, seed=3)
    for game in games:
        _replay_and_check(oracle, game)


def test_same_seeds_give_the_same_games():
    from kingdom_ai.gpu_puct import HashEvaluator

    a = _collect(HashEvaluator(), 6, batch_size=3, seed=21)
    b = _collect(HashEvaluator(), 6, batch_size=3, seed=21)
    assert [g.action_history for g in a] == [g.action_history for g in b]
    c = _collect(HashEvaluator(), 6, batch_size=3, seed=22)
    assert [g.action_history for g in a] != [g.action_history for g in c]


def test_zero_temperature_plays_the_search_best_move():
    from kingdom_ai.gpu_puct import HashEvaluator

    games = _collect(HashEvaluator(), 3, batch_size=3, temperature=0.0, seed=1, noise_seed=1)
    for game in games:
        for sample, action in zip(game.samples, game.action_history):
            visits = sample.policy
            assert visits[action] == visits.max()


def test_games_do_not_depend_on_batch_size_or_run_split(monkeypatch):
    """The device engine keys each game's randomness by its index, so neither
    the number of lanes nor splitting the call into runs changes a game."""
    from kingdom_ai import training
    from kingdom_ai.gpu_puct import HashEvaluator

    whole = _collect(HashEvaluator(), 10, batch_size=10, seed=4)
    narrow = _collect(HashEvaluator(), 10, batch_size=3, seed=4)
    monkeypatch.setattr(training, "_GAMES_PER_RUN", 4)
    split = _collect(HashEvaluator(), 10, batch_size=3, seed=4)
    for a, b, c in zip(whole, narrow, split):
        assert a.action_history == b.action_history == c.action_history
        assert a.winner == b.winner == c.winner and a.reason == b.reason == c.reason
        for x, y in zip(a.samples, c.samples):
            assert np.array_equal(x.policy.numpy(), y.policy.numpy()) and x.value == y.value


def test_other_modules_run_through_gpupuct(oracle):
    """A module the native kernels do not run is evaluated by torch inside
    GpuPUCT, ply by ply; its games replay exactly too."""
    import torch
    from torch import nn

    class Flat(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc = nn.Linear(810, 83)

        def forward(self, x):
            out = self.fc(x.flatten(1))
            return out[:, :82], torch.tanh(out[:, 82])

    torch.manual_seed(0)
    games = _collect(Flat(), 4, batch_size=4, seed=8)
    for game in games:
        _replay_and_check(oracle, game)


def test_the_callers_model_is_left_untouched():
    import torch
    from kingdom_ai.model import random_network

    model = random_network(64, 1, 3).train()
    before = {k: v.clone() for k, v in model.state_dict().items()}
    _collect(model, 2, batch_size=2, seed=1)
    assert model.training
    assert all(torch.equal(before[k], v) for k, v in model.state_dict().items())
