"""Model-versus-model evaluation games on the GPU.

The reference plays evaluation pairs one game per worker thread, each game
with one ``engine.BatchedPUCT`` per model (python/kingdom_ai/evaluation.py:
174-231, 235-360). ``evaluate_models_gpu`` plays every game of a match at once:
one ``GpuBatchedPUCT`` per model holds a tree per game, each model searches
the games where it is to move (their leaves in one network batch per wave),
and both models' trees advance after every move, as the reference does.

Pairing, seeds and move choice are the reference's: pair i uses
``(seed + i) % 2**64`` for both of its games, the candidate playing Black in
the first and White in the second; during the first ``opening_moves`` plies a
move is sampled from the root visits with weights exp((log n - log n_max)/T)
by that game's own CPU generator (python/kingdom_ai/puct.py:40-64), and the
most visited action is played afterwards.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from numbers import Real

import torch

from .batched_puct import GpuBatchedPUCT, PUCTOptions
from .gpu_rules import GPU_ACTOR, GPU_CELL_COUNT, GPU_REASON, GPU_WINNER, GpuStateBatch
from .training import _REASONS

MAX_PLIES = 2 * GPU_CELL_COUNT + 2  # evaluation.py:219-220


@dataclass
class EvaluationResult:
    """Results from the candidate's perspective (evaluation.py:22-36);
    ``endings`` counts games by end-reason name."""
    games: int
    wins: int
    losses: int
    wins_as_black: int
    wins_as_white: int
    total_plies: int
    endings: dict = field(default_factory=dict)

    @property
    def win_rate(self) -> float:
        return self.wins / self.games


def sample_visit_action(visits, temperature: float, generator: torch.Generator) -> int:
    """One action drawn from root visit counts as python/kingdom_ai/puct.py:
    50-63 does: weights exp((log n - log n_max) / T) in double precision for
    visited actions, then one multinomial draw from the caller's generator."""
    counts = [int(v) for v in visits]
    if max(counts) < 1:
        raise ValueError("A searched result must contain positive visit counts")
    largest_log = math.log(max(counts))
    weights = torch.tensor([math.exp((math.log(c) - largest_log) / temperature) if c > 0 else 0.0
                            for c in counts], dtype=torch.float64)
    return int(torch.multinomial(weights, 1, generator=generator).item())


def _check(name, value, low, kind=int):
    if kind is int:
        if type(value) is not int or value < low:
            raise ValueError(f"{name} must be an integer >= {low}")
    elif isinstance(value, bool) or not isinstance(value, Real) or not math.isfinite(value) or value < low:
        raise ValueError(f"{name} must be a finite real >= {low}")


def evaluate_models_gpu(candidate, reference, *, games: int = 20, simulations: int = 128, c_puct: float = 1.5,
                        seed: int = 42, opening_moves: int = 6, opening_temperature: float = 1.0,
                        leaf_batch_size: int = 8, reuse_tree: bool = True, device="cuda") -> EvaluationResult:
    """Play ``games`` evaluation games (an even number: pairs with the
    candidate first Black, then White) between two models on the GPU.

    ``candidate`` and ``reference`` are evaluators of ``GpuBatchedPUCT.search``
    (a network of this package runs on the native kernels). Results count from
    the candidate's side, as ``evaluate_models`` reports them
    (python/kingdom_ai/evaluation.py:235-360)."""
    _check("games", games, 2)
    if games % 2:
        raise ValueError("games must be even: each pair plays both colours")
    _check("simulations", simulations, 1)
    _check("opening_moves", opening_moves, 0)
    _check("leaf_batch_size", leaf_batch_size, 1)
    _check("c_puct", c_puct, 0.0, float)
    _check("opening_temperature", opening_temperature, 0.0, float)
    if type(seed) is not int or not 0 <= seed < 2 ** 64:
        raise ValueError("seed must be an unsigned 64-bit integer")
    options = PUCTOptions(simulations=simulations, c_puct=float(c_puct), seed=seed, dirichlet_epsilon=0.0)
    # Game 2i + c: pair i, candidate Black for c = 0 and White for c = 1.
    candidate_color = torch.tensor([1 if g % 2 == 0 else 2 for g in range(games)], dtype=torch.int32)
    generators = [torch.Generator(device="cpu").manual_seed((seed + g // 2) % 2 ** 64) for g in range(games)]
    searchers = {"candidate": GpuBatchedPUCT(games, options, leaf_batch_size, reuse_tree, device),
                 "reference": GpuBatchedPUCT(games, options, leaf_batch_size, reuse_tree, device)}
    models = {"candidate": candidate, "reference": reference}
    state = GpuStateBatch.initial(games, device=device)
    dev = state.device
    cand_color = candidate_color.to(dev)
    plies = torch.zeros(games, dtype=torch.int64)
    with torch.inference_mode():
        for ply in range(MAX_PLIES + 1):
            records = state.states
            live = records[:, GPU_REASON] == 0
            if not bool(live.any()):
                break
            if ply == MAX_PLIES:
                raise RuntimeError("Evaluation game exceeded its finite move bound")
            mover = records[:, GPU_ACTOR]
            moves = torch.zeros(games, dtype=torch.int64, device=dev)
            for name, searcher in searchers.items():
                own = (mover == cand_color) if name == "candidate" else (mover != cand_color)
                active = live & own
                if not bool(active.any()):
                    continue
                result = searcher.search(state, models[name], active=active)
                moves = torch.where(active, result.actions, moves)
                if ply < opening_moves and opening_temperature > 0:
                    visits = result.visits.cpu()
                    chosen = moves.cpu()
                    for g in active.nonzero().flatten().tolist():
                        chosen[g] = sample_visit_action(visits[g], float(opening_temperature), generators[g])
                    moves = chosen.to(dev)
            accepted = state.play(torch.where(live, moves, torch.zeros_like(moves)))
            if not bool(accepted[live].all()):
                raise RuntimeError("Evaluation search produced a rejected move")
            for searcher in searchers.values():
                searcher.advance(moves, active=live)
            plies += live.cpu().to(torch.int64)
    final = state.states.cpu()
    winners, reasons = final[:, GPU_WINNER], final[:, GPU_REASON]
    if not bool(((winners == 1) | (winners == 2)).all()):
        raise RuntimeError("A completed evaluation game must have a winner")
    won = winners == candidate_color
    endings: dict = {}
    for r in reasons.tolist():
        name = _REASONS[int(r)].name
        endings[name] = endings.get(name, 0) + 1
    return EvaluationResult(games=games, wins=int(won.sum()), losses=int((~won).sum()),
                            wins_as_black=int((won & (candidate_color == 1)).sum()),
                            wins_as_white=int((won & (candidate_color == 2)).sum()),
                            total_plies=int(plies.sum()), endings=endings)
