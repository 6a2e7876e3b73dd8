"""Complete self-play games in the reference's replay-sample schema.

``collect_gpu_puct_games`` is the drop-in for the reference's
``collect_gpu_puct_games`` (python/kingdom_ai/gpu_training.py:124-175), the
call behind the Trainer's CUDA self-play hook (python/kingdom_ai/loop.py:
524-541). For the networks the native kernels run (``PolicyValueNet``,
``GroupNormPolicyValueNet``) and for ``HashEvaluator`` it drives the
device-resident engine (``SelfPlayEngine``, ``gk_selfplay_ply``): a whole ply
per call with no host synchronisation inside it, ``batch_size`` lanes that
start the next game as soon as one ends, and per-game action histories and
replay rows kept on the device until the call's games are done, then copied to
the host in one copy per tensor. Any other ``nn.Module`` runs through
``GpuPUCT`` ply by ply with torch evaluating the leaves, in chunks of
``batch_size`` games as the reference does. The returned ``GameData`` /
``TrainingSample`` carry the fields of the reference types
(python/kingdom_ai/training.py:17-30).
"""

from __future__ import annotations

import copy
import enum
import math
from dataclasses import dataclass

import torch

from . import _native as native
from .gpu_puct import GpuPUCT, GpuPUCTOptions
from .gpu_rules import (GPU_ACTION_SIZE, GPU_ACTOR, GPU_CAPTURE, GPU_REASON, GPU_SUICIDE, GPU_TWO_PASSES,
                        GPU_WINNER, GpuStateBatch)

MAX_PLIES = 2 * 81 + 2  # every ply places a stone or passes; 41 stones each, two closing passes
_SAMPLING_SALT = 0x9E3779B97F4A7C15  # move sampling draws from seed ^ salt, root noise from the seed


class Cell(enum.IntEnum):
    """Cell values of the engine (engine/include/board/Board.h:11)."""
    Empty = 0
    Black = 1
    White = 2
    Neutral = 3


class EndReason(enum.IntEnum):
    """Game-end reasons of the engine (engine/include/board/GameResult.h:7)."""
    None_ = 0
    Capture = 1
    TwoPasses = 2
    Suicide = 3


_REASONS = {GPU_CAPTURE: EndReason.Capture, GPU_SUICIDE: EndReason.Suicide, GPU_TWO_PASSES: EndReason.TwoPasses}


@dataclass(frozen=True)
class TrainingSample:
    features: torch.Tensor    # float32 [10,9,9]
    legal_mask: torch.Tensor  # bool [82]
    policy: torch.Tensor      # float32 [82] root visit proportions
    value: float              # +1 if the player to move won the game, else -1
    to_play: Cell


@dataclass(frozen=True)
class TrainingBatch:
    """A sampled minibatch (python/kingdom_ai/training.py:33-38)."""
    features: torch.Tensor    # float32 [N,10,9,9]
    legal_mask: torch.Tensor  # bool [N,82]
    policy: torch.Tensor      # float32 [N,82]
    value: torch.Tensor       # float32 [N]


@dataclass(frozen=True)
class GameData:
    samples: list
    winner: Cell
    reason: EndReason
    action_history: tuple | None = None


def _check_schedule(temperature, temperature_moves, final_temperature):
    for name, t in (("Temperature", temperature), ("Final temperature", final_temperature)):
        if not isinstance(t, (int, float)) or isinstance(t, bool):
            raise TypeError(f"{name} must be a real number")
        if not math.isfinite(t) or t < 0:
            raise ValueError(f"{name} must be finite and non-negative")
    if temperature_moves is not None and (type(temperature_moves) is not int or temperature_moves < 0):
        raise ValueError("temperature_moves must be None or a non-negative integer")


def visit_sampling_weights(visits: torch.Tensor, temperature: float) -> torch.Tensor:
    """Weights proportional to visits**(1/T), computed as exp((log n - log n_max) / T).

    The same weights as gpu_training.py:28-37: working in relative logs keeps
    tiny temperatures from overflowing, and unvisited actions get weight 0.
    """
    visited = visits > 0
    logs = visits.to(torch.float64).clamp_min(1).log()
    logs = logs - logs.amax(dim=1, keepdim=True)
    t = max(float(temperature), torch.finfo(torch.float64).tiny)
    return (logs / t).exp().masked_fill(~visited, 0.0)


def _play_chunk(searcher, state, temperature, generator, temperature_moves, final_temperature, record_history):
    lanes, device = len(state), state.device
    feats = torch.empty((MAX_PLIES, lanes, 10, 9, 9), dtype=torch.float32, device=device)
    masks = torch.empty((MAX_PLIES, lanes, GPU_ACTION_SIZE), dtype=torch.bool, device=device)
    policies = torch.empty((MAX_PLIES, lanes, GPU_ACTION_SIZE), dtype=torch.float32, device=device)
    actors = torch.empty((MAX_PLIES, lanes), dtype=torch.int32, device=device)
    actions_seen = torch.empty((MAX_PLIES, lanes), dtype=torch.int32, device=device) if record_history else None
    lengths = torch.zeros(lanes, dtype=torch.int32, device=device)
    rejected = torch.zeros((), dtype=torch.bool, device=device)
    plies = 0
    for ply in range(MAX_PLIES):
        alive = state.states[:, GPU_REASON] == 0
        if not bool(alive.any()):
            break
        f, m = state.encode()
        feats[ply].copy_(f)
        masks[ply].copy_(m)
        actors[ply].copy_(state.states[:, GPU_ACTOR])  # the mover, recorded before the move
        result = searcher.search(state)
        policies[ply].copy_(result.policy)  # targets are raw visit shares at any temperature
        t = temperature if temperature_moves is None or ply < temperature_moves else final_temperature
        if t == 0:
            actions = result.actions
        else:
            weights = visit_sampling_weights(result.visits, t)
            # Finished lanes have no visits; give them a dummy pass weight so one
            # fixed-size multinomial serves the batch. Their action stays -1.
            weights[:, -1] += (~alive).to(weights.dtype)
            drawn = torch.multinomial(weights, 1, generator=generator).flatten()
            actions = torch.where(alive, drawn, result.actions)
        if actions_seen is not None:
            actions_seen[ply].copy_(actions)
        accepted = state.play(actions)
        rejected |= (alive & ~accepted).any()
        lengths += alive.to(lengths.dtype)
        plies = ply + 1
    if bool(rejected):
        raise RuntimeError("GPU PUCT produced a move the rules rejected")
    if bool((state.states[:, GPU_REASON] == 0).any()):
        raise RuntimeError("a game exceeded its finite move bound")

    feats, masks, policies, actors = (t[:plies].cpu() for t in (feats, masks, policies, actors))
    actions_seen = None if actions_seen is None else actions_seen[:plies].cpu()
    meta = torch.stack((lengths, state.states[:, GPU_WINNER], state.states[:, GPU_REASON]), dim=1).cpu().tolist()
    games = []
    for lane, (length, winner_code, reason_code) in enumerate(meta):
        winner = Cell(winner_code)
        samples = [TrainingSample(feats[p, lane], masks[p, lane], policies[p, lane],
                                  1.0 if Cell(int(actors[p, lane])) == winner else -1.0, Cell(int(actors[p, lane])))
                   for p in range(length)]
        history = None if actions_seen is None else tuple(actions_seen[:length, lane].tolist())
        games.append(GameData(samples, winner, _REASONS[reason_code], history))
    return games


# Games per engine run: their replay rows (at most 166 per game, 3,655 B each)
# stay on the device until the run ends, so a larger request runs in id ranges
# of this size (about 3.7 GB of rows). Game randomness is keyed by game id, so
# the split does not change any game.
_GAMES_PER_RUN = 6144


def _run_engine(engine, count):
    """Step `engine` until `count` games have finished.

    The host reads the finished-game counter one ply behind the GPU: after
    enqueueing ply p it waits for ply p-1's counter copy, so the device always
    has the next ply queued and never idles on the host. Plies after the first
    replay a CUDA graph of its launches.
    """
    from .selfplay import GAME_ACTIONS

    stream = torch.cuda.current_stream(engine.device)
    host = torch.zeros((2, engine.counters.numel()), dtype=torch.int64).pin_memory()
    done = [torch.cuda.Event(), torch.cuda.Event()]
    bound = (-(-count // engine.lanes)) * GAME_ACTIONS + 2
    for ply in range(bound + 1):
        engine.step()
        if ply == 0:
            engine.capture()  # later plies replay the first one's launches as a CUDA graph
        host[ply % 2].copy_(engine.counters, non_blocking=True)
        done[ply % 2].record(stream)
        if ply >= 1:
            done[(ply - 1) % 2].synchronize()
            if int(host[(ply - 1) % 2, 1]) >= count:
                break
    stream.synchronize()
    engine.check()
    if engine.stats()["games"] != count:
        raise RuntimeError("a game exceeded its finite move bound")


def _engine_games(net, games, options, temperature, batch_size, seed, device, temperature_moves, final_temperature,
                  record_history):
    from .selfplay import GAME_ACTIONS, SelfPlayEngine

    out = []
    for start in range(0, games, _GAMES_PER_RUN):
        count = min(_GAMES_PER_RUN, games - start)
        lanes = min(batch_size, count)
        engine = SelfPlayEngine(net, lanes, options, temperature=temperature, temperature_moves=temperature_moves,
                                final_temperature=final_temperature, replay_capacity=count * GAME_ACTIONS,
                                seed=options.seed, sample_seed=seed, device=device, game_log=count,
                                game_limit=start + count, first_game=start)
        _run_engine(engine, count)
        rows = engine.stats()["rows"]
        ring = engine.replay
        feats, masks, policy, value, to_play = (t[:rows].cpu() for t in (ring.features, ring.masks, ring.policy,
                                                                           ring.value, ring.to_play))
        log = engine.games.read(count)
        order = log["game_id"].argsort(kind="stable")
        values, actors = value.tolist(), to_play.tolist()
        for slot in order:
            first, plies = int(log["first_row"][slot]), int(log["plies"][slot])
            winner = Cell(int(log["winner"][slot]))
            samples = [TrainingSample(feats[r], masks[r], policy[r], values[r], Cell(actors[r]))
                       for r in range(first, first + plies)]
            history = tuple(log["actions"][slot, :plies].tolist()) if record_history else None
            out.append(GameData(samples, winner, _REASONS[int(log["reason"][slot])], history))
        del engine
    return out


def collect_gpu_puct_games(model, games, *, options=None, temperature=1.0, batch_size=128, seed=42, device="cuda",
                           temperature_moves=None, final_temperature=0.0, record_history=False) -> list:
    """Play `games` complete games with GPU PUCT; return them in order as GameData.

    Same contract as the reference (gpu_training.py:124-175): ``options.seed``
    drives root noise and ``seed`` drives move sampling (default options use
    ``seed`` for both, with root noise epsilon 0.25); at most ``batch_size``
    games are in flight; ``temperature_moves`` switches each game to
    ``final_temperature`` after that many plies; ``record_history`` keeps the
    played actions, which replay the game from the default start. The caller's
    model and the global RNG state are left untouched. Sample values are +1
    for the winner's moves. With the device engine, game k's randomness is
    keyed by (seed, k, ply), so a game does not depend on ``batch_size``.
    """
    if type(games) is not int or games < 0:
        raise ValueError("games must be a non-negative integer")
    if type(batch_size) is not int or batch_size < 1:
        raise ValueError("batch_size must be a positive integer")
    if type(seed) is not int or not 0 <= seed < 2**64:
        raise ValueError("Seed must be an unsigned 64-bit integer")
    _check_schedule(temperature, temperature_moves, final_temperature)
    if type(record_history) is not bool:
        raise TypeError("record_history must be bool")
    if options is None:
        options = GpuPUCTOptions(seed=seed)
    if not isinstance(options, GpuPUCTOptions):
        raise TypeError("options must be GpuPUCTOptions")
    if games == 0:
        return []
    from .gpu_puct import HashEvaluator
    from .model import NativePolicyValueNet, native_supported

    if isinstance(model, HashEvaluator) or native_supported(model):
        dev = native.require_cuda(device)
        net = None
        if not isinstance(model, HashEvaluator):
            net = NativePolicyValueNet(copy.deepcopy(model).cpu().float(), dev)
        with torch.cuda.device(dev), torch.no_grad():
            return _engine_games(net, games, options, temperature, batch_size, seed, dev, temperature_moves,
                                 final_temperature, record_history)
    searcher = GpuPUCT(model, options=options, device=device)
    generator = torch.Generator(device=searcher.device).manual_seed(seed ^ _SAMPLING_SALT)
    out = []
    with torch.cuda.device(searcher.device), torch.no_grad():
        for first in range(0, games, batch_size):
            state = GpuStateBatch.initial(min(batch_size, games - first), device=searcher.device)
            out.extend(_play_chunk(searcher, state, temperature, generator, temperature_moves, final_temperature,
                                   record_history))
    return out
