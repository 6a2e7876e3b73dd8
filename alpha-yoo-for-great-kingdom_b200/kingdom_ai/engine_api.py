"""The ``my_board_engine`` side of the drop-in boundary, on the GPU kernels.

``encode_puct_batch(states)`` stands in for ``my_board_engine.encode_puct_batch``
(bindings/batched_puct.cpp:140-148): schema-1 features and legal masks of a
batch of positions, returned as numpy arrays the caller owns.

``BatchedPUCT(options, leaf_batch_size, reuse_tree)`` stands in for
``my_board_engine.BatchedPUCT`` (bindings/batched_puct.cpp:52-139, over
mcts/src/BatchedPUCT.cpp): ``search(state, evaluator)`` takes one engine
``State`` and the reference's batch callback
``evaluator(features f32[N,10,9,9], masks bool[N,82]) -> (policy[N,82], values[N])``
on numpy arrays, and returns the fields of ``PUCTSearchResult``
(mcts/include/PUCT.h:38-51); ``advance``, ``clear``, ``stats``, ``options``,
``leaf_batch_size`` and ``reuse_tree`` follow the binding. The search runs on
this package's batched-search kernels (one tree of a ``GpuBatchedPUCT``);
the callback is called once per wave with that wave's leaves, as the
reference calls it. ``HashEvaluator()`` or a native network may be passed
instead of a callback.

Positions are accepted as engine ``State`` objects (``my_board_engine.State``,
read through their public attributes as ``GpuStateBatch.from_engine`` does),
a ``GpuStateBatch``, or wire records int32 [N,170]. Moves are action indices
(``row * 9 + col``, 81 = pass); ``advance`` also accepts an engine ``Move``.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as native
from .batched_puct import STAT_NAMES, GpuBatchedPUCT, PUCTOptions
from .gpu_puct import HashEvaluator
from .gpu_rules import GPU_ACTION_SIZE, GpuStateBatch

ACTION_SIZE = GPU_ACTION_SIZE
PASS_ACTION = ACTION_SIZE - 1


def _records(states, device) -> torch.Tensor:
    """Wire records int32 [N,170] on `device` for any accepted form of positions."""
    if isinstance(states, GpuStateBatch):
        return states.states.to(device)
    if isinstance(states, (torch.Tensor, np.ndarray)):
        recs = torch.as_tensor(states)
        if recs.dim() != 2 or recs.shape[1] != 170:
            raise ValueError("records must have shape [N, 170]")
        return GpuStateBatch(recs.to(device=device, dtype=torch.int32).contiguous()).states
    return GpuStateBatch.from_engine(list(states), device=device).states


def encode_puct_batch(states, device="cuda"):
    """Schema-1 features float32 [N,10,9,9] and legal masks bool [N,82] as numpy.

    Same contract as the reference binding (bindings/batched_puct.cpp:140-148,
    encode_puct_position per state, mcts/src/BatchedPUCT.cpp:25-50): the
    inputs are copied and the returned arrays are independently owned. The
    encoder runs on the GPU (``gk_encode_records``)."""
    device = native.require_cuda(device)
    if isinstance(states, (list, tuple)) and len(states) == 0:
        return np.zeros((0, 10, 9, 9), dtype=np.float32), np.zeros((0, ACTION_SIZE), dtype=bool)
    with torch.cuda.device(device):
        features, masks = GpuStateBatch(_records(states, device)).encode()
        return features.cpu().numpy(), masks.cpu().numpy()


def _action(move) -> int:
    """Action index of an int or an engine Move (is_pass(), point.row/col)."""
    if isinstance(move, (int, np.integer)) and not isinstance(move, bool):
        action = int(move)
    elif hasattr(move, "is_pass"):
        action = PASS_ACTION if move.is_pass() else int(move.point.row) * 9 + int(move.point.col)
    else:
        raise TypeError("move must be an action index or an engine Move")
    if not 0 <= action < ACTION_SIZE:
        raise ValueError("action index out of range")
    return action


@dataclass(frozen=True)
class PUCTMoveStatistics:
    """One root move of a search (mcts/include/PUCT.h:31-36); `move` is its action index."""
    move: int
    prior: float
    visits: int
    value: float


@dataclass(frozen=True)
class PUCTSearchResult:
    """The reference's search result (mcts/include/PUCT.h:38-51); moves as action indices."""
    best_move: int | None
    simulations: int
    nodes: int
    network_evaluations: int
    root_value: float
    best_value: float
    elapsed_seconds: float
    moves: tuple


def _numpy_callback(evaluator):
    """Adapt the reference's numpy batch callback to the device searcher."""

    def evaluate(features: torch.Tensor, masks: torch.Tensor):
        returned = evaluator(features.cpu().numpy(), masks.cpu().numpy())
        # bindings/batched_puct.cpp:32-51: a (policy, values) pair of the batch's shapes.
        if not isinstance(returned, tuple) or len(returned) != 2:
            raise ValueError("Batch evaluator must return (policy[N,82], values[N])")
        policy = np.ascontiguousarray(returned[0], dtype=np.float64)
        values = np.ascontiguousarray(returned[1], dtype=np.float64)
        n = features.shape[0]
        if policy.ndim != 2 or values.ndim != 1 or policy.shape != (n, ACTION_SIZE) or values.shape[0] != n:
            raise ValueError("Batch evaluator returned unexpected policy/value shapes")
        return torch.from_numpy(policy).to(features.device), torch.from_numpy(values).to(features.device)

    return evaluate


class BatchedPUCT:
    """One evaluation searcher with leaf batches, virtual loss and subtree reuse."""

    def __init__(self, options: PUCTOptions | None = None, leaf_batch_size: int = 8, reuse_tree: bool = True,
                 device="cuda"):
        self._searcher = GpuBatchedPUCT(1, options, leaf_batch_size, reuse_tree, device=device)
        self._searching = False

    @property
    def options(self) -> PUCTOptions:
        return self._searcher.options

    @property
    def leaf_batch_size(self) -> int:
        return self._searcher.leaf_batch_size

    @property
    def reuse_tree(self) -> bool:
        return self._searcher.reuse_tree

    def _check_idle(self):
        if self._searching:
            raise RuntimeError("Recursive access to an active BatchedPUCT is not supported")

    def search(self, state, evaluator) -> PUCTSearchResult:
        """BatchedPUCT::search of one position (BatchedPUCT.cpp:328-442)."""
        self._check_idle()
        device = self._searcher.device
        recs = _records([state] if not isinstance(state, (GpuStateBatch, torch.Tensor, np.ndarray)) else state,
                        device)
        if recs.shape[0] != 1:
            raise ValueError("search takes one position")
        from .model import NativePolicyValueNet, native_supported
        if not (isinstance(evaluator, (HashEvaluator, NativePolicyValueNet)) or native_supported(evaluator)):
            if not callable(evaluator):
                raise TypeError("PUCT requires a policy/value evaluator")
            evaluator = _numpy_callback(evaluator)
        self._searching = True
        started = time.perf_counter()
        try:
            r = self._searcher.search(GpuStateBatch(recs), evaluator)
            legal = r.legal[0].cpu()
        finally:
            self._searching = False
        elapsed = time.perf_counter() - started
        priors, visits, values = (t[0].cpu() for t in (r.priors, r.visits, r.move_values))
        moves = tuple(PUCTMoveStatistics(int(a), float(priors[a]), int(visits[a]), float(values[a]))
                      for a in legal.nonzero().flatten().tolist())
        best = int(r.actions[0])
        return PUCTSearchResult(best_move=None if best < 0 else best, simulations=int(r.simulations[0]),
                                nodes=int(r.nodes[0]), network_evaluations=int(r.network_evaluations[0]),
                                root_value=float(r.root_values[0]), best_value=float(r.best_values[0]),
                                elapsed_seconds=elapsed, moves=moves)

    def advance(self, move) -> bool:
        """BatchedPUCT::advance (BatchedPUCT.cpp:290-326): keep the played move's subtree."""
        self._check_idle()
        return bool(self._searcher.advance([_action(move)])[0])

    def clear(self) -> None:
        self._check_idle()
        self._searcher.clear()

    @property
    def stats(self) -> dict:
        """BatchedPUCTStatistics (mcts/include/BatchedPUCT.h:21-31) as ints."""
        self._check_idle()
        table = self._searcher.stats
        return {name: int(table[name][0]) for name in STAT_NAMES}
