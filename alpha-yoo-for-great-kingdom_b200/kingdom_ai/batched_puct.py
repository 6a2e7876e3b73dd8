"""Batched evaluation search on the GPU: drop-in for ``engine.BatchedPUCT``.

The reference's evaluation and match paths (python/kingdom_ai/evaluation.py:
174-231, match.py:121-254) keep one ``kingdom::BatchedPUCT`` per game and
model (mcts/src/BatchedPUCT.cpp): leaf batches gathered under a virtual loss,
one callback per batch, and the played move's subtree kept between searches.
``GpuBatchedPUCT`` holds many such searchers (``trees``) in one device
workspace and searches any subset of them together, so the leaves of every
game of a match go to the evaluator in one batch. Per tree, every result and
statistic is the reference searcher's, bit for bit for a deterministic
evaluator.

Evaluators, passed to each ``search`` like the reference's callback:

* ``HashEvaluator()`` - the injected evaluator of include/gk_common.h, run on
  the device (the whole search is then one kernel launch);
* a ``PolicyValueNet`` of this package (or a prepared
  ``NativePolicyValueNet``) - the native sm_100a network, masked softmax
  policy; no host synchronisation inside a search;
* any callable ``fn(features, masks) -> (policy, values)`` taking CUDA tensors
  fp32 [N,10,9,9] and bool [N,82] and returning non-negative policy weights
  [N,82] and values [N] (the batch callback of the reference binding, with
  device tensors in place of numpy arrays).
"""

from __future__ import annotations

import copy
import ctypes
import itertools
import math
import threading
import time
from dataclasses import dataclass
from numbers import Real

import torch

from . import _native as native
from .gpu_puct import HashEvaluator, encode_packed
from .gpu_rules import GPU_ACTION_SIZE, GpuStateBatch, _launch_scope

ACTION_SIZE = GPU_ACTION_SIZE
STAT_NAMES = ("network_evaluations", "inference_batches", "max_observed_batch_size", "reused_nodes",
              "inherited_visits", "advance_calls", "reuse_hits")
_ERR_CAPACITY, _ERR_VALUE, _ERR_POLICY, _ERR_NO_WEIGHT = 1, 2, 16, 32
_MESSAGES = (  # BatchedPUCT.cpp:72-81, 233-236, in the order the reference checks
    (_ERR_VALUE, ValueError, "PUCT evaluator value must be finite and in [-1, 1]"),
    (_ERR_POLICY, ValueError, "PUCT policy weights must be finite and non-negative"),
    (_ERR_NO_WEIGHT, ValueError, "PUCT policy must give positive weight to a legal action"),
    (_ERR_CAPACITY, RuntimeError, "Batched PUCT could not schedule a simulation"),
)


@dataclass(frozen=True)
class PUCTOptions:
    """``kingdom::PUCTOptions`` (mcts/include/PUCT.h:12-22) with the checks of
    PUCT::PUCT (mcts/src/PUCT.cpp:161-175)."""
    simulations: int = 128
    c_puct: float = 1.5
    seed: int = 42
    time_limit_ms: int = 0
    dirichlet_alpha: float = 0.3
    dirichlet_epsilon: float = 0.0

    def __post_init__(self):
        if type(self.simulations) is not int or not 1 <= self.simulations <= 2**31 - 2:
            raise ValueError("PUCT needs at least one simulation")
        for name in ("seed", "time_limit_ms"):
            value = getattr(self, name)
            if type(value) is not int or not 0 <= value <= 2**64 - 1:
                raise ValueError(f"{name} must be an unsigned 64-bit integer")
        values = {n: getattr(self, n) for n in ("c_puct", "dirichlet_alpha", "dirichlet_epsilon")}
        if any(isinstance(v, bool) or not isinstance(v, Real) for v in values.values()):
            raise ValueError("PUCT options must be real numbers")
        if not math.isfinite(self.c_puct) or self.c_puct <= 0:
            raise ValueError("PUCT exploration coefficient must be finite and positive")
        if not math.isfinite(self.dirichlet_alpha) or self.dirichlet_alpha <= 0:
            raise ValueError("Dirichlet alpha must be finite and positive")
        if not math.isfinite(self.dirichlet_epsilon) or not 0 <= self.dirichlet_epsilon <= 1:
            raise ValueError("Dirichlet epsilon must be finite and in [0, 1]")


class _Results(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "actions", "visits", "priors", "move_values", "legal", "simulations", "nodes", "root_values",
        "best_values", "stats", "errors", "status")]


class _Buffers(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "needs_eval", "leaf_bits", "policy", "value", "policy_f", "value_f", "active", "active_count", "pending",
        "node_count", "remaining", "stats")]


_c = ctypes
_BOUND = False


def _bind():
    global _BOUND
    if _BOUND:
        return
    vp, i64, i32, dbl = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_double
    native.register("gk_bpuct_workspace_bytes", [i64, i32, i32], _c.c_size_t)
    native.register("gk_bpuct_buffers", [vp, i64, i32, i32, _c.POINTER(_Buffers)])
    native.register("gk_bpuct_init", [vp, i64, i32, i32, vp])
    native.register("gk_bpuct_clear", [vp, i64, i32, i32, vp, vp])
    native.register("gk_bpuct_begin", [vp, i64, i32, i32, vp, vp, i32, i32, vp])
    native.register("gk_bpuct_root_expand", [vp, i64, i32, i32, i32, vp])
    native.register("gk_bpuct_collect", [vp, i64, i32, i32, dbl, vp])
    native.register("gk_bpuct_hash_eval", [vp, i64, i32, i32, vp])
    native.register("gk_bpuct_compact", [vp, i64, i32, i32, vp])
    native.register("gk_bpuct_expand", [vp, i64, i32, i32, i32, vp])
    native.register("gk_bpuct_finish", [vp, i64, i32, i32, _c.POINTER(_Results), vp])
    native.register("gk_bpuct_advance", [vp, i64, i32, i32, vp, vp, i32, vp, vp])
    native.register("gk_bpuct_search_hash", [vp, i64, i32, i32, vp, vp, i32, i32, dbl, _c.POINTER(_Results), vp])
    native.register("gk_bpuct_grow", [vp, i32, vp, i32, i64, i32, vp])
    native.register("gk_net_evaluate_states", [_c.POINTER(native.NetStruct), vp, vp, vp, i64, vp, vp, vp, vp, vp])
    _BOUND = True


@dataclass
class BatchedSearchResult:
    """Per-tree ``PUCTSearchResult`` fields (mcts/include/PUCT.h:38-51) as
    device tensors; rows of trees outside the search are empty (action -1)."""
    actions: torch.Tensor          # int64 [T] best action, -1 when none
    visits: torch.Tensor           # int32 [T,82] visits gained in this search
    priors: torch.Tensor           # float64 [T,82]
    move_values: torch.Tensor      # float64 [T,82] mean value for the root player
    legal: torch.Tensor            # bool [T,82] the root's moves
    simulations: torch.Tensor      # int32 [T]
    nodes: torch.Tensor            # int32 [T]
    network_evaluations: torch.Tensor  # int32 [T]
    root_values: torch.Tensor      # float64 [T]
    best_values: torch.Tensor      # float64 [T]
    searched: torch.Tensor         # bool [T] tree took part in this search

    def moves(self, tree: int):
        """The reference's ``moves`` list for one tree: (action, prior, visits,
        value) for every legal root action in action order."""
        legal = self.legal[tree].cpu()
        prior, visits, values = (t[tree].cpu() for t in (self.priors, self.visits, self.move_values))
        return [(int(a), float(prior[a]), int(visits[a]), float(values[a])) for a in legal.nonzero().flatten()]


class _Workspace:
    def __init__(self, trees, capacity, leaf_batch, device):
        lib = native.library()
        _bind()
        nbytes = lib.gk_bpuct_workspace_bytes(trees, capacity, leaf_batch)
        if nbytes == 0:
            raise ValueError("invalid batched search size")
        self.trees, self.capacity, self.leaf_batch, self.device = trees, capacity, leaf_batch, device
        self.storage = torch.empty(nbytes, dtype=torch.uint8, device=device)
        b = _Buffers()
        native.call("gk_bpuct_buffers", self.pointer, trees, capacity, leaf_batch, b)
        base = self.storage.data_ptr()

        def view(address, count, dtype, shape):
            offset = address - base
            width = torch.empty((), dtype=dtype).element_size()
            return self.storage[offset:offset + count * width].view(dtype).view(shape)

        S = trees * leaf_batch
        self.needs_eval = view(b.needs_eval, S, torch.uint8, (S,))
        self.leaf_bits = view(b.leaf_bits, S * 16, torch.int32, (S, 16))
        self.policy = view(b.policy, S * ACTION_SIZE, torch.float64, (S, ACTION_SIZE))
        self.value = view(b.value, S, torch.float64, (S,))
        self.policy_f = view(b.policy_f, S * ACTION_SIZE, torch.float32, (S, ACTION_SIZE))
        self.value_f = view(b.value_f, S, torch.float32, (S,))
        self.active = view(b.active, S, torch.int32, (S,))
        self.active_count = view(b.active_count, 1, torch.int32, (1,))
        self.node_count = view(b.node_count, trees, torch.int32, (trees,))
        self.remaining = view(b.remaining, 1, torch.int32, (1,))
        self.stats = view(b.stats, trees * len(STAT_NAMES), torch.int32, (trees, len(STAT_NAMES)))

    @property
    def pointer(self):
        return native.ptr(self.storage)

    def args(self):
        return self.pointer, self.trees, self.capacity, self.leaf_batch


class GpuBatchedPUCT:
    """``trees`` independent BatchedPUCT searchers (mcts/include/BatchedPUCT.h:38-60)
    in one device workspace.

    ``search(states, evaluator, active=None)`` searches the trees selected by
    ``active`` (bool [T], default all) from ``states`` (a GpuStateBatch or
    packed states int32 [T,16], one root per tree; rows of inactive trees are
    ignored). ``advance(actions, active=None)`` keeps each selected tree's
    subtree of its played action; ``clear`` drops trees. The workspace grows
    when a search could overflow it, so no tree is ever truncated.
    """

    def __init__(self, trees: int, options: PUCTOptions | None = None, leaf_batch_size: int = 8,
                 reuse_tree: bool = True, device="cuda", capacity: int | None = None):
        if options is None:
            options = PUCTOptions()
        if not isinstance(options, PUCTOptions):
            raise TypeError("options must be PUCTOptions")
        if type(trees) is not int or trees < 1:
            raise ValueError("trees must be a positive integer")
        if type(leaf_batch_size) is not int or leaf_batch_size < 1:
            raise ValueError("Batched PUCT needs a positive leaf batch size")
        if options.dirichlet_epsilon != 0.0:
            raise ValueError("Batched PUCT evaluation requires root Dirichlet noise to be disabled")
        if not isinstance(reuse_tree, bool):
            raise TypeError("reuse_tree must be a bool")
        self._options, self._leaf_batch, self._reuse = options, leaf_batch_size, reuse_tree
        self.trees = trees
        self.device = native.require_cuda(device)
        if capacity is None:
            capacity = 2 * (options.simulations + 1)
        self._lock = threading.Lock()
        self._ws = _Workspace(trees, max(capacity, options.simulations + 1), leaf_batch_size, self.device)
        self._node_bound = 0
        # The injected evaluator runs a whole search in one launch; with this
        # off the same search goes through the per-wave kernels.
        self._fuse_hash = True
        self._headfeat = None
        self._native_cache = (None, None)
        with torch.cuda.device(self.device):
            native.call("gk_bpuct_init", *self._ws.args(), native.stream_of(self.device))

    # -- reference accessors (BatchedPUCT.h:51-56) -------------------------------
    @property
    def options(self) -> PUCTOptions:
        return self._options

    @property
    def leaf_batch_size(self) -> int:
        return self._leaf_batch

    @property
    def reuse_tree(self) -> bool:
        return self._reuse

    @property
    def capacity(self) -> int:
        return self._ws.capacity

    @property
    def stats(self) -> dict:
        """BatchedPUCTStatistics (BatchedPUCT.h:21-31) per tree: int32 [T] each,
        copied from the device."""
        with self._lock:
            table = self._ws.stats.clone()
        return {name: table[:, i] for i, name in enumerate(STAT_NAMES)}

    def clear(self, trees=None) -> None:
        """BatchedPUCT::clear for the selected trees (all by default)."""
        with self._lock, torch.cuda.device(self.device):
            mask = self._mask(trees)
            stream = _launch_scope(self.device, self._ws.storage)
            native.call("gk_bpuct_clear", *self._ws.args(), native.ptr(mask), stream)
            if mask is None:
                self._node_bound = 0

    def advance(self, actions, active=None) -> torch.Tensor:
        """BatchedPUCT::advance (BatchedPUCT.cpp:290-326) per selected tree:
        bool [T], True where the played action's subtree was kept."""
        with self._lock, torch.cuda.device(self.device):
            acts = torch.as_tensor(actions, device=self.device).to(torch.int32).reshape(-1).contiguous()
            if acts.numel() != self.trees:
                raise ValueError("advance needs one action per tree")
            mask = self._mask(active)
            advanced = torch.zeros(self.trees, dtype=torch.uint8, device=self.device)
            stream = _launch_scope(self.device, acts, advanced, self._ws.storage)
            native.call("gk_bpuct_advance", *self._ws.args(), native.ptr(acts), native.ptr(mask), int(self._reuse),
                        native.ptr(advanced), stream)
            return advanced.bool()

    def search(self, states, evaluator, active=None) -> BatchedSearchResult:
        """BatchedPUCT::search (BatchedPUCT.cpp:328-442) of the selected trees."""
        if isinstance(states, GpuStateBatch):
            if states.device != self.device:
                raise ValueError("State and searcher must use the same CUDA device")
            roots = states.to_bits()
        elif isinstance(states, torch.Tensor) and states.dtype == torch.int32 and states.shape[1:] == (16,):
            roots = states.to(self.device)
        else:
            raise TypeError("states must be a GpuStateBatch or packed states int32 [T,16]")
        if roots.shape[0] != self.trees:
            raise ValueError("search needs one root per tree")
        with self._lock, torch.cuda.device(self.device), torch.inference_mode():
            return self._search(roots.contiguous(), evaluator, self._mask(active))

    # -- internals ---------------------------------------------------------------
    def _mask(self, trees):
        if trees is None:
            return None
        mask = torch.as_tensor(trees, device=self.device)
        if mask.dtype != torch.bool or mask.shape != (self.trees,):
            raise ValueError("tree selection must be a bool tensor [trees]")
        return mask.to(torch.uint8).contiguous()

    def _ensure_capacity(self, stream):
        if not self._reuse:
            # every searched tree starts empty (BatchedPUCT.cpp:346)
            self._node_bound = 0
        need = self._node_bound + self._options.simulations + 1
        if need <= self._ws.capacity:
            return
        self._node_bound = int(self._ws.node_count.max().item())
        need = self._node_bound + self._options.simulations + 1
        if need <= self._ws.capacity:
            return
        old = self._ws
        grown = _Workspace(old.trees, max(need, 2 * old.capacity), old.leaf_batch, self.device)
        native.call("gk_bpuct_grow", old.pointer, old.capacity, grown.pointer, grown.capacity, old.trees,
                    old.leaf_batch, stream)
        torch.cuda.current_stream(self.device).synchronize()
        self._ws = grown

    def _kind(self, evaluator):
        from .model import NativePolicyValueNet, native_supported
        if isinstance(evaluator, HashEvaluator):
            return "hash", None
        if isinstance(evaluator, NativePolicyValueNet):
            return "native", evaluator
        if native_supported(evaluator):
            # Packed once per model and weight version: any in-place update of
            # a parameter or buffer bumps its version counter.
            key = (id(evaluator), tuple((t.data_ptr(), t._version)
                                        for t in itertools.chain(evaluator.parameters(), evaluator.buffers())))
            cached_key, cached_net = self._native_cache
            if cached_key != key:
                cached_net = NativePolicyValueNet(copy.deepcopy(evaluator).cpu(), device=self.device)
                self._native_cache = (key, cached_net)
            return "native", cached_net
        if callable(evaluator):
            return "callback", evaluator
        raise TypeError("PUCT requires a policy/value evaluator")

    def _results(self):
        """Result tensors carved from one allocation. The finish kernel writes
        every field of every tree, so nothing needs clearing first."""
        T = self.trees
        fields = (("actions", (T,), torch.int64), ("priors", (T, ACTION_SIZE), torch.float64),
                  ("move_values", (T, ACTION_SIZE), torch.float64), ("root_values", (T,), torch.float64),
                  ("best_values", (T,), torch.float64), ("visits", (T, ACTION_SIZE), torch.int32),
                  ("simulations", (T,), torch.int32), ("nodes", (T,), torch.int32),
                  ("stats", (T, len(STAT_NAMES)), torch.int32), ("errors", (T,), torch.int32),
                  ("status", (1,), torch.int32), ("legal", (T, ACTION_SIZE), torch.uint8))
        sizes = [math.prod(shape) * torch.empty((), dtype=dtype).element_size() for _, shape, dtype in fields]
        padded = [(n + 255) // 256 * 256 for n in sizes]
        storage = torch.empty(sum(padded), dtype=torch.uint8, device=self.device)
        out, offset = {}, 0
        for (name, shape, dtype), n, step in zip(fields, sizes, padded):
            out[name] = storage[offset:offset + n].view(dtype).view(shape)
            offset += step
        struct = _Results(*(out[name].data_ptr() for name, _ in _Results._fields_))
        return out, struct

    def _evaluate(self, kind, evaluator, stream):
        """Evaluations of every slot that needs one. Returns the float_eval flag."""
        ws = self._ws
        if kind == "hash":
            native.call("gk_bpuct_hash_eval", *ws.args(), stream)
            return 0
        if kind == "native":
            n = ws.trees * ws.leaf_batch
            if self._headfeat is None or self._headfeat.shape[0] < n:
                self._headfeat = torch.empty((n, 243), dtype=torch.float32, device=self.device)
            native.call("gk_bpuct_compact", *ws.args(), stream)
            native.call("gk_net_evaluate_states", evaluator.struct, native.ptr(ws.leaf_bits), native.ptr(ws.active),
                        native.ptr(ws.active_count), n, native.ptr(ws.policy_f), native.ptr(ws.value_f),
                        native.ptr(self._headfeat), native.ptr(evaluator.status), stream)
            return 1
        slots = ws.needs_eval.nonzero(as_tuple=False).flatten()
        if slots.numel() == 0:
            return 0
        features, masks = encode_packed(ws.leaf_bits.index_select(0, slots))
        policy, values = evaluator(features, masks)
        policy = torch.as_tensor(policy, device=self.device)
        values = torch.as_tensor(values, device=self.device)
        n = slots.numel()
        if policy.shape != (n, ACTION_SIZE) or values.reshape(-1).shape != (n,):
            raise ValueError("Batched PUCT evaluator must return one result per position")
        if not policy.is_floating_point() or not values.is_floating_point():
            raise TypeError("evaluator policy and values must be floating-point tensors")
        ws.policy.index_copy_(0, slots, policy.to(torch.float64))
        ws.value.index_copy_(0, slots, values.reshape(-1).to(torch.float64))
        return 0

    def _search(self, roots, evaluator, mask):
        kind, ev = self._kind(evaluator)
        o = self._options
        stream = _launch_scope(self.device, roots, self._ws.storage)
        self._ensure_capacity(stream)
        ws = self._ws
        out, struct = self._results()
        started = time.perf_counter()
        reuse = int(self._reuse)
        try:
            if kind == "hash" and o.time_limit_ms == 0 and self._fuse_hash:
                native.call("gk_bpuct_search_hash", *ws.args(), native.ptr(roots), native.ptr(mask), o.simulations,
                            reuse, float(o.c_puct), struct, stream)
            else:
                native.call("gk_bpuct_begin", *ws.args(), native.ptr(roots), native.ptr(mask), o.simulations, reuse,
                            stream)
                flt = self._evaluate(kind, ev, stream)
                native.call("gk_bpuct_root_expand", *ws.args(), flt, stream)
                waves = -(-o.simulations // ws.leaf_batch)
                # Every wave completes at least one simulation of each tree
                # that still has budget, so this many waves always suffice.
                allowance = o.simulations + 1
                while True:
                    if waves > allowance:
                        raise RuntimeError("Batched PUCT could not schedule a simulation")
                    allowance -= waves
                    for _ in range(waves):
                        native.call("gk_bpuct_collect", *ws.args(), float(o.c_puct), stream)
                        flt = self._evaluate(kind, ev, stream)
                        native.call("gk_bpuct_expand", *ws.args(), flt, stream)
                        if o.time_limit_ms and (time.perf_counter() - started) * 1e3 >= o.time_limit_ms:
                            break
                    left = int(ws.remaining.item())
                    if left == 0 or (o.time_limit_ms and (time.perf_counter() - started) * 1e3 >= o.time_limit_ms):
                        break
                    waves = -(-left // ws.leaf_batch)
                native.call("gk_bpuct_finish", *ws.args(), struct, stream)
        except BaseException:
            # A failed evaluation leaves reservations behind: drop the trees of
            # this search, as the reference does (BatchedPUCT.cpp:435-440).
            native.call("gk_bpuct_clear", *ws.args(), native.ptr(mask), stream)
            raise
        self._node_bound += o.simulations + 1
        code = int(out["status"].item())
        if kind == "native":
            ev.check()
        if code:
            for bit, error, message in _MESSAGES:
                if code & bit:
                    raise error(message)
            raise RuntimeError(f"batched search failed with error bits {code:#x}")
        searched = torch.ones(self.trees, dtype=torch.bool, device=self.device) if mask is None else mask.bool()
        return BatchedSearchResult(actions=out["actions"], visits=out["visits"], priors=out["priors"],
                                   move_values=out["move_values"], legal=out["legal"].bool(),
                                   simulations=out["simulations"], nodes=out["nodes"],
                                   network_evaluations=out["stats"][:, 0].clone(), root_values=out["root_values"],
                                   best_values=out["best_values"], searched=searched)
