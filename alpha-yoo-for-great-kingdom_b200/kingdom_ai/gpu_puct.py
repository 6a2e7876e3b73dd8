"""Batched CUDA PUCT: drop-in for ``kingdom_ai.gpu_puct`` (python/kingdom_ai/gpu_puct.py).

Each lane owns one independent tree stored as structure-of-arrays in one
device workspace (see ``gk_puct.cuh``). Select, expand/backup and finish are
warp-per-tree kernels of libgk.so; the leaf evaluator is one of

* ``HashEvaluator()`` - the injected deterministic evaluator (weights
  w_a = exp(z_a), uniform value) that reproduces the C++ ``PUCT::search``
  visit counts bit for bit;
* a ``PolicyValueNet`` of this package - evaluated by the native sm_100a
  network kernels, with no host synchronisation inside a search;
* any other ``torch.nn.Module`` returning (logits [N,82], values [N]) - run
  by PyTorch on the compacted leaf batch, exactly as the reference does
  (one ``nonzero`` synchronisation per simulation).

Root noise is drawn on the device from a PCG32 stream per (search call, tree);
``reset_seed`` restarts it. Like the reference, the stream differs from the
C++ implementation's ``std::gamma_distribution``.
"""

from __future__ import annotations

import copy
import math
import threading
from dataclasses import dataclass
from numbers import Real

import torch
from torch import nn

from . import _native as native
from .gpu_rules import GPU_ACTION_SIZE, GpuStateBatch, _launch_scope

ACTION_SIZE = GPU_ACTION_SIZE


@dataclass(frozen=True)
class GpuPUCTOptions:
    """Opt-in root safety and value-based first-play urgency preserve defaults.

    Same fields, defaults and validation as python/kingdom_ai/gpu_puct.py:26-63.
    """
    simulations: int = 32
    c_puct: float = 1.5
    dirichlet_alpha: float = 0.3
    dirichlet_epsilon: float = 0.25
    seed: int = 42
    tactical_checks: bool = False
    fpu_reduction: float | None = None

    def __post_init__(self):
        if type(self.simulations) is not int or not 1 <= self.simulations <= 2**31 - 2:
            raise ValueError("simulations must be an integer in [1, 2147483646]")
        for name in ("c_puct", "dirichlet_alpha", "dirichlet_epsilon"):
            value = getattr(self, name)
            if isinstance(value, bool) or not isinstance(value, Real) or not math.isfinite(value):
                raise ValueError(f"{name} must be finite and real")
        if self.c_puct <= 0 or self.dirichlet_alpha <= 0:
            raise ValueError("c_puct and dirichlet_alpha must be positive")
        if not 0 <= self.dirichlet_epsilon <= 1:
            raise ValueError("dirichlet_epsilon must be in [0, 1]")
        if type(self.seed) is not int or not 0 <= self.seed <= 2**64 - 1:
            raise ValueError("seed must be an unsigned 64-bit integer")
        if type(self.tactical_checks) is not bool:
            raise TypeError("tactical_checks must be a bool")
        if self.fpu_reduction is not None and (
                isinstance(self.fpu_reduction, bool)
                or not isinstance(self.fpu_reduction, Real)
                or not math.isfinite(self.fpu_reduction)
                or self.fpu_reduction < 0):
            raise ValueError("fpu_reduction must be None or a finite non-negative real")


@dataclass(frozen=True)
class GpuSearchResult:
    actions: torch.Tensor
    visits: torch.Tensor
    policy: torch.Tensor
    values: torch.Tensor
    simulations: torch.Tensor
    network_evaluations: torch.Tensor
    priors: torch.Tensor
    best_values: torch.Tensor
    nodes: torch.Tensor
    root_values: torch.Tensor | None = None


class HashEvaluator:
    """The injected evaluator: a pure hash of the leaf state (include/gk_common.h)."""


class SearchWorkspace:
    """One device allocation holding every tree array of a batched search."""

    _FIELDS = ("needs_eval", "leaf_bits", "leaf_value", "policy", "noise", "active", "active_count", "errors",
               "leaf", "root_allow")

    def __init__(self, batch: int, capacity: int, device: torch.device):
        lib = native.library()
        nbytes = lib.gk_puct_workspace_bytes(batch, capacity)
        if nbytes == 0:
            raise ValueError("invalid search size")
        self.batch, self.capacity, self.device = batch, capacity, device
        self.storage = torch.empty(nbytes, dtype=torch.uint8, device=device)
        buffers = native.PuctBuffers()
        native.call("gk_puct_buffers", native.ptr(self.storage), batch, capacity, buffers)
        base = self.storage.data_ptr()

        def view(address, count, dtype, shape):
            offset = address - base
            width = torch.empty((), dtype=dtype).element_size()
            return self.storage[offset:offset + count * width].view(dtype).view(shape)

        self.needs_eval = view(buffers.needs_eval, batch, torch.uint8, (batch,))
        self.leaf_bits = view(buffers.leaf_bits, batch * 16, torch.int32, (batch, 16))
        self.leaf_value = view(buffers.leaf_value, batch, torch.float32, (batch,))
        self.policy = view(buffers.policy, batch * ACTION_SIZE, torch.float32, (batch, ACTION_SIZE))
        self.noise = view(buffers.noise, batch * ACTION_SIZE, torch.float32, (batch, ACTION_SIZE))
        self.active = view(buffers.active, batch, torch.int32, (batch,))
        self.active_count = view(buffers.active_count, 1, torch.int32, (1,))
        self.errors = view(buffers.errors, batch, torch.int32, (batch,))
        self.leaf = view(buffers.leaf, batch, torch.int32, (batch,))
        self.root_allow = view(buffers.root_allow, batch * 3, torch.int32, (batch, 3))
        self.node_visits = view(buffers.node_visits, batch * capacity, torch.int32, (batch, capacity))

    def root_masks(self, rows: torch.Tensor) -> torch.Tensor:
        """bool [len(rows), 82]: the root candidates of the given trees."""
        actions = torch.arange(ACTION_SIZE, device=rows.device)
        words = self.root_allow.index_select(0, rows)[:, actions // 32]
        return ((words >> (actions % 32)) & 1).bool()

    @property
    def pointer(self):
        return native.ptr(self.storage)


def encode_packed(bits: torch.Tensor):
    """Schema-1 features [N,10,9,9] and masks [N,82] of packed states."""
    n = bits.shape[0]
    features = torch.empty((n, 10, 9, 9), dtype=torch.float32, device=bits.device)
    masks = torch.empty((n, ACTION_SIZE), dtype=torch.bool, device=bits.device)
    if n:
        stream = _launch_scope(bits.device, bits, features, masks)
        native.call("gk_encode_bits", native.ptr(bits), native.ptr(features), native.ptr(masks), n, stream)
    return features, masks


class GpuPUCT:
    """Independent GPU trees, one leaf per tree per simulation.

    Mirrors python/kingdom_ai/gpu_puct.py:383-542: the model is copied to the
    search device in eval mode (the caller's module is never modified), calls
    are serialised by a lock, and one aggregate error word is read after all
    simulations (bit 2: invalid model output -> ValueError; otherwise
    RuntimeError).
    """

    def __init__(self, model, options=None, device="cuda"):
        if options is None:
            options = GpuPUCTOptions()
        if not isinstance(options, GpuPUCTOptions):
            raise TypeError("options must be GpuPUCTOptions")
        self.options = options
        self.device = native.require_cuda(device)
        if isinstance(model, HashEvaluator):
            self.model = model
            self._kind = "hash"
        elif isinstance(model, nn.Module):
            self.model = copy.deepcopy(model).to(device=self.device, dtype=torch.float32).eval()
            self._kind = "module"
            from .model import NativePolicyValueNet, native_supported
            if native_supported(self.model):
                self._native_net = NativePolicyValueNet(self.model.cpu(), device=self.device)
                self._kind = "native"
        else:
            raise TypeError("model must be a torch.nn.Module or a HashEvaluator")
        native.library()
        self._noise_calls = 0
        self._seed = options.seed
        self._lock = threading.Lock()
        self._workspace = None

    def reset_seed(self, seed=None):
        """Restart the dedicated root-noise stream without changing global RNGs."""
        if seed is None:
            seed = self.options.seed
        if type(seed) is not int or not 0 <= seed <= 2**64 - 1:
            raise ValueError("seed must be an unsigned 64-bit integer")
        with self._lock:
            self._seed = seed
            self._noise_calls = 0

    def search(self, state: GpuStateBatch) -> GpuSearchResult:
        if not isinstance(state, GpuStateBatch):
            raise TypeError("Expected a GpuStateBatch")
        GpuStateBatch(state.states)
        if state.device != self.device:
            raise ValueError("State and searcher must use the same CUDA device")
        with self._lock, torch.cuda.device(self.device), torch.inference_mode():
            return self._search(state.to_bits())

    def search_packed(self, roots: torch.Tensor) -> GpuSearchResult:
        """Search from packed states (int32 [N,16]) already on the device."""
        with self._lock, torch.cuda.device(self.device), torch.inference_mode():
            return self._search(roots)

    # -- internals -----------------------------------------------------------
    def _options_struct(self):
        o = self.options
        return native.PuctOptions(float(o.c_puct), float(o.dirichlet_epsilon),
                                  1 if o.fpu_reduction is not None else 0, float(o.fpu_reduction or 0.0))

    def _workspace_for(self, batch, capacity):
        ws = self._workspace
        if ws is None or ws.batch != batch or ws.capacity != capacity:
            self._workspace = None
            ws = self._workspace = SearchWorkspace(batch, capacity, self.device)
        return ws

    def _evaluate(self, ws: SearchWorkspace, stream):
        if self._kind == "hash":
            native.call("gk_puct_hash_eval", ws.pointer, ws.batch, ws.capacity, stream)
            return
        if self._kind == "native":
            self._native_net.evaluate_workspace(ws, stream)
            return
        active = ws.needs_eval.nonzero(as_tuple=False).flatten()
        if active.numel() == 0:
            return
        features, masks = encode_packed(ws.leaf_bits.index_select(0, active))
        if self.options.tactical_checks:
            # A root leaf's mask is its tactically narrowed candidate set
            # (gpu_puct.py:475-479, 499); the features keep rule legality.
            at_root = ws.leaf.index_select(0, active) == 0
            masks = torch.where(at_root[:, None], masks & ws.root_masks(active), masks)
        logits, values = self.model(features)
        if logits.shape != (active.numel(), ACTION_SIZE) or values.shape != (active.numel(),):
            raise ValueError("model must return logits [N, 82] and values [N]")
        if logits.device != self.device or values.device != self.device:
            raise ValueError("model outputs must stay on the search CUDA device")
        if not logits.is_floating_point() or not values.is_floating_point():
            raise TypeError("model logits and values must be floating-point tensors")
        logits = logits.to(dtype=torch.float32)
        values = values.to(dtype=torch.float32)
        weights = torch.softmax(logits.masked_fill(~masks, -torch.inf), dim=1).masked_fill(~masks, 0.0)
        ws.policy.index_copy_(0, active, weights)
        ws.leaf_value.index_copy_(0, active, values)

    def _search(self, roots: torch.Tensor) -> GpuSearchResult:
        batch = roots.shape[0]
        if batch < 1:
            raise ValueError("Search needs at least one state")
        capacity = self.options.simulations + 1
        device = self.device
        ws = self._workspace_for(batch, capacity)
        roots = roots.contiguous()
        opts = self._options_struct()
        stream = _launch_scope(device, roots, ws.storage)
        native.call("gk_puct_begin", ws.pointer, batch, capacity, native.ptr(roots), stream)
        if self.options.tactical_checks:
            native.call("gk_puct_root_tactics", ws.pointer, batch, capacity, stream)
        self._evaluate(ws, stream)
        if self.options.dirichlet_epsilon:
            native.call("gk_puct_noise", ws.pointer, batch, capacity, self._seed & (2**64 - 1),
                        (self._noise_calls << 32) & (2**64 - 1), float(self.options.dirichlet_alpha), stream)
            self._noise_calls += 1
        native.call("gk_puct_expand_backup", ws.pointer, batch, capacity, opts, 0, stream)
        for _ in range(self.options.simulations):
            native.call("gk_puct_select", ws.pointer, batch, capacity, opts, stream)
            self._evaluate(ws, stream)
            native.call("gk_puct_expand_backup", ws.pointer, batch, capacity, opts, 1, stream)
        out = _allocate_results(batch, device)
        native.call("gk_puct_finish", ws.pointer, batch, capacity, out.struct, stream)
        code = int(out.status.item())
        if self._kind == "native":
            self._native_net.check()
        if code:
            if code & 2:
                raise ValueError("PUCT model must return finite logits and finite values in [-1, 1]")
            raise RuntimeError("CUDA PUCT detected an illegal edge or exhausted tree capacity")
        return out.result()


class _Results:
    def __init__(self, batch, device):
        z = lambda shape, dtype: torch.zeros(shape, dtype=dtype, device=device)  # noqa: E731
        self.actions = torch.full((batch,), -1, dtype=torch.int64, device=device)
        self.visits = z((batch, ACTION_SIZE), torch.int32)
        self.policy = z((batch, ACTION_SIZE), torch.float32)
        self.values = z((batch,), torch.float32)
        self.simulations = z((batch,), torch.int32)
        self.evaluations = z((batch,), torch.int32)
        self.priors = z((batch, ACTION_SIZE), torch.float64)
        self.best_values = z((batch,), torch.float32)
        self.nodes = z((batch,), torch.int32)
        self.root_values = z((batch,), torch.float64)
        self.status = z((1,), torch.int32)
        p = lambda t: t.data_ptr()  # noqa: E731
        self.struct = native.PuctResults(
            p(self.actions), p(self.visits), p(self.policy), p(self.values), p(self.simulations),
            p(self.evaluations), p(self.priors), p(self.best_values), p(self.nodes), p(self.root_values),
            p(self.status))

    def result(self):
        return GpuSearchResult(actions=self.actions, visits=self.visits, policy=self.policy, values=self.values,
                               simulations=self.simulations, network_evaluations=self.evaluations,
                               priors=self.priors, best_values=self.best_values, nodes=self.nodes,
                               root_values=self.root_values)


def _allocate_results(batch, device):
    return _Results(batch, device)


def search_hash(roots: torch.Tensor, simulations: int, c_puct: float = 1.5,
                workspace: SearchWorkspace | None = None) -> GpuSearchResult:
    """Full injected-evaluator search in one native call (no host synchronisation).

    `workspace` (batch, simulations + 1) may be passed to reuse it and read
    the trees afterwards."""
    batch = roots.shape[0]
    device = roots.device
    ws = workspace if workspace is not None else SearchWorkspace(batch, simulations + 1, device)
    if (ws.batch, ws.capacity) != (batch, simulations + 1):
        raise ValueError("workspace size does not match the search")
    out = _allocate_results(batch, device)
    opts = native.PuctOptions(float(c_puct), 0.0, 0, 0.0)
    with torch.cuda.device(device):
        stream = _launch_scope(device, roots, ws.storage)
        native.call("gk_puct_search_hash", ws.pointer, batch, simulations, native.ptr(roots.contiguous()), opts,
                    out.struct, stream)
    return out.result()
