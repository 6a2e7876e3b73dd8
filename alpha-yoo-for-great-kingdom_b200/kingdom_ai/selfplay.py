"""Continuous batched self-play on one GPU (native network, no host syncs per ply).

``SelfPlayEngine`` keeps `lanes` games in flight; ``step()`` plays one ply in
every lane through a single ``gk_selfplay_ply`` call: a full PUCT search per
lane with the tcgen05 network as leaf evaluator, then one move per lane.
Finished games write their samples to a device FIFO ``ReplayRing`` in the row
schema of the reference ReplayBuffer (python/kingdom_ai/replay.py:106-125)
and their lanes start the next game.

Randomness is keyed by (seed, game id, ply), so the games played are the same
however lanes are split across GPUs: rank r of W plays game ids
r*lanes + i, then + W*lanes per finished game.

Each finished game is also written to an optional device ``GameLog``: its id,
the actions played (which replay it from the start position), winner, end
reason, final position and the index of its first replay row. With
``game_limit`` set, a lane whose next game id would reach the limit parks on
its finished position, so a run plays exactly the games below the limit.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as native
from .gpu_puct import GpuPUCTOptions, SearchWorkspace
from .gpu_rules import _launch_scope
from .model import NativePolicyValueNet, PolicyValueNet

COUNTER_NAMES = ("moves", "games", "rows", "errors", "black_wins", "white_wins", "capture_endings",
                 "evaluations")


class SelfPlayParams(ctypes.Structure):
    _fields_ = [("simulations", ctypes.c_int), ("c_puct", ctypes.c_double), ("dirichlet_alpha", ctypes.c_double),
                ("dirichlet_epsilon", ctypes.c_double), ("fpu_enabled", ctypes.c_int),
                ("fpu_reduction", ctypes.c_double), ("temperature_moves", ctypes.c_int),
                ("temperature", ctypes.c_double), ("final_temperature", ctypes.c_double),
                ("seed", ctypes.c_uint64), ("game_stride", ctypes.c_uint64), ("neutral_cell", ctypes.c_int),
                ("tactical_checks", ctypes.c_int), ("sample_seed", ctypes.c_uint64),
                ("game_limit", ctypes.c_uint64)]


class ReplayStruct(ctypes.Structure):
    _fields_ = [("features", ctypes.c_void_p), ("masks", ctypes.c_void_p), ("policy", ctypes.c_void_p),
                ("value", ctypes.c_void_p), ("to_play", ctypes.c_void_p), ("capacity", ctypes.c_int64)]


class GameLogStruct(ctypes.Structure):
    _fields_ = [("game_id", ctypes.c_void_p), ("first_row", ctypes.c_void_p), ("plies", ctypes.c_void_p),
                ("winner", ctypes.c_void_p), ("reason", ctypes.c_void_p), ("final_state", ctypes.c_void_p),
                ("actions", ctypes.c_void_p), ("capacity", ctypes.c_int64)]


GAME_ACTIONS = 2 * 81 + 4  # GK_GAME_ACTIONS: longest game plus slack


class SelfPlayBuffers(ctypes.Structure):
    _fields_ = [("states", ctypes.c_void_p), ("lane_ply", ctypes.c_void_p), ("game_id", ctypes.c_void_p),
                ("counters", ctypes.c_void_p), ("last_action", ctypes.c_void_p), ("last_policy", ctypes.c_void_p)]


def _bind():
    lib = native.library()
    if getattr(lib, "_selfplay_bound", False):
        return lib
    native.register("gk_selfplay_workspace_bytes", [ctypes.c_int64], ctypes.c_size_t)
    native.register("gk_selfplay_reset", [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64,
                                          ctypes.c_void_p])
    native.register("gk_selfplay_buffers", [ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(SelfPlayBuffers)])
    native.register("gk_selfplay_ply", [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                        ctypes.POINTER(native.NetStruct), ctypes.POINTER(SelfPlayParams),
                                        ctypes.POINTER(ReplayStruct), ctypes.POINTER(GameLogStruct),
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p])
    native.register("gk_timer_create", [ctypes.c_int], ctypes.c_void_p)
    native.register("gk_timer_destroy", [ctypes.c_void_p], None)
    native.register("gk_timer_reset", [ctypes.c_void_p], None)
    native.register("gk_timer_read", [ctypes.c_void_p, ctypes.POINTER(ctypes.c_double),
                                      ctypes.POINTER(ctypes.c_int)])
    lib._selfplay_bound = True
    return lib


class ReplayRing:
    """Device FIFO of training rows (features, legal mask, policy, value, to_play)."""

    ROW_BYTES = 810 * 4 + 82 + 82 * 4 + 4 + 1  # 3655, as replay.py:109

    def __init__(self, capacity: int, device):
        self.capacity = int(capacity)
        self.device = torch.device(device)
        c = max(self.capacity, 1)
        self.features = torch.zeros((c, 10, 9, 9), dtype=torch.float32, device=self.device)
        self.masks = torch.zeros((c, 82), dtype=torch.bool, device=self.device)
        self.policy = torch.zeros((c, 82), dtype=torch.float32, device=self.device)
        self.value = torch.zeros((c,), dtype=torch.float32, device=self.device)
        self.to_play = torch.zeros((c,), dtype=torch.int8, device=self.device)
        self.struct = ReplayStruct(self.features.data_ptr(), self.masks.data_ptr(), self.policy.data_ptr(),
                                   self.value.data_ptr(), self.to_play.data_ptr(), self.capacity)

    def rows(self, start: int, count: int):
        """Row indices [start, start + count) of the ring (modulo capacity)."""
        idx = (torch.arange(count, device=self.device, dtype=torch.int64) + start) % self.capacity
        return (self.features[idx], self.masks[idx], self.policy[idx], self.value[idx], self.to_play[idx])


class GameLog:
    """Device log of finished games; the k-th game to finish goes to slot k % capacity."""

    def __init__(self, capacity: int, device):
        self.capacity = int(capacity)
        self.device = torch.device(device)
        c = max(self.capacity, 1)
        z = lambda shape, dtype: torch.zeros(shape, dtype=dtype, device=self.device)  # noqa: E731
        self.game_id = z((c,), torch.int64)
        self.first_row = z((c,), torch.int64)
        self.plies = z((c,), torch.int32)
        self.winner = z((c,), torch.int8)
        self.reason = z((c,), torch.int8)
        self.final_state = z((c, 16), torch.int32)
        self.actions = z((c, GAME_ACTIONS), torch.uint8)
        self.struct = GameLogStruct(*(t.data_ptr() for t in (self.game_id, self.first_row, self.plies, self.winner,
                                                             self.reason, self.final_state, self.actions)),
                                    self.capacity)

    def read(self, count: int) -> dict:
        """The first `count` slots (count <= capacity) as host numpy arrays."""
        count = min(int(count), self.capacity)
        names = ("game_id", "first_row", "plies", "winner", "reason", "final_state", "actions")
        return {n: getattr(self, n)[:count].cpu().numpy() for n in names}


class Timer:
    """CUDA-event pairs recorded around the network tower inside a ply."""

    def __init__(self, pairs: int):
        lib = _bind()
        self.handle = lib.gk_timer_create(pairs)
        if not self.handle:
            raise RuntimeError("could not create CUDA events")

    def reset(self):
        native.library().gk_timer_reset(self.handle)

    def read(self):
        total, pairs = ctypes.c_double(), ctypes.c_int()
        native.call("gk_timer_read", self.handle, ctypes.byref(total), ctypes.byref(pairs))
        return total.value, pairs.value

    def __del__(self):
        try:
            native.library().gk_timer_destroy(self.handle)
        except Exception:
            pass


class SelfPlayEngine:
    """`lanes` concurrent games on one GPU, advanced one ply per ``step()``.

    `model` is a network the native kernels run (``PolicyValueNet``,
    ``GroupNormPolicyValueNet`` or a ``NativePolicyValueNet``), or
    ``HashEvaluator()`` / None for the injected evaluator. `seed` drives root
    noise and `sample_seed` (default: `seed`) move sampling. `game_log`
    slots record finished games; `game_limit` > 0 stops lanes at that game id.
    """

    def __init__(self, model, lanes: int, options: GpuPUCTOptions | None = None, *,
                 temperature: float = 1.0, temperature_moves: int | None = 10, final_temperature: float = 0.0,
                 replay_capacity: int = 1 << 20, seed: int | None = None, sample_seed: int | None = None,
                 rank: int = 0, world_size: int = 1, device="cuda", neutral=(4, 4), game_log: int = 0,
                 game_limit: int = 0, first_game: int | None = None, game_stride: int | None = None):
        from .gpu_puct import HashEvaluator

        lib = _bind()
        self.device = native.require_cuda(device)
        self.options = options or GpuPUCTOptions()
        self.lanes = int(lanes)
        if model is None or isinstance(model, HashEvaluator):
            self.net = None
        else:
            self.net = model if isinstance(model, NativePolicyValueNet) else NativePolicyValueNet(model, self.device)
        seed = self.options.seed if seed is None else seed
        sample_seed = seed if sample_seed is None else sample_seed
        neutral_cell = -1 if neutral is None else neutral[0] * 9 + neutral[1]
        self.params = SelfPlayParams(
            self.options.simulations, float(self.options.c_puct), float(self.options.dirichlet_alpha),
            float(self.options.dirichlet_epsilon), 1 if self.options.fpu_reduction is not None else 0,
            float(self.options.fpu_reduction or 0.0),
            self.options.simulations + 10**9 if temperature_moves is None else int(temperature_moves),
            float(temperature), float(final_temperature), seed & (2**64 - 1),
            world_size * self.lanes if game_stride is None else int(game_stride), neutral_cell,
            1 if self.options.tactical_checks else 0, sample_seed & (2**64 - 1), int(game_limit))
        self.first_game = rank * self.lanes if first_game is None else int(first_game)
        self.neutral_cell = neutral_cell
        nbytes = lib.gk_selfplay_workspace_bytes(self.lanes)
        self.storage = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.search = SearchWorkspace(self.lanes, self.options.simulations + 1, self.device)
        self.headfeat = torch.empty((self.lanes, 243), dtype=torch.float32, device=self.device)
        self.status = torch.zeros(2, dtype=torch.int32, device=self.device)
        self._load_status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.replay = ReplayRing(replay_capacity, self.device) if replay_capacity > 0 else None
        self.games = GameLog(game_log, self.device) if game_log > 0 else None
        bufs = SelfPlayBuffers()
        native.call("gk_selfplay_buffers", native.ptr(self.storage), self.lanes, bufs)
        base = self.storage.data_ptr()
        self.counters = self.storage[bufs.counters - base:bufs.counters - base + 64].view(torch.int64)
        self.states = self.storage[bufs.states - base:bufs.states - base + self.lanes * 64].view(torch.int32).view(
            self.lanes, 16)
        self.lane_ply = self.storage[bufs.lane_ply - base:bufs.lane_ply - base + self.lanes * 4].view(torch.int32)
        self.last_action = self.storage[bufs.last_action - base:bufs.last_action - base + self.lanes * 4].view(
            torch.int32)
        self.last_policy = self.storage[bufs.last_policy - base:bufs.last_policy - base + self.lanes * 82 * 4].view(
            torch.float32).view(self.lanes, 82)
        self.timer = None
        self._graph = None
        self._timed_graph = None  # (timer, graph): a ply whose tower launches record the timer's events
        self._stepped = False
        self.reset()

    def reset(self):
        with torch.cuda.device(self.device):
            stream = _launch_scope(self.device, self.storage)
            native.call("gk_selfplay_reset", native.ptr(self.storage), self.lanes, self.neutral_cell,
                        self.first_game, stream)

    def enable_timer(self, plies: int):
        """Record the network tower of the next `plies` plies with CUDA events."""
        self.timer = Timer(plies * (self.options.simulations + 1))
        return self.timer

    def set_simulations(self, simulations: int):
        """Search `simulations` per move from the next ply on (at most the options' count)."""
        if type(simulations) is not int or not 1 <= simulations <= self.options.simulations:
            raise ValueError("simulations must be an integer in [1, options.simulations]")
        if simulations != self.params.simulations:
            self._graph = self._timed_graph = None  # a captured ply has the old count baked in
        self.params.simulations = simulations

    def capture(self):
        """Record one ply as a CUDA graph; ``step()`` then replays it instead of
        issuing its 4 + 4 (S + 1) + S launches one by one.

        A ply's launches and their arguments are the same every ply (lane
        states, ply counters, game ids, counters and rings all live in device
        memory), so a replay is exactly a ``gk_selfplay_ply`` call. With a
        tower timer attached (``enable_timer``) a second graph is captured
        whose tower launches record the timer's first ply of event pairs;
        plies stepped with that timer replay it, so after them the timer holds
        the last such ply's tower times. Call after at least one ``step()`` at
        the current settings (the first ply sets per-device kernel attributes,
        which a capture may not do).
        """
        if not self._stepped:
            raise RuntimeError("step() once before capture()")
        self._graph = self._capture(None)
        if self.timer is not None:
            self.timer.reset()
            self._timed_graph = (self.timer, self._capture(self.timer))

    def _capture(self, timer):
        with torch.cuda.device(self.device):
            capture_stream = torch.cuda.Stream(self.device)
            capture_stream.wait_stream(torch.cuda.current_stream(self.device))
            graph = torch.cuda.CUDAGraph()
            # thread_local: other threads' CUDA calls (NCCL's, under torchrun)
            # do not invalidate this capture.
            with torch.cuda.stream(capture_stream), torch.cuda.graph(graph, stream=capture_stream,
                                                                     capture_error_mode="thread_local"):
                self._launch(1, timer=timer)
            torch.cuda.current_stream(self.device).wait_stream(capture_stream)
        return graph

    def step(self, plies: int = 1):
        graph = None
        if self.timer is None:
            graph = self._graph
        elif self._timed_graph is not None and self._timed_graph[0] is self.timer:
            graph = self._timed_graph[1]
        if graph is not None:
            with torch.cuda.device(self.device):
                for _ in range(plies):
                    graph.replay()
            return
        self._launch(plies, self.timer)
        self._stepped = True

    def _launch(self, plies: int, timer):
        with torch.cuda.device(self.device):
            stream = _launch_scope(self.device, self.storage, self.search.storage, self.headfeat)
            replay = self.replay.struct if self.replay is not None else None
            games = self.games.struct if self.games is not None else None
            net = self.net.struct if self.net is not None else None
            for _ in range(plies):
                native.call("gk_selfplay_ply", native.ptr(self.storage), self.search.pointer, self.lanes,
                            net, self.params, replay, games, native.ptr(self.headfeat),
                            native.ptr(self.status), timer.handle if timer else None, stream)

    def load_records(self, records: torch.Tensor):
        """Set every lane's position from wire records (int32 [lanes,170], host
        or device; a pinned host tensor is copied asynchronously). Lanes keep
        their game ids and ply counts; the next ply searches these positions."""
        if tuple(records.shape) != (self.lanes, 170) or records.dtype != torch.int32:
            raise ValueError("records must be int32 [lanes, 170]")
        with torch.cuda.device(self.device):
            dev = records.to(self.device, non_blocking=True) if records.device != self.device else records
            stream = _launch_scope(self.device, dev, self.storage)
            native.call("gk_records_to_bits", native.ptr(dev), native.ptr(self.states), native.ptr(self._load_status),
                        self.lanes, stream)

    def records(self, out: torch.Tensor | None = None) -> torch.Tensor:
        """Every lane's position as wire records (int32 [lanes,170] on the device)."""
        with torch.cuda.device(self.device):
            if out is None:
                out = torch.empty((self.lanes, 170), dtype=torch.int32, device=self.device)
            stream = _launch_scope(self.device, out, self.storage)
            native.call("gk_bits_to_records", native.ptr(self.states), native.ptr(out), self.lanes, stream)
        return out

    def stats(self) -> dict:
        values = self.counters.cpu().tolist()
        return dict(zip(COUNTER_NAMES, values))

    def check(self):
        if int(self._load_status.item()):
            raise ValueError("a loaded record is outside the wire format's value ranges")
        code = int(self.status[0].item())
        stats = self.stats()
        if code or stats["errors"]:
            raise RuntimeError(f"self-play reported status {code:#x}, {stats['errors']} rejected moves")
