"""ctypes bindings for the CPU checkers (TEST INFRASTRUCTURE ONLY).

``Oracle`` loads ``oracle/_build/libgkoracle.so`` (the plain-C restatement in
``oracle/gk_oracle.c``). ``Reference`` loads ``oracle/_ref/libgkref.so`` (the
reference C++ engine compiled from its own sources plus
``oracle/ref_harness.cpp``); it exists only where it was built.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module. The product never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libgkoracle.so"
REF_SO = HERE / "_ref" / "libgkref.so"
# Root of the reference sources, for building oracle/_ref: GK_REFERENCE_ROOT or
# the `root` argument of build_reference (no default).
REFERENCE_ROOT = os.environ.get("GK_REFERENCE_ROOT")

STATE_WIDTH = 170
ACTIONS = 82
FEATURES = 810

_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u64 = ctypes.c_uint64
_i64 = ctypes.c_int64
_int = ctypes.c_int


def build_oracle(force: bool = False) -> Path:
    """Compile the plain-C oracle with gcc (seconds) if it is missing."""
    if force or not ORACLE_SO.exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    return ORACLE_SO


def build_reference(force: bool = False, root: str | os.PathLike | None = None) -> Path | None:
    """Compile the reference engine from its sources under `root` (or
    GK_REFERENCE_ROOT) when they are present; else keep the built library."""
    if REF_SO.exists() and not force:
        return REF_SO
    root = root or REFERENCE_ROOT
    if root is None or not (Path(root) / "engine" / "src" / "State.cpp").exists():
        return REF_SO if REF_SO.exists() else None
    subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={Path(root)}"], check=True)
    return REF_SO


def _bind(lib, name, args, res=None):
    fn = getattr(lib, name)
    fn.argtypes = args
    fn.restype = res
    return fn


class Oracle:
    """The plain-C restatement of rules, encoder, generators and PUCT."""

    def __init__(self):
        self.lib = ctypes.CDLL(str(build_oracle()))
        L = self.lib
        _bind(L, "gko_initial", [_i32p, _int])
        _bind(L, "gko_play", [_i32p, _int], _int)
        _bind(L, "gko_legal", [_i32p, _int], _int)
        _bind(L, "gko_play_batch", [_i32p, _i32p, _u8p, _i64])
        _bind(L, "gko_encode_batch", [_i32p, _f32p, _u8p, _i64])
        _bind(L, "gko_random_playouts", [_u64, _u64, _i64, _int, _i8p, _i32p])
        _bind(L, "gko_gen_positions", [_u64, _u64, _i64, _i32p])
        _bind(L, "gko_eval", [_i32p, _f32p, _f32p])
        _bind(L, "gko_puct_search", [_i32p, _int, ctypes.c_double, _i32p, _f64p, _i32p, _f64p], _int)
        _bind(L, "gko_puct_search_uniform", [_i32p, _int, ctypes.c_double, _i32p, _f64p, _i32p, _f64p], _int)
        _bind(L, "gko_puct_search_batch", [_i32p, _i64, _int, ctypes.c_double, _i32p, _i32p, _f64p, _int], _int)
        _bind(L, "gko_root_tactics", [_i32p, _i8p, _u8p])
        _bind(L, "gko_puct_search_tactics", [_i32p, _int, ctypes.c_double, _int, _i32p, _f64p, _i32p, _f64p], _int)
        _bind(L, "gko_selfplay_hash_games", [_u64, _u64, _i64, _int, _int, ctypes.c_double, _int, ctypes.c_double,
                                             ctypes.c_double, _int, _u8p, _f32p, _i32p, _i32p, _int])
        _bind_batched(L, "gko")

    def selfplay_hash(self, sample_seed: int, games: int, simulations: int, *, first_game: int = 0,
                      c_puct: float = 1.5, temperature_moves: int = 10, temperature: float = 1.0,
                      final_temperature: float = 0.0, neutral: int = 40, tactics: bool = False,
                      threads: int | None = None):
        """Games first_game .. first_game + games - 1 as the device self-play
        engine plays them with the injected evaluator and no root noise.

        Returns (plies [n], actions [n, 166] uint8, policy [n, 166, 82] f32,
        final records [n, 170]); plies < 0 marks a failed game.
        """
        width = 2 * 81 + 4
        actions = np.zeros((games, width), dtype=np.uint8)
        policy = np.zeros((games, width, ACTIONS), dtype=np.float32)
        recs = np.zeros((games, STATE_WIDTH), dtype=np.int32)
        plies = np.zeros(games, dtype=np.int32)
        threads = threads or max(1, min(len(os.sched_getaffinity(0)), 64))
        self.lib.gko_selfplay_hash_games(sample_seed, first_game, games, neutral, simulations, c_puct,
                                         temperature_moves, temperature, final_temperature, int(tactics), actions,
                                         policy, recs, plies, threads)
        return plies, actions, policy, recs

    def batched(self, simulations, c_puct=1.5, leaf_batch=8, reuse=True, evaluator="hash"):
        """The restated BatchedPUCT searcher (oracle/gk_oracle.c)."""
        return BatchedSearcher(self.lib, "gko", simulations, c_puct, leaf_batch, reuse, evaluator)

    def initial(self, n: int = 1, neutral: int = 40) -> np.ndarray:
        recs = np.zeros((n, STATE_WIDTH), dtype=np.int32)
        for i in range(n):
            row = np.zeros(STATE_WIDTH, dtype=np.int32)
            self.lib.gko_initial(row, neutral)
            recs[i] = row
        return recs

    def play(self, recs: np.ndarray, actions) -> np.ndarray:
        """In-place batched transition; returns accepted flags (uint8)."""
        recs = np.ascontiguousarray(recs, dtype=np.int32)
        actions = np.ascontiguousarray(actions, dtype=np.int32)
        accepted = np.zeros(len(recs), dtype=np.uint8)
        self.lib.gko_play_batch(recs, actions, accepted, len(recs))
        return recs, accepted

    def encode(self, recs: np.ndarray):
        recs = np.ascontiguousarray(recs, dtype=np.int32)
        features = np.zeros((len(recs), FEATURES), dtype=np.float32)
        masks = np.zeros((len(recs), ACTIONS), dtype=np.uint8)
        self.lib.gko_encode_batch(recs, features, masks, len(recs))
        return features.reshape(len(recs), 10, 9, 9), masks.astype(bool)

    def random_playouts(self, seed: int, n: int, first: int = 0, neutral: int = 40):
        boards = np.zeros((n, 81), dtype=np.int8)
        infos = np.zeros((n, 5), dtype=np.int32)
        self.lib.gko_random_playouts(seed, first, n, neutral, boards, infos)
        return boards, infos

    def gen_positions(self, seed: int, n: int, first: int = 0) -> np.ndarray:
        recs = np.zeros((n, STATE_WIDTH), dtype=np.int32)
        self.lib.gko_gen_positions(seed, first, n, recs)
        return recs

    def evaluate(self, rec: np.ndarray):
        w = np.zeros(ACTIONS, dtype=np.float32)
        v = np.zeros(1, dtype=np.float32)
        self.lib.gko_eval(np.ascontiguousarray(rec, dtype=np.int32), w, v)
        return w, float(v[0])

    def root_tactics(self, rec: np.ndarray):
        """Per-action outcome (+1 win, -1 loss or losing reply, 0) and the narrowed root candidates."""
        outcome = np.zeros(ACTIONS, dtype=np.int8)
        allow = np.zeros(ACTIONS, dtype=np.uint8)
        self.lib.gko_root_tactics(np.ascontiguousarray(rec, dtype=np.int32), outcome, allow)
        return outcome, allow.astype(bool)

    def puct(self, rec: np.ndarray, simulations: int, c_puct: float = 1.5, uniform: bool = False,
             tactics: bool = False):
        visits = np.zeros(ACTIONS, dtype=np.int32)
        priors = np.zeros(ACTIONS, dtype=np.float64)
        stats = np.zeros(4, dtype=np.int32)
        values = np.zeros(2, dtype=np.float64)
        rec = np.ascontiguousarray(rec, dtype=np.int32)
        if tactics:
            status = self.lib.gko_puct_search_tactics(rec, simulations, c_puct, int(uniform), visits, priors, stats,
                                                      values)
        else:
            fn = self.lib.gko_puct_search_uniform if uniform else self.lib.gko_puct_search
            status = fn(rec, simulations, c_puct, visits, priors, stats, values)
        if status != 0:
            raise RuntimeError(f"oracle PUCT failed ({status})")
        return dict(visits=visits, priors=priors, best=int(stats[0]), simulations=int(stats[1]),
                    nodes=int(stats[2]), evaluations=int(stats[3]), root_value=float(values[0]),
                    best_value=float(values[1]))

    def puct_batch(self, recs: np.ndarray, simulations: int, c_puct: float = 1.5, threads: int = 1):
        recs = np.ascontiguousarray(recs, dtype=np.int32)
        n = len(recs)
        visits = np.zeros((n, ACTIONS), dtype=np.int32)
        best = np.zeros(n, dtype=np.int32)
        roots = np.zeros(n, dtype=np.float64)
        status = self.lib.gko_puct_search_batch(recs, n, simulations, c_puct, visits, best, roots, threads)
        if status != 0:
            raise RuntimeError(f"oracle PUCT failed ({status})")
        return visits, best, roots


EVALUATORS = {"hash": 0, "uniform": 1, "ramp": 2}
BATCHED_STATS = ("network_evaluations", "inference_batches", "max_observed_batch_size", "reused_nodes",
                 "inherited_visits", "advance_calls", "reuse_hits")


def _bind_batched(lib, prefix):
    vp = ctypes.c_void_p
    _bind(lib, f"{prefix}_bpuct_new", [_i64, ctypes.c_double, _i64, _int, _int], vp)
    _bind(lib, f"{prefix}_bpuct_free", [vp])
    _bind(lib, f"{prefix}_bpuct_clear", [vp])
    root = _i32p if prefix == "gko" else vp
    _bind(lib, f"{prefix}_bpuct_search", [vp, root, _i32p, _f64p, _f64p, _u8p, _i32p, _f64p], _int)
    _bind(lib, f"{prefix}_bpuct_advance", [vp, _int], _int)
    _bind(lib, f"{prefix}_bpuct_stats", [vp, ctypes.POINTER(ctypes.c_int64)])


class BatchedSearcher:
    """One BatchedPUCT searcher (leaf batches, virtual loss, subtree reuse):
    the plain-C restatement ("gko", searched from wire records) or the
    reference engine ("gkr", searched from RefState handles)."""

    def __init__(self, lib, prefix, simulations, c_puct, leaf_batch, reuse, evaluator):
        self.lib, self.prefix = lib, prefix
        self.h = getattr(lib, f"{prefix}_bpuct_new")(simulations, c_puct, leaf_batch, int(reuse),
                                                      EVALUATORS[evaluator])
        if not self.h:
            raise ValueError("invalid BatchedPUCT options")

    def __del__(self):
        try:
            getattr(self.lib, f"{self.prefix}_bpuct_free")(self.h)
        except Exception:
            pass

    def clear(self):
        getattr(self.lib, f"{self.prefix}_bpuct_clear")(self.h)

    def search(self, root):
        """root: a wire record (oracle) or a RefState (reference). Raises
        ValueError with the failure code when the search fails."""
        visits = np.zeros(ACTIONS, dtype=np.int32)
        priors = np.zeros(ACTIONS, dtype=np.float64)
        values = np.zeros(ACTIONS, dtype=np.float64)
        legal = np.zeros(ACTIONS, dtype=np.uint8)
        info = np.zeros(4, dtype=np.int32)
        out = np.zeros(2, dtype=np.float64)
        arg = root.h if isinstance(root, RefState) else np.ascontiguousarray(root, dtype=np.int32)
        status = getattr(self.lib, f"{self.prefix}_bpuct_search")(self.h, arg, visits, priors, values, legal, info,
                                                                  out)
        if status != 0:
            raise ValueError(f"BatchedPUCT search failed ({status})")
        return dict(visits=visits, priors=priors, move_values=values, legal=legal.astype(bool), best=int(info[0]),
                    simulations=int(info[1]), nodes=int(info[2]), evaluations=int(info[3]),
                    root_value=float(out[0]), best_value=float(out[1]))

    def advance(self, action):
        return bool(getattr(self.lib, f"{self.prefix}_bpuct_advance")(self.h, int(action)))

    @property
    def stats(self):
        out = (ctypes.c_int64 * len(BATCHED_STATS))()
        getattr(self.lib, f"{self.prefix}_bpuct_stats")(self.h, out)
        return dict(zip(BATCHED_STATS, (int(v) for v in out)))


class Reference:
    """Driver for the reference C++ engine compiled from its own sources."""

    def __init__(self):
        path = build_reference()
        if path is None:
            raise FileNotFoundError("the reference engine was not built (oracle/_ref)")
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        vp = ctypes.c_void_p
        _bind(L, "gkr_state_new", [_int], vp)
        _bind(L, "gkr_state_from_board", [_i32p, _int], vp)
        _bind(L, "gkr_state_copy", [vp], vp)
        _bind(L, "gkr_state_free", [vp])
        _bind(L, "gkr_state_play", [vp, _int], _int)
        _bind(L, "gkr_state_record", [vp, _i32p])
        _bind(L, "gkr_state_score", [vp, _i32p])
        _bind(L, "gkr_state_legal", [vp, _i32p], _int)
        _bind(L, "gkr_state_encode", [vp, _f32p, _u8p])
        _bind(L, "gkr_random_playouts", [_u64, _u64, _i64, _int, _int, _int, _i8p, _i32p])
        _bind(L, "gkr_gen_positions", [_u64, _u64, _i64, _int, _i32p])
        _bind(L, "gkr_gen_position_state", [_u64, _u64], vp)
        _bind(L, "gkr_encode_positions", [_u64, _u64, _i64, _int, _f32p, _u8p])
        _bind(L, "gkr_puct_search", [vp, _int, ctypes.c_double, _i32p, _f64p, _i32p, _f64p], _int)
        _bind(L, "gkr_puct_positions", [_u64, _u64, _i64, _int, ctypes.c_double, _int, _i32p, _i32p], _int)
        _bind(L, "gkr_states_generate", [_u64, _u64, _i64, _int], vp)
        _bind(L, "gkr_states_free", [vp])
        _bind(L, "gkr_states_encode", [vp, _int, _f32p, _u8p])
        _bind_batched(L, "gkr")

    def batched(self, simulations, c_puct=1.5, leaf_batch=8, reuse=True, evaluator="hash"):
        """The reference's own ``kingdom::BatchedPUCT`` (mcts/src/BatchedPUCT.cpp)."""
        return BatchedSearcher(self.lib, "gkr", simulations, c_puct, leaf_batch, reuse, evaluator)

    def random_playouts(self, seed, n, first=0, neutral=40, fast=False, threads=1):
        boards = np.zeros((n, 81), dtype=np.int8)
        infos = np.zeros((n, 5), dtype=np.int32)
        self.lib.gkr_random_playouts(seed, first, n, neutral, int(fast), threads, boards, infos)
        return boards, infos

    def gen_positions(self, seed, n, first=0, threads=1):
        recs = np.zeros((n, STATE_WIDTH), dtype=np.int32)
        self.lib.gkr_gen_positions(seed, first, n, threads, recs)
        return recs

    def encode_positions(self, seed, n, first=0, threads=1):
        features = np.zeros((n, FEATURES), dtype=np.float32)
        masks = np.zeros((n, ACTIONS), dtype=np.uint8)
        self.lib.gkr_encode_positions(seed, first, n, threads, features, masks)
        return features.reshape(n, 10, 9, 9), masks.astype(bool)

    def encode_timed(self, seed, n, threads=1, repeats=1):
        """Seconds per kingdom::encode_puct_position pass over n generated
        positions on `threads` workers (generation excluded), and the outputs."""
        import time
        h = self.lib.gkr_states_generate(seed, 0, n, threads)
        features = np.zeros((n, FEATURES), dtype=np.float32)
        masks = np.zeros((n, ACTIONS), dtype=np.uint8)
        try:
            self.lib.gkr_states_encode(h, threads, features, masks)  # warm
            start = time.perf_counter()
            for _ in range(repeats):
                self.lib.gkr_states_encode(h, threads, features, masks)
            seconds = (time.perf_counter() - start) / repeats
        finally:
            self.lib.gkr_states_free(h)
        return seconds, features.reshape(n, 10, 9, 9), masks.astype(bool)

    def puct_positions(self, seed, n, simulations, c_puct=1.5, first=0, threads=1):
        visits = np.zeros((n, ACTIONS), dtype=np.int32)
        best = np.zeros(n, dtype=np.int32)
        status = self.lib.gkr_puct_positions(seed, first, n, simulations, c_puct, threads, visits, best)
        if status != 0:
            raise RuntimeError("reference PUCT failed")
        return visits, best


class RefState:
    """A reference ``kingdom::State`` held through the harness."""

    def __init__(self, ref: Reference, handle):
        if not handle:
            raise ValueError("the reference rejected this position")
        self.ref, self.h = ref, handle

    @classmethod
    def initial(cls, ref, neutral=40):
        return cls(ref, ref.lib.gkr_state_new(neutral))

    @classmethod
    def from_board(cls, ref, cells, to_play):
        cells = np.ascontiguousarray(cells, dtype=np.int32).reshape(81)
        return cls(ref, ref.lib.gkr_state_from_board(cells, int(to_play)))

    @classmethod
    def generated(cls, ref, seed, index):
        return cls(ref, ref.lib.gkr_gen_position_state(seed, index))

    def copy(self):
        return RefState(self.ref, self.ref.lib.gkr_state_copy(self.h))

    def __del__(self):
        try:
            self.ref.lib.gkr_state_free(self.h)
        except Exception:
            pass

    def play(self, action: int) -> bool:
        return bool(self.ref.lib.gkr_state_play(self.h, int(action)))

    def record(self) -> np.ndarray:
        rec = np.zeros(STATE_WIDTH, dtype=np.int32)
        self.ref.lib.gkr_state_record(self.h, rec)
        return rec

    def score(self):
        out = np.zeros(2, dtype=np.int32)
        self.ref.lib.gkr_state_score(self.h, out)
        return int(out[0]), int(out[1])

    def legal(self):
        out = np.zeros(ACTIONS, dtype=np.int32)
        n = self.ref.lib.gkr_state_legal(self.h, out)
        return out[:n].tolist()

    def encode(self):
        features = np.zeros(FEATURES, dtype=np.float32)
        mask = np.zeros(ACTIONS, dtype=np.uint8)
        self.ref.lib.gkr_state_encode(self.h, features, mask)
        return features.reshape(10, 9, 9), mask.astype(bool)

    def puct(self, simulations, c_puct=1.5):
        visits = np.zeros(ACTIONS, dtype=np.int32)
        priors = np.zeros(ACTIONS, dtype=np.float64)
        stats = np.zeros(4, dtype=np.int32)
        values = np.zeros(2, dtype=np.float64)
        if self.ref.lib.gkr_puct_search(self.h, simulations, c_puct, visits, priors, stats, values) != 0:
            raise RuntimeError("reference PUCT failed")
        return dict(visits=visits, priors=priors, best=int(stats[0]), simulations=int(stats[1]),
                    nodes=int(stats[2]), evaluations=int(stats[3]), root_value=float(values[0]),
                    best_value=float(values[1]))


def replay_violation(features, legal_mask, policy, value, to_play):
    """Restatement of the reference's replay row checks (python/kingdom_ai/replay.py:35-74)
    in numpy: the message of the first check some row fails, or None. The
    policy sum is taken in float64."""
    f = np.asarray(features, dtype=np.float32).reshape(-1, 10, 9, 9)
    m = np.asarray(legal_mask, dtype=bool).reshape(-1, 82)
    p = np.asarray(policy, dtype=np.float32).reshape(-1, 82)
    v = np.asarray(value, dtype=np.float32).reshape(-1)
    t = np.asarray(to_play, dtype=np.int8).reshape(-1)
    if len(f) == 0:
        return None
    with np.errstate(invalid="ignore"):
        if not np.isfinite(f).all() or not np.isfinite(p).all():
            return "Replay features and policies must be finite"
        if ((f < 0) | (f > 1)).any():
            return "Replay features must lie between zero and one"
        if any(((f[:, q] != 0) & (f[:, q] != 1)).any() for q in (0, 1, 2, 3, 4, 5, 9)):
            return "Binary observation planes must contain only zero or one"
        if any((f[:, q].reshape(len(f), 81) != f[:, q, :1, :1].reshape(len(f), 1)).any() for q in (5, 6, 7, 8)):
            return "Scalar observation planes must be constant"
        if ((t != 1) & (t != 2)).any():
            return "Replay actors must be Black or White"
        if (f[:, 5, 0, 0] != (t == 1).astype(np.float32)).any():
            return "Observation player perspective does not match its actor"
        if ((f[:, 8, 0, 0] != 0) & (f[:, 8, 0, 0] != 0.5)).any():
            return "Replay observations must be taken before game termination"
        if not m[:, 81].all():
            return "Nonterminal replay observations must allow passing"
        if not np.array_equal(f[:, 9].reshape(len(f), 81) != 0, m[:, :81]):
            return "Observation legal placements do not match the action mask"
        if (f[:, :3].sum(axis=1) > 1).any():
            return "Stone observation planes cannot overlap"
        if (f[:, 2].sum(axis=(1, 2)) > 1).any():
            return "An observation can contain at most one neutral stone"
        if (f[:, 3] + f[:, 4] > 1).any():
            return "Opposing territory observation planes cannot overlap"
        if (p < 0).any() or (p[~m] != 0).any():
            return "Replay policies must assign non-negative mass to legal actions only"
        if not (np.abs(p.astype(np.float64).sum(axis=1) - 1.0) <= 1e-6).all():
            return "Each replay policy must sum to one"
        if not np.isfinite(v).all() or ((v != -1) & (v != 1)).any():
            return "Completed-game replay values must be -1 or +1"
    return None
