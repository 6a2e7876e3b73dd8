"""The my_board_engine side of the boundary: encode_puct_batch and BatchedPUCT.

Where the reference's own compiled module (``my_board_engine``, installed with
pip under baseline/_ref) can be imported, the GPU versions are compared with
it directly: the same engine States, the same numpy batch callback, bit-equal
features, masks, visit counts, priors, values and statistics across searches
with subtree reuse. Engine-like stand-ins built from oracle records cover the
State import path everywhere.
"""

import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF_INSTALL = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


@pytest.fixture(scope="module")
def engine():
    """The reference's compiled my_board_engine module, or skip."""
    if str(REF_INSTALL) not in sys.path:
        sys.path.append(str(REF_INSTALL))  # after this package, so kingdom_ai stays ours
    try:
        import my_board_engine
    except ImportError:
        pytest.skip("the reference's my_board_engine is not installed under baseline/_ref")
    return my_board_engine


def random_states(engine, n, seed, max_plies=60):
    rng = np.random.default_rng(seed)
    states = []
    for _ in range(n):
        s = engine.State()
        for _ in range(int(rng.integers(0, max_plies))):
            moves = s.legal_moves()
            if not moves or s.result.finished():
                break
            s.play(moves[int(rng.integers(len(moves)))])
        states.append(s)
    return states


def feature_callback(features, masks):
    """A deterministic row-wise evaluator on numpy arrays: positive weights on
    legal actions derived from the planes, a value in (-1, 1)."""
    n = features.shape[0]
    flat = features.reshape(n, -1).astype(np.float64)
    cells = flat[:, :81] - flat[:, 81:162] + 0.5 * flat[:, 162:243] + 0.25 * flat[:, 729:810]
    weights = np.concatenate([1.0 + np.abs(np.sin(3.0 * cells + np.arange(81))), np.full((n, 1), 0.5)], axis=1)
    policy = np.where(masks, weights, 0.0)
    values = np.tanh(flat.sum(axis=1) / 97.0 - 1.0)
    return policy, values


def test_encode_puct_batch_equals_the_reference_binding(engine):
    from kingdom_ai import encode_puct_batch

    states = random_states(engine, 300, 1) + [engine.State()]
    ref_f, ref_m = engine.encode_puct_batch(states)
    got_f, got_m = encode_puct_batch(states)
    assert got_f.dtype == np.float32 and got_m.dtype == np.bool_
    assert np.array_equal(got_f, ref_f) and np.array_equal(got_m, ref_m)
    empty_f, empty_m = encode_puct_batch([])
    assert empty_f.shape == (0, 10, 9, 9) and empty_m.shape == (0, 82)


def test_from_engine_imports_reference_states_exactly(engine, oracle):
    """Records imported from engine States replay the same positions in the oracle."""
    from kingdom_ai.gpu_rules import GpuStateBatch

    rng = np.random.default_rng(5)
    states, recs = [], []
    for _ in range(64):
        s, rec = engine.State(), oracle.initial(1)
        for _ in range(int(rng.integers(0, 80))):
            if s.result.finished():
                break
            moves = s.legal_moves()
            m = moves[int(rng.integers(len(moves)))]
            a = 81 if m.is_pass() else m.point.row * 9 + m.point.col
            assert s.play(m).accepted()
            rec, ok = oracle.play(rec, [a])
            assert ok[0]
        states.append(s)
        recs.append(rec)
    got = GpuStateBatch.from_engine(states).states.cpu().numpy()
    assert np.array_equal(got, np.concatenate(recs))


def test_batched_search_equals_the_reference_searcher(engine):
    """Search, advance (subtree reuse) and search again, with the same numpy
    callback on both sides: every result field and statistic is equal."""
    from kingdom_ai import BatchedPUCT, PUCTOptions

    for sims, leaf, reuse in ((64, 8, True), (48, 1, False), (96, 16, True)):
        ours = BatchedPUCT(PUCTOptions(simulations=sims, c_puct=1.5), leaf, reuse)
        ref = engine.BatchedPUCT(engine.PUCTOptions(simulations=sims, c_puct=1.5), leaf, reuse)
        assert (ours.leaf_batch_size, ours.reuse_tree) == (ref.leaf_batch_size, ref.reuse_tree)
        state = engine.State()
        for ply in range(6):
            a = ours.search(state, feature_callback)
            b = ref.search(state, feature_callback)
            assert (a.simulations, a.nodes, a.network_evaluations) == (b.simulations, b.nodes,
                                                                        b.network_evaluations), ply
            assert a.root_value == b.root_value and a.best_value == b.best_value
            bm = b.best_move
            assert a.best_move == (81 if bm.is_pass() else bm.point.row * 9 + bm.point.col)
            assert len(a.moves) == len(b.moves)
            for x, y in zip(a.moves, b.moves):
                ya = 81 if y.move.is_pass() else y.move.point.row * 9 + y.move.point.col
                assert (x.move, x.visits, x.prior, x.value) == (ya, y.visits, y.prior, y.value)
            assert ours.stats == dict(ref.stats)
            assert state.play(bm).accepted()
            if state.result.finished():
                break
            # advance takes the engine Move as the reference's does
            assert ours.advance(bm) == ref.advance(bm)


def test_batched_search_rejects_malformed_callbacks_like_the_reference():
    from kingdom_ai import BatchedPUCT, PUCTOptions
    from kingdom_ai.gpu_rules import GpuStateBatch

    searcher = BatchedPUCT(PUCTOptions(simulations=8))
    start = GpuStateBatch.initial(1)
    with pytest.raises(ValueError, match=r"must return \(policy\[N,82\], values\[N\]\)"):
        searcher.search(start, lambda f, m: [np.ones((len(f), 82)), np.zeros(len(f))])
    with pytest.raises(ValueError, match="unexpected policy/value shapes"):
        searcher.search(start, lambda f, m: (np.ones((len(f), 81)), np.zeros(len(f))))
    with pytest.raises(ValueError, match="finite and in"):
        searcher.search(start, lambda f, m: (np.ones((len(f), 82)), np.full(len(f), 2.0)))
    # A callback that re-enters the searcher is refused, as in the binding.
    def reenter(f, m):
        searcher.clear()
        return np.ones((len(f), 82)), np.zeros(len(f))
    with pytest.raises(RuntimeError, match="Recursive access"):
        searcher.search(start, reenter)
    result = searcher.search(start, lambda f, m: (np.where(m, 1.0, 0.0), np.zeros(len(f))))
    assert result.simulations == 8 and result.best_move is not None


class _Enum(int):
    def __new__(cls, value, name):
        obj = int.__new__(cls, value)
        obj.name = name
        return obj


class _Cell(_Enum):
    pass


_Cell.Black, _Cell.White = _Cell(1, "Black"), _Cell(2, "White")


def _engine_like(rec):
    """A stand-in with the public attributes of my_board_engine.State."""
    reasons = {0: "None_", 1: "Capture", 2: "Suicide", 3: "TwoPasses"}
    stock = {1: int(rec[163]), 2: int(rec[164])}
    return SimpleNamespace(
        board=SimpleNamespace(cells=[int(c) for c in rec[:81]]), ownership=[int(o) for o in rec[81:162]],
        to_play=_Cell(int(rec[162]), "Black" if rec[162] == 1 else "White"),
        remaining_stones=lambda player: stock[int(player)], consecutive_passes=int(rec[165]),
        result=SimpleNamespace(reason=SimpleNamespace(name=reasons[int(rec[166])]), winner=int(rec[167]),
                               captured_stones=int(rec[168])),
        rules=SimpleNamespace(suicide_rule=SimpleNamespace(name="Loses"), allow_own_territory_moves=False,
                              allow_single_edge_territory=True, stones_per_player=41))


def test_engine_like_states_encode_as_the_oracle(oracle):
    from kingdom_ai import encode_puct_batch

    recs = oracle.gen_positions(77, 200)
    features, masks = encode_puct_batch([_engine_like(r) for r in recs])
    ef, em = oracle.encode(recs)
    assert np.array_equal(features, ef) and np.array_equal(masks, em)
    # Records are accepted directly too.
    f2, m2 = encode_puct_batch(torch.from_numpy(recs))
    assert np.array_equal(f2, ef) and np.array_equal(m2, em)
