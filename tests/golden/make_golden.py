"""Generate the golden fixtures in this folder from the reference C++ engine.

The reference engine (engine/ and mcts/ of the reference repository) is
compiled from its own sources by ``oracle/Makefile`` into
``oracle/_ref/libgkref.so`` and driven through ``oracle/ref_harness.cpp``.
Run from the repository root with the reference source root in GK_REFERENCE
(both the engine build and the GroupNorm fixture read it):

    GK_REFERENCE=<reference root> GK_REFERENCE_ROOT=<reference root> python tests/golden/make_golden.py

Fixtures
  rules_<scenario>.npz  board set-ups and action sequences of the reference's
                        tests/gpu_rules_test.py (captures, suicide, territory,
                        closed house, illegal moves, stock, two-pass
                        threshold, seeded complete games); per step the
                        expected wire records, accepted flags and encodings.
  playouts.npz          uniform-random complete playouts (PCG32 per game).
  positions.npz         generated mid-game positions with their encodings.
  puct.npz              root visits / priors / best move / root value of the
                        reference PUCT::search with the injected evaluator.
  tactics.npz           root positions of the reference's tactical-check tests
                        (tests/gpu_puct_test.py:196-295) and generated
                        positions, with each root action's outcome found by
                        playing it and then every legal reply in the
                        reference engine (+1 win, -1 loss or a winning reply
                        for the opponent, 0 otherwise).

  batched.npz           evaluation games driven by the reference
                        kingdom::BatchedPUCT (mcts/src/BatchedPUCT.cpp): one
                        searcher per colour with subtree reuse, both advanced
                        after every move as python/kingdom_ai/evaluation.py:
                        174-231 does, under six (simulations, leaf batch,
                        c_puct, evaluator, reuse) configurations; per search
                        the root, every result field and the statistics, the
                        move played, the advance results and an occasional
                        illegal advance.

  groupnorm.npz         the reference's own PolicyValueNet (GroupNorm
                        everywhere) at 32 x 2 and 64 x 1: seeded weights as
                        its state_dict, generated positions' features and
                        the module's fp32 logits and values.

Run with the argument ``tactics``, ``batched`` or ``groupnorm`` to write only that fixture.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle.oracle import Reference, RefState  # noqa: E402

BLACK, WHITE = 1, 2


def board(black=(), white=(), neutral=None):
    cells = np.zeros(81, dtype=np.int32)
    if neutral is not None:
        cells[neutral[0] * 9 + neutral[1]] = 3
    for points, colour in ((black, BLACK), (white, WHITE)):
        for r, c in points:
            assert cells[r * 9 + c] == 0
            cells[r * 9 + c] = colour
    return cells


def last_liberty_cells():
    cells = np.zeros(81, dtype=np.int32)
    for r in range(9):
        for c in range(9):
            if c < 4 or (c == 4 and r < 4):
                cells[r * 9 + c] = BLACK
            elif c > 4 or (c == 4 and r > 4):
                cells[r * 9 + c] = WHITE
    return cells


def square_enclosure(neutral=None, enemy=False):
    points = []
    for k in range(2, 7):
        points += [(2, k), (6, k)]
    for r in range(3, 6):
        points += [(r, 2), (r, 6)]
    return board(points, ((4, 4),) if enemy else (), neutral=neutral)


def trajectory(ref, states, action_rows, encode_every=1):
    """Apply rows of actions; record records/accepted/encodings per step."""
    records = [np.stack([s.record() for s in states])]
    accepted, features, masks, enc_steps = [], [], [], []

    def encode(step):
        f, m = zip(*(s.encode() for s in states))
        features.append(np.stack(f).reshape(len(states), 810))
        masks.append(np.stack(m))
        enc_steps.append(step)

    encode(0)
    for step, row in enumerate(action_rows, start=1):
        accepted.append([s.play(int(a)) for s, a in zip(states, row)])
        records.append(np.stack([s.record() for s in states]))
        if step % encode_every == 0 or step == len(action_rows):
            encode(step)
    return dict(records=np.stack(records).astype(np.int32), actions=np.asarray(action_rows, dtype=np.int64),
                accepted=np.asarray(accepted, dtype=np.uint8), features=np.stack(features).astype(np.float32),
                masks=np.stack(masks).astype(np.uint8), encode_steps=np.asarray(enc_steps, dtype=np.int32))


def transform(point, symmetry):
    """tests/gpu_puct_test.py:35-41: the 8 board symmetries."""
    row, col = point
    if symmetry >= 4:
        col = 8 - col
    for _ in range(symmetry % 4):
        row, col = col, 8 - row
    return row, col


def brute_outcomes(state):
    """+1 / -1 / 0 per root action by exhaustive one-ply lookahead in the reference engine."""
    rec = state.record()
    actor = int(rec[162])
    out = np.zeros(82, dtype=np.int8)
    for a in state.legal():
        nxt = state.copy()
        assert nxt.play(a)
        r = nxt.record()
        if r[166] != 0:
            out[a] = 1 if r[167] == actor else -1
            continue
        for b in nxt.legal():
            reply = nxt.copy()
            assert reply.play(b)
            rr = reply.record()
            if rr[166] != 0 and rr[167] == 3 - actor:
                out[a] = -1
                break
    return out


def tactics_fixture(ref):
    from_board = lambda cells, to_play: RefState.from_board(ref, cells, to_play)  # noqa: E731
    states, group, expected = [], [], []
    # :196-229 a low-prior capture in every symmetry, for both colours
    for actor in (BLACK, WHITE):
        for sym in range(8):
            own = tuple(transform(p, sym) for p in ((0, 1), (1, 0), (2, 1)))
            other = (transform((1, 1), sym),)
            cells = board(own, other) if actor == BLACK else board(other, own)
            states.append(from_board(cells, actor))
            group.append(0)
            r, c = transform((1, 2), sym)
            expected.append(r * 9 + c)
    # :231-259 the one safe reply after a reported opening, in every symmetry
    opening = [(4, 8), (5, 8), (2, 8), (6, 8), (2, 4), (4, 4), (6, 2), (4, 7), (3, 7), (5, 9), (4, 6)]
    for sym in range(8):
        s = RefState.initial(ref, 40)
        for row, col in opening:
            r, c = transform((row - 1, col - 1), sym)
            assert s.play(r * 9 + c)
        states.append(s)
        group.append(1)
        r, c = transform((4, 6), sym)
        expected.append(r * 9 + c)
    # :261-295 suicide, simultaneous capture, pass win, pass loss, no safe move
    suicide = from_board(board(((0, 1), (6, 7), (7, 6), (8, 7)),
                               ((0, 0), (0, 2), (1, 0), (1, 2), (2, 1), (7, 7))), BLACK)
    capture = from_board(board(((0, 6), (1, 6), (1, 8), (2, 7)), ((0, 7), (1, 7), (2, 8))), BLACK)
    white_pass_win = RefState.initial(ref, 40)
    assert white_pass_win.play(81)
    black_pass_loss = from_board(board(neutral=(4, 4)), WHITE)
    assert black_pass_loss.play(81)
    full = np.asarray([BLACK] * 41 + [WHITE] * 40, dtype=np.int32)
    forced_loss = from_board(full, WHITE)
    assert forced_loss.play(81)
    for s, e in ((suicide, -1), (capture, 8), (white_pass_win, 81), (black_pass_loss, -1), (forced_loss, 81)):
        states.append(s)
        group.append(2)
        expected.append(e)
    # generated mid-game positions
    for i in range(48):
        states.append(RefState.generated(ref, 23, i))
        group.append(3)
        expected.append(-1)
    roots = np.stack([s.record() for s in states]).astype(np.int32)
    outcomes = np.stack([brute_outcomes(s) for s in states])
    return dict(roots=roots, group=np.asarray(group, np.int32), expected=np.asarray(expected, np.int32),
                outcomes=outcomes)


BATCHED_CONFIGS = (  # simulations, leaf batch, c_puct, evaluator (0 hash, 1 uniform, 2 ramp), reuse
    (16, 4, 1.5, 2, 1),
    (32, 8, 1.5, 0, 1),
    (24, 1, 0.7, 0, 1),
    (48, 16, 2.5, 1, 1),
    (40, 8, 1.5, 0, 0),
    (64, 64, 1.5, 0, 1),
)
BATCHED_GAMES = 6
BATCHED_PLIES = 60


def batched_fixture(ref):
    from oracle.oracle import EVALUATORS
    kinds = {v: k for k, v in EVALUATORS.items()}
    rows = {k: [] for k in ("cfg", "game", "ply", "root", "visits", "priors", "move_values", "legal", "info",
                            "values", "stats", "move", "advanced", "bad_action", "bad_advanced", "stats_after")}
    for ci, (sims, leaf, c, kind, reuse) in enumerate(BATCHED_CONFIGS):
        for g in range(BATCHED_GAMES):
            rng = np.random.default_rng(1000 * ci + g)
            searchers = [ref.batched(sims, c, leaf, bool(reuse), kinds[kind]) for _ in range(2)]
            state = RefState.initial(ref, 40) if g % 2 == 0 else RefState.generated(ref, 31, 10 * ci + g)
            for ply in range(BATCHED_PLIES):
                root = state.record()
                if root[166] != 0:
                    break
                who = 0 if root[162] == BLACK else 1
                r = searchers[who].search(state)
                stats = searchers[who].stats
                legal = np.flatnonzero(r["legal"])
                move = r["best"] if rng.random() < 0.7 else int(rng.choice(legal))
                assert state.play(move)
                advanced = [searchers[k].advance(move) for k in range(2)]
                bad, bad_adv = -100, [False, False]
                if rng.random() < 0.15:
                    bad = int(rng.choice([-1, 82, 90, 40]))
                    bad_adv = [searchers[k].advance(bad) for k in range(2)]
                after = [searchers[k].stats for k in range(2)]
                rows["cfg"].append(ci)
                rows["game"].append(g)
                rows["ply"].append(ply)
                rows["root"].append(root)
                for key in ("visits", "priors", "move_values", "legal"):
                    rows[key].append(r[key])
                rows["info"].append([r["best"], r["simulations"], r["nodes"], r["evaluations"]])
                rows["values"].append([r["root_value"], r["best_value"]])
                rows["stats"].append(list(stats.values()))
                rows["move"].append(move)
                rows["advanced"].append(advanced)
                rows["bad_action"].append(bad)
                rows["bad_advanced"].append(bad_adv)
                rows["stats_after"].append([list(a.values()) for a in after])
    out = {k: np.asarray(v) for k, v in rows.items()}
    out["root"] = out["root"].astype(np.int32)
    out["legal"] = out["legal"].astype(np.uint8)
    out["visits"] = out["visits"].astype(np.int32)
    for key in ("cfg", "game", "ply", "move", "bad_action"):
        out[key] = out[key].astype(np.int32)
    for key in ("info", "stats", "stats_after"):
        out[key] = out[key].astype(np.int64)
    out["advanced"] = out["advanced"].astype(np.uint8)
    out["bad_advanced"] = out["bad_advanced"].astype(np.uint8)
    out["configs"] = np.asarray(BATCHED_CONFIGS, dtype=np.float64)
    return out


def reference_model_module():
    """The reference's python/kingdom_ai/model.py, loaded on its own: its
    package imports the compiled engine, so the one module it needs
    (encoding's ACTION_SIZE, BOARD_SIZE, INPUT_CHANNELS) is stood in for."""
    import importlib.util
    import types
    ref = Path(os.environ["GK_REFERENCE"])  # the reference source root (required)
    package = types.ModuleType("refkingdom")
    package.__path__ = []
    encoding = types.ModuleType("refkingdom.encoding")
    encoding.ACTION_SIZE, encoding.BOARD_SIZE, encoding.INPUT_CHANNELS = 82, 9, 10
    sys.modules["refkingdom"], sys.modules["refkingdom.encoding"] = package, encoding
    spec = importlib.util.spec_from_file_location("refkingdom.model", ref / "python/kingdom_ai/model.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def groupnorm_fixture(ref):
    """The reference's PolicyValueNet (GroupNorm) at its default 32 x 2 and at
    64 x 1: seeded weights as saved by state_dict, schema-1 features of
    generated positions, and the reference module's fp32 outputs."""
    import torch
    model_module = reference_model_module()
    features, _ = ref.encode_positions(57, 96)
    out = {"features": features.astype(np.float32)}
    for tag, (channels, blocks) in (("c32", (32, 2)), ("c64", (64, 1))):
        torch.manual_seed(1000 + channels)
        net = model_module.PolicyValueNet(channels, blocks)
        with torch.no_grad():
            for name, tensor in net.named_parameters():
                if name.endswith("weight") and tensor.dim() == 1:  # GroupNorm affine
                    tensor.copy_(1.0 + 0.1 * torch.randn_like(tensor))
                elif name.endswith("bias"):
                    tensor.copy_(0.1 * torch.randn_like(tensor))
            logits, values = net.eval()(torch.from_numpy(out["features"]))
        for name, tensor in net.state_dict().items():
            out[f"{tag}/{name}"] = tensor.numpy()
        out[f"{tag}/logits"], out[f"{tag}/values"] = logits.numpy(), values.numpy()
    return out


def save(name, data):
    np.savez_compressed(HERE / name, **data)
    print(name, {k: v.shape for k, v in data.items()})


def main():
    ref = Reference()
    if len(sys.argv) > 1 and sys.argv[1] == "tactics":
        save("tactics.npz", tactics_fixture(ref))
        return
    if len(sys.argv) > 1 and sys.argv[1] == "groupnorm":
        save("groupnorm.npz", groupnorm_fixture(ref))
        return
    if len(sys.argv) > 1 and sys.argv[1] == "batched":
        save("batched.npz", batched_fixture(ref))
        return
    from_board = lambda cells, to_play: RefState.from_board(ref, cells, to_play)  # noqa: E731

    # tests/gpu_rules_test.py:137-148 (initial variants)
    for name, neutral in (("initial_center", 40), ("initial_corner", 8), ("initial_none", -1)):
        states = [RefState.initial(ref, neutral) for _ in range(3)]
        save(f"rules_{name}.npz", trajectory(ref, states, [[0, 1, 2]]))

    # tests/gpu_rules_test.py:150-169 (captures, simultaneous surround, neutral wall)
    states = [
        from_board(board(((1, 2), (2, 1), (3, 2)), ((2, 2),)), BLACK),
        from_board(board(((1, 2), (1, 3), (2, 1), (3, 2), (3, 3)), ((2, 2), (2, 3))), BLACK),
        from_board(board(((0, 6), (1, 6), (1, 8), (2, 7)), ((0, 7), (1, 7), (2, 8))), BLACK),
        from_board(board(((3, 3), (4, 2)), ((4, 3),), (4, 4)), BLACK),
        from_board(board(((2, 2),), ((1, 2), (2, 1), (3, 2))), WHITE),
        from_board(last_liberty_cells(), BLACK),
        from_board(last_liberty_cells(), WHITE),
    ]
    save("rules_captures.npz", trajectory(ref, states, [[21, 22, 8, 48, 21, 40, 40], [81] * 7]))

    # :171-177 remaining liberty
    states = [from_board(board(((1, 2), (2, 1), (3, 2), (3, 3)), ((2, 2), (2, 3))), BLACK)]
    save("rules_liberty.npz", trajectory(ref, states, [[12]]))

    # :179-191 suicide loses for both players
    b, w = ((0, 1),), ((0, 0), (0, 2), (1, 0), (1, 2), (2, 1))
    states = [from_board(board(b, w), BLACK), from_board(board(w, b), WHITE)]
    save("rules_suicide.npz", trajectory(ref, states, [[10, 10]]))

    # :193-215 territory edges, neutral walls, enemy exclusion
    three_edges = board(tuple((r, 2) for r in range(9)), ((0, 3),))
    boards = [
        board(((1, 2), (2, 1), (2, 3), (3, 2))),
        board(((0, 3), (1, 2), (1, 4), (2, 1), (2, 4), (3, 1), (3, 4), (4, 2), (4, 3), (4, 4))),
        board(((0, 2), (0, 5), (1, 3), (1, 4))),
        board(((0, 2), (1, 1), (2, 0))),
        three_edges,
        board(((4, 4),)),
        square_enclosure(enemy=True),
        square_enclosure((4, 4)),
        board(((3, 5), (4, 6), (5, 5)), neutral=(4, 4)),
    ]
    states = [from_board(cells, BLACK) for cells in boards]
    data = trajectory(ref, states, [[81] * 9, [81] * 9])
    data["scores"] = np.asarray([s.score() for s in [from_board(c, BLACK) for c in boards]], dtype=np.int32)
    save("rules_territory.npz", data)

    # :217-226 closed house persists and forbids both players
    states = [from_board(board(((1, 2), (2, 1), (2, 3))), BLACK)]
    save("rules_house.npz", trajectory(ref, states, [[29], [80], [20], [81], [20]]))

    # :228-238 illegal placements preserve actor, passes, stock and ownership
    states = []
    for _ in range(4):
        s = RefState.initial(ref, 40)
        assert s.play(0) and s.play(81)
        states.append(s)
    save("rules_illegal.npz", trajectory(ref, states, [[0, 40, -1, 82], [1, 2, 3, 4]]))

    # :240-250 the 41-stone stock cannot be exceeded
    states = [from_board(board(tuple(divmod(a, 9) for a in range(41))), BLACK)]
    save("rules_stock.npz", trajectory(ref, states, [[80], [81]]))

    # :252-264 two-pass threshold needs exactly three more house cells
    boards = [board(((0, 2), (1, 1), (2, 0))), board(((0, 2), (0, 5), (1, 3), (1, 4))), board(neutral=(4, 4))]
    states = [from_board(cells, BLACK) for cells in boards]
    save("rules_threshold.npz", trajectory(ref, states, [[81] * 3, [81] * 3]))

    # :277-292 seeded complete games from several neutral variants
    variants = [40, -1, 8, 40, -1, 72, 40, -1]
    states = [RefState.initial(ref, v) for v in variants]
    rng = np.random.default_rng(6800)
    probe = [RefState.initial(ref, v) for v in variants]
    rows = []
    for _ in range(170):
        if all(p.record()[166] != 0 for p in probe):
            break
        row = []
        for p in probe:
            legal = p.legal()
            a = 81 if not legal else int(legal[rng.integers(len(legal))])
            row.append(a)
            p.play(a)
        rows.append(row)
    save("rules_games.npz", trajectory(ref, states, rows, encode_every=7))

    # Uniform-random playouts (PCG32 stream per game), reference legal_moves().
    boards_out, infos = ref.random_playouts(2024, 256, neutral=40, fast=False, threads=8)
    save("playouts.npz", dict(seed=np.asarray([2024]), boards=boards_out, infos=infos))

    # Generated mid-game positions and their reference encodings.
    recs = ref.gen_positions(11, 256, threads=8)
    feats, masks = ref.encode_positions(11, 256, threads=8)
    save("positions.npz", dict(seed=np.asarray([11]), records=recs, features=feats.reshape(256, 810),
                               masks=masks.astype(np.uint8)))

    # Reference PUCT with the injected evaluator.
    n, sims = 48, 160
    visits = np.zeros((n, 82), np.int32)
    priors = np.zeros((n, 82), np.float64)
    stats = np.zeros((n, 4), np.int32)
    values = np.zeros((n, 2), np.float64)
    roots = np.zeros((n, 170), np.int32)
    for i in range(n):
        s = RefState.generated(ref, 5, i)
        roots[i] = s.record()
        r = s.puct(sims)
        visits[i], priors[i] = r["visits"], r["priors"]
        stats[i] = (r["best"], r["simulations"], r["nodes"], r["evaluations"])
        values[i] = (r["root_value"], r["best_value"])
    save("puct.npz", dict(seed=np.asarray([5]), simulations=np.asarray([sims]), roots=roots, visits=visits,
                          priors=priors, stats=stats, values=values))
    save("tactics.npz", tactics_fixture(ref))


if __name__ == "__main__":
    main()
