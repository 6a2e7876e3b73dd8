"""Pin the CPU oracle: golden vectors of the reference engine and its tests' known answers."""

import numpy as np
import pytest

RULE_FIXTURES = ["initial_center", "initial_corner", "initial_none", "captures", "liberty", "suicide",
                 "territory", "house", "illegal", "stock", "threshold", "games"]


def replay_oracle(oracle, data):
    """Replay a golden trajectory through the oracle; compare every step."""
    recs = data["records"][0].copy()
    enc = {int(s): i for i, s in enumerate(data["encode_steps"])}
    f, m = oracle.encode(recs)
    assert np.array_equal(f.reshape(len(recs), 810), data["features"][enc[0]])
    assert np.array_equal(m, data["masks"][enc[0]].astype(bool))
    for step, row in enumerate(data["actions"], start=1):
        actions = np.where((row >= 0) & (row < 82), row, -1).astype(np.int32)
        recs, accepted = oracle.play(recs, actions)
        assert np.array_equal(accepted, data["accepted"][step - 1]), f"accepted differs at step {step}"
        assert np.array_equal(recs, data["records"][step]), f"record differs at step {step}"
        if step in enc:
            f, m = oracle.encode(recs)
            assert np.array_equal(f.reshape(len(recs), 810), data["features"][enc[step]])
            assert np.array_equal(m, data["masks"][enc[step]].astype(bool))


@pytest.mark.parametrize("name", RULE_FIXTURES)
def test_oracle_rules_match_reference_fixtures(oracle, golden, name):
    replay_oracle(oracle, golden(f"rules_{name}.npz"))


def test_known_answers_of_reference_rule_tests(golden):
    # tests/gpu_rules_test.py:166-167 - capture reasons and captured counts.
    cap = golden("rules_captures.npz")
    assert cap["records"][1][:, 166].tolist() == [1] * 7
    assert cap["records"][1][:, 168].tolist() == [1, 2, 2, 1, 1, 40, 40]
    assert cap["accepted"][1].tolist() == [0] * 7
    # :206 - black territory of the nine fixture boards; :211-215 winners after two passes.
    terr = golden("rules_territory.npz")
    assert terr["scores"][:, 0].tolist() == [1, 5, 2, 3, 18, 0, 0, 8, 1]
    assert terr["records"][2][:, 167].tolist() == [2, 1, 2, 1, 1, 2, 2, 1, 2]
    # :263-264 - the 3-point black margin.
    thr = golden("rules_threshold.npz")
    assert thr["records"][2][:, 166].tolist() == [3, 3, 3]
    assert thr["records"][2][:, 167].tolist() == [1, 2, 2]
    # :179-191 - suicide is legal and loses for both colours.
    sui = golden("rules_suicide.npz")
    assert sui["accepted"][0].tolist() == [1, 1]
    assert sui["records"][1][:, 166].tolist() == [2, 2]
    # :217-226 - closed house forbids both players.
    house = golden("rules_house.npz")
    assert house["accepted"][:, 0].tolist() == [1, 1, 0, 1, 0]
    assert house["records"][1][0, 81 + 20] == 1
    # :240-250 - no stones left: only pass.
    stock = golden("rules_stock.npz")
    assert stock["masks"][0][0].sum() == 1 and stock["masks"][0][0][81] == 1


def test_oracle_playouts_match_reference(oracle, golden):
    g = golden("playouts.npz")
    boards, infos = oracle.random_playouts(int(g["seed"][0]), len(g["boards"]))
    assert np.array_equal(boards, g["boards"])
    assert np.array_equal(infos, g["infos"])


def test_oracle_positions_and_encoder_match_reference(oracle, golden):
    g = golden("positions.npz")
    recs = oracle.gen_positions(int(g["seed"][0]), len(g["records"]))
    assert np.array_equal(recs, g["records"])
    assert (recs[:, 166] == 0).all()
    f, m = oracle.encode(recs)
    assert np.array_equal(f.reshape(len(recs), 810), g["features"])
    assert np.array_equal(m, g["masks"].astype(bool))


def test_oracle_puct_matches_reference(oracle, golden):
    g = golden("puct.npz")
    sims = int(g["simulations"][0])
    for i, root in enumerate(g["roots"]):
        r = oracle.puct(root, sims)
        assert np.array_equal(r["visits"], g["visits"][i])
        assert np.array_equal(r["priors"], g["priors"][i])
        assert (r["best"], r["simulations"], r["nodes"], r["evaluations"]) == tuple(g["stats"][i])
        assert r["root_value"] == g["values"][i][0] and r["best_value"] == g["values"][i][1]


def test_oracle_matches_reference_engine_directly(oracle, reference):
    """Where the reference is built here, compare on fresh seeds as well."""
    b1, i1 = oracle.random_playouts(99, 300)
    b2, i2 = reference.random_playouts(99, 300, fast=True, threads=4)
    assert np.array_equal(b1, b2) and np.array_equal(i1, i2)
    assert np.array_equal(oracle.gen_positions(77, 200), reference.gen_positions(77, 200, threads=4))
    recs = oracle.gen_positions(3, 8)
    v, best, _ = oracle.puct_batch(recs, 120, threads=4)
    v2, best2 = reference.puct_positions(3, 8, 120, threads=4)
    assert np.array_equal(v, v2) and np.array_equal(best, best2)


def test_injected_evaluator_is_a_pure_function(oracle, golden):
    recs = golden("positions.npz")["records"][:4]
    for rec in recs:
        w1, v1 = oracle.evaluate(rec)
        w2, v2 = oracle.evaluate(rec.copy())
        assert np.array_equal(w1, w2) and v1 == v2
        assert (w1 > 0).all() and np.isfinite(w1).all() and -1.0 <= v1 < 1.0
    # Approximately standard-normal logits: log-weights have mean ~0, sd ~1.
    logs = np.log(np.concatenate([oracle.evaluate(r)[0] for r in golden("positions.npz")["records"]]))
    assert abs(logs.mean()) < 0.1 and abs(logs.std() - 1.0) < 0.1


def test_oracle_root_tactics_match_reference_engine_lookahead(oracle, golden):
    """Root tactical checks (gpu_puct.py:84-161) against the reference engine:
    each root action played, then every legal reply, in the compiled
    reference (tests/golden/tactics.npz)."""
    g = golden("tactics.npz")
    for rec, expected in zip(g["roots"], g["outcomes"]):
        outcome, allow = oracle.root_tactics(rec)
        legal = np.asarray([oracle.lib.gko_legal(rec, a) for a in range(82)], dtype=bool)
        assert np.array_equal(outcome[legal], expected[legal])
        winning, safe = (expected[legal] > 0).any(), (expected[legal] >= 0).any()
        keep = expected > 0 if winning else expected >= 0 if safe else np.ones(82, bool)
        assert np.array_equal(allow, legal & keep)


def test_oracle_tactical_search_known_answers(oracle, golden):
    """The expectations of the reference's tactical-check tests
    (tests/gpu_puct_test.py:196-295) with the oracle's search."""
    g = golden("tactics.npz")
    for rec, group, expected in zip(g["roots"], g["group"], g["expected"]):
        if group > 1:
            continue
        r = oracle.puct(rec, 8, uniform=True, tactics=True)
        assert r["best"] == expected and r["visits"][expected] == 8
    cases = [i for i, grp in enumerate(g["group"]) if grp == 2]
    suicide, capture, pass_win, pass_loss, forced = (g["roots"][i] for i in cases)
    r = oracle.puct(suicide, 8, uniform=True, tactics=True)
    assert r["visits"][10] == 0 and r["priors"][10] == 0.0
    r = oracle.puct(capture, 8, uniform=True, tactics=True)
    assert r["best"] == 8 and r["best_value"] == 1.0
    r = oracle.puct(pass_win, 8, uniform=True, tactics=True)
    assert r["best"] == 81 and r["best_value"] == 1.0
    assert oracle.puct(pass_loss, 8, uniform=True, tactics=True)["visits"][81] == 0
    r = oracle.puct(forced, 8, uniform=True, tactics=True)
    assert r["best"] == 81 and r["best_value"] == -1.0


def replay_sample(oracle, index=0, white=False):
    """The valid replay row of the reference's replay tests (tests/replay_test.py:16-25)."""
    rec = oracle.initial(1, 40)
    if white:
        oracle.play(rec, [81])
    features, masks = oracle.encode(rec)
    policy = np.zeros((1, 82), dtype=np.float32)
    policy[0, index % 40] = 1.0
    value = np.asarray([1.0 if index % 2 == 0 else -1.0], dtype=np.float32)
    return features, masks, policy, value, np.asarray([2 if white else 1], dtype=np.int8)


def replay_corruptions(oracle):
    """(message, row) pairs of the reference's rejected contents (tests/replay_test.py:237-274)."""
    f, m, p, v, t = replay_sample(oracle)
    cases = []

    def case(message, **changes):
        row = dict(features=f.copy(), legal_mask=m.copy(), policy=p.copy(), value=v.copy(), to_play=t.copy())
        for name, (index, value) in changes.items():
            row[name][(0, *index) if isinstance(index, tuple) else (0, index)] = value
        cases.append((message, row))

    case("Replay features and policies must be finite", features=((0, 0, 0), np.nan))
    case("Replay features must lie between zero and one", features=((6, 0, 0), -1.0))
    case("Binary observation planes must contain only zero or one", features=((0, 0, 0), 0.5))
    case("Scalar observation planes must be constant", features=((6, 0, 0), 0.7))
    case("Replay observations must be taken before game termination",
         features=((8, slice(None), slice(None)), 1.0))
    case("Replay policies must assign non-negative mass to legal actions only", policy=(0, -1.0))
    case("Replay policies must assign non-negative mass to legal actions only", policy=(40, 1.0))
    case("Replay features and policies must be finite", policy=(0, np.inf))
    case("Each replay policy must sum to one", policy=(slice(None), 0.0))
    case("Nonterminal replay observations must allow passing", legal_mask=(slice(None), False))
    case("Observation legal placements do not match the action mask", legal_mask=(0, False))
    case("Nonterminal replay observations must allow passing", legal_mask=(81, False))
    case("Completed-game replay values must be -1 or +1", value=((), np.nan))
    case("Completed-game replay values must be -1 or +1", value=((), 0.0))
    case("Replay actors must be Black or White", to_play=((), 3))
    case("Observation player perspective does not match its actor", to_play=((), 2))
    return cases


def test_replay_checks_restatement_rejects_reference_cases(oracle):
    from oracle.oracle import replay_violation
    for index, white in ((0, False), (3, False), (5, True)):
        assert replay_violation(*replay_sample(oracle, index, white)) is None
    for message, row in replay_corruptions(oracle):
        assert replay_violation(**row) == message


# ---- BatchedPUCT (mcts/src/BatchedPUCT.cpp) ------------------------------------------

BATCHED_FIELDS = ("visits", "priors", "move_values", "legal")
BATCHED_EVALUATORS = ("hash", "uniform", "ramp")


def batched_games(golden):
    """The golden evaluation games grouped by configuration: yields
    (config index, (simulations, leaf, c_puct, evaluator, reuse), [row indices of each game])."""
    g = golden("batched.npz")
    for ci, (sims, leaf, c, kind, reuse) in enumerate(g["configs"]):
        games = [np.flatnonzero((g["cfg"] == ci) & (g["game"] == game)) for game in np.unique(g["game"])]
        yield g, ci, (int(sims), int(leaf), float(c), BATCHED_EVALUATORS[int(kind)], bool(reuse)), games


def check_batched_row(g, i, result, stats):
    """One search of a golden game against the reference's outputs."""
    assert np.array_equal(np.asarray(result["visits"]), g["visits"][i])
    assert np.array_equal(np.asarray(result["priors"]), g["priors"][i])
    assert np.array_equal(np.asarray(result["move_values"]), g["move_values"][i])
    assert np.array_equal(np.asarray(result["legal"]).astype(np.uint8), g["legal"][i])
    info = [result["best"], result["simulations"], result["nodes"], result["evaluations"]]
    assert info == g["info"][i].tolist()
    assert [result["root_value"], result["best_value"]] == g["values"][i].tolist()
    assert list(stats) == g["stats"][i].tolist()


def test_oracle_batched_search_replays_reference_games(oracle, golden):
    """The restated BatchedPUCT reproduces, bit for bit, evaluation games
    played by the reference's own searcher (tests/golden/batched.npz)."""
    searches = 0
    for g, ci, (sims, leaf, c, kind, reuse), games in batched_games(golden):
        for rows in games:
            searchers = [oracle.batched(sims, c, leaf, reuse, kind) for _ in range(2)]
            for i in rows:
                root = g["root"][i]
                who = 0 if root[162] == 1 else 1
                result = searchers[who].search(root)
                check_batched_row(g, i, result, searchers[who].stats.values())
                searches += 1
                move = int(g["move"][i])
                assert [s.advance(move) for s in searchers] == g["advanced"][i].astype(bool).tolist()
                if g["bad_action"][i] != -100:
                    bad = int(g["bad_action"][i])
                    assert [s.advance(bad) for s in searchers] == g["bad_advanced"][i].astype(bool).tolist()
                assert [list(s.stats.values()) for s in searchers] == g["stats_after"][i].tolist()
    assert searches == len(g["cfg"])


def test_oracle_batched_search_matches_reference_engine_directly(oracle, reference):
    """Fresh games against the reference searcher, where it is built here."""
    from oracle.oracle import RefState
    rng = np.random.default_rng(5)
    for sims, leaf, c, kind in ((20, 5, 1.2, "hash"), (36, 12, 0.6, "hash"), (12, 2, 3.0, "ramp")):
        ours = [oracle.batched(sims, c, leaf, True, kind) for _ in range(2)]
        theirs = [reference.batched(sims, c, leaf, True, kind) for _ in range(2)]
        state = RefState.generated(reference, 91, sims)
        for _ in range(30):
            rec = state.record()
            if rec[166] != 0:
                break
            who = 0 if rec[162] == 1 else 1
            a, b = ours[who].search(rec), theirs[who].search(state)
            for key in BATCHED_FIELDS:
                assert np.array_equal(a[key], b[key])
            assert {k: a[k] for k in a if k not in BATCHED_FIELDS} == {k: b[k] for k in b if k not in BATCHED_FIELDS}
            assert ours[who].stats == theirs[who].stats
            move = a["best"] if rng.random() < 0.6 else int(rng.choice(np.flatnonzero(a["legal"])))
            assert state.play(move)
            assert [s.advance(move) for s in ours] == [s.advance(move) for s in theirs]


def split_board_record(oracle, actor):
    """tests/batched_puct_test.cpp:171-179: Black holds columns 0-3 and the top
    of column 4, White the rest; (4, 4) is the only empty cell."""
    rec = oracle.initial(1, -1)[0]
    for row in range(9):
        for col in range(9):
            if col < 4 or (col == 4 and row < 4):
                rec[row * 9 + col] = 1
            elif col > 4 or (col == 4 and row > 4):
                rec[row * 9 + col] = 2
    rec[162] = actor
    return rec


def test_oracle_batched_search_known_answers(oracle):
    """The assertions of the reference's tests/batched_puct_test.cpp on the
    restatement, with the tests' own fixed evaluator ("ramp")."""
    # :89-115 budgets, batch sizes and statistics
    for count in (1, 7, 19, 301):
        s = oracle.batched(count, 1.5, 8, False, "ramp")
        r = s.search(oracle.initial(1)[0])
        st = s.stats
        assert r["simulations"] == count and r["visits"].sum() == count
        assert r["evaluations"] == st["network_evaluations"] <= count + 1
        assert r["nodes"] <= count + 1 and st["max_observed_batch_size"] <= 8
        if count >= 8:
            assert st["max_observed_batch_size"] == 8
    # :117-150 subtree reuse and visits counted per search
    s = oracle.batched(64, 1.5, 8, True, "ramp")
    root = oracle.initial(1)[0]
    first = s.search(root)
    assert s.stats["reused_nodes"] == 0 and s.stats["inherited_visits"] == 0
    repeated = s.search(root)
    assert s.stats["reused_nodes"] == first["nodes"] and s.stats["inherited_visits"] == 64
    assert repeated["simulations"] == 64 and repeated["visits"].sum() == 64 and repeated["evaluations"] <= 64
    assert s.advance(repeated["best"])
    root, _ = oracle.play(root[None].copy(), [repeated["best"]])
    after = s.search(root[0])
    assert s.stats["reused_nodes"] > 0 and s.stats["inherited_visits"] > 0
    assert s.stats["advance_calls"] == 1 and s.stats["reuse_hits"] == 1
    assert after["visits"].sum() == 64 and after["nodes"] < repeated["nodes"] + 65
    assert not s.advance(40) and not s.advance(-1)
    again = s.search(root[0])
    assert s.stats["reused_nodes"] == after["nodes"] and again["visits"].sum() == 64
    assert s.stats["advance_calls"] == 3 and s.stats["reuse_hits"] == 1
    s.clear()
    assert s.search(root[0])["evaluations"] > 0 and s.stats["reused_nodes"] == 0
    # :152-169 a state that differs in any field starts a new tree
    s = oracle.batched(16, 1.5, 4, True, "ramp")
    start = oracle.initial(1)[0]
    s.search(start)
    passed, _ = oracle.play(start[None].copy(), [81])
    assert s.search(passed[0])["simulations"] == 16 and s.stats["reused_nodes"] == 0
    setup = passed[0].copy()
    setup[165] = 0
    assert s.search(setup)["simulations"] == 16 and s.stats["reused_nodes"] == 0
    assert s.search(oracle.initial(1, -1)[0])["simulations"] == 16 and s.stats["reused_nodes"] == 0
    # :171-209 capture values without the network, terminal roots
    for actor in (1, 2):
        s = oracle.batched(32, 1.5, 8, True, "ramp")
        rec = split_board_record(oracle, actor)
        r = s.search(rec)
        assert r["best"] == 40 and r["best_value"] == 1.0 and r["visits"].sum() == 32
        assert r["evaluations"] == 1 and s.stats["inference_batches"] == 1
        assert s.advance(40)
        done, _ = oracle.play(rec[None].copy(), [40])
        assert done[0][166] == 1  # capture
        t = s.search(done[0])
        assert t["root_value"] == -1.0 and s.stats["network_evaluations"] == 0 and t["best"] == -1
    two = oracle.initial(1)
    oracle.play(two, [81])
    oracle.play(two, [81])
    t = oracle.batched(8, 1.5, 8, True, "ramp").search(two[0])
    assert t["best"] == -1 and t["simulations"] == 0 and not t["legal"].any() and t["root_value"] == -1.0
    # :262-280 a whole game with two searchers that advance after every move
    rec = oracle.initial(1)[0]
    black, white = oracle.batched(16, 1.5, 4, True, "ramp"), oracle.batched(16, 1.5, 4, True, "ramp")
    plies = 0
    while rec[166] == 0 and plies < 164:
        r = (black if rec[162] == 1 else white).search(rec)
        assert r["visits"].sum() == 16
        nxt, ok = oracle.play(rec[None].copy(), [r["best"]])
        assert ok[0]
        rec = nxt[0]
        black.advance(r["best"])
        white.advance(r["best"])
        plies += 1
    assert rec[166] != 0
    # :57-87 one leaf per batch without reuse is the legacy search
    start, _ = oracle.play(oracle.initial(1), [0])
    start, _ = oracle.play(start, [81])
    for count in (1, 31, 300):
        legacy = oracle.puct(start[0], count)
        r = oracle.batched(count, 1.5, 1, False, "hash").search(start[0])
        assert np.array_equal(r["visits"], legacy["visits"]) and np.array_equal(r["priors"], legacy["priors"])
        assert (r["best"], r["nodes"], r["evaluations"]) == (legacy["best"], legacy["nodes"], legacy["evaluations"])
        assert (r["root_value"], r["best_value"]) == (legacy["root_value"], legacy["best_value"])


def test_oracle_selfplay_games_follow_the_reference_engine(oracle, reference):
    """The self-play restatement against the reference itself: every game
    replays in kingdom::State, every ply's visit-share target is the reference
    PUCT::search's visits over its simulations (the same injected evaluator),
    every move played after the sampled opening is the reference's best move,
    and the final position is the reference's."""
    import numpy as np

    from oracle.oracle import RefState

    sims = 24
    plies, actions, policy, finals = oracle.selfplay_hash(3, 6, sims, temperature_moves=4)
    for g in range(6):
        state = RefState.initial(reference)
        assert plies[g] > 0
        for ply in range(plies[g]):
            r = state.puct(sims)
            assert np.array_equal(policy[g, ply], (r["visits"].astype(np.float32) / np.float32(sims))), (g, ply)
            if ply >= 4:
                assert actions[g, ply] == r["best"], (g, ply)
            assert state.play(int(actions[g, ply]))
        assert np.array_equal(state.record(), finals[g])
