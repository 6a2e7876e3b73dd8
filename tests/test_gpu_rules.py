"""CUDA rules, encoder, playouts and generator against the oracle and the golden fixtures.

Follows the reference's tests/gpu_rules_test.py: exact [N,170] records and
exact encodings (rtol=atol=0) after every transition.
"""

import numpy as np
import pytest
import torch

from test_oracle import RULE_FIXTURES

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kai():
    import kingdom_ai
    return kingdom_ai


def assert_encoding(batch, features_expected, masks_expected):
    features, masks = batch.encode()
    assert features.dtype == torch.float32 and masks.dtype == torch.bool
    assert tuple(features.shape) == (len(batch), 10, 9, 9) and tuple(masks.shape) == (len(batch), 82)
    torch.testing.assert_close(features.cpu().reshape(len(batch), 810), torch.from_numpy(features_expected),
                               rtol=0, atol=0)
    assert np.array_equal(masks.cpu().numpy(), masks_expected.astype(bool))


@pytest.mark.parametrize("name", RULE_FIXTURES)
def test_records_and_encodings_match_reference_fixtures(kai, golden, name):
    data = golden(f"rules_{name}.npz")
    batch = kai.GpuStateBatch.from_records(data["records"][0])
    enc = {int(s): i for i, s in enumerate(data["encode_steps"])}
    assert_encoding(batch, data["features"][enc[0]], data["masks"][enc[0]])
    for step, row in enumerate(data["actions"], start=1):
        accepted = batch.play(torch.tensor(row, dtype=torch.int64, device="cuda"))
        assert accepted.dtype == torch.bool
        assert accepted.cpu().numpy().astype(np.uint8).tolist() == data["accepted"][step - 1].tolist()
        assert np.array_equal(batch.states.cpu().numpy(), data["records"][step]), f"step {step}"
        if step in enc:
            assert_encoding(batch, data["features"][enc[step]], data["masks"][enc[step]])


def test_int32_and_int64_actions_agree_and_huge_values_are_rejected(kai, oracle):
    recs = oracle.initial(2)
    batch = kai.GpuStateBatch.from_records(recs)
    before = batch.states.clone()
    accepted = batch.play(torch.tensor([-(2**40), 2**40], device="cuda", dtype=torch.int64))
    assert accepted.cpu().tolist() == [False, False]
    torch.testing.assert_close(batch.states, before, rtol=0, atol=0)
    # 2**32 + 5 must not wrap to action 5.
    accepted = batch.play(torch.tensor([2**32 + 5, 5], device="cuda", dtype=torch.int64))
    assert accepted.cpu().tolist() == [False, True]


def test_initial_clone_and_neutral_variants(kai, oracle):
    for neutral, cell in (((4, 4), 40), ((0, 8), 8), (None, -1)):
        batch = kai.GpuStateBatch.initial(3, device="cuda", neutral=neutral)
        expected = oracle.initial(3, cell)
        assert np.array_equal(batch.states.cpu().numpy(), expected)
        copied = batch.clone()
        assert copied.states.data_ptr() != batch.states.data_ptr()
        unchanged = batch.states.clone()
        copied.play(torch.tensor([0, 1, 2], device="cuda", dtype=torch.int32))
        torch.testing.assert_close(batch.states, unchanged, rtol=0, atol=0)
        exp, _ = oracle.play(expected, [0, 1, 2])
        assert np.array_equal(copied.states.cpu().numpy(), exp)


def test_nondefault_stream_orders_import_encode_and_play(kai, oracle):
    recs = np.concatenate([oracle.initial(1, 40), oracle.initial(1, -1)])
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        batch = kai.GpuStateBatch.from_records(recs)
        f0, m0 = batch.encode()
        accepted = batch.play(torch.tensor([0, 80], device="cuda", dtype=torch.int32))
        after = batch.states.clone()
        f1, m1 = batch.encode()
    stream.synchronize()
    ef0, em0 = oracle.encode(recs)
    nxt, acc = oracle.play(recs.copy(), [0, 80])
    ef1, em1 = oracle.encode(nxt)
    assert accepted.cpu().tolist() == [True, True] and acc.tolist() == [1, 1]
    assert np.array_equal(f0.cpu().numpy(), ef0) and np.array_equal(m0.cpu().numpy(), em0)
    assert np.array_equal(after.cpu().numpy(), nxt)
    assert np.array_equal(f1.cpu().numpy(), ef1) and np.array_equal(m1.cpu().numpy(), em1)


def test_batched_transitions_are_independent_of_partitions(kai, golden):
    recs = golden("rules_captures.npz")["records"][0]
    actions = [21, 22, 8, 48, 21, 40, 40]
    batched = kai.GpuStateBatch.from_records(recs)
    batched.play(torch.tensor(actions, device="cuda", dtype=torch.int32))
    for i, a in enumerate(actions):
        single = kai.GpuStateBatch.from_records(recs[i:i + 1])
        single.play(torch.tensor([a], device="cuda", dtype=torch.int32))
        torch.testing.assert_close(single.states[0], batched.states[i], rtol=0, atol=0)


def test_invalid_inputs_are_rejected_before_launch(kai):
    with pytest.raises(TypeError):
        kai.GpuStateBatch(np.zeros((2, 170), dtype=np.int32))
    with pytest.raises(ValueError):
        kai.GpuStateBatch(torch.zeros((2, 169), dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError):
        kai.GpuStateBatch(torch.zeros((2, 170), dtype=torch.int64, device="cuda"))
    with pytest.raises(ValueError):
        kai.GpuStateBatch.initial(0)
    with pytest.raises(ValueError):
        kai.GpuStateBatch.initial(2, neutral=(9, 0))
    bad = np.zeros((1, 170), dtype=np.int32)
    bad[0, 162] = 7
    with pytest.raises(ValueError):
        kai.GpuStateBatch.from_records(bad)
    batch = kai.GpuStateBatch.initial(2)
    before = batch.states.clone()
    for actions in (torch.tensor([0], device="cuda", dtype=torch.int32),
                    torch.tensor([[0, 1]], device="cuda", dtype=torch.int32),
                    torch.tensor([0.0, 1.0], device="cuda")):
        with pytest.raises((TypeError, ValueError)):
            batch.play(actions)
    torch.testing.assert_close(batch.states, before, rtol=0, atol=0)


def random_trajectory(oracle, n, seed, plies=200):
    """Records and actions of `n` uniform-random games driven by the oracle."""
    rng = np.random.default_rng(seed)
    recs = oracle.initial(n, 40)
    steps = []
    for _ in range(plies):
        acts = np.zeros(n, dtype=np.int32)
        for i in range(n):
            legal = [a for a in range(82) if oracle.lib.gko_legal(recs[i], a)]
            acts[i] = rng.choice(legal) if legal else 81
        steps.append((recs.copy(), acts))
        recs, _ = oracle.play(recs, acts)
        if (recs[:, 166] != 0).all():
            break
    return steps


def test_packed_state_kernels_match_the_record_kernels(kai, oracle):
    from kingdom_ai.gpu_rules import bits_to_records, records_to_bits
    from kingdom_ai.gpu_puct import encode_packed
    from kingdom_ai import _native as native

    steps = random_trajectory(oracle, 64, 5)
    recs0 = torch.from_numpy(steps[0][0]).cuda()
    bits = records_to_bits(recs0)
    for recs, acts in steps:
        exp_f, exp_m = oracle.encode(recs)
        f, m = encode_packed(bits)
        assert np.array_equal(f.cpu().numpy(), exp_f) and np.array_equal(m.cpu().numpy(), exp_m)
        assert np.array_equal(bits_to_records(bits).cpu().numpy()[:, :169], recs[:, :169])
        a = torch.from_numpy(acts).cuda()
        accepted = torch.empty(len(acts), dtype=torch.bool, device="cuda")
        native.call("gk_play_bits", native.ptr(bits), native.ptr(a), 4, native.ptr(accepted), len(acts),
                    native.stream_of(bits.device))
        exp, exp_acc = oracle.play(recs.copy(), acts)
        assert np.array_equal(accepted.cpu().numpy(), exp_acc.astype(bool))
    assert np.array_equal(bits_to_records(bits).cpu().numpy()[:, :169], exp[:, :169])


def _playouts(seed, n, neutral=40):
    from kingdom_ai import _native as native
    boards = torch.empty((n, 81), dtype=torch.int8, device="cuda")
    infos = torch.empty((n, 5), dtype=torch.int32, device="cuda")
    native.call("gk_random_playouts", seed, 0, n, neutral, native.ptr(boards), native.ptr(infos),
                native.stream_of(boards.device))
    return boards.cpu().numpy(), infos.cpu().numpy()


def test_playouts_match_golden(kai, golden):
    g = golden("playouts.npz")
    boards, infos = _playouts(int(g["seed"][0]), len(g["boards"]))
    assert np.array_equal(boards, g["boards"]) and np.array_equal(infos, g["infos"])


def test_playouts_full_size_bit_exact(kai, oracle):
    """4096 complete games from the default start: boards, winner, reason, score, plies."""
    boards, infos = _playouts(20241, 4096)
    eb, ei = oracle.random_playouts(20241, 4096)
    assert np.array_equal(boards, eb) and np.array_equal(infos, ei)
    for neutral in (-1, 8):
        boards, infos = _playouts(7, 512, neutral)
        eb, ei = oracle.random_playouts(7, 512, neutral=neutral)
        assert np.array_equal(boards, eb) and np.array_equal(infos, ei)


def test_generated_positions_and_encodings_full_size(kai, oracle, golden):
    from kingdom_ai import _native as native
    from kingdom_ai.gpu_rules import bits_to_records
    from kingdom_ai.gpu_puct import encode_packed

    g = golden("positions.npz")
    n = 65536
    bits = torch.empty((n, 16), dtype=torch.int32, device="cuda")
    native.call("gk_gen_positions", int(g["seed"][0]), 0, n, native.ptr(bits), native.stream_of(bits.device))
    recs = bits_to_records(bits).cpu().numpy()
    assert np.array_equal(recs[:256], g["records"])
    exp = oracle.gen_positions(int(g["seed"][0]), n)
    assert np.array_equal(recs, exp)
    f, m = encode_packed(bits)
    ef, em = oracle.encode(exp)
    assert np.array_equal(f.cpu().numpy(), ef) and np.array_equal(m.cpu().numpy(), em)
    # The wire-format encoder gives the same bits.
    batch = kai.GpuStateBatch.from_records(exp)
    f2, m2 = batch.encode()
    assert torch.equal(f2, f) and torch.equal(m2, m)


def test_settled_and_unsettled_packed_states_play_alike(kai, oracle):
    """Packed states carry a territory-settled flag (meta bit 27) that lets a
    placement re-examine only the empty component it splits. States packed
    from records have it clear and run the full claim; states whose owned
    territory was stripped (unclaimed territory far from the next move) must
    be claimed in full too. Every variant is played for several plies against
    the oracle."""
    from kingdom_ai import _native as native
    from kingdom_ai.gpu_rules import bits_to_records, records_to_bits

    n = 4096
    settled = torch.empty((n, 16), dtype=torch.int32, device="cuda")
    native.call("gk_gen_positions", 99, 0, n, native.ptr(settled), native.stream_of(settled.device))
    assert bool(((settled[:, 15] >> 27) & 1).all())
    recs = bits_to_records(settled).cpu().numpy()
    stripped = recs.copy()
    stripped[:, 81:162] = 0
    variants = [(settled, recs.copy()), (records_to_bits(torch.from_numpy(recs).cuda()), recs.copy()),
                (records_to_bits(torch.from_numpy(stripped).cuda()), stripped.copy())]
    assert not bool(((variants[1][0][:, 15] >> 27) & 1).any())
    rng = np.random.default_rng(5)
    for ply in range(12):
        base = variants[0][1]
        acts = np.full(n, 81, dtype=np.int32)
        for i in range(n):
            cand = [a for a in range(81) if base[i, a] == 0]
            if cand:
                acts[i] = rng.choice(cand)
        a = torch.from_numpy(acts).cuda()
        for k, (bits, exp) in enumerate(variants):
            accepted = torch.empty(n, dtype=torch.bool, device="cuda")
            native.call("gk_play_bits", native.ptr(bits), native.ptr(a), 4, native.ptr(accepted), n,
                        native.stream_of(bits.device))
            exp2, exp_acc = oracle.play(exp, acts)
            assert np.array_equal(accepted.cpu().numpy(), exp_acc.astype(bool)), (ply, k)
            assert np.array_equal(bits_to_records(bits).cpu().numpy()[:, :169], exp2[:, :169]), (ply, k)
            variants[k] = (bits, exp2)
