"""CUDA PUCT against the oracle and the reference fixtures (tests/gpu_puct_test.py in spirit).

With the injected evaluator, visits, priors, best move, node and evaluation
counts and the double root value must equal the C++ PUCT::search bit for bit.
"""

import numpy as np
import pytest
import torch

from conftest import cpu_threads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kai():
    import kingdom_ai
    return kingdom_ai


def opts(kai, simulations, epsilon=0.0, seed=742, **kw):
    return kai.GpuPUCTOptions(simulations=simulations, c_puct=1.5, dirichlet_alpha=0.3, dirichlet_epsilon=epsilon,
                              seed=seed, **kw)


def test_hash_search_matches_reference_fixture(kai, golden):
    g = golden("puct.npz")
    sims = int(g["simulations"][0])
    batch = kai.GpuStateBatch.from_records(g["roots"])
    result = kai.GpuPUCT(kai.HashEvaluator(), opts(kai, sims)).search(batch)
    assert np.array_equal(result.visits.cpu().numpy(), g["visits"])
    assert np.array_equal(result.priors.cpu().numpy(), g["priors"])
    assert result.actions.cpu().tolist() == g["stats"][:, 0].tolist()
    assert result.simulations.cpu().tolist() == g["stats"][:, 1].tolist()
    assert result.nodes.cpu().tolist() == g["stats"][:, 2].tolist()
    assert result.network_evaluations.cpu().tolist() == g["stats"][:, 3].tolist()
    assert np.array_equal(result.root_values.cpu().numpy(), g["values"][:, 0])
    assert np.array_equal(result.best_values.cpu().numpy(), g["values"][:, 1].astype(np.float32))


def test_hash_search_full_size_bit_exact(kai, oracle):
    """1024 generated roots x 800 simulations, c_puct 1.5, no noise."""
    from kingdom_ai import _native as native
    from kingdom_ai.gpu_puct import search_hash

    n, sims = 1024, 800
    bits = torch.empty((n, 16), dtype=torch.int32, device="cuda")
    native.call("gk_gen_positions", 4242, 0, n, native.ptr(bits), native.stream_of(bits.device))
    result = search_hash(bits, sims)
    recs = oracle.gen_positions(4242, n)
    visits, best, roots = oracle.puct_batch(recs, sims, threads=cpu_threads())
    assert np.array_equal(result.visits.cpu().numpy(), visits)
    assert np.array_equal(result.actions.cpu().numpy(), best.astype(np.int64))
    assert np.array_equal(result.root_values.cpu().numpy(), roots)



def test_fused_hash_search_equals_the_step_by_step_search(kai):
    """gk_puct_search_hash (one kernel, a warp per tree) against GpuPUCT's
    per-simulation select / evaluate / expand launches, c_puct 1.25, FPU 0.2."""
    from kingdom_ai import _native as native
    from kingdom_ai.gpu_puct import SearchWorkspace, _allocate_results

    n, sims = 300, 96
    bits = torch.empty((n, 16), dtype=torch.int32, device="cuda")
    native.call("gk_gen_positions", 99, 0, n, native.ptr(bits), native.stream_of(bits.device))
    options = kai.GpuPUCTOptions(simulations=sims, c_puct=1.25, dirichlet_epsilon=0.0, fpu_reduction=0.2, seed=1)
    step = kai.GpuPUCT(kai.HashEvaluator(), options).search_packed(bits)
    ws = SearchWorkspace(n, sims + 1, bits.device)
    out = _allocate_results(n, bits.device)
    native.call("gk_puct_search_hash", ws.pointer, n, sims, native.ptr(bits), native.PuctOptions(1.25, 0.0, 1, 0.2),
                out.struct, native.stream_of(bits.device))
    fused = out.result()
    for name in ("actions", "visits", "policy", "values", "simulations", "network_evaluations", "priors",
                 "best_values", "nodes", "root_values"):
        assert torch.equal(getattr(fused, name), getattr(step, name)), name

def zero_model(kai):
    from kingdom_ai.model import PolicyValueNet
    torch.manual_seed(829)
    model = PolicyValueNet(channels=8, residual_blocks=1)
    with torch.no_grad():
        for p in model.parameters():
            p.zero_()
    return model


class FixedPolicyValue(torch.nn.Module):
    """An adversarial prior and exact colour value (tests/gpu_puct_test.py:18-33)."""

    def __init__(self, preferred=0, rejected=None, color_value=False):
        super().__init__()
        logits = torch.zeros(82)
        logits[preferred] = 12.0
        if rejected is not None:
            logits[rejected] = -30.0
        self.register_buffer("logits", logits)
        self.color_value = color_value

    def forward(self, features):
        values = (2 * features[:, 5, 0, 0] - 1 if self.color_value
                  else torch.zeros(len(features), device=features.device))
        return self.logits.expand(len(features), -1), values


def assert_result(oracle, result, recs, simulations):
    """Invariants of tests/gpu_puct_test.py:93-150."""
    count = len(recs)
    for field, dtype, shape in (("actions", torch.int64, (count,)), ("visits", torch.int32, (count, 82)),
                                ("policy", torch.float32, (count, 82)), ("values", torch.float32, (count,)),
                                ("simulations", torch.int32, (count,)),
                                ("network_evaluations", torch.int32, (count,)), ("nodes", torch.int32, (count,)),
                                ("best_values", torch.float32, (count,))):
        tensor = getattr(result, field)
        assert tensor.device.type == "cuda" and tensor.dtype == dtype and tuple(tensor.shape) == shape, field
    actions = result.actions.cpu().tolist()
    visits = result.visits.cpu()
    policies = result.policy.cpu()
    values = result.values.cpu()
    sims = result.simulations.cpu().tolist()
    evals = result.network_evaluations.cpu().tolist()
    nodes = result.nodes.cpu().tolist()
    best_values = result.best_values.cpu()
    assert torch.isfinite(policies).all() and torch.isfinite(values).all() and (values.abs() <= 1).all()
    assert torch.isfinite(best_values).all() and (best_values.abs() <= 1).all() and (visits >= 0).all()
    _, masks = oracle.encode(recs)
    for i, rec in enumerate(recs):
        mask = torch.from_numpy(masks[i])
        assert (visits[i, ~mask] == 0).all() and (policies[i, ~mask] == 0).all()
        if rec[166] != 0:
            assert actions[i] == -1 and sims[i] == 0 and evals[i] == 0 and nodes[i] == 0
            assert best_values[i].item() == 0.0 and visits[i].sum() == 0 and policies[i].sum() == 0
            assert values[i].item() == (1.0 if rec[167] == rec[162] else -1.0)
        else:
            assert sims[i] == simulations and visits[i].sum() == simulations
            assert 1 <= evals[i] <= simulations + 1 and 1 <= nodes[i] <= simulations + 1
            assert mask[actions[i]] and visits[i, actions[i]] > 0
            torch.testing.assert_close(policies[i], visits[i].float() / simulations, rtol=0, atol=1e-7)


def terminal_records(oracle, golden):
    passed = oracle.initial(1, 40)
    passed, _ = oracle.play(passed, [81])
    passed, _ = oracle.play(passed, [81])
    cap = golden("rules_captures.npz")["records"][1][5:6]  # last-liberty capture, terminal
    sui = golden("rules_suicide.npz")["records"][1][0:1]
    return np.concatenate([passed, cap, sui])


def test_uniform_model_search_matches_oracle_exact_visits(kai, oracle, golden):
    cap = golden("rules_captures.npz")["records"][0]
    recs = np.concatenate([oracle.initial(1, 40), oracle.initial(1, -1), cap[5:7]])
    result = kai.GpuPUCT(zero_model(kai), opts(kai, 8)).search(kai.GpuStateBatch.from_records(recs))
    assert_result(oracle, result, recs, 8)
    for i, rec in enumerate(recs):
        r = oracle.puct(rec, 8, uniform=True)
        assert np.array_equal(result.visits[i].cpu().numpy(), r["visits"])
        assert result.actions[i].item() == r["best"]
        assert result.network_evaluations[i].item() == r["evaluations"]
        assert abs(result.values[i].item() - r["root_value"]) <= 1e-6


def test_forced_capture_wins_for_both_colours_and_input_is_unchanged(kai, oracle, golden):
    recs = golden("rules_captures.npz")["records"][0][5:7]
    batch = kai.GpuStateBatch.from_records(recs)
    result = kai.GpuPUCT(FixedPolicyValue(preferred=40), opts(kai, 8)).search(batch)
    assert_result(oracle, result, recs, 8)
    assert result.actions.cpu().tolist() == [40, 40]
    assert np.array_equal(batch.states.cpu().numpy(), recs)
    continued = batch.clone()
    assert continued.play(result.actions).all().item()
    assert continued.states[:, 166].cpu().tolist() == [1, 1]


def test_fpu_explores_optimistic_unvisited_moves(kai, oracle):
    model = FixedPolicyValue(preferred=52, color_value=True)
    state = kai.GpuStateBatch.initial(16)
    legacy = kai.GpuPUCT(model, kai.GpuPUCTOptions(simulations=128, dirichlet_epsilon=0.25, seed=103)).search(state)
    optimistic = kai.GpuPUCT(model, kai.GpuPUCTOptions(simulations=128, dirichlet_epsilon=0.25, seed=103,
                                                       fpu_reduction=0.0)).search(state)
    assert_result(oracle, optimistic, oracle.initial(16, 40), 128)
    assert (optimistic.visits > 0).sum().item() > (legacy.visits > 0).sum().item()
    torch.testing.assert_close(optimistic.priors, legacy.priors, rtol=0, atol=0)
    assert (legacy.visits[:, 52] == 128).all().item()
    assert (optimistic.visits[:, 52] < 128).all().item()


def test_terminal_roots_bypass_the_model(kai, oracle, golden):
    model = zero_model(kai)

    def reject(module, inputs):
        raise AssertionError("terminal rows must bypass the policy/value model")

    recs = terminal_records(oracle, golden)
    searcher = kai.GpuPUCT(model, opts(kai, 8))
    searcher.model.register_forward_pre_hook(reject)
    batch = kai.GpuStateBatch.from_records(recs)
    result = searcher.search(batch)
    assert_result(oracle, result, recs, 8)
    assert np.array_equal(batch.states.cpu().numpy(), recs)


def test_mixed_batch_only_forwards_active_rows(kai, oracle, golden):
    recs = np.concatenate([oracle.initial(1, 40), terminal_records(oracle, golden)[:1], oracle.initial(1, -1)])
    searcher = kai.GpuPUCT(zero_model(kai), opts(kai, 4))
    shapes = []
    searcher.model.register_forward_hook(lambda m, i, o: shapes.append((tuple(i[0].shape), torch.is_grad_enabled())))
    result = searcher.search(kai.GpuStateBatch.from_records(recs))
    assert_result(oracle, result, recs, 4)
    assert shapes[0][0] == (2, 10, 9, 9)
    assert all(s[1:] == (10, 9, 9) and 0 < s[0] <= 2 and not g for s, g in shapes)


def test_source_model_is_preserved(kai, oracle):
    model = zero_model(kai)
    model.train()
    weights = {k: v.clone() for k, v in model.state_dict().items()}
    recs = oracle.initial(2, 40)
    kai.GpuPUCT(model, opts(kai, 4)).search(kai.GpuStateBatch.from_records(recs))
    assert model.training
    for k, v in model.state_dict().items():
        assert v.device.type == "cpu" and torch.equal(v, weights[k])


def test_root_noise_repeats_with_the_same_seed_and_reset_seed_restarts(kai, oracle):
    model = zero_model(kai)
    recs = np.concatenate([oracle.initial(1, 40), oracle.initial(1, -1)])
    batch = kai.GpuStateBatch.from_records(recs)
    first = kai.GpuPUCT(model, opts(kai, 16, epsilon=0.25, seed=6502)).search(batch)
    second = kai.GpuPUCT(model, opts(kai, 16, epsilon=0.25, seed=6502)).search(batch)
    for field in ("actions", "visits", "policy", "values", "simulations", "network_evaluations", "priors"):
        torch.testing.assert_close(getattr(first, field), getattr(second, field), rtol=0, atol=0)
    assert_result(oracle, first, recs, 16)
    searcher = kai.GpuPUCT(model, opts(kai, 8, epsilon=0.25, seed=6502))
    cpu_rng = torch.get_rng_state().clone()
    a = searcher.search(batch)
    b = searcher.search(batch)
    assert not torch.equal(a.priors, b.priors)
    searcher.reset_seed()
    c = searcher.search(batch)
    for field in ("actions", "visits", "priors", "best_values", "nodes"):
        torch.testing.assert_close(getattr(a, field), getattr(c, field), rtol=0, atol=0)
    assert torch.equal(torch.get_rng_state(), cpu_rng)
    for invalid in (-1, 2**64, True, 1.5):
        with pytest.raises(ValueError):
            searcher.reset_seed(invalid)
    # Noise keeps priors a distribution over legal moves.
    pri = a.priors.cpu().numpy()
    assert np.allclose(pri.sum(axis=1), 1.0, atol=1e-12)


def test_nonfinite_model_outputs_raise_and_preserve_input(kai, oracle):
    for field in ("logits", "values"):
        model = zero_model(kai)
        searcher = kai.GpuPUCT(model, opts(kai, 8))

        def corrupt(module, inputs, output, field=field):
            logits, values = output
            if field == "logits":
                logits = logits.clone()
                logits[:, 0] = float("nan")
            else:
                values = torch.full_like(values, float("nan"))
            return logits, values

        searcher.model.register_forward_hook(corrupt)
        batch = kai.GpuStateBatch.initial(2)
        before = batch.states.clone()
        with pytest.raises(ValueError):
            searcher.search(batch)
        torch.testing.assert_close(batch.states, before, rtol=0, atol=0)


def test_wrong_search_input_is_rejected(kai):
    searcher = kai.GpuPUCT(zero_model(kai), opts(kai, 4))
    for invalid in (object(), torch.zeros((2, 170), device="cuda", dtype=torch.int32)):
        with pytest.raises((TypeError, ValueError)):
            searcher.search(invalid)


def test_nondefault_stream_orders_search(kai, oracle):
    recs = oracle.initial(2, 40)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        batch = kai.GpuStateBatch.from_records(recs)
        batch.play(torch.tensor([0, 80], device="cuda", dtype=torch.int32))
        result = kai.GpuPUCT(kai.HashEvaluator(), opts(kai, 16)).search(batch)
        summed = result.visits.sum(dim=1)
    stream.synchronize()
    played, _ = oracle.play(recs.copy(), [0, 80])
    assert summed.cpu().tolist() == [16, 16]
    for i in range(2):
        assert np.array_equal(result.visits[i].cpu().numpy(), oracle.puct(played[i], 16)["visits"])


def test_completed_selfplay_stays_legal(kai, oracle):
    recs = np.concatenate([oracle.initial(1, 40), oracle.initial(1, -1), oracle.initial(1, 8),
                           oracle.initial(1, 40)])
    batch = kai.GpuStateBatch.from_records(recs)
    searcher = kai.GpuPUCT(zero_model(kai), opts(kai, 4))
    for _ in range(170):
        if (recs[:, 166] != 0).all():
            break
        result = searcher.search(batch)
        assert_result(oracle, result, recs, 4)
        actions = result.actions.cpu().numpy().astype(np.int32)
        for i in range(len(recs)):
            if recs[i, 166] == 0:
                assert oracle.lib.gko_legal(recs[i], int(actions[i]))
        recs, expected = oracle.play(recs.copy(), actions)
        accepted = batch.play(result.actions)
        assert accepted.cpu().numpy().astype(np.uint8).tolist() == expected.tolist()
        assert np.array_equal(batch.states.cpu().numpy(), recs)
    assert (recs[:, 166] != 0).all()
