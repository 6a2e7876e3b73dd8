"""Root tactical checks of the CUDA search (GpuPUCTOptions.tactical_checks).

The root positions are those of the reference's tactical-check tests
(tests/gpu_puct_test.py:196-295) plus generated positions, recorded in
tests/golden/tactics.npz from the compiled reference engine. The expected
outcomes are the reference tests' own assertions; with the injected evaluator
the whole search must also equal the oracle's search with the same root
narrowing, bit for bit.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


class FixedPolicyValue(torch.nn.Module):
    """Constant logits: +12 on one action, -30 on another, 0 elsewhere; value 0.
    The same adversarial prior as the reference's tests (gpu_puct_test.py:18-32)."""

    def __init__(self, preferred=0, rejected=None):
        super().__init__()
        logits = torch.zeros(82)
        logits[preferred] = 12.0
        if rejected is not None:
            logits[rejected] = -30.0
        self.register_buffer("logits", logits)

    def forward(self, features):
        return self.logits.expand(len(features), -1), torch.zeros(len(features), device=features.device)


def options(simulations, epsilon, tactics=True, seed=5):
    from kingdom_ai.gpu_puct import GpuPUCTOptions
    return GpuPUCTOptions(simulations=simulations, c_puct=1.5, dirichlet_alpha=0.3, dirichlet_epsilon=epsilon,
                          seed=seed, tactical_checks=tactics)


def roots(golden, group):
    g = golden("tactics.npz")
    keep = g["group"] == group
    return g["roots"][keep], g["expected"][keep]


def search(model, recs, opts):
    from kingdom_ai import GpuPUCT, GpuStateBatch
    batch = GpuStateBatch.from_records(recs)
    before = batch.states.clone()
    result = GpuPUCT(model, opts).search(batch)
    assert torch.equal(batch.states, before)  # the input states stay untouched
    return result


def test_low_prior_capture_is_found(golden, oracle):
    # gpu_puct_test.py:196-229: the capture is the one action the model rejects.
    recs, expected = roots(golden, 0)
    model = FixedPolicyValue(preferred=80, rejected=11)
    plain = search(model, recs[:1], options(4, 0.0, tactics=False))
    assert plain.visits[0, 11].item() == 0
    finished = oracle.initial(1, 40)
    oracle.play(finished, [81])
    oracle.play(finished, [81])
    result = search(model, np.concatenate([recs, finished]), options(4, 0.25))
    assert result.actions[:-1].cpu().tolist() == expected.tolist()
    assert (result.best_values[:-1] == 1).all().item()
    assert result.network_evaluations[:-1].cpu().tolist() == [1] * len(recs)
    assert result.actions[-1].item() == -1


def test_last_liberty_defense_in_all_symmetries(golden):
    # gpu_puct_test.py:231-259: one reply avoids an immediate capture.
    recs, expected = roots(golden, 1)
    result = search(FixedPolicyValue(preferred=35), recs, options(8, 0.25))
    assert result.actions.cpu().tolist() == expected.tolist()
    for i, a in enumerate(expected):
        assert result.visits[i, a].item() == 8


def test_suicide_capture_passes_and_no_safe_fallback(golden):
    # gpu_puct_test.py:261-295.
    recs, _ = roots(golden, 2)
    result = search(FixedPolicyValue(preferred=10), recs, options(8, 0.0))
    assert result.visits[0, 10].item() == 0 and result.priors[0, 10].item() == 0
    assert result.actions[1].item() == 8 and result.best_values[1].item() == 1
    assert result.actions[2].item() == 81 and result.best_values[2].item() == 1
    assert result.visits[3, 81].item() == 0
    assert result.actions[4].item() == 81 and result.best_values[4].item() == -1


def test_injected_evaluator_search_equals_oracle_with_tactics(golden, oracle):
    from kingdom_ai import HashEvaluator
    g = golden("tactics.npz")
    recs, sims = g["roots"], 48
    result = search(HashEvaluator(), recs, options(sims, 0.0))
    for i, rec in enumerate(recs):
        r = oracle.puct(rec, sims, tactics=True)
        assert np.array_equal(result.visits[i].cpu().numpy(), r["visits"])
        assert np.array_equal(result.priors[i].cpu().numpy(), r["priors"])
        assert result.actions[i].item() == r["best"]
        assert result.nodes[i].item() == r["nodes"]
        assert result.root_values[i].item() == r["root_value"]


def test_native_network_keeps_to_the_candidates(golden, oracle):
    from kingdom_ai.model import random_network
    g = golden("tactics.npz")
    recs = g["roots"]
    result = search(random_network(64, 2, 9), recs, options(16, 0.25))
    visits = result.visits.cpu().numpy()
    priors = result.priors.cpu().numpy()
    for i, rec in enumerate(recs):
        _, allow = oracle.root_tactics(rec)
        assert (visits[i][~allow] == 0).all() and (priors[i][~allow] == 0).all()
        assert allow[result.actions[i].item()]
    first_two = g["group"] < 2
    assert np.array_equal(result.actions.cpu().numpy()[first_two], g["expected"][first_two])


def test_selfplay_engine_plays_tactical_candidates(oracle):
    from kingdom_ai.gpu_rules import bits_to_records
    from kingdom_ai.model import random_network
    from kingdom_ai.selfplay import SelfPlayEngine

    engine = SelfPlayEngine(random_network(64, 2, 3), 64, options(16, 0.25, seed=11), replay_capacity=1 << 12)
    checked = 0
    for _ in range(10):
        before = bits_to_records(engine.states).cpu().numpy()
        engine.step(1)
        torch.cuda.synchronize()
        engine.check()
        after = bits_to_records(engine.states).cpu().numpy()
        allow_words = engine.search.root_allow.cpu().numpy().astype(np.uint32)
        for lane, rec in enumerate(before):
            _, allow = oracle.root_tactics(rec)
            bits = np.asarray([(allow_words[lane, a >> 5] >> (a & 31)) & 1 for a in range(82)], dtype=bool)
            legal = oracle.encode(rec[None])[1][0]
            assert np.array_equal(bits & legal, allow)
            for a in np.flatnonzero(legal):
                nxt, _ = oracle.play(rec[None].copy(), [a])
                if np.array_equal(nxt[0, :169], after[lane, :169]):
                    assert allow[a]
                    checked += 1
                    break
    assert checked > 0
