"""The reference network restated in this package (CPU, no GPU needed)."""

import numpy as np
import pytest
import torch


def load_reference(golden, tag):
    from kingdom_ai.model import GroupNormPolicyValueNet
    g = golden("groupnorm.npz")
    state = {k.split("/", 1)[1]: torch.from_numpy(v) for k, v in g.items() if k.startswith(tag + "/")
             and k.split("/", 1)[1] not in ("logits", "values")}
    channels = state["trunk.0.weight"].shape[0]
    blocks = sum(1 for k in state if k.endswith("layers.0.weight"))
    net = GroupNormPolicyValueNet(channels, blocks)
    net.load_state_dict(state, strict=True)
    return g, net.eval()


def test_groupnorm_network_loads_reference_checkpoints_and_matches_its_outputs(golden):
    # tests/golden/groupnorm.npz: the reference's own PolicyValueNet
    # (python/kingdom_ai/model.py:30-84) at 32 x 2 and 64 x 1.
    for tag in ("c32", "c64"):
        g, net = load_reference(golden, tag)
        with torch.no_grad():
            logits, values = net(torch.from_numpy(g["features"]))
        np.testing.assert_allclose(logits.numpy(), g[f"{tag}/logits"], rtol=0, atol=1e-5)
        np.testing.assert_allclose(values.numpy(), g[f"{tag}/values"], rtol=0, atol=1e-6)
        assert net.model_config == {"channels": net.channels, "residual_blocks": net.residual_blocks}


def test_reference_checkpoint_payloads_load_with_the_reference_checks(golden):
    # python/kingdom_ai/checkpoint.py:14-90: the schema-1 payload and its checks.
    from kingdom_ai.model import FEATURE_NAMES, load_reference_model
    g, net = load_reference(golden, "c32")
    payload = {"format_version": 1, "board_size": 9, "action_size": 82, "feature_names": list(FEATURE_NAMES),
               "perspective": "to_play", "model_config": net.model_config,
               "state_dict": {k: v.clone() for k, v in net.state_dict().items()}}
    loaded = load_reference_model(payload)
    with torch.no_grad():
        logits, _ = loaded(torch.from_numpy(g["features"]))
    np.testing.assert_allclose(logits.numpy(), g["c32/logits"], rtol=0, atol=1e-5)
    bad = [dict(payload, extra=1), dict(payload, format_version=2), dict(payload, board_size=True),
           dict(payload, feature_names=list(FEATURE_NAMES)[::-1]), dict(payload, perspective="black"),
           dict(payload, model_config={"channels": 32}),
           dict(payload, model_config={"channels": 32, "residual_blocks": 3})]
    for key, change in (("trunk.0.weight", lambda t: t.double()), ("trunk.1.bias", lambda t: t[:-1]),
                        ("policy_head.4.bias", lambda t: t.fill_(float("nan")))):
        state = dict(payload["state_dict"])
        state[key] = change(state[key].clone())
        bad.append(dict(payload, state_dict=state))
    for candidate in bad:
        with pytest.raises(ValueError):
            load_reference_model(candidate)
