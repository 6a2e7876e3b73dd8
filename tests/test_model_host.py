"""The reference network restated in this package (CPU, no GPU needed)."""

import numpy as np
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
