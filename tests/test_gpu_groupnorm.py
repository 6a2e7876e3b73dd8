"""The reference's own network (GroupNorm everywhere, python/kingdom_ai/model.py:
13-84) on the native tcgen05 kernels.

Tolerances against the fp32 PyTorch module (bf16 operands, fp32 accumulation
and statistics): max |logit - fp32| <= 2e-2 * max |logit| + 5e-3 and
max |value - fp32| <= 4e-2, about twice the largest errors measured on a
B200 (logits 0.044 at max |logit| 3.63, values 0.021, 128 x 2 on 517
positions). The reference checkpoints come from tests/golden/groupnorm.npz
(the reference module's own weights and outputs).
"""

import json
import os

import pytest
import torch

from test_gpu_net import native_or_fail, positions, selftest  # noqa: F401
from test_model_host import load_reference

pytestmark = pytest.mark.gpu

RTOL, ATOL, VTOL = 2e-2, 5e-3, 4e-2


def check(model, features, bits=None):
    from kingdom_ai.model import NativePolicyValueNet
    with torch.no_grad():
        ref_logits, ref_values = model.cpu()(features.cpu())
    net = NativePolicyValueNet(model, device="cuda")
    logits, values = net.forward_features(features.cuda())
    torch.cuda.synchronize()
    net.check()
    scale = ref_logits.abs().max().item()
    err_logit = (logits.cpu() - ref_logits).abs().max().item()
    err_value = (values.cpu() - ref_values).abs().max().item()
    stats = dict(norm="group", channels=model.channels, blocks=model.residual_blocks, n=features.shape[0],
                 logit_scale=scale, fp32_max_abs_logit=err_logit, fp32_max_abs_value=err_value)
    print(json.dumps(stats))
    if os.environ.get("GK_NET_STATS"):
        with open(os.environ["GK_NET_STATS"], "a") as f:
            f.write(json.dumps(stats) + "\n")
    assert err_logit <= RTOL * scale + ATOL
    assert err_value <= VTOL
    if bits is not None:
        l2, v2 = net.forward_states(bits)
        assert torch.equal(l2, logits) and torch.equal(v2, values)
    return net


def test_reference_checkpoints(selftest, golden):  # noqa: F811
    native_or_fail(selftest)
    for tag in ("c32", "c64"):
        g, net = load_reference(golden, tag)
        features = torch.from_numpy(g["features"])
        check(net, features)
        # the stored reference outputs themselves
        from kingdom_ai.model import NativePolicyValueNet
        logits, values = NativePolicyValueNet(net, device="cuda").forward_features(features.cuda())
        ref = torch.from_numpy(g[f"{tag}/logits"])
        assert (logits.cpu() - ref).abs().max().item() <= RTOL * ref.abs().max().item() + ATOL
        assert (values.cpu() - torch.from_numpy(g[f"{tag}/values"])).abs().max().item() <= VTOL


@pytest.mark.parametrize("channels,blocks,n", [(32, 2, 1), (32, 2, 23), (32, 4, 1000), (64, 2, 333),
                                               (128, 2, 517)])
def test_random_groupnorm_networks(selftest, channels, blocks, n):  # noqa: F811
    from kingdom_ai.gpu_puct import encode_packed
    from kingdom_ai.model import random_groupnorm_network
    native_or_fail(selftest)
    bits = positions(n, channels + blocks)
    features, _ = encode_packed(bits)
    check(random_groupnorm_network(channels, blocks, 7), features, bits)


def test_groupnorm_network_in_both_searches(selftest, oracle):  # noqa: F811
    from kingdom_ai import GpuBatchedPUCT, GpuPUCT, GpuPUCTOptions, PUCTOptions
    from kingdom_ai.model import random_groupnorm_network
    native_or_fail(selftest)
    model = random_groupnorm_network(32, 2, 3)
    bits = positions(96, 11)
    r = GpuPUCT(model, GpuPUCTOptions(simulations=16, seed=1)).search_packed(bits)
    assert (r.visits.sum(1) == 16).all().item()
    s = GpuBatchedPUCT(96, PUCTOptions(simulations=24), 8)
    b = s.search(bits, model)
    assert (b.visits.sum(1) == 24).all().item() and (b.simulations == 24).all().item()
    legal = b.legal.gather(1, b.actions[:, None]).flatten()
    assert legal.all().item()


def test_selfplay_with_the_reference_network(selftest):  # noqa: F811
    """Self-play ply by ply with the reference's own 32 x 2 network: the rows
    it writes pass the reference's replay checks."""
    from kingdom_ai import GpuPUCTOptions, validate_rows
    from kingdom_ai.model import random_groupnorm_network
    from kingdom_ai.selfplay import SelfPlayEngine
    native_or_fail(selftest)
    engine = SelfPlayEngine(random_groupnorm_network(32, 2, 5), 64, GpuPUCTOptions(simulations=8, seed=2),
                            replay_capacity=1 << 13)
    engine.step(70)
    torch.cuda.synchronize()
    engine.check()
    n = min(engine.stats()["rows"], engine.replay.capacity)
    assert n > 0
    validate_rows(*engine.replay.rows(0, n))
