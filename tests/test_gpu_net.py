"""Native tcgen05 network against the fp32 PyTorch model of the same layout.

Tolerance (bf16 operands, fp32 accumulation, stated here and in the design
notes): max |logit - logit_fp32| <= 0.08 and max |value - value_fp32| <= 0.03,
both measured on Kaiming-initialised networks with randomised batch norms.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_TOL = 0.08
VALUE_TOL = 0.03


@pytest.fixture(scope="module")
def selftest():
    """One tcgen05 MMA whose addresses stay in range under any stride reading."""
    from kingdom_ai import _native as native

    g = torch.Generator().manual_seed(7)
    a = torch.randn(128, 16, generator=g).bfloat16()
    b = torch.randn(64, 16, generator=g).bfloat16()
    d = torch.zeros(128, 64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ac, bc = a.view(torch.int16).cuda(), b.view(torch.int16).cuda()
    native.call("gk_mma_selftest", native.ptr(ac), native.ptr(bc), native.ptr(d), native.ptr(status),
                native.stream_of(d.device))
    torch.cuda.synchronize()
    expected = a.float() @ b.float().T
    return d.cpu(), expected, int(status.item())


def test_tensor_core_selftest(selftest):
    d, expected, status = selftest
    assert status == 0
    torch.testing.assert_close(d, expected, rtol=1e-5, atol=1e-4)


def native_or_skip(selftest):
    d, expected, status = selftest
    if status != 0 or not torch.allclose(d, expected, rtol=1e-5, atol=1e-4):
        pytest.skip("tensor-core self-test failed; the network kernels are not run")


def positions(n, seed):
    from kingdom_ai import _native as native
    bits = torch.empty((n, 16), dtype=torch.int32, device="cuda")
    native.call("gk_gen_positions", seed, 0, n, native.ptr(bits), native.stream_of(bits.device))
    return bits


def compare(channels, blocks, n, seed, selftest):
    from kingdom_ai.gpu_puct import encode_packed
    from kingdom_ai.model import NativePolicyValueNet, random_network

    native_or_skip(selftest)
    model = random_network(channels, blocks, seed)
    bits = positions(n, seed)
    features, _ = encode_packed(bits)
    with torch.no_grad():
        ref_logits, ref_values = model.cuda()(features)
    net = NativePolicyValueNet(model.cpu(), device="cuda")
    logits, values = net.forward_states(bits)
    logits2, values2 = net.forward_features(features)
    torch.cuda.synchronize()
    net.check()
    dl = (logits - ref_logits).abs().max().item()
    dv = (values - ref_values).abs().max().item()
    print(f"C={channels} R={blocks} n={n}: max |dlogit| {dl:.4g}, max |dvalue| {dv:.4g}")
    assert dl <= LOGIT_TOL and dv <= VALUE_TOL
    # The state-fed and feature-fed stems see identical bf16 inputs.
    assert torch.equal(logits, logits2) and torch.equal(values, values2)
    return dl, dv


@pytest.mark.parametrize("n", [1, 5, 7, 64])
def test_small_batches_and_ragged_groups(selftest, n):
    compare(64, 1, n, 11 + n, selftest)


def test_selfplay_network_full_batch(selftest):
    """6 blocks x 64 channels, 4096 leaves (the self-play evaluation batch)."""
    compare(64, 6, 4096, 5, selftest)


def test_large_network(selftest):
    """10 blocks x 128 channels, 8192 positions."""
    compare(128, 10, 8192, 8, selftest)


def test_native_network_in_search(selftest, oracle):
    """GpuPUCT routes a PolicyValueNet to the native evaluator; results are a valid search."""
    import kingdom_ai
    from kingdom_ai.model import random_network

    native_or_skip(selftest)
    from test_gpu_puct import assert_result

    model = random_network(64, 2, 3)
    recs = oracle.gen_positions(21, 37)
    batch = kingdom_ai.GpuStateBatch.from_records(recs)
    opts = kingdom_ai.GpuPUCTOptions(simulations=24, dirichlet_epsilon=0.0)
    native = kingdom_ai.GpuPUCT(model, opts).search(batch)
    assert_result(oracle, native, recs, 24)
    # The fp32 PyTorch evaluator gives nearly the same root priors.
    ref = kingdom_ai.GpuPUCT(_AsModule(model), opts).search(batch)
    diff = (native.priors - ref.priors).abs().max().item()
    assert diff < 0.05


class _AsModule(torch.nn.Module):
    """Wraps a PolicyValueNet so GpuPUCT evaluates it with PyTorch instead of natively."""

    def __init__(self, model):
        super().__init__()
        self.inner = model

    def forward(self, features):
        return self.inner(features)
