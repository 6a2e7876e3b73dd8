"""Native tcgen05 network against PyTorch models of the same layout.

Two references:
  * the fp32 PyTorch model (TF32 off) - the accuracy statement for bf16
    arithmetic: max |logit - logit_fp32| <= rtol * max |logit_fp32| + 5e-3 and
    max |value - value_fp32| <= vtol (Kaiming initialisation, batch norms
    calibrated on generated positions; rounding differences compound with
    depth);
  * a PyTorch model that rounds to bf16 exactly where the kernels do (inputs,
    folded weights, every stored activation). It differs from the kernels
    only by fp32 summation order; with integer-valued networks, whose
    arithmetic is exact, the two must agree to fp32 round-off in the heads.

Each tolerance is about twice the error measured on a B200 (max over the
batch, TF32 off in the reference):

  network, positions                 |logit - fp32| (max |logit|)  |value - fp32|
  1 block x 64, 4096                 0.0196 (3.16)                 0.0023
  1 block x 64, 5                    0.0018 (0.17)                 0.0153
  6 x 64 calibrated, 4096            0.0891 (7.16)                 0.0432
  6 x 64 uncalibrated, 2048          0.297 (17.3)                  0 (tanh saturated)
  10 x 128 calibrated, 8192          0.129 (5.03)                  0.0713
"""

import json
import os

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-2   # vs fp32, relative to the largest |logit|
LOGIT_ATOL = 5e-3   # vs fp32, absolute floor for networks with tiny logits
VALUE_ATOL = 3e-2   # vs fp32 (1 block: measured <= 0.0153)
EMU_RTOL = 2e-3     # vs the bf16-rounding emulation, relative to the largest |logit|
EMU_VALUE_ATOL = 1e-3  # (1 block: measured <= 3.7e-4)


def bf16_emulation(model, features):
    """Forward with bf16 rounding at the kernel's rounding points, fp32 elsewhere."""
    from kingdom_ai.model import fold

    r = lambda t: t.bfloat16().float()  # noqa: E731
    layers = [fold(model.stem, model.stem_bn)]
    for block in model.blocks:
        layers += [fold(block.conv1, block.bn1), fold(block.conv2, block.bn2)]
    x = r(features)
    skip = None
    for i, (w, b) in enumerate(layers):
        y = F.conv2d(x, r(w.to(features.device)), b.to(features.device), padding=1)
        if i >= 2 and i % 2 == 0:
            y = y + skip
        # Every layer's output is stored in bf16, including the last, which
        # the head pass reads back.
        x = r(torch.relu(y))
        if i % 2 == 0:
            skip = x
    pw, pb = fold(model.policy_conv, model.policy_bn)
    vw, vb = fold(model.value_conv, model.value_bn)
    p = torch.relu(F.conv2d(x, pw.to(x.device), pb.to(x.device))).flatten(1)
    v = torch.relu(F.conv2d(x, vw.to(x.device), vb.to(x.device))).flatten(1)
    logits = model.policy_fc(p)
    value = torch.tanh(model.value_fc2(torch.relu(model.value_fc1(v)))).squeeze(1)
    return logits, value


@pytest.fixture(scope="module")
def selftest():
    """One tcgen05 MMA whose addresses stay in range under any stride reading."""
    from kingdom_ai import _native as native

    g = torch.Generator().manual_seed(7)
    a = torch.randn(128, 16, generator=g).bfloat16()
    b = torch.randn(64, 16, generator=g).bfloat16()
    d = torch.zeros(128, 64, device="cuda")
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    ac, bc = a.view(torch.int16).cuda(), b.view(torch.int16).cuda()
    native.call("gk_mma_selftest", native.ptr(ac), native.ptr(bc), native.ptr(d), native.ptr(status),
                native.stream_of(d.device))
    torch.cuda.synchronize()
    expected = a.float() @ b.float().T
    return d.cpu(), expected, int(status[0].item())


def test_tensor_core_selftest(selftest):
    d, expected, status = selftest
    assert status == 0
    torch.testing.assert_close(d, expected, rtol=1e-5, atol=1e-4)


def native_or_fail(selftest):
    """The network kernels run on the tensor cores: a broken tcgen05 path
    fails every network test rather than skipping it."""
    d, expected, status = selftest
    assert status == 0, f"tensor-core self-test reported status {status:#x}"
    torch.testing.assert_close(d, expected, rtol=1e-5, atol=1e-4)


@pytest.fixture(autouse=True)
def true_fp32():
    """The fp32 reference forward runs in fp32: cuDNN's TF32 convolutions off."""
    saved = (torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32)
    torch.backends.cudnn.allow_tf32 = torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = saved


def positions(n, seed):
    from kingdom_ai import _native as native
    bits = torch.empty((n, 16), dtype=torch.int32, device="cuda")
    native.call("gk_gen_positions", seed, 0, n, native.ptr(bits), native.stream_of(bits.device))
    return bits


def compare(channels, blocks, n, seed, selftest, calibrate=False, emu_rtol=EMU_RTOL, rtol=LOGIT_RTOL,
            emu_vtol=EMU_VALUE_ATOL, vtol=VALUE_ATOL):
    from kingdom_ai.gpu_puct import encode_packed
    from kingdom_ai.model import NativePolicyValueNet, calibrate_batchnorm, random_network

    native_or_fail(selftest)
    model = random_network(channels, blocks, seed)
    bits = positions(n, seed)
    features, _ = encode_packed(bits)
    model = model.cuda()
    if calibrate:
        calibrate_batchnorm(model, features)
    with torch.no_grad():
        ref_logits, ref_values = model(features)
        emu_logits, emu_values = bf16_emulation(model, features)
    net = NativePolicyValueNet(model.cpu(), device="cuda")
    logits, values = net.forward_states(bits)
    logits2, values2 = net.forward_features(features)
    torch.cuda.synchronize()
    net.check()
    scale = ref_logits.abs().max().item()
    stats = dict(channels=channels, blocks=blocks, n=n, logit_scale=scale,
                 fp32_max_abs_logit=(logits - ref_logits.cuda()).abs().max().item(),
                 fp32_max_abs_value=(values - ref_values.cuda()).abs().max().item(),
                 emu_max_abs_logit=(logits - emu_logits.cuda()).abs().max().item(),
                 emu_max_abs_value=(values - emu_values.cuda()).abs().max().item())
    print(json.dumps(stats))
    out = os.environ.get("GK_NET_STATS")
    if out:
        with open(out, "a") as f:
            f.write(json.dumps(stats) + "\n")
    assert stats["emu_max_abs_logit"] <= emu_rtol * scale and stats["emu_max_abs_value"] <= emu_vtol
    assert stats["fp32_max_abs_logit"] <= rtol * scale + LOGIT_ATOL and stats["fp32_max_abs_value"] <= vtol
    # The state-fed and feature-fed stems see identical bf16 inputs.
    assert torch.equal(logits, logits2) and torch.equal(values, values2)
    return stats


@pytest.mark.parametrize("n", [1, 5, 7, 64])
def test_small_batches_and_ragged_groups(selftest, n):
    compare(64, 1, n, 11 + n, selftest)


def test_many_groups_per_cta(selftest):
    """4096 positions = 820 groups over 148 CTAs: barrier phases across groups."""
    compare(64, 1, 4096, 9, selftest)
    compare(128, 1, 1001, 10, selftest)


def test_selfplay_network_full_batch(selftest):
    """6 blocks x 64 channels, 4096 leaves (the self-play evaluation batch)."""
    compare(64, 6, 4096, 5, selftest, calibrate=True, emu_rtol=1e-2, rtol=2e-2, emu_vtol=0.05, vtol=0.09)


def test_large_network(selftest):
    """10 blocks x 128 channels, 8192 positions."""
    compare(128, 10, 8192, 8, selftest, calibrate=True, emu_rtol=3e-2, rtol=4e-2, emu_vtol=0.1, vtol=0.15)


def test_uncalibrated_deep_network_stays_within_bf16_drift(selftest):
    """Arbitrary BN statistics blow logits up to ~30; the error stays a fraction of that."""
    compare(64, 6, 2048, 6, selftest, emu_rtol=2e-2, rtol=3e-2, emu_vtol=1e-3, vtol=1e-3)


def integer_network(channels, blocks, seed):
    """A network whose tower arithmetic is exact in bf16 and fp32.

    Conv weights are sparse in {-1, 0, 1} (the residual branch's second conv
    only {-1, 0}, so the residual stream cannot grow), batch norms fold to an
    identity scale with integer biases, and the stem ignores the two
    fractional stock planes. Every stored activation is then a small multiple
    of 1/2 and every fp32 sum is exact, so the native tower must reproduce
    the emulation to the last bit; only the fp32 fully connected heads see
    summation-order round-off.
    """
    from kingdom_ai.model import PolicyValueNet

    g = torch.Generator().manual_seed(seed)
    net = PolicyValueNet(channels, blocks)
    with torch.no_grad():
        for name, m in net.named_modules():
            if isinstance(m, torch.nn.Conv2d):
                if name.endswith("conv2"):
                    w = -(torch.rand(m.weight.shape, generator=g) < 0.01).float()
                else:
                    keep = (torch.rand(m.weight.shape, generator=g) < 0.1).float()
                    w = torch.randint(-1, 2, m.weight.shape, generator=g).float() * keep
                if name == "stem":
                    w[:, 6:8] = 0.0
                m.weight.copy_(w)
            elif isinstance(m, torch.nn.BatchNorm2d):
                m.eps = 2.0 ** -20
                m.running_mean.zero_()
                m.running_var.fill_(1.0 - 2.0 ** -20)  # var + eps == 1 exactly
                m.weight.fill_(1.0)
                lo, hi = (0, 2) if name.endswith("bn2") else (-1, 0)
                m.bias.copy_(torch.randint(lo, hi + 1, (m.num_features,), generator=g).float())
    return net.eval()


@pytest.mark.parametrize("channels,blocks,n", [(64, 6, 4096), (128, 10, 2048)])
def test_integer_network_is_exact(selftest, channels, blocks, n):
    from kingdom_ai.gpu_puct import encode_packed
    from kingdom_ai.model import NativePolicyValueNet

    native_or_fail(selftest)
    model = integer_network(channels, blocks, 13).cuda()
    bits = positions(n, 77)
    features, _ = encode_packed(bits)
    with torch.no_grad():
        emu_logits, emu_values = bf16_emulation(model, features)
        # float64 on the CPU: every convolution sum of this network is exact
        # (cuDNN's fp32 algorithms, Winograd among them, need not be).
        ref_logits, ref_values = (t.float().cuda() for t in model.cpu().double()(features.cpu().double()))
    net = NativePolicyValueNet(model.cpu().float(), device="cuda")
    logits, values = net.forward_states(bits)
    torch.cuda.synchronize()
    net.check()
    scale = max(1.0, emu_logits.abs().max().item())
    assert emu_logits.std(dim=0).mean().item() > 1e-3  # the network is not trivial
    assert (logits - emu_logits).abs().max().item() <= 1e-5 * scale
    assert (values - emu_values).abs().max().item() <= 1e-5
    # With exact arithmetic the bf16 network is also the fp32 network.
    assert (logits - ref_logits).abs().max().item() <= 1e-5 * scale


@pytest.mark.parametrize("channels,blocks", [(64, 6), (128, 2)])
def test_outputs_do_not_depend_on_batch_size_or_slot(selftest, channels, blocks):
    """A position's outputs are bit-identical whatever the batch around it.

    Every batch size maps images to different CTAs, image groups and 128-row
    tiles (full rounds of five-image groups, then the balanced tail of 2-5
    images per CTA), so sizes around the round boundaries of a 148-SM grid
    check that every image is computed exactly once; a permuted batch checks
    that the row a position lands on does not change its arithmetic.
    """
    from kingdom_ai.model import NativePolicyValueNet, random_network

    native_or_fail(selftest)
    n = 3001
    bits = positions(n, 4242)
    net = NativePolicyValueNet(random_network(channels, blocks, 5), device="cuda")
    full_logits, full_values = net.forward_states(bits)
    for m in (1, 2, 3, 7, 11, 147, 148, 149, 295, 296, 297, 739, 740, 741, 1479, 1481, 2221, 2960, 3000):
        logits, values = net.forward_states(bits[:m].contiguous())
        assert torch.equal(logits, full_logits[:m]), m
        assert torch.equal(values, full_values[:m]), m
    perm = torch.randperm(n, generator=torch.Generator().manual_seed(9)).cuda()
    logits, values = net.forward_states(bits[perm].contiguous())
    torch.cuda.synchronize()
    net.check()
    assert torch.equal(logits, full_logits[perm]) and torch.equal(values, full_values[perm])


def test_native_network_in_search(selftest, oracle):
    """GpuPUCT routes a PolicyValueNet to the native evaluator; results are a valid search."""
    import kingdom_ai
    from kingdom_ai.model import random_network

    native_or_fail(selftest)
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
