"""Policy/value network of the self-play workloads (fp32 PyTorch definition).

Layout (the batch-norm variant of python/kingdom_ai/model.py:30-84, with the
value head's hidden width fixed at 64):

    stem   conv3x3(10 -> C) + BN + ReLU
    blocks [conv3x3(C -> C) + BN + ReLU, conv3x3(C -> C) + BN, + skip, ReLU] x R
    policy conv1x1(C -> 2) + BN + ReLU -> flatten(162) -> Linear(162 -> 82) logits
    value  conv1x1(C -> 1) + BN + ReLU -> flatten(81) -> Linear(81 -> 64) -> ReLU
           -> Linear(64 -> 1) -> tanh

``GroupNormPolicyValueNet`` is the reference's own network (GroupNorm
everywhere, value hidden width C), which the native kernels also run.

This module is the fp32 reference the native bf16 kernels are judged
against; ``fold`` turns its eval-mode batch norms into per-channel scale and
bias, which is what the native network consumes.
"""

from __future__ import annotations

import math

import torch
from torch import nn

INPUT_CHANNELS = 10
BOARD = 9
ACTION_SIZE = 82
VALUE_HIDDEN = 64


class _Block(nn.Module):
    def __init__(self, channels):
        super().__init__()
        self.conv1 = nn.Conv2d(channels, channels, 3, padding=1, bias=False)
        self.bn1 = nn.BatchNorm2d(channels)
        self.conv2 = nn.Conv2d(channels, channels, 3, padding=1, bias=False)
        self.bn2 = nn.BatchNorm2d(channels)

    def forward(self, x):
        h = torch.relu(self.bn1(self.conv1(x)))
        return torch.relu(x + self.bn2(self.conv2(h)))


class PolicyValueNet(nn.Module):
    """Return policy logits [N, 82] and current-player values [N]."""

    def __init__(self, channels: int = 64, residual_blocks: int = 6):
        super().__init__()
        if type(channels) is not int or channels < 1:
            raise ValueError("channels must be a positive integer")
        if type(residual_blocks) is not int or residual_blocks < 0:
            raise ValueError("residual_blocks must be a non-negative integer")
        self.channels = channels
        self.residual_blocks = residual_blocks
        self.stem = nn.Conv2d(INPUT_CHANNELS, channels, 3, padding=1, bias=False)
        self.stem_bn = nn.BatchNorm2d(channels)
        self.blocks = nn.ModuleList([_Block(channels) for _ in range(residual_blocks)])
        self.policy_conv = nn.Conv2d(channels, 2, 1, bias=False)
        self.policy_bn = nn.BatchNorm2d(2)
        self.policy_fc = nn.Linear(2 * BOARD * BOARD, ACTION_SIZE)
        self.value_conv = nn.Conv2d(channels, 1, 1, bias=False)
        self.value_bn = nn.BatchNorm2d(1)
        self.value_fc1 = nn.Linear(BOARD * BOARD, VALUE_HIDDEN)
        self.value_fc2 = nn.Linear(VALUE_HIDDEN, 1)

    def forward(self, features: torch.Tensor):
        x = torch.relu(self.stem_bn(self.stem(features)))
        for block in self.blocks:
            x = block(x)
        p = torch.relu(self.policy_bn(self.policy_conv(x))).flatten(1)
        logits = self.policy_fc(p)
        v = torch.relu(self.value_bn(self.value_conv(x))).flatten(1)
        value = torch.tanh(self.value_fc2(torch.relu(self.value_fc1(v)))).squeeze(1)
        return logits, value


def random_network(channels: int, blocks: int, seed: int) -> PolicyValueNet:
    """Kaiming-normal weights and randomised batch-norm statistics from `seed`.

    The running statistics and affine parameters are drawn at random so that
    folding them into the convolutions is not the identity.
    """
    g = torch.Generator().manual_seed(seed)
    net = PolicyValueNet(channels, blocks)
    with torch.no_grad():
        for module in net.modules():
            if isinstance(module, (nn.Conv2d, nn.Linear)):
                fan_in = module.weight[0].numel()
                module.weight.copy_(torch.randn(module.weight.shape, generator=g) * (2.0 / fan_in) ** 0.5)
                if module.bias is not None:
                    module.bias.copy_(torch.randn(module.bias.shape, generator=g) * 0.05)
            elif isinstance(module, nn.BatchNorm2d):
                n = module.num_features
                module.weight.copy_(1.0 + 0.1 * torch.randn(n, generator=g))
                module.bias.copy_(0.1 * torch.randn(n, generator=g))
                module.running_mean.copy_(0.1 * torch.randn(n, generator=g))
                module.running_var.copy_(1.0 + 0.2 * torch.rand(n, generator=g))
    return net.eval()


def calibrate_batchnorm(model: PolicyValueNet, features: torch.Tensor) -> PolicyValueNet:
    """Set every batch norm's running statistics from one pass over `features`.

    A freshly initialised residual tower with arbitrary running statistics
    grows its activations layer after layer; calibrated statistics normalise
    each layer as a trained network's would, so the folded convolutions see
    realistic value ranges.
    """
    bns = [m for m in model.modules() if isinstance(m, nn.BatchNorm2d)]
    for bn in bns:
        bn.reset_running_stats()
        bn.momentum = None  # cumulative average over the calibration pass
    model.train()
    with torch.no_grad():
        model(features)
    for bn in bns:
        bn.momentum = 0.1
    return model.eval()


def fold(conv: nn.Conv2d, bn: nn.BatchNorm2d):
    """Eval-mode BN folded into the preceding bias-free conv: (weight, bias) fp32."""
    scale = bn.weight / torch.sqrt(bn.running_var + bn.eps)
    weight = conv.weight * scale.reshape(-1, *([1] * (conv.weight.dim() - 1)))
    bias = bn.bias - bn.running_mean * scale
    return weight.detach().float(), bias.detach().float()


class _GroupNormBlock(nn.Module):
    """Residual block of the reference network: conv, GroupNorm, ReLU, conv,
    GroupNorm, added to the input, ReLU (python/kingdom_ai/model.py:13-27)."""

    def __init__(self, channels):
        super().__init__()
        groups = math.gcd(8, channels)
        self.layers = nn.Sequential(
            nn.Conv2d(channels, channels, 3, padding=1, bias=False),
            nn.GroupNorm(groups, channels),
            nn.ReLU(),
            nn.Conv2d(channels, channels, 3, padding=1, bias=False),
            nn.GroupNorm(groups, channels),
        )
        self.activation = nn.ReLU()

    def forward(self, x):
        return self.activation(x + self.layers(x))


class GroupNormPolicyValueNet(nn.Module):
    """The reference's PolicyValueNet (python/kingdom_ai/model.py:30-84):
    GroupNorm(gcd(8, C), C) after every trunk convolution, GroupNorm(1, 2) and
    GroupNorm(1, 1) in the heads, and a value head of C hidden units. Module
    names and parameter shapes are the reference's, so its checkpoints'
    state_dicts load unchanged (checkpoint.py:86-89 stores ``model_config``
    {channels, residual_blocks} beside them)."""

    def __init__(self, channels: int = 32, residual_blocks: int = 2):
        super().__init__()
        if type(channels) is not int or channels < 1:
            raise ValueError("channels must be a positive integer")
        if type(residual_blocks) is not int or residual_blocks < 0:
            raise ValueError("residual_blocks must be a non-negative integer")
        self.channels = channels
        self.residual_blocks = residual_blocks
        self.trunk = nn.Sequential(
            nn.Conv2d(INPUT_CHANNELS, channels, 3, padding=1, bias=False),
            nn.GroupNorm(math.gcd(8, channels), channels),
            nn.ReLU(),
            *[_GroupNormBlock(channels) for _ in range(residual_blocks)],
        )
        self.policy_head = nn.Sequential(
            nn.Conv2d(channels, 2, 1, bias=False),
            nn.GroupNorm(1, 2),
            nn.ReLU(),
            nn.Flatten(),
            nn.Linear(2 * BOARD * BOARD, ACTION_SIZE),
        )
        self.value_head = nn.Sequential(
            nn.Conv2d(channels, 1, 1, bias=False),
            nn.GroupNorm(1, 1),
            nn.ReLU(),
            nn.Flatten(),
            nn.Linear(BOARD * BOARD, channels),
            nn.ReLU(),
            nn.Linear(channels, 1),
            nn.Tanh(),
        )

    @property
    def model_config(self) -> dict:
        return {"channels": self.channels, "residual_blocks": self.residual_blocks}

    def forward(self, features: torch.Tensor):
        shared = self.trunk(features)
        return self.policy_head(shared), self.value_head(shared).squeeze(-1)


def random_groupnorm_network(channels: int, blocks: int, seed: int) -> GroupNormPolicyValueNet:
    """Kaiming-normal weights and randomised GroupNorm affine parameters from `seed`."""
    g = torch.Generator().manual_seed(seed)
    net = GroupNormPolicyValueNet(channels, blocks)
    with torch.no_grad():
        for module in net.modules():
            if isinstance(module, (nn.Conv2d, nn.Linear)):
                fan_in = module.weight[0].numel()
                module.weight.copy_(torch.randn(module.weight.shape, generator=g) * (2.0 / fan_in) ** 0.5)
                if module.bias is not None:
                    module.bias.copy_(torch.randn(module.bias.shape, generator=g) * 0.05)
            elif isinstance(module, nn.GroupNorm):
                n = module.num_channels
                module.weight.copy_(1.0 + 0.1 * torch.randn(n, generator=g))
                module.bias.copy_(0.1 * torch.randn(n, generator=g))
    return net.eval()


# Schema-1 checkpoint fields (python/kingdom_ai/checkpoint.py:14-37): the
# observation planes in order, and the value perspective.
FEATURE_NAMES = ("own_stones", "opponent_stones", "neutral_stones", "own_territory", "opponent_territory",
                 "black_to_play", "own_remaining_fraction", "opponent_remaining_fraction",
                 "consecutive_passes_fraction", "legal_placements")
CHECKPOINT_FIELDS = {"format_version", "board_size", "action_size", "feature_names", "perspective",
                     "model_config", "state_dict"}


def load_reference_model(checkpoint, device="cpu") -> GroupNormPolicyValueNet:
    """A reference checkpoint (a path, or the payload torch.load returns) as a
    GroupNormPolicyValueNet in eval mode, with the checks of the reference's
    load_model (python/kingdom_ai/checkpoint.py:40-90)."""
    payload = checkpoint
    if not isinstance(checkpoint, dict):
        payload = torch.load(checkpoint, map_location="cpu", weights_only=True)
    if not isinstance(payload, dict) or set(payload) != CHECKPOINT_FIELDS:
        raise ValueError("checkpoint is missing or has unexpected schema fields")
    for key, expected in (("format_version", 1), ("board_size", BOARD), ("action_size", ACTION_SIZE)):
        if type(payload[key]) is not int or payload[key] != expected:
            raise ValueError(f"checkpoint {key} does not match the supported schema")
    names = payload["feature_names"]
    if type(names) is not list or any(type(n) is not str for n in names) or names != list(FEATURE_NAMES):
        raise ValueError("checkpoint feature_names do not match the input schema")
    if type(payload["perspective"]) is not str or payload["perspective"] != "to_play":
        raise ValueError("checkpoint value perspective must be to_play")
    config = payload["model_config"]
    if not isinstance(config, dict) or set(config) != {"channels", "residual_blocks"}:
        raise ValueError("checkpoint model_config is invalid")
    with torch.random.fork_rng(devices=[]):
        model = GroupNormPolicyValueNet(**config)
    state, expected = payload["state_dict"], model.state_dict()
    if not isinstance(state, dict) or set(state) != set(expected):
        raise ValueError("checkpoint parameters do not match the model configuration")
    for name, reference in expected.items():
        value = state[name]
        if not isinstance(value, torch.Tensor):
            raise ValueError(f"checkpoint parameter {name} is not a tensor")
        if value.layout != torch.strided or value.shape != reference.shape or value.dtype != reference.dtype:
            raise ValueError(f"checkpoint parameter {name} has the wrong shape or dtype")
        if not bool(torch.isfinite(value).all()):
            raise ValueError(f"checkpoint parameter {name} contains NaN or infinity")
    model.load_state_dict(state, strict=True)
    return model.to(device).eval()


def native_supported(model) -> bool:
    """Whether the native kernels can evaluate this module as it is."""
    return ((type(model) is PolicyValueNet and model.channels in (32, 64, 128))
            or (type(model) is GroupNormPolicyValueNet and model.channels in (32, 64, 128)))


# ---------------------------------------------------------------------------
# Native (sm_100a) network
# ---------------------------------------------------------------------------

def _pack_conv(weight: torch.Tensor, cin_pad: int, column_fused: bool) -> torch.Tensor:
    """[Cout][Cin][3][3] fp32 -> the bf16 operand layout of the native tower.

    Per tap (row-major over (dr, dc)) [Cin/8][Cout][8] for 128 channels; for 64
    channels, per row offset dr [Cin/8][3 (dc)][Cout][8], i.e. the three column
    taps of a row offset side by side, which the tower reads as one 192-column
    operand (include/gk.h, gk_net_t).
    """
    cout, cin = weight.shape[:2]
    w = torch.zeros((cout, cin_pad, 3, 3), dtype=torch.float32)
    w[:, :cin] = weight
    if column_fused:
        rows = w.permute(2, 1, 3, 0).reshape(3, cin_pad // 8, 8, 3, cout)  # [dr][k/8][k%8][dc][n]
        return rows.permute(0, 1, 3, 4, 2).contiguous().to(torch.bfloat16)  # [dr][k/8][dc][n][k%8]
    taps = w.permute(2, 3, 1, 0).reshape(9, cin_pad, cout)          # [tap][k][n]
    taps = taps.reshape(9, cin_pad // 8, 8, cout).permute(0, 1, 3, 2)  # [tap][k/8][n][k%8]
    return taps.contiguous().to(torch.bfloat16)


class NativePolicyValueNet:
    """A PolicyValueNet (BN folded) or GroupNormPolicyValueNet packed for the
    tcgen05 kernels (bf16 convolutions).

    ``forward_states`` / ``forward_features`` return raw logits [N,82] and
    values [N] (fp32); ``evaluate_workspace`` is the in-search leaf evaluator.
    Convolutions run in bf16 with fp32 accumulation; the 1x1 head convolutions
    and the fully connected heads run in fp32.
    """

    def __init__(self, model, device="cuda"):
        from . import _native as native
        self.native = native
        self.device = torch.device(device)
        if not native_supported(model):
            raise ValueError("the native network supports PolicyValueNet or GroupNormPolicyValueNet "
                             "with 32, 64 or 128 channels")
        self.channels, self.blocks = model.channels, model.residual_blocks
        self.norm = 1 if isinstance(model, GroupNormPolicyValueNet) else 0
        model = model.eval()
        with torch.no_grad():
            if self.norm:
                tensors = self._groupnorm_tensors(model)
            else:
                tensors = self._batchnorm_tensors(model)
        expected = native.library().gk_net_weight_bytes(self.channels, self.blocks)
        if tensors["conv_w"].numel() * 2 != expected:
            raise RuntimeError("packed weight size mismatch")
        self.tensors = {k: v.to(self.device).contiguous() for k, v in tensors.items()}
        t = self.tensors
        ptr = lambda name: t[name].data_ptr() if name in t else None  # noqa: E731
        self.struct = native.NetStruct(
            self.channels, self.blocks, ptr("conv_w"), ptr("conv_b"), ptr("head_w"), ptr("head_b"), ptr("pol_w"),
            ptr("pol_b"), ptr("val_w1"), ptr("val_b1"), ptr("val_w2"), ptr("val_b2"), self.norm, ptr("norm_w"),
            ptr("norm_b"), ptr("head_norm"))
        self._headfeat = None
        self.status = torch.zeros(2, dtype=torch.int32, device=self.device)

    def _batchnorm_tensors(self, model):
        convs = [fold(model.stem, model.stem_bn)]
        for block in model.blocks:
            convs.append(fold(block.conv1, block.bn1))
            convs.append(fold(block.conv2, block.bn2))
        fused = self.channels == 64
        packed = [_pack_conv(convs[0][0].cpu(), 16, fused)] + [_pack_conv(w.cpu(), self.channels, fused)
                                                                for w, _ in convs[1:]]
        pw, pb = fold(model.policy_conv, model.policy_bn)
        vw, vb = fold(model.value_conv, model.value_bn)
        return {
            "conv_w": torch.cat([p.reshape(-1) for p in packed]),
            "conv_b": torch.stack([b for _, b in convs]).float(),
            "head_w": torch.cat([pw.reshape(2, -1), vw.reshape(1, -1)]).float(),
            "head_b": torch.cat([pb, vb]).float(),
            # Fully connected heads feature-major ([162][82], [81][H]): the heads
            # kernel stages them with contiguous 16-byte copies.
            "pol_w": model.policy_fc.weight.detach().float().t().contiguous(),
            "pol_b": model.policy_fc.bias.detach().float(),
            "val_w1": model.value_fc1.weight.detach().float().t().contiguous(),
            "val_b1": model.value_fc1.bias.detach().float(),
            "val_w2": model.value_fc2.weight.detach().float().reshape(-1),
            "val_b2": model.value_fc2.bias.detach().float().reshape(-1),
        }

    def _groupnorm_tensors(self, model):
        """The reference layout (python/kingdom_ai/model.py:13-84): bias-free
        convolutions in the per-tap bf16 layout and each GroupNorm's affine
        parameters (include/gk.h, gk_net_t, norm 1)."""
        convs, norms = [(model.trunk[0], model.trunk[1])], []
        for block in list(model.trunk)[3:]:
            convs.append((block.layers[0], block.layers[1]))
            convs.append((block.layers[3], block.layers[4]))
        packed = [_pack_conv(convs[0][0].weight.detach().float().cpu(), 16, False)]
        packed += [_pack_conv(c.weight.detach().float().cpu(), self.channels, False) for c, _ in convs[1:]]
        for _, gn in convs:
            if gn.num_groups != 8 or abs(gn.eps - 1e-5) > 1e-12:
                raise ValueError("the native network expects GroupNorm(8, C) with eps 1e-5")
            norms.append(gn)
        ph, vh = model.policy_head, model.value_head
        return {
            "conv_w": torch.cat([p.reshape(-1) for p in packed]),
            "norm_w": torch.stack([g.weight.detach().float() for g in norms]),
            "norm_b": torch.stack([g.bias.detach().float() for g in norms]),
            "head_w": torch.cat([ph[0].weight.detach().float().reshape(2, -1),
                                 vh[0].weight.detach().float().reshape(1, -1)]),
            "head_norm": torch.cat([ph[1].weight.detach().float(), ph[1].bias.detach().float(),
                                    vh[1].weight.detach().float(), vh[1].bias.detach().float()]),
            "pol_w": ph[4].weight.detach().float().t().contiguous(), "pol_b": ph[4].bias.detach().float(),
            "val_w1": vh[4].weight.detach().float().t().contiguous(), "val_b1": vh[4].bias.detach().float(),
            "val_w2": vh[6].weight.detach().float().reshape(-1), "val_b2": vh[6].bias.detach().float().reshape(-1),
        }

    def _workspace(self, n):
        if self._headfeat is None or self._headfeat.shape[0] < n:
            self._headfeat = torch.empty((n, 243), dtype=torch.float32, device=self.device)
        return self._headfeat

    def _forward(self, states, features, n):
        native = self.native
        logits = torch.empty((n, ACTION_SIZE), dtype=torch.float32, device=self.device)
        values = torch.empty((n,), dtype=torch.float32, device=self.device)
        headfeat = self._workspace(n)
        with torch.cuda.device(self.device):
            stream = native.stream_of(self.device)
            native.call("gk_net_forward", self.struct, native.ptr(states), native.ptr(features), n,
                        native.ptr(headfeat), native.ptr(logits), native.ptr(values), native.ptr(self.status),
                        stream)
        return logits, values

    def forward_states(self, bits: torch.Tensor):
        """Packed states int32 [N,16] -> (logits [N,82], values [N])."""
        bits = bits.to(self.device).contiguous()
        return self._forward(bits, None, bits.shape[0])

    def forward_features(self, features: torch.Tensor):
        """Schema-1 features fp32 [N,10,9,9] -> (logits [N,82], values [N])."""
        features = features.to(device=self.device, dtype=torch.float32).contiguous()
        return self._forward(None, features, features.shape[0])

    def evaluate_workspace(self, ws, stream):
        """Fill the search workspace's policy/value for every leaf that needs it."""
        headfeat = self._workspace(ws.batch)
        self.native.call("gk_net_evaluate_puct", self.struct, ws.pointer, ws.batch, ws.capacity,
                         self.native.ptr(headfeat), self.native.ptr(self.status), stream)

    def check(self):
        """Raise if any kernel reported a bounded wait that gave up."""
        code, where = (int(v) for v in self.status.tolist())
        if code:
            raise RuntimeError(f"native network reported error bits {code:#x} (wait at {where & 0x7fffffff:#x}, "
                               f"parity {(where >> 31) & 1})")
