"""Policy/value network of the self-play workloads (fp32 PyTorch definition).

Layout (the batch-norm variant of python/kingdom_ai/model.py:30-84, with the
value head's hidden width fixed at 64):

    stem   conv3x3(10 -> C) + BN + ReLU
    blocks [conv3x3(C -> C) + BN + ReLU, conv3x3(C -> C) + BN, + skip, ReLU] x R
    policy conv1x1(C -> 2) + BN + ReLU -> flatten(162) -> Linear(162 -> 82) logits
    value  conv1x1(C -> 1) + BN + ReLU -> flatten(81) -> Linear(81 -> 64) -> ReLU
           -> Linear(64 -> 1) -> tanh

This module is the fp32 reference the native bf16 kernels are judged
against; ``fold`` turns its eval-mode batch norms into per-channel scale and
bias, which is what the native network consumes.
"""

from __future__ import annotations

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


def fold(conv: nn.Conv2d, bn: nn.BatchNorm2d):
    """Eval-mode BN folded into the preceding bias-free conv: (weight, bias) fp32."""
    scale = bn.weight / torch.sqrt(bn.running_var + bn.eps)
    weight = conv.weight * scale.reshape(-1, *([1] * (conv.weight.dim() - 1)))
    bias = bn.bias - bn.running_mean * scale
    return weight.detach().float(), bias.detach().float()
