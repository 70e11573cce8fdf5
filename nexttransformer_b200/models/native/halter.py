"""Circle's exit scorer: ``w . RMSNorm(after) + depth_bias[exit] + delta_scale * log(eps + |after -
before| / (eps + |before|))`` (norms divided by sqrt(width), all in fp32, token-local).  Depth biases
start at ``-Phi^-1(conditional survival)`` of the depth law so the initial exits follow it.
Behaviour: ``nexttransformer/models/native/halter.py:11-54``.
"""
import math

import torch
from torch import nn
import torch.nn.functional as F

from nexttransformer_b200.models.shell import norm


class DeltaDepthHalter(nn.Module):
    def __init__(self, width, exits, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(1, width))
        self.depth_bias = nn.Parameter(torch.empty(exits))
        self.delta_scale = nn.Parameter(torch.empty(()))
        self.eps = eps

    @torch.no_grad()
    def init_weights(self, conditional_survival):
        nn.init.normal_(self.weight, std=self.weight.shape[-1] ** -0.5)
        p = torch.tensor(conditional_survival, dtype=torch.float32).clamp(1e-4, 1 - 1e-4)
        self.depth_bias.copy_((-torch.distributions.Normal(0.0, 1.0).icdf(p)).to(self.depth_bias))
        nn.init.zeros_(self.delta_scale)

    def relative_change(self, before, after):
        before, after = before.float(), after.float()
        root = math.sqrt(before.shape[-1])
        change = torch.linalg.vector_norm(after - before, dim=-1) / root
        size = torch.linalg.vector_norm(before, dim=-1) / root
        return torch.log(self.eps + change / (self.eps + size))

    def forward(self, before, after, exit_index):
        with torch.autocast(device_type=after.device.type, enabled=False):
            s = F.linear(norm(after.float()), self.weight).squeeze(-1) + self.depth_bias[exit_index]
            return s + self.delta_scale * self.relative_change(before, after)


def feature_forward_ops(config):
    """Extra element/reduction operations of the exit features per token (outside the matrix count)."""
    if config.architecture != "circle":
        return 0
    from nexttransformer_b200.models.native.depth import depth_reference
    _, surv = depth_reference(config.core_layers, config.circle_max_steps, config.circle_target_steps)
    return sum(surv[config.core_layers - 1:-1]) * (5 * config.width + 10)
