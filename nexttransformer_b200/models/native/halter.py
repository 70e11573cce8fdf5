"""Circle's per-token exit scorer.

For a token whose state moved from ``before`` to ``after`` in ring step ``k`` the score is

    score = <w, RMSNorm(after)> + b_k + s * log(eps + rms(after - before) / (eps + rms(before)))

with ``rms(v) = |v| / sqrt(width)``, computed in fp32 and per token only.  The first term reads the
state, ``b_k`` is a learned per-exit offset and the last term measures how much the step changed the
token relative to its size (a converged token changes little).  A token continues while
``sigmoid(-score) >= 0.5``.  The offsets start at ``-Phi^-1(c_k)`` where ``c_k`` is the depth law's
conditional survival at exit k, so an untrained scorer (``w`` small, ``s = 0``) already exits tokens
at the law's rates.  Parameter names (``weight``, ``depth_bias``, ``delta_scale``) are the
reference's checkpoint keys; behaviour matches ``nexttransformer/models/native/halter.py``.
"""
import math

import torch
from torch import nn
import torch.nn.functional as F

from nexttransformer_b200.models.shell import norm


def log_relative_step(before, after, eps):
    """log(eps + rms(after - before) / (eps + rms(before))) per token, fp32."""
    b32, a32 = before.float(), after.float()
    scale = 1.0 / math.sqrt(b32.shape[-1])
    moved = torch.linalg.vector_norm(a32 - b32, dim=-1) * scale
    size = torch.linalg.vector_norm(b32, dim=-1) * scale
    return (moved / (size + eps) + eps).log()


def survival_offsets(conditional_survival):
    """Exit offsets that reproduce the given per-exit continuation probabilities at zero features."""
    p = torch.as_tensor(conditional_survival, dtype=torch.float32).clamp(1e-4, 1 - 1e-4)
    return -torch.distributions.Normal(0.0, 1.0).icdf(p)


class DeltaDepthHalter(nn.Module):
    def __init__(self, width, exits, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(1, width))
        self.depth_bias = nn.Parameter(torch.empty(exits))
        self.delta_scale = nn.Parameter(torch.empty(()))
        self.eps = eps

    @torch.no_grad()
    def init_weights(self, conditional_survival):
        width = self.weight.shape[-1]
        self.weight.normal_(0.0, width ** -0.5)
        self.depth_bias.copy_(survival_offsets(conditional_survival).to(self.depth_bias))
        self.delta_scale.zero_()

    def relative_change(self, before, after):
        return log_relative_step(before, after, self.eps)

    def forward(self, before, after, exit_index):
        with torch.autocast(device_type=after.device.type, enabled=False):
            state_term = F.linear(norm(after.float()), self.weight)[..., 0]
            return state_term + self.depth_bias[exit_index] + self.delta_scale * log_relative_step(before, after,
                                                                                                   self.eps)


def feature_forward_ops(config):
    """Element and reduction operations of the exit features per input token (outside the matrix
    FLOPs): each scored token costs about 5 width + 10 operations, weighted by the depth law's
    expected number of scored steps."""
    if config.architecture != "circle":
        return 0
    from nexttransformer_b200.models.native.depth import depth_reference
    _, survival = depth_reference(config.core_layers, config.circle_max_steps, config.circle_target_steps)
    scored = sum(survival[config.core_layers - 1:config.circle_max_steps - 1])
    return scored * (5 * config.width + 10)
