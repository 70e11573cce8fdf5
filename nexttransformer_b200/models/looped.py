"""Looped / recurrent-depth building blocks: ACT halting, Ouro exit distribution and gate loss,
Huginn depth sampling and sandwich blocks, DeepLoop scaled post-norm blocks (reference:
``nexttransformer/models/looped.py``)."""
import math

import torch
from torch import nn
from torch.nn import functional as F

from nexttransformer_b200.models.shell import norm


def sinusoidal_coordinates(length, width, step, device, dtype):
    """Position + recurrence-step sinusoids added to the state at each UT-ACT loop."""
    inv = 10000. ** (-torch.arange(0, width, 2, device=device, dtype=torch.float32) / width)
    pos = torch.arange(length, device=device, dtype=torch.float32)[:, None] * inv
    dep = torch.tensor(float(step), device=device) * inv
    a = torch.stack((pos.sin(), pos.cos()), -1).flatten(-2)
    b = torch.stack((dep.sin(), dep.cos()), -1).flatten(-2)
    return (a + b).to(dtype)[None]


def act_weights(p, cumulative, alive, final=False, epsilon=.01):
    """ACT: tokens halt once the cumulative halting probability reaches 1 - eps (or at the last loop)."""
    stop = alive & ((cumulative + p >= 1 - epsilon) | final)
    w = torch.where(stop, 1 - cumulative, p) * alive.to(p.dtype)
    rem = torch.where(stop, 1 - cumulative, torch.zeros_like(p))
    return w, cumulative + w, alive & ~stop, rem


def exit_distribution(logits):
    """Exit probability per loop from per-loop hazards; the final loop takes the survival remainder."""
    surv = torch.ones_like(logits[0])
    mass = []
    for g in logits:
        h = g.sigmoid()
        mass.append(surv * h)
        surv = surv * (1 - h)
    return torch.stack((*mass, surv), -1)


def ouro_gate_loss(gates, token_losses, slope=50., threshold=.005):
    """Gate target: continue while the detached per-token loss still improves by > threshold."""
    L = torch.stack(token_losses, -1).detach()
    gain = (L[..., :-1] - L[..., 1:]).clamp_min(0)
    cont = torch.sigmoid(slope * (gain - threshold))
    return F.binary_cross_entropy_with_logits(torch.stack(gates, -1), 1 - cont, reduction="none")


def huginn_depth(config, step):
    """Clipped Poisson-lognormal depth, sampled from a step-keyed private RNG (resume-exact)."""
    g = torch.Generator(device="cpu").manual_seed(config.routing_seed + int(step))
    s = config.huginn_sigma
    tau = torch.randn((), generator=g) * s + math.log(config.huginn_mean - 1) - s * s / 2
    return min(int(torch.poisson(tau.exp(), generator=g)) + 1, config.max_loops)


class SandwichBlock(nn.Module):
    """x = norm(x + attn(norm x)); x = norm(x + mlp(norm x))."""

    def __init__(self, block):
        super().__init__()
        self.attn, self.mlp = block.attn, block.mlp

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        x = norm(x + self.attn(norm(x), ve, cos_sin, window_size, kv_cache))
        return norm(x + self.mlp(norm(x)))


class DeepLoopBlock(nn.Module):
    """Post-norm with residual scale alpha = sqrt(2 L_eff); beta = (8 L_eff)^-1/2 used at init."""

    def __init__(self, block, effective_depth):
        super().__init__()
        self.attn, self.mlp = block.attn, block.mlp
        self.alpha = (2 * effective_depth) ** .5
        self.beta = (8 * effective_depth) ** -.5

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        x = norm(self.alpha * x + self.attn(norm(x), ve, cos_sin, window_size, kv_cache))
        return norm(self.alpha * x + self.mlp(norm(x)))
