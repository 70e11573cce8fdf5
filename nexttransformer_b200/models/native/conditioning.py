"""LoopFormer's time conditioning of the shared ring.

Before pass ``r`` of ``R`` over the core ring the model embeds the pass's position ``t = r / R`` and
its step size ``1 / R``: each scalar becomes sinusoidal features (geometric frequencies
``10000^(-i / half)``, cosines then sines) fed through a two-layer SiLU MLP; the two embeddings are
summed and RMS-normalised into one conditioning vector.  One bias-free head per core layer maps
SiLU(conditioning) to four offsets, squashed to ``bound * tanh(.)``: attention output gate, MLP
output gate, attention input scale, MLP input scale, applied by the block as ``1 + offset``.
Everything runs in fp32.  The heads start at zero, so training begins from the unmodulated ring.
Module names are the reference's checkpoint keys; behaviour matches
``nexttransformer/models/native/conditioning.py``.
"""
import math

import torch
from torch import nn
import torch.nn.functional as F

from nexttransformer_b200.models.shell import norm


def fourier_features(values, dim):
    """[len(values), dim] cos / sin features of scalar positions (zero-padded to an odd dim)."""
    half = dim // 2
    rates = torch.exp(torch.arange(half, device=values.device, dtype=torch.float32) * (-math.log(10000) / half))
    phase = values.float().unsqueeze(-1) * rates
    return F.pad(torch.cat((phase.cos(), phase.sin()), -1), (0, dim - 2 * half))


class TimeEmbedding(nn.Module):
    """Scalar -> fourier features -> Linear -> SiLU -> Linear."""

    def __init__(self, width, fourier_dim):
        super().__init__()
        self.dim = fourier_dim
        self.mlp = nn.Sequential(nn.Linear(fourier_dim, width), nn.SiLU(), nn.Linear(width, width))

    def forward(self, t):
        return self.mlp(fourier_features(t, self.dim))


class LoopConditioner(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        width = config.width
        self.time = TimeEmbedding(width, config.fourier_dim)
        self.delta = TimeEmbedding(width, config.fourier_dim)
        self.modulation = nn.ModuleList(nn.Sequential(nn.SiLU(), nn.Linear(width, 4 * width, bias=False))
                                        for _ in range(config.core_layers))

    @torch.no_grad()
    def init_weights(self):
        for embedding in (self.time, self.delta):
            for layer in (embedding.mlp[0], embedding.mlp[2]):
                layer.weight.normal_(0.0, 0.02)
                layer.bias.zero_()
        for head in self.modulation:
            head[1].weight.zero_()

    def conditioning(self, recursion, batch, device):
        """The RMS-normalised [batch, width] conditioning vector of pass ``recursion``."""
        total = self.config.recursions
        position = torch.full((batch,), recursion / total, device=device, dtype=torch.float32)
        step = torch.full((batch,), 1 / total, device=device, dtype=torch.float32)
        return norm(self.time(position) + self.delta(step))

    def forward(self, recursion, batch, device):
        """Per core layer the [batch, 4 width] bounded offsets of pass ``recursion``."""
        bound = self.config.loop_modulation_bound
        with torch.autocast(device_type=device.type, enabled=False):
            cond = self.conditioning(recursion, batch, device)
            return [bound * torch.tanh(head(cond)) for head in self.modulation]

    @torch.no_grad()
    def diagnostics(self):
        device = next(self.parameters()).device
        offsets = torch.cat([o.flatten() for r in range(self.config.recursions) for o in self(r, 1, device)])
        bound = self.config.loop_modulation_bound
        return {"loop_modulation_absmax": float(offsets.abs().max()),
                "loop_modulation_saturated_fraction": float((offsets.abs() > .95 * bound).float().mean())}
