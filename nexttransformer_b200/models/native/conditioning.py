"""LoopFormer conditioning: recursion time t = r/R and step 1/R are embedded with sinusoidal
features and two-layer SiLU MLPs, summed and RMS-normalised; one bias-free projection per core
layer gives four bounded offsets ``bound * tanh(.)`` (attention gate, MLP gate, attention input
scale, MLP input scale) that the block applies as ``1 + offset``.  Evaluated in fp32.  The offset
projections start at zero (identity modulation).
Behaviour: ``nexttransformer/models/native/conditioning.py:10-59``.
"""
import math

import torch
from torch import nn
import torch.nn.functional as F

from nexttransformer_b200.models.shell import norm


class TimeEmbedding(nn.Module):
    def __init__(self, width, fourier_dim):
        super().__init__()
        self.dim = fourier_dim
        self.mlp = nn.Sequential(nn.Linear(fourier_dim, width), nn.SiLU(), nn.Linear(width, width))

    def forward(self, t):
        half = self.dim // 2
        freq = torch.exp(-math.log(10000) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
        ang = t.float()[:, None] * freq
        feats = torch.cat((ang.cos(), ang.sin()), dim=-1)
        if self.dim % 2:
            feats = F.pad(feats, (0, 1))
        return self.mlp(feats)


class LoopConditioner(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.time = TimeEmbedding(config.width, config.fourier_dim)
        self.delta = TimeEmbedding(config.width, config.fourier_dim)
        self.modulation = nn.ModuleList(nn.Sequential(nn.SiLU(), nn.Linear(config.width, 4 * config.width, bias=False))
                                        for _ in range(config.core_layers))

    @torch.no_grad()
    def init_weights(self):
        for emb in (self.time, self.delta):
            for m in emb.modules():
                if isinstance(m, nn.Linear):
                    nn.init.normal_(m.weight, std=0.02)
                    nn.init.zeros_(m.bias)
        for mod in self.modulation:
            nn.init.zeros_(mod[-1].weight)

    def forward(self, recursion, batch, device):
        c = self.config
        with torch.autocast(device_type=device.type, enabled=False):
            t = torch.full((batch,), recursion / c.recursions, device=device, dtype=torch.float32)
            step = torch.full_like(t, 1 / c.recursions)
            cond = norm(self.time(t) + self.delta(step))
            return [c.loop_modulation_bound * torch.tanh(m(cond)) for m in self.modulation]

    @torch.no_grad()
    def diagnostics(self):
        dev = next(self.parameters()).device
        vals = torch.cat([v.flatten() for r in range(self.config.recursions) for v in self(r, 1, dev)])
        bound = self.config.loop_modulation_bound
        return {"loop_modulation_absmax": float(vals.abs().max()),
                "loop_modulation_saturated_fraction": float((vals.abs() > .95 * bound).float().mean())}
