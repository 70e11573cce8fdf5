"""Block AttnRes with Canon layers at positions A-D (shared by ``attnres_full_canon_abcd``; this
package declares no method of its own).

A Canon layer is ``x + causal_depthwise_conv(x)`` over the last four positions with
zero-initialised taps, so every one starts as the identity.  They are placed

* A / C: on every sublayer input, after the AttnRes depth read (``LanguageModel._attnres_trunk``
  with an input hook);
* B: on the raw q, k and v projections, before the heads are split, RoPE and QK-norm (the shell
  attention's ``projections`` hook);
* D: on the MLP's hidden pre-activation, before the squared ReLU (the shell MLP's ``hidden`` hook).

The trunk is the Block AttnRes trunk of the residual family with the group starts taken from
the ``groups`` option.  Parameter names and the audited operator sequence (the ledger charges the
depthwise convolutions) are the reference's; behaviour matches
``nexttransformer/methods/attnres_canon_abcd/__init__.py``.
"""
import torch
from torch import nn
import torch.nn.functional as F

from nexttransformer_b200.models.lm import LanguageModel, shell_config
from nexttransformer_b200.models.shell import MLP, CausalSelfAttention
from nexttransformer_b200.ops import plugins as plugin_ops


class Canon(nn.Module):
    """``x + causal depthwise convolution of x`` over ``[B, T, C]`` (window ``size``)."""

    def __init__(self, width, size=4):
        super().__init__()
        self.size = size
        self.weight = nn.Parameter(torch.empty(width, 1, size))

    def forward(self, x):
        if plugin_ops.supported(x, head=False) and x.shape[-1] % 8 == 0 and self.size <= 4:
            return plugin_ops.canon(x, self.weight)  # one kernel each way, fp32 taps
        channels_first = F.pad(x.transpose(1, 2), (self.size - 1, 0))
        return x + F.conv1d(channels_first, self.weight.to(x.dtype), groups=x.shape[-1]).transpose(1, 2)


class CanonAttention(CausalSelfAttention):
    """Shell attention whose raw q, k, v pass through their own Canon layer (position B)."""

    def __init__(self, config, layer):
        super().__init__(config, layer)
        self.canon_qkv = nn.ModuleList(Canon(config.n_embd) for _ in range(3))

    def projections(self, x):
        return tuple(canon(p) for canon, p in zip(self.canon_qkv, super().projections(x)))


class CanonMLP(MLP):
    """Shell ReLU^2 MLP with a Canon layer on the hidden pre-activation (position D)."""

    def __init__(self, config):
        super().__init__(shell_config(config))
        self.canon = Canon(config.mlp_width)

    def hidden(self, x):
        return self.canon(super().hidden(x))


def group_starts(layers, groups):
    """First layer of each of ``groups`` AttnRes groups: sizes as equal as possible, larger first."""
    size, larger = divmod(layers, groups)
    firsts = [g * size + min(g, larger) for g in range(groups)]
    return tuple(firsts)


def _keep_draws():
    """The embedding tables are drawn by ``init_weights``; a second reset would shift the RNG stream."""


class CanonAttnRes(LanguageModel):
    @staticmethod
    def groups(config):
        return config.option("groups")

    def __init__(self, config):
        super().__init__(config)
        self.group_starts = group_starts(config.n_layer, self.groups(config))
        self.depth_queries = nn.Parameter(torch.empty(2 * config.n_layer + 1, config.width))
        self.canon = nn.ModuleList(Canon(config.width) for _ in range(2 * config.n_layer))   # positions A / C
        for module in self.modules():
            if isinstance(module, nn.Embedding):
                module.reset_parameters = _keep_draws

    def _ordinary_hidden(self, idx):
        trunk = self._attnres_trunk(idx, self._embed(idx), self.group_starts, adapt=lambda k, h: self.canon[k](h))
        return trunk, None


def mixer(config, layer):
    return CanonAttention(config, layer)


def ffn(config, layer):
    return CanonMLP(config)


model = CanonAttnRes
frozen = ("resid_lambdas", "x0_lambdas", "backout_lambda")


@torch.no_grad()
def init(model):
    for module in model.modules():
        if isinstance(module, Canon):
            module.weight.zero_()


def check(config):
    groups = config.option("groups")
    if type(groups) is not int or not 1 <= groups <= config.n_layer:
        raise ValueError(f"groups must be a whole number between 1 and the layer count ({config.n_layer})")
