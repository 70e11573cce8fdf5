"""Gated attention (Qiu et al., arXiv 2505.06708): ``y_h <- y_h * sigmoid(x W_theta)`` per head.

The gate multiplies each head's attention output before ``c_proj``.  ``granularity`` chooses one gate
value per head channel ("elementwise") or one per head ("headwise").  The gate is a separate bias-free
linear layer ``output_gate`` fed by the block's pre-normalised input (the same input as q/k/v); its
name puts it in the auxiliary AdamW group while q/k/v/proj stay on Muon.  It starts with the c_q
uniform rule.  Behaviour: ``nexttransformer/methods/gated_attention/__init__.py:29-67`` of the
reference.
"""
import torch
from torch import nn

from nexttransformer_b200.models import shell
from nexttransformer_b200.ops import plugins as plugin_ops
from nexttransformer_b200.models.shell import CausalSelfAttention, Linear

GRANULARITY = ("elementwise", "headwise")


class GatedAttention(CausalSelfAttention):
    def __init__(self, config, layer):
        super().__init__(config, layer)
        per_head = self.head_dim if config.option("granularity") == "elementwise" else 1
        self.gate_channels = per_head
        self.output_gate = Linear(config.n_embd, self.n_head * per_head, bias=False)

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        if kv_cache is not None:
            raise NotImplementedError("KV-cache decoding goes through nexttransformer_b200.inference")
        B, T, _ = x.shape
        q, k, v = self.project(x, ve, cos_sin)
        y = shell.sdpa(q, k, v, window_size[0])
        pre = self.output_gate(x).view(B, T, self.n_head, self.gate_channels)
        if plugin_ops.supported(y, pre):
            return self.c_proj(plugin_ops.gate_mul(y, pre).reshape(B, T, -1))  # one kernel each way
        return self.c_proj((y * torch.sigmoid(pre)).reshape(B, T, -1))


def mixer(config, layer):
    return GatedAttention(config, layer)


@torch.no_grad()
def init(model):
    bound = (3.0 / model.config.width) ** 0.5
    for block in model.transformer.h:
        nn.init.uniform_(block.attn.output_gate.weight, -bound, bound)


def check(config):
    if config.option("granularity") not in GRANULARITY:
        raise ValueError("granularity must be one of " + ", ".join(GRANULARITY))
