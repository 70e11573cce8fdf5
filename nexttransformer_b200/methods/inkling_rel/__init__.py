"""Inkling REL: content-dependent relative-position logits in place of RoPE.

Per query position i and head h, ``r = x W_r`` (``d_rel`` values) and the logit of key j <= i gains
``bias(i, j) = sum_a r(i, h, a) E[a, i - j]``; ``E`` (``[d_rel, rel_extent]``) is one table per layer
shared by the heads, and distance 0 (the token itself) is included.  The bias is added after the
``1/sqrt(head_dim)`` content scaling; QK RMS-norm with gain 1.2, value embeddings and the output
projection are the shell's; there is no RoPE.  ``W_r`` and ``E`` start as ``N(0, rel_init_std)``.
Behaviour: ``nexttransformer/methods/inkling_rel/__init__.py:21-78`` and ``reference.py:10-47``.
"""
import math

import torch
from torch import nn

from nexttransformer_b200.methods.inkling_rel.reference import relative_attention_edges
from nexttransformer_b200.models.shell import CausalSelfAttention, Linear, norm


class RelativeDistanceTable(nn.Module):
    def __init__(self, d_rel, extent, std):
        super().__init__()
        self.std = std
        self.proj = nn.Parameter(torch.empty(d_rel, extent))
        self.reset_parameters()

    def reset_parameters(self):
        nn.init.normal_(self.proj, std=self.std)


class RelativeSelfAttention(CausalSelfAttention):
    def __init__(self, config, layer):
        super().__init__(config, layer)
        self.d_rel = config.option("d_rel")
        self.rel_extent = config.option("rel_extent")
        self.rel_init_std = config.option("rel_init_std")
        self.c_r = Linear(config.n_embd, self.n_head * self.d_rel, bias=False)
        self.rel_logits_proj = RelativeDistanceTable(self.d_rel, self.rel_extent, self.rel_init_std)

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        if kv_cache is not None:
            raise ValueError("REL supports full-sequence training and evaluation only")
        B, T, _ = x.shape
        if T > self.rel_extent:
            raise ValueError("the relative table does not cover this context")
        q = self.c_q(x).view(B, T, self.n_head, self.head_dim)
        k = self.c_k(x).view(B, T, self.n_kv_head, self.head_dim)
        v = self.c_v(x).view(B, T, self.n_kv_head, self.head_dim)
        if ve is not None and self.ve_gate is not None:
            gate = 3 * torch.sigmoid(self.ve_gate(x[..., :self.ve_gate_channels]))
            v = v + gate.unsqueeze(-1) * ve.view_as(v)
        q, k = norm(q) * 1.2, norm(k) * 1.2
        r = self.c_r(x).view(B, T, self.n_head, self.d_rel)
        table = self.rel_logits_proj.proj.to(r.dtype)
        if q.is_cuda and q.dtype == torch.bfloat16 and self.head_dim == 128:
            # the block-sparse sm_100a kernels over dense causal lists, the bias read from r @ E
            from nexttransformer_b200.ops.sparse_attention import block_sparse_attention, causal_lists
            lists, masks = causal_lists(B, T, q.device)
            rel = (r.float() @ table.float()).transpose(1, 2).contiguous()       # [B, H, T, extent]
            y = block_sparse_attention(q, k, v, lists, masks, self.head_dim ** -0.5, rel)
        elif q.is_cuda:
            from nexttransformer_b200.methods.inkling_rel.dense import relative_attention_dense
            y = relative_attention_dense(q, k, v, r, table)
        else:
            y = relative_attention_edges(q, k, v, r, table)
        return self.c_proj(y.reshape(B, T, -1))


def mixer(config, layer):
    return RelativeSelfAttention(config, layer)


@torch.no_grad()
def init(model):
    for block in model.transformer.h:
        nn.init.normal_(block.attn.c_r.weight, std=block.attn.rel_init_std)
        block.attn.rel_logits_proj.reset_parameters()


def check(config):
    if config.window_pattern != "L":
        raise ValueError("REL needs full causal attention in every layer")
    if type(config.option("d_rel")) is not int or config.option("d_rel") <= 0:
        raise ValueError("d_rel must be a positive integer")
    if type(config.option("rel_extent")) is not int or config.option("rel_extent") < config.sequence_len:
        raise ValueError("rel_extent must cover every causal distance in the context")
    std = config.option("rel_init_std")
    if not math.isfinite(std) or std <= 0:
        raise ValueError("rel_init_std must be positive")
