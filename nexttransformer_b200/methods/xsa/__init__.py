"""Exclusive self attention (Zhai, arXiv 2603.09078): before ``c_proj`` each head's output loses
its component along the head's own (effective) value vector, ``z = y - <y, u> u`` with
``u = v / max(|v|, 1e-12)``.  Gradients flow through both y and v; 16-bit inputs are projected in
fp32.  The value is the one attention used (value embedding mixed in); with GQA each query head
uses its KV head's value.  Behaviour: ``nexttransformer/methods/xsa/__init__.py:19-58``.
"""
import torch
import torch.nn.functional as F

from nexttransformer_b200.models import shell
from nexttransformer_b200.ops import plugins as plugin_ops
from nexttransformer_b200.models.shell import CausalSelfAttention


def exclusive_projection(y, v):
    out_dtype = y.dtype
    if out_dtype in (torch.float16, torch.bfloat16):
        y, v = y.float(), v.float()
    u = F.normalize(v, dim=-1, eps=1e-12)
    return (y - (y * u).sum(-1, keepdim=True) * u).to(out_dtype)


class ExclusiveSelfAttention(CausalSelfAttention):
    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        if kv_cache is not None:
            raise NotImplementedError("KV-cache decoding goes through nexttransformer_b200.inference")
        B, T, _ = x.shape
        q, k, v = self.project(x, ve, cos_sin)
        y = shell.sdpa(q, k, v, window_size[0])
        if plugin_ops.supported(y, v):
            # one kernel each way; the KV head of each query head is read in place (no repeat)
            return self.c_proj(plugin_ops.exclusive_projection(y, v).reshape(B, T, -1))
        if self.n_head != self.n_kv_head:
            v = v.repeat_interleave(self.n_head // self.n_kv_head, dim=2)
        return self.c_proj(exclusive_projection(y, v).reshape(B, T, -1))


def mixer(config, layer):
    return ExclusiveSelfAttention(config, layer)


def check(config):
    if config.window_pattern != "L":
        raise ValueError("XSA needs full causal attention in every layer (window_pattern L)")
