"""Block AttnRes with Canon layers at positions A-D (shared by ``attnres_full_canon_abcd``; this
package declares no method of its own).

The trunk is Block AttnRes: every sublayer reads a softmax mixture over depth sources (embedding,
completed group sums, current partial sum) through its own zero-initialised pseudo-query.  Canon
layers - a causal depthwise convolution over the last four positions added to its input, with
zero-initialised weights so each starts as the identity - sit on every sublayer input after the
depth read (A, C), on q/k/v before RoPE and QK-norm (B) and on the MLP hidden activation before the
squared ReLU (D).  Behaviour: ``nexttransformer/methods/attnres_canon_abcd/__init__.py:25-150``.
"""
import torch
from torch import nn
import torch.nn.functional as F

from nexttransformer_b200.models import shell
from nexttransformer_b200.models.lm import LanguageModel
from nexttransformer_b200.models.residual import depth_attention
from nexttransformer_b200.models.shell import CausalSelfAttention, Linear, apply_rotary_emb, norm


class Canon(nn.Module):
    def __init__(self, width, size=4):
        super().__init__()
        self.size = size
        self.weight = nn.Parameter(torch.empty(width, 1, size))

    def forward(self, x):
        """``x + causal_depthwise_conv(x)`` over ``[B, T, C]``."""
        y = F.conv1d(F.pad(x.transpose(1, 2), (self.size - 1, 0)), self.weight.to(x.dtype), groups=x.shape[-1])
        return x + y.transpose(1, 2)


class CanonAttention(CausalSelfAttention):
    def __init__(self, config, layer):
        super().__init__(config, layer)
        self.canon_qkv = nn.ModuleList(Canon(config.n_embd) for _ in range(3))

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        if kv_cache is not None:
            raise NotImplementedError("training and full-sequence evaluation only")
        B, T, _ = x.shape
        q, k, v = (c(t) for c, t in zip(self.canon_qkv, (self.c_q(x), self.c_k(x), self.c_v(x))))
        q = q.view(B, T, self.n_head, self.head_dim)
        k = k.view(B, T, self.n_kv_head, self.head_dim)
        v = v.view(B, T, self.n_kv_head, self.head_dim)
        if ve is not None and self.ve_gate is not None:
            gate = 3 * torch.sigmoid(self.ve_gate(x[..., :self.ve_gate_channels]))
            v = v + gate.unsqueeze(-1) * ve.view(B, T, self.n_kv_head, self.head_dim)
        cos, sin = cos_sin
        q, k = apply_rotary_emb(q, cos, sin), apply_rotary_emb(k, cos, sin)
        q, k = norm(q) * 1.2, norm(k) * 1.2
        y = shell.sdpa(q, k, v, window_size[0])
        return self.c_proj(y.reshape(B, T, -1))


class CanonMLP(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.c_fc = Linear(config.width, config.mlp_width, bias=False)
        self.c_proj = Linear(config.mlp_width, config.width, bias=False)
        self.canon = Canon(config.mlp_width)

    def forward(self, x):
        return self.c_proj(F.relu(self.canon(self.c_fc(x))).square())


def group_starts(layers, groups):
    """First layer of each AttnRes group: sizes as equal as possible, the larger groups first."""
    base, extra = divmod(layers, groups)
    starts, at = [], 0
    for g in range(groups):
        starts.append(at)
        at += base + (1 if g < extra else 0)
    return tuple(starts)


def _skip_reset():
    """Embedding tables are drawn by ``init_weights``; an extra reset would shift the RNG stream."""


class CanonAttnRes(LanguageModel):
    @staticmethod
    def groups(config):
        return config.option("groups")

    def __init__(self, config):
        super().__init__(config)
        self.group_starts = group_starts(config.n_layer, self.groups(config))
        self.depth_queries = nn.Parameter(torch.empty(2 * config.n_layer + 1, config.width))
        self.canon = nn.ModuleList(Canon(config.width) for _ in range(2 * config.n_layer))
        for m in self.modules():
            if isinstance(m, nn.Embedding):
                m.reset_parameters = _skip_reset

    def _ordinary_hidden(self, idx):
        c = self.config
        x = self._embed(idx)
        starts = set(self.group_starts)
        blocks, keys, partial = [], [], x
        for k in range(2 * c.n_layer):
            key = norm(partial)
            h = depth_attention(self.depth_queries[k], blocks + [partial], keys + [key])
            self._record("depth_read", sublayer=k, sources=len(blocks) + 1, tokens=idx.numel())
            if k % 2 == 0 and k // 2 in starts:
                blocks.append(partial)
                keys.append(key)
                partial = None
            h = self.canon[k](h)
            if k % 2 == 0:
                out = self._attention_branch(h, idx, k // 2)
            else:
                out = self.transformer.h[k // 2].mlp(norm(h))
            partial = out if partial is None else partial + out
        h = depth_attention(self.depth_queries[-1], blocks + [partial], keys + [norm(partial)])
        self._record("depth_read", sublayer=2 * c.n_layer, sources=len(blocks) + 1, tokens=idx.numel())
        return h, None


def mixer(config, layer):
    return CanonAttention(config, layer)


def ffn(config, layer):
    return CanonMLP(config)


model = CanonAttnRes
frozen = ("resid_lambdas", "x0_lambdas", "backout_lambda")


@torch.no_grad()
def init(model):
    for m in model.modules():
        if isinstance(m, Canon):
            nn.init.zeros_(m.weight)


def check(config):
    g = config.option("groups")
    if not (type(g) is int and 1 <= g <= config.n_layer):
        raise ValueError(f"groups must be an integer from 1 to the layer count ({config.n_layer})")
