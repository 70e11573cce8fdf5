"""SimpleHC (Zhang et al., arXiv 2611.05984): hyper-connections with identity stream transitions and
gates shared across groups of sublayers.

The residual state is ``streams`` copies of the hidden vector (the embedding replicated; the final
streams are summed).  Sublayer j reads ``u_j = sum_n pre[j, n] X[n]`` and writes
``X[n] += post[j, n] o_j``; there is no stream mixing.  A group of ``group`` consecutive sublayers
computes all its read gates (``sigmoid``) and write gates (``2 sigmoid``) from the group-entry state,
``alpha * (RMSNorm(flatten X) W) + b``; inside the group a later sublayer sees an earlier sublayer's
output through the scalar correction ``pre_j . post_k`` instead of a materialised state, and the group
writes back once.  A trailing short group holds the remainder.  Init: ``W ~ N(0, init_std)``,
``alpha = alpha_init``, ``b = 0`` (read gates 0.5, write gates 1).
Behaviour: ``nexttransformer/methods/simplehc/__init__.py:25-86`` of the reference.
"""
import torch
from torch import nn

from nexttransformer_b200.models.lm import LanguageModel
from nexttransformer_b200.models.residual import coef
from nexttransformer_b200.models.shell import norm


def group_sizes(sublayers, group):
    full, rest = divmod(sublayers, group)
    return (group,) * full + ((rest,) if rest else ())


class GroupGates(nn.Module):
    def __init__(self, width, streams, size, init_std, alpha_init):
        super().__init__()
        self.streams, self.size, self.init_std, self.alpha_init = streams, size, init_std, alpha_init
        self.projection = nn.Parameter(torch.empty(streams * width, 2 * size * streams))
        self.alpha = nn.Parameter(torch.empty(2, size, 1))
        self.bias = nn.Parameter(torch.empty(2, size, streams))

    @torch.no_grad()
    def reset_parameters(self):
        nn.init.normal_(self.projection, std=self.init_std)
        self.alpha.fill_(self.alpha_init)
        self.bias.zero_()

    def forward(self, state):
        """Read and write gates ``[B, T, size, streams]`` of this group (coefficient precision)."""
        B, T, n, d = state.shape
        flat = norm(state.reshape(B, T, n * d))
        logits = coef(flat @ self.projection.to(flat.dtype)).unflatten(-1, (2, self.size, n))
        logits = self.alpha * logits + self.bias
        return torch.sigmoid(logits[..., 0, :, :]), 2 * torch.sigmoid(logits[..., 1, :, :])


class SimpleHC(LanguageModel):
    def __init__(self, config):
        super().__init__(config)
        self.residual_maps = nn.ModuleList(
            GroupGates(config.width, config.option("streams"), size, config.option("init_std"),
                       config.option("alpha_init"))
            for size in group_sizes(2 * config.n_layer, config.option("group")))

    def _sublayer(self, h, idx, k):
        if k % 2 == 0:
            return self._attention_branch(h, idx, k // 2)
        return self.transformer.h[k // 2].mlp(norm(h))

    def _ordinary_hidden(self, idx):
        n = self.config.option("streams")
        x = self._embed(idx)
        state = x[:, :, None].expand(-1, -1, n, -1)
        k = 0
        for gates in self.residual_maps:
            pre, post = gates(state)
            reads = torch.einsum("btjn,btnd->btjd", pre.to(state.dtype), state)
            outs = []
            for j in range(gates.size):
                h = reads[:, :, j]
                if j:
                    corr = (pre[:, :, j, None] * post[:, :, :j]).sum(-1).to(h.dtype)
                    for i, o in enumerate(outs):
                        h = h + corr[..., i, None] * o
                outs.append(self._sublayer(h, idx, k))
                self._record("residual_map", sublayer=k, streams=n, tokens=idx.numel())
                k += 1
            state = state + torch.einsum("btjn,btjd->btnd", post.to(state.dtype), torch.stack(outs, 2))
        return state.sum(2), None


model = SimpleHC
frozen = ("resid_lambdas", "x0_lambdas", "backout_lambda")


def check(config):
    for name in ("streams", "group"):
        v = config.option(name)
        if not (type(v) is int and v >= 1):
            raise ValueError(f"{name} must be a positive integer")
    for name in ("init_std", "alpha_init"):
        v = config.option(name)
        if type(v) not in (int, float) or not v > 0:
            raise ValueError(f"{name} must be positive")
