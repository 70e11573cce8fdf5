"""Residual-stream organisations: Hyper-Connections, manifold-constrained HC and Block AttnRes.

Semantics follow ``nexttransformer/models/residual.py`` of the reference: every attention or
FFN sublayer is one residual layer; HC keeps n streams mixed by static + tanh-gated dynamic
maps; mHC projects the flattened streams to pre / post / residual logits with a Sinkhorn-Knopp
(log-domain) doubly-stochastic residual map; AttnRes reads a softmax over depth sources with
zero-initialised pseudo-queries.  Coefficients are computed in at least fp32.
"""
import torch
from torch import nn

from nexttransformer_b200.models.shell import norm


def coef(x):
    return x.to(torch.promote_types(x.dtype, torch.float32))


class _SinkhornKernel(torch.autograd.Function):
    """The whole Sinkhorn-Knopp projection in one sm_100a kernel per direction (csrc/residual.cu)."""

    @staticmethod
    def forward(ctx, logits, iterations):
        from nexttransformer_b200.ops._ext import ext
        z = logits.float().contiguous()
        out = torch.empty_like(z)
        ext().sinkhorn_fwd(z, out, iterations)
        ctx.save_for_backward(z)
        ctx.iterations, ctx.dtype = iterations, logits.dtype
        return out

    @staticmethod
    def backward(ctx, dout):
        from nexttransformer_b200.ops._ext import ext
        (z,) = ctx.saved_tensors
        dz = torch.empty_like(z)
        ext().sinkhorn_bwd(z, dout.float().contiguous(), dz, ctx.iterations)
        return dz.to(ctx.dtype), None


def sinkhorn_knopp(logits, iterations):
    """Alternate column / row normalisation of exp(logits) kept in the log domain."""
    if logits.is_cuda and logits.shape[-1] == logits.shape[-2] == 4 and iterations <= 32 \
            and logits.dtype in (torch.float32, torch.bfloat16) and type(logits) is torch.Tensor:
        return _SinkhornKernel.apply(logits, iterations)

    def lognorm(z, dim):
        z = z - z.amax(dim, keepdim=True).detach()
        return z - z.exp().sum(dim, keepdim=True).log()
    z = logits
    for _ in range(iterations):
        z = lognorm(lognorm(z, -2), -1)
    return z.exp()


class HyperConnection(nn.Module):
    """Dynamic hyper-connection around one sublayer; streams are [B, T, n, D]."""

    def __init__(self, width, streams, index, gate_init):
        super().__init__()
        self.streams, self.index, self.gate_init = streams, index, gate_init
        self.static_alpha = nn.Parameter(torch.empty(streams, streams + 1))
        self.static_beta = nn.Parameter(torch.empty(streams))
        self.dynamic_alpha = nn.Parameter(torch.empty(width, streams + 1))
        self.dynamic_beta = nn.Parameter(torch.empty(width, 1))
        self.alpha_scale = nn.Parameter(torch.empty(1))
        self.beta_scale = nn.Parameter(torch.empty(1))

    @torch.no_grad()
    def reset_parameters(self):
        """Start equivalent to pre-norm: read stream (index mod n), identity residual, unit writes."""
        n = self.streams
        self.static_alpha.zero_()
        self.static_alpha[self.index % n, 0] = 1.
        self.static_alpha[:, 1:] = torch.eye(n, device=self.static_alpha.device)
        self.static_beta.fill_(1.)
        self.dynamic_alpha.zero_()
        self.dynamic_beta.zero_()
        self.alpha_scale.fill_(self.gate_init)
        self.beta_scale.fill_(self.gate_init)

    def read(self, streams):
        h = norm(streams)
        alpha = self.alpha_scale * torch.tanh(coef(h @ self.dynamic_alpha.to(h.dtype))) + self.static_alpha
        beta = self.beta_scale * torch.tanh(coef(h @ self.dynamic_beta.to(h.dtype)).squeeze(-1)) + self.static_beta
        mixed = torch.einsum("btjk,btjd->btkd", alpha.to(streams.dtype), streams)
        return mixed[:, :, 0], mixed[:, :, 1:], beta

    @staticmethod
    def write(residual, out, weights):
        return residual + weights.to(out.dtype)[..., None] * out[:, :, None]


class ManifoldHyperConnection(nn.Module):
    """mHC: one projection of the normalised flattened streams gives pre (sigmoid), post
    (2 sigmoid) and residual (Sinkhorn-Knopp) maps."""

    def __init__(self, width, streams, index, gate_init, iterations):
        super().__init__()
        self.streams, self.index, self.gate_init, self.iterations = streams, index, gate_init, iterations
        n = streams
        self.projection = nn.Parameter(torch.empty(n * width, n * n + 2 * n))
        self.bias = nn.Parameter(torch.empty(n * n + 2 * n))
        self.gates = nn.Parameter(torch.empty(3))

    @torch.no_grad()
    def reset_parameters(self):
        n = self.streams
        self.projection.zero_()
        self.bias.zero_()
        self.bias[self.index % n] = 1.
        self.bias[n:2 * n] = 1.
        self.bias[2 * n:] = torch.eye(n, device=self.bias.device).flatten()
        self.gates.fill_(self.gate_init)

    def maps(self, streams):
        B, T, n, d = streams.shape
        flat = norm(streams.reshape(B, T, n * d))
        logits = coef(flat @ self.projection.to(flat.dtype))
        pre, post, res = logits.split((n, n, n * n), -1)
        bp, bq, br = self.bias.split((n, n, n * n))
        pre = torch.sigmoid(self.gates[0] * pre + bp)
        post = 2 * torch.sigmoid(self.gates[1] * post + bq)
        res = sinkhorn_knopp((self.gates[2] * res + br).unflatten(-1, (n, n)), self.iterations)
        return pre, post, res

    def read(self, streams):
        pre, post, res = self.maps(streams)
        x = torch.einsum("btj,btjd->btd", pre.to(streams.dtype), streams)
        mixed = torch.einsum("btij,btjd->btid", res.to(streams.dtype), streams)
        return x, mixed, post

    write = staticmethod(HyperConnection.write)


def depth_attention(query, sources, keys):
    """Softmax over depth sources: keys are the normalised sources, query a learned pseudo-query."""
    q = query.to(keys[0].dtype)[:, None]
    logits = coef(torch.stack([(k @ q).squeeze(-1) for k in keys]))
    w = logits.softmax(0).to(sources[0].dtype)
    out = w[0, ..., None] * sources[0]
    for wi, s in zip(w[1:], sources[1:]):
        out = out + wi[..., None] * s
    return out
