"""MSAR arithmetic on ``[batch, time, stream, hidden]`` tensors.

* ``TemporalAugmentation``: a source becomes four streams - the raw source and three causal
  depthwise convolutions of it with kernel widths 4, 8 and 12 (zero-initialised taps, so the
  augmented streams start at zero).
* ``DepthRead``: four pseudo-queries (one per stream) read a softmax mixture over depth sources;
  the four read streams are then combined by per-stream sigmoid gates computed from the flattened
  streams (``alpha * (flat W) / rms(flat) + b``; all-zero rows use rms 1).
* ``completed_read`` reads the completed sources of a block for all of the block's consumers at
  once and returns each read with its log-sum-exp; ``merge_partial`` folds the current partial
  source in with a two-way softmax over (completed log-sum-exp, partial logit).
Source keys are RMS-normalised (eps 1e-6) in at least fp32.
Behaviour: ``nexttransformer/methods/msar/ops.py:17-100`` of the reference.
"""
import torch
from torch import nn
import torch.nn.functional as F

WIDTHS = (4, 8, 12)


def _coef(x):
    return x.to(torch.promote_types(x.dtype, torch.float32))


class TemporalAugmentation(nn.Module):
    def __init__(self, width):
        super().__init__()
        self.taps = nn.ParameterList(nn.Parameter(torch.empty(width, 1, w)) for w in WIDTHS)
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self):
        for t in self.taps:
            nn.init.zeros_(t)

    def forward(self, raw):
        from nexttransformer_b200.ops import msar as K
        if K.supported(raw) and raw.dim() == 3:
            return K.temporal(raw, tuple(self.taps))   # one kernel per direction (csrc/msar.cu)
        ch = raw.transpose(1, 2)
        out = [raw]
        for t in self.taps:
            y = F.conv1d(F.pad(ch, (t.shape[-1] - 1, 0)), t.to(raw.dtype), groups=raw.shape[-1])
            out.append(y.transpose(1, 2))
        return torch.stack(out, dim=2)


class DepthRead(nn.Module):
    def __init__(self, width):
        super().__init__()
        self.query = nn.Parameter(torch.empty(4, width))
        self.proj_pre = nn.Parameter(torch.empty(4 * width, 4))
        self.alpha_pre = nn.Parameter(torch.empty(1))
        self.bias_pre = nn.Parameter(torch.empty(4))
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self):
        nn.init.zeros_(self.query)
        nn.init.normal_(self.proj_pre, std=0.006)
        nn.init.constant_(self.alpha_pre, 0.01)
        nn.init.zeros_(self.bias_pre)

    def forward(self, streams):
        from nexttransformer_b200.ops import msar as K
        if K.supported(streams) and streams.shape[-2] == 4:
            return K.gate(streams, self.proj_pre, self.alpha_pre, self.bias_pre)
        flat = streams.flatten(-2)
        ms = flat.square().mean(-1, keepdim=True)
        ms = torch.where(ms > 0, ms, torch.ones_like(ms))   # before rsqrt: no inf/NaN gradient at zero
        logits = (flat @ self.proj_pre.to(flat.dtype)) * ms.rsqrt()
        gate = torch.sigmoid(logits * self.alpha_pre.to(flat.dtype) + self.bias_pre.to(flat.dtype))
        return (gate.unsqueeze(-1) * streams).sum(-2)


def source_key(source):
    k = _coef(source)
    return k * torch.rsqrt(k.square().mean(-1, keepdim=True) + 1e-6)


def completed_read(queries, sources, keys):
    """queries ``[Q, 4, C]``; sources/keys lists of ``[B, T, 4, C]`` -> (reads ``[Q, B, T, 4, C]``,
    log-sum-exp ``[Q, B, T, 4]``)."""
    kstack = torch.stack(keys)
    with torch.autocast(device_type=kstack.device.type, enabled=False):
        logits = torch.einsum("qnk,cbtnk->qcbtn", queries.to(kstack.dtype), kstack)
    top = logits.amax(1, keepdim=True).detach()
    e = (logits - top).exp()
    z = e.sum(1, keepdim=True)
    w = (e / z).to(sources[0].dtype)
    lse = (top + z.log()).squeeze(1)
    read = w[:, 0].unsqueeze(-1) * sources[0]
    for i, s in enumerate(sources[1:], 1):
        read = read + w[:, i].unsqueeze(-1) * s
    return read, lse


def merge_partial(completed, completed_lse, partial, partial_key, query):
    with torch.autocast(device_type=partial_key.device.type, enabled=False):
        logit = torch.einsum("nk,btnk->btn", query.to(partial_key.dtype), partial_key)
    w = torch.stack((completed_lse, logit)).softmax(0).to(partial.dtype)
    return w[0].unsqueeze(-1) * completed + w[1].unsqueeze(-1) * partial
