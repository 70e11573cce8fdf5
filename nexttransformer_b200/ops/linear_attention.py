"""CUDA entry points of the linear-attention mixers (DeltaNet / GDN / KDA).

* ``causal_conv_silu(x, w)``: the short causal depthwise convolution (width 4) with SiLU on
  ``[B, T, C]``, one sm_100a kernel each way (``csrc/linear_attn.cu``); the convolution output
  is kept for the backward.
* ``gated_rms_norm(y, gate, gain)``: ``RMSNorm(y) * gain * SiLU(gate)`` over the head dimension,
  one kernel each way.
* ``delta_chunk_cuda(...)``: the chunked (gated) delta rule.  It runs the chunk form of
  ``models/linear.py`` with fp32 matrix products on the GPU (q/k L2 normalisation for GDN first)
  until the fused chunk kernel replaces it.
"""
import torch
from torch.autograd import Function
import torch.nn.functional as F

from nexttransformer_b200.ops._ext import ext


class _ConvSiLU(Function):
    @staticmethod
    def forward(ctx, x, w):
        x = x.contiguous()
        B, T, C = x.shape
        wf = w.reshape(C, -1).float().contiguous()
        y = torch.empty_like(x)
        pre = torch.empty_like(x)
        ext().conv_silu_fwd(x, wf, y, pre)
        ctx.save_for_backward(x, pre, wf)
        ctx.wshape, ctx.wdtype = w.shape, w.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, pre, wf = ctx.saved_tensors
        dx = torch.empty_like(x)
        dw = torch.zeros_like(wf)
        ext().conv_silu_bwd(x, pre, dy.contiguous().to(x.dtype), wf, dx, dw)
        return dx, dw.reshape(ctx.wshape).to(ctx.wdtype)


def causal_conv_silu(x, w):
    if x.dtype != torch.bfloat16 or x.shape[-1] % 8:
        y = F.conv1d(F.pad(x.transpose(1, 2), (w.shape[-1] - 1, 0)), w.to(x.dtype), groups=x.shape[-1])
        return F.silu(y.transpose(1, 2))
    return _ConvSiLU.apply(x, w)


class _GatedRMSNorm(Function):
    @staticmethod
    def forward(ctx, y, gate, gain):
        y, gate = y.contiguous(), gate.contiguous()
        D = y.shape[-1]
        g32 = gain.float().contiguous()
        out = torch.empty_like(y)
        rstd = torch.empty(y.numel() // D, device=y.device, dtype=torch.float32)
        ext().gated_rmsnorm_fwd(y, gate, g32, out, rstd)
        ctx.save_for_backward(y, gate, g32, rstd)
        ctx.gdtype = gain.dtype
        return out

    @staticmethod
    def backward(ctx, dout):
        y, gate, g32, rstd = ctx.saved_tensors
        dy, dg = torch.empty_like(y), torch.empty_like(gate)
        dgain = torch.zeros_like(g32)
        ext().gated_rmsnorm_bwd(y, gate, g32, rstd, dout.contiguous().to(y.dtype), dy, dg, dgain)
        return dy, dg, dgain.to(ctx.gdtype)


def gated_rms_norm(y, gate, gain):
    if y.dtype != torch.bfloat16 or gate.dtype != torch.bfloat16 or y.shape[-1] not in (64, 128):
        from nexttransformer_b200.models.linear import gated_rms_norm as reference
        return reference(y, gate, gain)
    return _GatedRMSNorm.apply(y, gate, gain)


def delta_chunk_cuda(q, k, v, *, kind, g=None, beta=None, chunk, qk_l2norm_scale=None):
    from nexttransformer_b200.models.linear import chunk_scan
    dt = q.dtype
    if qk_l2norm_scale is not None:
        q, k = F.normalize(q.float(), dim=-1) * qk_l2norm_scale, F.normalize(k.float(), dim=-1)
    out = chunk_scan(q.float(), k.float(), v.float(), kind=kind, g=None if g is None else g.float(),
                     beta=None if beta is None else beta.float(), chunk=chunk)
    return out.to(dt)
