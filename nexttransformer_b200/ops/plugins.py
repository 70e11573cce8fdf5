"""CUDA entry points of the attention plugins' elementwise heads (``csrc/plugin_ops.cu``) and the
Canon layer (``csrc/linear_attn.cu``, the convolution kernels without the activation).

* ``gate_mul(y, g)``: ``y * sigmoid(g)`` with ``g`` per head channel or per head (gated attention);
* ``exclusive_projection(y, v)``: ``y - <y, u> u`` with ``u = v / max(|v|, 1e-12)`` of each query head's
  KV head (XSA), given the value heads un-repeated;
* ``canon(x, w)``: ``x + causal depthwise conv(x)`` (Canon layer).

Each takes bf16 CUDA tensors with heads of 128 channels (channels a multiple of 8 for ``canon``);
``supported`` says whether the kernels take a call, and callers keep their PyTorch expression
otherwise.  Each op is one kernel per direction, fp32 inside.
"""
import torch
from torch.autograd import Function

from nexttransformer_b200.ops._ext import ext


def supported(*tensors, head=True):
    return all(t.is_cuda and t.dtype == torch.bfloat16 for t in tensors) and (
        not head or tensors[0].shape[-1] == 128)


class _GateMul(Function):
    @staticmethod
    def forward(ctx, y, g):
        B, T, H, D = y.shape
        y3, g3 = y.reshape(B * T, H, D).contiguous(), g.reshape(B * T, H, -1).contiguous()
        z = torch.empty_like(y3)
        ext().gate_mul_fwd(y3, g3, z)
        ctx.save_for_backward(y3, g3)
        ctx.shape = (y.shape, g.shape)
        return z.view(y.shape)

    @staticmethod
    def backward(ctx, dz):
        y3, g3 = ctx.saved_tensors
        dy, dg = torch.empty_like(y3), torch.empty_like(g3)
        ext().gate_mul_bwd(y3, g3, dz.reshape(y3.shape).to(y3.dtype).contiguous(), dy, dg)
        return dy.view(ctx.shape[0]), dg.view(ctx.shape[1])


def gate_mul(y, g):
    """y [B, T, H, 128] * sigmoid(g), g [B, T, H, 128] or [B, T, H, 1]."""
    return _GateMul.apply(y, g)


class _Exclusive(Function):
    @staticmethod
    def forward(ctx, y, v):
        B, T, H, D = y.shape
        y3, v3 = y.reshape(B * T, H, D).contiguous(), v.reshape(B * T, v.shape[2], D).contiguous()
        z = torch.empty_like(y3)
        ext().xsa_fwd(y3, v3, z)
        ctx.save_for_backward(y3, v3)
        ctx.shape = (y.shape, v.shape)
        return z.view(y.shape)

    @staticmethod
    def backward(ctx, dz):
        y3, v3 = ctx.saved_tensors
        dy, dv = torch.empty_like(y3), torch.empty_like(v3)
        ext().xsa_bwd(y3, v3, dz.reshape(y3.shape).to(y3.dtype).contiguous(), dy, dv)
        return dy.view(ctx.shape[0]), dv.view(ctx.shape[1])


def exclusive_projection(y, v):
    """y [B, T, H, 128] minus its component along the unit value of each head's KV head (v [B, T, Hk, 128])."""
    return _Exclusive.apply(y, v)


class _Canon(Function):
    @staticmethod
    def forward(ctx, x, w):
        x = x.contiguous()
        C = x.shape[-1]
        wf = w.reshape(C, -1).float().contiguous()
        y = torch.empty_like(x)
        ext().canon_conv_fwd(x, wf, y)
        ctx.save_for_backward(x, wf)
        ctx.wshape, ctx.wdtype = w.shape, w.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, wf = ctx.saved_tensors
        dx = torch.empty_like(x)
        dw = torch.zeros_like(wf)
        ext().canon_conv_bwd(x, dy.contiguous().to(x.dtype), wf, dx, dw)
        return dx, dw.reshape(ctx.wshape).to(ctx.wdtype)


def canon(x, w):
    """x [B, T, C] + causal depthwise convolution with taps w [C, 1, K] (K <= 4)."""
    return _Canon.apply(x, w)
