"""MSAR element kernels (``csrc/msar.cu``) as autograd functions.

``temporal(raw, taps)``: the four streams [B, T, 4, C] of a source (itself and causal depthwise
convolutions of widths 4, 8, 12); ``taps`` are the three [C, 1, w] parameters.  ``gate(streams, P,
alpha, bias)``: the depth-read mixture of ``methods/msar/ops.py``'s ``DepthRead``.  Both take bf16 or
fp32 activations, accumulate in fp32 and return gradients for every input; the token reductions
of the parameter gradients are fixed-order sums.
"""
import torch
from torch.autograd import Function

from nexttransformer_b200.ops._ext import ext


class _Temporal(Function):
    @staticmethod
    def forward(ctx, raw, t4, t8, t12):
        C = raw.shape[-1]
        taps = torch.cat([t.reshape(C, -1) for t in (t4, t8, t12)], 1).to(raw.dtype).float().contiguous()
        x = raw.contiguous()
        ctx.save_for_backward(x, taps)
        ctx.dtypes = (t4.dtype, t8.dtype, t12.dtype)
        return ext().msar_temporal_fwd(x, taps)

    @staticmethod
    def backward(ctx, dy):
        x, taps = ctx.saved_tensors
        dx, dtaps = ext().msar_temporal_bwd(x, taps, dy.contiguous().to(x.dtype))
        C = x.shape[-1]
        d4, d8, d12 = dtaps[:, :4], dtaps[:, 4:12], dtaps[:, 12:]
        return (dx, d4.reshape(C, 1, 4).to(ctx.dtypes[0]), d8.reshape(C, 1, 8).to(ctx.dtypes[1]),
                d12.reshape(C, 1, 12).to(ctx.dtypes[2]))


class _Gate(Function):
    @staticmethod
    def forward(ctx, streams, P, alpha, bias):
        shape = streams.shape
        s = streams.reshape(-1, 4, shape[-1]).contiguous()
        Pf, af, bf = P.float().contiguous(), alpha.float().contiguous(), bias.float().contiguous()
        out, zr = ext().msar_gate_fwd(s, Pf, af, bf)
        ctx.save_for_backward(s, Pf, af, bf, zr)
        ctx.meta = (shape, P.dtype, alpha.dtype, bias.dtype)
        return out.view(*shape[:-2], shape[-1])

    @staticmethod
    def backward(ctx, dout):
        s, Pf, af, bf, zr = ctx.saved_tensors
        shape, pd, ad, bd = ctx.meta
        ds, dP, da, db = ext().msar_gate_bwd(s, Pf, af, bf, zr, dout.reshape(-1, shape[-1]).contiguous().to(s.dtype))
        return ds.view(shape), dP.to(pd), da.to(ad), db.to(bd)


def supported(x):
    return x.is_cuda and x.dtype in (torch.bfloat16, torch.float32) and getattr(ext(), "msar_gate_fwd", None)


def temporal(raw, taps):
    return _Temporal.apply(raw, *taps)


def gate(streams, P, alpha, bias):
    return _Gate.apply(streams, P, alpha, bias)
