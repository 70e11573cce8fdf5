"""Kernel autograd functions shared by every model family on CUDA.

These are the building blocks of the generic sm_100a execution path: any ``Linear`` whose
weight has been given a bf16 shadow and an fp32 gradient slot (``models.fused_dense.FusedState``)
runs its forward, input gradient and weight gradient on the tcgen05 GEMM engine
(``csrc/gemm_sm100.cu``), and the RMSNorms around every mixer / FFN run on the row kernels of
``csrc/elementwise.cu``.  The reference runs the same projections through ``F.linear`` (cuBLAS)
and ``F.rms_norm`` (``nexttransformer/models/backbone.py:45-50``, ``models/lm.py:198-231``).

Parameter gradients never pass through autograd here: the weight-gradient GEMM writes the first
contribution of an update into ``weight.main_grad`` and accumulates every later one (the slot's
``fresh`` flag), so repeated uses of one weight (several micro-batches, looped blocks) sum in
fp32 inside the GEMM epilogue.
"""
import torch
from torch.autograd import Function

from nexttransformer_b200.ops import gemm as G
from nexttransformer_b200.ops._ext import ext

# Weights narrower than this, or with sizes that are not multiples of it, stay on F.linear
# (router columns, value-embedding gates, smear gate): too small to fill a 128-row tile.
MIN_KERNEL_DIM = 64


def linear_eligible(weight):
    """True when a Linear weight [out, in] can run on the GEMM engine."""
    out_f, in_f = weight.shape
    return (out_f % MIN_KERNEL_DIM == 0 and in_f % MIN_KERNEL_DIM == 0 and out_f >= MIN_KERNEL_DIM
            and in_f >= MIN_KERNEL_DIM)


def norm_eligible(x):
    """RMSNorm row kernels: bf16 rows of at most 2048 features, a multiple of 8."""
    d = x.shape[-1]
    return x.is_cuda and x.dtype == torch.bfloat16 and d % 8 == 0 and d <= 2048


class KernelLinear(Function):
    """y = x W^T with the bf16 shadow ``lin._w``; dW accumulates into ``lin.weight.main_grad``."""

    @staticmethod
    def forward(ctx, x, weight, lin):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y = G.linear(x2, lin._w)
        ctx.save_for_backward(x2)
        ctx.lin, ctx.shape = lin, shape
        return y.view(*shape[:-1], y.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        (x2,) = ctx.saved_tensors
        lin = ctx.lin
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        if dy2.dtype != torch.bfloat16:
            dy2 = dy2.to(torch.bfloat16)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = G.dgrad(dy2, lin._w).view(ctx.shape)
        if ctx.needs_input_grad[1]:
            buf, acc = lin._g.take()
            G.wgrad(dy2, x2, buf, accumulate=acc)
        return dx, None, None


def kernel_linear(x, lin):
    return KernelLinear.apply(x, lin.weight, lin)


class NormFn(Function):
    """h = RMSNorm(x) over the last dimension (no weight), bf16 in and out."""

    @staticmethod
    def forward(ctx, x):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        h = torch.empty_like(x2)
        ext().mix_norm_fwd(x2, None, None, None, h, None, 1.0)
        ctx.save_for_backward(x2)
        ctx.shape = shape
        return h.view(shape)

    @staticmethod
    def backward(ctx, dh):
        (x2,) = ctx.saved_tensors
        dx = torch.empty_like(x2)
        ext().norm_bwd(x2, dh.reshape(x2.shape).contiguous().to(torch.bfloat16), None, dx)
        return dx.view(ctx.shape)


def rms_norm(x):
    return NormFn.apply(x)


class MixNormFn(Function):
    """xm = a x + b x0 and h = RMSNorm(xm) for layer ``layer`` of a shell (``ab = (a, b)``).

    The gradient of x0 accumulates in ``scratch.dx0`` (added to the embedding's gradient once, at
    the embedding) and the two scalars' gradients land in the shell's ``resid_lambdas`` /
    ``x0_lambdas`` ``main_grad``."""

    @staticmethod
    def forward(ctx, x, x0, ab, model, scratch, layer):
        xm = torch.empty_like(x)
        h = torch.empty_like(x)
        ext().mix_norm_fwd(x, x0, ab, xm, h, None, 1.0)
        ctx.save_for_backward(x, x0, ab, xm)
        ctx.model, ctx.scratch, ctx.layer = model, scratch, layer
        return xm, h

    @staticmethod
    def backward(ctx, dxm, dh):
        x, x0, ab, xm = ctx.saved_tensors
        model, layer = ctx.model, ctx.layer
        if dxm is None:
            dxm = torch.zeros_like(x)
        if dh is None:
            dh = torch.zeros_like(x)
        dx = torch.empty_like(x)
        part = torch.empty(x.shape[0], 2, device=x.device, dtype=torch.float32)
        ext().mix_norm_bwd(x, x0, xm, dh.contiguous(), dxm.contiguous(), ab, dx, ctx.scratch.dx0, part)
        dab = part.sum(0)
        model.resid_lambdas.main_grad[layer:layer + 1] += dab[0:1]
        model.x0_lambdas.main_grad[layer:layer + 1] += dab[1:2]
        # the layer's value-embedding rows are scattered by a separate node the engine may run
        # later, so only the layer's own weights are final here
        model._fused.grads_ready(layer, tables=False)
        return dx, None, None, None, None, None


class TableLookupFn(Function):
    """rows = table[idx] (bf16); the gradient scatters (fp32 atomics) into ``table.main_grad``."""

    @staticmethod
    def forward(ctx, idx, table):
        out = table.detach().index_select(0, idx)
        ctx.save_for_backward(idx)
        ctx.table = table
        return out

    @staticmethod
    def backward(ctx, dout):
        (idx,) = ctx.saved_tensors
        ext().embed_scatter(dout.contiguous(), idx, ctx.table.main_grad)
        return None, None


def table_lookup(idx, table):
    return TableLookupFn.apply(idx, table)
