"""bf16 GEMM entry points on the sm_100a engine (csrc/gemm_sm100.cu).

Conventions: a Linear weight ``w`` is ``[out, in]``.  Forward ``y = x w^T``, input gradient
``dx = dy w``, weight gradient ``dW = dy^T x`` (reduction over tokens).  The engine takes
both operands in either storage order, so no transpose is ever materialised.
"""
import torch

from nexttransformer_b200.ops._ext import ext

EPI_BF16, EPI_F32, EPI_F32_ACC, EPI_BF16_AXPBY, EPI_RELU2, EPI_RELU2_BWD = range(6)


def gemm(a, b, out, *, a_mn=False, b_mn=False, epi=EPI_BF16, r=None, p=None, s_acc=1.0, s_res=1.0, s_dev=None):
    """out = epilogue(A B^T); A logical [M,K] (stored [K,M] if a_mn), B logical [N,K] (stored [K,N] if b_mn).

    ``s_dev`` (optional one-element fp32 CUDA tensor) multiplies ``s_acc`` on the device, so a
    loss scale produced by autograd never needs a host synchronisation.
    """
    ext().gemm(a, a_mn, b, b_mn, out, epi, r, p, float(s_acc), float(s_res), s_dev)
    return out


def linear(x, w, out=None, *, s_acc=1.0):
    """y = x w^T in bf16 (x [M,K], w [N,K])."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], device=x.device, dtype=torch.bfloat16)
    return gemm(x, w, out, s_acc=s_acc)


def linear_residual(x, w, res, out=None, *, s_acc=1.0, s_res=1.0):
    """y = bf16(s_acc x w^T) + s_res res."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], device=x.device, dtype=torch.bfloat16)
    return gemm(x, w, out, epi=EPI_BF16_AXPBY, r=res, s_acc=s_acc, s_res=s_res)


def linear_relu2(x, w):
    """(pre, relu(pre)^2) with pre = x w^T, both bf16."""
    pre = torch.empty(x.shape[0], w.shape[0], device=x.device, dtype=torch.bfloat16)
    out = torch.empty_like(pre)
    gemm(x, w, out, epi=EPI_RELU2, p=pre)
    return pre, out


def dgrad(dy, w, out=None, *, s_acc=1.0, s_dev=None):
    """dx = s_acc dy w  (dy [M,N], w [N,K] -> [M,K])."""
    if out is None:
        out = torch.empty(dy.shape[0], w.shape[1], device=dy.device, dtype=torch.bfloat16)
    return gemm(dy, w, out, b_mn=True, s_acc=s_acc, s_dev=s_dev)


def dgrad_relu2(dy, w, pre):
    """d pre = (dy w) * 2 relu(pre)."""
    out = torch.empty(dy.shape[0], w.shape[1], device=dy.device, dtype=torch.bfloat16)
    return gemm(dy, w, out, b_mn=True, epi=EPI_RELU2_BWD, r=pre)


def wgrad(dy, x, grad, *, accumulate, s_acc=1.0, s_dev=None):
    """grad (fp32 [N,K]) (+)= s_acc dy^T x   (dy [M,N], x [M,K])."""
    return gemm(dy, x, grad, a_mn=True, b_mn=True, epi=EPI_F32_ACC if accumulate else EPI_F32, s_acc=s_acc,
                s_dev=s_dev)
