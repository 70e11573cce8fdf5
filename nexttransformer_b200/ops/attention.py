"""Causal (optionally sliding-window, GQA) attention on the packed q|k|v projection.

``attention_fn(qkv, B, T, H, Hk, D, window)`` takes the ``[B*T, (H + 2 Hk) D]`` output of the
QKV GEMM (after RoPE / QK-norm) and returns ``y [B*T, H D]``; its backward returns ``dqkv`` in
the same packed layout, which the QKV input-gradient GEMM consumes directly.

On CUDA the forward and backward run the sm_100a flash-attention kernels of
``csrc/attention_sm100.cu``.  ``window`` is the reference's left window: a query at position t
sees keys t - window .. t; a window >= T - 1 is plain causal attention.
"""
import math

import torch
from torch.autograd import Function

from nexttransformer_b200.ops._ext import ext
from nexttransformer_b200.models.shell import sdpa

# Set by the kernel module once the tcgen05 path is validated for a (D, dtype) pair.
KERNEL_HEAD_DIMS = (128,)
# Deterministic backward: every key tile writes its dQ contribution to its own fp32 slice and the
# slices are summed in key-tile order (bitwise reproducible; ceil(T / 128) x the dQ workspace).
# Default: contributions are added into one buffer with bulk reductions whose order is not fixed.
_deterministic = False


def set_deterministic(on=True):
    """Select the deterministic attention backward (the reference's ``--deterministic-attention``)."""
    global _deterministic
    _deterministic = bool(on)


def _dq_workspace(M, cols, T, device):
    """(zeroed fp32 dQ workspace, slice count) for the current backward mode."""
    slices = (T + 127) // 128 if _deterministic else 0
    return torch.zeros(max(slices, 1) * M, cols, device=device, dtype=torch.float32), slices


def _use_kernel(qkv, D):
    return qkv.is_cuda and D in KERNEL_HEAD_DIMS and getattr(ext(), "attn_fwd", None) is not None and _kernel_enabled


_kernel_enabled = True


class _KernelAttn(Function):
    @staticmethod
    def forward(ctx, qkv, B, T, H, Hk, D, window):
        lib = ext()
        M = B * T
        q = qkv[:, :H * D]
        k = qkv[:, H * D:(H + Hk) * D]
        v = qkv[:, (H + Hk) * D:]
        o = torch.empty(M, H * D, device=qkv.device, dtype=torch.bfloat16)
        lse = torch.empty(B, H, T, device=qkv.device, dtype=torch.float32)
        w = window if 0 <= window < T - 1 else -1
        lib.attn_fwd(q, k, v, o, lse, B, T, H, Hk, D, w, 1.0 / math.sqrt(D))
        ctx.save_for_backward(qkv, o, lse)
        ctx.shape = (B, T, H, Hk, D, w)
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        B, T, H, Hk, D, w = ctx.shape
        lib = ext()
        M = B * T
        dqkv = torch.empty_like(qkv)
        dq_acc, slices = _dq_workspace(M, H * D, T, qkv.device)
        delta = torch.empty(B, H, T, device=qkv.device, dtype=torch.float32)
        lib.attn_bwd(qkv[:, :H * D], qkv[:, H * D:(H + Hk) * D], qkv[:, (H + Hk) * D:], o, lse, do.contiguous(),
                     dqkv[:, :H * D], dqkv[:, H * D:(H + Hk) * D], dqkv[:, (H + Hk) * D:], dq_acc, delta,
                     B, T, H, Hk, D, w, 1.0 / math.sqrt(D), None, slices)
        return dqkv, None, None, None, None, None, None


class _LibraryAttn(Function):
    """PyTorch SDPA inside a private autograd graph (oracle, CPU, unsupported head dims)."""

    @staticmethod
    def forward(ctx, qkv, B, T, H, Hk, D, window):
        with torch.enable_grad():
            leaf = qkv.detach().requires_grad_()
            v4 = leaf.view(B, T, H + 2 * Hk, D)
            y = sdpa(v4[:, :, :H], v4[:, :, H:H + Hk], v4[:, :, H + Hk:], window).reshape(B * T, H * D)
        ctx.leaf, ctx.y = leaf, y
        return y.detach()

    @staticmethod
    def backward(ctx, dy):
        (dqkv,) = torch.autograd.grad(ctx.y, ctx.leaf, dy)
        ctx.leaf = ctx.y = None
        return dqkv, None, None, None, None, None, None


class _KernelAttnBTHD(Function):
    """The same kernels on separate ``[B, T, H, D]`` q / ``[B, T, Hk, D]`` k, v tensors (the layout
    of the eager mixers); gradients come back in that layout."""

    @staticmethod
    def forward(ctx, q, k, v, window):
        B, T, H, D = q.shape
        Hk = k.shape[2]
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        o = torch.empty(B * T, H * D, device=q.device, dtype=torch.bfloat16)
        lse = torch.empty(B, H, T, device=q.device, dtype=torch.float32)
        w = window if 0 <= window < T - 1 else -1
        ext().attn_fwd(q.view(B * T, H * D), k.view(B * T, Hk * D), v.view(B * T, Hk * D), o, lse, B, T, H, Hk, D,
                       w, 1.0 / math.sqrt(D))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.w = w
        return o.view(B, T, H, D)

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        B, T, H, D = q.shape
        Hk = k.shape[2]
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        dq_acc, slices = _dq_workspace(B * T, H * D, T, q.device)
        delta = torch.empty(B, H, T, device=q.device, dtype=torch.float32)
        ext().attn_bwd(q.view(B * T, -1), k.view(B * T, -1), v.view(B * T, -1), o, lse,
                       do.contiguous().view(B * T, -1), dq.view(B * T, -1), dk.view(B * T, -1), dv.view(B * T, -1),
                       dq_acc, delta, B, T, H, Hk, D, ctx.w, 1.0 / math.sqrt(D), None, slices)
        return dq, dk, dv, None


def kernel_supports(q, k, v):
    """True when the sm_100a kernels take these ``[B, T, H, D]`` tensors."""
    return (_kernel_enabled and q.is_cuda and q.dtype == k.dtype == v.dtype == torch.bfloat16
            and q.shape[-1] in KERNEL_HEAD_DIMS and k.shape == v.shape and q.shape[2] % k.shape[2] == 0
            and type(q) is torch.Tensor)


def attention_bthd(q, k, v, window):
    """Causal (windowed) GQA attention on ``[B, T, H, D]`` tensors through the sm_100a kernels."""
    return _KernelAttnBTHD.apply(q, k, v, window)


def attention_fn(qkv, B, T, H, Hk, D, window):
    if _use_kernel(qkv, D):
        return _KernelAttn.apply(qkv, B, T, H, Hk, D, window)
    return _LibraryAttn.apply(qkv, B, T, H, Hk, D, window)
