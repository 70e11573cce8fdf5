"""Tensor-parallel linears (new capability; the reference pins TP = 1).

Column-parallel: each rank holds an output slice W_r [N / P, K]; y_r = x W_r^T, optionally
all-gathered.  Row-parallel: each rank holds an input slice W_r [N, K / P] and its activation
slice x_r; y = sum_r x_r W_r^T via a reduce-scatter over tokens (sequence-parallel output) or an
all-reduce.  ``MLPTP`` pairs them (column fc -> ReLU^2 -> row proj), the standard Megatron split
with one collective per direction.  The collectives are NCCL (gloo on CPU) calls around the GEMMs:
this is the baseline form; the all-gather -> GEMM and GEMM -> reduce-scatter pairs are not yet fused
into peer-memory kernels.
"""
import torch
import torch.distributed as dist
from torch import nn
import torch.nn.functional as F


class _ReduceScatterRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        size = dist.get_world_size(group)
        out = x.new_empty((x.shape[0] // size, *x.shape[1:]))
        dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        size = dist.get_world_size(ctx.group)
        out = g.new_empty((g.shape[0] * size, *g.shape[1:]))
        dist.all_gather_into_tensor(out, g.contiguous(), group=ctx.group)
        return out, None


class _AllGatherRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        size = dist.get_world_size(group)
        out = x.new_empty((x.shape[0] * size, *x.shape[1:]))
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        size = dist.get_world_size(ctx.group)
        out = g.new_empty((g.shape[0] // size, *g.shape[1:]))
        dist.reduce_scatter_tensor(out, g.contiguous(), group=ctx.group)
        return out, None


def reduce_scatter_rows(x, group=None):
    return _ReduceScatterRows.apply(x, group)


def all_gather_rows(x, group=None):
    return _AllGatherRows.apply(x, group)


class MLPTP(nn.Module):
    """ReLU^2 MLP split over a tensor-parallel group; input and output are sequence-sharded rows."""

    def __init__(self, width, hidden, group=None):
        super().__init__()
        self.group = group
        size = dist.get_world_size(group)
        if hidden % size:
            raise ValueError("hidden width must divide over the tensor-parallel group")
        self.c_fc = nn.Linear(width, hidden // size, bias=False)
        self.c_proj = nn.Linear(hidden // size, width, bias=False)

    @classmethod
    def from_dense(cls, mlp, group=None):
        size, rank = dist.get_world_size(group), dist.get_rank(group)
        width, hidden = mlp.c_fc.weight.shape[1], mlp.c_fc.weight.shape[0]
        m = cls(width, hidden, group)
        sl = slice(rank * hidden // size, (rank + 1) * hidden // size)
        with torch.no_grad():
            m.c_fc.weight.copy_(mlp.c_fc.weight[sl])
            m.c_proj.weight.copy_(mlp.c_proj.weight[:, sl])
        return m

    def forward(self, x_shard):
        x = all_gather_rows(x_shard, self.group)                       # all-gather -> GEMM
        h = F.relu(F.linear(x, self.c_fc.weight.to(x.dtype))).square()
        y = F.linear(h, self.c_proj.weight.to(x.dtype))
        return reduce_scatter_rows(y, self.group)                      # GEMM -> reduce-scatter
