"""Tensor-parallel linears (new capability; the reference pins TP = 1).

Column-parallel: each rank holds an output slice W_r [N / P, K]; y_r = x W_r^T, optionally
all-gathered.  Row-parallel: each rank holds an input slice W_r [N, K / P] and its activation
slice x_r; y = sum_r x_r W_r^T via a reduce-scatter over tokens (sequence-parallel output) or an
all-reduce.  ``MLPTP`` pairs them (column fc -> ReLU^2 -> row proj), the standard Megatron split
with one collective per direction.  The collectives are NCCL (gloo on CPU) calls around the GEMMs:
this is the baseline form; the all-gather -> GEMM and GEMM -> reduce-scatter pairs are not yet fused
into peer-memory kernels.

``enable_tensor_parallel(model, group)`` puts a model's plain ReLU^2 MLPs on the group: every rank keeps
the rest of the block replicated, takes its slice of the block's rows into ``MLPTP`` and gathers the
rows back, so replicated parameters see the same gradient on every rank and each rank holds and
updates only its slices of the MLP matrices (an optimizer then sees the shards: Muon orthogonalises
each shard on its own, which is not the full matrix's update).
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


class _ScatterToRanks(torch.autograd.Function):
    """Forward: this rank's slice of the rows (no communication).  Backward: the rows' gradients of
    every rank gathered, so the replicated computation upstream sees the full gradient everywhere."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        size, rank = dist.get_world_size(group), dist.get_rank(group)
        n = x.shape[0] // size
        return x[rank * n:(rank + 1) * n].contiguous()

    @staticmethod
    def backward(ctx, g):
        return all_gather_rows_plain(g, ctx.group), None


class _GatherFromRanks(torch.autograd.Function):
    """Forward: every rank's rows gathered.  Backward: the (replicated, hence equal) gradient's slice of
    this rank's rows; no sum, which would count the replicated gradient once per rank."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return all_gather_rows_plain(x, group)

    @staticmethod
    def backward(ctx, g):
        size, rank = dist.get_world_size(ctx.group), dist.get_rank(ctx.group)
        n = g.shape[0] // size
        return g[rank * n:(rank + 1) * n].contiguous(), None


def all_gather_rows_plain(x, group=None):
    size = dist.get_world_size(group)
    out = x.new_empty((x.shape[0] * size, *x.shape[1:]))
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


class TensorParallelMLP(nn.Module):
    """A block's MLP on a tensor-parallel group: [B, T, d] in and out, replicated on every rank."""

    def __init__(self, mlp, group=None):
        super().__init__()
        self.group = group
        self.tp = MLPTP.from_dense(mlp, group)

    def forward(self, x):
        rows = x.reshape(-1, x.shape[-1])
        if rows.shape[0] % dist.get_world_size(self.group):
            raise ValueError("tokens per micro-batch must divide over the tensor-parallel group")
        y = _GatherFromRanks.apply(self.tp(_ScatterToRanks.apply(rows, self.group)), self.group)
        return y.view_as(x)


def enable_tensor_parallel(model, group=None):
    """Replace every plain shell ``MLP`` under ``model`` by its tensor-parallel form on ``group``
    (weights sliced from the current ones).  Returns the number of MLPs replaced.  Variants that
    transform the hidden layer (a ``hidden`` override) stay replicated."""
    from nexttransformer_b200.models.shell import MLP
    replaced = 0
    for module in list(model.modules()):
        for name, child in list(module.named_children()):
            if type(child) is MLP:
                setattr(module, name, TensorParallelMLP(child, group))
                replaced += 1
    return replaced
