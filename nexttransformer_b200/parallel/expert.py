"""Expert parallelism for ``models.moe.MoEFFN``.

With an expert-parallel group of size E_p, rank r holds experts [r E/E_p, (r+1) E/E_p).  Each
rank routes its own tokens, sends every (token, expert) assignment to the expert's owner with
one all-to-all (counts exchanged first), the owner runs its experts on the received rows in
grouped order, and a second all-to-all returns the weighted outputs, which are summed back per
token.  Autograd flows through both exchanges (the backward of an all-to-all is the reverse
all-to-all).  Gradients of expert weights are then local to their owner; the dense and router
parameters are reduced over the data-parallel group as usual.
"""
import torch
import torch.distributed as dist


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send_counts, recv_counts, group):
        ctx.counts = (send_counts, recv_counts)
        ctx.group = group
        out = x.new_empty((sum(recv_counts), *x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv_counts, send_counts, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        send, recv = ctx.counts
        out = g.new_empty((sum(send), *g.shape[1:]))
        dist.all_to_all_single(out, g.contiguous(), send, recv, group=ctx.group)
        return out, None, None, None


def all_to_all(x, send_counts, recv_counts, group=None):
    return _AllToAll.apply(x, list(send_counts), list(recv_counts), group)


def enable_expert_parallel(model, group=None):
    """Shard every MoE layer's experts over `group`; returns the number of local experts."""
    from nexttransformer_b200.models.moe import MoEFFN
    size = dist.get_world_size(group)
    rank = dist.get_rank(group)
    local = None
    for m in model.modules():
        if isinstance(m, MoEFFN):
            if m.num_experts % size:
                raise ValueError("experts must divide evenly over the expert-parallel group")
            per = m.num_experts // size
            m.ep_group, m.ep_rank, m.ep_size, m.ep_per = group, rank, size, per
            for i, e in enumerate(m.experts):
                for p in e.parameters():
                    p.requires_grad_(rank * per <= i < (rank + 1) * per)
                    p.expert_owner = i // per
            local = per
    return local


def expert_parallel_combine(moe, rows, choice, w):
    """Routed-expert output for `rows` under expert parallelism (see module docstring)."""
    group, size, per, me = moe.ep_group, moe.ep_size, moe.ep_per, moe.ep_rank
    k = moe.top_k
    flat = choice.flatten()
    owner = flat // per
    order = torch.argsort(owner * moe.num_experts + flat, stable=True)   # by owner, then expert
    send_counts = torch.bincount(owner, minlength=size)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    tokens = order // k
    xs = rows.index_select(0, tokens)
    es = flat.index_select(0, order)
    ws = w.flatten().index_select(0, order)
    rx = all_to_all(xs, sc, rc, group)
    re = all_to_all(es.to(rows.dtype).unsqueeze(-1), sc, rc, group).squeeze(-1).round().long()
    local = re - me * per
    srt = torch.argsort(local, stable=True)
    counts = torch.bincount(local, minlength=per).tolist()
    xin = rx.index_select(0, srt)
    outs, start = [], 0
    for e, n in enumerate(counts):
        if n:
            outs.append(moe.experts[me * per + e](xin[start:start + n]))
        start += n
    y = torch.cat(outs) if outs else xin[:0]
    back = torch.empty_like(y).index_copy(0, srt, y) if y.shape[0] else y
    ret = all_to_all(back, rc, sc, group)
    contrib = ret * ws[:, None].to(ret.dtype)
    return torch.zeros_like(rows).index_add(0, tokens, contrib)
