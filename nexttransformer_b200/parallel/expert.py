"""Expert parallelism for ``models.moe.MoEFFN``.

With an expert-parallel group of size E_p, rank r holds experts [r E/E_p, (r+1) E/E_p) and no
others: ``enable_expert_parallel`` drops the other experts' modules, so each rank stores only its
own shard (the kept experts keep their global names in the state dict).  Each rank routes its own
tokens; every (token, expert) assignment is processed by the expert's owner and the weighted
outputs are summed back per token on the token's rank.  Gradients of expert weights are local to
their owner; ``expert_data_parallel_groups`` gives the groups over which copies of one expert
shard (one per expert-parallel group) average their gradients, and the dense and router
parameters are reduced over the whole data-parallel group as usual.

Two exchanges implement this:

* ``PeerExpertExchange`` (CUDA, NVLink peers): every rank writes its assignments, sorted by
  expert, into a send buffer in symmetric memory and publishes its per-expert counts into every
  peer's count table; after a flag barrier each owner pulls its rows straight from the peers'
  send buffers into its grouped-GEMM layout (``csrc/moe.cu``, plain peer loads), runs the
  grouped expert GEMMs, and pushes the result rows into the sources' return buffers (plain peer
  stores); a second barrier, and each source combines its rows locally.  The backward runs the
  same movement on the gradients.  Two barriers per direction, no NCCL call.
* ``expert_parallel_combine`` (any backend, the CPU tests use gloo): counts exchanged with an
  all-to-all, rows sent with ``all_to_all_single``, whose backward is the reverse all-to-all.
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
    """Shard every MoE layer's experts over `group` (this rank keeps only its own experts); returns
    the number of local experts.  Call before the optimizer and the kernel state are built."""
    from nexttransformer_b200.models.moe import MoEFFN
    size = dist.get_world_size(group)
    rank = dist.get_rank(group)
    local = None
    for m in model.modules():
        if isinstance(m, MoEFFN):
            if m.num_experts % size:
                raise ValueError("experts must divide evenly over the expert-parallel group")
            if m._w_fc is not None:
                raise RuntimeError("enable expert parallelism before building the kernel state")
            per = m.num_experts // size
            m.ep_group, m.ep_rank, m.ep_size, m.ep_per = group, rank, size, per
            m.keep_experts(rank * per, per)
            for e in m.local_experts():
                for p in e.parameters():
                    p.expert_owner = rank
                    p.expert_parallel = True
            local = per
    return local


def expert_data_parallel_groups(world, ep_size):
    """Rank lists of the expert-data-parallel groups: ranks holding the same expert shard.

    With ``world = ep_size * dp`` ranks laid out as consecutive expert-parallel groups
    (ranks [g ep_size, (g + 1) ep_size) form group g), shard s is held by ranks s, s + ep_size, ...
    (the reference's Megatron ``expt_dp`` groups, ``nexttransformer/scaling/megatron_optimizer.py``)."""
    if ep_size <= 0 or world % ep_size:
        raise ValueError("the expert-parallel size must divide the world size")
    return [list(range(s, world, ep_size)) for s in range(ep_size)]


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
            outs.append(moe.expert(me * per + e)(xin[start:start + n]))
        start += n
    y = torch.cat(outs) if outs else xin[:0]
    back = torch.empty_like(y).index_copy(0, srt, y) if y.shape[0] else y
    ret = all_to_all(back, rc, sc, group)
    contrib = ret * ws[:, None].to(ret.dtype)
    return torch.zeros_like(rows).index_add(0, tokens, contrib)


# ---------------------------------------------------------------------------- peer-memory exchange
EPI_BF16, EPI_F32, EPI_F32_ACC, EPI_BF16_AXPBY, EPI_RELU2, EPI_RELU2_BWD = range(6)
PAD = 128


class PeerExpertExchange:
    """Symmetric send / return row buffers and the count table of one expert-parallel group."""

    def __init__(self, group, rows, d, num_experts, device, timeout_s=60.0):
        import torch.distributed._symmetric_memory as symm
        group = group if group is not None else dist.group.WORLD
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.rows, self.d, self.E, self.timeout_s = rows, d, num_experts, timeout_s
        row_bytes = rows * d * 2
        self.ret_off = row_bytes
        self.cnt_off = 2 * row_bytes
        cnt_bytes = (self.world * num_experts * 4 + 255) // 256 * 256
        self.buf = symm.empty(2 * row_bytes + cnt_bytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        h = symm.rendezvous(self.buf, group)
        self.handle = h
        from nexttransformer_b200.parallel.symmetric import peer_pointers
        base = torch.tensor(peer_pointers(self.buf, h, self.rank), dtype=torch.int64, device=device)
        self.send_peers = base.clone()
        self.ret_peers = base + self.ret_off
        self.cnt_peers = base + self.cnt_off
        self.pads = torch.tensor(list(h.signal_pad_ptrs), dtype=torch.int64, device=device)
        self.send = self.buf[:row_bytes].view(torch.bfloat16).view(rows, d)
        self.ret = self.buf[self.ret_off:self.ret_off + row_bytes].view(torch.bfloat16).view(rows, d)
        self.counts = self.buf[self.cnt_off:self.cnt_off + self.world * num_experts * 4].view(torch.int32)
        self.counts = self.counts.view(self.world, num_experts)
        self.epoch = 0

    def barrier(self):
        from nexttransformer_b200.ops._ext import ext
        self.epoch += 1
        ext().p2p_barrier(self.pads, self.rank, self.world, self.epoch, self.timeout_s)

    def publish_counts(self, counts):
        from nexttransformer_b200.ops._ext import ext
        ext().p2p_put(self.cnt_peers, self.world, self.rank * self.E * 4, counts.to(torch.int32).contiguous())


_EXCHANGES = {}


def peer_exchange(moe, rows_needed, d, device):
    """The group's exchange, (re)allocated collectively when a larger row count is needed."""
    key = (id(moe.ep_group), d, moe.num_experts)
    ex = _EXCHANGES.get(key)
    if ex is None or ex.rows < rows_needed:
        ex = PeerExpertExchange(moe.ep_group, rows_needed, d, moe.num_experts, device)
        _EXCHANGES[key] = ex
    return ex


def _owner_tables(cnt, me, per):
    """Row layout of the owner's experts from the count table cnt [W, E] (device): per local row
    its source rank and row in that source's send buffer (-1: padding), grp_m, grp_k and P."""
    W = cnt.shape[0]
    dev = cnt.device
    cnt = cnt.long()
    loc = cnt[:, me * per:(me + 1) * per]                       # [W, per]
    tot = loc.sum(0)
    padded = (tot + PAD - 1) // PAD * PAD
    end = padded.cumsum(0)
    start = end - padded
    P, n = (int(v) for v in torch.stack((end[-1], tot.sum())).tolist())
    send_start = (cnt.cumsum(1) - cnt)[:, me * per:(me + 1) * per]   # [W, per]
    within = loc.cumsum(0) - loc
    seg_len = loc.t().reshape(-1)                                  # segments ordered (expert, source)
    seg_dst = (start[:, None] + within.t()).reshape(-1)
    seg_rank = torch.arange(W, device=dev).repeat(per)
    seg_src = send_start.t().reshape(-1)
    src_rank = torch.full((P,), -1, dtype=torch.int32, device=dev)
    src_row = torch.zeros(P, dtype=torch.int32, device=dev)
    if n:
        idx = torch.repeat_interleave(torch.arange(seg_len.numel(), device=dev), seg_len, output_size=n)
        pos = torch.arange(n, device=dev) - (seg_len.cumsum(0) - seg_len)[idx]
        dst = seg_dst[idx] + pos
        src_rank[dst] = seg_rank[idx].to(torch.int32)
        src_row[dst] = (seg_src[idx] + pos).to(torch.int32)
    tile_row = torch.arange(max(P, 0) // PAD, device=dev) * PAD
    grp_m = torch.searchsorted(end, tile_row, right=True).to(torch.int32)
    grp_k = torch.cat((end.new_zeros(1), end)).to(torch.int32)
    return src_rank, src_row, grp_m, grp_k, P


class _PeerExperts(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, w_fc, w_proj, choice, ex, per, state):
        from nexttransformer_b200.ops._ext import ext
        lib = ext()
        T, k = choice.shape
        d = x.shape[-1]
        F = w_fc.shape[1]
        n = T * k
        dev = x.device
        flat = choice.reshape(-1).long()
        order = torch.argsort(flat, stable=True)
        send_row_of = torch.empty(n, dtype=torch.int32, device=dev)
        send_row_of[order] = torch.arange(n, dtype=torch.int32, device=dev)
        xb = x.to(torch.bfloat16).contiguous()
        lib.moe_gather_rows(xb, (order // k).to(torch.int32), ex.send[:n])
        ex.publish_counts(torch.bincount(flat, minlength=ex.E))
        ex.barrier()                                       # counts and send rows are in place everywhere
        src_rank, src_row, grp_m, grp_k, P = _owner_tables(ex.counts.clone(), ex.rank, per)
        wf = w_fc.to(torch.bfloat16).contiguous()
        wp = w_proj.to(torch.bfloat16).contiguous()
        x_perm = torch.empty(P, d, device=dev, dtype=torch.bfloat16)
        h_pre = torch.empty(P, F, device=dev, dtype=torch.bfloat16)
        h = torch.empty_like(h_pre)
        y_perm = torch.empty(P, d, device=dev, dtype=torch.bfloat16)
        if P:
            lib.moe_pull_rows(ex.send_peers, src_rank, src_row, x_perm)
            lib.gemm_grouped(x_perm, False, wf, False, h, EPI_RELU2, grp_m, False, None, h_pre, 1.0)
            lib.gemm_grouped(h, False, wp, False, y_perm, EPI_BF16, grp_m, False, None, None, 1.0)
            lib.moe_push_rows(y_perm, ex.ret_peers, src_rank, src_row)
        ex.barrier()                                       # every owner has pushed its rows back
        w32 = w.float().contiguous()
        out = torch.empty(T, d, device=dev, dtype=torch.bfloat16)
        lib.moe_combine(ex.ret[:n], send_row_of, w32, None, out)
        y_rows = ex.ret[:n].clone()
        ctx.save_for_backward(x_perm, h_pre, h, wf, wp, src_rank, src_row, grp_m, grp_k, send_row_of, w32, y_rows)
        ctx.ex, ctx.P, ctx.state = ex, P, state
        ctx.dtypes = (x.dtype, w.dtype, w_fc.dtype, w_proj.dtype)
        return out.to(x.dtype)

    @staticmethod
    def backward(ctx, dout):
        from nexttransformer_b200.ops._ext import ext
        lib = ext()
        x_perm, h_pre, h, wf, wp, src_rank, src_row, grp_m, grp_k, send_row_of, w32, y_rows = ctx.saved_tensors
        ex, P = ctx.ex, ctx.P
        T = dout.shape[0]
        n = send_row_of.numel()
        d = dout.shape[-1]
        E_loc, F = wf.shape[0], wf.shape[1]
        dev = dout.device
        dy = dout.to(torch.bfloat16).contiguous()
        dw = torch.empty_like(w32)
        lib.moe_combine_bwd(dy, y_rows, send_row_of, w32, ex.send[:n], dw)
        ex.barrier()                                       # weighted output gradients are in the send buffers
        state = ctx.state
        if state is not None:      # accumulate straight into the experts' main_grad stacks
            dwf, dwp = state._g_fc, state._g_proj
        else:
            dwf = torch.zeros(E_loc, F, d, device=dev, dtype=torch.float32)
            dwp = torch.zeros(E_loc, d, F, device=dev, dtype=torch.float32)
        if P:
            d_rows = torch.empty(P, d, device=dev, dtype=torch.bfloat16)
            lib.moe_pull_rows(ex.send_peers, src_rank, src_row, d_rows)
            dh_pre = torch.empty(P, F, device=dev, dtype=torch.bfloat16)
            lib.gemm_grouped(d_rows, False, wp, True, dh_pre, EPI_RELU2_BWD, grp_m, False, h_pre, None, 1.0)
            lib.gemm_grouped(d_rows, True, h, True, dwp, EPI_F32_ACC, grp_k, True, None, None, 1.0)
            dx_perm = torch.empty(P, d, device=dev, dtype=torch.bfloat16)
            lib.gemm_grouped(dh_pre, False, wf, True, dx_perm, EPI_BF16, grp_m, False, None, None, 1.0)
            lib.gemm_grouped(dh_pre, True, x_perm, True, dwf, EPI_F32_ACC, grp_k, True, None, None, 1.0)
            lib.moe_push_rows(dx_perm, ex.ret_peers, src_rank, src_row)
        ex.barrier()                                       # input gradients are back on their token's rank
        dx = torch.empty(T, d, device=dev, dtype=torch.bfloat16)
        lib.moe_combine(ex.ret[:n], send_row_of, None, None, dx)
        xd, wd, fd, pd = ctx.dtypes
        if state is not None:
            return dx.to(xd), dw.view(T, -1).to(wd), None, None, None, None, None, None
        return dx.to(xd), dw.view(T, -1).to(wd), dwf.to(fd), dwp.to(pd), None, None, None, None


def peer_expert_combine(moe, rows, choice, w):
    """Routed-expert output for `rows` [T, d] (CUDA) through the peer-memory exchange."""
    per, me = moe.ep_per, moe.ep_rank
    ex = peer_exchange(moe, choice.numel(), rows.shape[-1], rows.device)
    if moe._w_fc is not None:     # kernel state: stacked bf16 shadows, gradients into main_grad
        return _PeerExperts.apply(rows, w, moe._w_fc, moe._w_proj, choice, ex, per, moe)
    local = moe.local_experts()
    w_fc = torch.stack([e.c_fc.weight for e in local])
    w_proj = torch.stack([e.c_proj.weight for e in local])
    return _PeerExperts.apply(rows, w, w_fc, w_proj, choice, ex, per, None)


def peer_exchange_supported(moe, rows):
    if not rows.is_cuda or rows.shape[-1] % 64 or moe.local_experts()[0].c_fc.weight.shape[0] % 64:
        return False
    try:
        import torch.distributed._symmetric_memory  # noqa: F401
    except ImportError:
        return False
    return dist.get_backend(moe.ep_group) == "nccl"
