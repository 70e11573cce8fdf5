"""Megatron-style mixture-of-experts FFN: softmax top-k router with aux-loss-free balancing,
one shared expert, ReLU^2 experts.

Routing: router logits in fp32; expert choice = top-k of (softmax probabilities + per-expert
bias); combine weights = the chosen probabilities renormalised to sum 1 (with zero bias this is
exactly the reference's normalised top-k softmax, ``nexttransformer/scaling/reference_blocks.py:
20-45``).  The bias is not trained by gradients: after each update it moves by ``moe_bias_rate``
towards balance (sign of mean load minus expert load), as in aux-loss-free load balancing.

Execution: tokens are sorted by expert and each expert runs on its contiguous slice (grouped
execution).  On CUDA all experts run in one grouped GEMM per projection (``ops.moe``); on the CPU
each expert runs on its slice in turn.  With an expert-parallel group set (``parallel.expert``)
tokens are exchanged between the ranks before and after the experts.
"""
import torch
from torch import nn
import torch.nn.functional as F

from nexttransformer_b200.models.shell import Linear


class ExpertMLP(nn.Module):
    def __init__(self, width, hidden):
        super().__init__()
        self.c_fc = Linear(width, hidden, bias=False)
        self.c_proj = Linear(hidden, width, bias=False)

    def forward(self, x):
        return self.c_proj(F.relu(self.c_fc(x)).square())


class MoEFFN(nn.Module):
    def __init__(self, width, num_experts, top_k, expert_width, shared=1, bias_rate=1e-3):
        super().__init__()
        if not 1 <= top_k <= num_experts:
            raise ValueError("top_k must be in [1, num_experts]")
        self.num_experts, self.top_k, self.bias_rate = num_experts, top_k, bias_rate
        self.router = Linear(width, num_experts, bias=False)
        self.shared = ExpertMLP(width, expert_width * shared) if shared else None
        self.experts = nn.ModuleList(ExpertMLP(width, expert_width) for _ in range(num_experts))
        self.register_buffer("expert_bias", torch.zeros(num_experts), persistent=True)
        self.register_buffer("load", torch.zeros(num_experts), persistent=False)
        self.ep_group = None       # set by parallel.expert.enable_expert_parallel (None = world group)
        self.ep_size = 1
        self.ep_exchange = "peer"  # "peer": NVLink peer-memory exchange on CUDA; "nccl": all-to-all
        self.last_stats = {}

    def route(self, rows):
        logits = F.linear(rows.float(), self.router.weight.float())
        probs = logits.softmax(-1)
        choice = (probs + self.expert_bias).topk(self.top_k, dim=-1).indices
        w = probs.gather(-1, choice)
        w = w / w.sum(-1, keepdim=True)
        return choice, w

    def forward(self, x):
        rows = x.reshape(-1, x.shape[-1])
        choice, w = self.route(rows)
        with torch.no_grad():
            self.load += torch.bincount(choice.flatten(), minlength=self.num_experts).float()
        out = self.shared(rows) if self.shared is not None else torch.zeros_like(rows)
        if self.ep_size > 1:
            from nexttransformer_b200.parallel import expert as ep
            if ep.peer_exchange_supported(self, rows) and self.ep_exchange == "peer":
                routed = ep.peer_expert_combine(self, rows, choice, w)
            else:
                routed = ep.expert_parallel_combine(self, rows, choice, w)
        elif rows.is_cuda and rows.shape[-1] % 64 == 0 and self.experts[0].c_fc.weight.shape[0] % 64 == 0:
            from nexttransformer_b200.ops.moe import grouped_experts
            w_fc = torch.stack([e.c_fc.weight for e in self.experts])
            w_proj = torch.stack([e.c_proj.weight for e in self.experts])
            routed = grouped_experts(rows, choice, w, w_fc, w_proj)
        else:
            routed = self.local_experts(rows, choice, w)
        out = out + routed
        self.last_stats = {"max_load_fraction": float(self.load.max() / self.load.sum().clamp_min(1))}
        return out.reshape_as(x)

    def local_experts(self, rows, choice, w, experts=None, offset=0):
        """Grouped execution: sort (token, slot) pairs by expert, run each expert on its slice."""
        experts = self.experts if experts is None else experts
        flat = choice.flatten()
        order = torch.argsort(flat, stable=True)
        tokens = order // self.top_k
        counts = torch.bincount(flat - offset, minlength=len(experts))[:len(experts)].tolist() if flat.numel() else []
        xs = rows.index_select(0, tokens)
        ws = w.flatten().index_select(0, order).to(rows.dtype)
        outs, start = [], 0
        for e, n in zip(experts, counts):
            if n:
                outs.append(e(xs[start:start + n]) * ws[start:start + n, None])
            start += n
        y = torch.cat(outs) if outs else xs.new_zeros(0, rows.shape[-1])
        return torch.zeros_like(rows).index_add(0, tokens[:y.shape[0]], y)

    @torch.no_grad()
    def update_bias(self):
        """Aux-loss-free balancing step; call once per optimizer update (loads summed over ranks)."""
        load = self.load
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            torch.distributed.all_reduce(load)
        if load.sum() > 0:
            self.expert_bias += self.bias_rate * torch.sign(load.mean() - load)
        self.load.zero_()
