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
    def __init__(self, width, num_experts, top_k, expert_width, shared=1, bias_rate=1e-3, aux_loss_coeff=0.0,
                 z_loss_coeff=0.0):
        super().__init__()
        if not 1 <= top_k <= num_experts:
            raise ValueError("top_k must be in [1, num_experts]")
        if aux_loss_coeff < 0 or z_loss_coeff < 0:
            raise ValueError("MoE loss coefficients must be non-negative")
        self.num_experts, self.top_k, self.bias_rate = num_experts, top_k, bias_rate
        self.aux_loss_coeff, self.z_loss_coeff = float(aux_loss_coeff), float(z_loss_coeff)
        self.router = Linear(width, num_experts, bias=False)
        self.shared = ExpertMLP(width, expert_width * shared) if shared else None
        self.experts = nn.ModuleList(ExpertMLP(width, expert_width) for _ in range(num_experts))
        self.register_buffer("expert_bias", torch.zeros(num_experts), persistent=True)
        self.register_buffer("load", torch.zeros(num_experts), persistent=False)
        self.ep_group = None       # set by parallel.expert.enable_expert_parallel (None = world group)
        self.ep_size = 1
        self.ep_rank = 0
        self.ep_per = num_experts
        self.ep_exchange = "peer"  # "peer": NVLink peer-memory exchange on CUDA; "nccl": all-to-all
        # Kernel state (models.fused_dense.FusedState): the experts' bf16 shadows and fp32 gradient
        # buffers stacked [E_local, F, d] / [E_local, d, F]; each expert's parameter keeps its own
        # name and owns one slice (its ``main_grad`` is a view), so no stack is built per forward.
        self._w_fc = self._w_proj = self._g_fc = self._g_proj = None
        self.last_aux = None
        self.last_stats = {}
        # CUDA routing through the fused kernels (ops.moe.fused_route); False: the torch ops below
        self.fused_route = True
        self._plan = None

    # -------------------------------------------------------------- experts held by this rank
    def local_experts(self):
        """This rank's experts in global order (all of them without expert parallelism)."""
        return list(self.experts.values()) if isinstance(self.experts, nn.ModuleDict) else list(self.experts)

    def expert(self, i):
        """Expert with global index ``i`` (must be held by this rank)."""
        return self.experts[str(i)] if isinstance(self.experts, nn.ModuleDict) else self.experts[i]

    def keep_experts(self, first, count):
        """Drop every expert outside [first, first + count): the others live on other ranks.  The kept
        ones keep their global names (``experts.<i>.*``) in the state dict."""
        kept = nn.ModuleDict({str(i): self.expert(i) for i in range(first, first + count)})
        self.experts = kept

    # -------------------------------------------------------------- routing
    def route(self, rows):
        """(choice [T, k], weights [T, k], aux loss or None); on CUDA the fused kernels also leave
        the grouped-GEMM row plan in ``self._plan`` and add the counts to ``self.load``."""
        logits = F.linear(rows.float(), self.router.weight.float())
        self._plan = None
        use_aux = self.training and bool(self.aux_loss_coeff or self.z_loss_coeff)
        if self.fused_route and rows.is_cuda:
            from nexttransformer_b200.ops.moe import fused_route, fused_route_supported
            if fused_route_supported(logits, self.top_k):
                choice, w, aux, self._plan = fused_route(
                    logits, self.expert_bias, self.top_k, self.aux_loss_coeff if use_aux else 0.0,
                    self.z_loss_coeff if use_aux else 0.0, self.load)
                return choice, w, aux if use_aux else None
        probs = logits.softmax(-1)
        choice = (probs + self.expert_bias).topk(self.top_k, dim=-1).indices
        w = probs.gather(-1, choice)
        w = w / w.sum(-1, keepdim=True)
        aux = None
        if use_aux:
            aux = logits.new_zeros(())
            if self.aux_loss_coeff:
                # Switch-style balance loss: E * sum_e (fraction of assignments to e) * (mean router prob of e)
                frac = torch.zeros(self.num_experts, device=rows.device, dtype=torch.float32).index_add_(
                    0, choice.flatten(), torch.ones(choice.numel(), device=rows.device)) / choice.numel()
                aux = aux + self.aux_loss_coeff * self.num_experts * (frac * probs.mean(0)).sum()
            if self.z_loss_coeff:
                aux = aux + self.z_loss_coeff * torch.logsumexp(logits, -1).square().mean()
        return choice, w, aux

    def forward(self, x):
        rows = x.reshape(-1, x.shape[-1])
        choice, w, self.last_aux = self.route(rows)
        if self._plan is None:
            with torch.no_grad():
                self.load += torch.bincount(choice.flatten(), minlength=self.num_experts).float()
        out = self.shared(rows) if self.shared is not None else torch.zeros_like(rows)
        if self.ep_size > 1:
            from nexttransformer_b200.parallel import expert as ep
            choice = choice.long()
            if ep.peer_exchange_supported(self, rows) and self.ep_exchange == "peer":
                routed = ep.peer_expert_combine(self, rows, choice, w)
            else:
                routed = ep.expert_parallel_combine(self, rows, choice, w)
        elif rows.is_cuda and self._w_fc is not None:
            from nexttransformer_b200.ops.moe import grouped_experts_state
            routed = grouped_experts_state(rows, choice, w, self, self._plan)
        elif rows.is_cuda and rows.shape[-1] % 64 == 0 and self.expert(0).c_fc.weight.shape[0] % 64 == 0:
            from nexttransformer_b200.ops.moe import grouped_experts
            w_fc = torch.stack([e.c_fc.weight for e in self.local_experts()])
            w_proj = torch.stack([e.c_proj.weight for e in self.local_experts()])
            routed = grouped_experts(rows, choice, w, w_fc, w_proj, self._plan)
        else:
            routed = self.run_experts(rows, choice, w)
        out = out + routed
        # a device tensor: reading it back is left to whoever reports it (no host sync per layer)
        self.last_stats = {"max_load_fraction": (self.load.max() / self.load.sum().clamp_min(1)).detach()}
        return out.reshape_as(x)

    def run_experts(self, rows, choice, w, experts=None, offset=0):
        """Grouped execution: sort (token, slot) pairs by expert, run each expert on its slice."""
        experts = self.local_experts() if experts is None else experts
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
