"""``LanguageModel``: one model class for every registered method on the shared shell.

Method dispatch follows the reference's ``ReferenceLM`` (``nexttransformer/models/lm.py``):
  * each block's mixer / FFN is swapped per family (linear, sparse, MLA, hybrid layouts, MoE,
    plugins), DeepLoop and Huginn wrap blocks, HC / mHC add residual maps, AttnRes depth queries;
  * ``forward`` runs the ordinary trunk (dense, sparse, linear, hybrids, fixed_recursive,
    deeploop, plugins), the looped trunk (UT-ACT, Huginn, Ouro) or the residual trunk, then
    the soft-capped readout and the mean token loss plus auxiliary losses;
  * methods whose blocks are all the shell's own dense attention + ReLU^2 MLP run the fused
    sm_100a path on CUDA (``models.fused_dense``).
An op trace (``last_trace``) records every embedding / block / head / depth read.
"""
from contextlib import nullcontext

import torch
from torch import nn
from torch.nn import functional as F

from nexttransformer_b200.models import plugins as plug
from nexttransformer_b200.models.config import HYBRID, LINEAR, LOOPED, MLA, MOE, RESIDUAL, SPARSE, ModelConfig
from nexttransformer_b200.models.linear import LinearMixer, init_gdn_gate
from nexttransformer_b200.models.looped import (DeepLoopBlock, SandwichBlock, act_weights, exit_distribution,
                                                huginn_depth, ouro_gate_loss, sinusoidal_coordinates)
from nexttransformer_b200.models.mla import MLAAttention
from nexttransformer_b200.models.moe import MoEFFN
from nexttransformer_b200.models.registry import PLUGIN_METHODS
from nexttransformer_b200.models.residual import HyperConnection, ManifoldHyperConnection, depth_attention
from nexttransformer_b200.models.shell import MLP, GPTShell, Linear, ShellConfig, norm
from nexttransformer_b200.models.sparse import BACKENDS as SPARSE_BACKENDS, SparseMixer
from nexttransformer_b200.utils.dtype import COMPUTE_DTYPE

# Shell scalars that a method's own residual path replaces (kept, frozen and unused).
FROZEN_NATIVE = {"deeploop": ("resid_lambdas", "x0_lambdas"),
                 **{m: ("resid_lambdas", "x0_lambdas", "backout_lambda") for m in RESIDUAL}}
PROTOCOL_STEPS = 46875


def shell_config(c: ModelConfig):
    return ShellConfig(sequence_len=c.sequence_len, vocab_size=c.vocab_size, n_layer=c.n_layer, n_head=c.heads,
                       n_kv_head=c.n_kv_head, n_embd=c.width, mlp_width=c.mlp_width, window_pattern=c.window_pattern,
                       value_embeddings=c.value_embeddings, attn_head_dim=c.attn_head_dim)


class LanguageModel(GPTShell):
    def __init__(self, config: ModelConfig):
        super().__init__(shell_config(config))
        self.config = config
        c = config
        self.optimizer_step = 0
        self.total_steps = PROTOCOL_STEPS
        self.last_trace, self.last_stats = [], {}
        self.last_aux_loss = self.last_lm_loss = None
        self.row_offset = 0
        # False keeps CUDA training on the plain PyTorch graph (a bf16 baseline for numerics checks)
        self.kernel_path = True
        self.plugin = plug.load(c.method) if c.method in PLUGIN_METHODS else None
        for i, blk in enumerate(self.transformer.h):
            kind = c.layer_mixers[i] if c.method in HYBRID else c.method
            if c.method in LINEAR:
                blk.attn = LinearMixer(c, i)
            elif c.method in SPARSE:
                blk.attn = SparseMixer(c, i)
            elif c.method in HYBRID and kind in LINEAR:
                blk.attn = LinearMixer(c, i, kind=kind)
            elif c.method in HYBRID and kind in SPARSE:
                blk.attn = SparseMixer(c, i, kind=kind)
            elif c.method in MLA or (c.method in HYBRID and kind in MLA):
                blk.attn = MLAAttention(c, i)
            if c.method in MOE and i >= c.moe_dense_layers:
                blk.mlp = MoEFFN(c.width, c.moe_experts, c.moe_topk, c.moe_ffn, c.moe_shared, c.moe_bias_rate,
                                 c.moe_aux_loss_coeff, c.moe_z_loss_coeff)
            if self.plugin and self.plugin.mixer:
                blk.attn = self.plugin.mixer(c, i)
            if self.plugin and self.plugin.ffn:
                blk.mlp = self.plugin.ffn(c, i)
            if not c.value_embeddings and hasattr(blk.attn, "ve_gate"):
                blk.attn.ve_gate = None
            if c.method == "deeploop":
                self.transformer.h[i] = DeepLoopBlock(blk, c.maximum_depth)
            elif c.method == "huginn":
                self.transformer.h[i] = SandwichBlock(blk)
            if self.plugin and self.plugin.block:
                self.transformer.h[i] = self.plugin.block(blk, c, i)
        if self.plugin:
            plug.check_shell(self)
        if c.method in ("ut_act", "ouro"):
            self.halter = nn.Linear(c.width, 1)
        if c.method == "huginn":
            self.state_adapter = Linear(2 * c.width, c.width, bias=False)
        if c.method == "hc":
            self.residual_maps = nn.ModuleList(HyperConnection(c.width, c.residual_streams, k, c.residual_gate_init)
                                               for k in range(2 * c.n_layer))
        elif c.method == "mhc":
            self.residual_maps = nn.ModuleList(ManifoldHyperConnection(c.width, c.residual_streams, k,
                                                                       c.residual_gate_init, c.sinkhorn_iterations)
                                               for k in range(2 * c.n_layer))
        elif c.method == "attnres":
            self.depth_queries = nn.Parameter(torch.empty(2 * c.n_layer + 1, c.width))
        for name in self._frozen_native():
            getattr(self, name).requires_grad_(False)

    # ------------------------------------------------------------------ init / state
    @torch.no_grad()
    def init_weights(self):
        super().init_weights()
        c = self.config
        if hasattr(self, "halter"):
            nn.init.normal_(self.halter.weight, std=c.width ** -.5)
            nn.init.constant_(self.halter.bias, -1.)
        if c.method == "deeploop":
            K = len(self.transformer.h)
            for blk in self.transformer.h:
                beta = blk.beta
                for proj, resid, gain in ((blk.attn.c_q, False, 1.), (blk.attn.c_k, False, 1.),
                                          (blk.attn.c_v, False, beta), (blk.attn.c_proj, True, beta),
                                          (blk.mlp.c_fc, False, beta), (blk.mlp.c_proj, True, beta)):
                    n_out, n_in = proj.weight.shape
                    std = (.5 / n_in ** .5) * min(1., (n_out / n_in) ** .5)
                    if resid:
                        std /= K
                    nn.init.normal_(proj.weight, mean=0., std=std * gain)
            for e in self.value_embeds.values():
                e.weight.mul_((8 * c.maximum_depth) ** -.5)
        for m in getattr(self, "residual_maps", ()):
            m.reset_parameters()
        if hasattr(self, "depth_queries"):
            nn.init.zeros_(self.depth_queries)
        for blk in self.transformer.h:
            if isinstance(blk.attn, MLAAttention):
                blk.attn.init_weights()
        if self.plugin and self.plugin.init:
            self.plugin.init(self)

    def _frozen_native(self):
        if self.plugin:
            return tuple(self.plugin.frozen or ())
        return FROZEN_NATIVE.get(self.config.method, ())

    def set_step(self, step):
        if not 0 <= step <= self.total_steps:
            raise ValueError("optimizer step outside the schedule")
        self.optimizer_step = int(step)
        for blk in self.transformer.h:
            if isinstance(blk.attn, SparseMixer):
                blk.attn.in_burnin = int(step) < self.config.burnin_steps
        if self.plugin:
            for m in self.modules():
                if m is not self and callable(getattr(m, "set_step", None)):
                    m.set_step(int(step))

    def set_sparse_backend(self, backend):
        if backend not in SPARSE_BACKENDS:
            raise ValueError(f"unknown sparse backend {backend!r}")
        for blk in self.transformer.h:
            if isinstance(blk.attn, SparseMixer):
                blk.attn.backend = backend

    def set_row_offset(self, offset):
        if offset < 0:
            raise ValueError("row offset must be non-negative")
        self.row_offset = int(offset)

    def routing_rng_state(self):
        return dict(policy="step-keyed-depth/row-keyed-state-v1", seed=self.config.routing_seed,
                    optimizer_step=self.optimizer_step, row_offset=self.row_offset)

    def restore_routing_rng(self, state):
        if state["policy"] != "step-keyed-depth/row-keyed-state-v1" or state["seed"] != self.config.routing_seed:
            raise ValueError("routing RNG policy changed")
        self.set_step(state["optimizer_step"])
        self.set_row_offset(state["row_offset"])

    def set_training_stage(self, step):
        """Ouro's last ``ouro_gate_steps`` updates train only the exit gate."""
        self.set_step(step)
        gate_only = self.config.method == "ouro" and step >= self.total_steps - self.config.ouro_gate_steps
        frozen = self._frozen_native()
        for name, p in self.named_parameters():
            if name in frozen:
                continue
            p.requires_grad_(not gate_only or name.startswith("halter."))
        return "gate_only" if gate_only else "joint"

    def update_router_bias(self):
        for m in self.modules():
            if isinstance(m, MoEFFN):
                m.update_bias()

    # ------------------------------------------------------------------ forward pieces
    def _record(self, kind, **fields):
        self.last_trace.append(dict(kind=kind, backward=torch.is_grad_enabled() and self.training, **fields))

    def _embed(self, idx):
        x = self.embed(idx)
        self._record("embedding", tokens=idx.numel())
        return x

    def _window(self, virtual, total):
        c = self.config
        if c.method in HYBRID:
            if c.layer_mixers[virtual] == "swa":
                return (c.sliding_window - 1, 0)
            return (c.sequence_len, 0)
        short = -(-c.sequence_len // 4 // 128) * 128
        long = virtual == total - 1 or c.window_pattern[virtual % len(c.window_pattern)] == "L"
        return (c.sequence_len if long else short, 0)

    def _cos_sin(self, T):
        return self.cos[:, :T], self.sin[:, :T]

    def _block(self, x, x0, idx, physical, virtual, total, alive=None):
        c = self.config
        mixed = x if c.method == "deeploop" else self.resid_lambdas[physical] * x + self.x0_lambdas[physical] * x0
        ve = self.value_embeds[str(physical)](idx).to(x.dtype) if str(physical) in self.value_embeds else None
        window = self._window(virtual, total)
        out = self.transformer.h[physical](mixed, ve, self._cos_sin(idx.shape[1]), window, None)
        if alive is not None:
            out = torch.where(alive[..., None], out, x)
        kind = c.layer_mixers[physical] if c.method in HYBRID else c.method
        self._record("block", physical=physical, virtual=virtual, window=window[0], tokens=idx.numel(),
                     sequence_len=idx.shape[1], ve=ve is not None,
                     mixer=kind if kind in LINEAR | SPARSE | MLA | PLUGIN_METHODS else "softmax")
        return out

    def _readout_trace(self, x, backout):
        logits = self.readout(x, backout)
        self._record("head", tokens=x.shape[0] * x.shape[1])
        return logits

    @staticmethod
    def _token_loss(logits, targets):
        return F.cross_entropy(logits.flatten(0, 1), targets.flatten(), ignore_index=-1,
                               reduction="none").reshape_as(targets)

    def _ordinary_hidden(self, idx):
        c = self.config
        x = self._embed(idx)
        x0, cached = x, None
        if c.method in LOOPED:
            core = list(range(c.pre_layers, c.pre_layers + c.core_layers))
            ids = [*range(c.pre_layers), *core * c.loops, *range(c.pre_layers + c.core_layers, c.n_layer)]
        else:
            ids = list(range(c.n_layer))
        for v, p in enumerate(ids):
            x = self._block(x, x0, idx, p, v, len(ids))
            if v == len(ids) // 2:
                cached = x
        return x, cached

    def _attention_branch(self, x, idx, physical):
        c = self.config
        T = idx.shape[1]
        ve = self.value_embeds[str(physical)](idx).to(x.dtype) if str(physical) in self.value_embeds else None
        window = self._window(physical, c.n_layer)
        out = self.transformer.h[physical].attn(norm(x), ve, self._cos_sin(T), window, None)
        self._record("block", physical=physical, virtual=physical, window=window[0], tokens=idx.numel(),
                     sequence_len=T, ve=ve is not None, mixer="softmax", residual=c.method)
        return out

    def _residual_hidden(self, idx):
        c = self.config
        x = self._embed(idx)
        mlp = lambda h, p: self.transformer.h[p].mlp(norm(h))
        if c.method == "residual_standard":
            for i in range(c.n_layer):
                x = x + self._attention_branch(x, idx, i)
                x = x + mlp(x, i)
            return x
        if c.method in ("hc", "mhc"):
            streams = x[:, :, None].expand(-1, -1, c.residual_streams, -1)
            for k, hyper in enumerate(self.residual_maps):
                h, mixed, w = hyper.read(streams)
                out = self._attention_branch(h, idx, k // 2) if k % 2 == 0 else mlp(h, k // 2)
                streams = hyper.write(mixed, out, w)
                self._record("residual_map", sublayer=k, streams=c.residual_streams, tokens=idx.numel())
            return streams.sum(2)
        return self._attnres_trunk(idx, x, c.attnres_group_starts)

    def _attnres_trunk(self, idx, x, group_starts, adapt=None):
        """Block AttnRes: sublayer k reads a softmax mixture over its depth sources (the embedding,
        the sums of completed groups and the current group's partial sum, keyed by their RMSNorm)
        through pseudo-query ``depth_queries[k]``; a group closes at each layer in
        ``group_starts``.  ``adapt(k, h)`` (optional) transforms a sublayer's input after the read."""
        c = self.config
        starts = set(group_starts)
        closed, keys, partial = [], [], x
        for k in range(2 * c.n_layer):
            layer, is_attention = divmod(k, 2)[0], k % 2 == 0
            key = norm(partial)
            h = depth_attention(self.depth_queries[k], closed + [partial], keys + [key])
            self._record("depth_read", sublayer=k, sources=len(closed) + 1, tokens=idx.numel())
            if is_attention and layer in starts:
                closed.append(partial)
                keys.append(key)
                partial = None
            if adapt is not None:
                h = adapt(k, h)
            out = self._attention_branch(h, idx, layer) if is_attention else self.transformer.h[layer].mlp(norm(h))
            partial = out if partial is None else partial + out
        h = depth_attention(self.depth_queries[-1], closed + [partial], keys + [norm(partial)])
        self._record("depth_read", sublayer=2 * c.n_layer, sources=len(closed) + 1, tokens=idx.numel())
        return h

    def _loop_hidden(self, idx, targets=None):
        c = self.config
        gate_stage = c.method == "ouro" and self.optimizer_step >= self.total_steps - c.ouro_gate_steps
        guard = torch.no_grad if gate_stage else nullcontext
        with guard():
            x = self._embed(idx)
            x0 = x
            for i in range(c.pre_layers):
                x = self._block(x, x0, idx, i, i, c.maximum_depth)
        prelude = x
        n = c.max_loops
        if c.method == "huginn":
            n = getattr(self, "accounting_depth", None) or (huginn_depth(c, self.optimizer_step) if self.training
                                                             else c.eval_loops)
            noise = []
            for row in range(idx.shape[0]):
                g = torch.Generator(device=idx.device).manual_seed(c.routing_seed + self.row_offset + row)
                noise.append(torch.randn((1, *x.shape[1:]), device=x.device, dtype=x.dtype, generator=g))
            x = torch.cat(noise, 0) * c.width ** -.5
        total = c.pre_layers + n * c.core_layers + c.post_layers
        alive = torch.ones(idx.shape, dtype=torch.bool, device=idx.device)
        cum = x.new_zeros(idx.shape, dtype=torch.float32)
        remainder = torch.zeros_like(cum)
        updates = torch.zeros_like(cum)
        weighted = torch.zeros_like(x)
        gates, logits_list, losses, masses = [], [], [], []
        for r in range(n):
            no_grad = gate_stage or (c.method == "huginn" and r < n - c.huginn_backprop_loops)
            with torch.no_grad() if no_grad else nullcontext():
                if c.method == "ut_act":
                    coords = sinusoidal_coordinates(idx.shape[1], c.width, r + 1, x.device, x.dtype)
                    x = torch.where(alive[..., None], x + coords, x)
                if c.method == "huginn":
                    if r == n - c.huginn_backprop_loops:
                        x = x.detach()
                    x = norm(self.state_adapter(torch.cat((x, prelude), -1)))
                    self._record("state_adapter", tokens=idx.numel())
                if c.method == "ut_act":
                    p = self.halter(norm(x.float())).squeeze(-1).sigmoid()
                    weight, cum, next_alive, rem = act_weights(p, cum, alive, r == n - 1, c.act_epsilon)
                    remainder = remainder + rem
                    updates = updates + alive
                    self._record("act_gate", tokens=idx.numel())
                for j in range(c.core_layers):
                    x = self._block(x, x0, idx, c.pre_layers + j, c.pre_layers + r * c.core_layers + j, total,
                                    alive=alive if c.method == "ut_act" else None)
                if c.method == "ut_act":
                    weighted = weighted + weight[..., None].to(x.dtype) * x
                    masses.append(weight)
                    alive = next_alive
            if c.method == "ouro":
                with guard():
                    y = x
                    for j in range(c.post_layers):
                        y = self._block(y, x0, idx, c.pre_layers + c.core_layers + j,
                                        c.pre_layers + (r + 1) * c.core_layers + j, total)
                    logits = self._readout_trace(y, prelude)
                    logits_list.append(logits)
                    if targets is not None:
                        losses.append(self._token_loss(logits, targets))
                if r < n - 1:
                    gates.append(self.halter(norm(y.detach().float() if gate_stage else y.float())).squeeze(-1))
                    self._record("ouro_gate", tokens=idx.numel())
        if c.method == "ouro":
            dist = exit_distribution(gates)
            self.last_stats.update(exit_distribution=dist.detach(), stage="gate_only" if gate_stage else "joint")
            if not self.training:
                sel = (dist.cumsum(-1) < c.ouro_exit_quantile).sum(-1).clamp_max(n - 1)
                stack = torch.stack(logits_list, -2)
                logits = stack.gather(-2, sel[..., None, None].expand(*sel.shape, 1, stack.shape[-1])).squeeze(-2)
                return logits, x.new_zeros(()), None
            if targets is None:
                return logits_list[-1], x.new_zeros(()), None
            mask = (targets != -1).to(dist.dtype)
            den = mask.sum().clamp_min(1)
            if gate_stage:
                aux = (ouro_gate_loss(gates, losses) * mask[..., None]).sum() / (den * n)
                token_loss, objective = losses[-1].detach(), aux
            else:
                token_loss = (dist * torch.stack(losses, -1)).sum(-1)
                ent = -(dist * dist.clamp_min(1e-12).log()).sum(-1)
                aux = -c.ouro_entropy_weight * (ent * mask).sum() / den
                objective = (token_loss * mask).sum() / den + aux
            return logits_list[-1], aux, (token_loss, objective)
        if c.method == "ut_act":
            x = weighted
            aux = c.ponder_weight * (updates + remainder).mean()
            self.last_stats.update(act_weights=torch.stack(masses, -1).detach(), mean_loops=float(updates.mean()))
        else:
            aux = x.new_zeros(())
            self.last_stats.update(sampled_loops=n, backprop_loops=min(n, c.huginn_backprop_loops))
        for j in range(c.post_layers):
            x = self._block(x, x0, idx, c.pre_layers + c.core_layers + j, c.pre_layers + n * c.core_layers + j, total)
        return self._readout_trace(x, prelude), aux, None

    def fused_supported(self):
        """True when the trunk runs ``models.fused_dense.fused_forward``: one ordinary pass over
        plain blocks (dense, sliding-window, linear, sparse, MLA, hybrid and MoE layers); looped,
        residual-stream and plugin methods run their own forward, with every eligible projection
        still on the GEMM engine."""
        from nexttransformer_b200.models.shell import Block
        c = self.config
        return (c.method not in LOOPED | RESIDUAL and self.plugin is None
                and all(type(b) is Block for b in self.transformer.h))

    def layer_window(self, i):
        return self._window(i, self.config.n_layer)[0]

    def forward(self, idx, targets=None, kv_cache=None, loss_reduction="mean"):
        c = self.config
        if idx.ndim != 2 or not 0 < idx.shape[1] <= c.sequence_len:
            raise ValueError("rows must be packed with 0 < T <= context")
        if kv_cache is not None:
            raise NotImplementedError("KV-cache decoding goes through nexttransformer_b200.inference")
        self.last_trace, self.last_stats = [], {}
        if (idx.is_cuda and targets is not None and loss_reduction == "mean" and self.training
                and self.kernel_path and self.fused_supported()):
            from nexttransformer_b200.models.fused_dense import fused_forward
            loss, aux = fused_forward(self, idx, targets, "mean")
            aux = loss.new_zeros(()) if aux is None else aux
            self.last_lm_loss, self.last_aux_loss = loss.detach(), aux
            self.last_stats = {"fused_dense": True}
            return loss + aux
        if c.method == "dense":
            # the SSSL anchor is the shell's own forward (same graph the cost anchor audits)
            out = self.forward_eager(idx, targets, loss_reduction)
            self.last_stats = {"native_dense_delegate": True}
            return out
        special = None
        if c.method in ("ut_act", "huginn", "ouro"):
            logits, aux, special = self._loop_hidden(idx, targets)
        elif c.method in RESIDUAL:
            logits = self._readout_trace(self._residual_hidden(idx), None)
            aux = logits.new_zeros(())
        else:
            x, cached = self._ordinary_hidden(idx)
            logits = self._readout_trace(x, cached)
            aux_src = (m for m in self.modules() if m is not self) if self.plugin else \
                [*(b.attn for b in self.transformer.h if isinstance(b.attn, (LinearMixer, SparseMixer))),
                 *(b.mlp for b in self.transformer.h if isinstance(b.mlp, MoEFFN))]
            aux = sum((m.last_aux for m in aux_src if torch.is_tensor(getattr(m, "last_aux", None))),
                      logits.new_zeros(()))
        self.last_aux_loss = aux
        if targets is None:
            return logits
        tok = self._token_loss(logits, targets)
        mask = (targets != -1).to(tok.dtype)
        self.last_lm_loss = (tok * mask).sum() / mask.sum().clamp_min(1)
        if loss_reduction == "none":
            return tok.flatten()
        if loss_reduction == "sum":
            return tok.sum()
        if loss_reduction != "mean":
            raise ValueError("invalid loss reduction")
        if self.training and special is not None:
            return special[1]
        return self.last_lm_loss + (aux if self.training else 0)


def construct(config: ModelConfig):
    """The model on the meta device (no storage)."""
    hooks = plug.load(config.method) if config.method in PLUGIN_METHODS else None
    with torch.device("meta"):
        return (hooks.model if hooks and hooks.model else LanguageModel)(config)


def materialize(model, device):
    """Allocate a meta-constructed model on `device` and run the reference-order initialisation."""
    config = model.config
    model.to_empty(device=device)
    from nexttransformer_b200.models.linear import CausalDepthwise
    for m in model.modules():
        if isinstance(m, (nn.Linear, nn.LayerNorm)):
            m.reset_parameters()
        elif isinstance(m, CausalDepthwise):
            nn.init.normal_(m.weight, std=m.size ** -.5)
    for m in model.modules():
        if isinstance(m, LinearMixer):
            if hasattr(m, "output_gain"):
                nn.init.ones_(m.output_gain)
            if m.kind == "gdn":
                init_gdn_gate(m.log_decay, m.dt_bias)
            elif hasattr(m, "log_decay"):
                nn.init.zeros_(m.log_decay)
                nn.init.constant_(m.dt_bias, -3.)
        if isinstance(m, SparseMixer) and hasattr(m, "compress_position"):
            nn.init.zeros_(m.compress_position)
        if isinstance(m, MoEFFN):
            m.expert_bias.zero_()
            m.load.zero_()
            nn.init.normal_(m.router.weight, std=0.02)
    if config.method in PLUGIN_METHODS:
        plug.reset(model)
    model.init_weights()
    return model


def build_model(config: ModelConfig, device="cpu", seed=42):
    """Meta construction -> materialise on `device` -> reference-order initialisation."""
    torch.manual_seed(seed)
    model = construct(config)
    if str(device) == "meta":
        return model
    return materialize(model, device)
