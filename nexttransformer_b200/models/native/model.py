"""Native-track models on the shared nanochat shell: SSSL Dense, MoR, LoopFormer, Circle.

* Dense is the shell's own forward.
* MoR runs the core ring three times; before recursions 2 and 3 a router scores every token
  (``sigmoid`` of a linear score of the RMS-normalised state) and hard-gated survivors (straight-
  through in training) are compacted: the surviving tokens of each row are gathered in position order,
  keep their original RoPE positions and window distances (explicit attention mask), and their block
  deltas are scattered back.  The recursion's update is weighted by the router probability.
* LoopFormer runs the ring twice with bounded, time-conditioned modulation of each block.
* Circle: see ``circle.py``.
Training returns the loss dict of the reference (``loss, lm_loss, router_loss, objective,
compute_loss``) with every parameter kept in the graph (zero-weighted) so skipped blocks still get
gradients on every rank.  ``last_stats`` counts forward FLOPs of the executed (padded) work.
Behaviour: ``nexttransformer/models/native/model.py:21-297`` of the reference.
"""
import torch
from torch import nn
import torch.nn.functional as F

from nexttransformer_b200.models.native.budget import CircleBudget, SurvivalBudget
from nexttransformer_b200.models.native.circle import SparseCircleMixin
from nexttransformer_b200.models.native.conditioning import LoopConditioner
from nexttransformer_b200.models.native.depth import depth_reference
from nexttransformer_b200.models.native.halter import DeltaDepthHalter
from nexttransformer_b200.models.shell import GPTShell, ShellConfig, apply_rotary_emb, norm
from nexttransformer_b200.models import shell
from nexttransformer_b200.utils.dtype import COMPUTE_DTYPE


def uses_value_embeddings(config):
    return getattr(config, "value_embeddings", True)


def _causal_route(x, w, n):
    """Compacted attention through the causal kernel: on CUDA when the window covers the sequence."""
    return x.is_cuda and w[0] >= n - 1


def window(config, virtual):
    short = -(-config.sequence_len // 4 // 128) * 128
    full = virtual == config.max_depth - 1 or config.window_pattern[virtual % len(config.window_pattern)] == "L"
    return (config.sequence_len if full else short, 0)


def block_forward_flops(config, batch, queries, keys=None, window_size=None):
    """Matmul FLOPs of one block's forward (the upstream ``estimate_flops / 3`` convention; padded
    rectangular attention for the compacted sparse paths)."""
    d = config.width
    k = queries if keys is None else keys
    seen = min(k, window_size[0]) if window_size is not None else k
    return batch * (24 * queries * d * d + 4 * queries * seen * d)


def _physical(c, j, n_virtual):
    if c.architecture == "dense" or j < c.pre_layers:
        return j
    if j >= n_virtual - c.post_layers:
        return c.pre_layers + c.core_layers + j - (n_virtual - c.post_layers)
    return c.pre_layers + (j - c.pre_layers) % c.core_layers


def theoretical_training_flops(config):
    """Training FLOPs per token at the ideal (target) route capacities."""
    c = config
    t, d = c.sequence_len, c.width
    if c.architecture == "mor":
        rates = [1.0] * c.pre_layers
        for r in (1.0, *c.mor_target_survival):
            rates += [r] * c.core_layers
        rates += [1.0] * c.post_layers
    elif c.architecture == "circle":
        _, ring = depth_reference(c.core_layers, c.circle_max_steps, c.circle_target_steps)
        rates = [1.0] * c.pre_layers + list(ring) + [1.0] * c.post_layers
    else:
        rates = [1.0] * c.max_depth
    fwd = 2 * t * d * c.vocab_size + 2 * t * 24
    for j, rate in enumerate(rates):
        n = t * rate
        sparse = ((c.architecture == "mor" and rate < 1)
                  or (c.architecture == "circle" and c.pre_layers + c.core_layers <= j < len(rates) - c.post_layers))
        fwd += block_forward_flops(c, 1, n, window_size=None if sparse else window(c, j))
        if uses_value_embeddings(c) and _physical(c, j, len(rates)) % 2 == (c.n_layer - 1) % 2:
            fwd += 24 * c.heads * n
    if c.architecture == "mor":
        fwd += 2 * (c.recursions - 1) * t * d
    if c.architecture == "circle":
        fwd += 2 * t * d * sum(ring[c.core_layers - 1:-1])
    if c.architecture == "loopformer":
        fwd += c.recursions * (4 * (c.fourier_dim * d + d * d) + 8 * c.core_layers * d * d)
    return 3 * fwd / t


class NativeExperiment(SparseCircleMixin, GPTShell):
    def __init__(self, config):
        super().__init__(ShellConfig(sequence_len=config.sequence_len, vocab_size=config.vocab_size,
                                     n_layer=config.n_layer, n_head=config.heads, n_kv_head=config.heads,
                                     n_embd=config.width, window_pattern=config.window_pattern))
        self.config = config
        self.max_seq_len = config.sequence_len
        self.last_stats = {}
        # Dense training steps on CUDA may run the shell's fused sm_100a path; the trainer that sets
        # this also owns the bf16 shadows (optimizer) and zeroes the fused gradients per update.
        self.use_fused = False
        if not uses_value_embeddings(config):
            self.value_embeds = nn.ModuleDict()
            for blk in self.transformer.h:
                blk.attn.ve_gate = None
        arch = config.architecture
        if arch == "mor":
            self.routers = nn.ModuleList(nn.Linear(config.width, 1) for _ in range(config.recursions - 1))
            self.survival_budget = SurvivalBudget(config)
        elif arch == "circle":
            self.halter = DeltaDepthHalter(config.width, config.circle_max_steps - config.core_layers,
                                           config.circle_halter_eps)
            self.circle_budget = CircleBudget(config)
        elif arch == "loopformer":
            self.conditioner = LoopConditioner(config)

    @torch.no_grad()
    def init_weights(self):
        super().init_weights()
        c = self.config
        if c.architecture == "mor":
            prev = 1.0
            for router, target in zip(self.routers, c.mor_target_survival):
                nn.init.normal_(router.weight, std=c.width ** -0.5)
                # scores have about unit variance after RMSNorm: start at the target quantile
                nn.init.constant_(router.bias, float(torch.distributions.Normal(0., 1.).icdf(
                    torch.tensor(target / prev))))
                prev = target
            self.survival_budget.reset()
        elif c.architecture == "circle":
            self.circle_budget.reset()
            _, surv = depth_reference(c.core_layers, c.circle_max_steps, c.circle_target_steps)
            self.halter.init_weights([surv[s] / surv[s - 1] for s in range(c.core_layers, c.circle_max_steps)])
        elif c.architecture == "loopformer":
            self.conditioner.init_weights()

    def _fresh_stats(self, idx):
        return dict(input_tokens=idx.numel(), forward_flops=0., recompute_flops=0.,
                    active_tokens=[0] * self.config.routing_steps, active_depth_sum=0., halter_extra_forward_ops=0.)

    def _embed_native(self, idx):
        x = self.embed(idx)
        self.last_stats["forward_flops"] += 2 * idx.numel() * 24
        return x

    # ------------------------------------------------------------------ one block, three ways
    def _full_block(self, h, ve, blk, w, rope, conditioning):
        """The block on every token: plain, or with LoopFormer's bounded offsets around identity
        (output gates and input scales act as ``1 + offset``, so zero offsets leave the block as is
        and a zero-initialised output projection still receives gradient)."""
        if conditioning is None:
            return blk(h, ve, rope, w, None)
        gate_attn, gate_mlp, scale_attn, scale_mlp = (o[:, None] for o in conditioning.to(h.dtype).chunk(4, -1))
        mixed = h + (1 + gate_attn) * blk.attn(norm(h) * (1 + scale_attn), ve, rope, w, None)
        return mixed + (1 + gate_mlp) * blk.mlp(norm(mixed) * (1 + scale_mlp))

    def _compacted_block(self, x, x0, idx, physical, w, active):
        """The block on the active tokens only: each row's active tokens are gathered in position
        order (padded to the longest row), attend with their original RoPE positions and window
        distances (explicit mask), and their block updates are scattered back.  Returns the new
        state and the number of gathered rows per sequence (None when no token is active)."""
        b, n, d = x.shape
        width = int(active.sum(1).max().item())
        if width == 0:
            return x, None
        c = self.config
        blk, a = self.transformer.h[physical], self.transformer.h[physical].attn
        order = torch.arange(n, device=x.device).expand(b, -1).masked_fill(~active, n).sort(1).values[:, :width]
        valid = order < n
        pos = order.clamp_max(n - 1)
        rows = pos[:, :, None].expand(-1, -1, d)
        mixed = self.resid_lambdas[physical] * x.gather(1, rows) + self.x0_lambdas[physical] * x0.gather(1, rows)
        z = norm(mixed)
        hd = d // c.heads
        q = a.c_q(z).view(b, width, c.heads, hd)
        k = a.c_k(z).view_as(q)
        v = a.c_v(z).view_as(q)
        if str(physical) in self.value_embeds:
            table = self.value_embeds[str(physical)](idx.gather(1, pos)).to(x.dtype).view_as(v)
            v = v + 3 * torch.sigmoid(a.ve_gate(z[..., :12])).unsqueeze(-1) * table
        cos, sin = self.cos[0, pos], self.sin[0, pos]
        q = norm(apply_rotary_emb(q, cos, sin)) * 1.2
        k = norm(apply_rotary_emb(k, cos, sin)) * 1.2
        if _causal_route(x, w, n):
            # full window: rows are sorted by position and padding rows follow every valid row, so the
            # mask below is plain causal in the compacted order for every valid query; the causal
            # attention kernel takes it (padding queries' outputs are discarded by `valid`)
            y = shell.sdpa(q, k, v, -1).reshape(b, width, d)
        else:
            lag = pos[:, :, None] - pos[:, None, :]
            visible = (lag >= 0) & (lag <= w[0]) & valid[:, :, None] & valid[:, None, :]
            y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               attn_mask=visible[:, None]).transpose(1, 2).reshape(b, width, d)
        out = mixed + a.c_proj(y)
        out = out + blk.mlp(norm(out))
        update = (out - x.gather(1, rows)) * valid[:, :, None].to(x.dtype)
        return x.scatter_add(1, rows, update), width

    def _layer(self, x, x0, idx, physical, virtual, conditioning=None, active=None):
        c = self.config
        b, n, _ = x.shape
        w = window(c, virtual)
        if active is None:
            h = self.resid_lambdas[physical] * x + self.x0_lambdas[physical] * x0
            ve = self.value_embeds[str(physical)](idx).to(x.dtype) if str(physical) in self.value_embeds else None
            out = self._full_block(h, ve, self.transformer.h[physical], w, (self.cos[:, :n], self.sin[:, :n]),
                                   conditioning)
            cost, rows = block_forward_flops(c, b, n, window_size=w), b * n
        else:
            out, width = self._compacted_block(x, x0, idx, physical, w, active)
            if width is None:
                return x
            cost, rows = block_forward_flops(c, b, width), b * width
        if str(physical) in self.value_embeds:
            cost += 24 * c.heads * rows
        self.last_stats["forward_flops"] += cost
        return out

    # ------------------------------------------------------------------ trunks
    def _mor_core(self, trunk, x_of, b, n, device):
        """Three passes over the ring; before passes 2 and 3 a router keeps tokens (hard gate in
        the forward, straight-through in training) and the pass's update is weighted by the router
        probability.  Returns the survival penalty."""
        c = self.config
        alive = torch.ones((b, n), device=device)
        means = []
        for r in range(c.recursions):
            prob = None
            if r:
                with torch.autocast(device_type=device.type, enabled=False):
                    logit = self.routers[r - 1](norm(x_of().float())).squeeze(-1)
                    prob = logit.sigmoid()
                    hard = (logit >= 0).float()
                    alive = alive * (hard - prob.detach() + prob if self.training else hard)
                means.append(alive.mean())
                self.last_stats["forward_flops"] += 2 * b * n * c.width
            active = alive.detach() > 0.5
            self.last_stats["active_tokens"][r] = int(active.sum())
            start = x_of()
            for i in range(c.core_layers):
                trunk(c.pre_layers + i, active=None if r == 0 else active)
            if prob is not None:
                trunk.state = start + prob.to(start.dtype)[:, :, None] * (trunk.state - start)
        self.last_stats["active_depth_sum"] = (b * n * (c.pre_layers + c.post_layers)
                                               + c.core_layers * sum(self.last_stats["active_tokens"]))
        return self.survival_budget.penalty(torch.stack(means)) if self.training else x_of().new_zeros(())

    def _loopformer_core(self, trunk, b, n, device):
        c = self.config
        for r in range(c.recursions):
            offsets = self.conditioner(r, b, device)
            self.last_stats["forward_flops"] += 4 * b * (c.fourier_dim * c.width + c.width * c.width)
            for i, offset in enumerate(offsets):
                self.last_stats["forward_flops"] += 8 * b * c.width * c.width
                trunk(c.pre_layers + i, conditioning=offset)
            self.last_stats["active_tokens"][r] = b * n
        self.last_stats["active_depth_sum"] = b * n * c.max_depth

    def _variant_hidden(self, idx):
        c = self.config
        b, n = idx.shape
        trunk = _Trunk(self, idx, self._embed_native(idx))
        for i in range(c.pre_layers):
            trunk(i)
        if c.architecture == "loopformer":
            self._loopformer_core(trunk, b, n, idx.device)
            penalty = trunk.state.new_zeros((), dtype=torch.float32)
        elif c.architecture == "mor":
            penalty = self._mor_core(trunk, lambda: trunk.state, b, n, idx.device)
        else:
            def step(physical, current, active=None):
                trunk.state = current
                trunk(physical, active=active)
                return trunk.state
            trunk.state, penalty, trunk.backout = self._sparse_circle(trunk.state, idx, step)
            trunk.state = norm(trunk.state)
        for i in range(c.post_layers):
            trunk(c.pre_layers + c.core_layers + i)
        x = trunk.state
        if trunk.backout is not None:
            x = x - self.backout_lambda.to(x.dtype) * trunk.backout
        return norm(x), penalty

    def forward(self, idx, targets=None, loss_reduction=None):
        if idx.shape[1] > self.max_seq_len:
            raise ValueError("input exceeds experiment context")
        self.last_stats = self._fresh_stats(idx)
        c = self.config
        if c.architecture == "dense":
            d = c.width
            per_tok = 2 * self.num_matmul_params() + sum(4 * d * min(w[0], idx.shape[1]) for w in self.window_sizes)
            self.last_stats.update(forward_flops=idx.numel() * per_tok, active_depth_sum=idx.numel() * c.dense_layers)
            if (self.use_fused and idx.is_cuda and targets is not None and loss_reduction is None and self.training
                    and self.fused_supported()):
                from nexttransformer_b200.models.fused_dense import fused_forward
                lm = fused_forward(self, idx, targets, "mean")[0]
                zero = lm.new_zeros(())
                return dict(loss=lm, lm_loss=lm, router_loss=zero, objective=lm.detach(), compute_loss=zero)
            logits = self.forward_eager(idx)
            penalty = logits.new_zeros(())
        else:
            hidden, penalty = self._variant_hidden(idx)
            logits = self.lm_head(hidden)[..., :c.vocab_size].float()
            logits = 15 * torch.tanh(logits / 15)
            self.last_stats["forward_flops"] += 2 * idx.numel() * c.width * self.lm_head.out_features
        if targets is None:
            return logits
        losses = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1), reduction="none",
                                 ignore_index=-1)
        if loss_reduction is not None:
            if loss_reduction == "none":
                return losses
            if loss_reduction == "sum":
                return losses.sum()
            if loss_reduction == "mean":
                return losses.mean()
            raise ValueError("invalid loss reduction")
        lm = losses.mean()
        keep = sum(p.reshape(-1)[0] * 0 for p in self.parameters()) if self.training else lm.new_zeros(())
        return dict(loss=lm + penalty + keep, lm_loss=lm, router_loss=penalty, objective=lm + penalty.detach(),
                    compute_loss=self.last_stats.get("circle_depth_loss", lm.new_zeros(())))

    def update_route_budget(self, counts, tokens, step):
        if not self.training:
            raise ValueError("cannot change routing budgets in evaluation")
        if self.config.architecture == "mor":
            return self.survival_budget.update(counts[1:], tokens, step)
        if self.config.architecture == "circle":
            return self.circle_budget.update(counts, tokens, step)
        return {}

    def estimate_flops(self):
        return theoretical_training_flops(self.config)


def build_model(config, device, seed=None):
    if seed is not None:
        torch.manual_seed(seed)
    with torch.device("meta"):
        model = NativeExperiment(config)
    model.to_empty(device=device)
    model.init_weights()
    return model


class _Trunk:
    """Runs blocks in depth order on a shared state: counts virtual depth and keeps the mid-depth
    state for the backout."""

    def __init__(self, model, idx, x):
        self.model, self.idx = model, idx
        self.state, self.x0 = x, x
        self.virtual = 0
        self.backout = None

    def __call__(self, physical, active=None, conditioning=None):
        model = self.model
        self.state = model._layer(self.state, self.x0, self.idx, physical, self.virtual, conditioning, active)
        if self.virtual == model.config.max_depth // 2:
            self.backout = self.state
        self.virtual += 1
