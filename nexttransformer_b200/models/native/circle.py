"""Circle: a ring of ``core_layers`` blocks run for up to ``circle_max_steps`` steps with sparse,
absorbing per-token exits.

The first full ring is dense.  After each later step every still-active token gets an exit score
from the halter (from the states before and after the step); a token continues while
``sigmoid(-score) >= 0.5``, its update ``before + q * (candidate - before)`` is weighted by that gate,
and once stopped it never resumes.  During the random warm-up and the route transition a growing
fraction of tokens follows depths drawn from the depth law instead (routing RNG per rank, saved in
checkpoints).  The budget sees the hard survival counts in forward and local straight-through gate
derivatives in backward.  Behaviour: ``nexttransformer/models/native/circle.py:6-93``.
"""
import torch
import torch.distributed as dist


class SparseCircleMixin:
    def set_circle_step(self, step):
        if step < 0:
            raise ValueError("Circle curriculum step must be nonnegative")
        self.circle_step = step

    def learned_route_fraction(self):
        if not self.training:
            return 1.0
        c = self.config
        since = getattr(self, "circle_step", 0) - c.circle_random_warmup
        if since < 0:
            return 0.0
        return min(1.0, (since + 1) / max(1, c.circle_route_transition))

    def circle_stage(self):
        f = self.learned_route_fraction()
        return "random_warmup" if f == 0 else "learned" if f == 1 else "route_transition"

    def routing_generator(self, device):
        if getattr(self, "_routing_generator", None) is None:
            rank = dist.get_rank() if dist.is_initialized() else 0
            gen = torch.Generator(device=device).manual_seed(self.config.circle_routing_seed + rank)
            saved = getattr(self, "_routing_state", None)
            if saved is not None:
                gen.set_state(saved)
                self._routing_state = None
            self._routing_generator = gen
        return self._routing_generator

    def routing_rng_state(self):
        gen = getattr(self, "_routing_generator", None)
        return gen.get_state() if gen is not None else getattr(self, "_routing_state", None)

    def restore_routing_rng(self, state):
        self._routing_generator = None
        self._routing_state = state

    def _circle_random_routes(self, idx):
        f = self.learned_route_fraction()
        if f == 1:
            return torch.zeros_like(idx, dtype=torch.bool), None
        gen = self.routing_generator(idx.device)
        forced = torch.rand(idx.shape, device=idx.device, generator=gen) >= f
        u = torch.rand(idx.shape, device=idx.device, generator=gen)
        c = self.config
        depth = torch.searchsorted(self.circle_budget.probabilities.cumsum(0), u.double().contiguous())
        return forced, depth.clamp_max(c.circle_max_steps - c.core_layers) + c.core_layers

    def _sparse_circle(self, x, idx, run):
        c = self.config
        active = torch.ones_like(idx, dtype=torch.bool)
        forced, depths = self._circle_random_routes(idx)
        gate, survival = None, []
        pending = x.new_tensor(1.0, dtype=torch.float32)
        anchor = x.new_zeros((), dtype=torch.float32)
        backout = None
        for s in range(1, c.circle_max_steps + 1):
            n_active = int(active.sum())
            self.last_stats["active_tokens"][s - 1] = n_active
            survival.append(pending)
            before = x
            cand = run(c.pre_layers + (s - 1) % c.core_layers, x, active=None if s <= c.core_layers else active)
            x = cand if gate is None else before + gate.to(x.dtype)[..., None] * (cand - before)
            if c.pre_layers + s - 1 == c.max_depth // 2:
                backout = x
            if s < c.core_layers:
                continue
            if s == c.circle_max_steps:
                break
            score = self.halter(before[active], x[active], s - c.core_layers)
            q = torch.zeros_like(idx, dtype=torch.float32).masked_scatter(active, torch.sigmoid(-score))
            self.last_stats["forward_flops"] += 2 * n_active * c.width
            self.last_stats["halter_extra_forward_ops"] += n_active * (5 * c.width + 10)
            keep = q >= 0.5
            if depths is not None:
                keep = torch.where(forced, depths > s, keep)
            nxt = active & keep
            straight = nxt.float() + (active & ~forced).float() * (q - q.detach())
            pending = straight.mean() + anchor
            anchor = anchor + q.sum() * 0      # keeps every gate in the graph after an empty tail
            active, gate = nxt, q
        penalty, depth_loss, shape_loss = self.circle_budget.penalty(torch.stack(survival))
        if not self.training:
            penalty = x.new_zeros((), dtype=torch.float32)
        self.last_stats["active_depth_sum"] = (idx.numel() * (c.pre_layers + c.post_layers)
                                               + sum(self.last_stats["active_tokens"]))
        self.last_stats["circle_depth_loss"] = depth_loss.detach()
        self.last_stats["circle_shape_loss"] = shape_loss.detach()
        return x, penalty, backout
