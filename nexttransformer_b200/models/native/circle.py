"""Circle: the core ring of ``core_layers`` blocks run for up to ``circle_max_steps`` steps with
sparse, absorbing per-token exits.

Schedule of one forward:

* steps 1 .. ring: every token runs (the first pass around the ring is dense);
* after each step s in [ring, max_steps): the halter scores every still-active token from its
  states before and after the step; the continue-gate is ``q = sigmoid(-score)`` and the token
  stays active for step s + 1 iff ``q >= 0.5``.  A stopped token never resumes.  The next step's
  update of a token is ``before + q (candidate - before)``, so the gate is trained through the
  states it blends;
* curriculum: during the random warm-up every token (during the route transition a growing
  fraction of tokens) instead follows a depth drawn from the population depth law, with a
  per-rank routing generator whose state is checkpointed.

The budget sees the hard survival fractions in the forward and the straight-through derivative
of the learned gates in the backward.  Behaviour matches ``nexttransformer/models/native/circle.py``.
"""
import torch
import torch.distributed as dist


class _Route:
    """Per-forward routing state: which tokens are active, the gate of the last exit decision, the
    tokens forced onto law-drawn depths, and the survival curve the budget penalises."""

    def __init__(self, model, idx, like):
        self.active = torch.ones_like(idx, dtype=torch.bool)
        self.forced, self.law_depth = model._circle_random_routes(idx)
        self.gate = None
        self.curve = []
        self.carry = like.new_tensor(1.0, dtype=torch.float32)
        # a zero-valued term that keeps every gate in the graph even after the last token has stopped
        self.anchor = like.new_zeros((), dtype=torch.float32)

    def enter(self, step, stats):
        """Record the active count and the survival value of step ``step`` (1-based)."""
        count = int(self.active.sum())
        stats["active_tokens"][step - 1] = count
        self.curve.append(self.carry)
        return count

    def blend(self, before, candidate):
        if self.gate is None:
            return candidate
        return before + self.gate.to(candidate.dtype)[..., None] * (candidate - before)

    def decide(self, model, step, before, after, count):
        """Score the active tokens after ``step`` and choose who continues."""
        c = model.config
        live = self.active
        score = model.halter(before[live], after[live], step - c.core_layers)
        q = torch.zeros(live.shape, device=live.device, dtype=torch.float32).masked_scatter(live, torch.sigmoid(-score))
        model.last_stats["forward_flops"] += 2 * count * c.width
        model.last_stats["halter_extra_forward_ops"] += count * (5 * c.width + 10)
        stay = q >= 0.5
        if self.law_depth is not None:
            stay = torch.where(self.forced, self.law_depth > step, stay)
        nxt = live & stay
        learned = (live & ~self.forced).float()
        self.carry = (nxt.float() + learned * (q - q.detach())).mean() + self.anchor
        self.anchor = self.anchor + q.sum() * 0
        self.active, self.gate = nxt, q


class SparseCircleMixin:
    # ------------------------------------------------------------------ curriculum
    def set_circle_step(self, step):
        if step < 0:
            raise ValueError("the Circle curriculum step cannot be negative")
        self.circle_step = step

    def learned_route_fraction(self):
        """Share of tokens routed by the halter: 0 in the warm-up, ramping to 1 over the transition
        (always 1 outside training)."""
        if not self.training:
            return 1.0
        c = self.config
        elapsed = getattr(self, "circle_step", 0) - c.circle_random_warmup + 1
        if elapsed <= 0:
            return 0.0
        return min(1.0, elapsed / max(1, c.circle_route_transition))

    def circle_stage(self):
        share = self.learned_route_fraction()
        if share == 0:
            return "random_warmup"
        return "learned" if share == 1 else "route_transition"

    # ------------------------------------------------------------------ routing generator
    def routing_generator(self, device):
        gen = getattr(self, "_routing_generator", None)
        if gen is None:
            rank = dist.get_rank() if dist.is_initialized() else 0
            gen = torch.Generator(device=device).manual_seed(self.config.circle_routing_seed + rank)
            pending = getattr(self, "_routing_state", None)
            if pending is not None:
                gen.set_state(pending)
                self._routing_state = None
            self._routing_generator = gen
        return gen

    def routing_rng_state(self):
        gen = getattr(self, "_routing_generator", None)
        return getattr(self, "_routing_state", None) if gen is None else gen.get_state()

    def restore_routing_rng(self, state):
        self._routing_generator, self._routing_state = None, state

    def _circle_random_routes(self, idx):
        """(forced mask, law-drawn total depth) per token; (all False, None) once fully learned."""
        share = self.learned_route_fraction()
        if share == 1:
            return torch.zeros_like(idx, dtype=torch.bool), None
        gen = self.routing_generator(idx.device)
        forced = torch.rand(idx.shape, device=idx.device, generator=gen) >= share
        draw = torch.rand(idx.shape, device=idx.device, generator=gen)
        c = self.config
        cdf = self.circle_budget.probabilities.cumsum(0)
        extra = torch.searchsorted(cdf, draw.double().contiguous()).clamp_max(c.circle_max_steps - c.core_layers)
        return forced, extra + c.core_layers

    # ------------------------------------------------------------------ the ring
    def _sparse_circle(self, x, idx, run):
        c = self.config
        ring, limit = c.core_layers, c.circle_max_steps
        route = _Route(self, idx, x)
        backout = None
        for step in range(1, limit + 1):
            count = route.enter(step, self.last_stats)
            before = x
            candidate = run(c.pre_layers + (step - 1) % ring, x, active=route.active if step > ring else None)
            x = route.blend(before, candidate)
            if c.pre_layers + step - 1 == c.max_depth // 2:
                backout = x
            if ring <= step < limit:
                route.decide(self, step, before, x, count)
        penalty, depth_loss, shape_loss = self.circle_budget.penalty(torch.stack(route.curve))
        if not self.training:
            penalty = x.new_zeros((), dtype=torch.float32)
        stats = self.last_stats
        stats["active_depth_sum"] = idx.numel() * (c.pre_layers + c.post_layers) + sum(stats["active_tokens"])
        stats["circle_depth_loss"] = depth_loss.detach()
        stats["circle_shape_loss"] = shape_loss.detach()
        return x, penalty, backout
