"""Compute budgets of the native track: Lagrangian dual ascent on measured route statistics.

Both budgets keep fp64 dual variables as buffers and move them once per complete optimizer update
from the globally reduced counts of that update (never from one micro-batch):

* MoR (``SurvivalBudget``): one dual per routed recursion on the survival error
  ``e = survival - target``; the training penalty is ``dual e + strength / 2 e^2`` (the forward
  measures hard survival, the backward follows the straight-through router surrogate) and the
  dual steps by ``dual_lr e``, clamped to ``+-dual_limit``.
* Circle (``CircleBudget``): one dual on the relative mean-depth error
  ``e = sum(survival) / target - 1``, smoothed by an EMA and enabled after the random warm-up,
  plus a weak quadratic pull of the survival curve beyond the first ring towards the depth law.

Buffer names are the reference's checkpoint keys; behaviour matches
``nexttransformer/models/native/budget.py``.
"""
import math

import torch
from torch import nn

from nexttransformer_b200.models.native.depth import depth_reference


class _UpdateClock(nn.Module):
    """Refuses a second budget update for the same optimizer step."""

    def __init__(self):
        super().__init__()
        self.register_buffer("updates", torch.zeros((), dtype=torch.long))
        self.register_buffer("last_step", torch.tensor(-1, dtype=torch.long))

    def admit(self, step, tokens, what):
        if tokens <= 0 or step <= int(self.last_step):
            raise ValueError(f"the {what} moves once per complete optimizer update")

    def tick(self, step):
        self.last_step.fill_(step)
        self.updates.add_(1)

    @torch.no_grad()
    def restart(self):
        self.updates.zero_()
        self.last_step.fill_(-1)


def dual_ascent(dual, step_size, error, limit):
    """dual <- clamp(dual + step_size * error, -limit, limit) in place."""
    dual.add_(step_size * error).clamp_(-limit, limit)


def quadratic_penalty(dual, error, weight):
    """dual . error + weight / 2 |error|^2 with the dual treated as a constant."""
    return dual.detach().clone().to(error) * error + 0.5 * weight * error.square()


class CircleBudget(_UpdateClock):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self._probs, self._surv = depth_reference(config.core_layers, config.circle_max_steps,
                                                  config.circle_target_steps)
        self.register_buffer("probabilities", torch.tensor(self._probs, dtype=torch.float64))
        self.register_buffer("survival", torch.tensor(self._surv, dtype=torch.float64))
        self.register_buffer("dual", torch.zeros((), dtype=torch.float64))
        self.register_buffer("ema", torch.zeros((), dtype=torch.float64))

    @torch.no_grad()
    def reset(self):
        """Every buffer back to its initial value (they are uninitialised after ``to_empty``)."""
        self.probabilities.copy_(torch.tensor(self._probs, dtype=torch.float64))
        self.survival.copy_(torch.tensor(self._surv, dtype=torch.float64))
        self.dual.zero_()
        self.ema.zero_()
        self.restart()

    def penalty(self, survival):
        """(total, depth term, shape term) for the survival curve of one forward."""
        c = self.config
        ring = c.core_layers
        depth = quadratic_penalty(self.dual, survival.sum() / c.circle_target_steps - 1, c.circle_depth_rho)
        gap = survival[ring:] - self.survival[ring:].to(survival)
        shape = c.circle_shape_weight * gap.square().mean()
        return depth + shape, depth, shape

    @staticmethod
    def _absorbing(surv, ring):
        """Counts of an absorbing exit process: in [0, 1], non-increasing, 1 through the first ring."""
        in_range = all(math.isfinite(v) and 0 <= v <= 1 for v in surv)
        monotone = all(nxt <= cur + 1e-9 for cur, nxt in zip(surv, surv[1:]))
        dense_ring = all(abs(v - 1) <= 1e-9 for v in surv[:ring])
        return in_range and monotone and dense_ring

    @torch.no_grad()
    def update(self, counts, tokens, step):
        c = self.config
        self.admit(step, tokens, "Circle budget")
        if len(counts) != c.circle_max_steps:
            raise ValueError("the Circle budget needs the active-token count of every step")
        surv = [float(n) / tokens for n in counts]
        if not self._absorbing(surv, c.core_layers):
            raise ValueError("Circle survival counts are not those of an absorbing exit process")
        error = sum(surv) / c.circle_target_steps - 1
        before = float(self.dual)
        smoothed = c.circle_budget_beta * float(self.ema) + (1 - c.circle_budget_beta) * error
        self.ema.fill_(smoothed)
        if step >= c.circle_random_warmup:
            dual_ascent(self.dual, c.circle_dual_lr, smoothed, c.circle_dual_limit)
        self.tick(step)
        gaps = [v - law for v, law in zip(surv, self._surv)]
        beyond = gaps[c.core_layers:]
        return dict(budget_target_steps=c.circle_target_steps, budget_error=error, budget_error_ema=smoothed,
                    budget_weight_used=before, budget_weight_next=float(self.dual), budget_survival=surv,
                    budget_survival_error=gaps,
                    budget_shape_rmse=math.sqrt(sum(g * g for g in beyond) / len(beyond)),
                    budget_updates=int(self.updates))


class SurvivalBudget(_UpdateClock):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.register_buffer("dual", torch.zeros(config.recursions - 1, dtype=torch.float64))

    @torch.no_grad()
    def reset(self):
        self.dual.zero_()
        self.restart()

    def _target(self, like):
        return like.new_tensor(self.config.mor_target_survival)

    def penalty(self, means):
        return quadratic_penalty(self.dual, means - self._target(means), self.config.mor_budget_strength).sum()

    @torch.no_grad()
    def update(self, counts, tokens, step):
        c = self.config
        self.admit(step, tokens, "MoR budget")
        survival = self.dual.new_tensor(counts) / tokens
        if not bool(torch.isfinite(survival).all()) or bool(((survival < 0) | (survival > 1)).any()):
            raise ValueError("MoR survival counts outside [0, tokens]")
        error = survival - self._target(survival)
        dual_ascent(self.dual, c.mor_dual_lr, error, c.mor_dual_limit)
        self.tick(step)
        return {"budget_survival": survival.tolist(), "budget_error": error.tolist(), "budget_dual": self.dual.tolist(),
                "budget_updates": int(self.updates)}
