"""Route budgets of the native track, updated once per complete optimizer update.

``SurvivalBudget`` (MoR): per recursion a dual variable on the survival error
``hard_mean - target``; penalty ``dual * e + strength/2 * e^2`` (forward measures hard survival,
backward follows the straight-through route surrogate); the dual moves by ``dual_lr * measured
error`` and is clamped.  ``CircleBudget``: a signed mean-depth dual (EMA-smoothed error, enabled
after the random warm-up) plus a weak quadratic pull of the survival curve towards the depth law.
Behaviour: ``nexttransformer/models/native/budget.py:8-96``.
"""
import math

import torch
from torch import nn

from nexttransformer_b200.models.native.depth import depth_reference


class CircleBudget(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self._probs, self._surv = depth_reference(config.core_layers, config.circle_max_steps,
                                                  config.circle_target_steps)
        self.register_buffer("probabilities", torch.tensor(self._probs, dtype=torch.float64))
        self.register_buffer("survival", torch.tensor(self._surv, dtype=torch.float64))
        self.register_buffer("dual", torch.zeros((), dtype=torch.float64))
        self.register_buffer("ema", torch.zeros((), dtype=torch.float64))
        self.register_buffer("updates", torch.zeros((), dtype=torch.long))
        self.register_buffer("last_step", torch.tensor(-1, dtype=torch.long))

    @torch.no_grad()
    def reset(self):
        """Buffers are uninitialised after ``to_empty``; restore every one."""
        self.probabilities.copy_(torch.tensor(self._probs, dtype=torch.float64))
        self.survival.copy_(torch.tensor(self._surv, dtype=torch.float64))
        for b in (self.dual, self.ema, self.updates):
            b.zero_()
        self.last_step.fill_(-1)

    def penalty(self, survival):
        c = self.config
        err = survival.sum() / c.circle_target_steps - 1
        depth = self.dual.detach().clone().to(err) * err + 0.5 * c.circle_depth_rho * err.square()
        tail = survival[c.core_layers:] - self.survival[c.core_layers:].to(survival)
        shape = c.circle_shape_weight * tail.square().mean()
        return depth + shape, depth, shape

    @torch.no_grad()
    def update(self, counts, tokens, step):
        c = self.config
        if step <= int(self.last_step) or tokens <= 0:
            raise ValueError("update Circle budget once per complete optimizer step")
        if len(counts) != c.circle_max_steps:
            raise ValueError("Circle budget needs counts at every block")
        surv = [float(n) / tokens for n in counts]
        ok = (all(math.isfinite(v) and 0 <= v <= 1 for v in surv)
              and all(a + 1e-9 >= b for a, b in zip(surv, surv[1:]))
              and all(abs(v - 1) <= 1e-9 for v in surv[:c.core_layers]))
        if not ok:
            raise ValueError("invalid absorbing Circle survival counts")
        err = sum(surv) / c.circle_target_steps - 1
        used = float(self.dual)
        ema = c.circle_budget_beta * float(self.ema) + (1 - c.circle_budget_beta) * err
        if step >= c.circle_random_warmup:
            self.dual.add_(c.circle_dual_lr * ema).clamp_(-c.circle_dual_limit, c.circle_dual_limit)
        self.ema.fill_(ema)
        self.last_step.fill_(step)
        self.updates.add_(1)
        gaps = [a - b for a, b in zip(surv, self._surv)]
        tail = gaps[c.core_layers:]
        return dict(budget_target_steps=c.circle_target_steps, budget_error=err, budget_error_ema=ema,
                    budget_weight_used=used, budget_weight_next=float(self.dual), budget_survival=surv,
                    budget_survival_error=gaps, budget_shape_rmse=math.sqrt(sum(g * g for g in tail) / len(tail)),
                    budget_updates=int(self.updates))


class SurvivalBudget(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.register_buffer("dual", torch.zeros(config.recursions - 1, dtype=torch.float64))
        self.register_buffer("updates", torch.zeros((), dtype=torch.long))
        self.register_buffer("last_step", torch.tensor(-1, dtype=torch.long))

    def penalty(self, means):
        err = means - means.new_tensor(self.config.mor_target_survival)
        return (self.dual.detach().clone().to(err) * err + 0.5 * self.config.mor_budget_strength * err.square()).sum()

    @torch.no_grad()
    def update(self, counts, tokens, step):
        if step <= int(self.last_step) or tokens <= 0:
            raise ValueError("update budget once per complete optimizer step")
        mean = self.dual.new_tensor(counts) / tokens
        if not torch.isfinite(mean).all() or (mean < 0).any() or (mean > 1).any():
            raise ValueError("invalid survival counts")
        err = mean - self.dual.new_tensor(self.config.mor_target_survival)
        self.dual.add_(self.config.mor_dual_lr * err).clamp_(-self.config.mor_dual_limit, self.config.mor_dual_limit)
        self.last_step.fill_(step)
        self.updates.add_(1)
        return {"budget_survival": mean.tolist(), "budget_error": err.tolist(), "budget_dual": self.dual.tolist(),
                "budget_updates": int(self.updates)}
