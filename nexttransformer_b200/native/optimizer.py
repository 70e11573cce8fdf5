"""Native-track parameter groups, gradient clips and schedule.

AdamW: lm_head, wte, value embeddings, the shell scalars, router/halter parameters (Circle's at
``circle_halter_lr_multiplier``), LoopFormer's conditioner (at ``loop_condition_lr_multiplier``) and
any other non-matrix parameter; Muon: every 2-D matrix, grouped by shape, weight decay scaled by the
d12/d24 parameter ratio.  LRs scale by sqrt(batch / 524288) and (width / 768)^-1/2.  Schedule: linear
warm-up, flat, linear warm-down over ``warmdown_ratio`` to ``final_lr_fraction``; Muon momentum
0.85 -> 0.97 over 400 updates and back to 0.90 in the warm-down; Muon weight decay cosine-decays.
Behaviour: ``nexttransformer/native/optimizer.py:12-84``.
"""
from collections import defaultdict
import math

import torch

from nexttransformer_b200.optim.muon_adamw import MuonAdamW

D12_SCALING_PARAMS = 110100912
D24_SCALING_PARAMS = 729810624


def build_optimizer(model, config, shadows=None):
    c = model.config
    ds = (c.width / 768) ** -0.5
    bs = math.sqrt(config.global_batch_tokens / 524288)
    wd = config.weight_decay * bs * D12_SCALING_PARAMS / D24_SCALING_PARAMS
    groups = []

    def adam(params, lr, betas, decay):
        params = list(params)
        if params:
            groups.append(dict(kind="adamw", params=params, lr=lr, initial_lr=lr, betas=betas, eps=1e-10,
                               weight_decay=decay))

    adam(model.lm_head.parameters(), config.unembedding_lr * bs * ds, (.8, .96), .01)
    adam(model.transformer.wte.parameters(), config.embedding_lr * bs * ds, (.8, .995), .001)
    adam(model.value_embeds.parameters(), config.embedding_lr * bs * ds * .5, (.8, .995), .01)
    adam([model.resid_lambdas], config.scalar_lr * bs * .01, (.8, .95), .05)
    adam([model.x0_lambdas], config.scalar_lr * bs, (.96, .95), 0.)
    adam([model.smear_gate.weight, model.smear_lambda, model.backout_lambda], .2, (.8, .95), 0.)
    routed = [p for n, p in model.named_parameters() if n.startswith(("routers.", "halter."))]
    adam(routed, config.adamw_lr * bs * (c.circle_halter_lr_multiplier if c.architecture == "circle" else 1.),
         (.9, .95), 0.)
    if c.architecture == "loopformer":
        adam(model.conditioner.parameters(), config.adamw_lr * bs * c.loop_condition_lr_multiplier, (.9, .95), 0.)
    taken = {id(p) for g in groups for p in g["params"]}
    matrices, rest = defaultdict(list), []
    for p in model.parameters():
        if id(p) not in taken:
            (matrices[tuple(p.shape)] if p.ndim == 2 else rest).append(p)
    adam(rest, config.adamw_lr * bs, (.9, .95), 0.)
    for shape in sorted(matrices):
        groups.append(dict(kind="muon", params=matrices[shape], lr=config.muon_lr * bs,
                           initial_lr=config.muon_lr * bs, momentum=.95, ns_steps=5, beta2=.9, weight_decay=wd,
                           initial_weight_decay=wd))
    ids = [id(p) for g in groups for p in g["params"]]
    if len(ids) != len(set(ids)) or set(ids) != {id(p) for p in model.parameters()}:
        raise RuntimeError("optimizer must cover all parameters exactly once")
    names = {id(p): n for n, p in model.named_parameters()}
    for g in groups:
        g["parameter_names"] = [names[id(p)] for p in g["params"]]
    return MuonAdamW(groups, shadows=shadows)


def clip_halter_gradients(model):
    """Clip Circle's exit scorer after accumulation, before the update."""
    if model.config.architecture != "circle":
        return 0.
    return float(torch.nn.utils.clip_grad_norm_(model.halter.parameters(), model.config.circle_halter_grad_clip,
                                                error_if_nonfinite=True))


def clip_condition_gradients(model):
    if model.config.architecture != "loopformer":
        return 0.
    return float(torch.nn.utils.clip_grad_norm_(model.conditioner.parameters(), model.config.loop_condition_grad_clip,
                                                error_if_nonfinite=True))


def set_schedule(optimizer, step, config):
    down = round(config.warmdown_ratio * config.steps)
    start = config.steps - down
    if step < config.warmup_steps:
        mult = (step + 1) / max(1, config.warmup_steps)
    elif step <= start:
        mult = 1.
    else:
        left = (config.steps - step) / max(1, down)
        mult = left + (1 - left) * config.final_lr_fraction
    if step < 400:
        momentum = .85 + (.97 - .85) * step / 400
    elif step >= start:
        momentum = .97 + (.90 - .97) * (step - start) / max(1, down)
    else:
        momentum = .97
    for g in optimizer.param_groups:
        g["lr"] = g["initial_lr"] * mult
        if g["kind"] == "muon":
            g["momentum"] = momentum
            g["weight_decay"] = g["initial_weight_decay"] * .5 * (1 + math.cos(math.pi * step / config.steps))
    return mult
