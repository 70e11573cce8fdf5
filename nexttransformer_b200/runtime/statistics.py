"""Per-update accounting vector of the native track (shared by its trainer and benchmark).

Layout (fp64): [0] lm loss, [1] router loss, [2] training FLOPs (3 x forward + recompute),
[3] recompute FLOPs, [4] input tokens, [5] active depth sum, [6 : 6+R] active tokens per routing
step, then total loss, logical sparse FLOPs, compute loss and objective.  Losses are pre-divided by
accumulation x world so one all-reduce SUM gives the global means.
Behaviour: ``nexttransformer/runtime/statistics.py:1-21``.
"""
import torch


def training_stats(config, device):
    return torch.zeros(10 + config.routing_steps, dtype=torch.float64, device=device)


def accumulate_stats(stats, out, path, accumulation, world, config):
    share = accumulation * world
    stats[0] += out["lm_loss"].detach() / share
    stats[1] += out["router_loss"].detach() / share
    stats[2] += 3 * path["forward_flops"] + path["recompute_flops"]
    stats[3] += path["recompute_flops"]
    stats[4] += path["input_tokens"]
    stats[5] += path["active_depth_sum"]
    for i, n in enumerate(path["active_tokens"]):
        stats[6 + i] += n
    k = 6 + config.routing_steps
    stats[k] += out["loss"].detach() / share
    stats[k + 1] += path.get("logical_sparse_flops", path["forward_flops"])
    stats[k + 2] += out.get("compute_loss", out["lm_loss"].new_zeros(())).detach() / share
    stats[k + 3] += out.get("objective", out["loss"]).detach() / share
