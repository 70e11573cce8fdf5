"""Native Muon/AdamW groups with nanochat's weight-decay rule applied to the model actually trained:
Muon weight decay scales inversely with the matrix parameter count (blocks plus output head), which
agrees with the native d24 pin for d24 (``nexttransformer/scaling/optimizer.py`` of the reference).

``bf16_reduce=True`` sends gradients to their owners in bf16 (half the reduce-scatter / reduce
traffic of fp32 gradients; the role of DDP's bf16 compression hook in the reference's scaling
trainer): before each step every gradient is exposed to the optimizer as a bf16 ``main_grad`` copy,
which its collectives reduce and its update rules read back in fp32.
"""
import torch
import torch.distributed as dist

from nexttransformer_b200.native.optimizer import D12_SCALING_PARAMS, build_optimizer as native_optimizer


def scaling_params(model):
    return sum(p.numel() for p in model.transformer.h.parameters()) + model.lm_head.weight.numel()


def muon_weight_decay(model, config):
    return config.weight_decay * config.batch_scale * D12_SCALING_PARAMS / scaling_params(model)


def _bf16_reduce_step(optimizer):
    step = optimizer.step

    @torch.no_grad()
    def wrapped():
        if not (dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1):
            return step()
        exposed = []
        for group in optimizer.param_groups:
            for p in group["params"]:
                if getattr(p, "main_grad", None) is None and p.grad is not None and p.grad.dtype != torch.bfloat16:
                    p.main_grad = p.grad.to(torch.bfloat16)
                    exposed.append(p)
        try:
            return step()
        finally:
            for p in exposed:
                p.main_grad = None
    optimizer.step = wrapped
    return optimizer


def build_optimizer(model, config, shadows=None, bf16_reduce=False):
    optimizer = native_optimizer(model, config, shadows=shadows)
    decay = muon_weight_decay(model, config)
    for group in optimizer.param_groups:
        if group["kind"] == "muon":
            group["weight_decay"] = group["initial_weight_decay"] = decay
    return _bf16_reduce_step(optimizer) if bf16_reduce else optimizer
