"""Parameter groups and learning-rate schedule of the Muon + AdamW recipe.

Two group layouts exist, as in the reference:
  * ``shell_groups`` - the upstream shell's own recipe (``nexttransformer/models/backbone.py:
    419-457``): AdamW for head / embeddings / value embeddings / scalars with LR scaled by
    (d / 768)^-1/2, Muon for every same-shape group of block matrices.
  * ``protocol_groups`` - the frozen protocol's recipe (``nexttransformer/training/optimizer.py:
    11-51``): batch-scaled LRs, method-auxiliary parameters (halters, indexers, gates, decay
    parameters, residual maps, depth queries) on AdamW, every other 2-D matrix on Muon, and an
    exactly-once ownership check.
``set_schedule`` is the protocol schedule (``nexttransformer/native/optimizer.py:68-84``).
"""
from collections import defaultdict
from dataclasses import dataclass
import math

D12_SCALING_PARAMS = 110100912
D24_SCALING_PARAMS = 729810624
AUXILIARY_KEYS = ("halter.", ".index_", ".beta_proj.", ".gate_down.", ".gate_up.", ".decay_proj.", ".slot_proj.",
                  ".branch_gate.", ".output_gate.", ".log_decay", ".dt_bias", ".compress_position", "residual_maps.",
                  "depth_queries", ".router.", "routers.")


@dataclass(frozen=True)
class TrainConfig:
    """Learning-rate recipe and budget of a run (defaults: the frozen reference protocol)."""
    seed: int = 42
    total_tokens: int = 49_152_000_000
    global_batch_tokens: int = 1_048_576
    muon_lr: float = .02
    adamw_lr: float = .0006
    embedding_lr: float = .3
    unembedding_lr: float = .008
    scalar_lr: float = .5
    weight_decay: float = .28
    warmup_steps: int = 40
    warmdown_ratio: float = .65
    final_lr_fraction: float = .05
    grad_clip: float = 0.

    @property
    def steps(self):
        if self.total_tokens <= 0 or self.total_tokens % self.global_batch_tokens:
            raise ValueError("total_tokens must be a positive multiple of global_batch_tokens")
        return self.total_tokens // self.global_batch_tokens


def _adam(groups, params, lr, betas, wd):
    params = [p for p in params if p.requires_grad]
    if params:
        groups.append(dict(kind="adamw", params=params, lr=lr, initial_lr=lr, betas=betas, eps=1e-10,
                           weight_decay=wd))


def _muon_groups(groups, matrices, lr, wd):
    for shape in sorted(matrices):
        groups.append(dict(kind="muon", params=matrices[shape], lr=lr, initial_lr=lr, momentum=.95, ns_steps=5,
                           beta2=.9, weight_decay=wd, initial_weight_decay=wd))


def _check_ownership(model, groups):
    ids = [id(p) for g in groups for p in g["params"]]
    want = {id(p) for p in model.parameters() if p.requires_grad}
    if len(ids) != len(set(ids)) or set(ids) != want:
        raise RuntimeError("trainable parameters must have exactly one optimizer owner")
    names = {id(p): n for n, p in model.named_parameters()}
    for g in groups:
        g["parameter_names"] = [names[id(p)] for p in g["params"]]
    return groups


def shell_groups(model, unembedding_lr=0.004, embedding_lr=0.2, matrix_lr=0.02, weight_decay=0.0, scalar_lr=0.5):
    d = model.lm_head.weight.shape[1]
    ds = (d / 768) ** -0.5
    groups = []
    _adam(groups, model.lm_head.parameters(), unembedding_lr * ds, (0.8, 0.96), 0.01)
    _adam(groups, model.transformer.wte.parameters(), embedding_lr * ds, (0.8, 0.995), 0.001)
    _adam(groups, model.value_embeds.parameters(), embedding_lr * ds * 0.5, (0.8, 0.995), 0.01)
    _adam(groups, [model.resid_lambdas], scalar_lr * 0.01, (0.8, 0.95), 0.05)
    _adam(groups, [model.x0_lambdas], scalar_lr, (0.96, 0.95), 0.0)
    _adam(groups, [model.smear_gate.weight, model.smear_lambda, model.backout_lambda], 0.2, (0.8, 0.95), 0.0)
    matrices = defaultdict(list)
    taken = {id(p) for g in groups for p in g["params"]}
    for p in model.transformer.h.parameters():
        if p.requires_grad and id(p) not in taken:
            matrices[tuple(p.shape)].append(p)
    _muon_groups(groups, matrices, matrix_lr, weight_decay)
    return _check_ownership(model, groups)


def protocol_groups(model, train=None, d12_d24_decay=True):
    c = train or TrainConfig()
    ds = (model.lm_head.weight.shape[1] / 768) ** -0.5
    bs = math.sqrt(c.global_batch_tokens / 524288)
    groups = []
    _adam(groups, model.lm_head.parameters(), c.unembedding_lr * bs * ds, (.8, .96), .01)
    _adam(groups, model.transformer.wte.parameters(), c.embedding_lr * bs * ds, (.8, .995), .001)
    _adam(groups, model.value_embeds.parameters(), c.embedding_lr * bs * ds * .5, (.8, .995), .01)
    _adam(groups, [model.resid_lambdas], c.scalar_lr * bs * .01, (.8, .95), .05)
    _adam(groups, [model.x0_lambdas], c.scalar_lr * bs, (.96, .95), 0.)
    _adam(groups, [model.smear_gate.weight, model.smear_lambda, model.backout_lambda], .2, (.8, .95), 0.)
    extras = [p for n, p in model.named_parameters() if any(k in n for k in AUXILIARY_KEYS)]
    _adam(groups, extras, c.adamw_lr * bs, (.9, .95), 0.)
    taken = {id(p) for g in groups for p in g["params"]}
    matrices, other = defaultdict(list), []
    for p in model.parameters():
        if not p.requires_grad or id(p) in taken:
            continue
        (matrices[tuple(p.shape)] if p.ndim == 2 else other).append(p)
    _adam(groups, other, c.adamw_lr * bs, (.9, .95), 0.)
    wd = c.weight_decay * bs * (D12_SCALING_PARAMS / D24_SCALING_PARAMS if d12_d24_decay else 1.0)
    _muon_groups(groups, matrices, c.muon_lr * bs, wd)
    return _check_ownership(model, groups)


def set_schedule(optimizer, step, train=None):
    """Linear warmup, flat, linear warmdown to ``final_lr_fraction``; Muon momentum ramp and cosine decay."""
    c = train or TrainConfig()
    steps = c.steps
    warmdown = round(c.warmdown_ratio * steps)
    start = steps - warmdown
    if step < c.warmup_steps:
        mult = (step + 1) / max(1, c.warmup_steps)
    elif step <= start:
        mult = 1.
    else:
        prog = (steps - step) / max(1, warmdown)
        mult = prog + (1 - prog) * c.final_lr_fraction
    if step < 400:
        mom = .85 + (.97 - .85) * step / 400
    elif step >= start:
        mom = .97 + (.90 - .97) * (step - start) / max(1, warmdown)
    else:
        mom = .97
    for g in optimizer.param_groups:
        g["lr"] = g["initial_lr"] * mult
        if g["kind"] == "muon":
            g["momentum"] = mom
            g["weight_decay"] = g["initial_weight_decay"] * .5 * (1 + math.cos(math.pi * step / steps))
    return mult
