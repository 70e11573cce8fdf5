"""Configuration of the native d24 comparison (model and training sections of one JSON file).

Field names, defaults and validation rules are those of the reference
(``nexttransformer/models/native/config.py:10-188``): native configuration files must load in both
trees.  Architectures: ``dense`` (24 layers), ``mor`` (3 + 9x3 + 3, token routing), ``loopformer``
(3 + 9x2 + 3, time-conditioned modulation) and ``circle`` (3 + ring of 9 up to 27 steps + 3, sparse
absorbing exits with a depth budget).
"""
from dataclasses import asdict, dataclass
import json
import math
from pathlib import Path

UPSTREAM_COMMIT = "92d63d4e8bb4df75c3b71618f31ddde2378b2bcd"
RECURSIONS = {"dense": 1, "mor": 3, "loopformer": 2, "circle": 3}


@dataclass(frozen=True)
class NativeModelConfig:
    architecture: str = "dense"
    dense_layers: int = 24
    pre_layers: int = 3
    core_layers: int = 9
    post_layers: int = 3
    recursions: int | None = None
    activation_checkpointing: bool = False
    fourier_dim: int = 256
    loop_modulation_bound: float = .5
    loop_condition_lr_multiplier: float = .5
    loop_condition_grad_clip: float = 1.
    vocab_size: int = 32768
    sequence_len: int = 2048
    width: int = 1536
    heads: int = 12
    mlp_width: int = 6144
    window_pattern: str = "SSSL"
    circle_max_steps: int = 27
    circle_target_steps: float = 17.5
    circle_method: str = "sparse_gate"
    circle_budget_mode: str = "mean_survival"
    circle_halter: str = "delta_depth"
    circle_halter_eps: float = 1e-6
    circle_exit_interval: int = 1
    circle_threshold: float = .5
    circle_routing_seed: int = 1729
    circle_budget_beta: float = .9
    circle_random_warmup: int = 256
    circle_route_transition: int = 768
    circle_depth_rho: float = 1.0
    circle_shape_weight: float = 0.1
    circle_dual_lr: float = 0.05
    circle_dual_limit: float = 2.0
    circle_halter_lr_multiplier: float = 0.5
    circle_halter_grad_clip: float = 1.0
    mor_target_survival: tuple = (.64, .32)
    mor_budget_strength: float = 1.0
    mor_dual_lr: float = .05
    mor_dual_limit: float = 10.0

    def __post_init__(self):
        if self.architecture not in RECURSIONS:
            raise ValueError(f"native architecture must be one of {sorted(RECURSIONS)}, got {self.architecture!r}")
        if self.recursions is None:
            object.__setattr__(self, "recursions", RECURSIONS[self.architecture])
        for scope, holds, message in _RULES:
            if scope in ("any", self.architecture) and not holds(self):
                raise ValueError(message)

    @property
    def n_layer(self):
        if self.architecture == "dense":
            return self.dense_layers
        return self.pre_layers + self.core_layers + self.post_layers

    @property
    def max_depth(self):
        if self.architecture == "dense":
            return self.dense_layers
        middle = self.circle_max_steps if self.architecture == "circle" else self.core_layers * self.recursions
        return self.pre_layers + middle + self.post_layers

    @property
    def routing_steps(self):
        return self.circle_max_steps if self.architecture == "circle" else self.recursions

    @property
    def n_embd(self):
        return self.width

    @property
    def n_head(self):
        return self.heads

    @property
    def n_kv_head(self):
        return self.heads


def _finite_positive(*values):
    return all(math.isfinite(v) and v > 0 for v in values)


def _decreasing(values):
    return all(a > b for a, b in zip(values, values[1:]))


# (scope, condition that must hold, message): scope "any" applies to every architecture.
_RULES = (
    ("any", lambda c: min(c.width, c.heads, c.sequence_len, c.pre_layers, c.core_layers, c.post_layers,
                          c.dense_layers, c.fourier_dim) > 0 and c.width % c.heads == 0,
     "native model sizes must be positive and the heads must divide the width"),
    ("any", lambda c: c.recursions == RECURSIONS[c.architecture],
     "the shared core protocol fixes the recursion count (MoR and Circle at most 3, LoopFormer exactly 2)"),
    ("any", lambda c: 0 < c.circle_halter_eps < 1, "circle_halter_eps must be strictly between 0 and 1"),
    ("any", lambda c: not c.activation_checkpointing,
     "the native FLOP accounting assumes no activation checkpointing"),
    ("any", lambda c: c.mlp_width == 4 * c.width and c.width >= 24 and (c.width // c.heads) % 2 == 0,
     "the native shell needs a 4x MLP, width of at least 24 and an even head size"),
    ("any", lambda c: bool(c.window_pattern) and set(c.window_pattern) <= set("SL"),
     "window_pattern may only use the letters S and L"),
    ("any", lambda c: len(c.mor_target_survival) == 2 and _decreasing((1., *c.mor_target_survival, 0.)),
     "MoR takes two survival targets, strictly decreasing inside (0, 1)"),
    ("any", lambda c: min(c.mor_budget_strength, c.mor_dual_lr, c.mor_dual_limit) > 0,
     "MoR budget strength, dual step and dual limit must be positive"),
    ("loopformer", lambda c: 0 < c.loop_modulation_bound < 1,
     "the LoopFormer modulation bound must be strictly between 0 and 1"),
    ("loopformer", lambda c: _finite_positive(c.loop_condition_lr_multiplier, c.loop_condition_grad_clip),
     "the LoopFormer conditioning learning-rate multiplier and clip must be finite and positive"),
    ("circle", lambda c: c.circle_halter == "delta_depth",
     "Circle uses the delta_depth halter (other halters belong to the frozen legacy source)"),
    ("circle", lambda c: (c.circle_method, c.circle_budget_mode, c.circle_exit_interval) ==
     ("sparse_gate", "mean_survival", 1),
     "Circle is the sparse-gate, mean-survival variant with an exit after every block"),
    ("circle", lambda c: c.circle_max_steps == c.core_layers * c.recursions,
     "Circle's step limit is exactly three passes around the ring"),
    ("circle", lambda c: c.core_layers < c.circle_target_steps < c.circle_max_steps,
     "Circle's target depth must lie strictly between one ring and the step limit"),
    ("circle", lambda c: c.circle_threshold == .5, "sparse Circle exits at a fixed gate threshold of 0.5"),
    ("circle", lambda c: all(math.isfinite(v) for v in (
        c.circle_target_steps, c.circle_depth_rho, c.circle_shape_weight, c.circle_dual_lr, c.circle_dual_limit,
        c.circle_budget_beta, c.circle_halter_lr_multiplier, c.circle_halter_grad_clip)),
     "every Circle setting must be finite"),
    ("circle", lambda c: _finite_positive(c.circle_depth_rho, c.circle_dual_lr, c.circle_dual_limit,
                                          c.circle_halter_lr_multiplier, c.circle_halter_grad_clip),
     "Circle's depth weight, dual step and limit, and halter optimizer settings must be positive"),
    ("circle", lambda c: c.circle_shape_weight >= 0 and 0 <= c.circle_budget_beta < 1,
     "Circle's shape weight must be non-negative and its smoothing in [0, 1)"),
    ("circle", lambda c: min(c.circle_random_warmup, c.circle_route_transition) >= 0,
     "Circle's warm-up and transition lengths cannot be negative"),
)


@dataclass(frozen=True)
class NativeTrainConfig:
    seed: int = 42
    total_tokens: int = 49152000000
    checkpoint_every: int = 5000
    muon_lr: float = .02
    adamw_lr: float = .0006
    global_batch_tokens: int = 1048576
    val_tokens: int = 80 * 524288
    val_every: int = 250
    final_bpb_tokens: int = 40 * 524288
    core_every: int = 8000
    core_max_per_task: int = -1
    warmup_steps: int = 40
    warmdown_ratio: float = .65
    final_lr_fraction: float = .05
    embedding_lr: float = .3
    unembedding_lr: float = .008
    scalar_lr: float = .5
    weight_decay: float = .28
    grad_clip: float = 0.0          # the native recipe does not clip

    @property
    def steps(self):
        if self.total_tokens <= 0 or self.global_batch_tokens <= 0 or self.total_tokens % self.global_batch_tokens:
            raise ValueError("total_tokens must be a positive multiple of global_batch_tokens")
        return self.total_tokens // self.global_batch_tokens

    def accumulation(self, model, world_size, micro_batch):
        per = world_size * micro_batch * model.sequence_len
        if per <= 0 or self.global_batch_tokens % per:
            raise ValueError("global batch must be divisible by world_size * micro_batch * sequence_len")
        return self.global_batch_tokens // per

    def validation_steps(self):
        return sorted({0, self.steps, *range(self.val_every, self.steps, self.val_every)})

    def core_steps(self, include_final=True):
        mid = list(range(self.core_every, self.steps, self.core_every)) if self.core_every > 0 else []
        return mid + ([self.steps] if include_final else [])


def load_config(path):
    raw = json.loads(Path(path).read_text())
    if set(raw) != {"model", "train"}:
        raise ValueError("configuration requires model and train sections")
    model = dict(raw["model"])
    if "mor_target_survival" in model:
        model["mor_target_survival"] = tuple(model["mor_target_survival"])
    mc, tc = NativeModelConfig(**model), NativeTrainConfig(**raw["train"])
    tc.steps
    if tc.val_tokens % mc.sequence_len or tc.final_bpb_tokens % mc.sequence_len:
        raise ValueError("evaluation budgets must contain whole sequences")
    return mc, tc


def write_config(path, mc, tc):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps({"model": asdict(mc), "train": asdict(tc)}, indent=2) + "\n")
