"""Configuration of a scaling-stage run: the native backbone (plus the shell switches the scaling
protocol varies) and a training section that names its own protocol, budget, batch and cadence.

Field names, defaults and validation rules follow ``nexttransformer/scaling/config.py`` of the
reference, so scaling configuration files load in both trees and hash alike.
"""
from dataclasses import asdict, dataclass, fields
import hashlib
import json
import math
from pathlib import Path

from nexttransformer_b200.models.native.config import NativeModelConfig

# Tokens per update at which the nanochat learning rates were tuned; larger batches scale them by
# sqrt(B / B0).
REFERENCE_BATCH_TOKENS = 524288
# Model settings the earlier comparison never varied: left out of the serialized form while at their
# default, so hashes recorded before they existed still match.
SCOPED_FIELDS = ("value_embeddings",)


@dataclass(frozen=True)
class ScalingModelConfig(NativeModelConfig):
    value_embeddings: bool = True

    def serialized(self):
        data = asdict(self)
        defaults = {f.name: f.default for f in fields(self)}
        for name in SCOPED_FIELDS:
            if data[name] == defaults[name]:
                data.pop(name)
        return data

    def matches(self, recorded):
        defaults = {f.name: f.default for f in fields(self)}
        kept = {k: v for k, v in recorded.items() if not (k in SCOPED_FIELDS and v == defaults[k])}
        return kept == self.serialized()


@dataclass(frozen=True)
class ScalingTrainConfig:
    protocol: str = "nextt-scale-200b-4k-v1"
    seed: int = 42
    total_tokens: int = 199_999_094_784
    global_batch_tokens: int = 2_097_152
    val_every: int = 1000
    val_tokens: int = 80 * 524288
    final_bpb_tokens: int = 40 * 524288
    core_every: int = 20_000
    core_max_per_task: int = -1
    checkpoint_every: int = 1000
    milestone_every: int = 10_000
    warmup_steps: int = 40
    warmdown_ratio: float = .65
    final_lr_fraction: float = .05
    muon_lr: float = .02
    adamw_lr: float = .0006
    embedding_lr: float = .3
    unembedding_lr: float = .008
    scalar_lr: float = .5
    weight_decay: float = .28
    grad_clip: float = 0.

    def __post_init__(self):
        if not self.protocol or not self.protocol.strip():
            raise ValueError("a scaling run names its protocol version")
        positive = (self.total_tokens, self.global_batch_tokens, self.val_every, self.val_tokens,
                    self.final_bpb_tokens, self.checkpoint_every, self.milestone_every)
        if min(positive) <= 0:
            raise ValueError("budgets and intervals must be positive")
        if self.milestone_every % self.checkpoint_every:
            raise ValueError("milestones must fall on checkpoint steps")
        if not (0 <= self.warmdown_ratio <= 1 and 0 <= self.final_lr_fraction <= 1 and self.warmup_steps >= 0):
            raise ValueError("invalid learning-rate schedule")
        lrs = (self.muon_lr, self.adamw_lr, self.embedding_lr, self.unembedding_lr, self.scalar_lr)
        if self.grad_clip < 0 or not all(math.isfinite(v) and v > 0 for v in lrs):
            raise ValueError("learning rates must be positive and clipping nonnegative")
        self.steps

    @property
    def steps(self):
        if self.total_tokens % self.global_batch_tokens:
            raise ValueError("total_tokens must be a multiple of global_batch_tokens")
        return self.total_tokens // self.global_batch_tokens

    @property
    def batch_scale(self):
        return math.sqrt(self.global_batch_tokens / REFERENCE_BATCH_TOKENS)

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

    def is_milestone(self, step):
        return step % self.milestone_every == 0 or step == self.steps


def load_config(path):
    raw = json.loads(Path(path).read_text())
    if set(raw) != {"model", "train"}:
        raise ValueError("a scaling configuration has model and train sections")
    model = dict(raw["model"])
    if "mor_target_survival" in model:
        model["mor_target_survival"] = tuple(model["mor_target_survival"])
    mc, tc = ScalingModelConfig(**model), ScalingTrainConfig(**raw["train"])
    if mc.architecture != "dense":
        raise ValueError("the scaling stage trains the dense backbone")
    for name in ("global_batch_tokens", "val_tokens", "final_bpb_tokens"):
        if getattr(tc, name) % mc.sequence_len:
            raise ValueError(f"{name} must contain whole sequences")
    return mc, tc


def config_hash(mc, tc):
    blob = json.dumps({"model": mc.serialized(), "train": asdict(tc)}, sort_keys=True).encode()
    return hashlib.sha256(blob).hexdigest()


def write_config(path, mc, tc):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps({"model": mc.serialized(), "train": asdict(tc)}, indent=2) + "\n")
