"""Event schedule, data layout and the cumulative budget ledger of a formal run.

``BudgetState`` charges every optimizer update its audited cost and checks the token cursor
and evaluation events; ``data_layout`` / ``share_batches`` let 16/32/64 ranks reproduce the
eight-stream row order of an eight-rank run (reference: ``nexttransformer/protocol/
admission.py:20-149``).  ``review_config`` checks a configuration against its cost proof.
"""
from dataclasses import asdict, dataclass, field
import json
import math
from pathlib import Path

import torch

from nexttransformer_b200.protocol.spec import Protocol, load_config


def review_config(path):
    """(config, proof, findings): the proof must describe this configuration; findings are stale or
    out-of-budget evidence (formal admission refuses any, research mode records them)."""
    path = Path(path)
    config = load_config(path)
    raw = json.loads(path.read_text())
    cal = raw["calibration"]
    findings = []
    proof_path = path.parent / cal.get("cost_record", "missing.json")
    if not proof_path.exists():
        raise ValueError("configuration has no cost proof")
    proof = json.loads(proof_path.read_text())
    p = Protocol()
    if proof["model_hash"] != config.fingerprint or proof["protocol_hash"] != p.fingerprint or proof.get("unknown"):
        raise ValueError("cost proof does not cover this model/protocol")
    if cal.get("status") != "theoretical_preflight_passed":
        findings.append("configuration has not passed cost preflight")
    if cal.get("torch") != torch.__version__:
        findings.append("PyTorch version differs from the cost evidence; re-audit in the target environment")
    if sum(s["optimizer_steps"] for s in proof["stages"]) != p.steps:
        raise ValueError("cost proof misses training stages")
    weighted = sum(s["optimizer_steps"] * s["cost"]["total"] for s in proof["stages"])
    if weighted != proof["total_training_flops"]:
        raise ValueError("stage-weighted cost mismatch")
    per_token = weighted / p.total_tokens
    if not math.isclose(per_token, cal["flops_per_token"], rel_tol=1e-12):
        raise ValueError("configuration cost mismatch")
    err = per_token / cal["dense_flops_per_token"] - 1
    if abs(err) > p.preflight_tolerance:
        findings.append(f"theoretical training budget mismatch ({err:+.3%} versus the "
                        f"{p.preflight_tolerance:.0%} preflight)")
    return config, proof, findings


def admit_config(path):
    config, proof, findings = review_config(path)
    if findings:
        raise ValueError(findings[0])
    return config, proof


def events_at(step):
    p = Protocol()
    if not 0 <= step <= p.steps:
        raise ValueError("step outside the training budget")
    return dict(val=step in p.validation_steps, core=step in p.core_steps, final=step == p.steps)


def data_layout(rank, world):
    """(stream rank, stream world, shares): multiples of eight ranks share the eight streams."""
    p = Protocol()
    if world % p.data_parallel_size:
        return rank, world, 1
    shares = world // p.data_parallel_size
    return rank // shares, p.data_parallel_size, shares


def share_batches(stream, batch, period, share, shares, device):
    """``batch``-row pieces of rows [share n, (share + 1) n) of the stream's next ``period`` rows.
    Every copy packs all ``period`` rows, so stream state stays that of an unshared stream."""
    own, rest = divmod(period, shares)
    if rest or own % batch:
        raise ValueError("a rank share must hold whole batches")
    cpu = torch.device("cpu")
    if share:
        stream.batch(share * own, cpu)
    for _ in range(own // batch):
        yield stream.batch(batch, device)
    if share < shares - 1:
        stream.batch((shares - 1 - share) * own, cpu)


@dataclass
class BudgetState:
    protocol_hash: str = field(default_factory=lambda: Protocol().fingerprint)
    optimizer_step: int = 0
    input_tokens: int = 0
    theory_flops: int = 0
    val_steps: list = field(default_factory=list)
    core_steps: list = field(default_factory=list)

    def validate(self):
        p = Protocol()
        if self.protocol_hash != p.fingerprint:
            raise ValueError("protocol changed on resume")
        if self.input_tokens != self.optimizer_step * p.global_batch_tokens:
            raise ValueError("token/step cursor mismatch")
        if not 0 <= self.optimizer_step <= p.steps or self.theory_flops < 0:
            raise ValueError("invalid cumulative state")
        for label, got, allowed in (("val", self.val_steps, p.validation_steps), ("core", self.core_steps, p.core_steps)):
            if got != sorted(set(got)) or any(s > self.optimizer_step or s not in allowed for s in got):
                raise ValueError(label + " event cursor mismatch")

    def advance(self, input_tokens, theory_flops):
        self.validate()
        p = Protocol()
        if input_tokens != p.global_batch_tokens or self.optimizer_step >= p.steps or theory_flops <= 0:
            raise ValueError("an update consumes exactly the global batch and a positive audited cost")
        self.optimizer_step += 1
        self.input_tokens += input_tokens
        self.theory_flops += int(theory_flops)

    def record_eval(self, kind):
        self.validate()
        if kind not in ("val", "core") or not events_at(self.optimizer_step)[kind]:
            raise ValueError("evaluation not scheduled at this step")
        hist = self.val_steps if kind == "val" else self.core_steps
        if self.optimizer_step in hist:
            raise ValueError("evaluation already recorded")
        hist.append(self.optimizer_step)

    def state_dict(self):
        self.validate()
        return asdict(self)

    @classmethod
    def from_state_dict(cls, state):
        s = cls(**state)
        s.validate()
        return s

    def final_status(self, dense_flops_per_token):
        self.validate()
        p = Protocol()
        if self.input_tokens != p.total_tokens:
            return "incomplete_training"
        if self.val_steps != list(p.validation_steps) or self.core_steps != list(p.core_steps):
            return "incomplete_eval"
        err = abs(self.theory_flops / (p.total_tokens * dense_flops_per_token) - 1)
        return "matched" if err <= p.cumulative_tolerance else "budget_mismatch"
