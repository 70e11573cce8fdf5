"""Cost calibration: audited FLOPs per input token of a method, and the budget-matching search.

``method_cost(config)`` weights the audited cost of one update by the number of updates each
training stage runs (sparse burn-in, Ouro gate-only stage, Huginn's sampled depths, plugin
stages).  Token-recurrent linear methods are audited at three short lengths and extrapolated
operator by operator (the counts are affine in T; the third length verifies it), chunked ones
are audited at full length.  ``calibrate`` searches the registered grid (depth, then FFN width
3d..5d in steps of 128) for the configuration closest to the SSSL anchor, as the reference's
``nexttransformer/protocol/calibrate.py`` does, and writes the configuration file and its proof.

    python -m nexttransformer_b200.protocol.calibrate --methods gdn nsa --out configs
"""
import argparse
from collections import Counter
from dataclasses import replace
import hashlib
import json
from pathlib import Path

import torch

from nexttransformer_b200.models.config import CHUNK_BACKENDS, LINEAR, LOOPED, candidate_config
from nexttransformer_b200.models.looped import huginn_depth
from nexttransformer_b200.models.registry import PLUGIN_METHODS
from nexttransformer_b200.protocol.compute import FORMULA_VERSION, audit_graph
from nexttransformer_b200.protocol.spec import Protocol, config_file, write_config

BATCH = 512
FIELDS = ("calls", "theory", "padded_envelope", "matrix")


def stages(c):
    """[(stage, depth, optimizer steps)] of a method's training schedule."""
    p = Protocol()
    if c.method in PLUGIN_METHODS:
        from nexttransformer_b200.models.plugins import stages as plugin_stages
        return [(name, None, n) for name, n in plugin_stages(c)]
    if c.method == "huginn":
        counts = Counter(huginn_depth(c, s) for s in range(p.steps))
        return [("joint", d, counts[d]) for d in sorted(counts)]
    if c.method == "ouro":
        return [("joint", None, p.steps - c.ouro_gate_steps), ("gate_only", None, c.ouro_gate_steps)]
    if c.has_sparse_burnin:
        return [("burnin", None, c.burnin_steps), ("joint", None, p.steps - c.burnin_steps)]
    return [("joint", None, p.steps)]


def _affine(c, stage, depth):
    """Operator-wise affine extrapolation of a token-recurrent audit to the full context."""
    chunk = CHUNK_BACKENDS.get(c.backend)
    lengths = (16, 32, 48) if chunk is None else (3 * chunk, 4 * chunk, 5 * chunk)
    probes = [audit_graph(c, sequence_len=t, batch=BATCH, stage=stage, depth=depth) for t in lengths]
    step = lengths[1] - lengths[0]
    keys = set().union(*(r["operators"] for r in probes))
    ops = {}
    for key in keys:
        item = {}
        for f in FIELDS:
            a, b, t3 = [r["operators"].get(key, {}).get(f, 0) for r in probes]
            if t3 != 2 * b - a:
                raise RuntimeError(f"non-affine count: {key}/{f}")
            num = (b - a) * (c.sequence_len - lengths[0])
            if num % step:
                raise RuntimeError("non-integral extrapolated count")
            item[f] = a + num // step
        ops[key] = item
    total = sum(v["theory"] for v in ops.values())
    return dict(probes[0], operators=dict(sorted(ops.items())), total=total, sequence_len=c.sequence_len,
                extrapolation={"kind": "operator-wise affine", "verified_lengths": list(lengths)})


def full_cost(c, stage="joint", depth=None):
    if c.method in LINEAR and c.backend not in CHUNK_BACKENDS:
        return _affine(c, stage, depth)
    return audit_graph(c, batch=BATCH, stage=stage, depth=depth)


def method_cost(c):
    """(flops per input token, proof record) of one configuration."""
    p = Protocol()
    records, weighted = [], 0
    for stage, depth, steps in stages(c):
        r = full_cost(c, stage, depth)
        if r["unknown"]:
            raise RuntimeError(f"uncovered floating operators: {r['unknown']}")
        records.append(dict(stage=stage, depth=depth, optimizer_steps=steps,
                            cost={k: r[k] for k in ("total", "phases", "matrix_total", "padded_envelope",
                                                    "parameters")}))
        weighted += steps * r["total"]
    proof = dict(method=c.method, model_hash=c.fingerprint, protocol_hash=p.fingerprint,
                 formula_version=FORMULA_VERSION, torch=torch.__version__, total_training_flops=weighted,
                 flops_per_token=weighted / p.total_tokens, stages=records, unknown={})
    return weighted / p.total_tokens, proof


def search(c, anchor, tolerance=.01):
    """Closest registered configuration to the anchor: FFN width on the 3d..5d grid (step 128)."""
    best = (abs(method_cost(c)[0] / anchor - 1), c)
    if best[0] <= tolerance:
        return best[1]
    lo, hi = 3 * c.width, 5 * c.width
    for width in range(lo - lo % 128 + (128 if lo % 128 else 0), hi + 1, 128):
        cand = replace(c, mlp_width=width)
        err = abs(method_cost(cand)[0] / anchor - 1)
        if err < best[0]:
            best = (err, cand)
    return best[1]


def calibrate(method, out_dir, anchor=None):
    anchor = anchor or method_cost(candidate_config("dense"))[0]
    c = search(candidate_config(method), anchor)
    per_token, proof = method_cost(c)
    path = config_file(out_dir, method)
    proof_path = path.with_name(f"{method}.cost.json")
    path.parent.mkdir(parents=True, exist_ok=True)
    proof_path.write_text(json.dumps(proof, indent=1) + "\n")
    write_config(path, c, dict(status="theoretical_preflight_passed", formula_version=FORMULA_VERSION,
                               flops_per_token=per_token, dense_flops_per_token=anchor,
                               relative_error=per_token / anchor - 1, cost_record=proof_path.name,
                               torch=torch.__version__))
    return path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--methods", nargs="+", required=True)
    ap.add_argument("--out", type=Path, default=Path("configs"))
    a = ap.parse_args(argv)
    anchor = method_cost(candidate_config("dense"))[0]
    for m in a.methods:
        print(calibrate(m, a.out, anchor))


if __name__ == "__main__":
    main()
