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
from nexttransformer_b200.protocol import fingerprint
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
    executed = set()
    for stage, depth, steps in stages(c):
        with fingerprint.traced() as ran:
            r = full_cost(c, stage, depth)
        executed |= ran
        if r["unknown"]:
            raise RuntimeError(f"uncovered floating operators: {r['unknown']}")
        records.append(dict(stage=stage, depth=depth, optimizer_steps=steps,
                            cost={k: r[k] for k in ("total", "phases", "matrix_total", "padded_envelope",
                                                    "parameters")}))
        weighted += steps * r["total"]
    proof = dict(method=c.method, model_hash=c.fingerprint, protocol_hash=p.fingerprint,
                 formula_version=FORMULA_VERSION, torch=torch.__version__, total_training_flops=weighted,
                 flops_per_token=weighted / p.total_tokens, stages=records, unknown={},
                 method_source=fingerprint.record(executed))
    return weighted / p.total_tokens, proof


def ffn_slope(c):
    """d(FLOPs per token)/d(FFN width) from the exact difference of two short-length audits per stage."""
    other = replace(c, mlp_width=c.mlp_width + 128)
    chunk = CHUNK_BACKENDS.get(c.backend)
    first, second = (16, 32) if chunk is None else (3 * chunk, 4 * chunk)
    weighted = 0
    for stage, depth, steps in stages(c):
        delta = [audit_graph(other, sequence_len=t, batch=BATCH, stage=stage, depth=depth)["total"]
                 - audit_graph(c, sequence_len=t, batch=BATCH, stage=stage, depth=depth)["total"] for t in (first, second)]
        weighted += steps * (delta[0] + (delta[1] - delta[0]) * (c.sequence_len - first) // (second - first))
    return weighted / Protocol().total_tokens / 128


def structure(c, initial, target, tol):
    """Adjacent integer depths first (layers 16..32, or core layers 1..16 for looped stacks), stopping
    at the first bracket around the target."""
    if abs(initial / target - 1) <= tol:
        return c, initial, []
    field = "core_layers" if c.method in LOOPED else "layers"
    lo, hi = (1, 16) if field == "core_layers" else (16, 32)
    step = 1 if initial < target else -1
    best_c, best, trials, prev = c, initial, [], initial - target
    for value in range(getattr(c, field) + step, (hi + 1) if step > 0 else (lo - 1), step):
        cand = replace(c, **{field: value})
        cost = method_cost(cand)[0]
        trials.append(dict(field=field, value=value, flops_per_token=cost))
        if abs(cost - target) < abs(best - target):
            best_c, best = cand, cost
        if (cost - target) * prev <= 0 or abs(cost / target - 1) <= tol:
            break
        prev = cost - target
    return best_c, best, trials


def v2_grid(c, target, tol):
    """Hybrids, no-VE controls and plugins: audit every allowed depth 16..32 at the starting FFN with its
    FFN slope, estimate every width on the [3d, 5d] 128-grid, then fully audit the estimated-within-tolerance
    candidates in tie-break order (width closest to the start, smallest |error|, depth closest to the
    start, shallower) and keep the first whose audit is within tolerance."""
    from nexttransformer_b200.models.config import LAYER_MULTIPLE
    depths, cands = [], []
    for n in range(16, 33):
        if n % LAYER_MULTIPLE.get(c.method, 1):
            continue
        trial = replace(c, layers=n)
        cost, slope = method_cost(trial)[0], ffn_slope(trial)
        depths.append(dict(layers=n, flops_per_token=cost, ffn_slope=slope))
        for width in range(3 * c.width, 5 * c.width + 1, 128):
            est = (cost + (width - c.mlp_width) * slope) / target - 1
            if abs(est) <= tol:
                cands.append(dict(layers=n, mlp_width=width, estimated_error=est))
    cands.sort(key=lambda t: (abs(t["mlp_width"] - c.mlp_width), abs(t["estimated_error"]), abs(t["layers"] - c.layers),
                              t["layers"]))
    table = dict(rule="v2 tie-break", start=dict(layers=c.layers, mlp_width=c.mlp_width), depths=depths,
                 candidates=cands)
    for cand in cands:
        chosen = replace(c, layers=cand["layers"], mlp_width=cand["mlp_width"])
        cost = method_cost(chosen)[0]
        cand["audited_error"] = cost / target - 1
        if abs(cand["audited_error"]) <= tol:
            return chosen, cost, table
    raise RuntimeError(f"{c.method}: no registered-grid candidate within tolerance")


def search(c, anchor, tol=None):
    """Registered selection: v2 grid for hybrids/no-VE/plugins; otherwise depth structure search, then
    the FFN width from the exact slope, rounded to the 128-grid inside [3d, 5d]."""
    from nexttransformer_b200.models.config import V2_CALIBRATION
    tol = Protocol().preflight_tolerance if tol is None else tol
    if c.method in V2_CALIBRATION:
        return v2_grid(c, anchor, tol)[0]
    chosen, cost, _ = structure(c, method_cost(c)[0], anchor, tol)
    if abs(cost / anchor - 1) > tol:
        wanted = chosen.mlp_width + (anchor - cost) / ffn_slope(chosen)
        width = 128 * round(wanted / 128)
        if not 3 * c.width <= width <= 5 * c.width:
            raise RuntimeError(f"{c.method}: the FFN grid cannot meet the budget")
        chosen = replace(chosen, mlp_width=width)
    return chosen


def calibrate(method, out_dir, anchor=None, reuse=None):
    """Audit a method and write its configuration and cost proof.  With ``reuse`` (a configuration
    directory) the stored structure is re-audited unchanged instead of searched."""
    from nexttransformer_b200.protocol.spec import load_config
    anchor = anchor or method_cost(candidate_config("dense"))[0]
    previous = config_file(reuse, method) if reuse else None
    if previous is not None and previous.exists():
        c = load_config(previous)
    elif method == "dense":
        c = candidate_config("dense")
    else:
        c = search(candidate_config(method), anchor)
    per_token, proof = method_cost(c)
    path = config_file(out_dir, method)
    proof_path = path.with_name(f"{method}.cost.json")
    path.parent.mkdir(parents=True, exist_ok=True)
    proof_path.write_text(json.dumps(proof, indent=1) + "\n")
    deviation = per_token / anchor - 1
    status = "theoretical_preflight_passed" if abs(deviation) <= Protocol().preflight_tolerance else "budget_mismatch"
    write_config(path, c, dict(status=status, formula_version=FORMULA_VERSION,
                               flops_per_token=per_token, dense_flops_per_token=anchor,
                               relative_error=deviation, cost_record=proof_path.name,
                               torch=torch.__version__, method_source_hash=proof["method_source"]["hash"]))
    return path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--methods", nargs="+", required=True)
    ap.add_argument("--out", type=Path, default=Path("configs"))
    ap.add_argument("--reuse-configs", type=Path, help="re-audit the structures stored here instead of searching")
    a = ap.parse_args(argv)
    anchor = method_cost(candidate_config("dense"))[0]
    for m in a.methods:
        print(calibrate(m, a.out, anchor, a.reuse_configs), flush=True)


if __name__ == "__main__":
    main()
