"""Numerics of the chunked delta-rule paths (DeltaNet, Gated DeltaNet, KDA) against an FP64 oracle.

    python -m nexttransformer_b200.checks.linear [--kinds gdn kda deltanet] [--seq 4096] [--batch 1]
    python -m nexttransformer_b200.checks.linear --checkpoint runs/x/checkpoint_00001000 [--output r.json]

Candidates: ``fused`` (the sm_100a chunk-term and scan kernels on bf16 operands, as in training; CUDA
only) and ``chunk_fp32`` (the plain torch chunk form in fp32, any device).  The oracle is the FP64
token-by-token recurrence (``models.linear.recurrent_scan``), which does not use the chunk form's
within-chunk exponentials, so it stays exact where trained gates push a chunk's cumulative log decay
below the fp32 exp range.  Outputs and the gradients of every raw input (q, k, v, the log decay and
beta) under a fixed random upstream gradient are compared by relative L2 error against tolerances
fixed before running: outputs <= 1e-2, gradients <= 3e-2 (the reference's bar,
``nexttransformer/checks/fla.py:44-376``).

Random mode draws inputs at the formal head shape [B, T, 12, 128].  Checkpoint mode runs the trained
model on one row (a validation row of the data directory when given, else a synthetic one), records
the actual mixer inputs of every delta-rule layer, and checks each of them, with the gate statistics
(smallest within-chunk cumulative log decay, share of chunks beyond the fp32 exp range) beside.
The command exits 1 when any error exceeds its tolerance.
"""
import argparse
import json
import math
from pathlib import Path

import torch
import torch.nn.functional as F

TOLERANCE = dict(output=1e-2, gradient=3e-2)
KINDS = ("gdn", "kda", "deltanet")
HEADS, DIM, CHUNK = 12, 128, 64
EXP_RANGE = -87.0   # exp(x) of fp32 underflows / exp(-x) overflows beyond this


def random_inputs(kind, batch, seq, seed, device):
    """Raw mixer inputs of one delta-rule kind (fp64): q, k, v, the log decay g, beta."""
    gen = torch.Generator(device=device).manual_seed(seed)

    def normal(*shape):
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.float64)
    q, k, v = (normal(batch, seq, HEADS, DIM) for _ in range(3))
    beta = torch.sigmoid(normal(batch, seq, HEADS))
    g = None
    if kind == "gdn":
        g = -F.softplus(normal(batch, seq, HEADS)) * 0.3
    elif kind == "kda":
        g = -F.softplus(normal(batch, seq, HEADS, DIM)) * 0.05
    if kind != "gdn":
        # the DeltaNet / KDA mixers L2-normalise q and k before the kernel (GDN does it inside)
        q, k = F.normalize(q, dim=-1) * DIM ** -.5, F.normalize(k, dim=-1)
    return dict(kind=kind, q=q, k=k, v=v, g=g, beta=beta,
                qk_l2norm_scale=DIM ** -.5 if kind == "gdn" else None)


def _oracle_forward(inp):
    from nexttransformer_b200.models.linear import recurrent_scan
    q, k = inp["q"], inp["k"]
    if inp["qk_l2norm_scale"] is not None:
        q, k = F.normalize(q, dim=-1) * inp["qk_l2norm_scale"], F.normalize(k, dim=-1)
    decay = None
    if inp["g"] is not None:
        decay = inp["g"].exp()
        if inp["kind"] == "gdn":
            decay = decay[..., None]
    kind = "kda" if inp["kind"] in ("gdn", "kda") else "deltanet"
    y, _ = recurrent_scan(q, k, inp["v"], kind=kind, decay=decay, beta=inp["beta"])
    return y


def _candidate_forward(name, inp):
    if name == "fused":
        from nexttransformer_b200.ops.linear_attention import delta_chunk_cuda
        return delta_chunk_cuda(inp["q"], inp["k"], inp["v"], kind=inp["kind"], g=inp["g"], beta=inp["beta"],
                                chunk=CHUNK, qk_l2norm_scale=inp["qk_l2norm_scale"])
    from nexttransformer_b200.models.linear import chunk_scan
    q, k = inp["q"], inp["k"]
    if inp["qk_l2norm_scale"] is not None:
        q, k = F.normalize(q, dim=-1) * inp["qk_l2norm_scale"], F.normalize(k, dim=-1)
    return chunk_scan(q, k, inp["v"], kind=inp["kind"], g=inp["g"], beta=inp["beta"], chunk=CHUNK)


NAMES = ("q", "k", "v", "g", "beta")


def _run(inp, fn, dtype, probe):
    leaves = {n: inp[n].detach().to(dtype).requires_grad_() for n in NAMES if inp[n] is not None}
    # the kernels take bf16 q / k / v and fp32 gates, as the training mixers pass them
    args = dict(inp, **leaves)
    y = fn(args)
    grads = torch.autograd.grad(y, list(leaves.values()), probe.to(y.dtype))
    return y.detach().double(), {n: g.double() for n, g in zip(leaves, grads)}


def rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def gate_stats(inp):
    """Smallest within-chunk cumulative log decay and the share of chunks beyond the fp32 exp range."""
    if inp["g"] is None:
        return None
    g = inp["g"].double()
    B, T, H = g.shape[:3]
    n = (T + CHUNK - 1) // CHUNK
    pad = F.pad(g.movedim(1, -1), (0, n * CHUNK - T)).reshape(*g.movedim(1, -1).shape[:-1], n, CHUNK)
    last = pad.sum(-1)
    return dict(min_chunk_log_decay=float(last.min()), beyond_fp32_exp_range=float((last < EXP_RANGE).double().mean()))


def check_one(inp, candidates, seed=0):
    """Relative errors of each candidate against the FP64 oracle; ``ok`` against the tolerances."""
    dev = inp["q"].device
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    probe = torch.randn(inp["v"].shape, generator=gen, device=dev, dtype=torch.float64)
    y_ref, g_ref = _run(inp, _oracle_forward, torch.float64, probe)
    out = {"kind": inp["kind"], "shape": list(inp["q"].shape), "gates": gate_stats(inp), "candidates": {}}
    for name in candidates:
        if name == "fused":
            # the fused path takes bf16 q / k / v (fp32 gates and beta)
            def fn(a):
                a = dict(a, q=a["q"].to(torch.bfloat16), k=a["k"].to(torch.bfloat16), v=a["v"].to(torch.bfloat16))
                return _candidate_forward("fused", a)
            y, g = _run(inp, fn, torch.float32, probe)
        else:
            y, g = _run(inp, lambda a: _candidate_forward(name, a), torch.float32, probe)
        errs = {"output": rel(y, y_ref), **{f"d{n}": rel(g[n], g_ref[n]) for n in g}}
        ok = errs["output"] <= TOLERANCE["output"] and all(v <= TOLERANCE["gradient"]
                                                           for n, v in errs.items() if n != "output")
        out["candidates"][name] = dict(errors=errs, ok=ok)
    out["ok"] = all(c["ok"] for c in out["candidates"].values())
    return out


def capture_mixer_inputs(model, idx):
    """Run ``model`` on ``idx`` and return the inputs of every delta-rule chunk call, in layer order."""
    from nexttransformer_b200.models import linear as L
    captured = []
    original = L.chunk_attention

    def spy(q, k, v, *, kind, g=None, beta=None, chunk, qk_l2norm_scale=None):
        if kind in KINDS:
            captured.append(dict(kind=kind, q=q.detach().double(), k=k.detach().double(), v=v.detach().double(),
                                 g=None if g is None else g.detach().double(),
                                 beta=None if beta is None else beta.detach().double(),
                                 qk_l2norm_scale=qk_l2norm_scale))
        return original(q, k, v, kind=kind, g=g, beta=beta, chunk=chunk, qk_l2norm_scale=qk_l2norm_scale)
    L.chunk_attention = spy
    try:
        with torch.no_grad():
            model(idx)
    finally:
        L.chunk_attention = original
    return captured


def checkpoint_row(model, data_dir=None, tokenizer_dir=None, device="cpu", seed=0):
    """One row of token ids: the first validation row of the data when given, else synthetic."""
    T = model.config.sequence_len
    if data_dir is not None and tokenizer_dir is not None:
        from nexttransformer_b200.runtime.data import BestFitStream
        from nexttransformer_b200.runtime.tokenizer import BPETokenizer
        x, _ = BestFitStream(data_dir, BPETokenizer.from_directory(tokenizer_dir), "val", 0, 1, T).batch(1, device)
        return x
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, model.config.vocab_size, (1, T), generator=gen).to(device)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--kinds", nargs="+", choices=KINDS, default=list(KINDS))
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--checkpoint", type=Path, help="check the mixer inputs of this trained checkpoint")
    ap.add_argument("--data-dir", type=Path)
    ap.add_argument("--tokenizer", type=Path)
    ap.add_argument("--candidates", nargs="+", choices=("fused", "chunk_fp32"))
    ap.add_argument("--output", type=Path)
    a = ap.parse_args(argv)
    dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    candidates = a.candidates or (["fused", "chunk_fp32"] if dev.type == "cuda" else ["chunk_fp32"])
    if "fused" in candidates and dev.type != "cuda":
        ap.error("the fused candidate needs CUDA")
    results = []
    if a.checkpoint is not None:
        from nexttransformer_b200.models import load_model
        model, _ = load_model(a.checkpoint, dev)
        model.eval()
        for layer, inp in enumerate(capture_mixer_inputs(model, checkpoint_row(model, a.data_dir, a.tokenizer, dev,
                                                                                 a.seed))):
            results.append(dict(layer=layer, **check_one(inp, candidates, a.seed)))
    else:
        for kind in a.kinds:
            results.append(check_one(random_inputs(kind, a.batch, a.seq, a.seed, dev), candidates, a.seed))
    report = dict(tolerance=TOLERANCE, device=dev.type, candidates=candidates, results=results,
                  ok=all(r["ok"] for r in results))
    text = json.dumps(report, indent=1)
    if a.output:
        a.output.write_text(text + "\n")
    print(text)
    return 0 if report["ok"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
