"""Bitwise comparison of every registered method at debug size between two source trees.

    python -m nexttransformer_b200.checks.golden --base origin/main
    python -m nexttransformer_b200.checks.golden --dump OUT.json [--methods dense_full gdn]

``--dump`` builds each method at debug size (seed 0), runs one forward/backward on fixed tokens and
records the loss (hex float), parameter names, sha256 digests of all parameters and all gradients,
and the model hash.  ``--base REF`` dumps REF (a temporary git worktree) and the working tree in
fresh CPU-only fp32 interpreters and lists every method whose values differ.  GPU-only kernels need
their own bounded check (``checks.kernels``).
Behaviour: ``nexttransformer/checks/golden.py:26-107``.
"""
import argparse
import hashlib
import json
import os
from pathlib import Path
import subprocess
import sys
import tempfile

REPO = Path(__file__).resolve().parents[2]
ENV = dict(CUDA_VISIBLE_DEVICES="", NANOCHAT_DTYPE="float32", OMP_NUM_THREADS="1")


def digest(items):
    h = hashlib.sha256()
    for name, t in items:
        h.update(name.encode())
        h.update(b"none" if t is None else t.detach().cpu().contiguous().numpy().tobytes())
    return h.hexdigest()


def dump(methods=None):
    import torch
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.lm import build_model
    from nexttransformer_b200.models.registry import METHODS
    torch.use_deterministic_algorithms(True)
    out = {}
    for method in methods or METHODS:
        c = debug_config(method)
        model = build_model(c, "cpu", seed=0)
        model.set_step(c.burnin_steps + 1)
        g = torch.Generator().manual_seed(1)
        x = torch.randint(c.vocab_size, (2, c.sequence_len), generator=g)
        y = torch.randint(c.vocab_size, x.shape, generator=g)
        loss = model(x, y)
        loss.backward()
        named = sorted(model.named_parameters())
        out[method] = dict(loss=float(loss.detach()).hex(), names=[n for n, _ in named], parameters=digest(named),
                           gradients=digest([(n, q.grad) for n, q in named]), model_hash=c.fingerprint)
    return out


def dump_tree(root, path, methods):
    env = dict(os.environ, **ENV, PYTHONPATH=str(root))
    cmd = [sys.executable, "-m", "nexttransformer_b200.checks.golden", "--dump", str(path)]
    if methods:
        cmd += ["--methods", *methods]
    subprocess.run(cmd, cwd=root, env=env, check=True)
    return json.loads(Path(path).read_text())


def compare(base, methods=None):
    def git(*args):
        return subprocess.run(["git", *args], cwd=REPO, capture_output=True, text=True, check=True).stdout
    with tempfile.TemporaryDirectory() as tmp:
        tree = Path(tmp) / "base"
        git("worktree", "add", "--detach", str(tree), git("merge-base", base, "HEAD").strip())
        try:
            # the extension build lives outside git; reuse this tree's build for the CPU paths
            before = dump_tree(tree, Path(tmp) / "base.json", methods)
        finally:
            git("worktree", "remove", "--force", str(tree))
        after = dump_tree(REPO, Path(tmp) / "head.json", methods)
    diff = {}
    for m in sorted(set(before) | set(after)):
        a, b = before.get(m), after.get(m)
        if a != b:
            diff[m] = "added" if a is None else "removed" if b is None else ", ".join(k for k in a if a[k] != b.get(k))
    return diff


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    act = p.add_mutually_exclusive_group(required=True)
    act.add_argument("--base")
    act.add_argument("--dump", type=Path)
    p.add_argument("--methods", nargs="+")
    a = p.parse_args(argv)
    if a.dump:
        for k, v in ENV.items():
            os.environ.setdefault(k, v)
        a.dump.write_text(json.dumps(dump(a.methods), indent=1) + "\n")
        return None
    diff = compare(a.base, a.methods)
    for m, what in diff.items():
        print(f"{m:24} differs: {what}")
    print("all methods are bitwise identical" if not diff else f"{len(diff)} method(s) differ")
    raise SystemExit(1 if diff else 0)


if __name__ == "__main__":
    main()
