"""What a change set touches and which checks it needs (reads git only; does not import torch).

    python -m nexttransformer_b200.checks.changes --base origin/main [--github-output FILE]

* ``tests``: the CPU suite runs unless only documentation or profiles changed.
* ``gpu``: CUDA/C++ sources, their bindings or the fused paths changed - run ``pytest -m gpu`` and
  ``checks.kernels`` on a GPU.
* ``contract``: files of the training contract changed (protocol, ledger, evaluation, trainer, data,
  optimizer, shell); admitted configurations must be re-audited.
* ``affected``: registered methods whose model files changed (family module, plugin package or the
  shared shell).
Behaviour: ``nexttransformer/checks/changes.py`` of the reference, with a GPU category added.
"""
import argparse
import subprocess
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
PKG = "nexttransformer_b200/"
NO_TESTS = ("profiles/", "docs/")      # plus every top-level Markdown file (prose only)
GPU = (PKG + "csrc/", PKG + "ops/", PKG + "models/fused_dense.py", PKG + "optim/muon_adamw.py", PKG + "build.py")
CONTRACT = (PKG + "protocol/", PKG + "evaluation/", PKG + "training/", PKG + "runtime/", PKG + "train.py",
            PKG + "evaluate.py", PKG + "optim/", PKG + "models/shell.py", PKG + "models/lm.py", PKG + "models/config.py")
FAMILY_FILES = {"linear": "models/linear.py", "sparse": "models/sparse.py", "residual": "models/residual.py",
                "looped": "models/looped.py", "moe": "models/moe.py"}


def changed(base):
    def git(*args):
        return subprocess.run(["git", *args], cwd=REPO, capture_output=True, text=True, check=True).stdout
    mb = git("merge-base", base, "HEAD").strip()
    rows = git("diff", "--name-status", "--no-renames", mb, "HEAD").splitlines()
    return [tuple(r.split("\t", 1)) for r in rows if r]


def affected_methods(paths):
    from nexttransformer_b200.models.registry import FAMILY, PLUGINS
    touched = set(paths)
    shared = any(p in touched for p in (PKG + "models/shell.py", PKG + "models/lm.py", PKG + "models/config.py"))
    out = set()
    for method, fam in FAMILY.items():
        if shared:
            out.add(method)
        elif fam in FAMILY_FILES and PKG + FAMILY_FILES[fam] in touched:
            out.add(method)
        elif method in PLUGINS and any(p.startswith(f"{PKG}methods/{method}/") for p in touched):
            out.add(method)
        elif method == "mla_nope" and PKG + "models/mla.py" in touched:
            out.add(method)
    return sorted(out)


def classify(paths):
    paths = list(paths)
    return dict(tests=any(not (p.startswith(NO_TESTS) or ("/" not in p and p.endswith(".md"))) for p in paths),
                gpu=any(p.startswith(GPU) for p in paths),
                contract=sorted(p for p in paths if p.startswith(CONTRACT)),
                affected=affected_methods(paths))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--base", default="origin/main")
    ap.add_argument("--github-output", type=Path)
    a = ap.parse_args(argv)
    paths = [p for _, p in changed(a.base)]
    r = classify(paths)
    print(f"{len(paths)} changed file(s)")
    print(f"CPU tests:  {'run' if r['tests'] else 'skipped (documentation or profiles only)'}")
    print(f"GPU tests:  {'run' if r['gpu'] else 'not needed'}")
    if r["contract"]:
        print("training contract changed: " + ", ".join(r["contract"]))
    if r["affected"]:
        print("methods whose model files changed: " + ", ".join(r["affected"]))
    if a.github_output:
        with open(a.github_output, "a") as f:
            f.write(f"tests={str(r['tests']).lower()}\ngpu={str(r['gpu']).lower()}\n")
            f.write(f"contract={str(bool(r['contract'])).lower()}\naffected={','.join(r['affected'])}\n")
    return r


if __name__ == "__main__":
    main()
