"""Per-method source fingerprints of cost proofs.

While a method's cost is audited, the package files whose Python code runs are recorded; the
package modules those files import are added (transitively, except through the hub modules that
import every family), plus a fixed core (ledger, protocol, calibration, optimizer, shell).  The
fingerprint hashes those files with comments, docstrings and layout removed, so editing comments or
another family's module keeps a proof valid while any change to code the method runs needs a new
audit.  (The reference additionally projects module-level data tables onto the method's own
entries; here a table edit in a shared file re-fingerprints every method that runs the file.)
Behaviour: ``nexttransformer/protocol/fingerprint.py`` of the reference.

    python -m nexttransformer_b200.protocol.fingerprint [--config-dir configs] [--all]
"""
import argparse
import ast
from contextlib import contextmanager
import hashlib
import io
import json
from pathlib import Path
import sys
import tokenize

ROOT = Path(__file__).resolve().parents[2]
PACKAGE = "nexttransformer_b200"
VERSION = "method-source-v1"
CORE = tuple(f"{PACKAGE}/{p}" for p in ("protocol/compute.py", "protocol/spec.py", "protocol/calibrate.py",
                                        "protocol/fingerprint.py", "optim/muon_adamw.py", "optim/groups.py",
                                        "models/shell.py"))
HUBS = frozenset(f"{PACKAGE}/{p}" for p in ("models/__init__.py", "models/lm.py", "models/registry.py"))


def _relative(filename):
    try:
        path = Path(filename).resolve().relative_to(ROOT)
    except (OSError, ValueError):
        return None
    return path.as_posix() if path.parts and path.parts[0] == PACKAGE and path.suffix == ".py" else None


@contextmanager
def traced():
    """Package files whose code runs inside the block (this thread)."""
    files, known = set(), {}

    def trace(frame, event, arg):
        name = frame.f_code.co_filename
        if name not in known:
            known[name] = _relative(name)
        if known[name]:
            files.add(known[name])
        return None

    previous = sys.gettrace()
    sys.settrace(trace)
    try:
        yield files
    finally:
        sys.settrace(previous)


def imports(path):
    """Package modules imported anywhere in the file."""
    out = set()
    for node in ast.walk(ast.parse((ROOT / path).read_text())):
        if isinstance(node, ast.Import):
            mods = [a.name for a in node.names]
        elif isinstance(node, ast.ImportFrom) and node.module and not node.level:
            mods = [node.module, *(f"{node.module}.{a.name}" for a in node.names)]
        else:
            continue
        for mod in mods:
            if mod.split(".")[0] != PACKAGE:
                continue
            base = ROOT / Path(*mod.split("."))
            for cand in (base.with_suffix(".py"), base / "__init__.py"):
                if cand.is_file():
                    out.add(cand.relative_to(ROOT).as_posix())
                    break
    return out


def method_files(executed):
    files, pending = set(), list(executed)
    while pending:
        path = pending.pop()
        if path in files:
            continue
        files.add(path)
        if path not in HUBS and path not in CORE:
            pending += [o for o in imports(path) if o not in files]
    return sorted(files)


def normalized(source):
    """Token stream without comments, docstrings or layout."""
    tree = ast.parse(source)
    docs = {(n.body[0].lineno, n.body[0].col_offset) for n in ast.walk(tree)
            if isinstance(n, (ast.Module, ast.ClassDef, ast.FunctionDef, ast.AsyncFunctionDef)) and n.body
            and isinstance(n.body[0], ast.Expr) and isinstance(n.body[0].value, ast.Constant)
            and isinstance(n.body[0].value.value, str)}
    out, skip_newline = [], False
    for tok in tokenize.generate_tokens(io.StringIO(source).readline):
        kind = tokenize.tok_name[tok.type]
        if kind in ("COMMENT", "NL", "ENCODING", "ENDMARKER"):
            continue
        if kind == "STRING" and tok.start in docs:
            skip_newline = True
            continue
        if kind == "NEWLINE" and skip_newline:
            skip_newline = False
            continue
        skip_newline = False
        out.append(kind if kind in ("NEWLINE", "INDENT", "DEDENT") else f"{kind} {tok.string}")
    return out


def method_source(files):
    h = hashlib.sha256(VERSION.encode())
    for path in sorted(set(files) | set(CORE)):
        f = ROOT / path
        h.update(f"\0{path}\0".encode())
        h.update(("\n".join(normalized(f.read_text())) if f.is_file() else "MISSING").encode())
    return h.hexdigest()


def record(executed):
    files = method_files(executed)
    return dict(version=VERSION, files=files, hash=method_source(files))


def status(path):
    """(recorded hash, current hash) of a configuration file whose cost record has a method source."""
    path = Path(path)
    cal = json.loads(path.read_text())["calibration"]
    proof = json.loads((path.parent / cal["cost_record"]).read_text())
    src = proof.get("method_source")
    return cal.get("method_source_hash"), (method_source(src["files"]) if src else None)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config-dir", type=Path, default=ROOT / "configs")
    ap.add_argument("--all", action="store_true", help="fail when any configuration no longer matches its proof")
    a = ap.parse_args(argv)
    stale = []
    for path in sorted(a.config_dir.glob("*/*.json")):
        if path.name.endswith(".cost.json") or path.parent.name in ("native", "scaling"):
            continue
        recorded, current = status(path)
        ok = current is not None and recorded == current
        if not ok:
            stale.append(path.stem)
        print(f"{path.stem:26} {'matches its proof' if ok else 'needs a new audit' if current else 'no fingerprint'}")
    if a.all and stale:
        raise SystemExit(1)
    return stale


if __name__ == "__main__":
    main()
